// Neighbour-graph builder kernels (see nlist.cuh).
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>

#include "nlist.cuh"

namespace b200dp {

// ---------------------------------------------------------------- host helpers
void make_box_inverse(const double* box, double* Binv, double* width) {
  // Same operation order as the oracle's make_cell (host code is compiled
  // with -ffp-contract=off), so wrapped coordinates agree bit for bit.
  double B[3][3];
  for (int a = 0; a < 3; ++a)
    for (int b = 0; b < 3; ++b) B[a][b] = box[3 * a + b];
  double c00 = B[1][1] * B[2][2] - B[1][2] * B[2][1];
  double c01 = B[1][2] * B[2][0] - B[1][0] * B[2][2];
  double c02 = B[1][0] * B[2][1] - B[1][1] * B[2][0];
  double det = (B[0][0] * c00 + B[0][1] * c01) + B[0][2] * c02;
  double id = 1.0 / det;
  double I[3][3];
  I[0][0] = c00 * id;
  I[1][0] = c01 * id;
  I[2][0] = c02 * id;
  I[0][1] = (B[0][2] * B[2][1] - B[0][1] * B[2][2]) * id;
  I[1][1] = (B[0][0] * B[2][2] - B[0][2] * B[2][0]) * id;
  I[2][1] = (B[0][1] * B[2][0] - B[0][0] * B[2][1]) * id;
  I[0][2] = (B[0][1] * B[1][2] - B[0][2] * B[1][1]) * id;
  I[1][2] = (B[0][2] * B[1][0] - B[0][0] * B[1][2]) * id;
  I[2][2] = (B[0][0] * B[1][1] - B[0][1] * B[1][0]) * id;
  for (int a = 0; a < 3; ++a)
    for (int b = 0; b < 3; ++b) Binv[3 * a + b] = I[a][b];
  double vol = std::fabs(det);
  for (int d = 0; d < 3; ++d) {
    const double* u = B[(d + 1) % 3];
    const double* v = B[(d + 2) % 3];
    double x = u[1] * v[2] - u[2] * v[1], y = u[2] * v[0] - u[0] * v[2], z = u[0] * v[1] - u[1] * v[0];
    width[d] = vol / std::sqrt(x * x + y * y + z * z);
  }
}

int make_grid(bool periodic, const double* box, const double* region, double rcut, long long max_cells, GridSpec& g) {
  std::memset(&g, 0, sizeof(g));
  g.periodic = periodic ? 1 : 0;
  double width[3], ext[3];
  if (periodic) {
    for (int k = 0; k < 9; ++k) g.B[k] = box[k];
    make_box_inverse(box, g.Binv, width);
    for (int d = 0; d < 3; ++d)
      if (!(width[d] > 0) || !std::isfinite(width[d])) return 1;
  } else {
    for (int d = 0; d < 3; ++d) {
      g.lo[d] = region[d];
      ext[d] = std::max(region[3 + d] - region[d], 1e-9);
      width[d] = ext[d];
    }
  }
  double scale = 1.0;
  for (;;) {
    long long tot = 1;
    for (int d = 0; d < 3; ++d) {
      g.n[d] = std::max(1, (int)std::floor(width[d] * kCellsPerCut / (rcut * scale)));
      tot *= g.n[d];
    }
    if (tot <= max_cells) break;
    scale *= 1.25;
  }
  for (int d = 0; d < 3; ++d) {
    // cells are width / n wide; reach = ceil(rcut / cell width)
    g.reach[d] = (int)std::ceil(rcut * g.n[d] / width[d] * (1.0 + 1e-12));
    if (!periodic) {
      // open grid: atoms outside the region are clamped into the edge cells,
      // and nothing lies beyond the grid
      g.inv_h[d] = g.n[d] / ext[d];
      g.reach[d] = std::min(g.reach[d], g.n[d] - 1);
    }
    if (2 * g.reach[d] + 1 > 31) return 2;
  }
  g.ncells = g.n[0] * g.n[1] * g.n[2];
  if (periodic && box[1] == 0.0 && box[2] == 0.0 && box[3] == 0.0 && box[5] == 0.0 && box[6] == 0.0 &&
      box[7] == 0.0) {
    g.prune = 1;
    for (int d = 0; d < 3; ++d) g.cw[d] = box[4 * d] / g.n[d];
  }
  return 0;
}

int make_grid_dbox(const double* box_ref, double min_scale, const double* dbox, double rcut, long long max_cells,
                   GridSpec& g) {
  double b[9];
  for (int k = 0; k < 9; ++k) b[k] = box_ref[k] * min_scale;
  const int rc = make_grid(true, b, nullptr, rcut, max_cells, g);
  g.dB = dbox;
  g.prune = 0;  // the device box may differ from the reference box
  return rc;
}

// The inverse of the box rows on the device, in the same operation order as
// make_box_inverse (explicit round-to-nearest operations, no contraction).
__global__ void k_box_setup(const double* __restrict__ box, double* __restrict__ bb) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  double B[3][3];
  for (int a = 0; a < 3; ++a)
    for (int b = 0; b < 3; ++b) B[a][b] = box[3 * a + b];
  const double c00 = dsub(dmul(B[1][1], B[2][2]), dmul(B[1][2], B[2][1]));
  const double c01 = dsub(dmul(B[1][2], B[2][0]), dmul(B[1][0], B[2][2]));
  const double c02 = dsub(dmul(B[1][0], B[2][1]), dmul(B[1][1], B[2][0]));
  const double det = dadd(dadd(dmul(B[0][0], c00), dmul(B[0][1], c01)), dmul(B[0][2], c02));
  const double id = __drcp_rn(det);
  double I[3][3];
  I[0][0] = dmul(c00, id);
  I[1][0] = dmul(c01, id);
  I[2][0] = dmul(c02, id);
  I[0][1] = dmul(dsub(dmul(B[0][2], B[2][1]), dmul(B[0][1], B[2][2])), id);
  I[1][1] = dmul(dsub(dmul(B[0][0], B[2][2]), dmul(B[0][2], B[2][0])), id);
  I[2][1] = dmul(dsub(dmul(B[0][1], B[2][0]), dmul(B[0][0], B[2][1])), id);
  I[0][2] = dmul(dsub(dmul(B[0][1], B[1][2]), dmul(B[0][2], B[1][1])), id);
  I[1][2] = dmul(dsub(dmul(B[0][2], B[1][0]), dmul(B[0][0], B[1][2])), id);
  I[2][2] = dmul(dsub(dmul(B[0][0], B[1][1]), dmul(B[0][1], B[1][0])), id);
  for (int k = 0; k < 9; ++k) bb[k] = box[k];
  for (int a = 0; a < 3; ++a)
    for (int b = 0; b < 3; ++b) bb[9 + 3 * a + b] = I[a][b];
}

void launch_box_setup(cudaStream_t st, const double* d_box, double* d_bb) {
  count_launch();
  k_box_setup<<<1, 1, 0, st>>>(d_box, d_bb);
}

// The box rows and their inverse of a grid: from device memory when the box
// lives there, else the host-built copies in the grid.
// DB: the box lives in device memory (a barostat's), else in the grid's host-built copies
// (kernel parameters); the kernels are instantiated for both, so the common case keeps
// its constant-bank operands.
template <bool DB>
__device__ __forceinline__ double gB(const GridSpec& g, int k) {
  if constexpr (DB) return __ldg(g.dB + k);
  return g.B[k];
}
template <bool DB>
__device__ __forceinline__ double gBinv(const GridSpec& g, int k) {
  if constexpr (DB) return __ldg(g.dB + 9 + k);
  return g.Binv[k];
}

// ---------------------------------------------------------------- binning
template <bool DB>
__global__ void k_bin(int nall, const double* __restrict__ coord, GridSpec g, double* __restrict__ xw,
                      int* __restrict__ cell_of, int* __restrict__ cell_count, int* __restrict__ lshift,
                      const int* __restrict__ gate) {
  if (gate && *gate == 0) return;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= nall) return;
  const double x[3] = {coord[3 * i], coord[3 * i + 1], coord[3 * i + 2]};
  double w[3];
  int c[3];
  if (g.periodic) {
    double f[3];
#pragma unroll
    for (int d = 0; d < 3; ++d) {
      const double s = dadd(dadd(dmul(x[0], gBinv<DB>(g, d)), dmul(x[1], gBinv<DB>(g, 3 + d))), dmul(x[2], gBinv<DB>(g, 6 + d)));
      f[d] = floor(s);
      if (lshift) lshift[3 * i + d] = (int)f[d];
    }
#pragma unroll
    for (int k = 0; k < 3; ++k)
      w[k] = dsub(x[k], dadd(dadd(dmul(f[0], gB<DB>(g, k)), dmul(f[1], gB<DB>(g, 3 + k))), dmul(f[2], gB<DB>(g, 6 + k))));
#pragma unroll
    for (int d = 0; d < 3; ++d) {
      const double s = (w[0] * gBinv<DB>(g, d) + w[1] * gBinv<DB>(g, 3 + d)) + w[2] * gBinv<DB>(g, 6 + d);
      double v = floor(s * g.n[d]);
      v = fmin(fmax(v, 0.0), (double)(g.n[d] - 1));
      c[d] = (int)v;
    }
  } else {
#pragma unroll
    for (int d = 0; d < 3; ++d) {
      w[d] = x[d];
      double v = floor((x[d] - g.lo[d]) * g.inv_h[d]);
      v = fmin(fmax(v, 0.0), (double)(g.n[d] - 1));
      c[d] = (int)v;
    }
  }
  xw[3 * i] = w[0];
  xw[3 * i + 1] = w[1];
  xw[3 * i + 2] = w[2];
  const int cell = (c[0] * g.n[1] + c[1]) * g.n[2] + c[2];
  cell_of[i] = cell;
  atomicAdd(cell_count + cell, 1);
}

void launch_bin(cudaStream_t st, int nall, const double* coord, const GridSpec& g, double* xw, int* cell_of,
                int* cell_count, int* lshift, const int* gate) {
  if (nall <= 0) return;
  count_launch();
  if (g.dB)
    k_bin<true><<<(nall + 255) / 256, 256, 0, st>>>(nall, coord, g, xw, cell_of, cell_count, lshift, gate);
  else
    k_bin<false><<<(nall + 255) / 256, 256, 0, st>>>(nall, coord, g, xw, cell_of, cell_count, lshift, gate);
}

// Single-block exclusive scan; out has n+1 entries (out[n] = total).  Each
// pass stages 8192 values through shared memory so that global loads and
// stores are coalesced 16-byte vectors while every thread scans 8
// consecutive values.
constexpr int kScanPer = 8;
constexpr int kScanPass = 1024 * kScanPer;

__global__ void __launch_bounds__(1024) k_exclusive_scan(int n, const int* __restrict__ in, int* __restrict__ out,
                                                         const int* __restrict__ gate) {
  if (gate && *gate == 0) return;
  __shared__ __align__(16) int stage[kScanPass];
  __shared__ int warp_ex[32];
  __shared__ int block_total;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const bool vec_in = (reinterpret_cast<uintptr_t>(in) & 15) == 0;
  const bool vec_out = (reinterpret_cast<uintptr_t>(out) & 15) == 0;
  int carry = 0;
  for (int base = 0; base < n; base += kScanPass) {
    const int m = min(kScanPass, n - base);
    if (vec_in && m == kScanPass) {
#pragma unroll
      for (int k = 0; k < kScanPer / 4; ++k) {
        const int q = tid + 1024 * k;
        reinterpret_cast<int4*>(stage)[q] = __ldg(reinterpret_cast<const int4*>(in + base) + q);
      }
    } else {
      for (int q = tid; q < kScanPass; q += 1024) stage[q] = q < m ? in[base + q] : 0;
    }
    __syncthreads();
    int v[kScanPer];
    const int4 a = reinterpret_cast<const int4*>(stage)[2 * tid];
    const int4 b = reinterpret_cast<const int4*>(stage)[2 * tid + 1];
    v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
    int local = 0;
#pragma unroll
    for (int q = 0; q < kScanPer; ++q) local += v[q];
    int wt;
    const int ex = warp_exclusive_scan(local, lane, wt);
    if (lane == 0) warp_ex[warp] = wt;
    __syncthreads();
    if (warp == 0) {
      int tot;
      const int e = warp_exclusive_scan(warp_ex[lane], lane, tot);
      warp_ex[lane] = e;
      if (lane == 0) block_total = tot;
    }
    __syncthreads();
    int run = carry + warp_ex[warp] + ex;
    int w[kScanPer];
#pragma unroll
    for (int q = 0; q < kScanPer; ++q) {
      w[q] = run;
      run += v[q];
    }
    reinterpret_cast<int4*>(stage)[2 * tid] = make_int4(w[0], w[1], w[2], w[3]);
    reinterpret_cast<int4*>(stage)[2 * tid + 1] = make_int4(w[4], w[5], w[6], w[7]);
    carry += block_total;
    __syncthreads();
    if (vec_out && m == kScanPass) {
#pragma unroll
      for (int k = 0; k < kScanPer / 4; ++k) {
        const int q = tid + 1024 * k;
        reinterpret_cast<int4*>(out + base)[q] = reinterpret_cast<const int4*>(stage)[q];
      }
    } else {
      for (int q = tid; q < m; q += 1024) out[base + q] = stage[q];
    }
    __syncthreads();
  }
  if (tid == 0) out[n] = carry;
}

// Multi-block exclusive scan: tile sums, a single-block scan of the sums, and
// a per-tile scan that adds the tile's offset (fixed order, deterministic).
constexpr int kScanTile = 4096;

__global__ void __launch_bounds__(1024) k_scan_tile_sums(int n, const int* __restrict__ in, int* __restrict__ sums,
                                                         const int* __restrict__ gate) {
  if (gate && *gate == 0) return;
  __shared__ int warp_tot[32];
  const int base = blockIdx.x * kScanTile;
  int local = 0;
  for (int i = base + threadIdx.x; i < min(n, base + kScanTile); i += 1024) local += in[i];
  local = warp_sum(local);
  if ((threadIdx.x & 31) == 0) warp_tot[threadIdx.x >> 5] = local;
  __syncthreads();
  if (threadIdx.x < 32) {
    int v = warp_sum(warp_tot[threadIdx.x]);
    if (threadIdx.x == 0) sums[blockIdx.x] = v;
  }
}

__global__ void __launch_bounds__(1024) k_scan_tile_apply(int n, const int* __restrict__ in,
                                                          const int* __restrict__ offs, int* __restrict__ out,
                                                          const int* __restrict__ gate) {
  if (gate && *gate == 0) return;
  __shared__ int warp_ex[32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int i0 = blockIdx.x * kScanTile + tid * 4;
  int v[4], local = 0;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    v[q] = (i0 + q < n) ? in[i0 + q] : 0;
    local += v[q];
  }
  int wt;
  const int ex = warp_exclusive_scan(local, lane, wt);
  if (lane == 0) warp_ex[warp] = wt;
  __syncthreads();
  if (warp == 0) {
    const int mine = warp_ex[lane];
    int tot;
    warp_ex[lane] = warp_exclusive_scan(mine, lane, tot);
  }
  __syncthreads();
  int run = offs[blockIdx.x] + warp_ex[warp] + ex;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    if (i0 + q < n) out[i0 + q] = run;
    run += v[q];
  }
  if (blockIdx.x == gridDim.x - 1 && tid == 0) out[n] = offs[gridDim.x];
}

size_t scan_scratch_ints(int n) { return 2 * ((size_t)n / kScanTile + 2); }

void launch_exclusive_scan(cudaStream_t st, int n, const int* in, int* out, int* scratch, const int* gate) {
  const int nb = (n + kScanTile - 1) / kScanTile;
  if (nb <= 8 || scratch == nullptr) {
    count_launch();
    k_exclusive_scan<<<1, 1024, 0, st>>>(n, in, out, gate);
    return;
  }
  int* sums = scratch;
  int* offs = scratch + nb + 1;
  count_launch();
  k_scan_tile_sums<<<nb, 1024, 0, st>>>(n, in, sums, gate);
  count_launch();
  k_exclusive_scan<<<1, 1024, 0, st>>>(nb, sums, offs, gate);
  count_launch();
  k_scan_tile_apply<<<nb, 1024, 0, st>>>(n, in, offs, out, gate);
}

// Order within a cell follows the atomics and is not fixed; the list kernel's
// ranking does not depend on it.
__global__ void k_fill_cells(int nall, const double* __restrict__ xw, const int* __restrict__ atype,
                             const int* __restrict__ cell_of, const int* __restrict__ cell_start,
                             int* __restrict__ cursor, CellRec* __restrict__ cell_rec, const int* __restrict__ gate) {
  if (gate && *gate == 0) return;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= nall) return;
  const int c = cell_of[i];
  CellRec r;
  r.x = xw[3 * i];
  r.y = xw[3 * i + 1];
  r.z = xw[3 * i + 2];
  r.j = i;
  r.t = atype[i];
  cell_rec[cell_start[c] + atomicAdd(cursor + c, 1)] = r;
}

void launch_fill_cells(cudaStream_t st, int nall, const double* xw, const int* atype, const int* cell_of,
                       const int* cell_start, int* cursor, CellRec* cell_rec, const int* gate) {
  if (nall <= 0) return;
  count_launch();
  k_fill_cells<<<(nall + 255) / 256, 256, 0, st>>>(nall, xw, atype, cell_of, cell_start, cursor, cell_rec, gate);
}

// ---------------------------------------------------------------- format
constexpr int kFmtWarps = 8;

__device__ __forceinline__ int floor_div(int a, int n) { return a >= 0 ? a / n : -((-a + n - 1) / n); }

void format_caps(FormatSpec& f) {
  f.cap_off[0] = 0;
  f.cap_max = 0;
  for (int t = 0; t < f.ntypes; ++t) {
    const int c = (std::max(128, 2 * f.sel[t]) + 31) / 32 * 32;
    f.cap_off[t + 1] = f.cap_off[t] + c;
    f.cap_max = std::max(f.cap_max, c);
  }
}

// Per warp: r2 (8 bytes), j, image code, source index and rank (16 bytes) per
// candidate slot, plus a rank bitmap of the largest type region.
__host__ __device__ inline size_t cand_bytes(int capsum, int cap_max) {
  return ((size_t)capsum * 24 + ((size_t)cap_max / 32 + 1) * 4 + 15) / 16 * 16;
}
size_t format_smem_bytes(const FormatSpec& f) {
  return (size_t)kFmtWarps * cand_bytes(f.cap_off[f.ntypes], f.cap_max);
}

struct CandBuf {
  double* r2;
  int* j;
  int* code;
  int* src;   // kernel-specific handle from which the centre-to-neighbour vector is recomputed
  int* rank;
  unsigned* seen;  // rank bitmap (tie detection)
};

__device__ __forceinline__ CandBuf cand_buf(unsigned char* smem, int warp, const FormatSpec& f) {
  const int capsum = f.cap_off[f.ntypes];
  unsigned char* base = smem + (size_t)warp * cand_bytes(capsum, f.cap_max);
  CandBuf b;
  b.r2 = reinterpret_cast<double*>(base);
  b.j = reinterpret_cast<int*>(b.r2 + capsum);
  b.code = b.j + capsum;
  b.src = b.code + capsum;
  b.rank = b.src + capsum;
  b.seen = reinterpret_cast<unsigned*>(b.rank + capsum);
  return b;
}

// Appends the valid lanes' candidates to their type regions (warp ballots per
// type; ncnt[t] keeps counting past the capacity so overflow is seen).
__device__ __forceinline__ void cand_push(const FormatSpec& f, const CandBuf& b, int (&ncnt)[kMaxTypes], bool valid,
                                          int tj, double r2, int j, int code, int src, unsigned lt_mask) {
#pragma unroll
  for (int t = 0; t < kMaxTypes; ++t) {
    if (t >= f.ntypes) break;
    const bool mine = valid && tj == t;
    const unsigned m = __ballot_sync(0xffffffffu, mine);
    const int pos = ncnt[t] + __popc(m & lt_mask);
    if (mine && pos < f.cap_off[t + 1] - f.cap_off[t]) {
      const int o = f.cap_off[t] + pos;
      b.r2[o] = r2;
      b.j[o] = j;
      b.code[o] = code;
      b.src[o] = src;
    }
    ncnt[t] += __popc(m);
  }
}

// Orders one centre's candidates and writes its row: each candidate is ranked
// against the candidates of its own type by (r^2, j, image).  Keys are unique
// (j, image) pairs, so the order is total and does not depend on the order in
// which the candidates were found.  r^2 alone decides almost always: each
// member counts the smaller r^2 of its type (warp-uniform broadcast reads);
// two members landing on the same rank reveal a tie, and only then is the
// type re-ranked with the full key.  rvec(src, code, r) recomputes the
// centre-to-neighbour vector of a kept candidate.
template <typename RVec>
__device__ void emit_row(const FormatSpec& f, int i, const CandBuf& b, const int (&ncnt)[kMaxTypes], int lane,
                         int* __restrict__ nl_j, int* __restrict__ nl_code, double* __restrict__ nl_rij,
                         int* __restrict__ nl_cnt, int* __restrict__ err, RVec rvec) {
  const int zero_code = image_code(0, 0, 0);
#pragma unroll 1
  for (int t = 0; t < f.ntypes; ++t) {
    const int cap_t = f.cap_off[t + 1] - f.cap_off[t];
    const int o = f.cap_off[t];
    int nt = ncnt[0];
#pragma unroll
    for (int u = 1; u < kMaxTypes; ++u)
      if (u == t) nt = ncnt[u];
    if (nt > cap_t) {
      if (lane == 0) atomicAdd(err + kErrCandCapacity, 1);
      nt = cap_t;
    }
    const int sel = f.sel[t];
    const int keep = nt < sel ? nt : sel;
    const double* r2v = b.r2 + o;
    if (nt > 0) {
      for (int w = lane; w <= nt / 32; w += 32) b.seen[w] = 0u;
      __syncwarp();
      bool tie = false;
      for (int base = 0; base < nt; base += 64) {
        const int ma = base + lane, mb = base + 32 + lane;
        const double ra = ma < nt ? r2v[ma] : 0.0, rb = mb < nt ? r2v[mb] : 0.0;
        int ka = 0, kb = 0;
        for (int k = 0; k < nt; ++k) {
          const double q = r2v[k];
          ka += (q < ra);
          kb += (q < rb);
        }
        if (ma < nt) {
          tie |= (atomicOr(&b.seen[ka >> 5], 1u << (ka & 31)) >> (ka & 31)) & 1u;
          b.rank[o + ma] = ka;
        }
        if (mb < nt) {
          tie |= (atomicOr(&b.seen[kb >> 5], 1u << (kb & 31)) >> (kb & 31)) & 1u;
          b.rank[o + mb] = kb;
        }
      }
      tie = __any_sync(0xffffffffu, tie);
      __syncwarp();
      for (int m = lane; m < nt; m += 32) {
        int rank = b.rank[o + m];
        const int j = b.j[o + m], code = b.code[o + m];
        if (tie) {  // full key (r^2, j, image)
          const double r2 = r2v[m];
          rank = 0;
          for (int k = 0; k < nt; ++k) {
            const double q = r2v[k];
            if (q < r2) {
              ++rank;
            } else if (q == r2 && k != m) {
              const int j2 = b.j[o + k];
              rank += (j2 < j || (j2 == j && b.code[o + k] < code));
            }
          }
        }
        if (rank < sel) {
          double r[3];
          rvec(b.src[o + m], code, r);
          const size_t slot = (size_t)i * f.selt + f.off[t] + rank;
          nl_j[slot] = j;
          nl_code[slot] = code;
          nl_rij[3 * slot] = r[0];
          nl_rij[3 * slot + 1] = r[1];
          nl_rij[3 * slot + 2] = r[2];
        }
      }
      __syncwarp();
    }
    for (int s = keep + lane; s < sel; s += 32) {
      const size_t slot = (size_t)i * f.selt + f.off[t] + s;
      nl_j[slot] = -1;
      nl_code[slot] = zero_code;
      nl_rij[3 * slot] = 0.0;
      nl_rij[3 * slot + 1] = 0.0;
      nl_rij[3 * slot + 2] = 0.0;
    }
    if (lane == 0) {
      nl_cnt[(size_t)i * f.ntypes + t] = keep;
      if (nt > sel) atomicAdd(err + kErrSelOverflow, nt - sel);
    }
  }
}

// Shift of periodic image (n0, n1, n2) and the vector from centre xi to
// neighbour xj in that image: (xj + shift) - xi, fp64, fixed operation order.
template <bool DB>
__device__ __forceinline__ void image_vector(const GridSpec& g, const double (&xi)[3], double x0, double x1,
                                             double x2, int code, double (&r)[3]) {
  double sh[3] = {0, 0, 0};
  if (g.periodic) {
    const double m0 = (double)(((code >> 20) & 1023) - kImageBias), m1 = (double)(((code >> 10) & 1023) - kImageBias),
                 m2 = (double)((code & 1023) - kImageBias);
#pragma unroll
    for (int c = 0; c < 3; ++c) sh[c] = dadd(dadd(dmul(m0, gB<DB>(g, c)), dmul(m1, gB<DB>(g, 3 + c))), dmul(m2, gB<DB>(g, 6 + c)));
  }
  r[0] = dsub(dadd(x0, sh[0]), xi[0]);
  r[1] = dsub(dadd(x1, sh[1]), xi[1]);
  r[2] = dsub(dadd(x2, sh[2]), xi[2]);
}

// Stencil cells handled per pass: kStencilPerLane consecutive cells per lane.
constexpr int kStencilPerLane = 4;
constexpr int kStencilChunk = 32 * kStencilPerLane;
constexpr int kGatherBatch = 4;  // candidate records loaded per lane before any is used

template <auto Kernel>
static void format_attr(size_t smem) {
  // the attribute is raised (never lowered) as larger type capacities arrive; one
  // record per kernel instantiation
  static size_t set = 48 * 1024;
  if (smem > set) {
    cudaFuncSetAttribute(Kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    set = smem;
  }
}

// Candidates of centre i (one warp): the stencil (every cell within reach,
// periodic images included) is flattened; a warp scan over the cells' atom
// counts numbers the candidates, and each lane takes every 32nd candidate,
// finds its cell by a binary search over the scanned counts and loads the
// cell-sorted record.  push(valid, tj, r2, j, code, ridx) is called by all
// lanes together for each batch slot (r2 < rc2, not the centre itself, type
// in range).
template <bool DB, typename Push>
__device__ __forceinline__ void gather_stencil(const FormatSpec& f, const GridSpec& g, const double (&xi)[3], int i,
                                               int cell, double rc2, const int* __restrict__ cell_start,
                                               const CellRec* __restrict__ cell_rec, int* __restrict__ err,
                                               int* c_start, int* c_pref, int* c_code, int lane, Push push) {
  const int ci[3] = {cell / (g.n[1] * g.n[2]), (cell / g.n[2]) % g.n[1], cell % g.n[2]};
  const int sy = 2 * g.reach[1] + 1, sz = 2 * g.reach[2] + 1;
  const int nstencil = (2 * g.reach[0] + 1) * sy * sz;
  // a stencil that reaches at most one cell row past the box wraps by one image
  // per dimension (no division); wider reaches (boxes thinner than the cutoff)
  // take the general floor division
  const bool one_image = g.reach[0] <= g.n[0] && g.reach[1] <= g.n[1] && g.reach[2] <= g.n[2];
  for (int s0 = 0; s0 < nstencil; s0 += kStencilChunk) {
    // counts of this lane's cells, then a warp scan
    int cnt[kStencilPerLane], st[kStencilPerLane], cd[kStencilPerLane];
    int local = 0;
    // this lane's first stencil cell, decoded once; the next ones step in z with carries
    const int sfirst = s0 + lane * kStencilPerLane;
    int dz = sfirst % sz, dy = (sfirst / sz) % sy, dx = sfirst / (sz * sy);
#pragma unroll
    for (int u = 0; u < kStencilPerLane; ++u) {
      const int sidx = sfirst + u;
      cnt[u] = 0;
      st[u] = 0;
      cd[u] = 0;
      if (sidx < nstencil) {
        int uu[3] = {ci[0] + dx - g.reach[0], ci[1] + dy - g.reach[1], ci[2] + dz - g.reach[2]};
        int img[3] = {0, 0, 0};
        bool ok = true;
#pragma unroll
        for (int d = 0; d < 3; ++d) {
          if (g.periodic) {
            if (one_image) {
              img[d] = uu[d] < 0 ? -1 : (uu[d] >= g.n[d] ? 1 : 0);
            } else {
              img[d] = floor_div(uu[d], g.n[d]);
            }
            uu[d] -= img[d] * g.n[d];
          } else {
            ok = ok && uu[d] >= 0 && uu[d] < g.n[d];
          }
        }
        if (!DB && ok && g.prune) {  // distance from the centre to the cell's box
          const int o[3] = {dx - g.reach[0], dy - g.reach[1], dz - g.reach[2]};
          double d2 = 0.0;
#pragma unroll
          for (int d = 0; d < 3; ++d) {
            const double pc = xi[d] - ci[d] * g.cw[d];  // the centre's offset inside its cell
            const double gap = o[d] > 0 ? o[d] * g.cw[d] - pc : (o[d] < 0 ? pc + (-o[d] - 1) * g.cw[d] : 0.0);
            const double gm = fmax(gap - 1e-6, 0.0);
            d2 += gm * gm;
          }
          ok = d2 < rc2;
        }
        if (ok) {
          const int cc = (uu[0] * g.n[1] + uu[1]) * g.n[2] + uu[2];
          st[u] = cell_start[cc];
          cnt[u] = cell_start[cc + 1] - st[u];
          cd[u] = image_code(img[0], img[1], img[2]);
        }
      }
      local += cnt[u];
      if (++dz == sz) {
        dz = 0;
        if (++dy == sy) {
          dy = 0;
          ++dx;
        }
      }
    }
    int total;
    int run = warp_exclusive_scan(local, lane, total);
#pragma unroll
    for (int u = 0; u < kStencilPerLane; ++u) {
      const int q = lane * kStencilPerLane + u;
      c_start[q] = st[u];
      c_pref[q] = run;  // cells past the stencil get pref == total and are never chosen
      c_code[q] = cd[u];
      run += cnt[u];
    }
    __syncwarp();
    for (int k0 = 0; k0 < total; k0 += 32 * kGatherBatch) {
      double2 ra[kGatherBatch], rc[kGatherBatch];
      int rcode[kGatherBatch], ridx[kGatherBatch];
#pragma unroll
      for (int u = 0; u < kGatherBatch; ++u) {
        const int k = k0 + 32 * u + lane;
        rcode[u] = -1;
        ridx[u] = 0;
        ra[u] = make_double2(0.0, 0.0);
        rc[u] = make_double2(0.0, 0.0);
        if (k < total) {
          int q = 0;  // last cell with c_pref[q] <= k (that cell holds k)
#pragma unroll
          for (int step = kStencilChunk / 2; step > 0; step >>= 1)
            if (c_pref[q + step] <= k) q += step;
          ridx[u] = c_start[q] + (k - c_pref[q]);
          const double2* src = reinterpret_cast<const double2*>(cell_rec + ridx[u]);
          ra[u] = __ldg(src);
          rc[u] = __ldg(src + 1);
          rcode[u] = c_code[q];
        }
      }
#pragma unroll
      for (int u = 0; u < kGatherBatch; ++u) {
        const long long jt = __double_as_longlong(rc[u].y);  // {int j, int t}, little-endian
        const int j = (int)(unsigned)(jt & 0xffffffffll), tj = (int)(jt >> 32), code = rcode[u];
        bool valid = false;
        double r2 = 0;
        if (code >= 0) {
          double r[3];
          image_vector<DB>(g, xi, ra[u].x, ra[u].y, rc[u].x, code, r);
          r2 = dadd(dadd(dmul(r[0], r[0]), dmul(r[1], r[1])), dmul(r[2], r[2]));
          const bool self = (j == i) && code == image_code(0, 0, 0);
          const bool type_ok = (tj >= 0 && tj < f.ntypes);
          if (!type_ok && !self && r2 < rc2) atomicAdd(err + kErrBadType, 1);
          valid = !self && type_ok && (r2 < rc2);
        }
        push(valid, tj, r2, j, code, ridx[u]);
      }
    }
    __syncwarp();
  }
}

template <bool DB>
__global__ void __launch_bounds__(kFmtWarps * 32, 3)
    k_format(FormatSpec f, GridSpec g, const double* __restrict__ xw, const int* __restrict__ cell_of,
             const int* __restrict__ cell_start, const CellRec* __restrict__ cell_rec, int* __restrict__ nl_j,
             int* __restrict__ nl_code, double* __restrict__ nl_rij, int* __restrict__ nl_cnt,
             int* __restrict__ err) {
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ int s_start[kFmtWarps][kStencilChunk], s_pref[kFmtWarps][kStencilChunk], s_code[kFmtWarps][kStencilChunk];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int i = blockIdx.x * kFmtWarps + warp;
  if (i >= f.nloc) return;  // warp-uniform; no block-level barrier follows
  const CandBuf b = cand_buf(smem, warp, f);
  const double xi[3] = {xw[3 * i], xw[3 * i + 1], xw[3 * i + 2]};
  const unsigned lt_mask = (1u << lane) - 1u;
  int ncnt[kMaxTypes];
#pragma unroll
  for (int t = 0; t < kMaxTypes; ++t) ncnt[t] = 0;
  gather_stencil<DB>(f, g, xi, i, cell_of[i], f.rc2, cell_start, cell_rec, err, s_start[warp], s_pref[warp],
                 s_code[warp], lane, [&](bool valid, int tj, double r2, int j, int code, int ridx) {
                   cand_push(f, b, ncnt, valid, tj, r2, j, code, ridx, lt_mask);
                 });
  __syncwarp();
  emit_row(f, i, b, ncnt, lane, nl_j, nl_code, nl_rij, nl_cnt, err,
           [&](int src, int code, double (&r)[3]) {
             const double2* p = reinterpret_cast<const double2*>(cell_rec + src);
             const double2 a = __ldg(p), c = __ldg(p + 1);
             image_vector<DB>(g, xi, a.x, a.y, c.x, code, r);
           });
}

// ---------------------------------------------------------------- neighbour reuse
// Skin (Verlet) candidates: every (j, image) within rc + skin of a centre,
// kept for several evaluations.  The rows are then formed from the candidates
// with the positions of each call, shifted by the lattice vectors each atom
// was wrapped by when the candidates were built (so the image codes stay
// valid as atoms cross the cell boundary, and under a changing cell).
template <bool DB>
__global__ void __launch_bounds__(kFmtWarps * 32)
    k_verlet_build(FormatSpec f, GridSpec g, double rcand2, int capS, const double* __restrict__ xw,
                   const int* __restrict__ cell_of, const int* __restrict__ cell_start,
                   const CellRec* __restrict__ cell_rec, int* __restrict__ cand_j, int* __restrict__ cand_code,
                   int* __restrict__ cand_cnt, int* __restrict__ err, const int* __restrict__ gate) {
  if (gate && *gate == 0) return;
  __shared__ int s_start[kFmtWarps][kStencilChunk], s_pref[kFmtWarps][kStencilChunk], s_code[kFmtWarps][kStencilChunk];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int i = blockIdx.x * kFmtWarps + warp;
  if (i >= f.nloc) return;
  const double xi[3] = {xw[3 * i], xw[3 * i + 1], xw[3 * i + 2]};
  const unsigned lt_mask = (1u << lane) - 1u;
  int n = 0;
  int* cj = cand_j + (size_t)i * capS;
  int* cc = cand_code + (size_t)i * capS;
  gather_stencil<DB>(f, g, xi, i, cell_of[i], rcand2, cell_start, cell_rec, err, s_start[warp], s_pref[warp],
                 s_code[warp], lane, [&](bool valid, int, double, int j, int code, int) {
                   const unsigned m = __ballot_sync(0xffffffffu, valid);
                   const int pos = n + __popc(m & lt_mask);
                   if (valid && pos < capS) {
                     cj[pos] = j;
                     cc[pos] = code;
                   }
                   n += __popc(m);
                 });
  if (lane == 0) {
    if (n > capS) atomicAdd(err + kErrCandCapacity, 1);
    cand_cnt[i] = n < capS ? n : capS;
  }
}

// Position of atom j shifted by its build-time lattice shift, with the
// arithmetic of k_bin's wrap (so a call right after a build sees the wrapped
// coordinates bit for bit).
template <bool DB>
__device__ __forceinline__ void shifted(const GridSpec& g, const double* __restrict__ x, const int* __restrict__ ls,
                                        int j, double (&w)[3]) {
  const double f0 = (double)ls[3 * j], f1 = (double)ls[3 * j + 1], f2 = (double)ls[3 * j + 2];
#pragma unroll
  for (int k = 0; k < 3; ++k)
    w[k] = dsub(x[3 * j + k], dadd(dadd(dmul(f0, gB<DB>(g, k)), dmul(f1, gB<DB>(g, 3 + k))), dmul(f2, gB<DB>(g, 6 + k))));
}

template <bool DB>
__global__ void __launch_bounds__(kFmtWarps * 32)
    k_format_verlet(FormatSpec f, GridSpec g, int capS, double half_skin2, const double* __restrict__ x,
                    const int* __restrict__ atype, const int* __restrict__ lshift, const double* __restrict__ xref,
                    const int* __restrict__ cand_j, const int* __restrict__ cand_code,
                    const int* __restrict__ cand_cnt, int* __restrict__ nl_j, int* __restrict__ nl_code,
                    double* __restrict__ nl_rij, int* __restrict__ nl_cnt, int* __restrict__ err,
                    int* __restrict__ stale) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int i = blockIdx.x * kFmtWarps + warp;
  if (i >= f.nloc) return;
  const CandBuf b = cand_buf(smem, warp, f);
  double xi[3];
  shifted<DB>(g, x, lshift, i, xi);
  if (lane == 0) {
    double d2 = 0;
#pragma unroll
    for (int k = 0; k < 3; ++k) {
      const double d = x[3 * i + k] - xref[3 * i + k];
      d2 += d * d;
    }
    if (d2 > half_skin2) atomicOr(stale, 1);
  }
  const unsigned lt_mask = (1u << lane) - 1u;
  int ncnt[kMaxTypes];
#pragma unroll
  for (int t = 0; t < kMaxTypes; ++t) ncnt[t] = 0;
  const int n = cand_cnt[i];
  const int* cj = cand_j + (size_t)i * capS;
  const int* cc = cand_code + (size_t)i * capS;
  for (int k0 = 0; k0 < n; k0 += 32) {
    const int k = k0 + lane;
    bool valid = false;
    int j = 0, code = 0, tj = 0;
    double r2 = 0;
    if (k < n) {
      j = cj[k];
      code = cc[k];
      tj = atype[j];
      double xj[3], r[3];
      shifted<DB>(g, x, lshift, j, xj);
      image_vector<DB>(g, xi, xj[0], xj[1], xj[2], code, r);
      r2 = dadd(dadd(dmul(r[0], r[0]), dmul(r[1], r[1])), dmul(r[2], r[2]));
      valid = (tj >= 0 && tj < f.ntypes) && r2 < f.rc2;
    }
    cand_push(f, b, ncnt, valid, tj, r2, j, code, k, lt_mask);
  }
  __syncwarp();
  emit_row(f, i, b, ncnt, lane, nl_j, nl_code, nl_rij, nl_cnt, err, [&](int src, int code, double (&r)[3]) {
    double xj[3];
    shifted<DB>(g, x, lshift, cj[src], xj);
    image_vector<DB>(g, xi, xj[0], xj[1], xj[2], code, r);
  });
}

void launch_verlet_build(cudaStream_t st, const FormatSpec& f, const GridSpec& g, double rcand, int capS,
                         const double* xw, const int* cell_of, const int* cell_start, const CellRec* cell_rec,
                         int* cand_j, int* cand_code, int* cand_cnt, int* err, const int* gate) {
  if (f.nloc <= 0) return;
  count_launch();
  const dim3 grid((f.nloc + kFmtWarps - 1) / kFmtWarps);
  if (g.dB)
    k_verlet_build<true><<<grid, kFmtWarps * 32, 0, st>>>(f, g, rcand * rcand, capS, xw, cell_of, cell_start,
                                                          cell_rec, cand_j, cand_code, cand_cnt, err, gate);
  else
    k_verlet_build<false><<<grid, kFmtWarps * 32, 0, st>>>(f, g, rcand * rcand, capS, xw, cell_of, cell_start,
                                                           cell_rec, cand_j, cand_code, cand_cnt, err, gate);
}

// Displacement check of every atom against the positions the candidates were
// built from: sets *trig when one moved more than skin / 2, and clears the
// other call's flag (its readers have completed: same stream).
__global__ void k_skin_check(int n, const double* __restrict__ x, const double* __restrict__ xref, double half_skin2,
                             int* __restrict__ trig, int* __restrict__ trig_prev) {
  if (blockIdx.x == 0 && threadIdx.x == 0) *trig_prev = 0;
  bool moved = false;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    double d2 = 0;
#pragma unroll
    for (int k = 0; k < 3; ++k) {
      const double d = x[3 * i + k] - xref[3 * i + k];
      d2 += d * d;
    }
    moved |= d2 > half_skin2;
  }
  if (__syncthreads_or(moved) && threadIdx.x == 0) atomicOr(trig, 1);
}

// When *gate: the reference positions become x and the rebuild is counted.
__global__ void k_xref_update(int n, const double* __restrict__ x, double* __restrict__ xref,
                              const int* __restrict__ gate, unsigned long long* __restrict__ count) {
  if (*gate == 0) return;
  if (blockIdx.x == 0 && threadIdx.x == 0) ++*count;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < 3 * n; i += gridDim.x * blockDim.x) xref[i] = x[i];
}

void launch_skin_check(cudaStream_t st, int n, const double* x, const double* xref, double skin, int* trig,
                       int* trig_prev) {
  if (n <= 0) return;
  count_launch();
  const int blocks = std::min((n + 255) / 256, 148 * 8);
  k_skin_check<<<blocks, 256, 0, st>>>(n, x, xref, 0.25 * skin * skin, trig, trig_prev);
}

void launch_xref_update(cudaStream_t st, int n, const double* x, double* xref, const int* gate,
                        unsigned long long* count) {
  if (n <= 0) return;
  count_launch();
  const int blocks = std::min((3 * n + 255) / 256, 148 * 8);
  k_xref_update<<<blocks, 256, 0, st>>>(n, x, xref, gate, count);
}

void launch_format_verlet(cudaStream_t st, const FormatSpec& f, const GridSpec& g, int capS, double skin,
                          const double* x, const int* atype, const int* lshift, const double* xref,
                          const int* cand_j, const int* cand_code, const int* cand_cnt, int* nl_j, int* nl_code,
                          double* nl_rij, int* nl_cnt, int* err, int* stale) {
  if (f.nloc <= 0) return;
  const size_t smem = format_smem_bytes(f);
  const dim3 grid((f.nloc + kFmtWarps - 1) / kFmtWarps);
  count_launch();
  if (g.dB) {
    format_attr<k_format_verlet<true>>(smem);
    k_format_verlet<true><<<grid, kFmtWarps * 32, smem, st>>>(f, g, capS, 0.25 * skin * skin, x, atype, lshift, xref,
                                                              cand_j, cand_code, cand_cnt, nl_j, nl_code, nl_rij,
                                                              nl_cnt, err, stale);
  } else {
    format_attr<k_format_verlet<false>>(smem);
    k_format_verlet<false><<<grid, kFmtWarps * 32, smem, st>>>(f, g, capS, 0.25 * skin * skin, x, atype, lshift,
                                                               xref, cand_j, cand_code, cand_cnt, nl_j, nl_code,
                                                               nl_rij, nl_cnt, err, stale);
  }
}

void launch_format(cudaStream_t st, const FormatSpec& f, const GridSpec& g, const double* xw, const int* cell_of,
                   const int* cell_start, const CellRec* cell_rec, int* nl_j, int* nl_code, double* nl_rij,
                   int* nl_cnt, int* err) {
  if (f.nloc <= 0) return;
  const size_t smem = format_smem_bytes(f);
  const dim3 grid((f.nloc + kFmtWarps - 1) / kFmtWarps);
  count_launch();
  if (g.dB) {
    format_attr<k_format<true>>(smem);
    k_format<true><<<grid, kFmtWarps * 32, smem, st>>>(f, g, xw, cell_of, cell_start, cell_rec, nl_j, nl_code, nl_rij,
                                                       nl_cnt, err);
  } else {
    format_attr<k_format<false>>(smem);
    k_format<false><<<grid, kFmtWarps * 32, smem, st>>>(f, g, xw, cell_of, cell_start, cell_rec, nl_j, nl_code,
                                                        nl_rij, nl_cnt, err);
  }
}

// Caller-provided candidates (LAMMPS full list): cand_start is a CSR over
// ilist order.  No periodic images: r = x_j - x_i on raw coordinates.
__global__ void __launch_bounds__(kFmtWarps * 32)
    k_format_candidates(FormatSpec f, const double* __restrict__ coord, const int* __restrict__ atype,
                        const int* __restrict__ ilist, const int* __restrict__ cand_start,
                        const int* __restrict__ cand, int* __restrict__ nl_j, int* __restrict__ nl_code,
                        double* __restrict__ nl_rij, int* __restrict__ nl_cnt, int* __restrict__ err) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * kFmtWarps + warp;
  if (row >= f.nloc) return;
  const int i = ilist[row];
  if (i < 0 || i >= f.nloc) return;
  const CandBuf b = cand_buf(smem, warp, f);
  const double xi[3] = {coord[3 * i], coord[3 * i + 1], coord[3 * i + 2]};
  const unsigned lt_mask = (1u << lane) - 1u;
  const int beg = cand_start[row], end = cand_start[row + 1];
  int ncnt[kMaxTypes];
#pragma unroll
  for (int t = 0; t < kMaxTypes; ++t) ncnt[t] = 0;
  for (int k = beg + lane; k - lane < end; k += 32) {
    bool valid = false;
    int j = -1, tj = 0;
    double r2 = 0;
    if (k < end) {
      j = cand[k];
      if (j >= 0 && j < f.nall && j != i) {
        double r[3];
#pragma unroll
        for (int c = 0; c < 3; ++c) r[c] = dsub(coord[3 * j + c], xi[c]);
        r2 = dadd(dadd(dmul(r[0], r[0]), dmul(r[1], r[1])), dmul(r[2], r[2]));
        tj = atype[j];
        const bool type_ok = (tj >= 0 && tj < f.ntypes);
        if (!type_ok && r2 < f.rc2) atomicAdd(err + kErrBadType, 1);
        valid = type_ok && r2 < f.rc2;
      }
    }
    cand_push(f, b, ncnt, valid, tj, r2, j, image_code(0, 0, 0), j, lt_mask);
  }
  __syncwarp();
  const double xi0 = xi[0], xi1 = xi[1], xi2 = xi[2];
  emit_row(f, i, b, ncnt, lane, nl_j, nl_code, nl_rij, nl_cnt, err, [=](int src, int, double (&r)[3]) {
    r[0] = dsub(coord[3 * src], xi0);
    r[1] = dsub(coord[3 * src + 1], xi1);
    r[2] = dsub(coord[3 * src + 2], xi2);
  });
}

// Canonical destination-major graph (the reference's direct-engine input):
// node i's edges are [row_ptr[i], row_ptr[i+1]), each with a source node j and
// the fp32 vector x_j - x_i.  Every edge is a candidate; periodic images are
// separate edges of the same source, told apart by their position in the
// row (the tie-break key in place of the image code).  Also writes the int32
// type of every node.
__global__ void __launch_bounds__(kFmtWarps * 32)
    k_format_graph(FormatSpec f, const int64_t* __restrict__ atype64, const int64_t* __restrict__ row_ptr,
                   const uint32_t* __restrict__ source, const float* __restrict__ edge_vec, int* __restrict__ atype32,
                   int* __restrict__ nl_j, int* __restrict__ nl_code, double* __restrict__ nl_rij,
                   int* __restrict__ nl_cnt, int* __restrict__ err, RawGeometry raw) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int i = blockIdx.x * kFmtWarps + warp;
  if (i >= f.nloc) return;
  if (lane == 0) {
    const int64_t ti = atype64[i];
    atype32[i] = (ti >= 0 && ti < f.ntypes) ? (int)ti : -1;
    if (ti < 0 || ti >= f.ntypes) atomicAdd(err + kErrBadType, 1);
  }
  const CandBuf b = cand_buf(smem, warp, f);
  const unsigned lt_mask = (1u << lane) - 1u;
  const int64_t beg = row_ptr[i], end = row_ptr[i + 1];
  // the edge vector: the graph's fp32 one, or recomputed in fp64 from the bound positions
  const double* xi = raw.x ? raw.x + (long long)raw.m2a[i] * raw.sa : nullptr;
  auto edge = [&](int64_t k, double (&r)[3]) {
    if (raw.x) {
      const double* xj = raw.x + (long long)raw.cand[k] * raw.sa;
#pragma unroll
      for (int c = 0; c < 3; ++c) r[c] = dmul(dsub(xj[c * raw.sx], xi[c * raw.sx]), raw.unit);
    } else {
#pragma unroll
      for (int c = 0; c < 3; ++c) r[c] = (double)edge_vec[3 * k + c];
    }
  };
  int ncnt[kMaxTypes];
#pragma unroll
  for (int t = 0; t < kMaxTypes; ++t) ncnt[t] = 0;
  for (int64_t k = beg + lane; k - lane < end; k += 32) {
    bool valid = false;
    int j = -1, tj = 0;
    double r2 = 0;
    if (k < end) {
      const uint32_t src = source[k];
      if (src < (uint32_t)f.nall) {
        j = (int)src;
        double r[3];
        edge(k, r);
        r2 = dadd(dadd(dmul(r[0], r[0]), dmul(r[1], r[1])), dmul(r[2], r[2]));
        const int64_t t64 = atype64[j];
        const bool type_ok = (t64 >= 0 && t64 < f.ntypes);
        tj = type_ok ? (int)t64 : 0;
        if (!type_ok && r2 < f.rc2) atomicAdd(err + kErrBadType, 1);
        valid = type_ok && r2 > 0.0 && r2 < f.rc2;
      }
    }
    // the image code is the edge's position in the row
    cand_push(f, b, ncnt, valid, tj, r2, j, (int)(k - beg), (int)(k - beg), lt_mask);
  }
  __syncwarp();
  emit_row(f, i, b, ncnt, lane, nl_j, nl_code, nl_rij, nl_cnt, err, [&](int src, int, double (&r)[3]) {
    edge(beg + src, r);
  });
}

void launch_format_graph(cudaStream_t st, const FormatSpec& f, const int64_t* atype64, const int64_t* row_ptr,
                         const uint32_t* source, const float* edge_vec, int* atype32, int* nl_j, int* nl_code,
                         double* nl_rij, int* nl_cnt, int* err, const RawGeometry& raw) {
  if (f.nloc <= 0) return;
  const size_t smem = format_smem_bytes(f);
  format_attr<k_format_graph>(smem);
  count_launch();
  k_format_graph<<<(f.nloc + kFmtWarps - 1) / kFmtWarps, kFmtWarps * 32, smem, st>>>(
      f, atype64, row_ptr, source, edge_vec, atype32, nl_j, nl_code, nl_rij, nl_cnt, err, raw);
}

void launch_format_candidates(cudaStream_t st, const FormatSpec& f, const double* coord, const int* atype,
                              const int* ilist, const int* cand_start, const int* cand, int* nl_j, int* nl_code,
                              double* nl_rij, int* nl_cnt, int* err) {
  if (f.nloc <= 0) return;
  const size_t smem = format_smem_bytes(f);
  format_attr<k_format_candidates>(smem);
  count_launch();
  k_format_candidates<<<(f.nloc + kFmtWarps - 1) / kFmtWarps, kFmtWarps * 32, smem, st>>>(
      f, coord, atype, ilist, cand_start, cand, nl_j, nl_code, nl_rij, nl_cnt, err);
}

// ---------------------------------------------------------------- type partition
// Stable partition of local atoms by type: perm_pos[i] is atom i's row in the
// type-grouped order, perm_atom the inverse, type_start[t] the first row of t.
constexpr int kPartBlock = 1024;

size_t type_partition_blocks(int nloc) { return (size_t)(nloc + kPartBlock - 1) / kPartBlock; }

__global__ void __launch_bounds__(kPartBlock) k_type_count(int nloc, int ntypes, const int* __restrict__ atype,
                                                            int* __restrict__ blk_counts, int* __restrict__ err) {
  __shared__ int cnt[kMaxTypes];
  if (threadIdx.x < kMaxTypes) cnt[threadIdx.x] = 0;
  __syncthreads();
  const int i = blockIdx.x * kPartBlock + threadIdx.x;
  if (i < nloc) {
    const int t = atype[i];
    if (t >= 0 && t < ntypes)
      atomicAdd(cnt + t, 1);
    else
      atomicAdd(err + kErrBadType, 1);
  }
  __syncthreads();
  if (threadIdx.x < ntypes) blk_counts[blockIdx.x * ntypes + threadIdx.x] = cnt[threadIdx.x];
}

// One warp: per type, the blocks' counts in chunks of 32 by a warp scan (each
// count becomes its block's base), then type_start and the row tables.
__global__ void k_type_scan(int nblk, int ntypes, int* __restrict__ blk_counts, int* __restrict__ type_start,
                            RowTables tab) {
  if (blockIdx.x != 0) return;
  const int lane = threadIdx.x & 31;
  int base = 0;
  for (int t = 0; t < ntypes; ++t) {
    if (lane == 0) type_start[t] = base;
    for (int b0 = 0; b0 < nblk; b0 += 32) {
      const int b = b0 + lane;
      const int c = b < nblk ? blk_counts[b * ntypes + t] : 0;
      int incl = c;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
      }
      if (b < nblk) blk_counts[b * ntypes + t] = base + incl - c;
      base += __shfl_sync(0xffffffffu, incl, 31);
    }
  }
  if (lane != 0) return;
  type_start[ntypes] = base;
  __threadfence_block();
  if (tab.istart) {
    int acc = 0;
    tab.istart[0] = 0;
    for (int q = 0; q < tab.nnets; ++q) {
      const int ti = q / ntypes;
      const int rows = tab.tos ? base : type_start[ti + 1] - type_start[ti];
      const int items = (rows + tab.item_rows - 1) / tab.item_rows;
      acc += (items + tab.item_pad - 1) / tab.item_pad * tab.item_pad;
      tab.istart[q + 1] = acc;
    }
  }
  if (tab.ftile) {
    int acc = 0;
    tab.ftile[0] = 0;
    for (int t = 0; t < ntypes; ++t) {
      acc += (type_start[t + 1] - type_start[t] + 127) / 128;
      tab.ftile[t + 1] = acc;
    }
  }
}

__global__ void __launch_bounds__(kPartBlock) k_type_place(int nloc, int ntypes, const int* __restrict__ atype,
                                                            const int* __restrict__ blk_base,
                                                            int* __restrict__ perm_pos, int* __restrict__ perm_atom) {
  __shared__ int wcount[32][kMaxTypes];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int i = blockIdx.x * kPartBlock + threadIdx.x;
  const int t = (i < nloc) ? atype[i] : -1;
  const unsigned lt = (1u << lane) - 1u;
  int my_rank = 0;
  for (int q = 0; q < ntypes; ++q) {
    const unsigned m = __ballot_sync(0xffffffffu, t == q);
    if (t == q) my_rank = __popc(m & lt);
    if (lane == 0) wcount[warp][q] = __popc(m);
  }
  __syncthreads();
  if (threadIdx.x < ntypes) {
    int run = 0;
    for (int w = 0; w < 32; ++w) {
      const int c = wcount[w][threadIdx.x];
      wcount[w][threadIdx.x] = run;
      run += c;
    }
  }
  __syncthreads();
  if (i < nloc) {
    if (t >= 0 && t < ntypes) {
      const int pos = blk_base[blockIdx.x * ntypes + t] + wcount[warp][t] + my_rank;
      perm_pos[i] = pos;
      perm_atom[pos] = i;
    } else {
      perm_pos[i] = -1;  // invalid type: the model kernels skip this centre
    }
  }
}

void launch_type_partition(cudaStream_t st, int nloc, int ntypes, const int* atype, int* blk_counts,
                           int* type_start, int* perm_pos, int* perm_atom, int* err, const RowTables& tables) {
  const int nblk = (int)type_partition_blocks(nloc);
  if (nblk == 0) {
    cudaMemsetAsync(type_start, 0, sizeof(int) * (ntypes + 1), st);
    if (tables.istart) cudaMemsetAsync(tables.istart, 0, sizeof(int) * (tables.nnets + 1), st);
    if (tables.ftile) cudaMemsetAsync(tables.ftile, 0, sizeof(int) * (ntypes + 1), st);
    return;
  }
  count_launch();
  k_type_count<<<nblk, kPartBlock, 0, st>>>(nloc, ntypes, atype, blk_counts, err);
  count_launch();
  k_type_scan<<<1, 32, 0, st>>>(nblk, ntypes, blk_counts, type_start, tables);
  count_launch();
  k_type_place<<<nblk, kPartBlock, 0, st>>>(nloc, ntypes, atype, blk_counts, perm_pos, perm_atom);
}

}  // namespace b200dp
