// fp64 embedding forward and backward over the compacted edge lists (see
// embed_f64.cuh).
#include <algorithm>

#include "common.cuh"
#include "embed_f64.cuh"
#include "simt_gemm.cuh"

namespace b200dp {

namespace {

constexpr int kW = kF64Warps;
constexpr int kCh = 8;  // edges per chunk: the M (or N) extent of one m8n8k4 product

constexpr int resid(int din, int dout) { return dout == din ? 1 : (dout == 2 * din ? 2 : 0); }
// input feature feeding the residual of output n (DeePMD's identity / concat rule)
template <int DIN, int DOUT>
__device__ __forceinline__ int src_of(int n) {
  return resid(DIN, DOUT) == 1 ? n : (n < DIN ? n : n - DIN);
}

// tanh in fp64 from e^(2|x|) = 2^n e^r (Cody and Waite's reduction: n the nearest
// integer to 2|x| / ln 2, r = 2|x| - n ln 2 in two parts, ln 2 split after its
// 32nd significant bit so that n times the high part is exact), e^r by its Taylor
// series to degree 11 (|r| <= ln 2 / 2: remainder < 7e-15 relative), then
// 1 - 2 / (e^(2|x|) + 1) with the reciprocal from a single-precision estimate and
// two Newton steps.  Absolute error < 5e-15 over the real line (a host emulation
// of these steps against the C library's tanh on 220,000 points); 2|x| is capped
// at 80, where tanh is 1 in fp64.  About 30 fp64 operations.
__device__ __forceinline__ double tanh_d(double x) {
  constexpr double kLn2Hi = 0.6931471803691238, kLn2Lo = 1.9082149292705877e-10, kInvLn2 = 1.4426950408889634;
  const double y = fmin(2.0 * fabs(x), 80.0);
  const double n = rint(y * kInvLn2);
  double r = fma(-n, kLn2Hi, y);
  r = fma(-n, kLn2Lo, r);
  double p = 2.505210838544172e-08;          // 1/11!
  p = fma(p, r, 2.755731922398589e-07);      // 1/10!
  p = fma(p, r, 2.7557319223985893e-06);     // 1/9!
  p = fma(p, r, 2.48015873015873e-05);       // 1/8!
  p = fma(p, r, 0.0001984126984126984);      // 1/7!
  p = fma(p, r, 0.001388888888888889);       // 1/6!
  p = fma(p, r, 0.008333333333333333);       // 1/5!
  p = fma(p, r, 0.041666666666666664);       // 1/4!
  p = fma(p, r, 0.16666666666666666);        // 1/3!
  p = fma(p, r, 0.5);
  p = fma(p, r, 1.0);
  p = fma(p, r, 1.0);
  const double E = __longlong_as_double(__double_as_longlong(p) + ((long long)n << 52));
  const double d = E + 1.0;  // in [2, 6e34]
  float rf;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(rf) : "f"((float)d));
  double q = (double)rf;
  q = fma(q, fma(-d, q, 1.0), q);
  q = fma(q, fma(-d, q, 1.0), q);
  const double t = fma(-2.0, q, 1.0);
  return isnan(x) ? x : copysign(t, x);
}

// Environment row R~ = (sw/r, sw x/r^2, sw y/r^2, sw z/r^2) of one edge.
__device__ __forceinline__ void env_row64(const double* r, double rc, double rs, double* rt) {
  const double r2 = r[0] * r[0] + r[1] * r[1] + r[2] * r[2];
  const double rr = sqrt(r2);
  double sw, dsw;
  smooth_switch(rr, rs, rc, sw, dsw);
  const double inv_r = 1.0 / rr, inv_r2 = inv_r * inv_r;
  rt[0] = sw * inv_r;
#pragma unroll
  for (int c = 0; c < 3; ++c) rt[1 + c] = sw * r[c] * inv_r2;
}

// Padded extents of one net and its layout in shared memory (doubles): layer-1
// weights and biases, then W2, b2, W3, b3, every weight matrix in the swizzled
// 8 x 8 block layout of swz().
template <int D1, int D2, int D3>
struct Dims {
  static constexpr int K1 = (D1 + 7) / 8 * 8, F2 = (D2 + 7) / 8 * 8, P3 = (D3 + 7) / 8 * 8;
  static constexpr int NK = K1 / 8, NF = F2 / 8, NP = P3 / 8;
  static constexpr int W1 = 0, B1 = K1, W2 = 2 * K1, B2 = W2 + K1 * F2, W3 = B2 + F2, B3 = W3 + F2 * P3;
  static constexpr int NET = (B3 + P3 + 1) / 2 * 2;
};

// W[r][c] (r the layer input, c its output, both padded to multiples of 8) in
// 8 x 8 blocks, row-block major; inside a block, row ri starts at
// 16 ((ri & 1) + 2 (ri >> 2)) and is rotated by (ri & 1) + 8 ((ri >> 1) & 1) + 4 (ri >> 2)
// within its 16 doubles.  The two fragment patterns of the products,
//   A: r = 8i + 2 (lane & 3) + s, c = 8j + (lane >> 2)   (the input index is K)
//   B: r = 8i + (lane >> 2), c = 8j + 2 (lane & 3) + s   (the output index is K)
// then touch 16 distinct 8-byte bank pairs in each half warp, so one copy of the
// weights serves the forward products and the transposed backward products.
__host__ __device__ constexpr int swz_rot(int ri) { return (ri & 1) + 8 * ((ri >> 1) & 1) + 4 * (ri >> 2); }
__host__ __device__ constexpr int swz_row(int ri) { return 16 * ((ri & 1) + 2 * (ri >> 2)); }
__device__ __forceinline__ int swz(int r, int c, int nc8) {
  const int ri = r & 7, ci = c & 7;
  return 64 * ((r >> 3) * nc8 + (c >> 3)) + swz_row(ri) + ((ci + swz_rot(ri)) & 15);
}

// The net of pair q from the SIMT layout (W[k][n] row-major [din][dout] at
// w_off[l], biases at b_off[l]), zero-padded.
template <int D1, int D2, int D3>
__device__ void load_net_sw(double* net, const double* __restrict__ emb, const SeaDev& s, int q) {
  using Dm = Dims<D1, D2, D3>;
  const double* src = emb + (size_t)q * s.net_stride;
  for (int i = threadIdx.x; i < Dm::K1; i += blockDim.x) {
    net[Dm::W1 + i] = i < D1 ? src[s.w_off[0] + i] : 0.0;
    net[Dm::B1 + i] = i < D1 ? src[s.b_off[0] + i] : 0.0;
  }
  for (int i = threadIdx.x; i < Dm::K1 * Dm::F2; i += blockDim.x) {
    const int r = i / Dm::F2, c = i - r * Dm::F2;
    net[Dm::W2 + swz(r, c, Dm::NF)] = (r < D1 && c < D2) ? src[s.w_off[1] + r * D2 + c] : 0.0;
  }
  for (int i = threadIdx.x; i < Dm::F2; i += blockDim.x) net[Dm::B2 + i] = i < D2 ? src[s.b_off[1] + i] : 0.0;
  for (int i = threadIdx.x; i < Dm::F2 * Dm::P3; i += blockDim.x) {
    const int r = i / Dm::P3, c = i - r * Dm::P3;
    net[Dm::W3 + swz(r, c, Dm::NP)] = (r < D2 && c < D3) ? src[s.w_off[2] + r * D3 + c] : 0.0;
  }
  for (int i = threadIdx.x; i < Dm::P3; i += blockDim.x) net[Dm::B3 + i] = i < D3 ? src[s.b_off[2] + i] : 0.0;
}

// First work item whose first edge is at or after e (the items are in net
// order with non-decreasing first edges).
__device__ __forceinline__ int first_item_at(const TcLists& L, int nitems, long long e) {
  int lo = 0, hi = nitems;
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if ((long long)L.items[2 * mid].w < e)
      lo = mid + 1;
    else
      hi = mid;
  }
  return lo;
}

// One chunk's inputs (lanes 0-7, one edge each): environment row and slot;
// edges past ne get a zero row.
__device__ __forceinline__ void stage_chunk(const TcLists& L, const double* __restrict__ rij, const SeaDev& s,
                                            int c0, int ne, int lane, double* rt, int* slotS) {
  if (lane < kCh) {
    double r4[4] = {0.0, 0.0, 0.0, 0.0};
    int slot = -1;
    if (lane < ne) {
      slot = L.slot[c0 + lane];
      const double r[3] = {rij[3 * (size_t)slot], rij[3 * (size_t)slot + 1], rij[3 * (size_t)slot + 2]};
      env_row64(r, s.rcut, s.rcut_smth, r4);
    }
    *reinterpret_cast<double2*>(rt + 4 * lane) = make_double2(r4[0], r4[1]);
    *reinterpret_cast<double2*>(rt + 4 * lane + 2) = make_double2(r4[2], r4[3]);
    if (slotS) slotS[lane] = slot;
  }
}

// Lane offsets of the two fragment patterns inside a swizzled 8 x 8 block.
__device__ __forceinline__ void frag_offsets(int g, int t, int (&oA)[2], int (&oB)[2]) {
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int ri = 2 * t + h;
    oA[h] = swz_row(ri) + ((g + swz_rot(ri)) & 15);
    oB[h] = swz_row(g) + ((2 * t + h + swz_rot(g)) & 15);
  }
}

// Layers 1 and 2 of one chunk, shared by both kernels.  Lane (g, t) =
// (lane >> 2, lane & 3) owns edge g in the row-major fragments.  Layer 1 is
// formed directly in the A fragments of layer 2, with K permuted so that
// k-step (nk, h) holds feature 8 nk + 2t + h (the positions a C fragment
// holds); h2 stays in its C fragments (edge g, feature 8 nt + 2t + h), which
// the next product takes as an operand with the same permutation.  t1s[e][k]
// and h2s[e][f] keep the values other lanes need (residuals, derivatives).
template <int D1, int D2, int D3>
__device__ __forceinline__ void layers12(const double* net, const double* rt, double* t1s, double* h2s, int g, int t,
                                         const int (&oA)[2], double (&acc2)[Dims<D1, D2, D3>::NF][2]) {
  using Dm = Dims<D1, D2, D3>;
  constexpr int NK = Dm::NK, NF = Dm::NF, R2 = resid(D1, D2);
  const double sv = rt[4 * g];
  double a1[NK][2];
#pragma unroll
  for (int nk = 0; nk < NK; ++nk)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int k = 8 * nk + 2 * t + h;
      double v = 0.0;
      if (k < D1) {
        v = tanh_d(fma(sv, net[Dm::W1 + k], net[Dm::B1 + k]));
        t1s[g * D1 + k] = v;
      }
      a1[nk][h] = v;
    }
#pragma unroll
  for (int nt = 0; nt < NF; ++nt)
#pragma unroll
    for (int h = 0; h < 2; ++h) acc2[nt][h] = net[Dm::B2 + 8 * nt + 2 * t + h];
#pragma unroll
  for (int nk = 0; nk < NK; ++nk)
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
      for (int nt = 0; nt < NF; ++nt) dmma_8x8x4(acc2[nt], a1[nk][h], net[Dm::W2 + 64 * (nk * NF + nt) + oA[h]]);
  __syncwarp();  // t1s complete
#pragma unroll
  for (int nt = 0; nt < NF; ++nt)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int f = 8 * nt + 2 * t + h;
      double v = 0.0;
      if (f < D2) {
        v = tanh_d(acc2[nt][h]);
        if (R2 != 0) v += t1s[g * D1 + src_of<D1, D2>(f)];
        h2s[g * D2 + f] = v;
      }
      acc2[nt][h] = v;
    }
  __syncwarp();  // h2s complete
}

// Per-warp shared buffers (doubles).
template <int D1, int D2, int D3>
struct FwdWarp {
  static constexpr int TS = Dims<D1, D2, D3>::P3 + 4;  // T row stride: rows 2 apart land 8 bank pairs apart
  static constexpr int RT = 0, T1 = RT + 4 * kCh, H2 = T1 + kCh * D1, TA = H2 + kCh * D2,
                       SIZE = (TA + 4 * TS + 1) / 2 * 2;
};
template <int D1, int D2, int D3>
struct BwdWarp {
  static constexpr int RT = 0, T1 = RT + 4 * kCh, H2 = T1 + kCh * D1, DG = H2 + kCh * D2, SL = DG + kCh * D2,
                       SIZE = (SL + kCh / 2 + 1) / 2 * 2;  // slots: kCh ints
};

}  // namespace

// The [25, 50, 100] embedding (the water model); wider nets keep the SIMT path.
bool f64_tiled_supported(const SeaDev& s) {
  return s.nl == 3 && s.ed[1] == 25 && s.ed[2] == 50 && s.ed[3] == 100;
}

namespace {

// ---------------------------------------------------------------- forward
// One block per SM takes the work items whose first edges fall in its share of
// the edge list (consecutive items of one net form a segment: the net is loaded
// once per segment); its warps take the segment's centre rows one at a time (a
// shared counter), and a warp runs its row's edges in chunks of 8 through
//   layer 1 (scalar input), layer 2 (edges x features),
//   layer 3 transposed (G^T: positions x edges, so that G^T is the A operand of)
//   T^T[p][c] += sum_e G^T[p][e] R~[e][c]   (N = the 4 components, padded to 8).
// T of the row accumulates in shared memory in chunk order and is written once
// (rows without edges write zeros): results do not depend on which warp or
// block ran a row.
template <int D1, int D2, int D3>
__global__ void __launch_bounds__(32 * kW, 1) k_embed_fwd_f64(TcLists L, SeaDev s, const double* __restrict__ rij,
                                                             const double* __restrict__ emb, double* __restrict__ Tq) {
  using Dm = Dims<D1, D2, D3>;
  using Wb = FwdWarp<D1, D2, D3>;
  constexpr int NF = Dm::NF, NP = Dm::NP, TS = Wb::TS, R3 = resid(D2, D3);
  static_assert(resid(1, D1) == 0, "layer 1 without residual");
  static_assert((2 * TS) % 16 == 8, "T rows 2t and 2t + 2 on different bank pairs");
  extern __shared__ __align__(16) double sm[];
  __shared__ int s_next;
  double* net = sm;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
  double* wb = sm + Dm::NET + warp * Wb::SIZE;
  double* rt = wb + Wb::RT;
  double* t1s = wb + Wb::T1;
  double* h2s = wb + Wb::H2;
  double* tacc = wb + Wb::TA;
  int oA[2], oB[2];
  frag_offsets(g, t, oA, oB);
  const int nitems = L.istart[L.nnets];
  const long long E = L.eoff[(size_t)L.nnets * L.nloc];
  const int it0 = first_item_at(L, nitems, E * blockIdx.x / gridDim.x);
  const int it1 = blockIdx.x + 1 == gridDim.x ? nitems : first_item_at(L, nitems, E * (blockIdx.x + 1) / gridDim.x);
  for (int it = it0; it < it1;) {
    const int q = L.items[2 * it].x;
    int seg = it + 1;
    while (seg < it1 && L.items[2 * seg].x == q) ++seg;
    __syncthreads();  // the previous segment's rows are done with the net
    load_net_sw<D1, D2, D3>(net, emb, s, q);
    if (tid == 0) s_next = 0;
    __syncthreads();
    const int nslots = (seg - it) * kItemRows;
    for (;;) {
      int j = 0;
      if (lane == 0) j = atomicAdd(&s_next, 1);
      j = __shfl_sync(0xffffffffu, j, 0);
      if (j >= nslots) break;
      const int4 rec = L.items[2 * (it + j / kItemRows)];
      const int row = rec.y + j % kItemRows;
      if (row >= rec.z) continue;  // short or padding item
      const int rs = L.eoff[(size_t)q * L.nloc + row], re = L.eoff[(size_t)q * L.nloc + row + 1];
      __syncwarp();
      for (int i = lane; i < 4 * TS; i += 32) tacc[i] = 0.0;
      for (int c0 = rs; c0 < re; c0 += kCh) {
        __syncwarp();  // the previous chunk's readers are done
        stage_chunk(L, rij, s, c0, min(kCh, re - c0), lane, rt, nullptr);
        __syncwarp();
        double acc2[NF][2];
        layers12<D1, D2, D3>(net, rt, t1s, h2s, g, t, oA, acc2);
        // layer 3 transposed: lane holds G^T[p = 8 mt + g][e = 2t + h]
        double acc3[NP][2];
#pragma unroll
        for (int mt = 0; mt < NP; ++mt) acc3[mt][0] = acc3[mt][1] = net[Dm::B3 + 8 * mt + g];
#pragma unroll
        for (int kt = 0; kt < NF; ++kt)
#pragma unroll
          for (int h = 0; h < 2; ++h)
#pragma unroll
            for (int mt = 0; mt < NP; ++mt)
              dmma_8x8x4(acc3[mt], net[Dm::W3 + 64 * (kt * NP + mt) + oA[h]], acc2[kt][h]);
#pragma unroll
        for (int mt = 0; mt < NP; ++mt)
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int p = 8 * mt + g;
            double v = 0.0;
            if (p < D3) {
              v = tanh_d(acc3[mt][h]);
              if (R3 != 0) v += h2s[(2 * t + h) * D2 + src_of<D2, D3>(p)];
            }
            acc3[mt][h] = v;
          }
        // T^T[p][c] += sum_e G^T[p][e] R~[e][c]: k-step h takes edges 2t + h
        double bR[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) bR[h] = g < 4 ? rt[4 * (2 * t + h) + g] : 0.0;
#pragma unroll
        for (int mt = 0; mt < NP; ++mt) {
          const int p = 8 * mt + g;
          double tc[2];
          tc[0] = t < 2 ? tacc[(2 * t) * TS + p] : 0.0;
          tc[1] = t < 2 ? tacc[(2 * t + 1) * TS + p] : 0.0;
          dmma_8x8x4(tc, acc3[mt][0], bR[0]);
          dmma_8x8x4(tc, acc3[mt][1], bR[1]);
          if (t < 2) {
            tacc[(2 * t) * TS + p] = tc[0];
            tacc[(2 * t + 1) * TS + p] = tc[1];
          }
        }
      }
      __syncwarp();
      double* dst = Tq + ((size_t)q * L.nloc + row) * 4 * D3;
      for (int i = lane; i < 4 * D3; i += 32) {
        const int c = i / D3, p = i - c * D3;
        dst[i] = tacc[c * TS + p];
      }
    }
    it = seg;
  }
}

// T_i = sum over nets (fixed order) / N -> T (atom order), D = T^T T_< (row order).
template <int D3>
__global__ void k_t_combine_f64(TcLists L, int M2, double inv_nnei, const int* __restrict__ perm_atom,
                                const double* __restrict__ Tq, double* __restrict__ T, double* __restrict__ D) {
  __shared__ double sT[4 * D3];
  __shared__ int s_t;
  const int r = blockIdx.x;
  const int nrows = L.type_start[L.ntypes];
  if (r >= nrows) return;
  if (threadIdx.x == 0) {
    int t = 0;
    while (t + 1 < L.ntypes && L.type_start[t + 1] <= r) ++t;
    s_t = t;
  }
  __syncthreads();
  const int t = s_t;
  const int q0 = L.type_one_side ? 0 : t * L.ntypes;
  const int q1 = L.type_one_side ? L.nnets : q0 + L.ntypes;
  const int atom = perm_atom[r];
  for (int i = threadIdx.x; i < 4 * D3; i += blockDim.x) {
    double acc = 0.0;
    for (int q = q0; q < q1; ++q) acc += Tq[((size_t)q * L.nloc + r) * 4 * D3 + i];
    const double v = acc * inv_nnei;
    sT[i] = v;
    T[(size_t)atom * 4 * D3 + i] = v;
  }
  __syncthreads();
  double* drow = D + (size_t)r * D3 * M2;
  for (int idx = threadIdx.x; idx < D3 * M2; idx += blockDim.x) {
    const int a = idx / M2, b = idx - a * M2;
    double acc = 0.0;
#pragma unroll
    for (int k = 0; k < 4; ++k) acc += sT[k * D3 + a] * sT[k * D3 + b];
    drow[idx] = acc;
  }
}

// dT[row][k][a] = (sum_b dD[a][b] T[k][b] + [a < M2] sum_c dD[c][a] T[k][c]) / N
template <int D3>
__global__ void k_dT_f64(int nloc, int ntypes, int M2, double inv_nnei, const int* __restrict__ type_start,
                         const int* __restrict__ perm_atom, const double* __restrict__ T,
                         const double* __restrict__ dD, double* __restrict__ dT) {
  extern __shared__ double sd[];
  double* sT = sd;            // 4 D3
  double* sdD = sd + 4 * D3;  // D3 rows of (M2 + 1)
  const int r = blockIdx.x;
  if (r >= type_start[ntypes]) return;
  const int atom = perm_atom[r];
  const int ld = M2 + 1;
  for (int i = threadIdx.x; i < 4 * D3; i += blockDim.x) sT[i] = T[(size_t)atom * 4 * D3 + i];
  const double* src = dD + (size_t)r * D3 * M2;
  for (int i = threadIdx.x; i < D3 * M2; i += blockDim.x) {
    const int a = i / M2, b = i - a * M2;
    sdD[a * ld + b] = src[i];
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < 4 * D3; idx += blockDim.x) {
    const int k = idx / D3, a = idx - k * D3;
    const double* tk = sT + k * D3;
    double acc = 0.0;
    for (int b = 0; b < M2; ++b) acc += sdD[a * ld + b] * tk[b];
    if (a < M2)
      for (int c = 0; c < D3; ++c) acc += sdD[c * ld + a] * tk[c];
    dT[(size_t)r * 4 * D3 + idx] = acc * inv_nnei;
  }
}

// ---------------------------------------------------------------- backward
// Same division of work as the forward.  Per chunk: layers 1-3 recomputed
// (layer 3 row-major this time: lane holds z3[e = g][p = 8 nt + 2t + h]), then
//   dG[e][p] = sum_c R~[e][c] dT[row][c][p],  dR~[e][c] = sum_p G[e][p] dT[row][c][p]
//   dz3 = dG (1 - t3^2);  dh2 = dz3 W3^T + residual(dG);  dz2 = dh2 (1 - t2^2)
//   dh1 = dz2 W2^T + residual(dh2);  dz1 = dh1 (1 - t1^2);  dE/ds = dz1 . w1
// with dz3 and dz2 taken from their C fragments as the A operands of the next
// products (the weights' transposed fragments come from the same swizzled
// copy), and per slot the environment-row gradient (dR~_0 + dE/ds, dR~_1..3)
// for the assembly's chain rule.  The tanh outputs of layers 1 and 2 are
// recovered from the stored layer outputs.
template <int D1, int D2, int D3>
__global__ void __launch_bounds__(32 * kW, 1) k_embed_bwd_f64(TcLists L, SeaDev s, const double* __restrict__ rij,
                                                             const double* __restrict__ emb,
                                                             const double* __restrict__ dT, double* __restrict__ genv) {
  using Dm = Dims<D1, D2, D3>;
  using Wb = BwdWarp<D1, D2, D3>;
  constexpr int NK = Dm::NK, NF = Dm::NF, NP = Dm::NP, R2 = resid(D1, D2), R3 = resid(D2, D3);
  static_assert(resid(1, D1) == 0, "layer 1 without residual");
  static_assert(D3 % 2 == 0, "dT pairs as 16-byte loads");
  extern __shared__ __align__(16) double sm[];
  __shared__ int s_next;
  double* net = sm;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
  double* wb = sm + Dm::NET + warp * Wb::SIZE;
  double* rt = wb + Wb::RT;
  double* t1s = wb + Wb::T1;
  double* h2s = wb + Wb::H2;
  double* dgs = wb + Wb::DG;  // dG[e][D2 + f], later dh2[e][f]
  int* slotS = reinterpret_cast<int*>(wb + Wb::SL);
  int oA[2], oB[2];
  frag_offsets(g, t, oA, oB);
  const int nitems = L.istart[L.nnets];
  const long long E = L.eoff[(size_t)L.nnets * L.nloc];
  const int it0 = first_item_at(L, nitems, E * blockIdx.x / gridDim.x);
  const int it1 = blockIdx.x + 1 == gridDim.x ? nitems : first_item_at(L, nitems, E * (blockIdx.x + 1) / gridDim.x);
  for (int it = it0; it < it1;) {
    const int q = L.items[2 * it].x;
    int seg = it + 1;
    while (seg < it1 && L.items[2 * seg].x == q) ++seg;
    __syncthreads();
    load_net_sw<D1, D2, D3>(net, emb, s, q);
    if (tid == 0) s_next = 0;
    __syncthreads();
    const int nslots = (seg - it) * kItemRows;
    for (;;) {
      int j = 0;
      if (lane == 0) j = atomicAdd(&s_next, 1);
      j = __shfl_sync(0xffffffffu, j, 0);
      if (j >= nslots) break;
      const int4 rec = L.items[2 * (it + j / kItemRows)];
      const int row = rec.y + j % kItemRows;
      if (row >= rec.z) continue;
      const int rs = L.eoff[(size_t)q * L.nloc + row], re = L.eoff[(size_t)q * L.nloc + row + 1];
      const double* dtr = dT + (size_t)row * 4 * D3;
      for (int c0 = rs; c0 < re; c0 += kCh) {
        const int ne = min(kCh, re - c0);
        __syncwarp();
        stage_chunk(L, rij, s, c0, ne, lane, rt, slotS);
        __syncwarp();
        double acc2[NF][2];
        layers12<D1, D2, D3>(net, rt, t1s, h2s, g, t, oA, acc2);
        // layer 3: lane holds z3[e = g][p = 8 nt + 2t + h]
        double acc3[NP][2];
#pragma unroll
        for (int nt = 0; nt < NP; ++nt)
#pragma unroll
          for (int h = 0; h < 2; ++h) acc3[nt][h] = net[Dm::B3 + 8 * nt + 2 * t + h];
#pragma unroll
        for (int kt = 0; kt < NF; ++kt)
#pragma unroll
          for (int h = 0; h < 2; ++h)
#pragma unroll
            for (int nt = 0; nt < NP; ++nt)
              dmma_8x8x4(acc3[nt], acc2[kt][h], net[Dm::W3 + 64 * (kt * NP + nt) + oA[h]]);
        // dG, dR~ (partial over this lane's positions), dz3; the residual
        // gradient of layer 3 starts dh2 (own positions directly, the concat
        // rule's second half through dgs)
        const double2 ra = *reinterpret_cast<const double2*>(rt + 4 * g);
        const double2 rb = *reinterpret_cast<const double2*>(rt + 4 * g + 2);
        double qv[4] = {0.0, 0.0, 0.0, 0.0};
        double dh2[NF][2];
#pragma unroll
        for (int nt = 0; nt < NF; ++nt) dh2[nt][0] = dh2[nt][1] = 0.0;
#pragma unroll
        for (int nt = 0; nt < NP; ++nt) {
          const int p0 = 8 * nt + 2 * t;
          double2 d[4];
#pragma unroll
          for (int c = 0; c < 4; ++c)
            d[c] = p0 < D3 ? __ldg(reinterpret_cast<const double2*>(dtr + c * D3 + p0)) : make_double2(0.0, 0.0);
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int p = p0 + h;
            double dz = 0.0;
            if (p < D3) {
              const double d0 = h ? d[0].y : d[0].x, d1 = h ? d[1].y : d[1].x, d2 = h ? d[2].y : d[2].x,
                           d3 = h ? d[3].y : d[3].x;
              const double t3 = tanh_d(acc3[nt][h]);
              const double G = R3 != 0 ? t3 + h2s[g * D2 + src_of<D2, D3>(p)] : t3;
              const double dg = ((ra.x * d0 + ra.y * d1) + rb.x * d2) + rb.y * d3;
              qv[0] = fma(G, d0, qv[0]);
              qv[1] = fma(G, d1, qv[1]);
              qv[2] = fma(G, d2, qv[2]);
              qv[3] = fma(G, d3, qv[3]);
              if (R3 != 0) {
                if (p < D2) {
                  if (nt < NF) dh2[nt < NF ? nt : 0][h] += dg;
                } else {
                  dgs[g * D2 + (p - D2)] = dg;
                }
              }
              dz = dg * (1.0 - t3 * t3);
            }
            acc3[nt][h] = dz;
          }
        }
        __syncwarp();  // dgs complete
        if (R3 == 2) {
#pragma unroll
          for (int nt = 0; nt < NF; ++nt)
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const int f = 8 * nt + 2 * t + h;
              if (f < D2) dh2[nt][h] += dgs[g * D2 + f];
            }
        }
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          qv[c] += __shfl_xor_sync(0xffffffffu, qv[c], 1);
          qv[c] += __shfl_xor_sync(0xffffffffu, qv[c], 2);
        }
        // dh2 += dz3 W3^T (K = positions: k-step (kt, h) holds 8 kt + 2t + h)
#pragma unroll
        for (int kt = 0; kt < NP; ++kt)
#pragma unroll
          for (int h = 0; h < 2; ++h)
#pragma unroll
            for (int nt = 0; nt < NF; ++nt)
              dmma_8x8x4(dh2[nt], acc3[kt][h], net[Dm::W3 + 64 * (nt * NP + kt) + oB[h]]);
        __syncwarp();  // every lane has read dgs
        // dz2 = dh2 (1 - t2^2); dh2 to dgs for the layer-2 residual of dh1
#pragma unroll
        for (int nt = 0; nt < NF; ++nt)
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int f = 8 * nt + 2 * t + h;
            double dz = 0.0;
            if (f < D2) {
              const double dh = dh2[nt][h];
              if (R2 != 0) dgs[g * D2 + f] = dh;
              const double t2 = R2 != 0 ? h2s[g * D2 + f] - t1s[g * D1 + src_of<D1, D2>(f)] : h2s[g * D2 + f];
              dz = dh * (1.0 - t2 * t2);
            }
            dh2[nt][h] = dz;
          }
        __syncwarp();  // dh2 in dgs
        double dh1[NK][2];
#pragma unroll
        for (int nk = 0; nk < NK; ++nk)
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int k = 8 * nk + 2 * t + h;
            double v = 0.0;
            if (k < D1) {
              if (R2 == 2) v = dgs[g * D2 + k] + dgs[g * D2 + k + D1];
              if (R2 == 1) v = dgs[g * D2 + k];
            }
            dh1[nk][h] = v;
          }
#pragma unroll
        for (int kt = 0; kt < NF; ++kt)
#pragma unroll
          for (int h = 0; h < 2; ++h)
#pragma unroll
            for (int nk = 0; nk < NK; ++nk)
              dmma_8x8x4(dh1[nk], dh2[kt][h], net[Dm::W2 + 64 * (nk * NF + kt) + oB[h]]);
        // dz1 = dh1 (1 - t1^2), dE/ds = dz1 . w1 (this lane's features, then the quad)
        double ds = 0.0;
#pragma unroll
        for (int nk = 0; nk < NK; ++nk)
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int k = 8 * nk + 2 * t + h;
            if (k < D1) {
              const double t1 = t1s[g * D1 + k];
              ds = fma(dh1[nk][h] * (1.0 - t1 * t1), net[Dm::W1 + k], ds);
            }
          }
        ds += __shfl_xor_sync(0xffffffffu, ds, 1);
        ds += __shfl_xor_sync(0xffffffffu, ds, 2);
        if (g < ne) {
          const double v = t == 0 ? qv[0] + ds : (t == 1 ? qv[1] : (t == 2 ? qv[2] : qv[3]));
          genv[4 * (size_t)slotS[g] + t] = v;
        }
      }
    }
    it = seg;
  }
}

template <class K>
void allow_smem(K kern, size_t smem) {
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
}

template <int D1, int D2, int D3>
size_t fwd_smem() {
  return sizeof(double) * (Dims<D1, D2, D3>::NET + (size_t)kW * FwdWarp<D1, D2, D3>::SIZE);
}
template <int D1, int D2, int D3>
size_t bwd_smem() {
  return sizeof(double) * (Dims<D1, D2, D3>::NET + (size_t)kW * BwdWarp<D1, D2, D3>::SIZE);
}

template <int D1, int D2, int D3>
void run_fwd(cudaStream_t st, const SeaDev& s, const TcLists& L, int grid, const double* rij, const double* emb,
             double* Tq, double* T, double* D, const int* perm_atom, int nloc) {
  const size_t smem = fwd_smem<D1, D2, D3>();
  static bool attr = false;
  if (!attr) {
    allow_smem(k_embed_fwd_f64<D1, D2, D3>, smem);
    attr = true;
  }
  count_launch();
  k_embed_fwd_f64<D1, D2, D3><<<grid, 32 * kW, smem, st>>>(L, s, rij, emb, Tq);
  count_launch();
  k_t_combine_f64<D3><<<nloc, 256, 0, st>>>(L, s.M2, s.inv_nnei, perm_atom, Tq, T, D);
}

template <int D1, int D2, int D3>
void run_bwd(cudaStream_t st, const SeaDev& s, const TcLists& L, int grid, const double* rij, const double* emb,
             const double* T, const double* dD, double* dT, double* genv, const int* type_start,
             const int* perm_atom, int nloc) {
  const size_t dsm = sizeof(double) * (4 * D3 + (size_t)D3 * (s.M2 + 1));
  static size_t dattr = 0;
  if (dsm > dattr) {
    allow_smem(k_dT_f64<D3>, dsm);
    dattr = dsm;
  }
  count_launch();
  k_dT_f64<D3><<<nloc, 128, dsm, st>>>(nloc, s.ntypes, s.M2, s.inv_nnei, type_start, perm_atom, T, dD, dT);
  const size_t smem = bwd_smem<D1, D2, D3>();
  static bool attr = false;
  if (!attr) {
    allow_smem(k_embed_bwd_f64<D1, D2, D3>, smem);
    attr = true;
  }
  count_launch();
  k_embed_bwd_f64<D1, D2, D3><<<grid, 32 * kW, smem, st>>>(L, s, rij, emb, dT, genv);
}

}  // namespace

int embed_f64_grid(const SeaDev& s, bool backward) {
  (void)s;
  (void)backward;
  int dev = 0, nsm = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
  return nsm;  // one block of kF64Warps warps per SM
}

void launch_embed_fwd_f64(cudaStream_t st, const SeaDev& s, const TcLists& L, int grid, const double* rij,
                          const double* emb, double* Tq, double* T, double* D, const int* perm_atom, int nloc) {
  if (nloc <= 0) return;
  run_fwd<25, 50, 100>(st, s, L, grid, rij, emb, Tq, T, D, perm_atom, nloc);
}

void launch_embed_bwd_f64(cudaStream_t st, const SeaDev& s, const TcLists& L, int grid, const double* rij,
                          const double* emb, const double* T, const double* dD, double* dT, double* genv,
                          const int* type_start, const int* perm_atom, int nloc) {
  if (nloc <= 0) return;
  run_bwd<25, 50, 100>(st, s, L, grid, rij, emb, T, dD, dT, genv, type_start, perm_atom, nloc);
}

}  // namespace b200dp
