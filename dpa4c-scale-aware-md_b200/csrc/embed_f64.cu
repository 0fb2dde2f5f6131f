// fp64 embedding forward and backward over the compacted edge lists (see
// embed_f64.cuh).
#include <algorithm>

#include "common.cuh"
#include "embed_f64.cuh"

namespace b200dp {

namespace {

constexpr int kE = kF64Edges;  // edges per subtile
constexpr int kT = kF64Threads;

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

// One net in shared memory (the layout of the SIMT weights: W[k][n] row-major, then b).
template <int D1, int D2, int D3>
struct F64Net {
  static constexpr int W1 = 0, B1 = D1, W2 = 2 * D1, B2 = W2 + D1 * D2, W3 = B2 + D2, B3 = W3 + D2 * D3;
  static constexpr int N = (B3 + D3 + 1) / 2 * 2;  // doubles, even (16-byte aligned regions after it)
};

__device__ __forceinline__ void load_net(double* dst, const double* __restrict__ emb, const SeaDev& s, int q,
                                         int d1, int d2, int d3) {
  const double* src = emb + (size_t)q * s.net_stride;
  // the SIMT layout: layer l weights at w_off[l] ([din][dout]), biases at b_off[l]
  const int W1 = 0, B1 = d1, W2 = 2 * d1, B2 = W2 + d1 * d2, W3 = B2 + d2, B3 = W3 + d2 * d3;
  for (int i = threadIdx.x; i < d1; i += blockDim.x) {
    dst[W1 + i] = src[s.w_off[0] + i];
    dst[B1 + i] = src[s.b_off[0] + i];
  }
  for (int i = threadIdx.x; i < d1 * d2; i += blockDim.x) dst[W2 + i] = src[s.w_off[1] + i];
  for (int i = threadIdx.x; i < d2; i += blockDim.x) dst[B2 + i] = src[s.b_off[1] + i];
  for (int i = threadIdx.x; i < d2 * d3; i += blockDim.x) dst[W3 + i] = src[s.w_off[2] + i];
  for (int i = threadIdx.x; i < d3; i += blockDim.x) dst[B3 + i] = src[s.b_off[2] + i];
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

// Item record {net, first row, end row, first edge}, {end edge}.
struct F64Item {
  int q, rb, re, e0, e1;
};
__device__ __forceinline__ F64Item item_at(const TcLists& L, int it) {
  const int4 a = L.items[2 * it], b = L.items[2 * it + 1];
  return F64Item{a.x, a.y, a.z, a.w, b.x};
}

// Subtile inputs: slot, centre row (relative to the item) and environment row
// of each edge; edges past ne get a zero row.
__device__ __forceinline__ void stage_edges(const TcLists& L, const double* __restrict__ rij, const SeaDev& s,
                                            int sub, int ne, int rb, double* rtS, int* rowS, int* slotS) {
  for (int e = threadIdx.x; e < kE; e += blockDim.x) {
    double rt[4] = {0.0, 0.0, 0.0, 0.0};
    int row = 0, slot = -1;
    if (e < ne) {
      slot = L.slot[sub + e];
      row = L.row[sub + e] - rb;
      const double r[3] = {rij[3 * (size_t)slot], rij[3 * (size_t)slot + 1], rij[3 * (size_t)slot + 2]};
      env_row64(r, s.rcut, s.rcut_smth, rt);
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) rtS[4 * e + k] = rt[k];
    rowS[e] = row;
    if (slotS) slotS[e] = slot;
  }
}

// outT[n][e] = tanh(sum_k inT[k][e] W[k][n] + b[n]) (+ residual inT[src(n)][e]),
// thread tiles of 4 edges x TN outputs (TN = 2 for narrow layers, so that the
// block's threads have work); consecutive threads take consecutive edge groups
// (the weight loads of a warp then hit few addresses).
template <int DIN, int DOUT, int TN = 4>
__device__ __forceinline__ void dense_fwd(const double* inT, const double* W, const double* b, double* outT) {
  constexpr int EG = kE / 4, NG = (DOUT + TN - 1) / TN;
  constexpr int RM = resid(DIN, DOUT);
  for (int it = threadIdx.x; it < EG * NG; it += blockDim.x) {
    const int e0 = (it % EG) * 4, n0 = (it / EG) * TN;
    double acc[4][TN];
#pragma unroll
    for (int j = 0; j < TN; ++j) {
      const double bj = n0 + j < DOUT ? b[n0 + j] : 0.0;
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[i][j] = bj;
    }
#pragma unroll 5
    for (int k = 0; k < DIN; ++k) {
      const double2 xa = *reinterpret_cast<const double2*>(inT + k * kE + e0);
      const double2 xb = *reinterpret_cast<const double2*>(inT + k * kE + e0 + 2);
      const double x[4] = {xa.x, xa.y, xb.x, xb.y};
      double w[TN];
#pragma unroll
      for (int j = 0; j < TN; ++j) w[j] = n0 + j < DOUT ? W[k * DOUT + n0 + j] : 0.0;
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j) acc[i][j] = fma(x[i], w[j], acc[i][j]);
    }
#pragma unroll
    for (int j = 0; j < TN; ++j) {
      const int n = n0 + j;
      if (n >= DOUT) break;
      double h[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        h[i] = tanh_d(acc[i][j]);
        if (RM != 0) h[i] += inT[src_of<DIN, DOUT>(n) * kE + e0 + i];
      }
      *reinterpret_cast<double2*>(outT + n * kE + e0) = make_double2(h[0], h[1]);
      *reinterpret_cast<double2*>(outT + n * kE + e0 + 2) = make_double2(h[2], h[3]);
    }
  }
}

// First layer from the scalar input s = R~_0 (no residual: D1 > 2).
template <int D1>
__device__ __forceinline__ void layer1(const double* rtS, const double* net, double* A1T) {
  for (int i = threadIdx.x; i < D1 * kE; i += blockDim.x) {
    const int n = i / kE, e = i - n * kE;
    A1T[i] = tanh_d(rtS[4 * e] * net[n] + net[D1 + n]);
  }
}

}  // namespace

// The [25, 50, 100] embedding (the water model); wider nets keep the SIMT path
// (their backward's working set does not fit one block's shared memory).
bool f64_tiled_supported(const SeaDev& s) {
  return s.nl == 3 && s.ed[1] == 25 && s.ed[2] == 50 && s.ed[3] == 100;
}

namespace {

// ---------------------------------------------------------------- forward
// One block per item at a time (persistent over the items): the item's net
// in shared memory, its edges in subtiles of kE, layers 1-3 as register-tiled
// fp64 GEMMs over the subtile, then T[row][k][p] += R~[e][k] G[e][p] with
// one thread per (position, component pair) summing its edges in list order
// (fixed order: results are run-to-run identical).
template <int D1, int D2, int D3>
struct FwdSmem {
  static constexpr int NET = F64Net<D1, D2, D3>::N;
  static constexpr int RT = NET, A1 = RT + 4 * kE, A2 = A1 + D1 * kE, G = A2 + D2 * kE, END = G + D3 * kE;
  static constexpr size_t BYTES = (size_t)END * sizeof(double) + kE * sizeof(int);
};

template <int D1, int D2, int D3>
__global__ void __launch_bounds__(kT) k_embed_fwd_f64(TcLists L, SeaDev s, const double* __restrict__ rij,
                                                     const double* __restrict__ emb, double* __restrict__ Tq) {
  using N = F64Net<D1, D2, D3>;
  using S = FwdSmem<D1, D2, D3>;
  static_assert(resid(1, D1) == 0, "layer 1 without residual");
  static_assert(2 * D3 <= kT, "one thread per (position, component pair)");
  extern __shared__ __align__(16) double sm[];
  double* net = sm;
  double* rtS = sm + S::RT;
  double* A1T = sm + S::A1;
  double* A2T = sm + S::A2;
  double* GT = sm + S::G;
  int* rowS = reinterpret_cast<int*>(sm + S::END);
  const int tid = threadIdx.x;
  const int nitems = L.istart[L.nnets];
  const int p = tid % D3, kp = 2 * (tid / D3);  // contraction role (tid < 2 D3)
  int loaded = -1;
  for (int it = blockIdx.x; it < nitems; it += gridDim.x) {
    const F64Item I = item_at(L, it);
    if (I.re <= I.rb) continue;  // padding item (block-uniform); rows without edges still write zeros
    if (I.q != loaded) {
      __syncthreads();
      load_net(net, emb, s, I.q, D1, D2, D3);
      loaded = I.q;
    }
    double tacc[kItemRows][2];
#pragma unroll
    for (int r = 0; r < kItemRows; ++r) tacc[r][0] = tacc[r][1] = 0.0;
    for (int sub = I.e0; sub < I.e1; sub += kE) {
      const int ne = min(kE, I.e1 - sub);
      __syncthreads();  // the previous subtile's readers are done
      stage_edges(L, rij, s, sub, ne, I.rb, rtS, rowS, nullptr);
      __syncthreads();
      layer1<D1>(rtS, net + N::W1, A1T);
      __syncthreads();
      dense_fwd<D1, D2, 2>(A1T, net + N::W2, net + N::B2, A2T);
      __syncthreads();
      dense_fwd<D2, D3>(A2T, net + N::W3, net + N::B3, GT);
      __syncthreads();
      if (tid < 2 * D3) {
        // edges in list order; the running sum of a row goes to its slot when the row changes
        double c0 = 0.0, c1 = 0.0;
        int cur = rowS[0];
        for (int e = 0; e < ne; ++e) {
          const int r = rowS[e];
          if (r != cur) {
#pragma unroll
            for (int rr = 0; rr < kItemRows; ++rr)
              if (rr == cur) {
                tacc[rr][0] += c0;
                tacc[rr][1] += c1;
              }
            c0 = c1 = 0.0;
            cur = r;
          }
          const double g = GT[p * kE + e];
          c0 = fma(rtS[4 * e + kp], g, c0);
          c1 = fma(rtS[4 * e + kp + 1], g, c1);
        }
#pragma unroll
        for (int rr = 0; rr < kItemRows; ++rr)
          if (rr == cur) {
            tacc[rr][0] += c0;
            tacc[rr][1] += c1;
          }
      }
    }
    if (tid < 2 * D3) {
      for (int r = 0; r < I.re - I.rb; ++r) {
        double* dst = Tq + (((size_t)I.q * L.nloc + I.rb + r) * 4 + kp) * D3 + p;
        double v0 = 0.0, v1 = 0.0;
#pragma unroll
        for (int rr = 0; rr < kItemRows; ++rr)
          if (rr == r) {
            v0 = tacc[rr][0];
            v1 = tacc[rr][1];
          }
        dst[0] = v0;
        dst[D3] = v1;
      }
    }
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
// Per subtile: the forward recomputed (as above), then
//   dG[e][p] = sum_k R~[e][k] dT[row][k][p],  dR~[e][k] = sum_p G[e][p] dT[row][k][p]
//   dz3 = dG (1 - t3^2);  dh2 = dz3 W3^T + residual(dG);  dz2 = dh2 (1 - t2^2)
//   dh1 = dz2 W2^T + residual(dh2);  dz1 = dh1 (1 - t1^2);  dE/ds = dz1 . w1
// and per slot the environment-row gradient (dR~_0 + dE/ds, dR~_1..3) for the
// assembly's chain rule.  The tanh outputs are recovered from the layer
// outputs minus their residual inputs.
template <int D1, int D2, int D3>
struct BwdSmem {
  // G is overwritten by dz3 in place, the residual gradient of layer 3 goes to the
  // dz2 region (each element read back by the thread that writes dz2 over it),
  // the partial dR~ wait in registers until the dz3 region is free again, and dT
  // is read from global memory (L2): two blocks share an SM
  static constexpr int NET = F64Net<D1, D2, D3>::N;
  static constexpr int RT = NET, A1 = RT + 4 * kE, A2 = A1 + D1 * kE, G = A2 + D2 * kE, Z2 = G + D3 * kE,
                       END = Z2 + D2 * kE;
  static constexpr size_t BYTES = (size_t)END * sizeof(double) + 2 * kE * sizeof(int);
};

// gxT[m][e] = sum_n gzT[n][e] W[m][n] (the transposed product of a layer with
// weights W[DIN][DOUT]); thread tiles of 4 edges x 4 inputs m.
template <int DIN, int DOUT>
__device__ __forceinline__ void dense_bwd_tile(const double* gzT, const double* W, int it, double (&acc)[4][4],
                                               int& e0, int& m0) {
  constexpr int EG = kE / 4;
  e0 = (it % EG) * 4;
  m0 = (it / EG) * 4;
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.0;
#pragma unroll 4
  for (int n = 0; n < DOUT; ++n) {
    const double2 za = *reinterpret_cast<const double2*>(gzT + n * kE + e0);
    const double2 zb = *reinterpret_cast<const double2*>(gzT + n * kE + e0 + 2);
    const double z[4] = {za.x, za.y, zb.x, zb.y};
    double w[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) w[j] = m0 + j < DIN ? W[(m0 + j) * DOUT + n] : 0.0;
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[i][j] = fma(z[i], w[j], acc[i][j]);
  }
}

template <int D1, int D2, int D3>
__global__ void __launch_bounds__(kT, 2) k_embed_bwd_f64(TcLists L, SeaDev s, const double* __restrict__ rij,
                                                        const double* __restrict__ emb, const double* __restrict__ dT,
                                                        double* __restrict__ genv) {
  using N = F64Net<D1, D2, D3>;
  using S = BwdSmem<D1, D2, D3>;
  constexpr int R2 = resid(D1, D2), R3 = resid(D2, D3);
  static_assert(resid(1, D1) == 0, "layer 1 without residual");
  extern __shared__ __align__(16) double sm[];
  double* net = sm;
  double* rtS = sm + S::RT;   // [e][4]
  double* A1T = sm + S::A1;   // t1, later dz1
  double* A2T = sm + S::A2;   // h2, later dh2
  double* GT = sm + S::G;     // G, then dz3, then the partial dR~ [warp][e][4]
  double* Z2T = sm + S::Z2;   // residual gradient of layer 3, then dz2
  int* rowS = reinterpret_cast<int*>(sm + S::END);
  int* slotS = rowS + kE;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  constexpr int NW = kT / 32;
  static_assert(kE == 32, "one lane per edge in the dG pass");
  static_assert(NW * kE * 4 <= D3 * kE, "the partial dR~ fit the dz3 region");
  const int nitems = L.istart[L.nnets];
  int loaded = -1;
  for (int it = blockIdx.x; it < nitems; it += gridDim.x) {
    const F64Item I = item_at(L, it);
    if (I.e1 <= I.e0) continue;
    __syncthreads();
    if (I.q != loaded) {
      load_net(net, emb, s, I.q, D1, D2, D3);
      loaded = I.q;
    }
    for (int sub = I.e0; sub < I.e1; sub += kE) {
      const int ne = min(kE, I.e1 - sub);
      __syncthreads();
      stage_edges(L, rij, s, sub, ne, I.rb, rtS, rowS, slotS);
      __syncthreads();
      layer1<D1>(rtS, net + N::W1, A1T);
      __syncthreads();
      dense_fwd<D1, D2, 2>(A1T, net + N::W2, net + N::B2, A2T);
      __syncthreads();
      dense_fwd<D2, D3>(A2T, net + N::W3, net + N::B3, GT);
      __syncthreads();
      // dG, dz3 (over G), the residual gradient into layer 2, partial dR~:
      // lane = edge, warps over positions; the positions that share a residual
      // source (s and s + D2 under the concat rule) go to the same thread
      const int e = lane, row = rowS[e];
      const double r0 = rtS[4 * e], r1 = rtS[4 * e + 1], r2 = rtS[4 * e + 2], r3 = rtS[4 * e + 3];
      const double* dtr = dT + (size_t)(I.rb + row) * 4 * D3;
      double q0 = 0.0, q1 = 0.0, q2 = 0.0, q3 = 0.0;
      auto position = [&](int p, double base) -> double {  // returns dG
        const double d0 = __ldg(dtr + p), d1 = __ldg(dtr + D3 + p), d2 = __ldg(dtr + 2 * D3 + p),
                     d3 = __ldg(dtr + 3 * D3 + p);
        const double g = GT[p * kE + e];
        const double dg = ((r0 * d0 + r1 * d1) + r2 * d2) + r3 * d3;
        q0 = fma(g, d0, q0);
        q1 = fma(g, d1, q1);
        q2 = fma(g, d2, q2);
        q3 = fma(g, d3, q3);
        const double t3 = g - base;
        GT[p * kE + e] = dg * (1.0 - t3 * t3);
        return dg;
      };
      if constexpr (R3 == 2) {
        for (int sp = warp; sp < D2; sp += NW) {
          const double h2 = A2T[sp * kE + e];
          const double ga = position(sp, h2), gb = position(sp + D2, h2);
          Z2T[sp * kE + e] = ga + gb;
        }
      } else if constexpr (R3 == 1) {
        for (int p = warp; p < D3; p += NW) Z2T[p * kE + e] = position(p, A2T[p * kE + e]);
      } else {
        for (int p = warp; p < D3; p += NW) position(p, 0.0);
      }
      __syncthreads();
      // dh2 = dz3 W3^T + residual of layer 3; dz2 = dh2 (1 - t2^2)
      for (int it2 = tid; it2 < (kE / 4) * ((D2 + 3) / 4); it2 += kT) {
        double acc[4][4];
        int e0, m0;
        dense_bwd_tile<D2, D3>(GT, net + N::W3, it2, acc, e0, m0);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int m = m0 + j;
          if (m >= D2) break;
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int ee = e0 + i;
            double dh = acc[i][j];
            if (R3 != 0) dh += Z2T[m * kE + ee];
            const double h2 = A2T[m * kE + ee];
            const double t2 = R2 != 0 ? h2 - A1T[src_of<D1, D2>(m) * kE + ee] : h2;
            Z2T[m * kE + ee] = dh * (1.0 - t2 * t2);  // over the residual gradient read above
            A2T[m * kE + ee] = dh;                     // read above by this thread only
          }
        }
      }
      __syncthreads();
      {  // the dz3 region is free: the partial dR~ of this warp
        double* pr = GT + (warp * kE + e) * 4;
        pr[0] = q0;
        pr[1] = q1;
        pr[2] = q2;
        pr[3] = q3;
      }
      // dh1 = dz2 W2^T + residual of layer 2; dz1 = dh1 (1 - t1^2) over t1
      for (int it2 = tid; it2 < (kE / 4) * ((D1 + 3) / 4); it2 += kT) {
        double acc[4][4];
        int e0, m0;
        dense_bwd_tile<D1, D2>(Z2T, net + N::W2, it2, acc, e0, m0);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int m = m0 + j;
          if (m >= D1) break;
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int ee = e0 + i;
            double dh = acc[i][j];
            if (R2 == 1) dh += A2T[m * kE + ee];
            if (R2 == 2) dh += A2T[m * kE + ee] + A2T[(m + D1) * kE + ee];
            const double t1 = A1T[m * kE + ee];
            A1T[m * kE + ee] = dh * (1.0 - t1 * t1);
          }
        }
      }
      __syncthreads();
      if (tid < ne) {  // dE/ds, the partial dR~ in warp order, the slot's environment-row gradient
        const int ee = tid;
        double ds = 0.0;
        for (int m = 0; m < D1; ++m) ds = fma(A1T[m * kE + ee], net[N::W1 + m], ds);
        double g[4] = {0.0, 0.0, 0.0, 0.0};
        for (int w = 0; w < NW; ++w)
#pragma unroll
          for (int k = 0; k < 4; ++k) g[k] += GT[(w * kE + ee) * 4 + k];
        double2* go = reinterpret_cast<double2*>(genv + 4 * (size_t)slotS[ee]);
        go[0] = make_double2(g[0] + ds, g[1]);
        go[1] = make_double2(g[2], g[3]);
      }
    }
  }
}

template <int D1, int D2, int D3>
void run_fwd(cudaStream_t st, const SeaDev& s, const TcLists& L, int grid, const double* rij, const double* emb,
             double* Tq, double* T, double* D, const int* perm_atom, int nloc) {
  const size_t smem = FwdSmem<D1, D2, D3>::BYTES;
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(k_embed_fwd_f64<D1, D2, D3>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    attr = true;
  }
  count_launch();
  k_embed_fwd_f64<D1, D2, D3><<<grid, kT, smem, st>>>(L, s, rij, emb, Tq);
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
    cudaFuncSetAttribute(k_dT_f64<D3>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)dsm);
    dattr = dsm;
  }
  count_launch();
  k_dT_f64<D3><<<nloc, 128, dsm, st>>>(nloc, s.ntypes, s.M2, s.inv_nnei, type_start, perm_atom, T, dD, dT);
  const size_t smem = BwdSmem<D1, D2, D3>::BYTES;
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(k_embed_bwd_f64<D1, D2, D3>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    attr = true;
  }
  count_launch();
  k_embed_bwd_f64<D1, D2, D3><<<grid, kT, smem, st>>>(L, s, rij, emb, dT, genv);
}

}  // namespace

int embed_f64_grid(const SeaDev& s, bool backward) {
  int dev = 0, nsm = 148, occ = 1;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
  (void)s;
  const size_t smem = backward ? BwdSmem<25, 50, 100>::BYTES : FwdSmem<25, 50, 100>::BYTES;
  int smem_sm = 0;
  cudaDeviceGetAttribute(&smem_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev);
  occ = std::max(1, std::min(4, smem_sm / (int)(smem + 1024)));
  return nsm * occ;
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
