// DPA4C-style model kernels (see sea.cuh).  SIMT path, templated on the
// network precision P (double for the fp64 mode, float for the mixed mode);
// geometry, the chain rule to r_ij and every accumulation of energy, force
// and virial stay in fp64 in both modes.
#include <algorithm>

#include <type_traits>

#include "sea.cuh"
#include "simt_gemm.cuh"

namespace b200dp {

namespace {

// Residual rule of DeePMD's embedding net: d_out == d_in -> x + h,
// d_out == 2 d_in -> concat(x, x) + h, otherwise h.
__device__ __forceinline__ int resid_mode(int din, int dout) { return dout == din ? 1 : (dout == 2 * din ? 2 : 0); }

template <typename P>
struct SmemCarve {
  unsigned char* p;
  __device__ explicit SmemCarve(unsigned char* base) : p(base) {}
  template <typename T>
  __device__ T* take(size_t n) {
    T* r = reinterpret_cast<T*>(p);
    p += ((n * sizeof(T) + 15) / 16) * 16;
    return r;
  }
};

// Scalar-input first layer: out[e][n] = tanh(s_e * w[n] + b[n]) (+ residual).
template <typename P>
__device__ __forceinline__ void layer_from_scalar(const P* srt, int ne, P* out, int d1, const P* __restrict__ w,
                                                  const P* __restrict__ b) {
  const int rm = resid_mode(1, d1);
  for (int idx = threadIdx.x; idx < ne * d1; idx += blockDim.x) {
    const int e = idx / d1, n = idx - e * d1;
    const P x = srt[4 * e];
    P h = act_tanh<P>(x * __ldg(w + n) + __ldg(b + n));
    if (rm) h += x;
    out[idx] = h;
  }
}

// out[e][n] = tanh(sum_k in[e][k] W[k][n] + b[n]) (+ residual); 4 edges per
// thread share each weight load.  Rows >= ne of `in` may hold stale values;
// they are computed but never stored (buffers have a multiple of 4 rows).
template <typename P>
__device__ __forceinline__ void dense_layer(const P* in, int din, P* out, int dout, const P* __restrict__ W,
                                            const P* __restrict__ b, int ne) {
  const int rm = resid_mode(din, dout);
  const int groups = (ne + 3) >> 2;
  for (int idx = threadIdx.x; idx < groups * dout; idx += blockDim.x) {
    const int n = idx % dout, e0 = (idx / dout) * 4;
    const P bias = __ldg(b + n);
    P a0 = bias, a1 = bias, a2 = bias, a3 = bias;
    const P* x = in + e0 * din;
    for (int k = 0; k < din; ++k) {
      const P wv = __ldg(W + k * dout + n);
      a0 += x[k] * wv;
      a1 += x[din + k] * wv;
      a2 += x[2 * din + k] * wv;
      a3 += x[3 * din + k] * wv;
    }
    const P acc[4] = {a0, a1, a2, a3};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int e = e0 + q;
      if (e < ne) {
        P h = act_tanh<P>(acc[q]);
        if (rm == 1)
          h += in[e * din + n];
        else if (rm == 2)
          h += in[e * din + (n < din ? n : n - din)];
        out[e * dout + n] = h;
      }
    }
  }
}

// gx[e][k] = sum_n gz[e][n] W[k][n] (+ residual gradient from gy).  WT is
// W transposed ([dout][din]) so threads over k read consecutive weights.
template <typename P>
__device__ __forceinline__ void dense_bwd(const P* gz, const P* gy, int dout, P* gx, int din,
                                          const P* __restrict__ WT, int ne) {
  const int rm = resid_mode(din, dout);
  const int groups = (ne + 3) >> 2;
  for (int idx = threadIdx.x; idx < groups * din; idx += blockDim.x) {
    const int k = idx % din, e0 = (idx / din) * 4;
    P a0 = 0, a1 = 0, a2 = 0, a3 = 0;
    const P* z = gz + e0 * dout;
    for (int n = 0; n < dout; ++n) {
      const P wv = __ldg(WT + n * din + k);
      a0 += z[n] * wv;
      a1 += z[dout + n] * wv;
      a2 += z[2 * dout + n] * wv;
      a3 += z[3 * dout + n] * wv;
    }
    const P acc[4] = {a0, a1, a2, a3};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int e = e0 + q;
      if (e < ne) {
        P v = acc[q];
        if (rm == 1)
          v += gy[e * dout + k];
        else if (rm == 2)
          v += gy[e * dout + k] + gy[e * dout + k + din];
        gx[e * din + k] = v;
      }
    }
  }
}

// Environment row of one edge: rt = sw(r) * (1/r, x/r^2, y/r^2, z/r^2) and,
// when drt != nullptr, its Jacobian d rt_k / d r_c (fp64).
__device__ __forceinline__ void env_row(const SeaDev& s, const double* r, double* rt, double* drt) {
  const double r2 = r[0] * r[0] + r[1] * r[1] + r[2] * r[2];
  const double rr = sqrt(r2);
  double sw, dsw;
  smooth_switch(rr, s.rcut_smth, s.rcut, sw, dsw);
  const double inv_r = 1.0 / rr, inv_r2 = inv_r * inv_r;
  rt[0] = sw * inv_r;
#pragma unroll
  for (int c = 0; c < 3; ++c) rt[1 + c] = sw * r[c] * inv_r2;
  if (drt) {
    const double d0 = dsw * inv_r - sw * inv_r2;
#pragma unroll
    for (int c = 0; c < 3; ++c) drt[c] = d0 * r[c] * inv_r;
#pragma unroll
    for (int a = 0; a < 3; ++a)
#pragma unroll
      for (int c = 0; c < 3; ++c)
        drt[3 * (1 + a) + c] =
            dsw * r[c] * inv_r * r[a] * inv_r2 + sw * ((a == c ? inv_r2 : 0.0) - 2.0 * r[a] * r[c] * inv_r2 * inv_r2);
  }
}

}  // namespace

// ---------------------------------------------------------------- descriptor forward
template <typename P>
size_t descriptor_fwd_smem(const SeaDev& s, int ch) {
  auto al = [](size_t b) { return ((b + 15) / 16) * 16; };
  return al(sizeof(P) * ch * 4) + 2 * al(sizeof(P) * ch * s.maxd) + al(sizeof(P) * 4 * s.M1);
}

template <typename P>
__global__ void __launch_bounds__(kSeaThreads)
    k_descriptor_fwd(SeaDev s, int nloc, int ch, const double* __restrict__ rij, const int* __restrict__ cnt,
                     const int* __restrict__ atype, const int* __restrict__ perm_pos, const P* __restrict__ emb,
                     P* __restrict__ Tg, P* __restrict__ Dg) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  SmemCarve<P> sc(smem_raw);
  P* srt = sc.template take<P>((size_t)ch * 4);
  P* buf0 = sc.template take<P>((size_t)ch * s.maxd);
  P* buf1 = sc.template take<P>((size_t)ch * s.maxd);
  P* sT = sc.template take<P>((size_t)4 * s.M1);
  const int tid = threadIdx.x;
  for (int i = blockIdx.x; i < nloc; i += gridDim.x) {
    const int ti = atype[i];
    if (ti < 0 || ti >= s.ntypes) continue;  // reported by the type partition; block-uniform
    P tacc[4] = {0, 0, 0, 0};
    for (int t = 0; t < s.ntypes; ++t) {
      const int n_e = cnt[(size_t)i * s.ntypes + t];
      const int net = s.type_one_side ? t : ti * s.ntypes + t;
      const P* Wn = emb + (size_t)net * s.net_stride;
      const size_t base = (size_t)i * s.selt + s.off[t];
      for (int c0 = 0; c0 < n_e; c0 += ch) {
        const int ne = min(ch, n_e - c0);
        for (int e = tid; e < ne; e += blockDim.x) {
          const double* r = rij + 3 * (base + c0 + e);
          const double rv[3] = {r[0], r[1], r[2]};
          double rt[4];
          env_row(s, rv, rt, nullptr);
#pragma unroll
          for (int k = 0; k < 4; ++k) srt[4 * e + k] = (P)rt[k];
        }
        __syncthreads();
        layer_from_scalar<P>(srt, ne, buf0, s.ed[1], Wn + s.w_off[0], Wn + s.b_off[0]);
        __syncthreads();
        P* in = buf0;
        P* out = buf1;
        for (int l = 1; l < s.nl; ++l) {
          dense_layer<P>(in, s.ed[l], out, s.ed[l + 1], Wn + s.w_off[l], Wn + s.b_off[l], ne);
          __syncthreads();
          P* tmp = in;
          in = out;
          out = tmp;
        }
        if (tid < s.M1) {
          // one column of T per thread (M1 <= blockDim is checked at load)
          for (int e = 0; e < ne; ++e) {
            const P g = in[e * s.M1 + tid];
#pragma unroll
            for (int k = 0; k < 4; ++k) tacc[k] += srt[4 * e + k] * g;
          }
        }
        __syncthreads();
      }
    }
    const P inv = (P)s.inv_nnei;
    if (tid < s.M1) {
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const P v = tacc[k] * inv;
        sT[k * s.M1 + tid] = v;
        Tg[(size_t)i * 4 * s.M1 + k * s.M1 + tid] = v;
      }
    }
    __syncthreads();
    P* drow = Dg + (size_t)perm_pos[i] * s.dim;
    for (int idx = tid; idx < s.M1 * s.M2; idx += blockDim.x) {
      const int a = idx / s.M2, b = idx - a * s.M2;
      P acc = 0;
#pragma unroll
      for (int k = 0; k < 4; ++k) acc += sT[k * s.M1 + a] * sT[k * s.M1 + b];
      drow[idx] = acc;
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------- descriptor backward
template <typename P>
size_t descriptor_bwd_smem(const SeaDev& s, int ch) {
  auto al = [](size_t b) { return ((b + 15) / 16) * 16; };
  size_t acts = 0;
  for (int l = 1; l <= s.nl; ++l) acts += al(sizeof(P) * ch * s.ed[l]);
  return 2 * al(sizeof(P) * 4 * s.M1) + al(sizeof(P) * s.dim) + al(sizeof(P) * ch * 4) +
         al(sizeof(double) * ch * 12) + al(sizeof(P) * ch * 4) + acts + 3 * al(sizeof(P) * ch * s.maxd);
}

template <typename P>
__global__ void __launch_bounds__(kSeaThreads)
    k_descriptor_bwd(SeaDev s, int nloc, int ch, const double* __restrict__ rij, const int* __restrict__ cnt,
                     const int* __restrict__ atype, const int* __restrict__ perm_pos, const P* __restrict__ emb,
                     const P* __restrict__ embT, const P* __restrict__ Tg, const P* __restrict__ dDg,
                     double* __restrict__ gslot) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  SmemCarve<P> sc(smem_raw);
  P* sT = sc.template take<P>((size_t)4 * s.M1);
  P* sdT = sc.template take<P>((size_t)4 * s.M1);
  P* sdD = sc.template take<P>((size_t)s.dim);
  P* srt = sc.template take<P>((size_t)ch * 4);
  double* sdrt = sc.template take<double>((size_t)ch * 12);
  P* sdR = sc.template take<P>((size_t)ch * 4);
  P* act[kMaxLayers + 1];
  act[0] = nullptr;
  for (int l = 1; l <= s.nl; ++l) act[l] = sc.template take<P>((size_t)ch * s.ed[l]);
  P* gbuf[3];
  for (int q = 0; q < 3; ++q) gbuf[q] = sc.template take<P>((size_t)ch * s.maxd);
  const int tid = threadIdx.x;
  const int M1 = s.M1, M2 = s.M2;
  for (int i = blockIdx.x; i < nloc; i += gridDim.x) {
    const int ti = atype[i];
    if (ti < 0 || ti >= s.ntypes) continue;  // reported by the type partition; block-uniform
    const P* Ti = Tg + (size_t)i * 4 * M1;
    const P* dDi = dDg + (size_t)perm_pos[i] * s.dim;
    for (int idx = tid; idx < 4 * M1; idx += blockDim.x) sT[idx] = Ti[idx];
    for (int idx = tid; idx < s.dim; idx += blockDim.x) sdD[idx] = dDi[idx];
    __syncthreads();
    // dT[k][a] = (sum_b dD[a][b] T[k][b] + [a < M2] sum_c dD[c][a] T[k][c]) / N
    for (int idx = tid; idx < 4 * M1; idx += blockDim.x) {
      const int k = idx / M1, a = idx - k * M1;
      const P* tk = sT + k * M1;
      P acc = 0;
      for (int b = 0; b < M2; ++b) acc += sdD[a * M2 + b] * tk[b];
      if (a < M2)
        for (int c = 0; c < M1; ++c) acc += sdD[c * M2 + a] * tk[c];
      sdT[idx] = acc * (P)s.inv_nnei;
    }
    __syncthreads();
    for (int t = 0; t < s.ntypes; ++t) {
      const int n_e = cnt[(size_t)i * s.ntypes + t];
      const int net = s.type_one_side ? t : ti * s.ntypes + t;
      const P* Wn = emb + (size_t)net * s.net_stride;
      const P* WTn = embT + (size_t)net * s.net_stride;
      const size_t base = (size_t)i * s.selt + s.off[t];
      for (int c0 = 0; c0 < n_e; c0 += ch) {
        const int ne = min(ch, n_e - c0);
        for (int e = tid; e < ne; e += blockDim.x) {
          const double* r = rij + 3 * (base + c0 + e);
          const double rv[3] = {r[0], r[1], r[2]};
          double rt[4];
          env_row(s, rv, rt, sdrt + 12 * e);
#pragma unroll
          for (int k = 0; k < 4; ++k) srt[4 * e + k] = (P)rt[k];
        }
        __syncthreads();
        // forward recompute, keeping every layer output
        layer_from_scalar<P>(srt, ne, act[1], s.ed[1], Wn + s.w_off[0], Wn + s.b_off[0]);
        __syncthreads();
        for (int l = 1; l < s.nl; ++l) {
          dense_layer<P>(act[l], s.ed[l], act[l + 1], s.ed[l + 1], Wn + s.w_off[l], Wn + s.b_off[l], ne);
          __syncthreads();
        }
        const P* G = act[s.nl];
        // dG[e][a] = sum_k dT'[k][a] rt[e][k];  dR[e][k] = sum_a dT'[k][a] G[e][a]
        P* gy = gbuf[0];
        for (int idx = tid; idx < ne * M1; idx += blockDim.x) {
          const int e = idx / M1, a = idx - e * M1;
          P acc = 0;
#pragma unroll
          for (int k = 0; k < 4; ++k) acc += sdT[k * M1 + a] * srt[4 * e + k];
          gy[idx] = acc;
        }
        for (int idx = tid; idx < ne * 4; idx += blockDim.x) {
          const int e = idx >> 2, k = idx & 3;
          const P* g = G + e * M1;
          const P* dt = sdT + k * M1;
          P acc = 0;
          for (int a = 0; a < M1; ++a) acc += dt[a] * g[a];
          sdR[idx] = acc;
        }
        __syncthreads();
        // back through layers nl-1 .. 1
        P* gz = gbuf[1];
        P* gx = gbuf[2];
        for (int l = s.nl - 1; l >= 1; --l) {
          const int din = s.ed[l], dout = s.ed[l + 1];
          const int rm = resid_mode(din, dout);
          const P* x = act[l];
          const P* y = act[l + 1];
          for (int idx = tid; idx < ne * dout; idx += blockDim.x) {
            const int e = idx / dout, n = idx - e * dout;
            P th = y[idx];
            if (rm == 1)
              th -= x[e * din + n];
            else if (rm == 2)
              th -= x[e * din + (n < din ? n : n - din)];
            gz[idx] = gy[idx] * ((P)1 - th * th);
          }
          __syncthreads();
          dense_bwd<P>(gz, gy, dout, gx, din, WTn + s.w_off[l], ne);
          __syncthreads();
          P* tmp = gy;
          gy = gx;
          gx = tmp;
        }
        // first layer (scalar input) and the chain rule to r_ij
        {
          const int d1 = s.ed[1];
          const int rm = resid_mode(1, d1);
          const P* y = act[1];
          for (int idx = tid; idx < ne * d1; idx += blockDim.x) {
            const int e = idx / d1;
            P th = y[idx];
            if (rm) th -= srt[4 * e];
            gz[idx] = gy[idx] * ((P)1 - th * th);
          }
          __syncthreads();
          const P* w0 = Wn + s.w_off[0];
          for (int e = tid; e < ne; e += blockDim.x) {
            P ds = 0;
            for (int n = 0; n < d1; ++n) ds += gz[e * d1 + n] * __ldg(w0 + n);
            if (rm)
              for (int n = 0; n < d1; ++n) ds += gy[e * d1 + n];
            double dR[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) dR[k] = (double)sdR[4 * e + k];
            dR[0] += (double)ds;
            const double* J = sdrt + 12 * e;
            double* go = gslot + 3 * (base + c0 + e);
#pragma unroll
            for (int c = 0; c < 3; ++c) go[c] = ((dR[0] * J[c] + dR[1] * J[3 + c]) + dR[2] * J[6 + c]) + dR[3] * J[9 + c];
          }
          __syncthreads();
        }
      }
    }
  }
}

template <typename P>
int descriptor_grid(const SeaDev& s, int ch, bool bwd, int nloc) {
  int dev = 0, nsm = 148, occ = 1;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
  const size_t smem = bwd ? descriptor_bwd_smem<P>(s, ch) : descriptor_fwd_smem<P>(s, ch);
  if (bwd) {
    cudaFuncSetAttribute(k_descriptor_bwd<P>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, k_descriptor_bwd<P>, kSeaThreads, smem);
  } else {
    cudaFuncSetAttribute(k_descriptor_fwd<P>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, k_descriptor_fwd<P>, kSeaThreads, smem);
  }
  occ = std::max(occ, 1);
  return std::max(1, std::min(nloc, nsm * occ));
}

template <typename P>
void launch_descriptor_fwd(cudaStream_t st, const SeaDev& s, int nloc, int ch, int grid, const double* rij,
                           const int* cnt, const int* atype, const int* perm_pos, const P* emb, P* T, P* D) {
  if (nloc <= 0) return;
  count_launch();
  k_descriptor_fwd<P><<<grid, kSeaThreads, descriptor_fwd_smem<P>(s, ch), st>>>(s, nloc, ch, rij, cnt, atype,
                                                                                 perm_pos, emb, T, D);
}

template <typename P>
void launch_descriptor_bwd(cudaStream_t st, const SeaDev& s, int nloc, int ch, int grid, const double* rij,
                           const int* cnt, const int* atype, const int* perm_pos, const P* emb, const P* embT,
                           const P* T, const P* dD, double* gslot) {
  if (nloc <= 0) return;
  count_launch();
  k_descriptor_bwd<P><<<grid, kSeaThreads, descriptor_bwd_smem<P>(s, ch), st>>>(s, nloc, ch, rij, cnt, atype,
                                                                                 perm_pos, emb, embT, T, dD, gslot);
}

// ---------------------------------------------------------------- fitting GEMMs
namespace {
template <typename P>
struct EpiForward {
  const P* b;
  const P* X;
  int ldx;
  bool residual;
  P* th;
  P* Y;
  int ld;
  __device__ void operator()(int m, int n, P acc) const {
    const P h = act_tanh<P>(acc + b[n]);
    th[(size_t)m * ld + n] = h;
    Y[(size_t)m * ld + n] = residual ? X[(size_t)m * ldx + n] + h : h;
  }
};

template <typename P>
struct EpiBackward {
  const P* dy_next;  // residual gradient (same shape as the output), or null
  P* dX;
  const P* th_prev;  // tanh of the previous layer, or null (last step: dX is the input gradient)
  P* dz_prev;
  int ld;
  __device__ void operator()(int m, int n, P acc) const {
    const size_t o = (size_t)m * ld + n;
    const P v = dy_next ? acc + dy_next[o] : acc;
    dX[o] = v;
    if (th_prev) {
      const P t = th_prev[o];
      dz_prev[o] = v * ((P)1 - t * t);
    }
  }
};
}  // namespace

template <typename P>
void launch_fit_forward_layer(cudaStream_t st, int Mmax, const int* range, int N, int K, const P* X, int ldx,
                              const P* W, const P* b, bool residual, P* th, P* Y) {
  if (Mmax <= 0) return;
  EpiForward<P> epi{b, X, ldx, residual, th, Y, N};
  count_launch();
  if constexpr (std::is_same<P, double>::value) {
    dim3 grid((N + kDN - 1) / kDN, (Mmax + kDM - 1) / kDM);
    k_dgemm<false, EpiForward<P>><<<grid, 128, 0, st>>>(range, N, K, X, ldx, W, N, epi);
  } else {
    dim3 grid((N + kBN - 1) / kBN, (Mmax + kBM - 1) / kBM);
    k_gemm<P, false, EpiForward<P>><<<grid, 256, 0, st>>>(range, N, K, X, ldx, W, N, epi);
  }
}

template <typename P>
void launch_fit_backward_layer(cudaStream_t st, int Mmax, const int* range, int Nin, int Nout, const P* dZ,
                               const P* W, const P* dY_next, P* dX, const P* th_prev, P* dZ_prev) {
  if (Mmax <= 0) return;
  // dX[m][n] = sum_k dZ[m][k] W[n][k]   (W is [Nin][Nout] row-major)
  EpiBackward<P> epi{dY_next, dX, th_prev, dZ_prev, Nin};
  count_launch();
  if constexpr (std::is_same<P, double>::value) {
    dim3 grid((Nin + kDN - 1) / kDN, (Mmax + kDM - 1) / kDM);
    k_dgemm<true, EpiBackward<P>><<<grid, 128, 0, st>>>(range, Nin, Nout, dZ, Nout, W, Nout, epi);
  } else {
    dim3 grid((Nin + kBN - 1) / kBN, (Mmax + kBM - 1) / kBM);
    k_gemm<P, true, EpiBackward<P>><<<grid, 256, 0, st>>>(range, Nin, Nout, dZ, Nout, W, Nout, epi);
  }
}

template <typename P>
__global__ void k_fit_energy(const int* __restrict__ range, int N, const P* __restrict__ Y, const P* __restrict__ wo,
                             double bo, const int* __restrict__ perm_atom, double* __restrict__ atom_energy) {
  const int row0 = range[0], M = range[1] - row0;
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= M) return;
  const int row = row0 + warp;
  const P* y = Y + (size_t)row * N;
  double acc = 0;
  for (int n = lane; n < N; n += 32) acc += (double)(y[n] * wo[n]);
  acc = warp_sum(acc);
  if (lane == 0) atom_energy[perm_atom[row]] = acc + bo;
}

template <typename P>
void launch_fit_energy(cudaStream_t st, int Mmax, const int* range, int N, const P* Y, const P* wo,
                       double bo_plus_bias, const int* perm_atom, double* atom_energy) {
  if (Mmax <= 0) return;
  count_launch();
  k_fit_energy<P><<<(Mmax * 32 + 255) / 256, 256, 0, st>>>(range, N, Y, wo, bo_plus_bias, perm_atom, atom_energy);
}

template <typename P>
__global__ void k_fit_seed(const int* __restrict__ range, int N, const P* __restrict__ wo, const P* __restrict__ th,
                           P* __restrict__ dy, P* __restrict__ dz) {
  const size_t row0 = (size_t)range[0], M = (size_t)(range[1] - range[0]);
  const size_t total = M * N;
  for (size_t q = blockIdx.x * (size_t)blockDim.x + threadIdx.x; q < total; q += (size_t)gridDim.x * blockDim.x) {
    const size_t o = row0 * N + q;
    const int n = (int)(q % N);
    const P w = wo[n], t = th[o];
    dy[o] = w;
    dz[o] = w * ((P)1 - t * t);
  }
}

template <typename P>
void launch_fit_seed(cudaStream_t st, int Mmax, const int* range, int N, const P* wo, const P* th, P* dy, P* dz) {
  if (Mmax <= 0) return;
  const size_t total = (size_t)Mmax * N;
  const int blocks = (int)std::min<size_t>((total + 255) / 256, 148 * 32);
  count_launch();
  k_fit_seed<P><<<blocks, 256, 0, st>>>(range, N, wo, th, dy, dz);
}

// ---------------------------------------------------------------- assembly
// F_j = sum_{own row} g - sum_{edges into j} g.  One warp per centre i sums its
// own row in a fixed order (the row's occupied slots in slot order, dealt to
// the lanes in turn, then an xor-tree warp reduction) and scatters -g of every
// edge into the neighbour's accumulator.  The accumulators are 128-bit
// two's-complement fixed point with 64 fractional bits, added with integer
// atomics: integer addition is associative, so the sum does not depend on the
// order in which edges arrive (deterministic).  A second pass converts each
// accumulator to fp64, adds the own-row part and clears the accumulator for
// the next call.
//
// The total virial -sum g (x) r runs over every edge once and is summed over
// the own rows; the per-atom virial (edges into j) is scattered the same way
// when asked for.  Energy and virial are reduced in the first launch: each
// block writes its sums, and the last block to finish adds the blocks' sums
// in block order.
constexpr int kAsmWarps = 8;
constexpr int kAsmCols = 10;  // virial (9) + energy

// v * 2^64 as (lo, hi), truncated toward -inf at 2^-64; |v| < 2^63.  For
// |v| < 1 the high word's increment (integer part + carry) is usually zero
// and is then not sent.
__device__ __forceinline__ void fix_add(unsigned long long* __restrict__ p, double v) {
  const double fl = floor(v);
  const unsigned long long hi = (unsigned long long)(long long)fl;
  const unsigned long long lo = (unsigned long long)((v - fl) * 0x1p64);
  const unsigned long long old = atomicAdd(p, lo);
  const unsigned long long inc = hi + (old + lo < old ? 1ull : 0ull);
  if (inc) atomicAdd(p + 1, inc);
}

__device__ __forceinline__ double fix_value(unsigned long long lo, unsigned long long hi) {
  return (double)(long long)hi + (double)lo * 0x1p-64;
}

// (lo, hi) added to the 128-bit accumulator at p.
__device__ __forceinline__ void fix_add128(unsigned long long* p, unsigned long long lo, unsigned long long hi) {
  const unsigned long long old = atomicAdd(p, lo);
  const unsigned long long inc = hi + (old + lo < old ? 1ull : 0ull);
  if (inc) atomicAdd(p + 1, inc);
}

// Peer fold (domain decomposition): owned neighbours' contributions go to
// this rank's exported accumulator (own, own_nf) instead of acc_f, ghost rows
// stay in acc_f for k_fold_push.
struct FoldTargets {
  unsigned long long* own;
  unsigned* own_nf;
};

// dE/dr_ij from the environment-row gradient g4 = dE/dR~ (R~ = (sw/r, sw x/r^2,
// sw y/r^2, sw z/r^2)) by the chain rule through R~(r), in fp64.
__device__ __forceinline__ void env_chain(const double* g4, const double* r3, double rc, double rs, double* g3) {
  // with u = r / |r| and g = (g4[1], g4[2], g4[3]):
  //   d(sw/r)/dr_c = (dsw/r - sw/r^2) u_c,
  //   sum_a g_a d(sw r_a/r^2)/dr_c = r_c (g.r)(dsw/r^3 - 2 sw/r^4) + (sw/r^2) g_c
  const double x = r3[0], y = r3[1], zc = r3[2];
  const double r2 = x * x + y * y + zc * zc, rr = sqrt(r2);
  double sw, dsw;
  smooth_switch(rr, rs, rc, sw, dsw);
  const double ir = 1.0 / rr, ir2 = ir * ir;
  const double gr = g4[1] * x + g4[2] * y + g4[3] * zc;
  const double a = g4[0] * (dsw * ir - sw * ir2) * ir + gr * ir2 * (dsw * ir - 2.0 * sw * ir2);
  const double b = sw * ir2;
  g3[0] = a * x + b * g4[1];
  g3[1] = a * y + b * g4[2];
  g3[2] = a * zc + b * g4[3];
}

// One warp per centre over its slots.  gsrc holds per slot either dE/dr_ij
// (3 doubles) or, with kEnv, the environment-row gradient (4 doubles) that
// env_chain turns into dE/dr_ij.
template <bool kAtomVirial, bool kEnv>
__global__ void __launch_bounds__(kAsmWarps * 32)
    k_assemble(int nloc, int selt, const int* __restrict__ nl_j, const double* __restrict__ gsrc,
               const double* __restrict__ rij, const double* __restrict__ atom_e, double* __restrict__ force,
               unsigned long long* __restrict__ acc_f, unsigned long long* __restrict__ acc_v,
               unsigned* __restrict__ nonfinite, double* __restrict__ partial, unsigned* __restrict__ done,
               double* __restrict__ energy, double* __restrict__ virial, FoldTargets fold, double rc, double rs) {
  __shared__ double s_part[kAsmWarps][kAsmCols];
  __shared__ int s_last;
  __shared__ short s_slot[kAsmWarps][kAssembleMaxSlots];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  short* slots = s_slot[warp];
  double v[9] = {0, 0, 0, 0, 0, 0, 0, 0, 0};
  double e = 0;
  // a fixed grid strides over the atoms: the same atoms land in the same
  // block's sums on every call, and the final reduction stays short
  for (int i = blockIdx.x * kAsmWarps + warp; i < nloc; i += gridDim.x * kAsmWarps) {
    double f[3] = {0, 0, 0};
    const size_t row = (size_t)i * selt;
    // the row's occupied slots in slot order (a ballot per 32 slots)
    int nreal = 0;
    __syncwarp();
    for (int s0 = 0; s0 < selt; s0 += 32) {
      const int s = s0 + lane;
      const bool occ = s < selt && nl_j[row + s] >= 0;
      const unsigned m = __ballot_sync(0xffffffffu, occ);
      if (occ) slots[nreal + __popc(m & ((1u << lane) - 1u))] = (short)s;
      nreal += __popc(m);
    }
    __syncwarp();
    for (int k = lane; k < nreal; k += 32) {
      const int s = slots[k];
      const int j = nl_j[row + s];
      {
        const double* r = rij + 3 * (row + s);
        const double r3[3] = {r[0], r[1], r[2]};
        double g3[3];
        if (kEnv) {
          const double2* g = reinterpret_cast<const double2*>(gsrc + 4 * (row + s));
          const double2 ga = g[0], gb = g[1];
          const double g4[4] = {ga.x, ga.y, gb.x, gb.y};
          env_chain(g4, r3, rc, rs, g3);
        } else {
          const double* g = gsrc + 3 * (row + s);
          g3[0] = g[0];
          g3[1] = g[1];
          g3[2] = g[2];
        }
        f[0] += g3[0];
        f[1] += g3[1];
        f[2] += g3[2];
        double w[9];
#pragma unroll
        for (int a = 0; a < 3; ++a)
#pragma unroll
          for (int b = 0; b < 3; ++b) {
            w[3 * a + b] = -g3[a] * r3[b];
            v[3 * a + b] += w[3 * a + b];
          }
        bool finite = isfinite(g3[0]) && isfinite(g3[1]) && isfinite(g3[2]);
        if (finite) {
          unsigned long long* dst = (fold.own && j < nloc ? fold.own : acc_f) + 6 * (size_t)j;
#pragma unroll
          for (int c = 0; c < 3; ++c) fix_add(dst + 2 * c, -g3[c]);
          if (kAtomVirial) {
#pragma unroll
            for (int c = 0; c < 9; ++c) finite = finite && isfinite(w[c]);
            if (finite) {
#pragma unroll
              for (int c = 0; c < 9; ++c) fix_add(acc_v + 2 * (9 * (size_t)j + c), w[c]);
            }
          }
        }
        if (!finite) atomicOr((fold.own && j < nloc ? fold.own_nf : nonfinite) + j, 1u);
      }
    }
    if (lane == 0) e += atom_e[i];
#pragma unroll
    for (int c = 0; c < 3; ++c) f[c] = warp_sum(f[c]);
    if (lane == 0) {
      force[3 * (size_t)i] = f[0];
      force[3 * (size_t)i + 1] = f[1];
      force[3 * (size_t)i + 2] = f[2];
    }
  }
#pragma unroll
  for (int c = 0; c < 9; ++c) v[c] = warp_sum(v[c]);
  if (lane == 0) {
#pragma unroll
    for (int c = 0; c < 9; ++c) s_part[warp][c] = v[c];
    s_part[warp][9] = e;
  }
  __syncthreads();
  if (threadIdx.x < kAsmCols) {
    double acc = 0;
#pragma unroll
    for (int w = 0; w < kAsmWarps; ++w) acc += s_part[w][threadIdx.x];
    partial[(size_t)blockIdx.x * kAsmCols + threadIdx.x] = acc;
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) s_last = (atomicAdd(done, 1u) == gridDim.x - 1);
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  for (int c = warp; c < kAsmCols; c += kAsmWarps) {
    double acc = 0;
    for (int b = lane; b < (int)gridDim.x; b += 32) acc += __ldcg(partial + (size_t)b * kAsmCols + c);
    acc = warp_sum(acc);
    if (lane == 0) {
      if (c < 9)
        virial[c] = acc;
      else
        energy[0] = acc;
    }
  }
  if (threadIdx.x == 0) *done = 0u;  // ready for the next launch
}

// Adds the scattered sums to the own-row forces (ghost atoms have no own row),
// writes the per-atom virials, and clears the accumulators.
template <bool kAtomVirial>
__global__ void k_assemble_finish(int nloc, int nall, double* __restrict__ force, double* __restrict__ atom_virial,
                                  unsigned long long* __restrict__ acc_f, unsigned long long* __restrict__ acc_v,
                                  unsigned* __restrict__ nonfinite) {
  const int j = blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= nall) return;
  const bool bad = nonfinite[j] != 0u;
  if (bad) nonfinite[j] = 0u;
  const double nan = __longlong_as_double(0x7ff8000000000000ll);
#pragma unroll
  for (int c = 0; c < 3; ++c) {
    ulonglong2* a = reinterpret_cast<ulonglong2*>(acc_f) + 3 * (size_t)j + c;
    const ulonglong2 q = *a;
    const double own = j < nloc ? force[3 * (size_t)j + c] : 0.0;
    force[3 * (size_t)j + c] = bad ? nan : own + fix_value(q.x, q.y);
    *a = make_ulonglong2(0ull, 0ull);
  }
  if (kAtomVirial) {
#pragma unroll
    for (int c = 0; c < 9; ++c) {
      ulonglong2* a = reinterpret_cast<ulonglong2*>(acc_v) + 9 * (size_t)j + c;
      const ulonglong2 q = *a;
      atom_virial[9 * (size_t)j + c] = bad ? nan : fix_value(q.x, q.y);
      *a = make_ulonglong2(0ull, 0ull);
    }
  }
}

int assemble_blocks(int nloc) { return std::max(1, std::min((nloc + kAsmWarps - 1) / kAsmWarps, 148 * 8)); }

void launch_assemble(cudaStream_t st, int nloc, int nall, int selt, const int* nl_j, const double* gslot,
                     const double* rij, const double* atom_e, double* force, double* atom_virial,
                     unsigned long long* acc_f, unsigned long long* acc_v, unsigned* nonfinite, double* partial,
                     unsigned* done, double* energy, double* virial, const EnvChain& env) {
  if (nall <= 0) return;
  const int nb = assemble_blocks(nloc);
  const int fb = (nall + 255) / 256;
  count_launch();
  count_launch();
  const FoldTargets none{nullptr, nullptr};
  const double rc = env.rcut, rs = env.rcut_smth;
  if (atom_virial) {
    if (env.on)
      k_assemble<true, true><<<nb, kAsmWarps * 32, 0, st>>>(nloc, selt, nl_j, gslot, rij, atom_e, force, acc_f, acc_v,
                                                            nonfinite, partial, done, energy, virial, none, rc, rs);
    else
      k_assemble<true, false><<<nb, kAsmWarps * 32, 0, st>>>(nloc, selt, nl_j, gslot, rij, atom_e, force, acc_f,
                                                             acc_v, nonfinite, partial, done, energy, virial, none, rc,
                                                             rs);
    k_assemble_finish<true><<<fb, 256, 0, st>>>(nloc, nall, force, atom_virial, acc_f, acc_v, nonfinite);
  } else {
    if (env.on)
      k_assemble<false, true><<<nb, kAsmWarps * 32, 0, st>>>(nloc, selt, nl_j, gslot, rij, atom_e, force, acc_f,
                                                             nullptr, nonfinite, partial, done, energy, virial, none,
                                                             rc, rs);
    else
      k_assemble<false, false><<<nb, kAsmWarps * 32, 0, st>>>(nloc, selt, nl_j, gslot, rij, atom_e, force, acc_f,
                                                              nullptr, nonfinite, partial, done, energy, virial, none,
                                                              rc, rs);
    k_assemble_finish<false><<<fb, 256, 0, st>>>(nloc, nall, force, nullptr, acc_f, nullptr, nonfinite);
  }
}

// Each ghost row's sums (acc_f rows nloc..nall) are added to its owner's
// accumulator in the owner's memory (one 128-bit addition per component), and
// the local rows are cleared for the next call.
__global__ void k_fold_push(int nloc, int nghost, unsigned long long* __restrict__ acc_f,
                            unsigned* __restrict__ nonfinite, PeerSet peers, const int2* __restrict__ origin) {
  const int g = blockIdx.x * blockDim.x + threadIdx.x;
  if (g >= nghost) return;
  const size_t j = (size_t)nloc + g;
  const int2 o = origin[g];
  unsigned char* base = peers.base[o.x];
  unsigned long long* dst = reinterpret_cast<unsigned long long*>(base + peers.off_acc) + 6 * (size_t)o.y;
  ulonglong2* a = reinterpret_cast<ulonglong2*>(acc_f) + 3 * j;
#pragma unroll
  for (int c = 0; c < 3; ++c) {
    const ulonglong2 q = a[c];
    if (q.x | q.y) fix_add128(dst + 2 * c, q.x, q.y);
    a[c] = make_ulonglong2(0ull, 0ull);
  }
  if (nonfinite[j]) {
    nonfinite[j] = 0u;
    atomicOr(reinterpret_cast<unsigned*>(base + peers.off_nf) + o.y, 1u);
  }
  __threadfence_system();  // the additions are visible to the owner before this kernel completes
}

// Ghost rows of x from the owners' published positions plus the periodic shift
// (each component a sum of whole box lengths, applied as one addition, as the
// staged exchange does).
__global__ void k_halo_gather(int nloc, int nghost, double* __restrict__ x, PeerSet peers,
                              const int2* __restrict__ origin, const double* __restrict__ shift) {
  const int g = blockIdx.x * blockDim.x + threadIdx.x;
  if (g >= nghost) return;
  const int2 o = origin[g];
  const double* src = reinterpret_cast<const double*>(peers.base[o.x] + peers.off_x) + 3 * (size_t)o.y;
  const double s0 = src[0], s1 = src[1], s2 = src[2];
  double* dst = x + 3 * ((size_t)nloc + g);
  dst[0] = s0 + shift[3 * (size_t)g];
  dst[1] = s1 + shift[3 * (size_t)g + 1];
  dst[2] = s2 + shift[3 * (size_t)g + 2];
}

void launch_assemble_fold(cudaStream_t st, int nloc, int nall, int selt, const int* nl_j, const double* gslot,
                          const double* rij, const double* atom_e, double* force, unsigned long long* acc_f,
                          unsigned* nonfinite, unsigned long long* own_acc, unsigned* own_nf, const PeerSet& peers,
                          const int2* origin, double* partial, unsigned* done, double* energy, double* virial,
                          const EnvChain& env) {
  count_launch();
  const FoldTargets fold{own_acc, own_nf};
  if (env.on)
    k_assemble<false, true><<<assemble_blocks(nloc), kAsmWarps * 32, 0, st>>>(
        nloc, selt, nl_j, gslot, rij, atom_e, force, acc_f, nullptr, nonfinite, partial, done, energy, virial, fold,
        env.rcut, env.rcut_smth);
  else
    k_assemble<false, false><<<assemble_blocks(nloc), kAsmWarps * 32, 0, st>>>(
        nloc, selt, nl_j, gslot, rij, atom_e, force, acc_f, nullptr, nonfinite, partial, done, energy, virial, fold,
        env.rcut, env.rcut_smth);
  const int nghost = nall - nloc;
  if (nghost > 0) {
    count_launch();
    k_fold_push<<<(nghost + 255) / 256, 256, 0, st>>>(nloc, nghost, acc_f, nonfinite, peers, origin);
  }
}

void launch_fold_finish(cudaStream_t st, int nloc, double* force, unsigned long long* acc, unsigned* nonfinite) {
  if (nloc <= 0) return;
  count_launch();
  k_assemble_finish<false><<<(nloc + 255) / 256, 256, 0, st>>>(nloc, nloc, force, nullptr, acc, nullptr, nonfinite);
}

// shift[g][d] *= ratio[d] (an isotropic or orthorhombic rescaling of the box)
__global__ void k_scale_shifts(int nghost, double* __restrict__ shift, double r0, double r1, double r2) {
  const int g = blockIdx.x * blockDim.x + threadIdx.x;
  if (g >= nghost) return;
  shift[3 * (size_t)g] *= r0;
  shift[3 * (size_t)g + 1] *= r1;
  shift[3 * (size_t)g + 2] *= r2;
}

void launch_scale_shifts(cudaStream_t st, int nghost, double* shift, const double* ratio) {
  if (nghost <= 0) return;
  count_launch();
  k_scale_shifts<<<(nghost + 255) / 256, 256, 0, st>>>(nghost, shift, ratio[0], ratio[1], ratio[2]);
}

void launch_halo_gather(cudaStream_t st, int nloc, int nghost, double* x, const PeerSet& peers, const int2* origin,
                        const double* shift) {
  if (nghost <= 0) return;
  count_launch();
  k_halo_gather<<<(nghost + 255) / 256, 256, 0, st>>>(nloc, nghost, x, peers, origin, shift);
}

// One rendezvous of all ranks (see launch_peer_reduce).  One warp: lane q
// handles rank q (q < nranks <= 32 per pass of the loops below).
__global__ void __launch_bounds__(32) k_peer_reduce(PeerSync ps, unsigned long long* __restrict__ seqp,
                                                    const double* __restrict__ in, int nv, double* __restrict__ out,
                                                    int* __restrict__ err, long long limit) {
  const int lane = threadIdx.x;
  const unsigned long long seq = *seqp + 1;
  const size_t mail = ps.off_mail + sizeof(double) * ((size_t)(seq & 1) * kPeerMaxRanks * kPeerMaxValues +
                                                      (size_t)ps.rank * kPeerMaxValues);
  // 1. this rank's values into every rank's mailbox slot, then its arrival counter
  for (int q = lane; q < ps.nranks; q += 32) {
    double* dst = reinterpret_cast<double*>(ps.base[q] + mail);
    for (int v = 0; v < nv; ++v) dst[v] = in[v];
  }
  __threadfence_system();
  __syncwarp();
  for (int q = lane; q < ps.nranks; q += 32) {
    unsigned long long* flag = reinterpret_cast<unsigned long long*>(ps.base[q] + ps.off_flags) + ps.rank;
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(flag), "l"(seq) : "memory");
  }
  // 2. wait until every rank has arrived (bounded)
  const unsigned long long* own =
      reinterpret_cast<const unsigned long long*>(ps.base[ps.rank] + ps.off_flags);
  bool ok = true;
  for (int q = lane; q < ps.nranks; q += 32) {
    long long it = 0;
    for (;;) {
      unsigned long long f;
      asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(f) : "l"(own + q) : "memory");
      if (f >= seq) break;
      if (++it >= limit) {
        ok = false;
        break;
      }
      __nanosleep(64);
    }
  }
  ok = __all_sync(0xffffffffu, ok);
  if (!ok) {
    if (lane == 0) {
      atomicAdd(err, 1);
      *seqp = seq;
    }
    return;
  }
  __threadfence_system();
  // 3. the sum over ranks in rank order
  const double* box = reinterpret_cast<const double*>(ps.base[ps.rank] + ps.off_mail) +
                      (size_t)(seq & 1) * kPeerMaxRanks * kPeerMaxValues;
  for (int v = lane; v < nv; v += 32) {
    double acc = 0.0;
    for (int q = 0; q < ps.nranks; ++q) {
      const double* src = box + (size_t)q * kPeerMaxValues + v;
      double x;
      asm volatile("ld.relaxed.sys.global.f64 %0, [%1];" : "=d"(x) : "l"(src) : "memory");
      acc += x;
    }
    out[v] = acc;
  }
  if (lane == 0) *seqp = seq;
}

void launch_peer_reduce(cudaStream_t st, const PeerSync& ps, unsigned long long* seq, const double* in, int nv,
                        double* out, int* err, long long limit) {
  count_launch();
  k_peer_reduce<<<1, 32, 0, st>>>(ps, seq, in, nv, out, err, limit);
}

// ---------------------------------------------------------------- instantiations
#define B200DP_INST(P)                                                                                              \
  template size_t descriptor_fwd_smem<P>(const SeaDev&, int);                                                      \
  template size_t descriptor_bwd_smem<P>(const SeaDev&, int);                                                      \
  template int descriptor_grid<P>(const SeaDev&, int, bool, int);                                                  \
  template void launch_descriptor_fwd<P>(cudaStream_t, const SeaDev&, int, int, int, const double*, const int*,    \
                                         const int*, const int*, const P*, P*, P*);                                \
  template void launch_descriptor_bwd<P>(cudaStream_t, const SeaDev&, int, int, int, const double*, const int*,    \
                                         const int*, const int*, const P*, const P*, const P*, const P*, double*); \
  template void launch_fit_forward_layer<P>(cudaStream_t, int, const int*, int, int, const P*, int, const P*,   \
                                            const P*, bool, P*, P*);                                               \
  template void launch_fit_energy<P>(cudaStream_t, int, const int*, int, const P*, const P*, double, const int*,   \
                                     double*);                                                                     \
  template void launch_fit_seed<P>(cudaStream_t, int, const int*, int, const P*, const P*, P*, P*);              \
  template void launch_fit_backward_layer<P>(cudaStream_t, int, const int*, int, int, const P*, const P*,          \
                                             const P*, P*, const P*, P*);

B200DP_INST(double)
B200DP_INST(float)

}  // namespace b200dp
