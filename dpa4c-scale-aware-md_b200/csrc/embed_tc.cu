// Tensor-core embedding forward (see embed_tc.cuh).
#include <algorithm>
#include <cstring>

#include "common.cuh"
#include "embed_tc.cuh"
#include "umma.cuh"

namespace b200dp {

namespace {

// tanh from the exponential: 1 - 2 / (exp(2x) + 1).  Absolute error ~1e-7,
// saturates correctly at both ends (exp overflow -> 1, underflow -> -1).
__device__ __forceinline__ float tanh_fast(float x) { return 1.0f - __fdividef(2.0f, __expf(2.0f * x) + 1.0f); }

template <int D1, int D2, int D3>
struct TcShape {
  static constexpr int D1p = (D1 + 15) / 16 * 16;
  static constexpr int D2p = (D2 + 15) / 16 * 16;
  static constexpr int D3p = (D3 + 15) / 16 * 16;
  static constexpr int NT = 32;  // contraction MMA columns: 8 atoms x 4 environment components
  static constexpr uint32_t W2B = D2p * D1p * 2;
  static constexpr uint32_t W3B = D3p * D2p * 2;
  static constexpr uint32_t BUFB = 128 * 128 * 2;  // largest view: G^T, 128 (a) x 128 (edges)
  static constexpr uint32_t RB = NT * 128 * 2;
  static constexpr uint32_t NF = 2 * D1 + D2 + D3;  // w1, b1, b2, b3
  // shared memory map (bytes); every block is a multiple of 16
  static constexpr uint32_t O_W2 = 0;
  static constexpr uint32_t O_W3 = O_W2 + 2 * W2B;
  static constexpr uint32_t O_F = O_W3 + 2 * W3B;
  static constexpr uint32_t O_BUF = ((O_F + NF * 4 + 1023) / 1024) * 1024;
  static constexpr uint32_t O_R = O_BUF + 2 * BUFB;
  static constexpr uint32_t SMEM = O_R + 2 * RB;
  // packed net blob in global memory: [w2 hi|lo][w3 hi|lo][floats]
  static constexpr uint32_t BLOB = O_F + NF * 4;
  // canonical no-swizzle layouts
  static constexpr uint32_t SBO_A1 = (D1p / 8) * 128;  // K-major, K = D1p
  static constexpr uint32_t SBO_A2 = (D2p / 8) * 128;  // K-major, K = D2p
  static constexpr uint32_t SBO_W2 = (D1p / 8) * 128;
  static constexpr uint32_t SBO_W3 = (D2p / 8) * 128;
  static constexpr uint32_t LBO_G = (128 / 8) * 128, SBO_G = 128;  // MN-major, M = 128, K = 128
  static constexpr uint32_t LBO_R = (NT / 8) * 128, SBO_R = 128;   // MN-major, N = NT, K = 128
  // TMEM columns
  static constexpr uint32_t C_D2 = 0, C_D3 = D2p, C_T = D2p + D3p, NCOLS = 256;
  static_assert(C_T + NT <= NCOLS, "TMEM budget");
  static_assert(D1 > 2, "layer-1 residual is not handled by the tensor-core path");
};

constexpr long long kWaitLimit = 1LL << 26;

template <int D2>
__host__ __device__ constexpr int D2p_of() {
  return (D2 + 15) / 16 * 16;
}

template <int D2, int D1>
__device__ __forceinline__ float resid_of(const float* x, int n) {
  if constexpr (D2 == D1) return x[n];
  if constexpr (D2 == 2 * D1) return x[n < D1 ? n : n - D1];
  return 0.0f;
}

// Writes 8 consecutive fp32 values as bf16 hi and lo 16-byte chunks.
__device__ __forceinline__ void store8_split(unsigned char* hi, unsigned char* lo, const float* v) {
  uint32_t h[4], l[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    __nv_bfloat16 h0, l0, h1, l1;
    umma::split_bf16(v[2 * j], h0, l0);
    umma::split_bf16(v[2 * j + 1], h1, l1);
    h[j] = umma::pack2(h0, h1);
    l[j] = umma::pack2(l0, l1);
  }
  *reinterpret_cast<uint4*>(hi) = make_uint4(h[0], h[1], h[2], h[3]);
  *reinterpret_cast<uint4*>(lo) = make_uint4(l[0], l[1], l[2], l[3]);
}

struct FwdArgs {
  TcLists L;
  const unsigned char* nets;
  size_t net_bytes;
  float* partial;
  int* err;
  int M1;
};

// Issues the three split products of one K=16 step pair (hi*hi, hi*lo, lo*hi).
__device__ __forceinline__ void mma3(uint32_t d, uint32_t a_hi, uint32_t a_lo, uint32_t b_hi, uint32_t b_lo,
                                     uint32_t lbo_a, uint32_t sbo_a, uint32_t lbo_b, uint32_t sbo_b, uint32_t idesc,
                                     int steps, uint32_t step_a, uint32_t step_b) {
  for (int s = 0; s < steps; ++s) {
    const uint32_t oa = s * step_a, ob = s * step_b;
    umma::mma(d, umma::desc(a_hi + oa, lbo_a, sbo_a), umma::desc(b_hi + ob, lbo_b, sbo_b), idesc, s > 0 ? 1u : 0u);
    umma::mma(d, umma::desc(a_hi + oa, lbo_a, sbo_a), umma::desc(b_lo + ob, lbo_b, sbo_b), idesc, 1u);
    umma::mma(d, umma::desc(a_lo + oa, lbo_a, sbo_a), umma::desc(b_hi + ob, lbo_b, sbo_b), idesc, 1u);
  }
}

template <int D1, int D2, int D3>
__global__ void __launch_bounds__(128, 1) k_embed_fwd_tc(FwdArgs a) {
  using S = TcShape<D1, D2, D3>;
  extern __shared__ __align__(1024) unsigned char smem[];
  __shared__ uint64_t bar;
  __shared__ uint32_t tbase;
  __shared__ int s_row[128];
  __shared__ int s_lrow[128];
  __shared__ int s_wcnt[4];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const float* w1 = reinterpret_cast<const float*>(smem + S::O_F);
  const float* b1 = w1 + D1;
  const float* b2 = b1 + D1;
  const float* b3 = b2 + D2;
  unsigned char* w2h = smem + S::O_W2;
  unsigned char* w2l = w2h + S::W2B;
  unsigned char* w3h = smem + S::O_W3;
  unsigned char* w3l = w3h + S::W3B;
  unsigned char* bufh = smem + S::O_BUF;
  unsigned char* bufl = bufh + S::BUFB;
  unsigned char* rh = smem + S::O_R;
  unsigned char* rl = rh + S::RB;
  if (warp == 0) umma::tmem_alloc(&tbase, S::NCOLS);
  if (tid == 0) {
    umma::mbar_init(&bar, 1);
    umma::fence_mbar_init();
  }
  umma::fence_before_sync();
  __syncthreads();
  umma::fence_after_sync();
  const uint32_t tm = tbase;
  const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
  uint32_t phase = 0;
  int loaded = -1;
  const TcLists& L = a.L;
  const int ntiles = L.tstart[L.nnets];
  const uint32_t idesc2 = umma::idesc_bf16(128, S::D2p, false, false);
  const uint32_t idesc3 = umma::idesc_bf16(128, S::D3p, false, false);
  const uint32_t idescT = umma::idesc_bf16(128, S::NT, true, true);
  bool aborted = false;
  for (int g = blockIdx.x; g < ntiles && !aborted; g += gridDim.x) {
    int q = 0;
    while (q + 1 < L.nnets && L.tstart[q + 1] <= g) ++q;
    const int kt = g - L.tstart[q];
    const int lbase = L.eoff[(size_t)q * L.nloc];
    const int lend = L.eoff[(size_t)(q + 1) * L.nloc];
    const int e0 = lbase + kt * 128;
    const int ne = min(128, lend - e0);
    if (q != loaded) {
      __syncthreads();
      const uint4* src = reinterpret_cast<const uint4*>(a.nets + (size_t)q * a.net_bytes);
      uint4* dst = reinterpret_cast<uint4*>(smem);
      for (uint32_t i = tid; i < S::BLOB / 16; i += 128) dst[i] = src[i];
      loaded = q;
    }
    // environment rows of this tile and the local rank of each edge's centre
    const bool valid = tid < ne;
    const float4 rt = valid ? L.rt[e0 + tid] : make_float4(0.f, 0.f, 0.f, 0.f);
    const int row = valid ? L.row[e0 + tid] : -1;
    s_row[tid] = row;
    __syncthreads();
    const bool first = valid && (tid == 0 || s_row[tid - 1] != row);
    const unsigned fm = __ballot_sync(0xffffffffu, first);
    if (lane == 0) s_wcnt[warp] = __popc(fm);
    __syncthreads();
    int before = 0;
    for (int w = 0; w < warp; ++w) before += s_wcnt[w];
    const int na = s_wcnt[0] + s_wcnt[1] + s_wcnt[2] + s_wcnt[3];
    const unsigned le_mask = (lane == 31) ? 0xffffffffu : ((2u << lane) - 1u);
    const int lr = valid ? before + __popc(fm & le_mask) - 1 : -1;
    if (first) s_lrow[lr] = row;
    // layer 1 (scalar input, elementwise) -> A1
    float h1[D1];
#pragma unroll
    for (int n = 0; n < D1; ++n) h1[n] = valid ? tanh_fast(rt.x * w1[n] + b1[n]) : 0.f;
#pragma unroll
    for (int kg = 0; kg < S::D1p / 8; ++kg) {
      float v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = (kg * 8 + j < D1) ? h1[kg * 8 + j] : 0.f;
      const uint32_t o = (tid >> 3) * S::SBO_A1 + kg * 128 + (tid & 7) * 16;
      store8_split(bufh + o, bufl + o, v);
    }
    umma::fence_proxy_async();
    umma::fence_before_sync();
    __syncthreads();
    umma::fence_after_sync();
    if (tid == 0) {
      mma3(tm + S::C_D2, umma::smem_u32(bufh), umma::smem_u32(bufl), umma::smem_u32(w2h), umma::smem_u32(w2l), 128,
           S::SBO_A1, 128, S::SBO_W2, idesc2, S::D1p / 16, 256, 256);
      umma::commit(&bar);
    }
    bool ok = umma::mbar_wait(&bar, phase, kWaitLimit);
    phase ^= 1;
    if (__syncthreads_or(!ok)) {
      aborted = true;
      break;
    }
    umma::fence_after_sync();
    // layer 2 epilogue -> A2 (overwrites A1; the MMA that read it has completed)
    float h2[D2];
#pragma unroll
    for (int c = 0; c < S::D2p / 16; ++c) {
      float v[16];
      umma::ld16(tm + lane_base + S::C_D2 + c * 16, v);
      umma::wait_ld();
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int n = c * 16 + j;
        if (n < D2) h2[n] = valid ? tanh_fast(v[j] + b2[n]) + resid_of<D2, D1>(h1, n) : 0.f;
      }
    }
#pragma unroll
    for (int kg = 0; kg < S::D2p / 8; ++kg) {
      float v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = (kg * 8 + j < D2) ? h2[kg * 8 + j] : 0.f;
      const uint32_t o = (tid >> 3) * S::SBO_A2 + kg * 128 + (tid & 7) * 16;
      store8_split(bufh + o, bufl + o, v);
    }
    umma::fence_proxy_async();
    umma::fence_before_sync();
    __syncthreads();
    umma::fence_after_sync();
    if (tid == 0) {
      mma3(tm + S::C_D3, umma::smem_u32(bufh), umma::smem_u32(bufl), umma::smem_u32(w3h), umma::smem_u32(w3l), 128,
           S::SBO_A2, 128, S::SBO_W3, idesc3, S::D2p / 16, 256, 256);
      umma::commit(&bar);
    }
    ok = umma::mbar_wait(&bar, phase, kWaitLimit);
    phase ^= 1;
    if (__syncthreads_or(!ok)) {
      aborted = true;
      break;
    }
    umma::fence_after_sync();
    // layer 3 epilogue: G -> G^T (MN-major A operand of the contraction)
#pragma unroll
    for (int c = 0; c < S::D3p / 16; ++c) {
      float v[16];
      umma::ld16(tm + lane_base + S::C_D3 + c * 16, v);
      umma::wait_ld();
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int n = c * 16 + j;
        v[j] = (n < D3 && valid) ? tanh_fast(v[j] + b3[n]) + resid_of<D3, D2>(h2, n) : 0.f;
      }
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const uint32_t o = (2 * c + h) * S::SBO_G + (tid >> 3) * S::LBO_G + (tid & 7) * 16;
        store8_split(bufh + o, bufl + o, v + 8 * h);
      }
    }
    // contraction T^T[a][4r+k] = sum_e G_e[a] rt_e[k] over the edges of local atom r
    for (int ch = 0; ch * 8 < na; ++ch) {
      const int rr = lr - 8 * ch;
      const float rv[4] = {rt.x, rt.y, rt.z, rt.w};
#pragma unroll
      for (int ng = 0; ng < S::NT / 8; ++ng) {
        float v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int n = ng * 8 + j;
          v[j] = (valid && rr == (n >> 2)) ? rv[n & 3] : 0.f;
        }
        const uint32_t o = ng * S::SBO_R + (tid >> 3) * S::LBO_R + (tid & 7) * 16;
        store8_split(rh + o, rl + o, v);
      }
      umma::fence_proxy_async();
      umma::fence_before_sync();
      __syncthreads();
      umma::fence_after_sync();
      if (tid == 0) {
        mma3(tm + S::C_T, umma::smem_u32(bufh), umma::smem_u32(bufl), umma::smem_u32(rh), umma::smem_u32(rl),
             S::LBO_G, S::SBO_G, S::LBO_R, S::SBO_R, idescT, 128 / 16, 2 * S::LBO_G, 2 * S::LBO_R);
        umma::commit(&bar);
      }
      ok = umma::mbar_wait(&bar, phase, kWaitLimit);
      phase ^= 1;
      if (__syncthreads_or(!ok)) {
        aborted = true;
        break;
      }
      umma::fence_after_sync();
      float v[32];
      umma::ld16(tm + lane_base + S::C_T, v);
      umma::ld16(tm + lane_base + S::C_T + 16, v + 16);
      umma::wait_ld();
      if (tid < D3) {
        for (int r8 = 0; r8 < 8; ++r8) {
          const int r = 8 * ch + r8;
          if (r >= na) break;
          const int prow = s_lrow[r];
          const int lo = L.eoff[(size_t)q * L.nloc + prow] - lbase;
          const int piece = kt - lo / 128;
          float* dst = a.partial + (((size_t)q * L.nloc + prow) * L.pieces + piece) * 4 * D3;
#pragma unroll
          for (int k = 0; k < 4; ++k) dst[k * D3 + tid] = v[4 * r8 + k];
        }
      }
      umma::fence_before_sync();
      __syncthreads();
      umma::fence_after_sync();
    }
  }
  if (aborted && tid == 0) atomicAdd(a.err + kErrTcTimeout, 1);
  umma::fence_before_sync();
  __syncthreads();
  if (warp == 0) umma::tmem_dealloc(tm, S::NCOLS);
}

// ---------------------------------------------------------------- backward
// Shared-memory map of the backward tile kernel.  The forward weight blobs
// double as the backward B operands: read with MN-major descriptors they are
// W3 and W2 themselves (LBO and SBO swapped), so no transposed copy is kept.
template <int D1, int D2, int D3>
struct TcBwd {
  using F = TcShape<D1, D2, D3>;
  static constexpr int D1p = F::D1p, D2p = F::D2p, D3p = F::D3p, NT = 32;
  static constexpr uint32_t XB = 128 * D2p * 2;   // A1 / A2 / dz2 (one half)
  static constexpr uint32_t GB = 128 * D3p * 2;   // G, then dz3, K-major [edge][a]
  static constexpr uint32_t RB = 128 * NT * 2;    // environment rows, K-major [edge][n]
  static constexpr uint32_t TB = NT * D3p * 2;    // dT chunk stored [n][a]
  static constexpr uint32_t O_X = ((F::O_F + F::NF * 4 + 1023) / 1024) * 1024;
  static constexpr uint32_t O_G = O_X + 2 * XB;
  static constexpr uint32_t O_R = O_G + 2 * GB;
  static constexpr uint32_t O_T = O_R + 2 * RB;
  static constexpr uint32_t SMEM = O_T + 2 * TB;
  static constexpr uint32_t SBO_A1 = (D1p / 8) * 128, SBO_A2 = (D2p / 8) * 128, SBO_G = (D3p / 8) * 128;
  static constexpr uint32_t SBO_R = (NT / 8) * 128, SBO_T = (D3p / 8) * 128;
  // TMEM columns (512 allocated: one CTA per SM)
  static constexpr uint32_t C_D2 = 0, C_D3 = 64, C_DG = 192, C_DR = 320, C_DH1 = 352, NCOLS = 512;
  static_assert(D2p <= 64 && D3p <= 128 && D1p <= 32, "TMEM column plan");
};

struct BwdArgs {
  TcLists L;
  const unsigned char* nets;
  size_t net_bytes;
  const float* dT;     // [row][4][D3], already scaled by 1/N
  const double* rij;   // formatted neighbour list vectors
  double* gslot;       // dE/dr per slot
  int* err;
  double rcut, rcut_smth;
};

template <int D1, int D2, int D3>
__global__ void __launch_bounds__(128, 1) k_embed_bwd_tc(BwdArgs a) {
  using F = TcShape<D1, D2, D3>;
  using B = TcBwd<D1, D2, D3>;
  extern __shared__ __align__(1024) unsigned char smem[];
  __shared__ uint64_t bar;
  __shared__ uint32_t tbase;
  __shared__ int s_row[128];
  __shared__ int s_lrow[128];
  __shared__ int s_wcnt[4];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const float* w1 = reinterpret_cast<const float*>(smem + F::O_F);
  const float* b1 = w1 + D1;
  const float* b2 = b1 + D1;
  const float* b3 = b2 + D2;
  unsigned char* w2h = smem + F::O_W2;
  unsigned char* w2l = w2h + F::W2B;
  unsigned char* w3h = smem + F::O_W3;
  unsigned char* w3l = w3h + F::W3B;
  unsigned char* xh = smem + B::O_X;
  unsigned char* xl = xh + B::XB;
  unsigned char* gh = smem + B::O_G;
  unsigned char* gl = gh + B::GB;
  unsigned char* rh = smem + B::O_R;
  unsigned char* rl = rh + B::RB;
  unsigned char* th = smem + B::O_T;
  unsigned char* tl = th + B::TB;
  if (warp == 0) umma::tmem_alloc(&tbase, B::NCOLS);
  if (tid == 0) {
    umma::mbar_init(&bar, 1);
    umma::fence_mbar_init();
  }
  umma::fence_before_sync();
  __syncthreads();
  umma::fence_after_sync();
  const uint32_t tm = tbase;
  const uint32_t lb = (uint32_t)(warp * 32) << 16;
  uint32_t phase = 0;
  int loaded = -1;
  const TcLists& L = a.L;
  const int ntiles = L.tstart[L.nnets];
  const uint32_t id_2 = umma::idesc_bf16(128, D2p_of<D2>(), false, false);
  const uint32_t id_3 = umma::idesc_bf16(128, B::D3p, false, false);
  const uint32_t id_dg = umma::idesc_bf16(128, B::D3p, false, true);
  const uint32_t id_dr = umma::idesc_bf16(128, B::NT, false, false);
  const uint32_t id_h2 = umma::idesc_bf16(128, B::D2p, false, true);
  const uint32_t id_h1 = umma::idesc_bf16(128, B::D1p, false, true);
  bool aborted = false;
  auto sync_mma = [&]() {
    umma::fence_proxy_async();
    umma::fence_before_sync();
    __syncthreads();
    umma::fence_after_sync();
  };
  auto wait_mma = [&]() -> bool {
    const bool ok = umma::mbar_wait(&bar, phase, kWaitLimit);
    phase ^= 1;
    if (__syncthreads_or(!ok)) return false;
    umma::fence_after_sync();
    return true;
  };
  for (int g = blockIdx.x; g < ntiles && !aborted; g += gridDim.x) {
    int q = 0;
    while (q + 1 < L.nnets && L.tstart[q + 1] <= g) ++q;
    const int kt = g - L.tstart[q];
    const int lbase = L.eoff[(size_t)q * L.nloc];
    const int lend = L.eoff[(size_t)(q + 1) * L.nloc];
    const int e0 = lbase + kt * 128;
    const int ne = min(128, lend - e0);
    if (q != loaded) {
      __syncthreads();
      const uint4* src = reinterpret_cast<const uint4*>(a.nets + (size_t)q * a.net_bytes);
      uint4* dst = reinterpret_cast<uint4*>(smem);
      for (uint32_t i = tid; i < F::BLOB / 16; i += 128) dst[i] = src[i];
      loaded = q;
    }
    const bool valid = tid < ne;
    const float4 rt = valid ? L.rt[e0 + tid] : make_float4(0.f, 0.f, 0.f, 0.f);
    const int row = valid ? L.row[e0 + tid] : -1;
    const int slot = valid ? L.slot[e0 + tid] : -1;
    s_row[tid] = row;
    __syncthreads();
    const bool first = valid && (tid == 0 || s_row[tid - 1] != row);
    const unsigned fm = __ballot_sync(0xffffffffu, first);
    if (lane == 0) s_wcnt[warp] = __popc(fm);
    __syncthreads();
    int before = 0;
    for (int w = 0; w < warp; ++w) before += s_wcnt[w];
    const int na = s_wcnt[0] + s_wcnt[1] + s_wcnt[2] + s_wcnt[3];
    const unsigned le_mask = (lane == 31) ? 0xffffffffu : ((2u << lane) - 1u);
    const int lr = valid ? before + __popc(fm & le_mask) - 1 : -1;
    if (first) s_lrow[lr] = row;
    __syncthreads();
    const float rv[4] = {rt.x, rt.y, rt.z, rt.w};
    float dR[4] = {0.f, 0.f, 0.f, 0.f};
    // layer 1 recompute -> A1 (X)
    float h1[D1];
#pragma unroll
    for (int n = 0; n < D1; ++n) h1[n] = valid ? tanh_fast(rt.x * w1[n] + b1[n]) : 0.f;
#pragma unroll
    for (int kg = 0; kg < B::D1p / 8; ++kg) {
      float v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = (kg * 8 + j < D1) ? h1[kg * 8 + j] : 0.f;
      const uint32_t o = (tid >> 3) * B::SBO_A1 + kg * 128 + (tid & 7) * 16;
      store8_split(xh + o, xl + o, v);
    }
    sync_mma();
    if (tid == 0) {
      mma3(tm + B::C_D2, umma::smem_u32(xh), umma::smem_u32(xl), umma::smem_u32(w2h), umma::smem_u32(w2l), 128,
           B::SBO_A1, 128, F::SBO_W2, id_2, B::D1p / 16, 256, 256);
      umma::commit(&bar);
    }
    if (!wait_mma()) {
      aborted = true;
      break;
    }
    // layer 2 recompute -> A2 (X)
    float h2[D2];
#pragma unroll
    for (int c = 0; c < B::D2p / 16; ++c) {
      float v[16];
      umma::ld16(tm + lb + B::C_D2 + c * 16, v);
      umma::wait_ld();
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int n = c * 16 + j;
        if (n < D2) h2[n] = valid ? tanh_fast(v[j] + b2[n]) + resid_of<D2, D1>(h1, n) : 0.f;
      }
    }
#pragma unroll
    for (int kg = 0; kg < B::D2p / 8; ++kg) {
      float v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = (kg * 8 + j < D2) ? h2[kg * 8 + j] : 0.f;
      const uint32_t o = (tid >> 3) * B::SBO_A2 + kg * 128 + (tid & 7) * 16;
      store8_split(xh + o, xl + o, v);
    }
    sync_mma();
    if (tid == 0) {
      mma3(tm + B::C_D3, umma::smem_u32(xh), umma::smem_u32(xl), umma::smem_u32(w3h), umma::smem_u32(w3l), 128,
           B::SBO_A2, 128, F::SBO_W3, id_3, B::D2p / 16, 256, 256);
      umma::commit(&bar);
    }
    if (!wait_mma()) {
      aborted = true;
      break;
    }
    // layer 3 recompute: G -> K-major [edge][a] (A operand of dR = G dT^T)
#pragma unroll
    for (int c = 0; c < B::D3p / 16; ++c) {
      float v[16];
      umma::ld16(tm + lb + B::C_D3 + c * 16, v);
      umma::wait_ld();
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int n = c * 16 + j;
        v[j] = (n < D3 && valid) ? tanh_fast(v[j] + b3[n]) + resid_of<D3, D2>(h2, n) : 0.f;
      }
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const uint32_t o = (tid >> 3) * B::SBO_G + (2 * c + h) * 128 + (tid & 7) * 16;
        store8_split(gh + o, gl + o, v + 8 * h);
      }
    }
    // dG = R dT (accumulated over atom chunks) and dR = G dT^T (per chunk)
    for (int ch = 0; ch * 8 < na; ++ch) {
      const int rr = lr - 8 * ch;
#pragma unroll
      for (int ng = 0; ng < B::NT / 8; ++ng) {
        float v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int n = ng * 8 + j;
          v[j] = (valid && rr == (n >> 2)) ? rv[n & 3] : 0.f;
        }
        const uint32_t o = (tid >> 3) * B::SBO_R + ng * 128 + (tid & 7) * 16;
        store8_split(rh + o, rl + o, v);
      }
      for (int idx = tid; idx < B::NT * (B::D3p / 8); idx += 128) {
        const int n = idx / (B::D3p / 8), ag = idx - n * (B::D3p / 8);
        const int r = 8 * ch + (n >> 2), k = n & 3;
        float v[8];
        const float* src = (r < na) ? a.dT + ((size_t)s_lrow[r] * 4 + k) * D3 : nullptr;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int aa = ag * 8 + j;
          v[j] = (src && aa < D3) ? src[aa] : 0.f;
        }
        const uint32_t o = (n >> 3) * B::SBO_T + ag * 128 + (n & 7) * 16;
        store8_split(th + o, tl + o, v);
      }
      sync_mma();
      if (tid == 0) {
        // dG[e][a] += sum_n R[e][n] dT(a, n): B read MN-major from the [n][a] store
        for (int s = 0; s < B::NT / 16; ++s) {
          const uint32_t oa = s * 256, ob = s * 2 * B::SBO_T;
          const uint32_t ra = umma::smem_u32(rh) + oa, rla = umma::smem_u32(rl) + oa;
          const uint32_t tb = umma::smem_u32(th) + ob, tlb = umma::smem_u32(tl) + ob;
          umma::mma(tm + B::C_DG, umma::desc(ra, 128, B::SBO_R), umma::desc(tb, B::SBO_T, 128), id_dg,
                    (ch > 0 || s > 0) ? 1u : 0u);
          umma::mma(tm + B::C_DG, umma::desc(ra, 128, B::SBO_R), umma::desc(tlb, B::SBO_T, 128), id_dg, 1u);
          umma::mma(tm + B::C_DG, umma::desc(rla, 128, B::SBO_R), umma::desc(tb, B::SBO_T, 128), id_dg, 1u);
        }
        // dR[e][n] = sum_a G[e][a] dT(n, a): B read K-major from the same store
        mma3(tm + B::C_DR, umma::smem_u32(gh), umma::smem_u32(gl), umma::smem_u32(th), umma::smem_u32(tl), 128,
             B::SBO_G, 128, B::SBO_T, id_dr, B::D3p / 16, 256, 256);
        umma::commit(&bar);
      }
      if (!wait_mma()) {
        aborted = true;
        break;
      }
      float v[32];
      umma::ld16(tm + lb + B::C_DR, v);
      umma::ld16(tm + lb + B::C_DR + 16, v + 16);
      umma::wait_ld();
      if (rr >= 0 && rr < 8) {
#pragma unroll
        for (int r8 = 0; r8 < 8; ++r8)
          if (r8 == rr) {
#pragma unroll
            for (int k = 0; k < 4; ++k) dR[k] = v[4 * r8 + k];
          }
      }
      umma::fence_before_sync();
      __syncthreads();
      umma::fence_after_sync();
    }
    if (aborted) break;
    // dz3 = dG (1 - th3^2), th3 = G - residual; written over G (own row only)
#pragma unroll
    for (int c = 0; c < B::D3p / 16; ++c) {
      float dg[16];
      umma::ld16(tm + lb + B::C_DG + c * 16, dg);
      umma::wait_ld();
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const uint32_t o = (tid >> 3) * B::SBO_G + (2 * c + h) * 128 + (tid & 7) * 16;
        const uint4 uh = *reinterpret_cast<const uint4*>(gh + o);
        const uint4 ul = *reinterpret_cast<const uint4*>(gl + o);
        const uint32_t hw[4] = {uh.x, uh.y, uh.z, uh.w}, lw[4] = {ul.x, ul.y, ul.z, ul.w};
        float z[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int n = c * 16 + 8 * h + j;
          const uint32_t hb = (j & 1) ? (hw[j >> 1] & 0xFFFF0000u) : (hw[j >> 1] << 16);
          const uint32_t lbits = (j & 1) ? (lw[j >> 1] & 0xFFFF0000u) : (lw[j >> 1] << 16);
          const float gval = __uint_as_float(hb) + __uint_as_float(lbits);
          const float t3 = gval - resid_of<D3, D2>(h2, n);
          z[j] = (n < D3 && valid) ? dg[8 * h + j] * (1.f - t3 * t3) : 0.f;
        }
        store8_split(gh + o, gl + o, z);
      }
    }
    sync_mma();
    if (tid == 0) {
      // dh2[e][k2] = sum_a dz3[e][a] W3[k2][a]; W3 blob read MN-major
      mma3(tm + B::C_D2, umma::smem_u32(gh), umma::smem_u32(gl), umma::smem_u32(w3h), umma::smem_u32(w3l), 128,
           B::SBO_G, F::SBO_W3, 128, id_h2, B::D3p / 16, 256, 2 * F::SBO_W3);
      umma::commit(&bar);
    }
    if (!wait_mma()) {
      aborted = true;
      break;
    }
    // dh2 = MMA + residual gradient from dG; dz2 = dh2 (1 - th2^2) -> X.
    // TMEM is read in aligned 16-column chunks; the chunk holding dG[n + D2]
    // is known at compile time, so every register index below is static.
    float dh2[D2];
#pragma unroll
    for (int c = 0; c < B::D2p / 16; ++c) {
      float v[16], ga[16], gb[16], gc[16];
      umma::ld16(tm + lb + B::C_D2 + c * 16, v);
      umma::ld16(tm + lb + B::C_DG + c * 16, ga);
      constexpr int kShift = (D3 == 2 * D2) ? D2 : 0;
      const int cb = (c * 16 + kShift) / 16;
      umma::ld16(tm + lb + B::C_DG + min(cb, B::D3p / 16 - 1) * 16, gb);
      umma::ld16(tm + lb + B::C_DG + min(cb + 1, B::D3p / 16 - 1) * 16, gc);
      umma::wait_ld();
      float z[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int n = c * 16 + j;
        float r = v[j];
        if constexpr (D3 == D2) r += ga[j];
        if constexpr (D3 == 2 * D2) {
          const int m = n + D2;
          const int off = m - cb * 16;  // 0..31, static after unrolling
          r += ga[j] + (off < 16 ? gb[off & 15] : gc[off & 15]);
        }
        if (n < D2) {
          dh2[n] = valid ? r : 0.f;
          const float t2 = h2[n] - resid_of<D2, D1>(h1, n);
          z[j] = dh2[n] * (1.f - t2 * t2);
        } else {
          z[j] = 0.f;
        }
      }
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const uint32_t o = (tid >> 3) * B::SBO_A2 + (2 * c + h) * 128 + (tid & 7) * 16;
        store8_split(xh + o, xl + o, z + 8 * h);
      }
    }
    sync_mma();
    if (tid == 0) {
      // dh1[e][k1] = sum_n dz2[e][n] W2[k1][n]; W2 blob read MN-major
      mma3(tm + B::C_DH1, umma::smem_u32(xh), umma::smem_u32(xl), umma::smem_u32(w2h), umma::smem_u32(w2l), 128,
           B::SBO_A2, F::SBO_W2, 128, id_h1, B::D2p / 16, 256, 2 * F::SBO_W2);
      umma::commit(&bar);
    }
    if (!wait_mma()) {
      aborted = true;
      break;
    }
    float ds = 0.f;
#pragma unroll
    for (int c = 0; c < B::D1p / 16; ++c) {
      float v[16];
      umma::ld16(tm + lb + B::C_DH1 + c * 16, v);
      umma::wait_ld();
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int n = c * 16 + j;
        if (n < D1) {
          float r = v[j];
          if constexpr (D2 == D1) r += dh2[n];
          if constexpr (D2 == 2 * D1) r += dh2[n] + dh2[n + D1];
          ds += r * (1.f - h1[n] * h1[n]) * w1[n];
        }
      }
    }
    if (valid) {
      // chain rule to r_ij in fp64
      const double* rp = a.rij + 3 * (size_t)slot;
      const double x = rp[0], y = rp[1], z = rp[2];
      const double r2 = x * x + y * y + z * z, rr = sqrt(r2);
      double sw, dsw;
      smooth_switch(rr, a.rcut_smth, a.rcut, sw, dsw);
      const double ir = 1.0 / rr, ir2 = ir * ir;
      const double d0 = dsw * ir - sw * ir2;
      const double rvec[3] = {x, y, z};
      const double g0 = (double)dR[0] + (double)ds;
      double gout[3];
#pragma unroll
      for (int cc = 0; cc < 3; ++cc) {
        double acc = g0 * d0 * rvec[cc] * ir;
#pragma unroll
        for (int aa = 0; aa < 3; ++aa) {
          const double J = dsw * rvec[cc] * ir * rvec[aa] * ir2 +
                           sw * ((aa == cc ? ir2 : 0.0) - 2.0 * rvec[aa] * rvec[cc] * ir2 * ir2);
          acc += (double)dR[1 + aa] * J;
        }
        gout[cc] = acc;
      }
      double* go = a.gslot + 3 * (size_t)slot;
      go[0] = gout[0];
      go[1] = gout[1];
      go[2] = gout[2];
    }
    umma::fence_before_sync();
    __syncthreads();
    umma::fence_after_sync();
  }
  if (aborted && tid == 0) atomicAdd(a.err + kErrTcTimeout, 1);
  umma::fence_before_sync();
  __syncthreads();
  if (warp == 0) umma::tmem_dealloc(tm, B::NCOLS);
}

// dT[row][k][a] = (sum_b dD[a][b] T[k][b] + [a < M2] sum_c dD[c][a] T[k][c]) / N
template <int D3>
__global__ void __launch_bounds__(128) k_dT(int nloc, int ntypes, int M2, double inv_nnei,
                                            const int* __restrict__ type_start, const int* __restrict__ perm_atom,
                                            const float* __restrict__ T, const float* __restrict__ dD,
                                            float* __restrict__ dT) {
  extern __shared__ float sm[];
  float* sT = sm;             // 4 * D3
  float* sdD = sm + 4 * D3;   // D3 * M2
  const int r = blockIdx.x;
  if (r >= type_start[ntypes]) return;
  const int atom = perm_atom[r];
  for (int i = threadIdx.x; i < 4 * D3; i += blockDim.x) sT[i] = T[(size_t)atom * 4 * D3 + i];
  for (int i = threadIdx.x; i < D3 * M2; i += blockDim.x) sdD[i] = dD[(size_t)r * D3 * M2 + i];
  __syncthreads();
  for (int idx = threadIdx.x; idx < 4 * D3; idx += blockDim.x) {
    const int k = idx / D3, aa = idx - k * D3;
    const float* tk = sT + k * D3;
    float acc = 0.f;
    for (int b = 0; b < M2; ++b) acc += sdD[aa * M2 + b] * tk[b];
    if (aa < M2)
      for (int c = 0; c < D3; ++c) acc += sdD[c * M2 + aa] * tk[c];
    dT[(size_t)r * 4 * D3 + idx] = (float)(acc * inv_nnei);
  }
}

// T_i = (sum over nets and pieces, fixed order) / N; D = T^T T_< .
template <int D3>
__global__ void __launch_bounds__(128) k_t_combine(TcLists L, int ntypes, int M2, double inv_nnei,
                                                    const int* __restrict__ type_start,
                                                    const int* __restrict__ perm_atom,
                                                    const float* __restrict__ partial, float* __restrict__ T,
                                                    float* __restrict__ D) {
  __shared__ float sT[4 * D3];
  const int r = blockIdx.x;
  if (r >= type_start[ntypes]) return;
  const int tid = threadIdx.x;
  if (tid < D3) {
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int q = 0; q < L.nnets; ++q) {
      const size_t idx = (size_t)q * L.nloc + r;
      const int beg = L.eoff[idx], cnt = L.eoff[idx + 1] - beg;
      if (cnt <= 0) continue;
      const int base = L.eoff[(size_t)q * L.nloc];
      const int np = (beg + cnt - 1 - base) / 128 - (beg - base) / 128 + 1;
      for (int p = 0; p < np; ++p) {
        const float* src = partial + (idx * L.pieces + p) * 4 * D3;
#pragma unroll
        for (int k = 0; k < 4; ++k) acc[k] += src[k * D3 + tid];
      }
    }
    const int atom = perm_atom[r];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float v = (float)(acc[k] * inv_nnei);
      sT[k * D3 + tid] = v;
      T[(size_t)atom * 4 * D3 + k * D3 + tid] = v;
    }
  }
  __syncthreads();
  float* drow = D + (size_t)r * D3 * M2;
  for (int idx = tid; idx < D3 * M2; idx += blockDim.x) {
    const int aa = idx / M2, b = idx - aa * M2;
    float acc = 0.f;
#pragma unroll
    for (int k = 0; k < 4; ++k) acc += sT[k * D3 + aa] * sT[k * D3 + b];
    drow[idx] = acc;
  }
}

__global__ void k_edge_count(int nloc, int ntypes, int nnets, int tos, const int* __restrict__ type_start,
                             const int* __restrict__ perm_atom, const int* __restrict__ atype,
                             const int* __restrict__ cnt, int* __restrict__ ecount) {
  const size_t total = (size_t)nnets * nloc;
  const int nvalid = type_start[ntypes];
  for (size_t idx = blockIdx.x * (size_t)blockDim.x + threadIdx.x; idx < total;
       idx += (size_t)gridDim.x * blockDim.x) {
    const int q = (int)(idx / nloc), r = (int)(idx % nloc);
    int c = 0;
    if (r < nvalid) {
      const int atom = perm_atom[r];
      const int tj = tos ? q : q % ntypes;
      if (tos || q / ntypes == atype[atom]) c = cnt[(size_t)atom * ntypes + tj];
    }
    ecount[idx] = c;
  }
}

// One warp per (net, row): environment rows in fp64, stored as float4.
__global__ void k_edge_compact(SeaDev s, int nloc, const int* __restrict__ type_start,
                               const int* __restrict__ perm_atom, const int* __restrict__ atype,
                               const double* __restrict__ rij, const int* __restrict__ eoff,
                               float4* __restrict__ rt, int* __restrict__ rowv, int* __restrict__ slotv) {
  const size_t w = (blockIdx.x * (size_t)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= (size_t)s.nnets * nloc) return;
  const int q = (int)(w / nloc), r = (int)(w % nloc);
  const int beg = eoff[w], c = eoff[w + 1] - beg;
  if (c <= 0) return;
  const int atom = perm_atom[r];
  const int tj = s.type_one_side ? q : q % s.ntypes;
  const size_t base = (size_t)atom * s.selt + s.off[tj];
  for (int k = lane; k < c; k += 32) {
    const size_t sl = base + k;
    const double x = rij[3 * sl], y = rij[3 * sl + 1], z = rij[3 * sl + 2];
    const double rr = sqrt(x * x + y * y + z * z);
    double sw, dsw;
    smooth_switch(rr, s.rcut_smth, s.rcut, sw, dsw);
    const double ir = 1.0 / rr, s0 = sw * ir, s1 = s0 * ir;
    rt[beg + k] = make_float4((float)s0, (float)(s1 * x), (float)(s1 * y), (float)(s1 * z));
    rowv[beg + k] = r;
    slotv[beg + k] = (int)sl;
  }
}

__global__ void k_tile_table(int nnets, int nloc, const int* __restrict__ eoff, int* __restrict__ tstart) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  int t = 0;
  tstart[0] = 0;
  for (int q = 0; q < nnets; ++q) {
    const int e = eoff[(size_t)(q + 1) * nloc] - eoff[(size_t)q * nloc];
    t += (e + 127) / 128;
    tstart[q + 1] = t;
  }
}

template <int D1, int D2, int D3>
void pack_net(const std::vector<HostLayer>& net, std::vector<unsigned char>& out) {
  using S = TcShape<D1, D2, D3>;
  out.assign(S::BLOB, 0);
  auto put = [&](uint32_t base, uint32_t half, int rows, int K, auto val) {
    for (int r = 0; r < rows; ++r)
      for (int k = 0; k < K; ++k) {
        const float x = val(r, k);
        // round-to-nearest-even bf16 split on the host
        auto to_bf16 = [](float f) {
          uint32_t u;
          std::memcpy(&u, &f, 4);
          const uint32_t rnd = 0x7FFFu + ((u >> 16) & 1u);
          return (uint16_t)((u + rnd) >> 16);
        };
        auto from_bf16 = [](uint16_t h) {
          uint32_t u = (uint32_t)h << 16;
          float f;
          std::memcpy(&f, &u, 4);
          return f;
        };
        const uint16_t hi = to_bf16(x);
        const uint16_t lo = to_bf16(x - from_bf16(hi));
        const uint32_t o = (uint32_t)(r >> 3) * ((K / 8) * 128) + (uint32_t)(k >> 3) * 128 + (r & 7) * 16 + (k & 7) * 2;
        std::memcpy(&out[base + o], &hi, 2);
        std::memcpy(&out[base + half + o], &lo, 2);
      }
  };
  const HostLayer& L1 = net[0];
  const HostLayer& L2 = net[1];
  const HostLayer& L3 = net[2];
  put(S::O_W2, S::W2B, S::D2p, S::D1p,
      [&](int n, int k) { return (n < D2 && k < D1) ? (float)L2.w[(size_t)k * D2 + n] : 0.f; });
  put(S::O_W3, S::W3B, S::D3p, S::D2p,
      [&](int n, int k) { return (n < D3 && k < D2) ? (float)L3.w[(size_t)k * D3 + n] : 0.f; });
  float* f = reinterpret_cast<float*>(&out[S::O_F]);
  for (int n = 0; n < D1; ++n) f[n] = (float)L1.w[n];
  for (int n = 0; n < D1; ++n) f[D1 + n] = (float)L1.b[n];
  for (int n = 0; n < D2; ++n) f[2 * D1 + n] = (float)L2.b[n];
  for (int n = 0; n < D3; ++n) f[2 * D1 + D2 + n] = (float)L3.b[n];
}

enum class Inst { None, W25, W32 };
Inst which(const SeaDev& s) {
  if (s.nl != 3) return Inst::None;
  if (s.ed[1] == 25 && s.ed[2] == 50 && s.ed[3] == 100) return Inst::W25;
  if (s.ed[1] == 32 && s.ed[2] == 64 && s.ed[3] == 128) return Inst::W32;
  return Inst::None;
}

}  // namespace

bool tc_supported(const SeaDev& s) { return which(s) != Inst::None; }

size_t tc_net_bytes(const SeaDev& s) {
  switch (which(s)) {
    case Inst::W25:
      return TcShape<25, 50, 100>::BLOB;
    case Inst::W32:
      return TcShape<32, 64, 128>::BLOB;
    default:
      return 0;
  }
}

void tc_pack_net(const SeaDev& s, const std::vector<HostLayer>& net, std::vector<unsigned char>& out) {
  if (which(s) == Inst::W25) pack_net<25, 50, 100>(net, out);
  if (which(s) == Inst::W32) pack_net<32, 64, 128>(net, out);
}

int tc_pieces(const SeaDev& s) {
  int mx = 0;
  for (int t = 0; t < s.ntypes; ++t) mx = std::max(mx, s.sel[t]);
  return (mx + 127) / 128 + 1;
}

void launch_edge_count(cudaStream_t st, const SeaDev& s, int nloc, const int* type_start, const int* perm_atom,
                       const int* atype, const int* cnt, int* ecount) {
  const size_t total = (size_t)s.nnets * nloc;
  if (!total) return;
  const int blocks = (int)std::min<size_t>((total + 255) / 256, 148 * 8);
  count_launch();
  k_edge_count<<<blocks, 256, 0, st>>>(nloc, s.ntypes, s.nnets, s.type_one_side, type_start, perm_atom, atype, cnt,
                                       ecount);
}

void launch_edge_compact(cudaStream_t st, const SeaDev& s, int nloc, const int* type_start, const int* perm_atom,
                         const int* atype, const int* cnt, const double* rij, const int* eoff, float4* rt, int* row,
                         int* slot) {
  const size_t warps = (size_t)s.nnets * nloc;
  if (!warps) return;
  count_launch();
  k_edge_compact<<<(unsigned)((warps * 32 + 255) / 256), 256, 0, st>>>(s, nloc, type_start, perm_atom, atype, rij, eoff,
                                                                       rt, row, slot);
}

void launch_tile_table(cudaStream_t st, int nnets, int nloc, const int* eoff, int* tstart) {
  count_launch();
  k_tile_table<<<1, 32, 0, st>>>(nnets, nloc, eoff, tstart);
}

int embed_tc_grid(const SeaDev&) {
  int dev = 0, nsm = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
  return nsm;  // one CTA per SM (TMEM 256 columns and ~120 KB shared memory each)
}

template <int D1, int D2, int D3>
static void launch_fwd(cudaStream_t st, const SeaDev& s, const TcLists& L, int grid, const unsigned char* nets,
                       float* partial, int* err) {
  using S = TcShape<D1, D2, D3>;
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(k_embed_fwd_tc<D1, D2, D3>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)S::SMEM);
    attr = true;
  }
  FwdArgs a{L, nets, S::BLOB, partial, err, s.M1};
  count_launch();
  k_embed_fwd_tc<D1, D2, D3><<<grid, 128, S::SMEM, st>>>(a);
}

void launch_embed_fwd_tc(cudaStream_t st, const SeaDev& s, const TcLists& L, int grid, const unsigned char* nets,
                         float* partial, int* err) {
  if (which(s) == Inst::W25) launch_fwd<25, 50, 100>(st, s, L, grid, nets, partial, err);
  if (which(s) == Inst::W32) launch_fwd<32, 64, 128>(st, s, L, grid, nets, partial, err);
}

template <int D1, int D2, int D3>
static void launch_bwd(cudaStream_t st, const TcLists& L, int grid, const unsigned char* nets, const float* dT,
                       const double* rij, double* gslot, int* err, double rcut, double rs) {
  using Bw = TcBwd<D1, D2, D3>;
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(k_embed_bwd_tc<D1, D2, D3>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)Bw::SMEM);
    attr = true;
  }
  BwdArgs a{L, nets, TcShape<D1, D2, D3>::BLOB, dT, rij, gslot, err, rcut, rs};
  count_launch();
  k_embed_bwd_tc<D1, D2, D3><<<grid, 128, Bw::SMEM, st>>>(a);
}

void launch_embed_bwd_tc(cudaStream_t st, const SeaDev& s, const TcLists& L, int grid, const unsigned char* nets,
                         const float* dT, const double* rij, double* gslot, int* err) {
  if (which(s) == Inst::W25) launch_bwd<25, 50, 100>(st, L, grid, nets, dT, rij, gslot, err, s.rcut, s.rcut_smth);
  if (which(s) == Inst::W32) launch_bwd<32, 64, 128>(st, L, grid, nets, dT, rij, gslot, err, s.rcut, s.rcut_smth);
}

void launch_dT(cudaStream_t st, const SeaDev& s, int nloc, const int* type_start, const int* perm_atom, const float* T,
               const float* dD, float* dT) {
  if (nloc <= 0) return;
  const size_t smem = sizeof(float) * (4 + s.M2) * s.M1;
  count_launch();
  if (which(s) == Inst::W25)
    k_dT<100><<<nloc, 128, smem, st>>>(nloc, s.ntypes, s.M2, s.inv_nnei, type_start, perm_atom, T, dD, dT);
  else
    k_dT<128><<<nloc, 128, smem, st>>>(nloc, s.ntypes, s.M2, s.inv_nnei, type_start, perm_atom, T, dD, dT);
}

void launch_t_combine(cudaStream_t st, const SeaDev& s, const TcLists& L, const int* type_start, const int* perm_atom,
                      const float* partial, float* T, float* D) {
  if (L.nloc <= 0) return;
  count_launch();
  if (which(s) == Inst::W25)
    k_t_combine<100><<<L.nloc, 128, 0, st>>>(L, s.ntypes, s.M2, s.inv_nnei, type_start, perm_atom, partial, T, D);
  else
    k_t_combine<128><<<L.nloc, 128, 0, st>>>(L, s.ntypes, s.M2, s.inv_nnei, type_start, perm_atom, partial, T, D);
}

}  // namespace b200dp
