// Tensor-core embedding forward and backward (see embed_tc.cuh).
#include <algorithm>
#include <cmath>
#include <cstring>

#include "common.cuh"
#include "embed_tc.cuh"
#include "umma.cuh"

namespace b200dp {

namespace {


constexpr long long kWaitLimit = 1LL << 26;
constexpr int kFwdGroups = 2;  // groups of 8 warps per CTA in the forward kernel
static_assert(kFwdGroups == kItemPad, "the item table's padding is the forward's group count");

// Writes 8 consecutive fp32 values as bf16 hi and lo 16-byte chunks.
__device__ __forceinline__ void store8_split(unsigned char* hi, unsigned char* lo, const float* v) {
  uint32_t h[4], l[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) umma::split_pair(v[2 * j], v[2 * j + 1], h[j], l[j]);
  *reinterpret_cast<uint4*>(hi) = make_uint4(h[0], h[1], h[2], h[3]);
  *reinterpret_cast<uint4*>(lo) = make_uint4(l[0], l[1], l[2], l[3]);
}

// The three split products (hi*hi, hi*lo, lo*hi) of `steps` K = 16 steps from
// precomputed descriptors: K step s adds s * inc (bytes >> 4) to the
// start-address field of the A and B descriptors.
__device__ __forceinline__ void mma3d(uint32_t d, uint64_t a_hi, uint64_t a_lo, uint64_t b_hi, uint64_t b_lo,
                                      uint32_t idesc, int steps, uint32_t inc_a, uint32_t inc_b, bool accumulate) {
  for (int s = 0; s < steps; ++s) {
    const uint64_t oa = (uint64_t)(s * inc_a), ob = (uint64_t)(s * inc_b);
    umma::mma(d, a_hi + oa, b_hi + ob, idesc, (accumulate || s > 0) ? 1u : 0u);
    umma::mma(d, a_hi + oa, b_lo + ob, idesc, 1u);
    umma::mma(d, a_lo + oa, b_hi + ob, idesc, 1u);
  }
}

// Layer 2 with the hi and lo halves of W2 side by side as one N = 128 operand
// (they are adjacent in the blob: lo's rows follow hi's at the row-group stride):
// D[0, 64) += A_hi W_hi + A_lo W_hi, D[64, 128) += A_hi W_lo; the epilogue adds
// the two halves.  Four MMAs instead of six, and A_hi is read once per K step.
__device__ __forceinline__ void mma_l2(uint32_t d, uint64_t a_hi, uint64_t a_lo, uint64_t w_hi, uint32_t id128,
                                       uint32_t id64) {
#pragma unroll
  for (int s = 0; s < 2; ++s) {
    const uint64_t o = (uint64_t)(s * (256 >> 4));
    umma::mma(d, a_hi + o, w_hi + o, id128, s > 0 ? 1u : 0u);
    umma::mma(d, a_lo + o, w_hi + o, id64, 1u);
  }
}

// Work item -> (net, first row, end row) and its edge range.
struct Item {
  int q, rb, re, e0, e1;
};
__device__ __forceinline__ Item item_compute(const TcLists& L, int it) {
  Item r;
  int q = 0;
  while (q + 1 < L.nnets && L.istart[q + 1] <= it) ++q;
  r.q = q;
  int rb0 = 0, re0 = L.type_start[L.ntypes];
  if (!L.type_one_side) {
    const int ti = q / L.ntypes;
    rb0 = L.type_start[ti];
    re0 = L.type_start[ti + 1];
  }
  r.rb = min(rb0 + kItemRows * (it - L.istart[q]), re0);  // padded items are empty
  r.re = min(r.rb + kItemRows, re0);
  r.e0 = L.eoff[(size_t)q * L.nloc + r.rb];
  r.e1 = L.eoff[(size_t)q * L.nloc + r.re];
  return r;
}
// The kernels read the precomputed record (two 16-byte loads instead of a
// chain of dependent lookups).
__device__ __forceinline__ Item item_of(const TcLists& L, int it) {
  const int4 a = L.items[2 * it], b = L.items[2 * it + 1];
  return Item{a.x, a.y, a.z, a.w, b.x};
}

// ---------------------------------------------------------------- forward
// Two threads per edge.  Every layer's output features are divided between
// the two threads of an edge ("halves"), so that each thread owns the
// residual sources of its own features: with DeePMD's concat rule
// (d_out = 2 d_in, feature n uses input n mod d_in) the half that owns input
// feature i also owns outputs i and i + d_in; with the identity rule it owns
// output i.  The host permutes the weights into this order: positions
// [0, H) of a layer are half 0's features, [H, 2H) half 1's, with zero
// padding; H = 16, 32, 64 for layers 1, 2, 3.  The contraction operand G^T
// (128 positions x 128 edges) is written by all 256 threads of a group at
// once, and its rows stay in position order through the T accumulator; the
// store of T maps positions back to feature indices.
constexpr int res_kind(int dout, int din) { return dout == din ? 1 : (dout == 2 * din ? 2 : 0); }

template <int D1, int D2, int D3>
struct Split {
  static constexpr int H1 = 16, H2 = 32, H3 = 64;  // slots per half
  static constexpr int R2 = res_kind(D2, D1), R3 = res_kind(D3, D2);
  static constexpr int c1(int h) { return h == 0 ? (D1 + 1) / 2 : D1 / 2; }
  static constexpr int c2(int h) { return R2 == 1 ? c1(h) : R2 == 2 ? 2 * c1(h) : (h == 0 ? (D2 + 1) / 2 : D2 / 2); }
  static constexpr int c3(int h) { return R3 == 1 ? c2(h) : R3 == 2 ? 2 * c2(h) : (h == 0 ? (D3 + 1) / 2 : D3 / 2); }
  // input slot (same half) feeding the residual of output slot j, -1 for none
  static constexpr int src2(int h, int j) { return R2 == 1 ? j : R2 == 2 ? (j < c1(h) ? j : j - c1(h)) : -1; }
  static constexpr int src3(int h, int j) { return R3 == 1 ? j : R3 == 2 ? (j < c2(h) ? j : j - c2(h)) : -1; }
  static_assert(c1(0) <= H1 && c2(0) <= H2 && c3(0) <= H3, "widths of the split forward kernel");
  // A padding slot of half 0 carries a constant 1 whose weight row is the
  // next layer's bias, so the MMA adds the bias (when such a slot exists).
  static constexpr bool FOLD2 = c1(0) < H1, FOLD3 = c2(0) < H2;
};

// Pre-activations arrive scaled by c = 2 log2(e) (the host scales weights
// and biases), so tanh(z) = 1 - 2 / (1 + 2^(c z)); `base` is 1 plus the
// residual input, which turns the tanh and the residual add into one FMA.
constexpr float kTanhScale = 2.8853900817779268f;
__device__ __forceinline__ float tanh_scaled(float zc, float base) {
  float e, r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(zc));
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(1.0f + e));
  return fmaf(-2.0f, r, base);
}

// Host: original feature index of every position of the three layers (-1 = padding).
template <int D1, int D2, int D3>
void split_order(std::vector<int>& p1, std::vector<int>& p2, std::vector<int>& p3) {
  using P = Split<D1, D2, D3>;
  p1.assign(2 * P::H1, -1);
  p2.assign(2 * P::H2, -1);
  p3.assign(2 * P::H3, -1);
  for (int h = 0; h < 2; ++h) {
    for (int j = 0; j < P::c1(h); ++j) p1[h * P::H1 + j] = (h ? P::c1(0) : 0) + j;
    for (int j = 0; j < P::c2(h); ++j) {
      const int s = P::src2(h, j);
      p2[h * P::H2 + j] = P::R2 == 0 ? (h ? P::c2(0) : 0) + j : p1[h * P::H1 + s] + (j >= P::c1(h) ? D1 : 0);
    }
    for (int j = 0; j < P::c3(h); ++j) {
      const int s = P::src3(h, j);
      p3[h * P::H3 + j] = P::R3 == 0 ? (h ? P::c3(0) : 0) + j : p2[h * P::H2 + s] + (j >= P::c2(h) ? D2 : 0);
    }
  }
}

// Packed net (global memory and the front of shared memory), shared by the
// forward and backward kernels: W2 and W3 as K-major B operands in position
// order (element (n, k) = W[k][n], bf16 hi then lo), then fp32 w1, b1
// (layer-1 positions), b2, b3, and the feature index of each layer-3
// position.  Weights and biases are scaled by c = 2 log2(e).
struct FwdBlob {
  static constexpr uint32_t W2B = 64 * 32 * 2, W3B = 128 * 64 * 2;
  static constexpr uint32_t O_W2 = 0, O_W3 = 2 * W2B, O_F = O_W3 + 2 * W3B;
  static constexpr uint32_t O_MAP = O_F + (32 + 32 + 64 + 128) * 4;
  static constexpr uint32_t BLOB = O_MAP + 128 * 4;
  static constexpr uint32_t O_END = (BLOB + 1023) / 1024 * 1024;
  static constexpr uint32_t SBO_W2 = (32 / 8) * 128, SBO_W3 = (64 / 8) * 128;
};

template <int D1, int D2, int D3>
struct NetBlob {
  static_assert(D1 > 2, "a layer-1 residual is not handled by the tensor-core path");
  static constexpr uint32_t OFF_FWD = 0;
  static constexpr uint32_t BYTES = FwdBlob::O_END;
};

// Shared memory of one group (256 threads): A1 (layer-2 A), X (layer-3 A),
// then G^T (contraction A, MN-major, 128 positions x 128 edges) over both,
// and R~ (contraction B, MN-major, 32 columns x 128 edges, bf16 hi and lo side
// by side as 64 columns).
struct FwdGroup {
  static constexpr uint32_t A1B = 128 * 32 * 2, XB = 128 * 64 * 2, GB = 128 * 128 * 2, RB = 32 * 128 * 2;
  static constexpr uint32_t O_A1 = 0, O_X = 2 * A1B, O_G = 0, O_R = 2 * GB;
  static constexpr uint32_t BYTES = O_R + 2 * RB;
  static constexpr uint32_t SBO_A1 = (32 / 8) * 128, SBO_X = (64 / 8) * 128;
  static constexpr uint32_t SBO_G = 128, LBO_G = 16 * 128;  // MN-major, 16 position blocks per edge block
  // R~ as one MN-major operand of 64 columns: per block of 8 edges, the 4 column
  // blocks of the hi half, then the 4 of the lo half
  static constexpr uint32_t SBO_R = 128, LBO_R = 8 * 128;
  static constexpr uint32_t C_D = 0, C_T = 128, COLS = 256;  // TMEM columns per group (T: 64)
  static constexpr int NG = 2;
  static constexpr uint32_t SMEM = FwdBlob::O_END + NG * BYTES;
};
static_assert(FwdGroup::O_X + 2 * FwdGroup::XB <= FwdGroup::O_R, "A1 and X lie inside the G^T region");
static_assert(kFwdGroups == FwdGroup::NG, "item padding matches the groups per CTA");

struct FwdArgs {
  TcLists L;
  const unsigned char* nets;
  size_t net_bytes, fwd_off;
  float* Tq;
  int* err;
};

// The per-half pieces of one subtile (H = the thread's half, compile time).
// Rows of edges beyond the subtile compute finite values from a zero
// environment row; their R~ rows are zero, so they add nothing to T.
// h1 / h2 hold the activations to store, h1p / h2p hold 1 + activation for
// the next layer's residual (or 1 where a feature has no residual).
template <int D1, int D2, int D3, int H>
__device__ __forceinline__ void fwd_layer1(const float* f, float s, float (&h1)[16], float (&h1p)[16]) {
  using P = Split<D1, D2, D3>;
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    if (j < P::c1(H)) {
      const float y = tanh_scaled(fmaf(s, f[H * 16 + j], f[32 + H * 16 + j]), 1.0f);
      h1[j] = y;
      h1p[j] = y + 1.0f;
    } else {
      h1[j] = (P::FOLD2 && H == 0 && j == P::c1(0)) ? 1.0f : 0.0f;
      h1p[j] = 1.0f;
    }
  }
}

template <int D1, int D2, int D3, int H>
__device__ __forceinline__ void fwd_epi2(const float* f, uint32_t taddr, const float (&h1p)[16], float (&h2)[32],
                                         float (&h2p)[32]) {
  using P = Split<D1, D2, D3>;
  float v[32];
#pragma unroll
  for (int c = 0; c < 2; ++c) {  // the two column halves of the layer-2 accumulator
    float w[16];
    umma::ld16(taddr + H * 32 + 16 * c, v + 16 * c);
    umma::ld16(taddr + 64 + H * 32 + 16 * c, w);
    umma::wait_ld();
#pragma unroll
    for (int j = 0; j < 16; ++j) v[16 * c + j] += w[j];
  }
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    if (j < P::c2(H)) {
      const float z = P::FOLD2 ? v[j] : v[j] + f[64 + H * 32 + j];
      const float y = tanh_scaled(z, P::R2 != 0 ? h1p[P::src2(H, j)] : 1.0f);
      h2[j] = y;
      h2p[j] = y + 1.0f;
    } else {
      h2[j] = (P::FOLD3 && H == 0 && j == P::c2(0)) ? 1.0f : 0.0f;
      h2p[j] = 1.0f;
    }
  }
}

template <int D1, int D2, int D3, int H>
__device__ __forceinline__ void fwd_epi3(const float* f, uint32_t taddr, const float (&h2p)[32], unsigned char* gh,
                                         unsigned char* gl, int e) {
  using P = Split<D1, D2, D3>;
  using S = FwdGroup;
  // TMEM loads one chunk ahead: the load of chunk c + 1 overlaps the tanh of chunk c
  float nxt[16];
  umma::ld16(taddr + H * 64, nxt);
  umma::wait_ld();
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    float v[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = nxt[i];
    if (c + 1 < 4) umma::ld16(taddr + H * 64 + (c + 1) * 16, nxt);
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int j = c * 16 + i;
      if (j < P::c3(H)) {
        const float z = P::FOLD3 ? v[i] : v[i] + f[128 + H * 64 + j];
        v[i] = tanh_scaled(z, P::R3 != 0 ? h2p[P::src3(H, j)] : 1.0f);
      } else {
        v[i] = 0.f;
      }
    }
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const int mb = H * 8 + 2 * c + hh;
      const uint32_t o = mb * S::SBO_G + (e >> 3) * S::LBO_G + (e & 7) * 16;
      store8_split(gh + o, gl + o, v + 8 * hh);
    }
    if (c + 1 < 4) umma::wait_ld();
  }
}

template <int D1, int D2, int D3>
__global__ void __launch_bounds__(256 * FwdGroup::NG, 1) k_embed_fwd_tc(FwdArgs a) {
  using S = FwdGroup;
  using B = FwdBlob;
  extern __shared__ __align__(1024) unsigned char smem[];
  __shared__ uint64_t bars[S::NG];
  __shared__ uint32_t tbase;
  const int gtid = threadIdx.x, g = gtid >> 8, t = gtid & 255, hf = t >> 7, e = t & 127;
  const int bid = 1 + g;  // named barrier of this group
  const float* f = reinterpret_cast<const float*>(smem + B::O_F);
  const int* pmap = reinterpret_cast<const int*>(smem + B::O_MAP);
  unsigned char* gbase = smem + B::O_END + g * S::BYTES;
  unsigned char* a1h = gbase + S::O_A1;
  unsigned char* a1l = a1h + S::A1B;
  unsigned char* xh = gbase + S::O_X;
  unsigned char* xl = xh + S::XB;
  unsigned char* gh = gbase + S::O_G;
  unsigned char* gl = gh + S::GB;
  unsigned char* rh = gbase + S::O_R;

  uint64_t* bar = &bars[g];
  if ((gtid >> 5) == 0) umma::tmem_alloc(&tbase, 512);
  if (t == 0) {
    umma::mbar_init(bar, 1);
    umma::fence_mbar_init();
  }
  umma::fence_before_sync();
  __syncthreads();
  umma::fence_after_sync();
  const uint32_t tm = tbase + g * S::COLS;
  const uint32_t lane_base = (uint32_t)((e >> 5) * 32) << 16;
  uint32_t phase = 0;
  int loaded = -1;
  const TcLists& L = a.L;
  const int nitems = L.istart[L.nnets];
  // descriptors of the fixed operands (later K steps add (bytes >> 4))
  const uint64_t dw2h = umma::desc(umma::smem_u32(smem + B::O_W2), 128, B::SBO_W2);
  const uint64_t dw3h = umma::desc(umma::smem_u32(smem + B::O_W3), 128, B::SBO_W3);
  const uint64_t dw3l = umma::desc(umma::smem_u32(smem + B::O_W3 + B::W3B), 128, B::SBO_W3);
  const uint64_t da1h = umma::desc(umma::smem_u32(a1h), 128, S::SBO_A1);
  const uint64_t da1l = umma::desc(umma::smem_u32(a1l), 128, S::SBO_A1);
  const uint64_t dxh = umma::desc(umma::smem_u32(xh), 128, S::SBO_X);
  const uint64_t dxl = umma::desc(umma::smem_u32(xl), 128, S::SBO_X);
  const uint64_t dgh = umma::desc(umma::smem_u32(gh), S::LBO_G, S::SBO_G);
  const uint64_t dgl = umma::desc(umma::smem_u32(gl), S::LBO_G, S::SBO_G);
  const uint64_t drh = umma::desc(umma::smem_u32(rh), S::LBO_R, S::SBO_R);
  const uint32_t id2 = umma::idesc_bf16(128, 64, false, false);
  const uint32_t id3 = umma::idesc_bf16(128, 128, false, false);
  const uint32_t idT = umma::idesc_bf16(128, 32, true, true), idT64 = umma::idesc_bf16(128, 64, true, true);
  const uint32_t id2w = umma::idesc_bf16(128, 128, false, false);
  bool aborted = false;
  auto sync_mma = [&]() {
    umma::fence_proxy_async();
    umma::fence_before_sync();
    umma::bar_sync(bid, 256);
    umma::fence_after_sync();
  };
  auto wait_mma = [&]() -> bool {
    const bool ok = umma::mbar_wait(bar, phase, kWaitLimit);
    phase ^= 1;
    if (umma::bar_sync_or(bid, 256, !ok)) return false;
    umma::fence_after_sync();
    return true;
  };
  for (int base = blockIdx.x * S::NG; base < nitems; base += gridDim.x * S::NG) {
    const int qr = item_of(L, base).q;
    if (qr != loaded) {
      __syncthreads();
      const uint4* src = reinterpret_cast<const uint4*>(a.nets + (size_t)qr * a.net_bytes + a.fwd_off);
      uint4* dst = reinterpret_cast<uint4*>(smem);
      for (uint32_t i = gtid; i < B::BLOB / 16; i += 256 * S::NG) dst[i] = src[i];
      loaded = qr;
      __syncthreads();
    }
    if (aborted) continue;  // keep taking part in the CTA-wide barriers above
    const Item I = item_of(L, base + g);
    bool first = true, pending = false;
    for (int sub = I.e0; sub < I.e1; sub += 128) {
      const int ne = min(128, I.e1 - sub);
      const bool valid = e < ne;
      const float4 rt = valid ? L.rt[sub + e] : make_float4(0.f, 0.f, 0.f, 0.f);
      const int rloc = valid ? L.row[sub + e] - I.rb : -1;
      float h1[16], h1p[16], h2[32], h2p[32];
      if (hf == 0)
        fwd_layer1<D1, D2, D3, 0>(f, rt.x, h1, h1p);
      else
        fwd_layer1<D1, D2, D3, 1>(f, rt.x, h1, h1p);
      if (pending) {  // the previous contraction still reads G^T (over A1) and R~
        if (!wait_mma()) {
          aborted = true;
          break;
        }
        pending = false;
      }
#pragma unroll
      for (int kk = 0; kk < 2; ++kk) {
        const uint32_t o = (e >> 3) * S::SBO_A1 + (2 * hf + kk) * 128 + (e & 7) * 16;
        store8_split(a1h + o, a1l + o, h1 + 8 * kk);
      }
      {  // environment row in the column block of its centre; this half writes centres 4 hf .. 4 hf + 3
        const float rv[4] = {rt.x, rt.y, rt.z, rt.w};
#pragma unroll
        for (int nn = 0; nn < 2; ++nn) {
          float v[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const int n = 16 * hf + 8 * nn + j;
            v[j] = (rloc == (n >> 2)) ? rv[j & 3] : 0.f;
          }
          const int nb = 2 * hf + nn;
          const uint32_t o = nb * S::SBO_R + (e >> 3) * S::LBO_R + (e & 7) * 16;
          store8_split(rh + o, rh + o + 4 * S::SBO_R, v);
        }
      }
      sync_mma();
      if (t == 0) {
        mma_l2(tm + S::C_D, da1h, da1l, dw2h, id2w, id2);
        umma::commit(bar);
      }
      if (!wait_mma()) {
        aborted = true;
        break;
      }
      if (hf == 0)
        fwd_epi2<D1, D2, D3, 0>(f, tm + lane_base + S::C_D, h1p, h2, h2p);
      else
        fwd_epi2<D1, D2, D3, 1>(f, tm + lane_base + S::C_D, h1p, h2, h2p);
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const uint32_t o = (e >> 3) * S::SBO_X + (4 * hf + kk) * 128 + (e & 7) * 16;
        store8_split(xh + o, xl + o, h2 + 8 * kk);
      }
      sync_mma();  // also orders every D2 read before MMA3 overwrites the columns
      if (t == 0) {
        mma3d(tm + S::C_D, dxh, dxl, dw3h, dw3l, id3, 4, 256 >> 4, 256 >> 4, false);
        umma::commit(bar);
      }
      if (!wait_mma()) {
        aborted = true;
        break;
      }
      if (hf == 0)
        fwd_epi3<D1, D2, D3, 0>(f, tm + lane_base + S::C_D, h2p, gh, gl, e);
      else
        fwd_epi3<D1, D2, D3, 1>(f, tm + lane_base + S::C_D, h2p, gh, gl, e);
      sync_mma();
      if (t == 0) {
        // T[:, 0, 32) += G_hi R_hi + G_lo R_hi, T[:, 32, 64) += G_hi R_lo (summed at the store)
        const int steps = (ne + 15) / 16;
        for (int s2 = 0; s2 < steps; ++s2) {
          const uint64_t oa = (uint64_t)(s2 * ((2 * S::LBO_G) >> 4)), ob = (uint64_t)(s2 * ((2 * S::LBO_R) >> 4));
          umma::mma(tm + S::C_T, dgh + oa, drh + ob, idT64, (!first || s2 > 0) ? 1u : 0u);
          umma::mma(tm + S::C_T, dgl + oa, drh + ob, idT, 1u);
        }
        umma::commit(bar);
      }
      first = false;
      pending = true;
    }
    if (aborted) continue;
    if (pending && !wait_mma()) {
      aborted = true;
      continue;
    }
    // T[position][4 r + k] -> Tq[net][row][k][feature]; half hf stores centres 4 hf .. 4 hf + 3
    const int a_idx = pmap[e];
    float v[16];
    if (I.e1 > I.e0) {
      float w[16];
      umma::ld16(tm + lane_base + S::C_T + 16 * hf, v);
      umma::ld16(tm + lane_base + S::C_T + 32 + 16 * hf, w);
      umma::wait_ld();
#pragma unroll
      for (int j = 0; j < 16; ++j) v[j] += w[j];
    } else {
#pragma unroll
      for (int j = 0; j < 16; ++j) v[j] = 0.f;
    }
    if (a_idx >= 0) {
      for (int rr = 0; rr < 4; ++rr) {
        const int r = 4 * hf + rr;
        if (r >= I.re - I.rb) break;
        float* dst = a.Tq + (((size_t)I.q * L.nloc + I.rb + r) * 4) * D3 + a_idx;
#pragma unroll
        for (int k = 0; k < 4; ++k) dst[k * D3] = v[4 * rr + k];
      }
    }
    umma::fence_before_sync();
    umma::bar_sync(bid, 256);
    umma::fence_after_sync();
  }
  if (aborted && t == 0) atomicAdd(a.err + kErrTcTimeout, 1);
  umma::fence_before_sync();
  __syncthreads();
  if ((gtid >> 5) == 0) umma::tmem_dealloc(tbase, 512);
}

// ---------------------------------------------------------------- backward
// Same split as the forward: two threads per edge, each owning half of the
// positions of every layer (and the residual sources of its own positions).
// Per subtile the forward is recomputed with the same MMAs; then
//   dG[e][p] = sum_k R~[e][k] dT[row][k][p]    (rank 4: CUDA cores)
//   dR~[e][k] = sum_p G[e][p] dT[row][k][p]   (rank 4: CUDA cores)
//   dh2 = dz3 W3^T, dh1 = dz2 W2^T             (tcgen05 MMAs)
// dz3 is written back into the TMEM columns of the layer-3 pre-activations
// (bf16 hi and lo halves per K step) and read from there as the A operand;
// dz2 goes to the shared-memory slot of the layer-3 A operand.  The weights
// are the forward blob (scaled by c = 2 log2(e)); dT is staged scaled by 1/c,
// so the MMAs with scaled weights return true gradients.
struct BwdGroup {
  static constexpr uint32_t A1B = 128 * 32 * 2, XB = 128 * 64 * 2, DTB = kItemRows * 128 * 16;
  static constexpr uint32_t T2B = 16 * 256 * 4;  // layer-2 tanh outputs 16..31 (0..15 reuse the A1 slot)
  static constexpr uint32_t O_A1 = 0, O_X = 2 * A1B, O_DT = O_X + 2 * XB, O_T2 = O_DT + DTB, BYTES = O_T2 + T2B;
  static constexpr uint32_t SBO_A1 = (32 / 8) * 128, SBO_X = (64 / 8) * 128;
  static constexpr uint32_t C_D2 = 0, C_D3 = 64, C_DH1 = 192, COLS = 256;  // TMEM columns per group
  static constexpr int NG = 2;
  static constexpr uint32_t SMEM = FwdBlob::O_END + NG * BYTES;
};
static_assert(kFwdGroups == BwdGroup::NG, "item padding matches the groups per CTA");

struct BwdArgs {
  TcLists L;
  const unsigned char* nets;
  size_t net_bytes, fwd_off;
  const float* dT;    // [row][4][D3], already scaled by 1/N
  double* genv;       // per slot: dE/d(environment row) as (dE/ds + dE/dR~_0, dE/dR~_1..3), fp64
  int* err;
};

constexpr float kInvTanhScale = 0.34657359027997264f;  // 1 / c

// r = 1 / (1 + 2^zc): tanh(z) = 1 - 2 r for the scaled pre-activation zc = c z.
__device__ __forceinline__ float tanh_r(float zc) {
  float e, r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(zc));
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(1.0f + e));
  return r;
}


// D[tmem] (+)= A[tmem] * B^T: the A operand is read from tensor memory.
__device__ __forceinline__ void mma_ta(uint32_t d, uint32_t a_tmem, uint64_t b, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d),
      "r"(a_tmem), "l"(b), "r"(idesc), "r"(accumulate));
}

// The layer-2 tanh outputs of a group's 256 threads, [position j][thread] fp32
// (bank-conflict free): positions 0..15 in the layer-1 operand slot, which is
// free from the completion of the layer-2 MMA until the next subtile's layer-1
// stores (every read happens before the barrier ahead of the dh1 MMA),
// positions 16..31 in a slot of their own.  Keeping them out of registers
// leaves the backward epilogues without spills.
struct T2Slots {
  float* lo;
  float* hi;
  int t;
  __device__ __forceinline__ float& operator[](int j) const {
    return j < 16 ? lo[j * 256 + t] : hi[(j - 16) * 256 + t];
  }
};

template <int D1, int D2, int D3, int H>
__device__ __forceinline__ void bwd_epi2(const float* f, uint32_t taddr, const float (&h1p)[16], float (&h2)[32],
                                         const T2Slots& t2) {
  using P = Split<D1, D2, D3>;
  float v[32];
#pragma unroll
  for (int c = 0; c < 2; ++c) {  // the two column halves of the layer-2 accumulator
    float w[16];
    umma::ld16(taddr + H * 32 + 16 * c, v + 16 * c);
    umma::ld16(taddr + 64 + H * 32 + 16 * c, w);
    umma::wait_ld();
#pragma unroll
    for (int j = 0; j < 16; ++j) v[16 * c + j] += w[j];
  }
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    if (j < P::c2(H)) {
      const float r = tanh_r(P::FOLD2 ? v[j] : v[j] + f[64 + H * 32 + j]);
      t2[j] = fmaf(-2.0f, r, 1.0f);
      h2[j] = fmaf(-2.0f, r, P::R2 != 0 ? h1p[P::src2(H, j)] : 1.0f);  // t2 + h1 (1 + h1 - 2 r)
    } else {
      t2[j] = 0.f;
      h2[j] = (P::FOLD3 && H == 0 && j == P::c2(0)) ? 1.0f : 0.0f;
    }
  }
}

// Layer 3 with its gradient for the 64 positions of half H.  Returns the
// partial dR~' (over this half's positions) and accumulates racc' (residual
// gradient into layer 2, scaled by 1/c); writes dz3' into TMEM in place.
template <int D1, int D2, int D3, int H>
__device__ __forceinline__ void bwd_epi3(const float* f, uint32_t taddr, const float4* dts, float4 rt,
                                         const float (&h1p)[16], const T2Slots& t2, float (&racc)[32],
                                         float4& dR) {
  using P = Split<D1, D2, D3>;
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    float z[16];
    umma::ld16(taddr + H * 64 + c * 16, z);
    umma::wait_ld();
    float v[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int j = c * 16 + i;
      if (j < P::c3(H)) {
        const float4 d4 = dts[H * 64 + j];
        const float dg = fmaf(rt.x, d4.x, fmaf(rt.y, d4.y, fmaf(rt.z, d4.z, rt.w * d4.w)));
        const float r = tanh_r(P::FOLD3 ? z[i] : z[i] + f[128 + H * 64 + j]);
        const float t3 = fmaf(-2.0f, r, 1.0f);
        float gv = t3;
        if constexpr (P::R3 != 0) {
          const int s = P::src3(H, j);
          float h2s = t2[s];
          if constexpr (P::R2 != 0) h2s += h1p[P::src2(H, s)] - 1.0f;
          gv += h2s;
          racc[s] += dg;
        }
        dR.x = fmaf(gv, d4.x, dR.x);
        dR.y = fmaf(gv, d4.y, dR.y);
        dR.z = fmaf(gv, d4.z, dR.z);
        dR.w = fmaf(gv, d4.w, dR.w);
        v[i] = dg * fmaf(-t3, t3, 1.0f);
      } else {
        v[i] = 0.f;
      }
    }
    uint32_t pk[16];
#pragma unroll
    for (int q = 0; q < 8; ++q) umma::split_pair(v[2 * q], v[2 * q + 1], pk[q], pk[8 + q]);
    umma::st16(taddr + H * 64 + c * 16, pk);
  }
  umma::wait_st();
}

// dh2 total = MMA + layer-3 residual gradient; dz2' = dh2 (1 - t2^2) / c;
// racc1 collects the layer-2 residual gradient into layer 1.
template <int D1, int D2, int D3, int H>
__device__ __forceinline__ void bwd_epi_dh2(uint32_t taddr, const T2Slots& t2, const float (&racc)[32],
                                            float (&racc1)[16], float (&zz)[32]) {
  using P = Split<D1, D2, D3>;
  float v[32];
  umma::ld16(taddr + H * 32, v);
  umma::ld16(taddr + H * 32 + 16, v + 16);
  umma::wait_ld();
#pragma unroll
  for (int j = 0; j < 16; ++j) racc1[j] = 0.f;
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    if (j < P::c2(H)) {
      const float dh = fmaf(kTanhScale, racc[j], v[j]);
      if constexpr (P::R2 != 0) racc1[P::src2(H, j)] += dh;
      const float tj = t2[j];
      zz[j] = dh * kInvTanhScale * fmaf(-tj, tj, 1.0f);
    } else {
      zz[j] = 0.f;
    }
  }
}

// dE/ds of this half: sum over its layer-1 positions of (dh1 + residual) (1 - t1^2) w1.
template <int D1, int D2, int D3, int H>
__device__ __forceinline__ float bwd_ds(const float* f, uint32_t taddr, const float (&h1p)[16],
                                        const float (&racc1)[16]) {
  using P = Split<D1, D2, D3>;
  float v[16];
  umma::ld16(taddr + H * 16, v);
  umma::wait_ld();
  float ds = 0.f;
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    if (j < P::c1(H)) {
      const float t1 = h1p[j] - 1.0f;
      ds = fmaf((v[j] + racc1[j]) * fmaf(-t1, t1, 1.0f), f[H * 16 + j], ds);
    }
  }
  return ds * kInvTanhScale;
}

template <int D1, int D2, int D3>
__global__ void __launch_bounds__(256 * BwdGroup::NG, 1) k_embed_bwd_tc(BwdArgs a) {
  using S = BwdGroup;
  using B = FwdBlob;
  using P = Split<D1, D2, D3>;
  extern __shared__ __align__(1024) unsigned char smem[];
  __shared__ uint64_t bars[S::NG];
  __shared__ uint32_t tbase;
  __shared__ float4 xdr[S::NG][128];
  __shared__ float xds[S::NG][128];
  const int gtid = threadIdx.x, g = gtid >> 8, t = gtid & 255, hf = t >> 7, e = t & 127;
  const int bid = 1 + g;
  const float* f = reinterpret_cast<const float*>(smem + B::O_F);
  const int* pmap = reinterpret_cast<const int*>(smem + B::O_MAP);
  unsigned char* gbase = smem + B::O_END + g * S::BYTES;
  unsigned char* a1h = gbase + S::O_A1;
  unsigned char* a1l = a1h + S::A1B;
  unsigned char* xh = gbase + S::O_X;
  unsigned char* xl = xh + S::XB;
  float4* dts = reinterpret_cast<float4*>(gbase + S::O_DT);
  const T2Slots t2{reinterpret_cast<float*>(a1h), reinterpret_cast<float*>(gbase + S::O_T2), t};
  uint64_t* bar = &bars[g];
  if ((gtid >> 5) == 0) umma::tmem_alloc(&tbase, 512);
  if (t == 0) {
    umma::mbar_init(bar, 1);
    umma::fence_mbar_init();
  }
  umma::fence_before_sync();
  __syncthreads();
  umma::fence_after_sync();
  const uint32_t tm = tbase + g * S::COLS;
  const uint32_t lane_base = (uint32_t)((e >> 5) * 32) << 16;
  uint32_t phase = 0;
  int loaded = -1;
  const TcLists& L = a.L;
  const int nitems = L.istart[L.nnets];
  const uint64_t dw2h = umma::desc(umma::smem_u32(smem + B::O_W2), 128, B::SBO_W2);
  const uint64_t dw3h = umma::desc(umma::smem_u32(smem + B::O_W3), 128, B::SBO_W3);
  const uint64_t dw3l = umma::desc(umma::smem_u32(smem + B::O_W3 + B::W3B), 128, B::SBO_W3);
  // the same blobs read MN-major: W3 as B of dh2 (N = layer-2 positions, K = layer-3
  // positions), W2 as B of dh1 (N = layer-1 positions, K = layer-2 positions)
  const uint64_t dw3th = umma::desc(umma::smem_u32(smem + B::O_W3), B::SBO_W3, 128);
  const uint64_t dw3tl = umma::desc(umma::smem_u32(smem + B::O_W3 + B::W3B), B::SBO_W3, 128);
  const uint64_t dw2th = umma::desc(umma::smem_u32(smem + B::O_W2), B::SBO_W2, 128);
  const uint64_t dw2tl = umma::desc(umma::smem_u32(smem + B::O_W2 + B::W2B), B::SBO_W2, 128);
  const uint64_t da1h = umma::desc(umma::smem_u32(a1h), 128, S::SBO_A1);
  const uint64_t da1l = umma::desc(umma::smem_u32(a1l), 128, S::SBO_A1);
  const uint64_t dxh = umma::desc(umma::smem_u32(xh), 128, S::SBO_X);
  const uint64_t dxl = umma::desc(umma::smem_u32(xl), 128, S::SBO_X);
  const uint32_t id2w = umma::idesc_bf16(128, 128, false, false);
  const uint32_t id2 = umma::idesc_bf16(128, 64, false, false);
  const uint32_t id3 = umma::idesc_bf16(128, 128, false, false);
  const uint32_t id_h2 = umma::idesc_bf16(128, 64, false, true);
  const uint32_t id_h1 = umma::idesc_bf16(128, 32, false, true);
  bool aborted = false;
  auto sync_mma = [&]() {
    umma::fence_proxy_async();
    umma::fence_before_sync();
    umma::bar_sync(bid, 256);
    umma::fence_after_sync();
  };
  auto wait_mma = [&]() -> bool {
    const bool ok = umma::mbar_wait(bar, phase, kWaitLimit);
    phase ^= 1;
    if (umma::bar_sync_or(bid, 256, !ok)) return false;
    umma::fence_after_sync();
    return true;
  };
  for (int base = blockIdx.x * S::NG; base < nitems; base += gridDim.x * S::NG) {
    const int qr = item_of(L, base).q;
    if (qr != loaded) {
      __syncthreads();
      const uint4* src = reinterpret_cast<const uint4*>(a.nets + (size_t)qr * a.net_bytes + a.fwd_off);
      uint4* dst = reinterpret_cast<uint4*>(smem);
      for (uint32_t i = gtid; i < B::BLOB / 16; i += 256 * S::NG) dst[i] = src[i];
      loaded = qr;
      __syncthreads();
    }
    if (aborted) continue;  // keep taking part in the CTA-wide barriers above
    const Item I = item_of(L, base + g);
    if (I.e1 <= I.e0) continue;  // uniform over the group
    // dT of the item's rows in position order, [row][position] float4 over k, scaled by 1/c
    for (int idx = t; idx < kItemRows * 128; idx += 256) {
      const int r = idx >> 7, p = idx & 127, fa = pmap[p], row = I.rb + r;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (fa >= 0 && row < I.re) {
        const float* src = a.dT + (size_t)row * 4 * D3 + fa;
        v = make_float4(src[0] * kInvTanhScale, src[D3] * kInvTanhScale, src[2 * D3] * kInvTanhScale,
                        src[3 * D3] * kInvTanhScale);
      }
      dts[idx] = v;
    }
    umma::bar_sync(bid, 256);
    for (int sub = I.e0; sub < I.e1; sub += 128) {
      const int ne = min(128, I.e1 - sub);
      const bool valid = e < ne;
      const float4 rt = valid ? L.rt[sub + e] : make_float4(0.f, 0.f, 0.f, 0.f);
      const int rloc = valid ? L.row[sub + e] - I.rb : 0;
      float h1[16], h1p[16], h2[32];
      if (hf == 0)
        fwd_layer1<D1, D2, D3, 0>(f, rt.x, h1, h1p);
      else
        fwd_layer1<D1, D2, D3, 1>(f, rt.x, h1, h1p);
#pragma unroll
      for (int kk = 0; kk < 2; ++kk) {
        const uint32_t o = (e >> 3) * S::SBO_A1 + (2 * hf + kk) * 128 + (e & 7) * 16;
        store8_split(a1h + o, a1l + o, h1 + 8 * kk);
      }
      sync_mma();
      if (t == 0) {
        mma_l2(tm + S::C_D2, da1h, da1l, dw2h, id2w, id2);  // columns [0, 128): over the idle layer-3 region
        umma::commit(bar);
      }
      if (!wait_mma()) {
        aborted = true;
        break;
      }
      if (hf == 0)
        bwd_epi2<D1, D2, D3, 0>(f, tm + lane_base + S::C_D2, h1p, h2, t2);
      else
        bwd_epi2<D1, D2, D3, 1>(f, tm + lane_base + S::C_D2, h1p, h2, t2);
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const uint32_t o = (e >> 3) * S::SBO_X + (4 * hf + kk) * 128 + (e & 7) * 16;
        store8_split(xh + o, xl + o, h2 + 8 * kk);
      }
      sync_mma();
      if (t == 0) {
        mma3d(tm + S::C_D3, dxh, dxl, dw3h, dw3l, id3, 4, 256 >> 4, 256 >> 4, false);
        umma::commit(bar);
      }
      if (!wait_mma()) {
        aborted = true;
        break;
      }
      float racc[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) racc[j] = 0.f;
      float4 dR = make_float4(0.f, 0.f, 0.f, 0.f);
      const float4* drow = dts + rloc * 128;
      if (hf == 0)
        bwd_epi3<D1, D2, D3, 0>(f, tm + lane_base + S::C_D3, drow, rt, h1p, t2, racc, dR);
      else
        bwd_epi3<D1, D2, D3, 1>(f, tm + lane_base + S::C_D3, drow, rt, h1p, t2, racc, dR);
      umma::fence_before_sync();
      umma::bar_sync(bid, 256);
      umma::fence_after_sync();
      if (t == 0) {
        // dh2[e][q] = sum_p dz3'[e][p] W3s[q][p]; A = dz3' in TMEM (hi at +16 s, lo at +16 s + 8)
        const uint32_t az = tm + S::C_D3;
#pragma unroll
        for (int s = 0; s < 8; ++s) {
          const uint64_t ob = (uint64_t)(s * ((2 * B::SBO_W3) >> 4));
          mma_ta(tm + S::C_D2, az + 16 * s, dw3th + ob, id_h2, s > 0 ? 1u : 0u);
          mma_ta(tm + S::C_D2, az + 16 * s, dw3tl + ob, id_h2, 1u);
          mma_ta(tm + S::C_D2, az + 16 * s + 8, dw3th + ob, id_h2, 1u);
        }
        umma::commit(bar);
      }
      if (!wait_mma()) {
        aborted = true;
        break;
      }
      // dh2 total -> dz2' into the X slot (the A operand of dh1)
      float racc1[16];
      {
        float zz[32];
        if (hf == 0)
          bwd_epi_dh2<D1, D2, D3, 0>(tm + lane_base + S::C_D2, t2, racc, racc1, zz);
        else
          bwd_epi_dh2<D1, D2, D3, 1>(tm + lane_base + S::C_D2, t2, racc, racc1, zz);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          const uint32_t o = (e >> 3) * S::SBO_X + (4 * hf + kk) * 128 + (e & 7) * 16;
          store8_split(xh + o, xl + o, zz + 8 * kk);
        }
      }
      sync_mma();
      if (t == 0) {
        // dh1[e][l] = sum_q dz2'[e][q] W2s[l][q]
        mma3d(tm + S::C_DH1, dxh, dxl, dw2th, dw2tl, id_h1, 4, 256 >> 4, (2 * B::SBO_W2) >> 4, false);
        umma::commit(bar);
      }
      if (!wait_mma()) {
        aborted = true;
        break;
      }
      const float ds = hf == 0 ? bwd_ds<D1, D2, D3, 0>(f, tm + lane_base + S::C_DH1, h1p, racc1)
                               : bwd_ds<D1, D2, D3, 1>(f, tm + lane_base + S::C_DH1, h1p, racc1);
      if (hf == 1) {
        xdr[g][e] = dR;
        xds[g][e] = ds;
      }
      umma::fence_before_sync();
      umma::bar_sync(bid, 256);
      umma::fence_after_sync();
      if (hf == 0 && valid) {
        // the environment-row gradient in fp64; the chain rule to r_ij runs in the assembly
        const float4 o4 = xdr[g][e];
        const double dR0 = kTanhScale * ((double)dR.x + o4.x), dR1 = kTanhScale * ((double)dR.y + o4.y);
        const double dR2 = kTanhScale * ((double)dR.z + o4.z), dR3 = kTanhScale * ((double)dR.w + o4.w);
        const double dsum = (double)ds + xds[g][e];
        double2* go = reinterpret_cast<double2*>(a.genv + 4 * (size_t)L.slot[sub + e]);
        go[0] = make_double2(dR0 + dsum, dR1);
        go[1] = make_double2(dR2, dR3);
      }
    }
    if (aborted) continue;
    umma::bar_sync(bid, 256);  // every reader of dts is done before the next item restages it
  }
  if (aborted && t == 0) atomicAdd(a.err + kErrTcTimeout, 1);
  umma::fence_before_sync();
  __syncthreads();
  if ((gtid >> 5) == 0) umma::tmem_dealloc(tbase, 512);
}

// dT[row][k][a] = (sum_b dD[a][b] T[k][b] + [a < M2] sum_c dD[c][a] T[k][c]) / N
// dD rows are staged with a stride of M2 + 1 floats so that threads over a
// read distinct banks.
template <int D3>
__global__ void __launch_bounds__(128) k_dT(int nloc, int ntypes, int M2, float inv_nnei,
                                            const int* __restrict__ type_start, const int* __restrict__ perm_atom,
                                            const float* __restrict__ T, const float* __restrict__ dD,
                                            float* __restrict__ dT) {
  extern __shared__ float sm[];
  float* sT = sm;            // 4 * D3
  float* sdD = sm + 4 * D3;  // D3 rows of (M2 + 1)
  const int r = blockIdx.x;
  if (r >= type_start[ntypes]) return;
  const int atom = perm_atom[r];
  const int ld = M2 + 1;
  for (int i = threadIdx.x; i < 4 * D3; i += blockDim.x) sT[i] = T[(size_t)atom * 4 * D3 + i];
  const float* src = dD + (size_t)r * D3 * M2;
  for (int i = threadIdx.x; i < D3 * M2; i += blockDim.x) {
    const int aa = i / M2, b = i - aa * M2;
    sdD[aa * ld + b] = src[i];
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < 4 * D3; idx += blockDim.x) {
    const int k = idx / D3, aa = idx - k * D3;
    const float* tk = sT + k * D3;
    float acc = 0.f;
    for (int b = 0; b < M2; ++b) acc += sdD[aa * ld + b] * tk[b];
    if (aa < M2)
      for (int c = 0; c < D3; ++c) acc += sdD[c * ld + aa] * tk[c];
    dT[(size_t)r * 4 * D3 + idx] = acc * inv_nnei;
  }
}

// T_i = sum over nets (fixed order) / N; D = T^T T_< written as fp32 rows and,
// when requested, pre-tiled bf16 hi/lo for the fitting GEMMs.  A block takes
// kCombRows consecutive rows: in the tiled layout the same 8-column group of 8
// consecutive rows of a tile is one contiguous 128-byte line, so consecutive
// threads take consecutive rows and every line is written whole.
constexpr int kCombRows = 8;

template <int D3>
__global__ void __launch_bounds__(256) k_t_combine(TcLists L, int M2, float inv_nnei, const int* __restrict__ perm_atom,
                                                    const int* __restrict__ ftile, const float* __restrict__ Tq,
                                                    float* __restrict__ T, float* __restrict__ D,
                                                    unsigned char* __restrict__ Dt_hi,
                                                    unsigned char* __restrict__ Dt_lo, int tiled) {
  __shared__ float sT[kCombRows][4 * D3 + 1];  // odd row stride: the 8 rows of a warp read distinct banks
  __shared__ int s_type[kCombRows];
  const int nrows = L.type_start[L.ntypes];
  const int r0 = blockIdx.x * kCombRows;
  if (r0 >= nrows) return;
  const int tid = threadIdx.x;
  if (tid < kCombRows) {
    int t = 0;
    const int r = min(r0 + tid, nrows - 1);
    while (t + 1 < L.ntypes && L.type_start[t + 1] <= r) ++t;
    s_type[tid] = t;
  }
  __syncthreads();
  for (int idx = tid; idx < kCombRows * D3; idx += blockDim.x) {
    const int rr = idx / D3, c = idx - rr * D3, r = r0 + rr;
    if (r >= nrows) continue;
    const int t = s_type[rr];
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    const int q0 = L.type_one_side ? 0 : t * L.ntypes;
    const int q1 = L.type_one_side ? L.nnets : q0 + L.ntypes;
    for (int q = q0; q < q1; ++q) {
      const float* src = Tq + (((size_t)q * L.nloc + r) * 4) * D3;
#pragma unroll
      for (int k = 0; k < 4; ++k) acc[k] += src[k * D3 + c];
    }
    const int atom = perm_atom[r];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float v = acc[k] * inv_nnei;
      sT[rr][k * D3 + c] = v;
      if (!tiled) T[(size_t)atom * 4 * D3 + k * D3 + c] = v;
    }
  }
  __syncthreads();
  if (tiled) {
    // for the tensor-core fitting, T in its 128-row tiles, [tile][k][c][row in tile]: the
    // final fitting backward (one thread per row) then reads it coalesced
    for (int idx = tid; idx < kCombRows * 4 * D3; idx += blockDim.x) {
      const int rr = idx % kCombRows, kc = idx / kCombRows, r = r0 + rr;
      if (r >= nrows) continue;
      const int t = s_type[rr];
      const int prow = 128 * ftile[t] + (r - L.type_start[t]);
      T[((size_t)(prow >> 7) * 4 * D3 + kc) * 128 + (prow & 127)] = sT[rr][kc];
    }
  }
  const int dim = D3 * M2;
  for (int idx = tid; (D || Dt_hi) && idx < kCombRows * (dim / 8); idx += blockDim.x) {
    const int rr = idx % kCombRows, g = idx / kCombRows, r = r0 + rr;
    if (r >= nrows) continue;
    const float* st = sT[rr];
    const int k0 = g * 8;
    float v[8];
    // descriptor column k = aa M2 + b: one division per group of 8, then a carry
    int aa = k0 / M2, b = k0 - aa * M2;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      v[j] = st[aa] * st[b] + st[D3 + aa] * st[D3 + b] + st[2 * D3 + aa] * st[2 * D3 + b] +
             st[3 * D3 + aa] * st[3 * D3 + b];
      if (++b == M2) {
        b = 0;
        ++aa;
      }
    }
    if (D) {
      float4* drow = reinterpret_cast<float4*>(D + (size_t)r * dim + k0);
      drow[0] = make_float4(v[0], v[1], v[2], v[3]);
      drow[1] = make_float4(v[4], v[5], v[6], v[7]);
    }
    if (Dt_hi) {
      const int t = s_type[rr];
      const int prow = 128 * ftile[t] + (r - L.type_start[t]);
      const size_t o = umma::tiled_off(prow, k0, dim);
      store8_split(Dt_hi + o, Dt_lo + o, v);
    }
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

__global__ void k_item_records(TcLists L, int cap, int4* __restrict__ items) {
  const int n = min(L.istart[L.nnets], cap);
  for (int it = blockIdx.x * blockDim.x + threadIdx.x; it < n; it += gridDim.x * blockDim.x) {
    const Item I = item_compute(L, it);
    items[2 * it] = make_int4(I.q, I.rb, I.re, I.e0);
    items[2 * it + 1] = make_int4(I.e1, 0, 0, 0);
  }
}

template <int D1, int D2, int D3>
void pack_net(const std::vector<HostLayer>& net, std::vector<unsigned char>& out) {
  out.assign(NetBlob<D1, D2, D3>::BYTES, 0);
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
  const HostLayer& L1 = net[0];
  const HostLayer& L2 = net[1];
  const HostLayer& L3 = net[2];
  using FB = FwdBlob;
  const uint32_t fo = NetBlob<D1, D2, D3>::OFF_FWD;
  std::vector<int> p1, p2, p3;
  split_order<D1, D2, D3>(p1, p2, p3);
  auto putf = [&](uint32_t base, uint32_t half, int rows, int K, auto val) {
    for (int r = 0; r < rows; ++r)
      for (int k = 0; k < K; ++k) {
        const float x = val(r, k);
        const uint16_t hi = to_bf16(x);
        const uint16_t lo = to_bf16(x - from_bf16(hi));
        const uint32_t o = (uint32_t)(r >> 3) * ((K / 8) * 128) + (uint32_t)(k >> 3) * 128 + (r & 7) * 16 + (k & 7) * 2;
        std::memcpy(&out[fo + base + o], &hi, 2);
        std::memcpy(&out[fo + base + half + o], &lo, 2);
      }
  };
  // weights and biases scaled by 2 log2(e) (the kernel's tanh takes scaled
  // pre-activations); folded biases sit in the weight row of the constant slot
  using P = Split<D1, D2, D3>;
  const double c = 2.0 / std::log(2.0);
  const int one1 = P::FOLD2 ? P::c1(0) : -1, one2 = P::FOLD3 ? P::c2(0) : -1;
  putf(FB::O_W2, FB::W2B, 64, 32, [&](int n, int k) {
    if (p2[n] < 0) return 0.f;
    if (k == one1) return (float)(c * L2.b[p2[n]]);
    return p1[k] >= 0 ? (float)(c * L2.w[(size_t)p1[k] * D2 + p2[n]]) : 0.f;
  });
  putf(FB::O_W3, FB::W3B, 128, 64, [&](int n, int k) {
    if (p3[n] < 0) return 0.f;
    if (k == one2) return (float)(c * L3.b[p3[n]]);
    return p2[k] >= 0 ? (float)(c * L3.w[(size_t)p2[k] * D3 + p3[n]]) : 0.f;
  });
  float* ff = reinterpret_cast<float*>(&out[fo + FB::O_F]);
  for (int j = 0; j < 32; ++j) ff[j] = p1[j] >= 0 ? (float)(c * L1.w[p1[j]]) : 0.f;
  for (int j = 0; j < 32; ++j) ff[32 + j] = p1[j] >= 0 ? (float)(c * L1.b[p1[j]]) : 0.f;
  for (int j = 0; j < 64; ++j) ff[64 + j] = p2[j] >= 0 ? (float)(c * L2.b[p2[j]]) : 0.f;
  for (int j = 0; j < 128; ++j) ff[128 + j] = p3[j] >= 0 ? (float)(c * L3.b[p3[j]]) : 0.f;
  int* map = reinterpret_cast<int*>(&out[fo + FB::O_MAP]);
  for (int j = 0; j < 128; ++j) map[j] = p3[j];
}

enum class Inst { None, W25, W32 };
Inst which(const SeaDev& s) {
  if (s.nl != 3) return Inst::None;
  if (s.ed[1] == 25 && s.ed[2] == 50 && s.ed[3] == 100) return Inst::W25;
  if (s.ed[1] == 32 && s.ed[2] == 64 && s.ed[3] == 128) return Inst::W32;
  return Inst::None;
}

template <int D1, int D2, int D3>
void launch_fwd(cudaStream_t st, const TcLists& L, int grid, const unsigned char* nets, float* Tq, int* err) {
  using S = FwdGroup;
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(k_embed_fwd_tc<D1, D2, D3>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)S::SMEM);
    attr = true;
  }
  FwdArgs a{L, nets, NetBlob<D1, D2, D3>::BYTES, NetBlob<D1, D2, D3>::OFF_FWD, Tq, err};
  count_launch();
  k_embed_fwd_tc<D1, D2, D3><<<grid, 256 * S::NG, S::SMEM, st>>>(a);
}

template <int D1, int D2, int D3>
void launch_bwd(cudaStream_t st, const TcLists& L, int grid, const unsigned char* nets, const float* dT,
                double* genv, int* err) {
  using S = BwdGroup;
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(k_embed_bwd_tc<D1, D2, D3>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)S::SMEM);
    attr = true;
  }
  BwdArgs a{L, nets, NetBlob<D1, D2, D3>::BYTES, NetBlob<D1, D2, D3>::OFF_FWD, dT, genv, err};
  count_launch();
  k_embed_bwd_tc<D1, D2, D3><<<grid, 256 * S::NG, S::SMEM, st>>>(a);
}

}  // namespace

bool tc_supported(const SeaDev& s) { return which(s) != Inst::None; }

size_t tc_net_bytes(const SeaDev& s) {
  switch (which(s)) {
    case Inst::W25:
      return NetBlob<25, 50, 100>::BYTES;
    case Inst::W32:
      return NetBlob<32, 64, 128>::BYTES;
    default:
      return 0;
  }
}

void tc_pack_net(const SeaDev& s, const std::vector<HostLayer>& net, std::vector<unsigned char>& out) {
  if (which(s) == Inst::W25) pack_net<25, 50, 100>(net, out);
  if (which(s) == Inst::W32) pack_net<32, 64, 128>(net, out);
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

int tc_item_capacity(const SeaDev& s, int nloc) {
  return s.nnets * ((nloc + kItemRows - 1) / kItemRows + kFwdGroups) + kFwdGroups;
}

void launch_item_records(cudaStream_t st, const SeaDev& s, const TcLists& L, int4* items) {
  const int cap = tc_item_capacity(s, L.nloc);
  count_launch();
  k_item_records<<<std::max(1, std::min(148 * 4, (cap + 255) / 256)), 256, 0, st>>>(L, cap, items);
}

int embed_tc_grid(const SeaDev&, bool backward) {
  int dev = 0, nsm = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
  // one CTA per SM: the forward runs kFwdGroups groups of 8 warps in it, the backward one group of 4
  return nsm;
}

void launch_embed_fwd_tc(cudaStream_t st, const SeaDev& s, const TcLists& L, int grid, const unsigned char* nets,
                         float* Tq, int* err) {
  if (which(s) == Inst::W25) launch_fwd<25, 50, 100>(st, L, grid, nets, Tq, err);
  if (which(s) == Inst::W32) launch_fwd<32, 64, 128>(st, L, grid, nets, Tq, err);
}

void launch_embed_bwd_tc(cudaStream_t st, const SeaDev& s, const TcLists& L, int grid, const unsigned char* nets,
                         const float* dT, double* genv, int* err) {
  if (which(s) == Inst::W25) launch_bwd<25, 50, 100>(st, L, grid, nets, dT, genv, err);
  if (which(s) == Inst::W32) launch_bwd<32, 64, 128>(st, L, grid, nets, dT, genv, err);
}

void launch_dT(cudaStream_t st, const SeaDev& s, int nloc, const int* type_start, const int* perm_atom, const float* T,
               const float* dD, float* dT) {
  if (nloc <= 0) return;
  const size_t smem = sizeof(float) * (4 + s.M2 + 1) * s.M1;
  count_launch();
  if (which(s) == Inst::W25)
    k_dT<100><<<nloc, 128, smem, st>>>(nloc, s.ntypes, s.M2, (float)s.inv_nnei, type_start, perm_atom, T, dD, dT);
  else
    k_dT<128><<<nloc, 128, smem, st>>>(nloc, s.ntypes, s.M2, (float)s.inv_nnei, type_start, perm_atom, T, dD, dT);
}

void launch_t_combine(cudaStream_t st, const SeaDev& s, const TcLists& L, const int* perm_atom, const int* ftile,
                      const float* Tq, float* T, float* D, unsigned char* Dt_hi, unsigned char* Dt_lo, bool tiled) {
  if (L.nloc <= 0) return;
  count_launch();
  if (which(s) == Inst::W25)
    k_t_combine<100><<<(L.nloc + kCombRows - 1) / kCombRows, 256, 0, st>>>(L, s.M2, (float)s.inv_nnei, perm_atom,
                                                                            ftile, Tq, T, D, Dt_hi, Dt_lo, tiled);
  else
    k_t_combine<128><<<(L.nloc + kCombRows - 1) / kCombRows, 256, 0, st>>>(L, s.M2, (float)s.inv_nnei, perm_atom,
                                                                            ftile, Tq, T, D, Dt_hi, Dt_lo, tiled);
}

}  // namespace b200dp
