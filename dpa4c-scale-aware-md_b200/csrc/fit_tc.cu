// Tensor-core fitting net (see fit_tc.cuh).
#include <algorithm>
#include <cstring>
#include <functional>

#include "common.cuh"
#include "fit_tc.cuh"
#include "umma.cuh"

namespace b200dp {

namespace {

constexpr int kMaxStages = 8;
constexpr uint32_t kTSlice = 8 * 512;  // T of one layer-0 K chunk: 4 components x 2 a values x 128 rows
constexpr uint32_t kABlock = 128 * kFitBK * 2;  // one half of a 128 x 32 activation block (8 KB)
constexpr uint32_t kSbo = (kFitBK / 8) * 128;    // K-major SBO inside a block (512 B)
constexpr long long kWaitLimit = 1LL << 26;


using umma::tiled_off;

// fp32 activations of the fitting (tanh outputs, layer outputs, residual
// gradients) are stored per 128-row tile column by column, so the epilogue
// threads (one per row) read and write consecutive addresses.
__device__ __forceinline__ size_t colmajor_off(int prow, int col, int ncols) {
  return ((size_t)(prow >> 7) * ncols + col) * 128 + (prow & 127);
}

__device__ __forceinline__ void store8_split(unsigned char* hi, unsigned char* lo, const float* v) {
  uint32_t h[4], l[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) umma::split_pair(v[2 * j], v[2 * j + 1], h[j], l[j]);
  *reinterpret_cast<uint4*>(hi) = make_uint4(h[0], h[1], h[2], h[3]);
  *reinterpret_cast<uint4*>(lo) = make_uint4(l[0], l[1], l[2], l[3]);
}

enum Mode : int { kFwd = 0, kBwd = 1 };

struct GemmArgs {
  int ntypes;
  const int* type_start;
  const int* ftile;
  int nk;  // K chunks of 32
  const unsigned char* A_hi;
  const unsigned char* A_lo;
  // layer 0 with A formed in the kernel: the descriptor D = T^T T_< from T in the
  // fitting's row tiles ([tile][4][M1][128], already divided by N), axis 16
  const float* Tt;
  int M1;
  const unsigned char* B_hi[kMaxTypes];
  const unsigned char* B_lo[kMaxTypes];
  int BN, N;
  int mode;
  int stages;  // K-chunk pipeline depth
  // forward
  const float* bias[kMaxTypes];
  const float* Yprev;
  int ldprev;
  float* TH;
  float* Y;
  unsigned char* Anext_hi;
  unsigned char* Anext_lo;
  int kpad_next;
  int last;
  const float* wo[kMaxTypes];
  double bo[kMaxTypes];
  const int* perm_atom;
  double* atom_e;
  unsigned char* Z_hi;
  unsigned char* Z_lo;
  int kpad_z;
  // backward
  const float* DYnext;
  int dy_is_wo;
  float* DYout;
  const float* THprev;
  int* err;
};

// Warps 0-7 run the epilogue (2 warps per TMEM lane quadrant share a tile's
// columns); warp 8 streams the K chunks of A and B into a ring of
// shared-memory stages, warp 9 issues the MMAs, so loads, MMAs and their
// bookkeeping proceed independently.  Ring indices advance by increments
// (no runtime division in the issue loops).  320 threads at <= 102 registers
// and a 4-stage ring let two CTAs share an SM, so a layer's 3 x 98 tiles run
// as one wave.
constexpr int kFitEpiThreads = 256;
constexpr int kFitThreads = kFitEpiThreads + 64;

__global__ void __launch_bounds__(kFitThreads, 2) k_fit_gemm(GemmArgs a) {
  extern __shared__ __align__(1024) unsigned char smem[];
  __shared__ uint64_t full[kMaxStages], empty[kMaxStages], tfull[kMaxStages], done;
  __shared__ uint32_t tbase;
  __shared__ int s_ok;
  __shared__ double s_e[kFitEpiThreads / 128][128];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = blockIdx.x, nt = blockIdx.y;
  if (g >= a.ftile[a.ntypes]) return;  // CTA-uniform, before any TMEM allocation
  int t = 0;
  while (t + 1 < a.ntypes && a.ftile[t + 1] <= g) ++t;
  const int row0 = a.type_start[t] + 128 * (g - a.ftile[t]);
  const int nrows = min(128, a.type_start[t + 1] - row0);
  const uint32_t BB = (uint32_t)a.BN * kFitBK * 2;
  // a stage: A (hi, lo), B (hi, lo) and, when A is formed here, the chunk's slice of T
  const uint32_t SB = 2 * kABlock + 2 * BB + (a.Tt ? kTSlice : 0u);
  if (warp == 0) umma::tmem_alloc(&tbase, 256);
  const int S = a.stages;
  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      // the loader's arrival (with the bulk bytes), plus every epilogue thread's when it forms A
      umma::mbar_init(&full[s], a.Tt ? 1 + kFitEpiThreads : 1);
      umma::mbar_init(&empty[s], 1);
      umma::mbar_init(&tfull[s], 1);
    }
    umma::mbar_init(&done, 1);
    umma::fence_mbar_init();
    s_ok = 1;
  }
  umma::fence_before_sync();
  __syncthreads();
  umma::fence_after_sync();
  const uint32_t tm = tbase;
  if (warp == kFitEpiThreads / 32 && lane == 0) {  // loader
    const unsigned char* Ah = a.A_hi + (size_t)g * a.nk * kABlock;
    const unsigned char* Al = a.A_lo + (size_t)g * a.nk * kABlock;
    const unsigned char* Bh = a.B_hi[t] + (size_t)nt * a.nk * BB;
    const unsigned char* Bl = a.B_lo[t] + (size_t)nt * a.nk * BB;
    int s = 0, round = 0;
    for (int kc = 0; kc < a.nk; ++kc) {
      if (round > 0 && !umma::mbar_wait(&empty[s], (round - 1) & 1, kWaitLimit)) {
        s_ok = 0;
        break;
      }
      unsigned char* st = smem + s * SB;
      if (a.Tt) {  // T[tile][k][a][128 rows] for the chunk's two a values: 8 rows of 512 bytes
        umma::mbar_expect_tx(&tfull[s], kTSlice);
        const float* tsrc = a.Tt + (size_t)g * 4 * a.M1 * 128;
        for (int k = 0; k < 4; ++k)
          for (int q = 0; q < 2; ++q)
            umma::bulk_g2s(st + 2 * kABlock + 2 * BB + (2 * k + q) * 512,
                           tsrc + ((size_t)k * a.M1 + 2 * kc + q) * 128, 512, &tfull[s]);
      }
      umma::mbar_expect_tx(&full[s], a.Tt ? 2 * BB : SB);
      if (!a.Tt) {
        umma::bulk_g2s(st, Ah + (size_t)kc * kABlock, kABlock, &full[s]);
        umma::bulk_g2s(st + kABlock, Al + (size_t)kc * kABlock, kABlock, &full[s]);
      }
      umma::bulk_g2s(st + 2 * kABlock, Bh + (size_t)kc * BB, BB, &full[s]);
      umma::bulk_g2s(st + 2 * kABlock + BB, Bl + (size_t)kc * BB, BB, &full[s]);
      if (++s == S) {
        s = 0;
        ++round;
      }
    }
  } else if (warp == kFitEpiThreads / 32 + 1 && lane == 0) {  // MMA issuer
    const uint32_t idesc = umma::idesc_bf16(128, a.BN, false, false);
    const uint64_t d0 = umma::desc(umma::smem_u32(smem), 128, kSbo);
    const uint64_t sstep = SB >> 4, o_al = kABlock >> 4, o_bh = (2 * kABlock) >> 4, o_bl = (2 * kABlock + BB) >> 4;
    int s = 0, round = 0;
    bool ok = true;
    for (int kc = 0; kc < a.nk; ++kc) {
      ok = umma::mbar_wait(&full[s], round & 1, kWaitLimit);
      if (!ok) break;
      umma::fence_after_sync();
      const uint64_t ah = d0 + (uint64_t)s * sstep;
#pragma unroll
      for (int ks = 0; ks < kFitBK / 16; ++ks) {
        const uint64_t o = (uint64_t)(ks * (256 >> 4));
        umma::mma(tm, ah + o, ah + o_bh + o, idesc, (kc | ks) ? 1u : 0u);
        umma::mma(tm, ah + o, ah + o_bl + o, idesc, 1u);
        umma::mma(tm, ah + o_al + o, ah + o_bh + o, idesc, 1u);
      }
      umma::commit(&empty[s]);
      if (++s == S) {
        s = 0;
        ++round;
      }
    }
    umma::commit(&done);
    if (!ok) s_ok = 0;
  }
  if (a.Tt && warp < kFitEpiThreads / 32) {
    // producers of A: row r, descriptor columns a*16 + b of the chunk's two a
    // values, b in [8 h, 8 h + 8): D[r][a][b] = sum_k T[r][k][a] T[r][k][b],
    // written as bf16 hi / lo into the stage's A block (zero rows past the tile)
    const int r = tid & 127, h = tid >> 7;
    const bool rv = r < nrows;
    const float* Tg = a.Tt + (size_t)g * 4 * a.M1 * 128 + r;  // element (k, c) at Tg[(k M1 + c) 128]
    float tb[4][8];
#pragma unroll
    for (int k = 0; k < 4; ++k)
#pragma unroll
      for (int j = 0; j < 8; ++j) tb[k][j] = rv ? Tg[((size_t)k * a.M1 + 8 * h + j) * 128] : 0.f;
    const uint32_t o0 = (uint32_t)(r >> 3) * kSbo + (uint32_t)h * 128 + (uint32_t)(r & 7) * 16;
    const uint32_t o1 = o0 + 2 * 128;
    int s = 0, round = 0;
    for (int kc = 0; kc < a.nk; ++kc) {
      // the stage is free once its slice of T has landed (the loader waited for it)
      if (!umma::mbar_wait(&tfull[s], round & 1, kWaitLimit)) {
        s_ok = 0;
        break;
      }
      unsigned char* st = smem + s * SB;
      const float* ts = reinterpret_cast<const float*>(st + 2 * kABlock + 2 * BB) + r;
      float ta[4][2];
#pragma unroll
      for (int k = 0; k < 4; ++k)
#pragma unroll
        for (int q = 0; q < 2; ++q) ta[k][q] = rv ? ts[(2 * k + q) * 128] : 0.f;
      float v[2][8];
#pragma unroll
      for (int q = 0; q < 2; ++q)
#pragma unroll
        for (int j = 0; j < 8; ++j)
          v[q][j] = ta[0][q] * tb[0][j] + ta[1][q] * tb[1][j] + ta[2][q] * tb[2][j] + ta[3][q] * tb[3][j];
      store8_split(st + o0, st + kABlock + o0, v[0]);
      store8_split(st + o1, st + kABlock + o1, v[1]);
      umma::fence_proxy_async();
      umma::mbar_arrive(&full[s]);
      if (++s == S) {
        s = 0;
        ++round;
      }
    }
  }
  const bool ok = umma::mbar_wait(&done, 0, kWaitLimit);
  const int q = warp & 3, part = warp >> 2;  // lane quadrant, column part
  const int r = q * 32 + lane;               // row within the tile (TMEM lane)
  const bool valid = r < nrows;
  const int prow = g * 128 + r;  // padded row
  const int urow = row0 + r;     // row in type-grouped order
  const int nparts = warp < kFitEpiThreads / 32 ? kFitEpiThreads / 128 : 0;
  if (__syncthreads_or(!ok || !s_ok)) {
    if (tid == 0) atomicAdd(a.err + 3, 1);
  } else {
    umma::fence_after_sync();
    const uint32_t lb = (uint32_t)(q * 32) << 16;
    double e_acc = 0.0;
    for (int c = part; nparts && c < a.BN / 16; c += nparts) {
      float v[16];
      umma::ld16(tm + lb + c * 16, v);
      umma::wait_ld();
      if (!valid) continue;
      const int col0 = nt * a.BN + c * 16;
      // every global operand of the chunk is loaded before any store: the
      // stores below may alias them in the compiler's view, and loads issued
      // behind them would each wait a full L2 round trip
      if (a.mode == kFwd) {
        float y[16], zs[16], bb[16], yp[16], wo[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          bb[j] = __ldg(a.bias[t] + col0 + j);
          yp[j] = a.Yprev ? a.Yprev[colmajor_off(prow, col0 + j, a.ldprev)] : 0.f;
          wo[j] = a.last ? __ldg(a.wo[t] + col0 + j) : 0.f;
        }
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int col = col0 + j;
          const float th = umma::tanh_fast(v[j] + bb[j]);
          float yy = th;
          if (a.Yprev) yy += yp[j];
          a.TH[colmajor_off(prow, col, a.N)] = th;
          a.Y[colmajor_off(prow, col, a.N)] = yy;
          y[j] = yy;
          if (a.last) {
            e_acc += (double)(yy * wo[j]);
            zs[j] = wo[j] * (1.f - th * th);
          }
        }
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int k = col0 + 8 * h;
          if (a.last) {
            const size_t o = tiled_off(prow, k, a.kpad_z);
            store8_split(a.Z_hi + o, a.Z_lo + o, zs + 8 * h);
          } else {
            const size_t o = tiled_off(prow, k, a.kpad_next);
            store8_split(a.Anext_hi + o, a.Anext_lo + o, y + 8 * h);
          }
        }
      } else {
        float z[16], dn[16], thp[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int col = col0 + j;
          dn[j] = a.dy_is_wo ? __ldg(a.wo[t] + col) : (a.DYnext ? a.DYnext[colmajor_off(prow, col, a.N)] : 0.f);
          thp[j] = a.THprev[colmajor_off(prow, col, a.N)];
        }
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int col = col0 + j;
          const float d = v[j] + dn[j];
          if (a.DYout) a.DYout[colmajor_off(prow, col, a.N)] = d;
          z[j] = d * (1.f - thp[j] * thp[j]);
        }
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const size_t o = tiled_off(prow, col0 + 8 * h, a.kpad_z);
          store8_split(a.Z_hi + o, a.Z_lo + o, z + 8 * h);
        }
      }
    }
    if (a.mode == kFwd && a.last) {  // partial energies of the column parts, summed in a fixed order
      if (nparts) s_e[part][r] = e_acc;
      __syncthreads();
      if (nparts && part == 0 && valid) {
        double e = a.bo[t];
        for (int p2 = 0; p2 < kFitEpiThreads / 128; ++p2) e += s_e[p2][r];
        a.atom_e[a.perm_atom[urow]] = e;
      }
    }
  }
  umma::fence_before_sync();
  __syncthreads();
  if (warp == 0) umma::tmem_dealloc(tm, 256);
}

// ------------------------------------------------------------ hidden chain
// Layers 1 .. L-1 forward and then backward (down to dz0) for one 128-row
// tile per CTA, in one launch.  The tile's activation operand (at most 256
// columns, bf16 hi and lo, 128 KB) stays in shared memory from layer to layer:
// each epilogue writes the next GEMM's A operand in place, after the GEMM that
// read it has completed.  The weights of all steps stream through one ring of
// shared-memory stages (warp 16), so the next step's first K chunks arrive
// while the current epilogue runs; warp 17 issues the MMAs (N = the layer's
// whole width).  TMEM: the accumulator in columns [0, 256), and in [256, 512)
// the fp32 value a later epilogue of the same thread adds as a residual
// (layer output y_l in the forward, dE/dy_l in the backward).  The tanh
// outputs that the backward needs stay in global memory (L2-resident).
// Every step keeps the arithmetic of the per-layer kernel above (k_fit_gemm),
// column by column; the energy adds the partial sums of four column parts.
constexpr int kChainK = 256;  // widest activation operand (columns)
constexpr int kChainEpiWarps = 16;
constexpr int kChainThreads = kChainEpiWarps * 32 + 64;
constexpr uint32_t kChainAct = 2 * (kChainK / kFitBK) * kABlock;  // hi region, then lo region
constexpr size_t kChainSmemMax = 227 * 1024 - 8192;  // dynamic shared memory budget of k_fit_chain

struct ChainArgs {
  int ntypes;
  const int* type_start;
  const int* ftile;
  int L;
  int width[kFitMaxLayers], kpad[kFitMaxLayers], res[kFitMaxLayers];
  int bnf[kFitMaxLayers], bnb[kFitMaxLayers];
  const unsigned char* A_hi;  // tiled input of layer 1 (y0)
  const unsigned char* A_lo;
  const unsigned char* fB_hi[kMaxTypes][kFitMaxLayers];
  const unsigned char* fB_lo[kMaxTypes][kFitMaxLayers];
  const unsigned char* bB_hi[kMaxTypes][kFitMaxLayers];
  const unsigned char* bB_lo[kMaxTypes][kFitMaxLayers];
  const float* bias[kMaxTypes][kFitMaxLayers];
  const float* wo[kMaxTypes];
  double bo[kMaxTypes];
  const float* Y0;                  // layer-0 output (residual of layer 1)
  float* TH[kFitMaxLayers];         // tanh outputs (TH[0] written by the layer-0 launch)
  const int* perm_atom;
  double* atom_e;
  unsigned char* Z_hi;  // dz0, tiled (kpad_z columns), the final backward's A operand
  unsigned char* Z_lo;
  int kpad_z;
  int stages;
  int* err;
};

// GEMM step j: forward layer j + 1 for j < L - 1, then backward layers L - 1 .. 1.
struct ChainStep {
  int l, fwd, N, nk, bn;
};
__device__ __forceinline__ ChainStep chain_step(const ChainArgs& a, int j) {
  ChainStep c;
  c.fwd = j < a.L - 1;
  c.l = c.fwd ? j + 1 : 2 * a.L - 2 - j;
  c.N = c.fwd ? a.width[c.l] : a.width[c.l - 1];
  c.nk = c.fwd ? a.kpad[c.l] / kFitBK : (a.width[c.l] + kFitBK - 1) / kFitBK;
  c.bn = c.fwd ? a.bnf[c.l] : a.bnb[c.l];
  return c;
}

__device__ __forceinline__ uint32_t act_off(int r, int k) {
  return (uint32_t)(k / kFitBK) * kABlock + (uint32_t)(r >> 3) * kSbo + (uint32_t)((k % kFitBK) >> 3) * 128u +
         (uint32_t)(r & 7) * 16u;
}

__global__ void __launch_bounds__(kChainThreads, 1) k_fit_chain(ChainArgs a) {
  extern __shared__ __align__(1024) unsigned char smem[];
  __shared__ uint64_t full[kMaxStages], empty[kMaxStages], a_in, acc_full, act_full;
  __shared__ uint32_t tbase;
  __shared__ int s_fail;
  __shared__ double s_e[kChainEpiWarps / 4][128];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = blockIdx.x;
  if (g >= a.ftile[a.ntypes]) return;  // CTA-uniform, before any TMEM allocation
  int t = 0;
  while (t + 1 < a.ntypes && a.ftile[t + 1] <= g) ++t;
  const int row0 = a.type_start[t] + 128 * (g - a.ftile[t]);
  const int nrows = min(128, a.type_start[t + 1] - row0);
  const int nsteps = 2 * (a.L - 1);
  unsigned char* act = smem;
  unsigned char* ring = smem + kChainAct;
  uint32_t SB = 0;  // ring stage: the widest step's B chunk, hi then lo
  for (int j = 0; j < nsteps; ++j) SB = max(SB, (uint32_t)chain_step(a, j).N * kFitBK * 2 * 2);
  const int S = a.stages;
  if (warp == 0) umma::tmem_alloc(&tbase, 512);
  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      umma::mbar_init(&full[s], 1);
      umma::mbar_init(&empty[s], 1);
    }
    umma::mbar_init(&a_in, 1);
    umma::mbar_init(&acc_full, 1);
    umma::mbar_init(&act_full, kChainEpiWarps * 32);
    umma::fence_mbar_init();
    s_fail = 0;
  }
  umma::fence_before_sync();
  __syncthreads();
  umma::fence_after_sync();
  const int nk1 = a.kpad[1] / kFitBK;
  if (warp == kChainEpiWarps && lane == 0) {  // loader: y0 once, then every step's weights through the ring
    const uint32_t half = (uint32_t)nk1 * kABlock;
    umma::mbar_expect_tx(&a_in, 2 * half);
    umma::bulk_g2s(act, a.A_hi + (size_t)g * half, half, &a_in);
    umma::bulk_g2s(act + kChainAct / 2, a.A_lo + (size_t)g * half, half, &a_in);
    int s = 0, round = 0;
    bool ok = true;
    for (int j = 0; j < nsteps && ok; ++j) {
      const ChainStep c = chain_step(a, j);
      const unsigned char* Bh = c.fwd ? a.fB_hi[t][c.l] : a.bB_hi[t][c.l];
      const unsigned char* Bl = c.fwd ? a.fB_lo[t][c.l] : a.bB_lo[t][c.l];
      const uint32_t blk = (uint32_t)c.bn * kFitBK * 2, nb = (uint32_t)(c.N / c.bn);
      for (int kc = 0; kc < c.nk; ++kc) {
        if (round > 0 && !umma::mbar_wait(&empty[s], (round - 1) & 1, kWaitLimit)) {
          ok = false;
          break;
        }
        unsigned char* st = ring + s * SB;
        umma::mbar_expect_tx(&full[s], 2 * nb * blk);
        // the N blocks of the packed weights (BN rows each) side by side make one N-row operand
        for (uint32_t nt = 0; nt < nb; ++nt) {
          umma::bulk_g2s(st + nt * blk, Bh + ((size_t)nt * c.nk + kc) * blk, blk, &full[s]);
          umma::bulk_g2s(st + nb * blk + nt * blk, Bl + ((size_t)nt * c.nk + kc) * blk, blk, &full[s]);
        }
        if (++s == S) {
          s = 0;
          ++round;
        }
      }
    }
    if (!ok) s_fail = 1;
  } else if (warp == kChainEpiWarps + 1 && lane == 0) {  // MMA issuer
    bool ok = umma::mbar_wait(&a_in, 0, kWaitLimit);
    int s = 0, round = 0;
    for (int j = 0; j < nsteps && ok; ++j) {
      const ChainStep c = chain_step(a, j);
      // the A operand is ready: the zero fill (j = 0) or the previous epilogue
      ok = umma::mbar_wait(&act_full, j & 1, kWaitLimit);
      if (!ok) break;
      umma::fence_after_sync();
      const uint32_t idesc = umma::idesc_bf16(128, c.N, false, false);
      const uint64_t dah = umma::desc(umma::smem_u32(act), 128, kSbo);
      const uint64_t dal = umma::desc(umma::smem_u32(act + kChainAct / 2), 128, kSbo);
      const uint64_t db0 = umma::desc(umma::smem_u32(ring), 128, kSbo);
      const uint64_t o_bl = ((uint64_t)c.N * kFitBK * 2) >> 4, sstep = SB >> 4, kstep = kABlock >> 4;
      for (int kc = 0; kc < c.nk; ++kc) {
        ok = umma::mbar_wait(&full[s], round & 1, kWaitLimit);
        if (!ok) break;
        umma::fence_after_sync();
        const uint64_t ah = dah + (uint64_t)kc * kstep, al = dal + (uint64_t)kc * kstep;
        const uint64_t bh = db0 + (uint64_t)s * sstep, bl = bh + o_bl;
#pragma unroll
        for (int ks = 0; ks < kFitBK / 16; ++ks) {
          const uint64_t o = (uint64_t)(ks * (256 >> 4));
          umma::mma(tbase, ah + o, bh + o, idesc, (kc | ks) ? 1u : 0u);
          umma::mma(tbase, ah + o, bl + o, idesc, 1u);
          umma::mma(tbase, al + o, bh + o, idesc, 1u);
        }
        umma::commit(&empty[s]);
        if (++s == S) {
          s = 0;
          ++round;
        }
      }
      if (ok) umma::commit(&acc_full);
    }
    if (!ok) s_fail = 1;
  } else if (warp < kChainEpiWarps) {  // epilogue
    const int q = warp & 3, part = warp >> 2, nparts = kChainEpiWarps / 4;
    const int r = q * 32 + lane;  // row within the tile (TMEM lane)
    const bool valid = r < nrows;
    const int prow = g * 128 + r;
    const uint32_t lb = (uint32_t)(q * 32) << 16;
    const uint32_t acc = tbase + lb, car = tbase + lb + 256;
    unsigned char* ah = act;
    unsigned char* al = act + kChainAct / 2;
    // the activation chunks that y0 does not fill are zero (K padding of wider layers)
    for (uint32_t i = (uint32_t)nk1 * kABlock / 16 + (tid & 511); i < kChainAct / 32; i += kChainEpiWarps * 32) {
      reinterpret_cast<uint4*>(ah)[i] = make_uint4(0u, 0u, 0u, 0u);
      reinterpret_cast<uint4*>(al)[i] = make_uint4(0u, 0u, 0u, 0u);
    }
    umma::fence_proxy_async();
    umma::fence_before_sync();
    umma::mbar_arrive(&act_full);
    bool ok = true;
    double e_acc = 0.0;
    // the operand a chunk reads from global memory (L2): y0 for the residual of
    // layer 1, the tanh outputs of layer l - 1 in the backward; fetched one chunk
    // ahead, the first chunk of a step while its GEMM runs
    auto fetch = [&](const ChainStep& c, int cc, float* dst) {
      const int col0 = cc * 16;
      if (c.fwd) {
        const bool use = a.res[c.l] && c.l == 1 && valid;
#pragma unroll
        for (int i = 0; i < 16; ++i) dst[i] = use ? a.Y0[colmajor_off(prow, col0 + i, a.width[0])] : 0.f;
      } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) dst[i] = valid ? a.TH[c.l - 1][colmajor_off(prow, col0 + i, c.N)] : 0.f;
      }
    };
    for (int j = 0; j < nsteps; ++j) {
      const ChainStep c = chain_step(a, j);
      const int l = c.l, N = c.N;
      const bool last_fwd = c.fwd && l == a.L - 1;
      float gn[16];
      if (part < N / 16) fetch(c, part, gn);
      if (ok) ok = umma::mbar_wait(&acc_full, j & 1, kWaitLimit);
      ok = __all_sync(0xffffffffu, ok);  // the TMEM loads below are warp-collective
      umma::fence_after_sync();
      for (int cc = part; ok && cc < N / 16; cc += nparts) {
        const int col0 = cc * 16;
        float v[16], x[16], u[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) x[i] = gn[i];
        if (cc + nparts < N / 16) fetch(c, cc + nparts, gn);
        if (c.fwd) {
          // x: residual input (y_{l-1}; layer 1's came with the fetch), u: bias
          const bool res = a.res[l] != 0;
#pragma unroll
          for (int i = 0; i < 16; ++i) u[i] = __ldg(a.bias[t][l] + col0 + i);
          umma::ld16(acc + col0, v);
          if (res && l >= 2) umma::ld16(car + col0, x);
          umma::wait_ld();
          float y[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const float th = umma::tanh_fast(v[i] + u[i]);
            y[i] = res ? th + x[i] : th;
            v[i] = th;
          }
          if (l + 1 < a.L && a.res[l + 1]) umma::st16f(car + col0, y);
          if (valid) {
            if (!last_fwd) {
#pragma unroll
              for (int i = 0; i < 16; ++i) a.TH[l][colmajor_off(prow, col0 + i, N)] = v[i];
#pragma unroll
              for (int h = 0; h < 2; ++h) {
                const uint32_t o = act_off(r, col0 + 8 * h);
                store8_split(ah + o, al + o, y + 8 * h);
              }
            } else {
              float zs[16];
#pragma unroll
              for (int i = 0; i < 16; ++i) {
                const float w = __ldg(a.wo[t] + col0 + i);
                e_acc += (double)(y[i] * w);
                zs[i] = w * (1.f - v[i] * v[i]);
              }
#pragma unroll
              for (int h = 0; h < 2; ++h) {
                const uint32_t o = act_off(r, col0 + 8 * h);
                store8_split(ah + o, al + o, zs + 8 * h);
              }
            }
          }
        } else {
          // x: dE/dy_l (residual of layer l), u: tanh outputs of layer l - 1 (the fetch)
          const bool res = a.res[l] != 0, top = l == a.L - 1;
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            u[i] = x[i];
            x[i] = (res && top) ? __ldg(a.wo[t] + col0 + i) : 0.f;
          }
          umma::ld16(acc + col0, v);
          if (res && !top) umma::ld16(car + col0, x);
          umma::wait_ld();
          float z[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const float d = v[i] + x[i];
            v[i] = d;
            z[i] = d * (1.f - u[i] * u[i]);
          }
          if (a.res[l - 1]) umma::st16f(car + col0, v);
          if (valid) {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              if (l > 1) {
                const uint32_t o = act_off(r, col0 + 8 * h);
                store8_split(ah + o, al + o, z + 8 * h);
              } else {
                const size_t o = tiled_off(prow, col0 + 8 * h, a.kpad_z);
                store8_split(a.Z_hi + o, a.Z_lo + o, z + 8 * h);
              }
            }
          }
        }
      }
      umma::wait_st();
      if (last_fwd) {  // partial energies of the column parts, summed in part order
        s_e[part][r] = e_acc;
        umma::bar_sync(1, kChainEpiWarps * 32);
        if (part == 0 && valid && ok) {
          double e = a.bo[t];
          for (int p2 = 0; p2 < nparts; ++p2) e += s_e[p2][r];
          a.atom_e[a.perm_atom[row0 + r]] = e;
        }
      }
      umma::fence_proxy_async();
      umma::fence_before_sync();
      umma::mbar_arrive(&act_full);
    }
    if (!ok) s_fail = 1;
  }
  umma::fence_before_sync();
  __syncthreads();
  if (tid == 0 && s_fail) atomicAdd(a.err + 3, 1);
  if (warp == 0) umma::tmem_dealloc(tbase, 512);
}

// ------------------------------------------------------------ final backward
// dD = dz0 W0^T fused with the descriptor contraction (D = T^T T_<, with T
// already divided by N):
//   dT[k][a] = (sum_b dD[a][b] T[k][b] + [a < M2] sum_c dD[c][a] T[k][c]) / N
// One CTA per 128-row tile and chunk range: with few row tiles (small
// systems) the N chunks of a tile are split over gridDim.y CTAs so that the
// SMs are used; the second term's partial sums then go to dt_part and the
// last CTA of the tile to arrive adds them in split order (deterministic).
// The whole dz0 tile stays in shared memory; dD is
// produced in N chunks of BN = 16 NA columns (NA descriptor rows a) into two
// TMEM buffers, so the epilogue of chunk j overlaps the MMAs of chunk j + 1.
// Warps 0-15 run the epilogue: four warps per TMEM lane quadrant, one per
// environment component k, each reading the whole chunk of its rows; warp 16
// streams W0 through a ring of shared-memory stages and warp 17 issues the
// MMAs.  dD itself is written only when requested
// (descriptor inspection).
constexpr int kDtMaxStages = 16;
constexpr int kDtThreads = 576;
constexpr size_t kDtSmemMax = 227 * 1024 - 2048;  // dynamic shared memory budget of k_fit_dT

struct DtArgs {
  int ntypes;
  const int* type_start;
  const int* ftile;
  int nk;  // K chunks of dz0 (32 columns each)
  const unsigned char* A_hi;
  const unsigned char* A_lo;
  const unsigned char* B_hi[kMaxTypes];
  const unsigned char* B_lo[kMaxTypes];
  int BN, nchunks, M1, stages;
  float inv_nnei;
  const float* T;  // in the fitting's row tiles: [tile][4][M1][128]
  float* dT;  // [row][4][M1]
  float* dD;  // [row][16 M1] or null
  float* part;     // split partials (gridDim.y > 1)
  unsigned* cnt;   // per-tile arrival counters (gridDim.y > 1)
  int* err;
};

__global__ void __launch_bounds__(kDtThreads, 1) k_fit_dT(DtArgs a) {
  extern __shared__ __align__(1024) unsigned char smem[];
  __shared__ uint64_t a_full, b_full[kDtMaxStages], b_empty[kDtMaxStages], acc_full[2], acc_empty[2];
  __shared__ uint32_t tbase;
  __shared__ int s_fail, s_last;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = blockIdx.x;
  const int nsplit = gridDim.y, split = blockIdx.y;
  const int per = (a.nchunks + nsplit - 1) / nsplit;
  const int j0 = min(a.nchunks, split * per), j1 = min(a.nchunks, j0 + per);
  if (g >= a.ftile[a.ntypes]) return;  // CTA-uniform, before any TMEM allocation
  int t = 0;
  while (t + 1 < a.ntypes && a.ftile[t + 1] <= g) ++t;
  const int row0 = a.type_start[t] + 128 * (g - a.ftile[t]);
  const int nrows = min(128, a.type_start[t + 1] - row0);
  const uint32_t AH = (uint32_t)a.nk * kABlock;  // one half of the dz0 tile
  const uint32_t BB = (uint32_t)a.BN * kFitBK * 2;
  unsigned char* sA = smem;
  unsigned char* sB = smem + 2 * AH;
  if (warp == 0) umma::tmem_alloc(&tbase, 512);
  if (tid == 0) {
    umma::mbar_init(&a_full, 1);
    for (int s = 0; s < a.stages; ++s) {
      umma::mbar_init(&b_full[s], 1);
      umma::mbar_init(&b_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      umma::mbar_init(&acc_full[i], 1);
      umma::mbar_init(&acc_empty[i], 512);
    }
    umma::fence_mbar_init();
    s_fail = 0;
  }
  umma::fence_before_sync();
  __syncthreads();
  umma::fence_after_sync();
  const int total = (j1 - j0) * a.nk;
  const int S = a.stages;
  if (warp == 16 && lane == 0) {  // loader: the dz0 tile once, then the W0 blocks through the ring
    const unsigned char* Ah = a.A_hi + (size_t)g * AH;
    const unsigned char* Al = a.A_lo + (size_t)g * AH;
    umma::mbar_expect_tx(&a_full, 2 * AH);
    for (int kc = 0; kc < a.nk; ++kc) {
      umma::bulk_g2s(sA + kc * kABlock, Ah + (size_t)kc * kABlock, kABlock, &a_full);
      umma::bulk_g2s(sA + AH + kc * kABlock, Al + (size_t)kc * kABlock, kABlock, &a_full);
    }
    const unsigned char* Bh = a.B_hi[t] + (size_t)j0 * a.nk * BB;  // B blocks are ordered (N chunk, K chunk)
    const unsigned char* Bl = a.B_lo[t] + (size_t)j0 * a.nk * BB;
    int s = 0, round = 0;
    for (int it = 0; it < total; ++it) {
      if (round > 0 && !umma::mbar_wait(&b_empty[s], (round - 1) & 1, kWaitLimit)) {
        s_fail = 1;
        break;
      }
      unsigned char* st = sB + s * 2 * BB;
      umma::mbar_expect_tx(&b_full[s], 2 * BB);
      umma::bulk_g2s(st, Bh + (size_t)it * BB, BB, &b_full[s]);
      umma::bulk_g2s(st + BB, Bl + (size_t)it * BB, BB, &b_full[s]);
      if (++s == S) {
        s = 0;
        ++round;
      }
    }
  } else if (warp == 17 && lane == 0) {  // MMA issuer
    bool ok = umma::mbar_wait(&a_full, 0, kWaitLimit);
    umma::fence_after_sync();
    const uint32_t idesc = umma::idesc_bf16(128, a.BN, false, false);
    const uint64_t dah = umma::desc(umma::smem_u32(sA), 128, kSbo);
    const uint64_t dal = umma::desc(umma::smem_u32(sA + AH), 128, kSbo);
    const uint64_t db0 = umma::desc(umma::smem_u32(sB), 128, kSbo);
    const uint64_t sstep = (2 * BB) >> 4, o_bl = BB >> 4, kstep = kABlock >> 4;
    int s = 0, round = 0;
    for (int j = 0; j < j1 - j0 && ok; ++j) {  // j counts this CTA's chunks
      const int buf = j & 1;
      if (j >= 2) {
        ok = umma::mbar_wait(&acc_empty[buf], ((j - 2) >> 1) & 1, kWaitLimit);
        if (!ok) break;
        umma::fence_after_sync();
      }
      const uint32_t d = tbase + buf * 256;
      for (int kc = 0; kc < a.nk; ++kc) {
        ok = umma::mbar_wait(&b_full[s], round & 1, kWaitLimit);
        if (!ok) break;
        umma::fence_after_sync();
        const uint64_t ah = dah + (uint64_t)kc * kstep, al = dal + (uint64_t)kc * kstep;
        const uint64_t bh = db0 + (uint64_t)s * sstep, bl = bh + o_bl;
#pragma unroll
        for (int ks = 0; ks < kFitBK / 16; ++ks) {
          const uint64_t o = (uint64_t)(ks * (256 >> 4));
          umma::mma(d, ah + o, bh + o, idesc, (kc | ks) ? 1u : 0u);
          umma::mma(d, ah + o, bl + o, idesc, 1u);
          umma::mma(d, al + o, bh + o, idesc, 1u);
        }
        umma::commit(&b_empty[s]);
        if (++s == S) {
          s = 0;
          ++round;
        }
      }
      if (ok) umma::commit(&acc_full[buf]);
    }
    if (!ok) s_fail = 1;
  } else if (warp < 16) {  // epilogue
    const int k = warp >> 2, q = warp & 3, r = q * 32 + lane;
    const bool valid = r < nrows;
    const int urow = row0 + r;
    const int M1 = a.M1;
    const float* Tk = a.T + ((size_t)g * 4 + k) * M1 * 128 + r;  // element c at Tk[128 c]: lanes read a line
    float* dTk = a.dT + (size_t)urow * 4 * M1 + k * M1;
    const uint32_t lb = (uint32_t)(q * 32) << 16;
    float Tb[16], acc2[16];
#pragma unroll
    for (int b = 0; b < 16; ++b) {
      Tb[b] = valid ? Tk[128 * b] : 0.f;
      acc2[b] = 0.f;
    }
    const int NA = a.BN / 16;  // at most 16, even (BN is a multiple of 32)
    // dT rows are written as 8-byte pairs when a row's M1 floats keep them
    // aligned (one row per thread, so each access is its own sector)
    const bool pairs = (M1 & 1) == 0;
    bool ok = true;
    for (int jj = 0; jj < j1 - j0; ++jj) {
      const int j = j0 + jj, buf = jj & 1;
      float tav[16];  // T[k][a] of the chunk's rows a, loaded before waiting for the MMA
      float dtv[16];  // the chunk's first terms, stored after the loop
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        tav[i] = (valid && i < NA) ? Tk[128 * (j * NA + i)] : 0.f;
        dtv[i] = 0.f;
      }
      if (ok) ok = umma::mbar_wait(&acc_full[buf], (jj >> 1) & 1, kWaitLimit);
      umma::fence_after_sync();
      if (ok) {
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          if (i >= NA) break;
          const int aa = j * NA + i;
          float dv[16];
          umma::ld16(tbase + lb + buf * 256 + i * 16, dv);
          umma::wait_ld();
          if (valid) {
            const float ta = tav[i];
            float s0 = 0.f, s1 = 0.f;
#pragma unroll
            for (int b = 0; b < 16; b += 2) {
              s0 = fmaf(dv[b], Tb[b], s0);
              s1 = fmaf(dv[b + 1], Tb[b + 1], s1);
              acc2[b] = fmaf(dv[b], ta, acc2[b]);
              acc2[b + 1] = fmaf(dv[b + 1], ta, acc2[b + 1]);
            }
            dtv[i] = (s0 + s1) * a.inv_nnei;
            if (a.dD && k == 0) {
              float4* dst = reinterpret_cast<float4*>(a.dD + (size_t)urow * 16 * M1 + aa * 16);
#pragma unroll
              for (int b = 0; b < 16; b += 4) dst[b / 4] = make_float4(dv[b], dv[b + 1], dv[b + 2], dv[b + 3]);
            }
          }
        }
      }
      umma::fence_before_sync();
      umma::mbar_arrive(&acc_empty[buf]);
      if (valid && ok) {
#pragma unroll
        for (int i = 0; i < 16; i += 2) {
          if (i >= NA) break;
          if (pairs) {
            *reinterpret_cast<float2*>(dTk + j * NA + i) = make_float2(dtv[i], dtv[i + 1]);
          } else {
            dTk[j * NA + i] = dtv[i];
            dTk[j * NA + i + 1] = dtv[i + 1];
          }
        }
      }
    }
    if (nsplit == 1) {
      // second term for a < 16: this thread wrote the first term itself
      if (valid && ok) {
#pragma unroll
        for (int b = 0; b < 16; ++b) dTk[b] += acc2[b] * a.inv_nnei;
      }
    } else {
      float4* pp = reinterpret_cast<float4*>(a.part + (((size_t)split * gridDim.x + g) * 128 + r) * 64 + k * 16);
#pragma unroll
      for (int b = 0; b < 16; b += 4) pp[b / 4] = make_float4(acc2[b], acc2[b + 1], acc2[b + 2], acc2[b + 3]);
      __threadfence();
    }
    if (!ok) s_fail = 1;
  }
  umma::fence_before_sync();
  __syncthreads();
  if (tid == 0 && s_fail) atomicAdd(a.err + 3, 1);
  if (warp == 0) umma::tmem_dealloc(tbase, 512);
  if (nsplit == 1) return;
  // the tile's last CTA adds the splits' second terms, in split order
  if (tid == 0) {
    s_last = atomicAdd(a.cnt + g, 1u) == (unsigned)nsplit - 1;
    if (s_last) a.cnt[g] = 0u;  // ready for the next launch
  }
  __syncthreads();
  if (!s_last || warp >= 16 || s_fail) return;
  __threadfence();
  const int k = warp >> 2, r = (warp & 3) * 32 + lane;
  if (r >= nrows) return;
  float sum[16];
#pragma unroll
  for (int b = 0; b < 16; ++b) sum[b] = 0.f;
  for (int sp = 0; sp < nsplit; ++sp) {
    const float4* pp = reinterpret_cast<const float4*>(a.part + (((size_t)sp * gridDim.x + g) * 128 + r) * 64 + k * 16);
#pragma unroll
    for (int b = 0; b < 16; b += 4) {
      const float4 v = __ldcg(pp + b / 4);
      sum[b] += v.x;
      sum[b + 1] += v.y;
      sum[b + 2] += v.z;
      sum[b + 3] += v.w;
    }
  }
  float* dTk = a.dT + (size_t)(row0 + r) * 4 * a.M1 + k * a.M1;
#pragma unroll
  for (int b = 0; b < 16; ++b) dTk[b] = __ldcg(dTk + b) + sum[b] * a.inv_nnei;
}

int round32(int x) { return (x + 31) / 32 * 32; }

// Largest N tile that is a multiple of 16, at most 128 and divides w into at
// least two tiles (more CTAs per layer); w itself when no such tile exists.
int split_bn(int w) {
  for (int bn = 128; bn >= 16; bn -= 16)
    if (w % bn == 0 && w / bn >= 2) return bn;
  return w;
}

}  // namespace

FitTcPlan fit_tc_plan(const HostModel& m) {
  FitTcPlan p;
  p.L = (int)m.fit.size();
  p.dim = m.dim();
  if (p.L < 1 || p.L > kFitMaxLayers || p.dim % kFitBK != 0 || m.ntypes > kMaxTypes) return p;
  int din = p.dim;
  for (int l = 0; l < p.L; ++l) {
    const int w = m.fit[l];
    if (w % 16 != 0 || w > 256) return p;
    p.width[l] = w;
    p.kpad[l] = l == 0 ? p.dim : round32(m.fit[l - 1]);
    p.res[l] = (l >= 1 && w == din) ? 1 : 0;
    din = w;
  }
  for (int l = 0; l < p.L; ++l) {
    // layer 0 forms its operand (the descriptor) from T inside the GEMM: one CTA per
    // row tile takes the whole width, so that the operand is formed once
    p.bnf[l] = (l == p.L - 1 || l == 0) ? p.width[l] : split_bn(p.width[l]);
    p.bnb[l] = (l == 0) ? 0 : split_bn(p.width[l - 1]);
  }
  // final backward: N chunks of whole descriptor rows (16 columns each), an
  // even number of them, at most 256 columns; three W0 stages must fit beside
  // the resident dz0 tile
  p.bn_out = 0;
  if (m.axis == 16)
    for (int bn = 256; bn >= 32; bn -= 32)
      if (p.dim % bn == 0) {
        p.bn_out = bn;
        break;
      }
  if (p.L >= 1 && 2 * (size_t)(round32(p.width[0]) / kFitBK) * kABlock + 3 * 2 * (size_t)p.bn_out * kFitBK * 2 >
                      kDtSmemMax)
    p.bn_out = 0;
  p.ok = p.bn_out > 0;
  // hidden layers 1 .. L-1 in one launch: every operand at most kChainK wide, and the
  // activation tile plus two ring stages of the widest step fit in shared memory
  p.chain = p.ok && p.L >= 2;
  int nmax = 0;
  for (int l = 1; l < p.L && p.chain; ++l) {
    if (p.kpad[l] > kChainK || round32(p.width[l]) > kChainK) p.chain = false;
    nmax = std::max(nmax, std::max(p.width[l], p.width[l - 1]));
  }
  if (p.chain && kChainAct + 2 * (size_t)nmax * kFitBK * 4 > kChainSmemMax) p.chain = false;
  p.chain_stages = p.chain ? (int)std::min<size_t>(kMaxStages, (kChainSmemMax - kChainAct) / ((size_t)nmax * kFitBK * 4))
                           : 0;
  return p;
}

void fit_pack_B(int N, int Kp, int BN, const std::function<double(int, int)>& val, std::vector<unsigned char>& hi,
                std::vector<unsigned char>& lo) {
  const int nkc = Kp / kFitBK;
  const size_t bytes = (size_t)N * Kp * 2;
  hi.assign(bytes, 0);
  lo.assign(bytes, 0);
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
  for (int n = 0; n < N; ++n)
    for (int k = 0; k < Kp; ++k) {
      const float x = (float)val(n, k);
      const uint16_t h = to_bf16(x);
      const uint16_t l = to_bf16(x - from_bf16(h));
      const int nt = n / BN, nn = n % BN;
      const size_t o = ((size_t)nt * nkc + k / kFitBK) * ((size_t)BN * kFitBK * 2) + (size_t)(nn >> 3) * kSbo +
                       (size_t)((k % kFitBK) >> 3) * 128 + (nn & 7) * 16 + (k & 7) * 2;
      std::memcpy(&hi[o], &h, 2);
      std::memcpy(&lo[o], &l, 2);
    }
}

static void run_gemm(cudaStream_t st, GemmArgs& a, int row_tiles, int ntn) {
  // K chunks stream from L2: a deep pipeline hides its latency.  With several
  // N tiles two CTAs share an SM (4 stages each), else one CTA takes up to 8.
  const size_t sb = 2 * kABlock + 2 * (size_t)a.BN * kFitBK * 2 + (a.Tt ? kTSlice : 0);
  // (with the slice of T a stage is 4 KB larger: three stages keep two CTAs on an SM)
  a.stages = ntn > 1 ? (a.Tt ? 3 : 4) : (int)std::min<size_t>(kMaxStages, (200 * 1024) / sb);
  a.stages = std::max(2, std::min(a.stages, a.nk));
  const size_t smem = (size_t)a.stages * sb;
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(k_fit_gemm, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    attr = true;
  }
  count_launch();
  k_fit_gemm<<<dim3(row_tiles, ntn), kFitThreads, smem, st>>>(a);
}

void launch_fit_tc(cudaStream_t st, const FitTcPlan& p, int ntypes, int nloc, const int* type_start,
                   const int* ftile, const int* perm_atom, const FitTcWeights* w, const FitTcBuffers& b,
                   double* atom_energy, const float* T, float inv_nnei, float* dT, float* dD, int* err) {
  if (nloc <= 0) return;
  const int row_tiles = (nloc + 127) / 128 + ntypes;
  const int L = p.L;
  const bool chain = p.chain;
  for (int l = 0; l < (chain ? 1 : L); ++l) {
    GemmArgs a;
    std::memset(&a, 0, sizeof(a));
    a.ntypes = ntypes;
    a.type_start = type_start;
    a.ftile = ftile;
    a.nk = p.kpad[l] / kFitBK;
    a.A_hi = b.At_hi[l];
    a.A_lo = b.At_lo[l];
    if (l == 0) {  // the descriptor is formed from T inside the GEMM (no tiled copy of D)
      a.Tt = T;
      a.M1 = p.dim / 16;
    }
    for (int t = 0; t < ntypes; ++t) {
      a.B_hi[t] = w[t].fB_hi[l];
      a.B_lo[t] = w[t].fB_lo[l];
      a.bias[t] = w[t].bias[l];
      a.wo[t] = w[t].wo;
      a.bo[t] = w[t].bo;
    }
    a.BN = p.bnf[l];
    a.N = p.width[l];
    a.mode = kFwd;
    a.Yprev = p.res[l] ? b.Y[l - 1] : nullptr;
    a.ldprev = l > 0 ? p.width[l - 1] : 0;
    a.TH = b.TH[l];
    a.Y = b.Y[l];
    a.last = (l == L - 1);
    if (!a.last) {
      a.Anext_hi = b.At_hi[l + 1];
      a.Anext_lo = b.At_lo[l + 1];
      a.kpad_next = p.kpad[l + 1];
    } else {
      a.Z_hi = b.Z_hi[0];
      a.Z_lo = b.Z_lo[0];
      a.kpad_z = round32(p.width[l]);
      a.perm_atom = perm_atom;
      a.atom_e = atom_energy;
    }
    a.err = err;
    run_gemm(st, a, row_tiles, p.width[l] / p.bnf[l]);
  }
  if (chain) {
    ChainArgs c;
    std::memset(&c, 0, sizeof(c));
    c.ntypes = ntypes;
    c.type_start = type_start;
    c.ftile = ftile;
    c.L = L;
    for (int l = 0; l < L; ++l) {
      c.width[l] = p.width[l];
      c.kpad[l] = p.kpad[l];
      c.res[l] = p.res[l];
      c.bnf[l] = p.bnf[l];
      c.bnb[l] = p.bnb[l];
      c.TH[l] = b.TH[l];
      for (int t = 0; t < ntypes; ++t) {
        c.fB_hi[t][l] = w[t].fB_hi[l];
        c.fB_lo[t][l] = w[t].fB_lo[l];
        c.bB_hi[t][l] = w[t].bB_hi[l];
        c.bB_lo[t][l] = w[t].bB_lo[l];
        c.bias[t][l] = w[t].bias[l];
      }
    }
    for (int t = 0; t < ntypes; ++t) {
      c.wo[t] = w[t].wo;
      c.bo[t] = w[t].bo;
    }
    c.A_hi = b.At_hi[1];
    c.A_lo = b.At_lo[1];
    c.Y0 = b.Y[0];
    c.perm_atom = perm_atom;
    c.atom_e = atom_energy;
    c.Z_hi = b.Z_hi[(L - 1) & 1];  // where the final backward below reads dz0
    c.Z_lo = b.Z_lo[(L - 1) & 1];
    c.kpad_z = round32(p.width[0]);
    c.stages = p.chain_stages;
    c.err = err;
    int nmax = 0;
    for (int l = 1; l < L; ++l) nmax = std::max(nmax, std::max(p.width[l], p.width[l - 1]));
    const size_t smem = kChainAct + (size_t)c.stages * nmax * kFitBK * 4;
    static size_t attr = 0;
    if (smem > attr) {
      cudaFuncSetAttribute(k_fit_chain, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      attr = smem;
    }
    count_launch();
    k_fit_chain<<<row_tiles, kChainThreads, smem, st>>>(c);
  }
  for (int s = chain ? L - 1 : 0; s < L; ++s) {
    const int l = L - 1 - s;
    GemmArgs a;
    std::memset(&a, 0, sizeof(a));
    a.ntypes = ntypes;
    a.type_start = type_start;
    a.ftile = ftile;
    a.nk = round32(p.width[l]) / kFitBK;
    a.A_hi = b.Z_hi[s & 1];
    a.A_lo = b.Z_lo[s & 1];
    for (int t = 0; t < ntypes; ++t) {
      a.B_hi[t] = w[t].bB_hi[l];
      a.B_lo[t] = w[t].bB_lo[l];
      a.wo[t] = w[t].wo;
    }
    a.err = err;
    if (l >= 1) {
      a.BN = p.bnb[l];
      a.N = p.width[l - 1];
      a.mode = kBwd;
      a.dy_is_wo = (p.res[l] && l == L - 1) ? 1 : 0;
      a.DYnext = (p.res[l] && l < L - 1) ? b.DY[s & 1] : nullptr;
      a.DYout = p.res[l - 1] ? b.DY[(s + 1) & 1] : nullptr;
      a.THprev = b.TH[l - 1];
      a.Z_hi = b.Z_hi[(s + 1) & 1];
      a.Z_lo = b.Z_lo[(s + 1) & 1];
      a.kpad_z = round32(p.width[l - 1]);
      run_gemm(st, a, row_tiles, p.width[l - 1] / p.bnb[l]);
    } else {
      DtArgs d;
      std::memset(&d, 0, sizeof(d));
      d.ntypes = ntypes;
      d.type_start = type_start;
      d.ftile = ftile;
      d.nk = a.nk;
      d.A_hi = a.A_hi;
      d.A_lo = a.A_lo;
      for (int t = 0; t < ntypes; ++t) {
        d.B_hi[t] = a.B_hi[t];
        d.B_lo[t] = a.B_lo[t];
      }
      d.BN = p.bn_out;
      d.nchunks = p.dim / p.bn_out;
      d.M1 = p.dim / 16;
      d.inv_nnei = inv_nnei;
      d.T = T;
      d.dT = dT;
      d.dD = dD;
      d.part = b.dt_part;
      d.cnt = b.dt_cnt;
      d.err = err;
      // few row tiles: split each tile's chunks over CTAs so that the SMs are used
      // (splitting more tiles than fill one wave was measured slower: each split CTA
      // reloads the tile's whole dz0 operand and the partial sums add a pass)
      int nsplit = 1;
      if (b.dt_part && b.dt_cnt && row_tiles > 0) {
        nsplit = std::max(1, std::min(d.nchunks, kDtSplitSlots / row_tiles));
        const int per = (d.nchunks + nsplit - 1) / nsplit;
        nsplit = (d.nchunks + per - 1) / per;  // no CTA without a chunk
      }
      // as many W0 stages as fit beside the resident dz0 tile: the stream is L2-latency bound
      const size_t abytes = 2 * (size_t)d.nk * kABlock, sbytes = 2 * (size_t)d.BN * kFitBK * 2;
      d.stages = (int)std::min<size_t>(kDtMaxStages, (kDtSmemMax - abytes) / sbytes);
      const size_t smem = abytes + d.stages * sbytes;
      static size_t attr = 0;
      if (smem > attr) {
        cudaFuncSetAttribute(k_fit_dT, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        attr = smem;
      }
      count_launch();
      k_fit_dT<<<dim3(row_tiles, nsplit), kDtThreads, smem, st>>>(d);
    }
  }
}

}  // namespace b200dp
