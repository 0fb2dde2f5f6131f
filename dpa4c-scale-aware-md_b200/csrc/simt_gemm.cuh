// Tiled SIMT GEMM with a fused per-element epilogue, shared by the fitting
// nets of both model profiles (fp64 and fp32).
#pragma once

#include <cuda_runtime.h>

namespace b200dp {

constexpr int kBM = 64, kBN = 64, kBK = 16;

// Rows [range[0], range[1]) of A when range is given (a device pair), else
// rows [0, Mrows).
// C[m][n] = sum_k A[m][k] * B(k, n), B(k, n) = BT ? B[n*ldb + k] : B[k*ldb + n].
// 256 threads, 4x4 outputs each at stride 16 (bank-conflict free reads).
template <typename P, bool BT, class Epi>
__global__ void __launch_bounds__(256) k_gemm(const int* __restrict__ range, int N, int K, const P* __restrict__ A,
                                               int lda, const P* __restrict__ B, int ldb, Epi epi, int Mrows = 0) {
  __shared__ P As[kBK][kBM + 1];
  __shared__ P Bs[kBK][kBN + 1];
  const int row0 = range ? range[0] : 0, M = range ? range[1] - row0 : Mrows;
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int m0 = blockIdx.y * kBM, n0 = blockIdx.x * kBN;
  if (m0 >= M) return;
  A += (size_t)row0 * lda;
  P acc[4][4];
#pragma unroll
  for (int q = 0; q < 4; ++q)
#pragma unroll
    for (int r = 0; r < 4; ++r) acc[q][r] = 0;
  for (int k0 = 0; k0 < K; k0 += kBK) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int idx = tid + 256 * q;  // 0..1023
      const int mm = idx / kBK, kk = idx % kBK;
      const int m = m0 + mm, k = k0 + kk;
      As[kk][mm] = (m < M && k < K) ? A[(size_t)m * lda + k] : (P)0;
      if (BT) {
        const int nn = idx / kBK, kb = idx % kBK;
        const int n = n0 + nn, kx = k0 + kb;
        Bs[kb][nn] = (n < N && kx < K) ? B[(size_t)n * ldb + kx] : (P)0;
      } else {
        const int kb = idx / kBN, nn = idx % kBN;
        const int n = n0 + nn, kx = k0 + kb;
        Bs[kb][nn] = (n < N && kx < K) ? B[(size_t)kx * ldb + n] : (P)0;
      }
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < kBK; ++kk) {
      P a[4], b[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        a[q] = As[kk][ty + 16 * q];
        b[q] = Bs[kk][tx + 16 * q];
      }
#pragma unroll
      for (int q = 0; q < 4; ++q)
#pragma unroll
        for (int r = 0; r < 4; ++r) acc[q][r] += a[q] * b[r];
    }
    __syncthreads();
  }
#pragma unroll
  for (int q = 0; q < 4; ++q)
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int m = m0 + ty + 16 * q, n = n0 + tx + 16 * r;
      if (m < M && n < N) epi(row0 + m, n, acc[q][r]);
    }
}

// fp64 GEMM on the tensor cores (mma.sync m8n8k4 .f64: the fp64 tensor path of
// sm_100, which tcgen05 has no kind for), same contract and epilogue as k_gemm
// with P = double.  128 threads, block tile 64 x 64, K chunks of 16 staged in
// shared memory k-major ([k][m], rows padded to 68 doubles: a warp's fragment
// loads touch every bank twice, the minimum for 256 bytes); the next chunk is
// fetched into registers while the current one is multiplied.  Each warp
// computes a 32 x 32 sub-tile as 4 x 4 MMAs of 8 x 8 x 4.  Fragment layouts
// (PTX ISA, m8n8k4 .f64): A row-major, a0 = A[lane / 4][lane % 4]; B
// column-major, b0 = B[lane % 4][lane / 4]; C, D: c0, c1 = C[lane / 4][2 (lane % 4) + 0, 1].
constexpr int kDM = 64, kDN = 64, kDK = 16, kDS = 68;

__device__ __forceinline__ void dmma_8x8x4(double (&d)[2], double a, double b) {
  asm volatile("mma.sync.aligned.m8n8k4.row.col.f64.f64.f64.f64 {%0, %1}, {%2}, {%3}, {%0, %1};"
               : "+d"(d[0]), "+d"(d[1])
               : "d"(a), "d"(b));
}

template <bool BT, class Epi>
__global__ void __launch_bounds__(128) k_dgemm(const int* __restrict__ range, int N, int K,
                                               const double* __restrict__ A, int lda, const double* __restrict__ B,
                                               int ldb, Epi epi, int Mrows = 0) {
  __shared__ double As[kDK][kDS];
  __shared__ double Bs[kDK][kDS];
  const int row0 = range ? range[0] : 0, M = range ? range[1] - row0 : Mrows;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t4 = lane & 3;
  const int m0 = blockIdx.y * kDM, n0 = blockIdx.x * kDN;
  if (m0 >= M) return;
  A += (size_t)row0 * lda;
  const int wm = (warp >> 1) * 32, wn = (warp & 1) * 32;
  double acc[4][4][2];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j][0] = acc[i][j][1] = 0.0;
  double ra[8], rb[8];
  auto fetch = [&](int k0) {
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const int idx = tid + 128 * q;  // 0..1023
      {
        const int mm = idx >> 4, kk = idx & 15, m = m0 + mm, k = k0 + kk;
        ra[q] = (m < M && k < K) ? A[(size_t)m * lda + k] : 0.0;
      }
      if (BT) {
        const int nn = idx >> 4, kb = idx & 15, n = n0 + nn, k = k0 + kb;
        rb[q] = (n < N && k < K) ? B[(size_t)n * ldb + k] : 0.0;
      } else {
        const int kb = idx >> 6, nn = idx & 63, n = n0 + nn, k = k0 + kb;
        rb[q] = (n < N && k < K) ? B[(size_t)k * ldb + n] : 0.0;
      }
    }
  };
  fetch(0);
  for (int k0 = 0; k0 < K; k0 += kDK) {
    __syncthreads();  // the previous chunk's fragment loads are done
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const int idx = tid + 128 * q;
      As[idx & 15][idx >> 4] = ra[q];
      if (BT)
        Bs[idx & 15][idx >> 4] = rb[q];
      else
        Bs[idx >> 6][idx & 63] = rb[q];
    }
    __syncthreads();
    if (k0 + kDK < K) fetch(k0 + kDK);
#pragma unroll
    for (int ks = 0; ks < kDK; ks += 4) {
      double af[4], bf[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) af[i] = As[ks + t4][wm + 8 * i + g];
#pragma unroll
      for (int j = 0; j < 4; ++j) bf[j] = Bs[ks + t4][wn + 8 * j + g];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) dmma_8x8x4(acc[i][j], af[i], bf[j]);
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int m = m0 + wm + 8 * i + g, n = n0 + wn + 8 * j + 2 * t4 + h;
        if (m < M && n < N) epi(row0 + m, n, acc[i][j][h]);
      }
}

}  // namespace b200dp
