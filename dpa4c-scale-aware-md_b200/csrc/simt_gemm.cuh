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

}  // namespace b200dp
