// Self-test of the tcgen05 helper layer (umma.cuh): one CTA computes
// C[128 x N] = A[128 x K] * B[N x K]^T from fp32 inputs split into bf16 hi/lo,
// with 1 (hi*hi) or 3 (hi*hi + hi*lo + lo*hi) tensor-core products accumulated
// in TMEM, either operand in K-major or MN-major no-swizzle layout.
#include <cstdio>

#include "../../include/b200dp.h"
#include "common.cuh"
#include "umma.cuh"

namespace b200dp {

__global__ void __launch_bounds__(128)
    k_umma_selftest(int K, int N, int a_mn, int b_mn, int passes, const float* __restrict__ A,
                    const float* __restrict__ B, float* __restrict__ C, int* __restrict__ err) {
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ uint64_t bar;
  __shared__ uint32_t tbase;
  const int tid = threadIdx.x, warp = tid >> 5;
  unsigned char* a_hi = smem;
  unsigned char* a_lo = a_hi + 128 * K * 2;
  unsigned char* b_hi = a_lo + 128 * K * 2;
  unsigned char* b_lo = b_hi + N * K * 2;
  const uint32_t lboA = a_mn ? (128 / 8) * 128 : 128, sboA = a_mn ? 128 : (K / 8) * 128;
  const uint32_t lboB = b_mn ? (N / 8) * 128 : 128, sboB = b_mn ? 128 : (K / 8) * 128;
  for (int idx = tid; idx < 128 * K; idx += 128) {
    const int r = idx / K, k = idx % K;
    __nv_bfloat16 hi, lo;
    umma::split_bf16(A[idx], hi, lo);
    const uint32_t o = a_mn ? umma::off_mnmajor(r, k, lboA, sboA) : umma::off_kmajor(r, k, lboA, sboA);
    *reinterpret_cast<__nv_bfloat16*>(a_hi + o) = hi;
    *reinterpret_cast<__nv_bfloat16*>(a_lo + o) = lo;
  }
  for (int idx = tid; idx < N * K; idx += 128) {
    const int r = idx / K, k = idx % K;
    __nv_bfloat16 hi, lo;
    umma::split_bf16(B[idx], hi, lo);
    const uint32_t o = b_mn ? umma::off_mnmajor(r, k, lboB, sboB) : umma::off_kmajor(r, k, lboB, sboB);
    *reinterpret_cast<__nv_bfloat16*>(b_hi + o) = hi;
    *reinterpret_cast<__nv_bfloat16*>(b_lo + o) = lo;
  }
  uint32_t ncols = 32;
  while ((int)ncols < N) ncols <<= 1;
  if (warp == 0) umma::tmem_alloc(&tbase, ncols);
  if (tid == 0) {
    umma::mbar_init(&bar, 1);
    umma::fence_mbar_init();
  }
  umma::fence_proxy_async();
  umma::fence_before_sync();
  __syncthreads();
  umma::fence_after_sync();
  const uint32_t tmem = tbase;
  if (tid == 0) {
    const uint32_t idesc = umma::idesc_bf16(128, N, a_mn != 0, b_mn != 0);
    const unsigned char* as[3] = {a_hi, a_hi, a_lo};
    const unsigned char* bs[3] = {b_hi, b_lo, b_hi};
    for (int s = 0; s < K / 16; ++s)
      for (int p = 0; p < passes; ++p) {
        const uint64_t ad = umma::desc(umma::smem_u32(as[p]) + s * 2 * lboA, lboA, sboA);
        const uint64_t bd = umma::desc(umma::smem_u32(bs[p]) + s * 2 * lboB, lboB, sboB);
        umma::mma(tmem, ad, bd, idesc, (s > 0 || p > 0) ? 1u : 0u);
      }
    umma::commit(&bar);
  }
  const bool ok = umma::mbar_wait(&bar, 0, 1LL << 24);
  if (!ok && tid == 0) atomicAdd(err, 1);
  umma::fence_after_sync();
  if (ok) {
    for (int c0 = 0; c0 < N; c0 += 16) {
      float v[16];
      umma::ld16(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)c0, v);
      umma::wait_ld();
#pragma unroll
      for (int j = 0; j < 16; ++j) C[tid * N + c0 + j] = v[j];
    }
  }
  umma::fence_before_sync();
  __syncthreads();
  if (warp == 0) umma::tmem_dealloc(tmem, ncols);
}

}  // namespace b200dp

extern "C" b200dp_status b200dp_selftest_mma(int K, int N, int a_mn_major, int b_mn_major, int passes,
                                             const float* A, const float* B, float* C) {
  using namespace b200dp;
  if (K < 16 || K > 256 || K % 16 || N < 16 || N > 256 || N % 16 || (passes != 1 && passes != 3) || !A || !B || !C)
    return B200DP_ERR_INVALID;
  if ((size_t)4 * K * (128 + N) > 200 * 1024) return B200DP_ERR_INVALID;  // operands must fit in shared memory
  float *dA = nullptr, *dB = nullptr, *dC = nullptr;
  int* dErr = nullptr;
  b200dp_status st = B200DP_OK;
  const size_t smem = (size_t)2 * 128 * K * 2 + (size_t)2 * N * K * 2;
  int herr = 0;
  if (cudaMalloc(&dA, sizeof(float) * 128 * K) != cudaSuccess || cudaMalloc(&dB, sizeof(float) * N * K) != cudaSuccess ||
      cudaMalloc(&dC, sizeof(float) * 128 * N) != cudaSuccess || cudaMalloc(&dErr, sizeof(int)) != cudaSuccess) {
    st = B200DP_ERR_CUDA;
    goto done;
  }
  if (cudaMemcpy(dA, A, sizeof(float) * 128 * K, cudaMemcpyHostToDevice) != cudaSuccess ||
      cudaMemcpy(dB, B, sizeof(float) * N * K, cudaMemcpyHostToDevice) != cudaSuccess ||
      cudaMemset(dErr, 0, sizeof(int)) != cudaSuccess ||
      cudaFuncSetAttribute(k_umma_selftest, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess) {
    st = B200DP_ERR_CUDA;
    goto done;
  }
  count_launch();
  k_umma_selftest<<<1, 128, smem>>>(K, N, a_mn_major, b_mn_major, passes, dA, dB, dC, dErr);
  if (cudaDeviceSynchronize() != cudaSuccess || cudaGetLastError() != cudaSuccess) {
    st = B200DP_ERR_CUDA;
    goto done;
  }
  if (cudaMemcpy(&herr, dErr, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess || herr ||
      cudaMemcpy(C, dC, sizeof(float) * 128 * N, cudaMemcpyDeviceToHost) != cudaSuccess)
    st = B200DP_ERR_CUDA;
done:
  cudaFree(dA);
  cudaFree(dB);
  cudaFree(dC);
  cudaFree(dErr);
  return st;
}
