// Shared device helpers for the b200dp kernels (sm_100a).
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace b200dp {

// Host-side count of kernels this library has launched (diagnostic; read
// through b200dp_kernel_launches).
void count_launch();
long long launch_count();

constexpr int kWarp = 32;
constexpr int kMaxTypes = 8;
constexpr int kMaxLayers = 6;
constexpr int kImageBias = 512;

// Device-side error counters (one int each, in the engine's status block).
enum DeviceError : int {
  kErrSelOverflow = 0,   // candidates dropped because a type section held more than sel
  kErrCandCapacity = 1,  // a centre had more in-cutoff candidates than the per-warp buffer
  kErrBadType = 2,       // atom type outside [0, ntypes)
  kErrCount = 4
};

// Explicit round-to-nearest fp64 arithmetic: the neighbour builder must give
// the same bits as the host oracle, which is compiled without contraction.
__device__ __forceinline__ double dmul(double a, double b) { return __dmul_rn(a, b); }
__device__ __forceinline__ double dadd(double a, double b) { return __dadd_rn(a, b); }
__device__ __forceinline__ double dsub(double a, double b) { return __dsub_rn(a, b); }

__device__ __forceinline__ int image_code(int n0, int n1, int n2) {
  return ((n0 + kImageBias) << 20) | ((n1 + kImageBias) << 10) | (n2 + kImageBias);
}

template <typename T>
__device__ __forceinline__ T warp_sum(T v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ int warp_exclusive_scan(int v, int lane, int& total) {
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  total = __shfl_sync(0xffffffffu, x, 31);
  return x - v;
}

template <typename P>
__device__ __forceinline__ P act_tanh(P x);
template <>
__device__ __forceinline__ double act_tanh<double>(double x) {
  return tanh(x);
}
template <>
__device__ __forceinline__ float act_tanh<float>(float x) {
  return tanhf(x);
}

// Quintic switch of DeePMD's env_mat_a (1 below rs, 0 at rc) and its derivative.
__device__ __forceinline__ void smooth_switch(double r, double rs, double rc, double& sw, double& dsw) {
  if (r < rs) {
    sw = 1.0;
    dsw = 0.0;
  } else if (r < rc) {
    const double du = 1.0 / (rc - rs);
    const double u = (r - rs) * du;
    const double u2 = u * u, u3 = u2 * u;
    sw = u3 * (-6.0 * u2 + 15.0 * u - 10.0) + 1.0;
    dsw = (3.0 * u2 * (-6.0 * u2 + 15.0 * u - 10.0) + u3 * (-12.0 * u + 15.0)) * du;
  } else {
    sw = 0.0;
    dsw = 0.0;
  }
}

}  // namespace b200dp

#define B200DP_CUDA_TRY(expr)                                  \
  do {                                                         \
    cudaError_t _e = (expr);                                   \
    if (_e != cudaSuccess) return ::b200dp::cuda_fail(_e, #expr, __FILE__, __LINE__); \
  } while (0)
