// Thin inline-PTX layer over the sm_100a 5th-generation tensor cores
// (tcgen05): TMEM allocation, shared-memory matrix descriptors, MMA issue,
// commit to an mbarrier, and TMEM -> register loads.
//
// Operand layouts are the canonical no-swizzle ("interleave") layouts: a core
// matrix is 8 rows x 16 bytes stored contiguously (128 B).
//   K-major : element (r, k) of an R x K bf16 operand at
//             (r/8)*SBO + (k/8)*LBO + (r%8)*16 + (k%8)*2
//   MN-major: element (r, k) at (r/8)*SBO + (k/8)*LBO + (k%8)*16 + (r%8)*2
// LBO is the byte stride between core matrices along K, SBO along M/N.  One
// kind::f16 MMA consumes K = 16, i.e. two core matrices along K; the next
// K step starts 2*LBO bytes further.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace b200dp {
namespace umma {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// 64-bit shared-memory matrix descriptor, SWIZZLE_NONE, descriptor version 1.
__device__ __forceinline__ uint64_t desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1u << 46;
  return d;
}

// Instruction descriptor for kind::f16 with bf16 A and B, f32 accumulator.
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N, bool a_mn_major, bool b_mn_major) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((a_mn_major ? 1u : 0u) << 15) | ((b_mn_major ? 1u : 0u) << 16) |
         ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// Byte offset of element (r, k) in the canonical layouts above.
__host__ __device__ __forceinline__ uint32_t off_kmajor(int r, int k, uint32_t lbo, uint32_t sbo) {
  return (uint32_t)(r >> 3) * sbo + (uint32_t)(k >> 3) * lbo + (uint32_t)(r & 7) * 16u + (uint32_t)(k & 7) * 2u;
}
__host__ __device__ __forceinline__ uint32_t off_mnmajor(int r, int k, uint32_t lbo, uint32_t sbo) {
  return (uint32_t)(r >> 3) * sbo + (uint32_t)(k >> 3) * lbo + (uint32_t)(k & 7) * 16u + (uint32_t)(r & 7) * 2u;
}

// D[tmem] (+)= A * B^T over one K = 16 step.  Issued by a single thread.
__device__ __forceinline__ void mma(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate));
}

// Arrive once on `bar` when every MMA this thread issued so far has completed.
__device__ __forceinline__ void commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// Executed by one full warp; the TMEM base address is written to *dst.
__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)), "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void fence_before_sync() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_after_sync() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
// Generic-proxy shared-memory writes -> visible to the tensor core (async proxy).
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Each thread of the warp reads 16 consecutive 32-bit columns of its lane.
__device__ __forceinline__ void ld16(uint32_t taddr, float* v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
// Each thread of the warp reads 8 consecutive 32-bit columns of its lane.
__device__ __forceinline__ void ld8(uint32_t taddr, float* v) {
  uint32_t r[8];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// Each thread of the warp writes 16 consecutive 32-bit columns of its lane.
__device__ __forceinline__ void st16(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void st16f(uint32_t taddr, const float* v) {
  uint32_t r[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) r[i] = __float_as_uint(v[i]);
  st16(taddr, r);
}
__device__ __forceinline__ void wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

// Bounded wait for the phase with the given parity to complete.  Returns
// false after `max_iters` unsuccessful polls (the caller records an error and
// unwinds instead of hanging the GPU).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, long long max_iters) {
  const uint32_t addr = smem_u32(bar);
  for (long long it = 0; it < max_iters; ++it) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok)
        : "r"(addr), "r"(parity)
        : "memory");
    if (ok) return true;
  }
  return false;
}

// Plain arrive (one of the barrier's expected arrivals).
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Arrive on `bar` and add `bytes` to its expected transaction count.
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

// Bulk (non-tensor) async copy global -> shared, completing on `bar`.
// Addresses 16-byte aligned, size a multiple of 16.  No multicast.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

// Named barrier over `count` threads (id 1..15; id 0 is __syncthreads).
__device__ __forceinline__ void bar_sync(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}
// Named barrier that also ORs a predicate over the participating threads.
__device__ __forceinline__ bool bar_sync_or(int id, int count, bool pred) {
  uint32_t res;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}\n"
      : "=r"(res)
      : "r"((uint32_t)pred), "r"(id), "r"(count)
      : "memory");
  return res != 0;
}

// Byte offset of element (row, k) in a pre-tiled activation operand: blocks
// of 128 rows x 32 columns (8 KB per bf16 half), K-major no-swizzle inside,
// kpad columns per row (a multiple of 32).
__host__ __device__ __forceinline__ size_t tiled_off(int prow, int k, int kpad) {
  const int rt = prow >> 7, r = prow & 127;
  return ((size_t)rt * (kpad / 32) + k / 32) * 8192u + (uint32_t)(r >> 3) * 512u + (uint32_t)((k % 32) >> 3) * 128u +
         (uint32_t)(r & 7) * 16u + (uint32_t)(k & 7) * 2u;
}

// bf16 split of an fp32 value: x ~= hi + lo with |x - hi - lo| <~ 2^-17 |x|.
__device__ __forceinline__ void split_bf16(float x, __nv_bfloat16& hi, __nv_bfloat16& lo) {
  hi = __float2bfloat16_rn(x);
  lo = __float2bfloat16_rn(x - __bfloat162float(hi));
}
// bf16 split of two fp32 values with integer operations only: hi is x
// rounded to bf16 (to nearest, ties away from zero: add half an ulp of the
// 16 dropped bits, then truncate), lo is x - hi (exact in fp32) truncated to
// bf16, so |x - hi - lo| <= 2^-17 |x|; the sign of lo follows the rounding
// of hi, so the truncation is not biased.  Returns the packed pairs, first
// element in the low half.  The conversion instructions are left out because
// they share the pipe that the tanh epilogues' exponentials and reciprocals
// need.
__device__ __forceinline__ void split_pair(float a, float b, uint32_t& hi, uint32_t& lo) {
  const uint32_t ah = (__float_as_uint(a) + 0x8000u) & 0xFFFF0000u;
  const uint32_t bh = (__float_as_uint(b) + 0x8000u) & 0xFFFF0000u;
  const float ar = a - __uint_as_float(ah);
  const float br = b - __uint_as_float(bh);
  hi = __byte_perm(ah, bh, 0x7632);
  lo = __byte_perm(__float_as_uint(ar), __float_as_uint(br), 0x7632);
}

// tanh from the exponential: 1 - 2 / (exp(2x) + 1).  Absolute error ~1e-7,
// saturates correctly at both ends (exp overflow -> 1, underflow -> -1).
__device__ __forceinline__ float tanh_fast(float x) { return 1.0f - __fdividef(2.0f, __expf(2.0f * x) + 1.0f); }

// Packs two bf16 into one 32-bit word (first element in the low half).
__device__ __forceinline__ uint32_t pack2(__nv_bfloat16 a, __nv_bfloat16 b) {
  return (uint32_t)__bfloat16_as_ushort(a) | ((uint32_t)__bfloat16_as_ushort(b) << 16);
}
}  // namespace umma
}  // namespace b200dp
