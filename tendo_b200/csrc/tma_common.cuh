// tma_common.cuh — device helpers shared by the TMA-fed kernels: mbarrier
// pipeline primitives (every wait bounded), 1-D bulk copies, the integer
// tensor-core MMA, consumer-only named barriers and L1-bypassing loads.
#pragma once

#include <stdint.h>

namespace tb {

__device__ __forceinline__ uint32_t smem_addr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbarrier_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbarrier_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbarrier_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}
// Waits for the completion of the phase with parity `parity`; after a bounded
// number of polls (well over a second) it counts a timeout in *err and
// returns, so a broken pipeline ends the kernel instead of hanging the GPU.
__device__ __forceinline__ void mbarrier_wait(uint64_t* bar, uint32_t parity, int* err) {
  const uint32_t a = smem_addr(bar);
  for (uint32_t it = 0; it < (1u << 24); it++) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
        : "=r"(done)
        : "r"(a), "r"(parity)
        : "memory");
    if (done) return;
  }
  if (err) atomicAdd(err, 1);
}
// Global -> shared bulk copy completing on `bar` (16-byte aligned, bytes % 16 == 0).
__device__ __forceinline__ void bulk_copy_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_addr(dst)),
               "l"(src), "r"(bytes), "r"(smem_addr(bar))
               : "memory");
}
// The same copy with an L2 cache policy (createpolicy) for the source lines.
__device__ __forceinline__ void bulk_copy_g2s_hint(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                                   uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::
          "r"(smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
      : "memory");
}
// Named barrier 1 over the first `nthreads` threads (the consumer warps).
__device__ __forceinline__ void named_sync(int nthreads) {
  asm volatile("bar.sync 1, %0;" ::"r"(nthreads) : "memory");
}
// D[16x8] += A[16x32] . B[32x8], s8 x s8 -> s32 (exact).
__device__ __forceinline__ void mma_s8_16832(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                             uint32_t b0, uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
// Loads that skip L1: data written by other CTAs earlier in the same launch
// must not be served from a stale L1 line.
__device__ __forceinline__ float ldcg(const float* p) { return __ldcg(p); }
__device__ __forceinline__ float4 ldcg4(const float* p) { return __ldcg(reinterpret_cast<const float4*>(p)); }

// Shared-memory row stride for `bytes`-long rows read with 16-byte lane
// loads at 16 t + 64 kb: 64 (mod 128) puts rows g and g + 1 on disjoint banks.
__host__ __device__ __forceinline__ int bank_stride(int bytes) { return (bytes % 128 == 0) ? bytes + 64 : bytes; }

// Chunk width of a row of `bytes` (a multiple of 64): the largest divisor of
// bytes / 64 blocks that keeps a chunk within 4096 bytes.
__host__ __device__ __forceinline__ int chunk_bytes(int bytes) {
  const int kb = bytes / 64;
  int d = 1;
  while (kb / d > 64 || kb % d != 0) d++;
  return 64 * (kb / d);
}

}  // namespace tb
