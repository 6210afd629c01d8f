// common.cuh — shared helpers of libtendo_b200 (status handling, launch
// checks, host-side fault injection, small device utilities).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/tendo_b200.h"

namespace tb {

// Records the CUDA error text for tb_get_last_cuda_error_string() and maps
// the error onto a status.
tb_status_t cuda_fail(cudaError_t e, const char* where);
// Records `msg` as the last error text (tb_get_last_cuda_error_string) and returns TB_ERROR_CUDA.
tb_status_t fail_message(const char* msg);

// Status of the launch just issued (cudaGetLastError).
tb_status_t check_launch(const char* where);

// Host-side fault injection: TENDO_B200_INJECT=<name>[,<name>...] makes the
// named entry points return TB_ERROR_INJECTED before touching the GPU.
bool injected(const char* name);

// Number of SMs of the current device (cached per device).
int sm_count();

inline bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

inline unsigned ceil_div(int64_t a, int64_t b) { return (unsigned)((a + b - 1) / b); }

// KV cache elements: fp32 (the reference's cache) or bf16 (a model option;
// rounded to nearest even on the way in, widened exactly on the way out).
__device__ __forceinline__ void kv_put(float* p, float v) { *p = v; }
__device__ __forceinline__ void kv_put(__nv_bfloat16* p, float v) { *p = __float2bfloat16_rn(v); }
__device__ __forceinline__ float kv_get(const float* p) { return *p; }
__device__ __forceinline__ float kv_get(const __nv_bfloat16* p) { return __bfloat162float(*p); }

}  // namespace tb

#define TB_INJECT(name)                                 \
  do {                                                  \
    if (tb::injected(name)) return TB_ERROR_INJECTED;   \
  } while (0)

#define TB_REQUIRE(cond)                                \
  do {                                                  \
    if (!(cond)) return TB_ERROR_INVALID_ARGUMENT;      \
  } while (0)

#define TB_CUDA(call)                                   \
  do {                                                  \
    cudaError_t e_ = (call);                            \
    if (e_ != cudaSuccess) return tb::cuda_fail(e_, #call); \
  } while (0)

#define TB_TRY(call)                                    \
  do {                                                  \
    tb_status_t s_ = (call);                            \
    if (s_ != TB_SUCCESS) return s_;                    \
  } while (0)

// ---------------------------------------------------------------------------
// Device utilities
// ---------------------------------------------------------------------------
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Streaming 16-byte load that bypasses L1 (weights are read once per pass).
__device__ __forceinline__ int4 ld_stream_v4(const void* p) {
  int4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.s32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// Four signed bytes of w as exact fp32 values.  Each byte is biased to
// unsigned (xor 0x80), placed into the mantissa of 2^23 with a byte permute
// and the bias 2^23 + 128 is subtracted: one PRMT and one FADD per value.
__device__ __forceinline__ void i8x4_to_f32(uint32_t w, float& a, float& b, float& c, float& d) {
  const uint32_t u = w ^ 0x80808080u;
  const uint32_t hi = 0x4B000000u;
  a = __uint_as_float(__byte_perm(u, hi, 0x7650)) - 8388736.0f;
  b = __uint_as_float(__byte_perm(u, hi, 0x7651)) - 8388736.0f;
  c = __uint_as_float(__byte_perm(u, hi, 0x7652)) - 8388736.0f;
  d = __uint_as_float(__byte_perm(u, hi, 0x7653)) - 8388736.0f;
}

// Bulk L2 prefetch through the TMA unit: `bytes` (a multiple of 16) from a
// 16-byte aligned global address, no registers held while it is in flight.
__device__ __forceinline__ void prefetch_l2_bulk(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// Programmatic dependent launch: wait for the preceding grid's memory and
// let the next grid start launching.  Both are no-ops when the kernel was not
// launched with the programmatic-serialization attribute.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
