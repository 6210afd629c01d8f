// capi.cu — status strings, error capture, host-side fault injection and the
// DequantizeMatmul / MatMul dispatch of the C ABI.
#include <stdlib.h>
#include <string.h>

#include <mutex>
#include <string>

#include "common.cuh"
#include "kernels.h"

namespace tb {

namespace {
thread_local std::string g_last_cuda_error;
}

tb_status_t cuda_fail(cudaError_t e, const char* where) {
  g_last_cuda_error = std::string(where) + ": " + cudaGetErrorName(e) + ": " + cudaGetErrorString(e);
  if (e == cudaErrorMemoryAllocation) return TB_ERROR_OUT_OF_MEMORY;
  return TB_ERROR_CUDA;
}

tb_status_t fail_message(const char* msg) {
  g_last_cuda_error = msg;
  return TB_ERROR_CUDA;
}

tb_status_t check_launch(const char* where) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, where);
  return TB_SUCCESS;
}

bool injected(const char* name) {
  const char* env = getenv("TENDO_B200_INJECT");
  if (!env || !*env) return false;
  const size_t n = strlen(name);
  for (const char* p = env; *p;) {
    const char* comma = strchr(p, ',');
    const size_t len = comma ? (size_t)(comma - p) : strlen(p);
    if (len == n && strncmp(p, name, n) == 0) return true;
    if (len == 3 && strncmp(p, "all", 3) == 0) return true;
    if (!comma) break;
    p = comma + 1;
  }
  return false;
}

int sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cached[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cached[dev] = n;
  }
  return cached[dev];
}

}  // namespace tb

extern "C" const char* tb_get_error_string(tb_status_t status) {
  switch (status) {
    case TB_SUCCESS: return "success";
    case TB_ERROR_INVALID_ARGUMENT: return "invalid argument";
    case TB_ERROR_CUDA: return "CUDA error";
    case TB_ERROR_NOT_SUPPORTED: return "not supported";
    case TB_ERROR_OUT_OF_MEMORY: return "out of memory";
    case TB_ERROR_TIMEOUT: return "device-side wait timed out";
    case TB_ERROR_INJECTED: return "injected failure";
  }
  return "unknown status";
}

extern "C" const char* tb_get_last_cuda_error_string(void) { return tb::g_last_cuda_error.c_str(); }

extern "C" int tb_version(void) { return 100; }

namespace {

int gemm_planes(tb_gemm_mode_t mode) { return mode == TB_GEMM_I8X2 ? 2 : 3; }

size_t dqmm_workspace(int64_t M, int64_t N, int64_t K, int64_t group_size, tb_gemm_mode_t mode) {
  if (mode == TB_GEMM_SIMT) return 0;
  if (M <= 32) {  // the decode regime of the C ABI (per-group: groups of a multiple of 128)
    if (K % 128 != 0 || (group_size > 0 && group_size % 128 != 0)) return 0;
    return tb::gemv_tc_zeroed_bytes(M, N, K) + tb::gemv_tc_scratch_bytes(M, N, K, group_size);
  }
  // per-group: groups of a multiple of 128 and at most 128 groups per row
  if (group_size > 0 && (group_size % 128 != 0 || K % group_size != 0 || K / group_size > 128)) return 0;
  return tb::gemm_tc_workspace(M, K, gemm_planes(mode));
}

// Library-owned buffers per device for the entry points without a workspace
// argument: kind 0 is plain scratch, kind 1 is kept zero between calls (the
// GEMV's split-tile counters and sums).  Allocated on first use, grown (after
// a device synchronisation) when a larger call arrives.
std::mutex g_arena_mu;
struct ArenaSlot {
  void* p = nullptr;
  size_t n = 0;
};
ArenaSlot g_arena[2][64];

tb_status_t arena_get(int kind, size_t bytes, void** out) {
  int dev = 0;
  TB_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return TB_ERROR_NOT_SUPPORTED;
  std::lock_guard<std::mutex> lk(g_arena_mu);
  ArenaSlot& a = g_arena[kind][dev];
  if (a.n < bytes) {
    if (a.p) {
      TB_CUDA(cudaDeviceSynchronize());
      TB_CUDA(cudaFree(a.p));
      a.p = nullptr;
      a.n = 0;
    }
    const size_t want = bytes + bytes / 4;
    TB_CUDA(cudaMalloc(&a.p, want));
    if (kind == 1) TB_CUDA(cudaMemset(a.p, 0, want));
    a.n = want;
  }
  *out = a.p;
  return TB_SUCCESS;
}

tb_status_t dqmm(float* out, const float* x, const int8_t* q, const float* scale, int64_t M, int64_t N, int64_t K,
                 int64_t group_size, tb_gemm_mode_t mode, void* ws, size_t ws_bytes, bool arena, cudaStream_t st) {
  if (M <= 32) {
    // up to 5 rows with per-channel scales: one weight stream through a
    // shared-memory ring, no workspace
    if (mode != TB_GEMM_SIMT && group_size == 0 && tb::gemv_ring_ok(x, q, M, N, K))
      return tb::gemv_ring(out, x, q, scale, nullptr, (int)M, (int)N, (int)K, st);
    const size_t gneed = dqmm_workspace(M, N, K, group_size, mode);
    if (gneed > 0 && tb::gemv_tc_ok(q, M, N, K, group_size) && (uintptr_t)x % 16 == 0) {
      const size_t zb = tb::gemv_tc_zeroed_bytes(M, N, K), sb = tb::gemv_tc_scratch_bytes(M, N, K, group_size);
      void *zero = nullptr, *scratch = nullptr;
      if (arena) {
        TB_TRY(arena_get(1, zb, &zero));
        if (sb) TB_TRY(arena_get(0, sb, &scratch));
      } else {
        TB_REQUIRE(ws && ws_bytes >= gneed);
        zero = ws;
        scratch = static_cast<unsigned char*>(ws) + zb;
      }
      return tb::gemv_tc(out, x, q, scale, nullptr, (int)M, (int)N, (int)K, zero, !arena, scratch, st, nullptr, 0.f,
                         (int)group_size);
    }
    if (!arena && gneed > 0) TB_REQUIRE(ws && ws_bytes >= gneed);
    if (group_size == 0 && tb::gemv_fast_ok(x, q, K))
      return tb::gemv_plain(out, x, q, scale, nullptr, (int)M, (int)N, (int)K, nullptr, 0.f, st, false);
    return tb::gemv_generic(out, x, q, scale, (int)M, (int)N, (int)K, group_size > 0 ? (int)group_size : (int)K, st);
  }
  const size_t need = dqmm_workspace(M, N, K, group_size, mode);
  const bool tc = group_size > 0 ? tb::gemm_tc_grp_ok(q, M, N, K, group_size) : tb::gemm_tc_ok(q, M, N, K);
  if (need > 0 && tc && (uintptr_t)x % 16 == 0) {
    if (arena) {
      TB_TRY(arena_get(0, need, &ws));
    } else {
      TB_REQUIRE(ws && ws_bytes >= need);
    }
    if (group_size > 0)
      return tb::gemm_tc_grp(out, x, q, scale, nullptr, (int)M, (int)N, (int)K, (int)group_size, gemm_planes(mode), ws,
                             st);
    return tb::gemm_tc(out, x, q, scale, nullptr, (int)M, (int)N, (int)K, gemm_planes(mode), ws, st);
  }
  if (!arena && need > 0) TB_REQUIRE(ws && ws_bytes >= need);
  return tb::gemm_simt_i8(out, x, q, scale, nullptr, (int)M, (int)N, (int)K, (int)group_size, st);
}

}  // namespace

#define TB_DQMM_ARGS_CHECK()                                                 \
  do {                                                                        \
    TB_REQUIRE(M >= 0 && N >= 0 && K > 0 && group_size >= 0);                \
    TB_REQUIRE(group_size == 0 || K % group_size == 0);                       \
    TB_REQUIRE(M <= 0x7fffffff && N <= 0x7fffffff && K <= 0x7fffffff);        \
    TB_REQUIRE(mode == TB_GEMM_I8X3 || mode == TB_GEMM_I8X2 || mode == TB_GEMM_SIMT); \
  } while (0)

extern "C" size_t tb_dequant_matmul_workspace_size(int64_t M, int64_t N, int64_t K, int64_t group_size,
                                                   tb_gemm_mode_t mode) {
  if (M < 0 || N < 0 || K <= 0 || group_size < 0) return 0;
  return dqmm_workspace(M, N, K, group_size, mode);
}

extern "C" tb_status_t tb_dequant_matmul_i8f32_ws(float* out, const float* x, const int8_t* q, const float* scale,
                                                  int64_t M, int64_t N, int64_t K, int64_t group_size,
                                                  tb_gemm_mode_t mode, void* workspace, size_t workspace_bytes,
                                                  tb_stream_t stream) {
  TB_INJECT("tb_dequant_matmul_i8f32");
  TB_DQMM_ARGS_CHECK();
  if (M == 0 || N == 0) return TB_SUCCESS;
  TB_REQUIRE(out && x && q && scale);
  return dqmm(out, x, q, scale, M, N, K, group_size, mode, workspace, workspace_bytes, false, (cudaStream_t)stream);
}

extern "C" tb_status_t tb_dequant_matmul_i8f32_mode(float* out, const float* x, const int8_t* q, const float* scale,
                                                    int64_t M, int64_t N, int64_t K, int64_t group_size,
                                                    tb_gemm_mode_t mode, tb_stream_t stream) {
  TB_INJECT("tb_dequant_matmul_i8f32");
  TB_DQMM_ARGS_CHECK();
  if (M == 0 || N == 0) return TB_SUCCESS;
  TB_REQUIRE(out && x && q && scale);
  return dqmm(out, x, q, scale, M, N, K, group_size, mode, nullptr, 0, true, (cudaStream_t)stream);
}

extern "C" tb_status_t tb_dequant_matmul_i8f32(float* out, const float* x, const int8_t* q, const float* scale,
                                               int64_t M, int64_t N, int64_t K, int64_t group_size,
                                               tb_stream_t stream) {
  return tb_dequant_matmul_i8f32_mode(out, x, q, scale, M, N, K, group_size, TB_GEMM_I8X3, stream);
}

extern "C" tb_status_t tb_matmul_nt_f32(float* out, const float* a, const float* b, int64_t M, int64_t N, int64_t K,
                                        tb_stream_t stream) {
  TB_INJECT("tb_matmul_nt_f32");
  TB_REQUIRE(M >= 0 && N >= 0 && K > 0);
  TB_REQUIRE(M <= 0x7fffffff && N <= 0x7fffffff && K <= 0x7fffffff);
  if (M == 0 || N == 0) return TB_SUCCESS;
  TB_REQUIRE(out && a && b);
  return tb::gemm_f32_nt(out, a, b, (int)M, (int)N, (int)K, (cudaStream_t)stream);
}
