// quant.cu — int8 quantization, packing, dequantization and the synthetic
// weight generator (nn/quantize.go:42-229).
#include "../../include/tendo_synth.h"
#include "common.cuh"

namespace {

constexpr int kQuantThreads = 256;

__device__ __forceinline__ float block_max_256(float v, float* red) {
  v = warp_max(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();  // red may still be read by a previous call
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float r = red[0];
#pragma unroll
  for (int i = 1; i < kQuantThreads / 32; i++) r = fmaxf(r, red[i]);
  return r;
}

// One span (a row, or a group of a row) quantized exactly as
// quantizePerChannel / quantizePerGroup do: max |w| is order independent,
// scale = maxAbs / 127 (IEEE fp32 division), 1 when zero; q = clamp(
// round_half_away(w / scale)).  roundf is half away from zero, like Go's
// math.Round, and rounding an fp32 value through fp64 changes nothing.
__device__ __forceinline__ int8_t quant_one(float w, float scale) {
  float q = roundf(__fdiv_rn(w, scale));
  q = fminf(fmaxf(q, -128.0f), 127.0f);
  return (int8_t)(int)q;
}

__device__ __forceinline__ float scale_of(float max_abs) {
  float s = __fdiv_rn(max_abs, 127.0f);
  return s == 0.0f ? 1.0f : s;
}

// grid: (N, groups); one CTA per span.
__global__ void __launch_bounds__(kQuantThreads) quantize_kernel(int8_t* __restrict__ q, float* __restrict__ scale,
                                                                 const float* __restrict__ w, int64_t K,
                                                                 int64_t g) {
  __shared__ float red[kQuantThreads / 32];
  const int64_t n = blockIdx.x, j = blockIdx.y;
  const int64_t ng = K / g;
  const float* src = w + n * K + j * g;
  int8_t* dst = q + n * K + j * g;
  float m = 0.0f;
  for (int64_t i = threadIdx.x; i < g; i += kQuantThreads) m = fmaxf(m, fabsf(src[i]));
  m = block_max_256(m, red);
  const float s = scale_of(m);
  if (threadIdx.x == 0) scale[n * ng + j] = s;
  for (int64_t i = threadIdx.x; i < g; i += kQuantThreads) dst[i] = quant_one(src[i], s);
}

__global__ void pack_kernel(int8_t* __restrict__ q, const float* __restrict__ qf, int64_t n, int32_t* bad) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    float v = qf[i];
    bool ok = (v == rintf(v)) && v >= -128.0f && v <= 127.0f;
    if (!ok && bad) atomicAdd(bad, 1);
    q[i] = ok ? (int8_t)(int)v : (int8_t)0;
  }
}

__global__ void dequant_kernel(float* __restrict__ w, const int8_t* __restrict__ q, const float* __restrict__ scale,
                               int64_t N, int64_t K, int64_t g) {
  const int64_t total = N * K, ng = K / g;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    int64_t n = i / K, k = i - n * K;
    w[i] = __fmul_rn((float)q[i], scale[n * ng + k / g]);
  }
}

__global__ void synth_normal_kernel(float* __restrict__ w, int64_t total, uint64_t key, double std_) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x)
    w[i] = ts_normal_f32(key, (uint64_t)i, std_);
}

// One CTA per row: draws the row twice (max pass, quantize pass) instead of
// keeping an fp32 copy, so a 70B matrix never exists in fp32.
__global__ void __launch_bounds__(kQuantThreads) synth_quant_kernel(int8_t* __restrict__ q, float* __restrict__ scale,
                                                                    int64_t K, uint64_t key, double std_) {
  __shared__ float red[kQuantThreads / 32];
  const int64_t n = blockIdx.x;
  const uint64_t base = (uint64_t)(n * K);
  float m = 0.0f;
  for (int64_t i = threadIdx.x; i < K; i += kQuantThreads) m = fmaxf(m, fabsf(ts_normal_f32(key, base + i, std_)));
  m = block_max_256(m, red);
  const float s = scale_of(m);
  if (threadIdx.x == 0) scale[n] = s;
  for (int64_t i = threadIdx.x; i < K; i += kQuantThreads) q[n * K + i] = quant_one(ts_normal_f32(key, base + i, std_), s);
}

// A shard of a synthetic quantized matrix: local row n is global row
// row0 + n, drawn over all K columns (the per-channel scale needs the whole
// row) with the same element indices as the unsharded draw; columns
// [col0, col0 + cols) are kept.
__global__ void __launch_bounds__(kQuantThreads) synth_quant_shard_kernel(int8_t* __restrict__ q,
                                                                          float* __restrict__ scale, int64_t K,
                                                                          int64_t row0, int64_t col0, int64_t cols,
                                                                          uint64_t key, double std_) {
  __shared__ float red[kQuantThreads / 32];
  const int64_t n = blockIdx.x;
  const uint64_t base = (uint64_t)((row0 + n) * K);
  float m = 0.0f;
  for (int64_t i = threadIdx.x; i < K; i += kQuantThreads) m = fmaxf(m, fabsf(ts_normal_f32(key, base + i, std_)));
  m = block_max_256(m, red);
  const float s = scale_of(m);
  if (threadIdx.x == 0) scale[n] = s;
  for (int64_t i = threadIdx.x; i < cols; i += kQuantThreads)
    q[n * cols + i] = quant_one(ts_normal_f32(key, base + col0 + i, std_), s);
}

// The per-group form: block (n, j) quantizes kept group j (columns
// col0 + j g .. col0 + j g + g - 1 of global row row0 + n) with its own scale
// (nn/quantize.go:126-187); col0 is a multiple of g, so a shard keeps whole
// groups of the unsharded draw.
__global__ void __launch_bounds__(kQuantThreads) synth_quant_shard_grp_kernel(int8_t* __restrict__ q,
                                                                              float* __restrict__ scale, int64_t K,
                                                                              int64_t row0, int64_t col0,
                                                                              int64_t cols, int64_t g, uint64_t key,
                                                                              double std_) {
  __shared__ float red[kQuantThreads / 32];
  const int64_t n = blockIdx.x, j = blockIdx.y;
  const uint64_t base = (uint64_t)((row0 + n) * K + col0 + j * g);
  float m = 0.0f;
  for (int64_t i = threadIdx.x; i < g; i += kQuantThreads) m = fmaxf(m, fabsf(ts_normal_f32(key, base + i, std_)));
  m = block_max_256(m, red);
  const float s = scale_of(m);
  if (threadIdx.x == 0) scale[n * (cols / g) + j] = s;
  for (int64_t i = threadIdx.x; i < g; i += kQuantThreads)
    q[n * cols + j * g + i] = quant_one(ts_normal_f32(key, base + i, std_), s);
}

__global__ void synth_normal_offset_kernel(float* __restrict__ w, int64_t total, uint64_t first, uint64_t key,
                                           double std_) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x)
    w[i] = ts_normal_f32(key, first + (uint64_t)i, std_);
}

unsigned grid_for(int64_t n, int threads) {
  int64_t b = (n + threads - 1) / threads;
  int64_t cap = (int64_t)tb::sm_count() * 16;
  if (b > cap) b = cap;
  return (unsigned)(b < 1 ? 1 : b);
}

}  // namespace

extern "C" tb_status_t tb_quantize_i8_f32(int8_t* q, float* scale, const float* w, int64_t N, int64_t K,
                                          int64_t group_size, tb_stream_t stream) {
  TB_INJECT("tb_quantize_i8_f32");
  TB_REQUIRE(N >= 0 && K > 0 && group_size >= 0);
  const int64_t g = group_size == 0 ? K : group_size;
  TB_REQUIRE(K % g == 0);
  if (N == 0) return TB_SUCCESS;
  TB_REQUIRE(q && scale && w);
  TB_REQUIRE(N <= 0x7fffffff && K / g <= 65535);
  dim3 grid((unsigned)N, (unsigned)(K / g));
  quantize_kernel<<<grid, kQuantThreads, 0, (cudaStream_t)stream>>>(q, scale, w, K, g);
  return tb::check_launch("quantize_kernel");
}

extern "C" tb_status_t tb_pack_q_f32_to_i8(int8_t* q, const float* q_f32, int64_t n, int32_t* bad_count,
                                           tb_stream_t stream) {
  TB_INJECT("tb_pack_q_f32_to_i8");
  TB_REQUIRE(n >= 0);
  if (n == 0) return TB_SUCCESS;
  TB_REQUIRE(q && q_f32);
  pack_kernel<<<grid_for(n, 256), 256, 0, (cudaStream_t)stream>>>(q, q_f32, n, bad_count);
  return tb::check_launch("pack_kernel");
}

extern "C" tb_status_t tb_dequantize_i8_f32(float* w, const int8_t* q, const float* scale, int64_t N, int64_t K,
                                            int64_t group_size, tb_stream_t stream) {
  TB_INJECT("tb_dequantize_i8_f32");
  TB_REQUIRE(N >= 0 && K > 0 && group_size >= 0);
  const int64_t g = group_size == 0 ? K : group_size;
  TB_REQUIRE(K % g == 0);
  if (N == 0) return TB_SUCCESS;
  TB_REQUIRE(w && q && scale);
  dequant_kernel<<<grid_for(N * K, 256), 256, 0, (cudaStream_t)stream>>>(w, q, scale, N, K, g);
  return tb::check_launch("dequant_kernel");
}

extern "C" tb_status_t tb_synth_normal_f32(float* w, int64_t N, int64_t K, uint64_t seed, uint64_t stream_id,
                                           double std_, tb_stream_t stream) {
  TB_INJECT("tb_synth_normal_f32");
  TB_REQUIRE(N >= 0 && K >= 0);
  if (N * K == 0) return TB_SUCCESS;
  TB_REQUIRE(w);
  synth_normal_kernel<<<grid_for(N * K, 256), 256, 0, (cudaStream_t)stream>>>(w, N * K, ts_key(seed, stream_id),
                                                                               std_);
  return tb::check_launch("synth_normal_kernel");
}

extern "C" tb_status_t tb_synth_quantized_i8(int8_t* q, float* scale, int64_t N, int64_t K, uint64_t seed,
                                             uint64_t stream_id, double std_, tb_stream_t stream) {
  TB_INJECT("tb_synth_quantized_i8");
  TB_REQUIRE(N >= 0 && K > 0);
  if (N == 0) return TB_SUCCESS;
  TB_REQUIRE(q && scale && N <= 0x7fffffff);
  synth_quant_kernel<<<(unsigned)N, kQuantThreads, 0, (cudaStream_t)stream>>>(q, scale, K, ts_key(seed, stream_id),
                                                                               std_);
  return tb::check_launch("synth_quant_kernel");
}

namespace tb {

tb_status_t synth_quant_shard(int8_t* q, float* scale, int64_t rows, int64_t K, int64_t row0, int64_t col0,
                              int64_t cols, uint64_t seed, uint64_t stream_id, double std_, cudaStream_t st) {
  if (rows == 0) return TB_SUCCESS;
  synth_quant_shard_kernel<<<(unsigned)rows, kQuantThreads, 0, st>>>(q, scale, K, row0, col0, cols,
                                                                      ts_key(seed, stream_id), std_);
  return check_launch("synth_quant_shard_kernel");
}

tb_status_t synth_quant_shard_grp(int8_t* q, float* scale, int64_t rows, int64_t K, int64_t row0, int64_t col0,
                                  int64_t cols, int64_t group, uint64_t seed, uint64_t stream_id, double std_,
                                  cudaStream_t st) {
  if (rows == 0) return TB_SUCCESS;
  if (group <= 0 || cols % group != 0 || col0 % group != 0 || cols / group > 65535) return TB_ERROR_INVALID_ARGUMENT;
  synth_quant_shard_grp_kernel<<<dim3((unsigned)rows, (unsigned)(cols / group)), kQuantThreads, 0, st>>>(
      q, scale, K, row0, col0, cols, group, ts_key(seed, stream_id), std_);
  return check_launch("synth_quant_shard_grp_kernel");
}

tb_status_t synth_normal_rows(float* w, int64_t rows, int64_t K, int64_t row0, uint64_t seed, uint64_t stream_id,
                              double std_, cudaStream_t st) {
  if (rows * K == 0) return TB_SUCCESS;
  synth_normal_offset_kernel<<<grid_for(rows * K, 256), 256, 0, st>>>(w, rows * K, (uint64_t)(row0 * K),
                                                                      ts_key(seed, stream_id), std_);
  return check_launch("synth_normal_offset_kernel");
}

}  // namespace tb

extern "C" tb_status_t tb_synth_tokens_host(int64_t* ids, int64_t n, int64_t vocab, uint64_t seed) {
  TB_REQUIRE(n >= 0 && vocab > 0 && vocab <= 0xffffffffLL);
  if (n == 0) return TB_SUCCESS;
  TB_REQUIRE(ids);
  const uint64_t key = ts_key(seed, TS_STREAM_PROMPT);
  for (int64_t i = 0; i < n; i++) ids[i] = ts_uniform_int(key, (uint64_t)i, (uint32_t)vocab);
  return TB_SUCCESS;
}
