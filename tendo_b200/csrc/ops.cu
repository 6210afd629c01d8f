// ops.cu — the small glue kernels of the path: embedding gather, RMSNorm
// (optionally fused with the residual add), RoPE and the in-place KV append,
// SiLU / SwiGLU / Add, row argmax, and the decode-step tail.
#include <math.h>

#include <vector>

#include "../../include/tendo_synth.h"
#include "common.cuh"
#include "kernels.h"

namespace tb {
namespace {

unsigned grid_1d(int64_t n, int threads, int per_sm = 8) {
  int64_t b = (n + threads - 1) / threads;
  int64_t cap = (int64_t)sm_count() * per_sm;
  if (b > cap) b = cap;
  return (unsigned)(b < 1 ? 1 : b);
}

__global__ void embedding_kernel(float* out, const float* __restrict__ table, const int64_t* __restrict__ ids,
                                 int64_t n, int64_t vocab, int64_t dim, int32_t* bad) {
  pdl_wait();
  pdl_launch_dependents();
  for (int64_t r = blockIdx.x; r < n; r += gridDim.x) {
    const int64_t id = ids[r];
    const bool ok = id >= 0 && id < vocab;
    if (!ok && threadIdx.x == 0 && bad) atomicAdd(bad, 1);
    for (int64_t e = threadIdx.x; e < dim; e += blockDim.x) out[r * dim + e] = ok ? table[id * dim + e] : 0.f;
  }
}

// One CTA per row: x = in (+ resid), written to resid_out if given, then
// out = x / rms * w with rms = sqrt(mean(x^2) + eps) (cpu/backend.go:606-652).
__global__ void rmsnorm_kernel(float* out, float* resid_out, const float* in, const float* resid,
                               const float* __restrict__ w, int64_t d, float eps) {
  __shared__ float red[32];
  const int64_t r = blockIdx.x;
  const float* x = in + r * d;
  const float* rr = resid ? resid + r * d : nullptr;
  float ss = 0.f;
  for (int64_t i = threadIdx.x; i < d; i += blockDim.x) {
    float v = x[i];
    if (rr) v = __fadd_rn(v, rr[i]);
    ss = fmaf(v, v, ss);
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float s = 0.f;
  for (int i = 0; i < (int)(blockDim.x >> 5); i++) s += red[i];
  const float rms = __fsqrt_rn(__fadd_rn(__fdiv_rn(s, (float)d), eps));
  for (int64_t i = threadIdx.x; i < d; i += blockDim.x) {
    float v = x[i];
    if (rr) {
      v = __fadd_rn(v, rr[i]);
      if (resid_out) resid_out[r * d + i] = v;
    }
    float o = __fdiv_rn(v, rms);
    if (w) o = __fmul_rn(o, w[i]);
    out[r * d + i] = o;
  }
}

// x rows in the projection layout [B, S, Hx, D] with row stride ld (floats):
// rotate-half of every head at position pos + s (nn/rope.go:141-197).
__global__ void rope_rows_kernel(float* x, const float* __restrict__ cos_t, const float* __restrict__ sin_t,
                                 int64_t B, int64_t S, int64_t Hx, int64_t D, int64_t pos, int64_t ld) {
  const int64_t half = D / 2;
  const int64_t total = B * S * Hx * half;
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t i = t % half;
    const int64_t hh = (t / half) % Hx;
    const int64_t s = (t / (half * Hx)) % S;
    const int64_t b = t / (half * Hx * S);
    float* v = x + (b * S + s) * ld + hh * D;
    const float c = cos_t[(pos + s) * half + i], sn = sin_t[(pos + s) * half + i];
    const float x0 = v[i], x1 = v[i + half];
    v[i] = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, sn));
    v[i + half] = __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, c));
  }
}

// k, v [B, S, Hkv, D] (row stride ld) -> caches [B, Hkv, max_seq, D] at
// positions pos..pos+S-1, RoPE applied to k on the way; KT is the cache element.
template <typename KT>
__global__ void kv_append_rope_kernel(KT* kc, KT* vc, const float* __restrict__ k, const float* __restrict__ v,
                                      const float* __restrict__ cos_t, const float* __restrict__ sin_t, int64_t B,
                                      int64_t Hkv, int64_t S, int64_t D, int64_t pos, int64_t max_seq, int64_t ld) {
  const int64_t half = D / 2;
  const int64_t total = B * S * Hkv * half;
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t i = t % half;
    const int64_t hh = (t / half) % Hkv;
    const int64_t s = (t / (half * Hkv)) % S;
    const int64_t b = t / (half * Hkv * S);
    const float* ks = k + (b * S + s) * ld + hh * D;
    const float* vs = v + (b * S + s) * ld + hh * D;
    KT* kd = kc + ((b * Hkv + hh) * max_seq + pos + s) * D;
    KT* vd = vc + ((b * Hkv + hh) * max_seq + pos + s) * D;
    const float c = cos_t[(pos + s) * half + i], sn = sin_t[(pos + s) * half + i];
    const float x0 = ks[i], x1 = ks[i + half];
    kv_put(kd + i, __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, sn)));
    kv_put(kd + i + half, __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, c)));
    kv_put(vd + i, vs[i]);
    kv_put(vd + i + half, vs[i + half]);
  }
}

template <typename KT>
__global__ void qkv_rope_append_kernel(float* q, KT* kc, KT* vc, const float* __restrict__ qkv,
                                       const float* __restrict__ cos_t, const float* __restrict__ sin_t,
                                       const int64_t* pos_p, int64_t B, int64_t H, int64_t Hkv, int64_t D,
                                       int64_t max_seq) {
  const int64_t pos = *pos_p;
  const int64_t half = D / 2, NH = H + 2 * Hkv;
  const int64_t total = B * NH * half;
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t i = t % half;
    const int64_t hh = (t / half) % NH;
    const int64_t b = t / (half * NH);
    const float* src = qkv + (b * NH + hh) * D;
    const float x0 = src[i], x1 = src[i + half];
    if (hh < H + Hkv) {
      const float c = cos_t[pos * half + i], sn = sin_t[pos * half + i];
      const float r0 = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, sn));
      const float r1 = __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, c));
      if (hh < H) {
        float* d = q + (b * H + hh) * D;
        d[i] = r0;
        d[i + half] = r1;
      } else {
        KT* d = kc + ((b * Hkv + (hh - H)) * max_seq + pos) * D;
        kv_put(d + i, r0);
        kv_put(d + i + half, r1);
      }
    } else {
      KT* d = vc + ((b * Hkv + (hh - H - Hkv)) * max_seq + pos) * D;
      kv_put(d + i, x0);
      kv_put(d + i + half, x1);
    }
  }
}

__device__ __forceinline__ float silu_f(float g) { return g * (1.0f / (1.0f + expf(-g))); }

__global__ void silu_kernel(float* out, const float* in, int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    out[i] = silu_f(in[i]);
}

__global__ void silu_mul_kernel(float* out, const float* gate, const float* up, int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    out[i] = __fmul_rn(silu_f(gate[i]), up[i]);
}

// out[m, j] = silu(gu[m, j]) * gu[m, F + j]: rows of [gate | up] products.
__global__ void silu_mul_rows_kernel(float* out, const float* gu, int64_t B, int64_t F) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < B * F; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t m = i / F, j = i - m * F;
    out[i] = __fmul_rn(silu_f(gu[m * 2 * F + j]), gu[m * 2 * F + F + j]);
  }
}

__global__ void add_kernel(float* out, const float* a, const float* b, int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    out[i] = __fadd_rn(a[i], b[i]);
}

// One CTA per row; first index of the maximum (strict >, models/sampling.go:73-83).
// Greedy choice of a row as one orderable word: the logit's bits mapped to
// an order-preserving unsigned, then 2^32 - 1 - index, so the max over
// words is the largest logit with the lowest index on ties
// (models/sampling.go:73-83).
__device__ __forceinline__ unsigned long long packed_key(float v, int64_t idx) {
  uint32_t b = __float_as_uint(v);
  b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return ((unsigned long long)b << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)idx);
}

__global__ void argmax_keys_kernel(unsigned long long* keys, const float* x, int64_t n, int64_t v0) {
  __shared__ unsigned long long bk[8];
  const float* r = x + blockIdx.x * n;
  unsigned long long best = 0ull;
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
    const unsigned long long k = packed_key(r[i], v0 + i);
    best = k > best ? k : best;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long ok = __shfl_xor_sync(0xffffffffu, best, o);
    best = ok > best ? ok : best;
  }
  if ((threadIdx.x & 31) == 0) bk[threadIdx.x >> 5] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); w++) best = bk[w] > best ? bk[w] : best;
    atomicMax(keys + blockIdx.x, best);
  }
}

__global__ void argmax_kernel(int64_t* out, const float* x, int64_t n) {
  __shared__ float bv[32];
  __shared__ int64_t bi[32];
  const float* r = x + blockIdx.x * n;
  float best = -INFINITY;
  int64_t idx = -1;
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
    const float v = r[i];
    if (idx < 0 || v > best) {
      best = v;
      idx = i;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int64_t oi = __shfl_xor_sync(0xffffffffu, idx, o);
    if (oi >= 0 && (idx < 0 || ov > best || (ov == best && oi < idx))) {
      best = ov;
      idx = oi;
    }
  }
  if ((threadIdx.x & 31) == 0) {
    bv[threadIdx.x >> 5] = best;
    bi[threadIdx.x >> 5] = idx;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); w++) {
      if (bi[w] >= 0 && (idx < 0 || bv[w] > best || (bv[w] == best && bi[w] < idx))) {
        best = bv[w];
        idx = bi[w];
      }
    }
    out[blockIdx.x] = idx < 0 ? 0 : idx;
  }
}

__global__ void finish_step_kernel(unsigned long long* keys, int64_t* tokens, int64_t* history, int64_t* step,
                                   int64_t* pos, int M, int64_t hist_cap) {
  pdl_wait();
  pdl_launch_dependents();
  const int m = threadIdx.x;
  const int64_t st = *step;
  if (m < M) {
    const unsigned long long k = keys[m];
    const int64_t tok = (int64_t)(0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull));
    tokens[m] = tok;
    if (history && st < hist_cap) history[st * M + m] = tok;
    keys[m] = 0ull;
  }
  __syncthreads();
  if (m == 0) {
    *pos += 1;
    *step = st + 1;
  }
}

}  // namespace

tb_status_t embedding(float* out, const float* table, const int64_t* ids, int64_t n, int64_t vocab, int64_t dim,
                      int32_t* bad, cudaStream_t st, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid_1d(n, 1, 16));
  cfg.blockDim = dim3(256);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  cudaError_t e = cudaLaunchKernelEx(&cfg, embedding_kernel, out, table, ids, n, vocab, dim, bad);
  if (e != cudaSuccess) return cuda_fail(e, "embedding_kernel");
  return TB_SUCCESS;
}

tb_status_t rmsnorm(float* out, float* resid_out, const float* in, const float* resid, const float* w, int64_t rows,
                    int64_t d, float eps, cudaStream_t st) {
  if (rows == 0) return TB_SUCCESS;
  TB_REQUIRE(rows <= 0x7fffffff);
  rmsnorm_kernel<<<(unsigned)rows, 256, 0, st>>>(out, resid_out, in, resid, w, d, eps);
  return check_launch("rmsnorm_kernel");
}

tb_status_t kv_append_rope(void* kc, void* vc, const float* k, const float* v, const float* cos_t,
                           const float* sin_t, int64_t B, int64_t Hkv, int64_t S, int64_t D, int64_t pos,
                           int64_t max_seq, int64_t ld, cudaStream_t st, bool kv_bf16) {
  const int64_t total = B * S * Hkv * (D / 2);
  if (total == 0) return TB_SUCCESS;
  if (kv_bf16)
    kv_append_rope_kernel<<<grid_1d(total, 256), 256, 0, st>>>(static_cast<__nv_bfloat16*>(kc),
                                                               static_cast<__nv_bfloat16*>(vc), k, v, cos_t, sin_t, B,
                                                               Hkv, S, D, pos, max_seq, ld);
  else
    kv_append_rope_kernel<<<grid_1d(total, 256), 256, 0, st>>>(static_cast<float*>(kc), static_cast<float*>(vc), k, v,
                                                               cos_t, sin_t, B, Hkv, S, D, pos, max_seq, ld);
  return check_launch("kv_append_rope_kernel");
}

tb_status_t rope_rows(float* x, const float* cos_t, const float* sin_t, int64_t B, int64_t S, int64_t Hx, int64_t D,
                      int64_t pos, int64_t ld, cudaStream_t st) {
  const int64_t total = B * S * Hx * (D / 2);
  if (total == 0) return TB_SUCCESS;
  rope_rows_kernel<<<grid_1d(total, 256), 256, 0, st>>>(x, cos_t, sin_t, B, S, Hx, D, pos, ld);
  return check_launch("rope_rows_kernel");
}

tb_status_t silu_mul(float* out, const float* gate, const float* up, int64_t n, cudaStream_t st) {
  if (n == 0) return TB_SUCCESS;
  silu_mul_kernel<<<grid_1d(n, 256), 256, 0, st>>>(out, gate, up, n);
  return check_launch("silu_mul_kernel");
}

tb_status_t silu_mul_rows(float* out, const float* gu, int64_t B, int64_t F, cudaStream_t st) {
  if (B * F == 0) return TB_SUCCESS;
  silu_mul_rows_kernel<<<grid_1d(B * F, 256), 256, 0, st>>>(out, gu, B, F);
  return check_launch("silu_mul_rows_kernel");
}

tb_status_t argmax_rows(int64_t* out, const float* x, int64_t rows, int64_t n, cudaStream_t st) {
  if (rows == 0) return TB_SUCCESS;
  TB_REQUIRE(rows <= 0x7fffffff && n > 0);
  argmax_kernel<<<(unsigned)rows, 256, 0, st>>>(out, x, n);
  return check_launch("argmax_kernel");
}

tb_status_t qkv_rope_append(float* q, void* kc, void* vc, const float* qkv, const float* cos_t, const float* sin_t,
                            const int64_t* pos, int64_t B, int64_t H, int64_t Hkv, int64_t D, int64_t max_seq,
                            cudaStream_t st, bool kv_bf16) {
  const int64_t total = B * (H + 2 * Hkv) * (D / 2);
  if (total == 0) return TB_SUCCESS;
  const int64_t blocks = (total + 255) / 256 < 4096 ? (total + 255) / 256 : 4096;
  if (kv_bf16)
    qkv_rope_append_kernel<<<(unsigned)blocks, 256, 0, st>>>(q, static_cast<__nv_bfloat16*>(kc),
                                                             static_cast<__nv_bfloat16*>(vc), qkv, cos_t, sin_t, pos,
                                                             B, H, Hkv, D, max_seq);
  else
    qkv_rope_append_kernel<<<(unsigned)blocks, 256, 0, st>>>(q, static_cast<float*>(kc), static_cast<float*>(vc), qkv,
                                                             cos_t, sin_t, pos, B, H, Hkv, D, max_seq);
  return check_launch("qkv_rope_append_kernel");
}

// The sampler's draws for the token just generated (device step s counts it):
// u[b] = uniform(key, (s - 1) B + b).
__global__ void sample_uniforms_kernel(float* u, const int64_t* step, int64_t B, uint64_t key) {
  const int64_t b = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (b < B) u[b] = ts_uniform_f32(key, (uint64_t)((*step - 1) * B + b));
}

// The sampled tokens replace the step's greedy choice in the history.
__global__ void history_set_kernel(int64_t* history, const int64_t* tokens, const int64_t* step, int64_t B,
                                   int64_t hist_cap) {
  const int64_t b = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  const int64_t s = *step - 1;
  if (b < B && s >= 0 && s < hist_cap) history[s * B + b] = tokens[b];
}

tb_status_t sample_uniforms(float* u, const int64_t* step, int64_t B, uint64_t seed, cudaStream_t st) {
  sample_uniforms_kernel<<<(unsigned)((B + 127) / 128), 128, 0, st>>>(u, step, B, ts_key(seed, TS_STREAM_SAMPLE));
  return check_launch("sample_uniforms_kernel");
}

tb_status_t history_set(int64_t* history, const int64_t* tokens, const int64_t* step, int64_t B, int64_t hist_cap,
                        cudaStream_t st) {
  history_set_kernel<<<(unsigned)((B + 127) / 128), 128, 0, st>>>(history, tokens, step, B, hist_cap);
  return check_launch("history_set_kernel");
}

tb_status_t argmax_keys(unsigned long long* keys, const float* x, int64_t rows, int64_t n, int64_t v0,
                        cudaStream_t st) {
  if (rows == 0) return TB_SUCCESS;
  TB_REQUIRE(rows <= 0x7fffffff && n > 0 && v0 >= 0 && v0 + n <= 0x7fffffff);
  argmax_keys_kernel<<<(unsigned)rows, 256, 0, st>>>(keys, x, n, v0);
  return check_launch("argmax_keys_kernel");
}

tb_status_t finish_step(unsigned long long* keys, int64_t* tokens, int64_t* history, int64_t* step, int64_t* pos,
                        int M, int64_t hist_cap, cudaStream_t st, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1);
  cfg.blockDim = dim3(32 * ((M + 31) / 32));
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  cudaError_t e = cudaLaunchKernelEx(&cfg, finish_step_kernel, keys, tokens, history, step, pos, M, hist_cap);
  if (e != cudaSuccess) return cuda_fail(e, "finish_step_kernel");
  return TB_SUCCESS;
}

}  // namespace tb

// ---------------------------------------------------------------------------
// C ABI
// ---------------------------------------------------------------------------
extern "C" tb_status_t tb_rmsnorm_f32(float* out, const float* in, const float* weight, int64_t n, int64_t norm_size,
                                      float eps, tb_stream_t stream) {
  TB_INJECT("tb_rmsnorm_f32");
  TB_REQUIRE(n >= 0 && norm_size > 0);
  if (n == 0) return TB_SUCCESS;
  TB_REQUIRE(out && in);
  return tb::rmsnorm(out, nullptr, in, nullptr, weight, n, norm_size, eps, (cudaStream_t)stream);
}

extern "C" tb_status_t tb_add_rmsnorm_f32(float* out, float* residual_out, const float* in, const float* residual,
                                          const float* weight, int64_t n, int64_t norm_size, float eps,
                                          tb_stream_t stream) {
  TB_INJECT("tb_add_rmsnorm_f32");
  TB_REQUIRE(n >= 0 && norm_size > 0);
  if (n == 0) return TB_SUCCESS;
  TB_REQUIRE(out && in && residual);
  return tb::rmsnorm(out, residual_out, in, residual, weight, n, norm_size, eps, (cudaStream_t)stream);
}

extern "C" tb_status_t tb_silu_f32(float* out, const float* in, int64_t n, tb_stream_t stream) {
  TB_INJECT("tb_silu_f32");
  TB_REQUIRE(n >= 0);
  if (n == 0) return TB_SUCCESS;
  TB_REQUIRE(out && in);
  tb::silu_kernel<<<tb::grid_1d(n, 256), 256, 0, (cudaStream_t)stream>>>(out, in, n);
  return tb::check_launch("silu_kernel");
}

extern "C" tb_status_t tb_silu_mul_f32(float* out, const float* gate, const float* up, int64_t n,
                                       tb_stream_t stream) {
  TB_INJECT("tb_silu_mul_f32");
  TB_REQUIRE(n >= 0);
  if (n == 0) return TB_SUCCESS;
  TB_REQUIRE(out && gate && up);
  return tb::silu_mul(out, gate, up, n, (cudaStream_t)stream);
}

extern "C" tb_status_t tb_add_f32(float* out, const float* a, const float* b, int64_t n, tb_stream_t stream) {
  TB_INJECT("tb_add_f32");
  TB_REQUIRE(n >= 0);
  if (n == 0) return TB_SUCCESS;
  TB_REQUIRE(out && a && b);
  tb::add_kernel<<<tb::grid_1d(n, 256), 256, 0, (cudaStream_t)stream>>>(out, a, b, n);
  return tb::check_launch("add_kernel");
}

extern "C" tb_status_t tb_rope_tables_host(float* cos_t, float* sin_t, int dim, int max_seq, float base) {
  TB_REQUIRE(dim > 0 && dim % 2 == 0 && max_seq >= 0 && cos_t && sin_t);
  const int half = dim / 2;
  std::vector<float> inv(half);
  for (int i = 0; i < half; i++) inv[i] = 1.0f / (float)pow((double)base, (double)(2 * i) / (double)dim);
  for (int p = 0; p < max_seq; p++)
    for (int i = 0; i < half; i++) {
      const float f = (float)p * inv[i];
      cos_t[(int64_t)p * half + i] = (float)cos((double)f);
      sin_t[(int64_t)p * half + i] = (float)sin((double)f);
    }
  return TB_SUCCESS;
}

extern "C" tb_status_t tb_rope_apply_f32(float* out, const float* x, const float* cos_t, const float* sin_t,
                                         int64_t B, int64_t Hx, int64_t S, int64_t D, int64_t pos_offset,
                                         int64_t max_seq, tb_stream_t stream) {
  TB_INJECT("tb_rope_apply_f32");
  TB_REQUIRE(B >= 0 && Hx >= 0 && S >= 0 && D > 0 && D % 2 == 0 && pos_offset >= 0);
  TB_REQUIRE(pos_offset + S <= max_seq);  // nn/rope.go:109-111
  if (B * Hx * S == 0) return TB_SUCCESS;
  TB_REQUIRE(out && x && cos_t && sin_t);
  cudaStream_t st = (cudaStream_t)stream;
  if (out != x) TB_CUDA(cudaMemcpyAsync(out, x, sizeof(float) * B * Hx * S * D, cudaMemcpyDeviceToDevice, st));
  // [B, Hx, S, D] is the projection layout with B' = B * Hx "sequences" of one head.
  return tb::rope_rows(out, cos_t, sin_t, B * Hx, S, 1, D, pos_offset, D, st);
}

extern "C" tb_status_t tb_kv_append_rope_f32(float* kcache, float* vcache, const float* k, const float* v,
                                             const float* cos_t, const float* sin_t, int64_t B, int64_t Hkv,
                                             int64_t S, int64_t D, int64_t pos, int64_t max_seq,
                                             tb_stream_t stream) {
  TB_INJECT("tb_kv_append_rope_f32");
  TB_REQUIRE(B >= 0 && Hkv > 0 && S >= 0 && D > 0 && D % 2 == 0 && pos >= 0 && pos + S <= max_seq);
  if (B * S == 0) return TB_SUCCESS;
  TB_REQUIRE(kcache && vcache && k && v && cos_t && sin_t);
  return tb::kv_append_rope(kcache, vcache, k, v, cos_t, sin_t, B, Hkv, S, D, pos, max_seq, Hkv * D,
                            (cudaStream_t)stream);
}

extern "C" tb_status_t tb_embedding_f32(float* out, const float* table, const int64_t* ids, int64_t n, int64_t vocab,
                                        int64_t dim, int32_t* bad_count, tb_stream_t stream) {
  TB_INJECT("tb_embedding_f32");
  TB_REQUIRE(n >= 0 && vocab > 0 && dim > 0);
  if (n == 0) return TB_SUCCESS;
  TB_REQUIRE(out && table && ids);
  return tb::embedding(out, table, ids, n, vocab, dim, bad_count, (cudaStream_t)stream, false);
}

extern "C" tb_status_t tb_argmax_f32(int64_t* out_idx, const float* x, int64_t rows, int64_t n, tb_stream_t stream) {
  TB_INJECT("tb_argmax_f32");
  TB_REQUIRE(rows >= 0 && n > 0);
  if (rows == 0) return TB_SUCCESS;
  TB_REQUIRE(out_idx && x);
  return tb::argmax_rows(out_idx, x, rows, n, (cudaStream_t)stream);
}
