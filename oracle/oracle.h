/*
 * oracle.h — TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C restatement of the tendo (github.com/zoobzio/tendo) CPU path for
 * the int8 Llama decode hot path.  It is the checker for the CUDA library and
 * the CPU baseline that bench.py times; the library itself never links,
 * loads or calls anything in this directory.
 *
 * Arithmetic follows the Go code line by line (fp32 where Go uses float32,
 * fp64 where Go converts to float64, mul-then-add with no fused multiply-add).
 * GEMM order: gonum blas32.Gemm (v0.16.0, not vendored in the reference)
 * is restated as a sequential fp32 sum over k per output element, which is
 * what its serial kernel does for NoTrans x NoTrans (c[i,j] += a[i,l]*b[l,j],
 * l ascending).  That order is not pinned by any reference test.
 *
 * Every function is bit-identical whatever the thread count: threads split
 * output elements, never a sum.
 */
#ifndef TENDO_ORACLE_H
#define TENDO_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

void or_set_threads(int n);
int or_get_threads(void);

/* nn/quantize.go:67-124 (per channel) and :126-187 (per group, group > 0).
 * q_f32 receives the reference's float32-coded integers, q_i8 the same values
 * as int8; either may be NULL.  scale is [N] or [N, K/group]. */
void or_quantize(const float* w, int64_t N, int64_t K, int64_t group,
                 float* q_f32, int8_t* q_i8, float* scale);

/* nn/quantize.go:191-229: w = q * scale (fp32 multiply). */
void or_dequantize(const int8_t* q, const float* scale, int64_t N, int64_t K,
                   int64_t group, float* w);

/* y[M,N] = x[M,K] @ dequantize(q)^T — the reference CPU contract of
 * QuantizedLinearBackend.DequantizeMatmul (nn/quantize.go:251-258): dequantize
 * (nn/quantize.go:204-222) then cpu MatMul (cpu/backend.go:1976-2021). */
void or_dequant_matmul(const float* x, const int8_t* q, const float* scale,
                       int64_t M, int64_t N, int64_t K, int64_t group, float* y);

/* y[M,N] = a[M,K] @ b[N,K]^T in fp32 (the fp32 lm_head, models/llama/quantized.go:164-172). */
void or_matmul_nt(const float* a, const float* b, int64_t M, int64_t N, int64_t K, float* y);

/* y[M,N] = a[M,K] @ b[K,N] (cpu MatMul of two row-major matrices). */
void or_matmul_nn(const float* a, const float* b, int64_t M, int64_t N, int64_t K, float* y);

/* cpu/backend.go:606-652 (weight may be NULL). */
void or_rmsnorm(const float* x, const float* w, int64_t rows, int64_t d, float eps, float* out);

/* cpu/backend.go:193-198. */
void or_silu(const float* x, int64_t n, float* out);

/* cpu/backend.go:1690-1744 (softmax over the last dim of [rows, cols]). */
void or_softmax(const float* x, int64_t rows, int64_t cols, float* out);

/* nn/rope.go:22-52: cos/sin tables [max_seq, dim/2]. */
void or_rope_tables(int dim, int max_seq, float base, float* cos_t, float* sin_t);

/* nn/rope.go:141-197: rotate-half of x[B, Hx, S, D] (contiguous, in place)
 * at positions pos_offset .. pos_offset+S-1. */
void or_rope_apply(float* x, int64_t B, int64_t Hx, int64_t S, int64_t D,
                   const float* cos_t, const float* sin_t, int64_t pos_offset);

/* models/sampling.go:73-83: first index of the maximum. */
int64_t or_argmax(const float* v, int64_t n);

/* Embedding (cpu/backend.go:1289-1339): out[i, :] = table[ids[i], :].
 * Returns -1 (and writes nothing) if an id is outside [0, V). */
int or_embedding(const float* table, int64_t V, int64_t d, const int64_t* ids, int64_t n, float* out);

/* Synthetic inputs (include/tendo_synth.h): out[i] = N(0, std) draw
 * `offset + i` of (seed, stream); tokens uniform in [0, vocab). */
void or_synth_uniform(uint64_t seed, uint64_t stream, uint64_t offset, int64_t n, float* out);
void or_synth_normal(uint64_t seed, uint64_t stream, uint64_t offset, int64_t n, double std_, float* out);
void or_synth_tokens(uint64_t seed, int64_t n, int64_t vocab, int64_t* out);

/* ---------------------------------------------------------------------------
 * Quantized Llama (models/llama/quantized.go), batch of B sequences in lockstep
 * --------------------------------------------------------------------------- */
typedef struct {
  int vocab, dim, layers, heads, kv_heads, hidden, max_seq;
  float rope_base, eps;
} or_config;

typedef struct or_model or_model;

/* Allocates a model with weights drawn from the shared synthetic generator
 * (N(0, 0.02) fp32, seed) and quantized per channel (nn/quantize.go:67-124);
 * gains are 1.0, embedding and lm_head stay fp32.  With generate == 0 the
 * arrays are left zero for the caller to fill. */
or_model* or_model_create(const or_config* cfg, int batch, uint64_t seed, int generate);
/* The same model with every Linear quantized per group of `group` input
 * columns (QuantizeModel(m, groupSize), models/llama/quantized.go:52-73);
 * scales [N][K / group]; group 0 is per channel. */
or_model* or_model_create_grouped(const or_config* cfg, int batch, uint64_t seed, int generate, int64_t group);
void or_model_free(or_model* m);

/* Pointers into the model's arrays (mat: 0..6 = q,k,v,o,gate,up,down). */
int8_t* or_model_q(or_model* m, int layer, int mat);
float* or_model_scale(or_model* m, int layer, int mat);
float* or_model_norm(or_model* m, int layer, int which); /* 0 attn, 1 mlp; layer == -1: final */
float* or_model_embed(or_model* m);
float* or_model_lm_head(or_model* m);
float* or_model_kcache(or_model* m, int layer); /* [B, Hkv, max_seq, D] */
float* or_model_vcache(or_model* m, int layer);

void or_model_reset(or_model* m); /* empties the KV cache */
void or_model_set_pos(or_model* m, int64_t pos); /* cache length (timing samples) */
/* on != 0: K and V are rounded to bf16 (nearest even) as they are appended,
 * the restatement of a bf16 KV cache; off (default): the reference's fp32 cache. */
void or_model_set_kv_bf16(or_model* m, int on);
float or_round_bf16(float x); /* fp32 -> nearest-even bf16 value, as fp32 */
int64_t or_model_pos(const or_model* m);

/* QuantizedModel.Forward (models/llama/quantized.go:125-178) over tokens[B, S]
 * appended at the current cache position.  logits: [B, S, V] (or NULL);
 * last_logits: [B, V] (or NULL); hidden: [layers + 1, B, S, d] residual stream
 * after the embedding and after each layer (or NULL).  Returns 0, or -1 on a
 * bad token id / position overflow. */
int or_model_forward(or_model* m, const int64_t* tokens, int64_t S, float* logits,
                     float* last_logits, float* hidden);

/* GenerateGreedy (models/llama/generate.go:99-150) for B sequences: prefill
 * with prompt[B, S], then n_new greedy steps.  out_tokens [B, n_new];
 * margins [B, n_new] (top-1 minus top-2 logit, may be NULL).  Returns 0 / -1. */
int or_model_generate_greedy(or_model* m, const int64_t* prompt, int64_t S, int64_t n_new,
                             int64_t* out_tokens, float* margins);

/* One decode step for all B sequences (tokens[B]); next[B] gets the greedy
 * token.  Used for bounded CPU timing samples. */
int or_model_decode_step(or_model* m, const int64_t* tokens, int64_t* next);

#ifdef __cplusplus
}
#endif
#endif
