/*
 * oracle.c — TEST INFRASTRUCTURE ONLY: the CPU restatement of tendo's
 * int8 Llama path used to check the CUDA library and as the timed CPU
 * baseline.  Build: oracle/Makefile (gcc -O2 -ffp-contract=off -fopenmp).
 *
 * Citations are paths inside the tendo repository.
 */
#include "oracle.h"

#include <float.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#include "../include/tendo_synth.h"

#if defined(__FP_FAST_FMAF) && !defined(OR_ALLOW_FMA)
/* -ffp-contract=off is what matters; this only guards against -ffast-math. */
#endif

void or_set_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}

int or_get_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

/* ------------------------------------------------------------------------- */
/* nn/quantize.go:67-124 and :126-187.  maxAbs is a sequential fp32 max,
 * scale = maxAbs / 127 in fp32 (1 when zero), q = clamp(round(float64(w /
 * scale))) with the division in fp32 and Go's math.Round (half away from
 * zero), which C's round() also is. */
static void quantize_span(const float* w, int64_t n, float* q_f32, int8_t* q_i8, float* scale_out) {
  float max_abs = 0.0f;
  for (int64_t i = 0; i < n; i++) {
    float v = w[i];
    if (v < 0) v = -v;
    if (v > max_abs) max_abs = v;
  }
  float scale = max_abs / 127.0f;
  if (scale == 0) scale = 1.0f;
  *scale_out = scale;
  for (int64_t i = 0; i < n; i++) {
    float q = w[i] / scale;
    q = (float)round((double)q);
    if (q > 127) {
      q = 127;
    } else if (q < -128) {
      q = -128;
    }
    if (q_f32) q_f32[i] = q;
    if (q_i8) q_i8[i] = (int8_t)q;
  }
}

void or_quantize(const float* w, int64_t N, int64_t K, int64_t group, float* q_f32, int8_t* q_i8,
                 float* scale) {
  int64_t g = group > 0 ? group : K;
  int64_t ng = K / g;
#pragma omp parallel for schedule(static)
  for (int64_t n = 0; n < N; n++) {
    for (int64_t j = 0; j < ng; j++) {
      int64_t off = n * K + j * g;
      quantize_span(w + off, g, q_f32 ? q_f32 + off : NULL, q_i8 ? q_i8 + off : NULL,
                    scale + n * ng + j);
    }
  }
}

/* nn/quantize.go:191-229 */
void or_dequantize(const int8_t* q, const float* scale, int64_t N, int64_t K, int64_t group, float* w) {
  int64_t g = group > 0 ? group : K;
  int64_t ng = K / g;
#pragma omp parallel for schedule(static)
  for (int64_t n = 0; n < N; n++)
    for (int64_t k = 0; k < K; k++) w[n * K + k] = (float)q[n * K + k] * scale[n * ng + k / g];
}

/* ------------------------------------------------------------------------- */
/* Dequantize-then-MatMul.  Each output is a sequential fp32 sum over k of
 * x[m,k] * w[n,k], with w[n,k] = float(q) * scale rounded to fp32 first
 * (nn/quantize.go:204-212), products and sums rounded separately. */
void or_dequant_matmul(const float* x, const int8_t* q, const float* scale, int64_t M, int64_t N,
                       int64_t K, int64_t group, float* y) {
  int64_t g = group > 0 ? group : K;
  int64_t ng = K / g;
  int64_t nb = (N + 3) / 4;
#pragma omp parallel for schedule(static)
  for (int64_t b = 0; b < nb * M; b++) {
    int64_t m = b / nb;
    int64_t n0 = (b % nb) * 4;
    const float* xr = x + m * K;
    if (n0 + 4 <= N && group <= 0) {
      /* four rows at once: independent accumulators, identical per-row order */
      const int8_t* q0 = q + (n0 + 0) * K;
      const int8_t* q1 = q + (n0 + 1) * K;
      const int8_t* q2 = q + (n0 + 2) * K;
      const int8_t* q3 = q + (n0 + 3) * K;
      float s0 = scale[n0], s1 = scale[n0 + 1], s2 = scale[n0 + 2], s3 = scale[n0 + 3];
      float a0 = 0, a1 = 0, a2 = 0, a3 = 0;
      for (int64_t k = 0; k < K; k++) {
        float xv = xr[k];
        float w0 = (float)q0[k] * s0;
        float w1 = (float)q1[k] * s1;
        float w2 = (float)q2[k] * s2;
        float w3 = (float)q3[k] * s3;
        float p0 = xv * w0, p1 = xv * w1, p2 = xv * w2, p3 = xv * w3;
        a0 = a0 + p0;
        a1 = a1 + p1;
        a2 = a2 + p2;
        a3 = a3 + p3;
      }
      y[m * N + n0] = a0;
      y[m * N + n0 + 1] = a1;
      y[m * N + n0 + 2] = a2;
      y[m * N + n0 + 3] = a3;
    } else {
      for (int64_t n = n0; n < N && n < n0 + 4; n++) {
        const int8_t* qr = q + n * K;
        float acc = 0;
        for (int64_t k = 0; k < K; k++) {
          float w = (float)qr[k] * scale[n * ng + k / g];
          float p = xr[k] * w;
          acc = acc + p;
        }
        y[m * N + n] = acc;
      }
    }
  }
}

void or_matmul_nt(const float* a, const float* b, int64_t M, int64_t N, int64_t K, float* y) {
  int64_t nb = (N + 3) / 4;
#pragma omp parallel for schedule(static)
  for (int64_t t = 0; t < nb * M; t++) {
    int64_t m = t / nb;
    int64_t n0 = (t % nb) * 4;
    const float* ar = a + m * K;
    if (n0 + 4 <= N) {
      const float* b0 = b + (n0 + 0) * K;
      const float* b1 = b + (n0 + 1) * K;
      const float* b2 = b + (n0 + 2) * K;
      const float* b3 = b + (n0 + 3) * K;
      float a0 = 0, a1 = 0, a2 = 0, a3 = 0;
      for (int64_t k = 0; k < K; k++) {
        float av = ar[k];
        float p0 = av * b0[k], p1 = av * b1[k], p2 = av * b2[k], p3 = av * b3[k];
        a0 = a0 + p0;
        a1 = a1 + p1;
        a2 = a2 + p2;
        a3 = a3 + p3;
      }
      y[m * N + n0] = a0;
      y[m * N + n0 + 1] = a1;
      y[m * N + n0 + 2] = a2;
      y[m * N + n0 + 3] = a3;
    } else {
      for (int64_t n = n0; n < N; n++) {
        const float* br = b + n * K;
        float acc = 0;
        for (int64_t k = 0; k < K; k++) {
          float p = ar[k] * br[k];
          acc = acc + p;
        }
        y[m * N + n] = acc;
      }
    }
  }
}

void or_matmul_nn(const float* a, const float* b, int64_t M, int64_t N, int64_t K, float* y) {
#pragma omp parallel for schedule(static)
  for (int64_t t = 0; t < M * N; t++) {
    int64_t m = t / N, n = t % N;
    float acc = 0;
    for (int64_t k = 0; k < K; k++) {
      float p = a[m * K + k] * b[k * N + n];
      acc = acc + p;
    }
    y[t] = acc;
  }
}

/* cpu/backend.go:606-652 */
void or_rmsnorm(const float* x, const float* w, int64_t rows, int64_t d, float eps, float* out) {
  for (int64_t r = 0; r < rows; r++) {
    const float* xr = x + r * d;
    float sum_sq = 0;
    for (int64_t i = 0; i < d; i++) {
      float p = xr[i] * xr[i];
      sum_sq = sum_sq + p;
    }
    float ms = sum_sq / (float)d;
    float rms = (float)sqrt((double)(ms + eps));
    for (int64_t i = 0; i < d; i++) {
      float v = xr[i] / rms;
      if (w) v = v * w[i];
      out[r * d + i] = v;
    }
  }
}

/* cpu/backend.go:193-198 */
void or_silu(const float* x, int64_t n, float* out) {
  for (int64_t i = 0; i < n; i++) {
    float sig = (float)(1.0 / (1.0 + exp(-(double)x[i])));
    out[i] = x[i] * sig;
  }
}

/* cpu/backend.go:1690-1744 (non-log branch) */
void or_softmax(const float* x, int64_t rows, int64_t cols, float* out) {
  for (int64_t r = 0; r < rows; r++) {
    const float* xr = x + r * cols;
    float* o = out + r * cols;
    float max_v = -FLT_MAX;
    for (int64_t j = 0; j < cols; j++)
      if (xr[j] > max_v) max_v = xr[j];
    float sum = 0;
    for (int64_t j = 0; j < cols; j++) {
      float e = (float)exp((double)(xr[j] - max_v));
      o[j] = e;
      sum = sum + e;
    }
    for (int64_t j = 0; j < cols; j++) o[j] = o[j] / sum;
  }
}

/* nn/rope.go:22-52 */
void or_rope_tables(int dim, int max_seq, float base, float* cos_t, float* sin_t) {
  int half = dim / 2;
  float* inv = (float*)malloc(sizeof(float) * (size_t)half);
  for (int i = 0; i < half; i++) inv[i] = 1.0f / (float)pow((double)base, (double)(2 * i) / (double)dim);
  for (int p = 0; p < max_seq; p++) {
    for (int i = 0; i < half; i++) {
      float f = (float)p * inv[i];
      cos_t[(int64_t)p * half + i] = (float)cos((double)f);
      sin_t[(int64_t)p * half + i] = (float)sin((double)f);
    }
  }
  free(inv);
}

/* nn/rope.go:141-197: out0 = x0*cos - x1*sin, out1 = x0*sin + x1*cos,
 * each product and sum rounded to fp32 separately. */
void or_rope_apply(float* x, int64_t B, int64_t Hx, int64_t S, int64_t D, const float* cos_t,
                   const float* sin_t, int64_t pos_offset) {
  int64_t half = D / 2;
  for (int64_t bh = 0; bh < B * Hx; bh++) {
    for (int64_t s = 0; s < S; s++) {
      float* v = x + (bh * S + s) * D;
      const float* c = cos_t + (pos_offset + s) * half;
      const float* sn = sin_t + (pos_offset + s) * half;
      for (int64_t i = 0; i < half; i++) {
        float x0 = v[i], x1 = v[i + half];
        float x0c = x0 * c[i], x1s = x1 * sn[i];
        float x0s = x0 * sn[i], x1c = x1 * c[i];
        v[i] = x0c - x1s;
        v[i + half] = x0s + x1c;
      }
    }
  }
}

/* models/sampling.go:73-83 */
int64_t or_argmax(const float* v, int64_t n) {
  int64_t idx = 0;
  float best = v[0];
  for (int64_t i = 1; i < n; i++) {
    if (v[i] > best) {
      best = v[i];
      idx = i;
    }
  }
  return idx;
}

/* cpu/backend.go:1289-1339 (the Go code panics on an out-of-range id; this
 * returns -1 instead). */
int or_embedding(const float* table, int64_t V, int64_t d, const int64_t* ids, int64_t n, float* out) {
  for (int64_t i = 0; i < n; i++)
    if (ids[i] < 0 || ids[i] >= V) return -1;
  for (int64_t i = 0; i < n; i++) memcpy(out + i * d, table + ids[i] * d, sizeof(float) * (size_t)d);
  return 0;
}

/* The sampler's uniform draws (ts_uniform_f32): index offset .. offset + n - 1. */
void or_synth_uniform(uint64_t seed, uint64_t stream, uint64_t offset, int64_t n, float* out) {
  const uint64_t key = ts_key(seed, stream);
  for (int64_t i = 0; i < n; i++) out[i] = ts_uniform_f32(key, offset + (uint64_t)i);
}

void or_synth_normal(uint64_t seed, uint64_t stream, uint64_t offset, int64_t n, double std_, float* out) {
  uint64_t key = ts_key(seed, stream);
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; i++) out[i] = ts_normal_f32(key, offset + (uint64_t)i, std_);
}

void or_synth_tokens(uint64_t seed, int64_t n, int64_t vocab, int64_t* out) {
  uint64_t key = ts_key(seed, TS_STREAM_PROMPT);
  for (int64_t i = 0; i < n; i++) out[i] = ts_uniform_int(key, (uint64_t)i, (uint32_t)vocab);
}

/* ------------------------------------------------------------------------- */
/* Quantized Llama                                                            */
/* ------------------------------------------------------------------------- */
struct or_model {
  or_config c;
  int B;
  int64_t pos;
  int64_t n_out[7];
  int64_t n_in[7];
  int8_t* q[7];     /* per matrix: [layers][N][K] */
  float* scale[7];  /* [layers][N][K / group] (group 0: [layers][N]) */
  int64_t group;    /* 0: per output channel */
  int64_t ng[7];    /* scales per row */
  float* attn_norm; /* [layers][d] */
  float* mlp_norm;
  float* final_norm;
  float* embed;   /* [V][d] */
  float* lm_head; /* [V][d] */
  float* kc;      /* [layers][B][Hkv][max_seq][D] */
  float* vc;
  int kv_bf16;    /* values rounded to bf16 as they are appended */
  float* cos_t;
  float* sin_t;
};

static void* xcalloc(size_t n) {
  void* p = calloc(n, 1);
  return p;
}

or_model* or_model_create(const or_config* cfg, int batch, uint64_t seed, int generate) {
  return or_model_create_grouped(cfg, batch, seed, generate, 0);
}

/* QuantizeModel(m, groupSize) (models/llama/quantized.go:52-73): every
 * Linear quantized per group of `group` input columns (0: per channel). */
or_model* or_model_create_grouped(const or_config* cfg, int batch, uint64_t seed, int generate, int64_t group) {
  or_model* m = (or_model*)xcalloc(sizeof(or_model));
  if (!m) return NULL;
  m->c = *cfg;
  m->B = batch;
  m->group = group;
  int64_t d = cfg->dim, D = cfg->dim / cfg->heads;
  int64_t hq = (int64_t)cfg->heads * D, hkv = (int64_t)cfg->kv_heads * D, F = cfg->hidden;
  int64_t no[7] = {hq, hkv, hkv, d, F, F, d};
  int64_t ni[7] = {d, d, d, hq, d, d, F};
  int L = cfg->layers;
  int ok = 1;
  for (int i = 0; i < 7; i++) {
    m->n_out[i] = no[i];
    m->n_in[i] = ni[i];
    m->ng[i] = group > 0 ? ni[i] / group : 1;
    if (group > 0 && ni[i] % group != 0) ok = 0;
    m->q[i] = (int8_t*)malloc((size_t)L * no[i] * ni[i]);
    m->scale[i] = (float*)malloc(sizeof(float) * (size_t)L * no[i] * m->ng[i]);
    ok = ok && m->q[i] && m->scale[i];
  }
  m->attn_norm = (float*)malloc(sizeof(float) * (size_t)L * d);
  m->mlp_norm = (float*)malloc(sizeof(float) * (size_t)L * d);
  m->final_norm = (float*)malloc(sizeof(float) * (size_t)d);
  m->embed = (float*)malloc(sizeof(float) * (size_t)cfg->vocab * d);
  m->lm_head = (float*)malloc(sizeof(float) * (size_t)cfg->vocab * d);
  size_t kv = (size_t)L * batch * cfg->kv_heads * cfg->max_seq * D;
  m->kc = (float*)xcalloc(sizeof(float) * kv);
  m->vc = (float*)xcalloc(sizeof(float) * kv);
  m->cos_t = (float*)malloc(sizeof(float) * (size_t)cfg->max_seq * (D / 2));
  m->sin_t = (float*)malloc(sizeof(float) * (size_t)cfg->max_seq * (D / 2));
  ok = ok && m->attn_norm && m->mlp_norm && m->final_norm && m->embed && m->lm_head && m->kc && m->vc &&
       m->cos_t && m->sin_t;
  if (!ok) {
    or_model_free(m);
    return NULL;
  }
  for (int64_t i = 0; i < (int64_t)L * d; i++) m->attn_norm[i] = m->mlp_norm[i] = 1.0f;
  for (int64_t i = 0; i < d; i++) m->final_norm[i] = 1.0f;
  or_rope_tables((int)D, cfg->max_seq, cfg->rope_base, m->cos_t, m->sin_t);
  if (generate) {
    for (int l = 0; l < L; l++) {
      for (int i = 0; i < 7; i++) {
        uint64_t key = ts_key(seed, (uint64_t)l * TS_MATS + (uint64_t)i);
        int64_t N = no[i], K = ni[i];
#pragma omp parallel
        {
          float* row = (float*)malloc(sizeof(float) * (size_t)K);
#pragma omp for schedule(static)
          for (int64_t n = 0; n < N; n++) {
            for (int64_t k = 0; k < K; k++) row[k] = ts_normal_f32(key, (uint64_t)(n * K + k), 0.02);
            const int64_t ng = m->ng[i], g = K / ng;
            for (int64_t j = 0; j < ng; j++)
              quantize_span(row + j * g, g, NULL, m->q[i] + ((int64_t)l * N + n) * K + j * g,
                            m->scale[i] + ((int64_t)l * N + n) * ng + j);
          }
          free(row);
        }
      }
    }
    uint64_t ke = ts_key(seed, TS_STREAM_EMBED), kl = ts_key(seed, TS_STREAM_LMHEAD);
    int64_t vd = (int64_t)cfg->vocab * d;
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < vd; i++) {
      m->embed[i] = ts_normal_f32(ke, (uint64_t)i, 0.02);
      m->lm_head[i] = ts_normal_f32(kl, (uint64_t)i, 0.02);
    }
  }
  return m;
}

void or_model_free(or_model* m) {
  if (!m) return;
  for (int i = 0; i < 7; i++) {
    free(m->q[i]);
    free(m->scale[i]);
  }
  free(m->attn_norm);
  free(m->mlp_norm);
  free(m->final_norm);
  free(m->embed);
  free(m->lm_head);
  free(m->kc);
  free(m->vc);
  free(m->cos_t);
  free(m->sin_t);
  free(m);
}

int8_t* or_model_q(or_model* m, int layer, int mat) {
  return m->q[mat] + (int64_t)layer * m->n_out[mat] * m->n_in[mat];
}
float* or_model_scale(or_model* m, int layer, int mat) {
  return m->scale[mat] + (int64_t)layer * m->n_out[mat] * m->ng[mat];
}
float* or_model_norm(or_model* m, int layer, int which) {
  if (layer < 0) return m->final_norm;
  return (which ? m->mlp_norm : m->attn_norm) + (int64_t)layer * m->c.dim;
}
float* or_model_embed(or_model* m) { return m->embed; }
float* or_model_lm_head(or_model* m) { return m->lm_head; }
static int64_t kv_layer_elems(const or_model* m) {
  return (int64_t)m->B * m->c.kv_heads * m->c.max_seq * (m->c.dim / m->c.heads);
}
float* or_model_kcache(or_model* m, int layer) { return m->kc + layer * kv_layer_elems(m); }
float* or_model_vcache(or_model* m, int layer) { return m->vc + layer * kv_layer_elems(m); }
void or_model_reset(or_model* m) { m->pos = 0; }
void or_model_set_pos(or_model* m, int64_t pos) { m->pos = pos; }
void or_model_set_kv_bf16(or_model* m, int on) { m->kv_bf16 = on != 0; }

/* Round to nearest even at bit 16 of the fp32 pattern: the bf16 value with the
 * upper 16 bits (NaN stays NaN). */
float or_round_bf16(float x) {
  uint32_t u;
  memcpy(&u, &x, 4);
  if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x007FFFFFu)) {
    u |= 0x00400000u;
  } else {
    u += 0x7FFFu + ((u >> 16) & 1u);
  }
  u &= 0xFFFF0000u;
  memcpy(&x, &u, 4);
  return x;
}

/* dst[0..n) = src, rounded to bf16 when the model keeps a bf16 cache */
static void kv_store(const or_model* m, float* dst, const float* src, int64_t n) {
  if (!m->kv_bf16) {
    memcpy(dst, src, sizeof(float) * (size_t)n);
    return;
  }
  for (int64_t i = 0; i < n; i++) dst[i] = or_round_bf16(src[i]);
}
int64_t or_model_pos(const or_model* m) { return m->pos; }

/* models/llama/quantized.go:229-382 for one layer, batch-major activations
 * x[B*S, d].  Q/K/V projections, RoPE on q and k (nn/rope.go:102-197),
 * cache append of post-RoPE K and raw V (:282-299), GQA by kv head
 * h / (H/Hkv) (forward.go:345-370), scores = (q . k) then * (1/sqrt(D))
 * (:324-341), causal mask j <= i + (Sk - Sq) (forward.go:372-417), softmax
 * (:351), P.V (:358), then the O projection (:375). */
static void attention_layer(or_model* m, int l, const float* xn, int64_t S, float* out, float* scratch_q,
                            float* scratch_k, float* scratch_v, float* attn) {
  const or_config* c = &m->c;
  int64_t B = m->B, d = c->dim, H = c->heads, Hkv = c->kv_heads, D = d / H;
  int64_t P = m->pos, Sk = P + S, Ms = c->max_seq;
  or_dequant_matmul(xn, or_model_q(m, l, 0), or_model_scale(m, l, 0), B * S, H * D, d, m->group, scratch_q);
  or_dequant_matmul(xn, or_model_q(m, l, 1), or_model_scale(m, l, 1), B * S, Hkv * D, d, m->group, scratch_k);
  or_dequant_matmul(xn, or_model_q(m, l, 2), or_model_scale(m, l, 2), B * S, Hkv * D, d, m->group, scratch_v);
  /* permute [B,S,H,D] -> [B,H,S,D] */
  float* qh = (float*)malloc(sizeof(float) * (size_t)(B * H * S * D));
  float* kh = (float*)malloc(sizeof(float) * (size_t)(B * Hkv * S * D));
  for (int64_t b = 0; b < B; b++)
    for (int64_t s = 0; s < S; s++) {
      for (int64_t h = 0; h < H; h++)
        memcpy(qh + ((b * H + h) * S + s) * D, scratch_q + (b * S + s) * H * D + h * D, sizeof(float) * (size_t)D);
      for (int64_t h = 0; h < Hkv; h++)
        memcpy(kh + ((b * Hkv + h) * S + s) * D, scratch_k + (b * S + s) * Hkv * D + h * D,
               sizeof(float) * (size_t)D);
    }
  or_rope_apply(qh, B, H, S, D, m->cos_t, m->sin_t, P);
  or_rope_apply(kh, B, Hkv, S, D, m->cos_t, m->sin_t, P);
  float* kc = or_model_kcache(m, l);
  float* vc = or_model_vcache(m, l);
  for (int64_t b = 0; b < B; b++)
    for (int64_t h = 0; h < Hkv; h++)
      for (int64_t s = 0; s < S; s++) {
        kv_store(m, kc + ((b * Hkv + h) * Ms + P + s) * D, kh + ((b * Hkv + h) * S + s) * D, D);
        kv_store(m, vc + ((b * Hkv + h) * Ms + P + s) * D, scratch_v + (b * S + s) * Hkv * D + h * D, D);
      }
  float scale = 1.0f / (float)sqrt((double)D);
  int64_t rep = H / Hkv;
#pragma omp parallel
  {
    float* sc = (float*)malloc(sizeof(float) * (size_t)Sk);
    float* pr = (float*)malloc(sizeof(float) * (size_t)Sk);
#pragma omp for schedule(static) collapse(2)
    for (int64_t bh = 0; bh < B * H; bh++) {
      for (int64_t i = 0; i < S; i++) {
        int64_t b = bh / H, h = bh % H, hk = h / rep;
        const float* qv = qh + (bh * S + i) * D;
        const float* kb = kc + (b * Hkv + hk) * Ms * D;
        const float* vb = vc + (b * Hkv + hk) * Ms * D;
        for (int64_t j = 0; j < Sk; j++) {
          float acc = 0;
          for (int64_t e = 0; e < D; e++) {
            float p = qv[e] * kb[j * D + e];
            acc = acc + p;
          }
          acc = acc * scale;
          sc[j] = (j <= i + (Sk - S)) ? acc : -INFINITY;
        }
        or_softmax(sc, 1, Sk, pr);
        float* o = attn + (b * S + i) * H * D + h * D; /* permute back to [B,S,H*D] */
        for (int64_t e = 0; e < D; e++) {
          float acc = 0;
          for (int64_t j = 0; j < Sk; j++) {
            float p = pr[j] * vb[j * D + e];
            acc = acc + p;
          }
          o[e] = acc;
        }
      }
    }
    free(sc);
    free(pr);
  }
  or_dequant_matmul(attn, or_model_q(m, l, 3), or_model_scale(m, l, 3), B * S, d, H * D, m->group, out);
  free(qh);
  free(kh);
}

int or_model_forward(or_model* m, const int64_t* tokens, int64_t S, float* logits, float* last_logits,
                     float* hidden) {
  const or_config* c = &m->c;
  int64_t B = m->B, d = c->dim, H = c->heads, Hkv = c->kv_heads, D = d / H, F = c->hidden, V = c->vocab;
  int64_t rows = B * S;
  if (m->pos + S > c->max_seq) return -1;
  float* h = (float*)malloc(sizeof(float) * (size_t)(rows * d));
  float* xn = (float*)malloc(sizeof(float) * (size_t)(rows * d));
  float* t1 = (float*)malloc(sizeof(float) * (size_t)(rows * d));
  float* sq = (float*)malloc(sizeof(float) * (size_t)(rows * H * D));
  float* sk = (float*)malloc(sizeof(float) * (size_t)(rows * Hkv * D));
  float* sv = (float*)malloc(sizeof(float) * (size_t)(rows * Hkv * D));
  float* at = (float*)malloc(sizeof(float) * (size_t)(rows * H * D));
  float* g = (float*)malloc(sizeof(float) * (size_t)(rows * F));
  float* u = (float*)malloc(sizeof(float) * (size_t)(rows * F));
  int rc = 0;
  if (or_embedding(m->embed, V, d, tokens, rows, h) != 0) {
    rc = -1;
    goto done;
  }
  if (hidden) memcpy(hidden, h, sizeof(float) * (size_t)(rows * d));
  for (int l = 0; l < c->layers; l++) {
    /* forwardQuantizedLayer, models/llama/quantized.go:180-227 */
    or_rmsnorm(h, or_model_norm(m, l, 0), rows, d, c->eps, xn);
    attention_layer(m, l, xn, S, t1, sq, sk, sv, at);
    for (int64_t i = 0; i < rows * d; i++) h[i] = h[i] + t1[i];
    or_rmsnorm(h, or_model_norm(m, l, 1), rows, d, c->eps, xn);
    /* forwardQuantizedMLP, :385-417: down(silu(gate(x)) * up(x)) */
    or_dequant_matmul(xn, or_model_q(m, l, 4), or_model_scale(m, l, 4), rows, F, d, m->group, g);
    or_silu(g, rows * F, g);
    or_dequant_matmul(xn, or_model_q(m, l, 5), or_model_scale(m, l, 5), rows, F, d, m->group, u);
    for (int64_t i = 0; i < rows * F; i++) g[i] = g[i] * u[i];
    or_dequant_matmul(g, or_model_q(m, l, 6), or_model_scale(m, l, 6), rows, d, F, m->group, t1);
    for (int64_t i = 0; i < rows * d; i++) h[i] = h[i] + t1[i];
    if (hidden) memcpy(hidden + (int64_t)(l + 1) * rows * d, h, sizeof(float) * (size_t)(rows * d));
  }
  m->pos += S;
  /* final RMSNorm + fp32 lm_head, :154-172 */
  or_rmsnorm(h, m->final_norm, rows, d, c->eps, xn);
  if (logits) or_matmul_nt(xn, m->lm_head, rows, V, d, logits);
  if (last_logits) {
    for (int64_t b = 0; b < B; b++) {
      if (logits) {
        memcpy(last_logits + b * V, logits + ((b * S) + S - 1) * V, sizeof(float) * (size_t)V);
      } else {
        or_matmul_nt(xn + ((b * S) + S - 1) * d, m->lm_head, 1, V, d, last_logits + b * V);
      }
    }
  }
done:
  free(h);
  free(xn);
  free(t1);
  free(sq);
  free(sk);
  free(sv);
  free(at);
  free(g);
  free(u);
  return rc;
}

static void top2(const float* v, int64_t n, int64_t* idx, float* margin) {
  int64_t i1 = or_argmax(v, n);
  float second = -INFINITY;
  for (int64_t i = 0; i < n; i++)
    if (i != i1 && v[i] > second) second = v[i];
  *idx = i1;
  if (margin) *margin = v[i1] - second;
}

int or_model_generate_greedy(or_model* m, const int64_t* prompt, int64_t S, int64_t n_new, int64_t* out_tokens,
                             float* margins) {
  int64_t B = m->B, V = m->c.vocab;
  float* ll = (float*)malloc(sizeof(float) * (size_t)(B * V));
  int64_t* cur = (int64_t*)malloc(sizeof(int64_t) * (size_t)B);
  m->pos = 0;
  int rc = or_model_forward(m, prompt, S, NULL, ll, NULL);
  for (int64_t t = 0; t < n_new && rc == 0; t++) {
    for (int64_t b = 0; b < B; b++) {
      top2(ll + b * V, V, &cur[b], margins ? &margins[b * n_new + t] : NULL);
      out_tokens[b * n_new + t] = cur[b];
    }
    if (t + 1 < n_new) rc = or_model_forward(m, cur, 1, NULL, ll, NULL);
  }
  free(ll);
  free(cur);
  return rc;
}

int or_model_decode_step(or_model* m, const int64_t* tokens, int64_t* next) {
  int64_t B = m->B, V = m->c.vocab;
  float* ll = (float*)malloc(sizeof(float) * (size_t)(B * V));
  int rc = or_model_forward(m, tokens, 1, NULL, ll, NULL);
  for (int64_t b = 0; b < B && rc == 0; b++) next[b] = or_argmax(ll + b * V, V);
  free(ll);
  return rc;
}
