// engine.cu — the host side of the path in C++: tendo's QuantizedModel
// (models/llama/quantized.go:13-477) over the kernels of this library.
//
// Layout in HBM (one engine per GPU):
//   wqkv  [L][(H + 2 Hkv) D][d] int8   — q, k, v rows concatenated per layer
//   sqkv  [L][(H + 2 Hkv) D]    fp32   — their per-channel scales
//   wo    [L][d][H D], wgate/wup [L][F][d], wdown [L][d][F] int8 (+ scales)
//   embed, lm_head [V][d] fp32 (the reference keeps both fp32)
//   kc, vc [L][B][Hkv][max_seq][D] fp32 (the reference's cache layout,
//          preallocated; the Cat append becomes an in-place write)
//
// Prefill (and any batch too wide for the fused decode kernels) runs layer
// by layer: RMSNorm, the GEMM projections, RoPE + cache append, tiled causal
// attention, residual adds.  Decode runs one CUDA graph per step: embedding,
// then per layer [fused RMSNorm+QKV+RoPE+append GEMV] -> [split-K attention
// + combine] -> [O GEMV + residual] -> [fused RMSNorm+gate/up+SwiGLU GEMV]
// -> [down GEMV + residual], then the fused final-norm lm_head GEMV with
// greedy argmax, and a tail kernel that feeds the token back and advances
// the position — both live in device memory, so the same graph replays for
// every step with programmatic dependent launch between the kernels.
#include <math.h>
#include <string.h>

#include <vector>

#include "../../include/tendo_synth.h"
#include "common.cuh"
#include "gemv.cuh"
#include "kernels.h"

struct tb_model {
  tb_model_config c{};
  int device = 0;
  cudaStream_t stream = nullptr;
  int64_t d = 0, H = 0, Hkv = 0, D = 0, F = 0, V = 0, L = 0, Ms = 0, B = 0, NQKV = 0;
  int8_t *wqkv = nullptr, *wo = nullptr, *wgate = nullptr, *wup = nullptr, *wdown = nullptr;
  float *sqkv = nullptr, *so = nullptr, *sgate = nullptr, *sup = nullptr, *sdown = nullptr;
  float *attn_norm = nullptr, *mlp_norm = nullptr, *final_norm = nullptr;
  float *embed = nullptr, *lm_head = nullptr, *cos_t = nullptr, *sin_t = nullptr;
  void *kc = nullptr, *vc = nullptr;  // fp32, or bf16 with kv16
  bool kv16 = false;                   // bf16 KV cache (TB_MODEL_KV_BF16)
  float *h = nullptr, *xn = nullptr, *qkv = nullptr, *attn = nullptr, *g = nullptr, *u = nullptr;
  float* gu = nullptr;  // decode: [B, 2F] gate and up products of one launch
  int64_t group = 0;    // scales per group of this many input columns (0: per output channel)
  float *qbuf = nullptr, *partial = nullptr, *logits = nullptr, *last = nullptr;
  unsigned long long* keys = nullptr;
  int64_t *tokens = nullptr, *ids = nullptr, *history = nullptr, *pos = nullptr, *step = nullptr;
  int32_t* bad = nullptr;
  int64_t host_pos = 0, host_step = 0, hist_cap = 0, chunk_s = 0, rows_max = 0;
  int nsplit = 1;
  bool fused = false;
  bool pdl = true;
  bool mk = false;      // whole decode step as one persistent kernel (batch 1)
  int mk_nsplit = 1;
  unsigned int* bar_counter = nullptr;
  unsigned long long* mk_ll = nullptr;  // the persistent kernel's tagged exchange words (zeroed at creation)
  unsigned int* mk_epoch = nullptr;      // its decode-step counter (never reset: tags stay unique)
  int* err_word = nullptr;
  uint64_t* trace = nullptr;  // [2 + 2 * (1 + 5 L + 1)] phase stamps of the last decode step
  tb_comm* comm = nullptr;    // tensor-parallel group (null: the whole model on one GPU)
  int tp = 1, tp_rank = 0;
  int64_t Hg = 0, Hkvg = 0, Fg = 0, Vg = 0;  // unsharded heads, kv heads, hidden, vocabulary
  int64_t v0 = 0;                            // vocabulary index of this rank's first lm_head row
  float* samp_u = nullptr;    // the sampler's uniform draws [B]
  bool gv = false;            // decode projections of 2..64 sequences on the tcgen05 GEMV (one weight pass)
  int lm_rows = 8;            // rows of x the fused lm_head GEMV stages in shared memory (0: the GEMM path)
  void* gv_zero = nullptr;    // its split-tile counters and sums (kept zero between launches)
  void* gv_scratch = nullptr; // its digit rows
  int8_t* tcdig = nullptr;    // digit rows of the prefill projections' activations (tcgen05 GEMM)
  float* tcs = nullptr;       // their row scales
  int trace_n = 0;
  cudaGraphExec_t graph = nullptr;
  std::vector<void*> allocs;
};

namespace {

using tb::ceil_div;

constexpr int kTcPlanes = 3;  // digit rows of the prefill GEMM's activations
// decode steps of more sequences than this run the QKV, O and gate/up
// projections on the prefill GEMM instead of the split-K GEMV (7B shape, 64
// sequences: 42 / 34 / 72 us against 59 / 43 / 101 us per layer)
constexpr int kDecodeGemmRows = 32;

template <typename T>
tb_status_t dalloc(tb_model* m, T** p, size_t count) {
  void* v = nullptr;
  cudaError_t e = cudaMalloc(&v, count * sizeof(T) > 0 ? count * sizeof(T) : 16);
  if (e != cudaSuccess) return tb::cuda_fail(e, "cudaMalloc");
  m->allocs.push_back(v);
  *p = (T*)v;
  return TB_SUCCESS;
}

// layer l's slice of a KV cache [L][B][Hkv][max_seq][D] of either element type
void* kv_layer(const tb_model* m, void* base, int64_t l) {
  const size_t elems = (size_t)l * m->B * m->Hkv * m->Ms * m->D;
  return static_cast<unsigned char*>(base) + elems * (m->kv16 ? 2 : 4);
}

__global__ void fill_kernel(float* p, int64_t n, float v) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) p[i] = v;
}

size_t lin_rows(const tb_model* m, int mat) {
  const int64_t hq = m->H * m->D, hkv = m->Hkv * m->D;
  const int64_t r[7] = {hq, hkv, hkv, m->d, m->F, m->F, m->d};
  return (size_t)r[mat];
}
size_t lin_cols(const tb_model* m, int mat) {
  const int64_t c[7] = {m->d, m->d, m->d, m->H * m->D, m->d, m->d, m->F};
  return (size_t)c[mat];
}

// Scales per row of one Linear: K / group, or 1 per output channel.
size_t lin_ng(const tb_model* m, int mat) { return m->group ? lin_cols(m, mat) / (size_t)m->group : 1; }

// Pointers of one Linear inside the layer buffers (scales [rows][lin_ng]).
void lin_ptr(tb_model* m, int layer, int mat, int8_t** q, float** s) {
  const int64_t hq = m->H * m->D, hkv = m->Hkv * m->D;
  const size_t gd = m->group ? (size_t)(m->d / m->group) : 1, gh = lin_ng(m, 3), gf = lin_ng(m, 6);
  switch (mat) {
    case 0: *q = m->wqkv + (size_t)layer * m->NQKV * m->d; *s = m->sqkv + (size_t)layer * m->NQKV * gd; break;
    case 1:
      *q = m->wqkv + ((size_t)layer * m->NQKV + hq) * m->d;
      *s = m->sqkv + ((size_t)layer * m->NQKV + hq) * gd;
      break;
    case 2:
      *q = m->wqkv + ((size_t)layer * m->NQKV + hq + hkv) * m->d;
      *s = m->sqkv + ((size_t)layer * m->NQKV + hq + hkv) * gd;
      break;
    case 3: *q = m->wo + (size_t)layer * m->d * hq; *s = m->so + (size_t)layer * m->d * gh; break;
    // gate and up rows of a layer are adjacent (one [2F, d] matrix, gate first)
    case 4: *q = m->wgate + (size_t)layer * 2 * m->F * m->d; *s = m->sgate + (size_t)layer * 2 * m->F * gd; break;
    case 5: *q = m->wup + (size_t)layer * 2 * m->F * m->d; *s = m->sup + (size_t)layer * 2 * m->F * gd; break;
    default: *q = m->wdown + (size_t)layer * m->d * m->F; *s = m->sdown + (size_t)layer * m->d * gf; break;
  }
}

struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    if (prev != dev) cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    int cur = -1;
    if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
  }
};

// Layer-by-layer forward of S tokens per sequence already embedded in m->h
// (rows b * S + s), at cache positions host_pos .. host_pos + S - 1.
tb_status_t forward_layers(tb_model* m, int64_t S) {
  cudaStream_t st = m->stream;
  const int64_t rows = m->B * S;
  const int64_t P = m->host_pos;
  const float scale = 1.0f / (float)sqrt((double)m->D);
  // rows > 32: projections on the tcgen05 GEMM (digit rows of the activations)
  // per-group scales: every projection through the grouped DequantizeMatmul
  const bool tc = rows > 32 && !m->group && tb::gemm_tc_ok(m->wqkv, rows, m->NQKV, m->d) &&
                  tb::gemm_tc_ok(m->wo, rows, m->d, m->H * m->D) && tb::gemm_tc_ok(m->wdown, rows, m->d, m->F);
  for (int64_t l = 0; l < m->L; l++) {
    int8_t *wq, *wo, *wg, *wu, *wd;
    float *sq, *so, *sg, *su, *sd;
    lin_ptr(m, (int)l, 0, &wq, &sq);
    lin_ptr(m, (int)l, 3, &wo, &so);
    lin_ptr(m, (int)l, 4, &wg, &sg);
    lin_ptr(m, (int)l, 5, &wu, &su);
    lin_ptr(m, (int)l, 6, &wd, &sd);
    void* kcl = kv_layer(m, m->kc, l);
    void* vcl = kv_layer(m, m->vc, l);
    // attention block (models/llama/quantized.go:186-199)
    if (tc) {
      TB_TRY(tb::gemm_tc_digits(m->tcdig, m->tcs, m->h, (int)rows, (int)m->d, kTcPlanes, m->attn_norm + l * m->d,
                                m->c.eps, st));
      TB_TRY(tb::gemm_tc_run(m->qkv, m->tcdig, m->tcs, wq, sq, nullptr, (int)rows, (int)m->NQKV, (int)m->d, kTcPlanes,
                             st));
    } else {
      TB_TRY(tb::rmsnorm(m->xn, nullptr, m->h, nullptr, m->attn_norm + l * m->d, rows, m->d, m->c.eps, st));
      TB_TRY(tb_dequant_matmul_i8f32(m->qkv, m->xn, wq, sq, rows, m->NQKV, m->d, m->group, (tb_stream_t)st));
    }
    TB_TRY(tb::rope_rows(m->qkv, m->cos_t, m->sin_t, m->B, S, m->H, m->D, P, m->NQKV, st));
    TB_TRY(tb::kv_append_rope(kcl, vcl, m->qkv + m->H * m->D, m->qkv + (m->H + m->Hkv) * m->D, m->cos_t, m->sin_t,
                              m->B, m->Hkv, S, m->D, P, m->Ms, m->NQKV, st, m->kv16));
    // q rows have stride NQKV; the attention kernels take [B, S, H, D] rows of H * D
    TB_CUDA(cudaMemcpy2DAsync(m->g, sizeof(float) * m->H * m->D, m->qkv, sizeof(float) * m->NQKV,
                              sizeof(float) * m->H * m->D, rows, cudaMemcpyDeviceToDevice, st));
    if (S == 1) {
      tb::AttnDecodeArgs a{};
      a.q = m->g;
      a.kcache = kcl;
      a.vcache = vcl;
      a.out = m->attn;
      a.partial = m->partial;
      a.pos = nullptr;
      a.sk = P + 1;
      a.B = (int)m->B;
      a.H = (int)m->H;
      a.Hkv = (int)m->Hkv;
      a.D = (int)m->D;
      a.max_seq = (int)m->Ms;
      a.nsplit = m->nsplit;
      a.scale = scale;
      a.kv_bf16 = m->kv16;
      TB_TRY(tb::attn_decode(a, st, false));
    } else {
      TB_TRY(tb::attn_prefill(m->attn, m->g, kcl, vcl, (int)m->B, (int)m->H, (int)m->Hkv, (int)S, P + S, (int)m->D,
                              (int)m->Ms, scale, st, m->kv16));
    }
    // o projection + residual; row-parallel under tensor parallelism: each
    // rank's partial product, the residual on rank 0 only, summed over ranks
    const float* resid = m->tp_rank == 0 ? m->h : nullptr;
    if (rows <= 32 || m->group) {
      TB_TRY(tb_dequant_matmul_i8f32(m->xn, m->attn, wo, so, rows, m->d, m->H * m->D, m->group, (tb_stream_t)st));
      TB_TRY(tb::allreduce(m->comm, m->xn, (size_t)(rows * m->d), false, st, m->err_word));
      TB_TRY(tb_add_f32(m->h, m->h, m->xn, rows * m->d, (tb_stream_t)st));
    } else if (tc) {
      const int HD = (int)(m->H * m->D);
      TB_TRY(tb::gemm_tc_digits(m->tcdig, m->tcs, m->attn, (int)rows, HD, kTcPlanes, nullptr, 0.f, st));
      TB_TRY(tb::gemm_tc_run(m->h, m->tcdig, m->tcs, wo, so, resid, (int)rows, (int)m->d, HD, kTcPlanes, st));
      TB_TRY(tb::allreduce(m->comm, m->h, (size_t)(rows * m->d), false, st, m->err_word));
    } else {
      TB_TRY(tb::gemm_simt_i8(m->h, m->attn, wo, so, resid, (int)rows, (int)m->d, (int)(m->H * m->D), 0, st));
      TB_TRY(tb::allreduce(m->comm, m->h, (size_t)(rows * m->d), false, st, m->err_word));
    }
    // MLP block (models/llama/quantized.go:206-219, :385-417)
    if (tc) {
      TB_TRY(tb::gemm_tc_digits(m->tcdig, m->tcs, m->h, (int)rows, (int)m->d, kTcPlanes, m->mlp_norm + l * m->d,
                                m->c.eps, st));
      TB_TRY(tb::gemm_tc_run(m->g, m->tcdig, m->tcs, wg, sg, nullptr, (int)rows, (int)m->F, (int)m->d, kTcPlanes, st));
      TB_TRY(tb::gemm_tc_run(m->u, m->tcdig, m->tcs, wu, su, nullptr, (int)rows, (int)m->F, (int)m->d, kTcPlanes, st));
    } else {
      TB_TRY(tb::rmsnorm(m->xn, nullptr, m->h, nullptr, m->mlp_norm + l * m->d, rows, m->d, m->c.eps, st));
      TB_TRY(tb_dequant_matmul_i8f32(m->g, m->xn, wg, sg, rows, m->F, m->d, m->group, (tb_stream_t)st));
      TB_TRY(tb_dequant_matmul_i8f32(m->u, m->xn, wu, su, rows, m->F, m->d, m->group, (tb_stream_t)st));
    }
    TB_TRY(tb::silu_mul(m->g, m->g, m->u, rows * m->F, st));
    if (rows <= 32 || m->group) {
      TB_TRY(tb_dequant_matmul_i8f32(m->xn, m->g, wd, sd, rows, m->d, m->F, m->group, (tb_stream_t)st));
      TB_TRY(tb::allreduce(m->comm, m->xn, (size_t)(rows * m->d), false, st, m->err_word));
      TB_TRY(tb_add_f32(m->h, m->h, m->xn, rows * m->d, (tb_stream_t)st));
    } else if (tc) {
      TB_TRY(tb::gemm_tc_digits(m->tcdig, m->tcs, m->g, (int)rows, (int)m->F, kTcPlanes, nullptr, 0.f, st));
      TB_TRY(tb::gemm_tc_run(m->h, m->tcdig, m->tcs, wd, sd, resid, (int)rows, (int)m->d, (int)m->F, kTcPlanes, st));
      TB_TRY(tb::allreduce(m->comm, m->h, (size_t)(rows * m->d), false, st, m->err_word));
    } else {
      TB_TRY(tb::gemm_simt_i8(m->h, m->g, wd, sd, resid, (int)rows, (int)m->d, (int)m->F, 0, st));
      TB_TRY(tb::allreduce(m->comm, m->h, (size_t)(rows * m->d), false, st, m->err_word));
    }
  }
  return TB_SUCCESS;
}

// Final RMSNorm + lm_head on the last row of each sequence, greedy argmax
// into m->tokens (and the history), position set to host_pos.
tb_status_t finish_logits(tb_model* m, int64_t S) {
  cudaStream_t st = m->stream;
  // gather the last rows: h[b * S + S - 1] -> last[b]
  TB_CUDA(cudaMemcpy2DAsync(m->last, sizeof(float) * m->d, m->h + (S - 1) * m->d, sizeof(float) * m->d * S,
                            sizeof(float) * m->d, m->B, cudaMemcpyDeviceToDevice, st));
  // greedy keys of this rank's vocabulary rows, max over the ranks, then the
  // tail kernel turns them into tokens (it advances the position by one:
  // pre-compensate)
  if (m->B <= 8 && tb::gemv_smem_bytes(8, (int)m->d) <= 200 * 1024) {
    tb::LmHeadArgs a{};
    a.h = m->last;
    a.norm_w = m->final_norm;
    a.eps = m->c.eps;
    a.w = m->lm_head;
    a.logits = m->logits;
    a.argmax_keys = m->keys;
    a.M = (int)m->B;
    a.d = (int)m->d;
    a.V = (int)m->V;
    a.v0 = (int)m->v0;
    a.l2_prefetch = tb::l2_prefetch_enabled();
    TB_TRY(tb::gemv_lmhead(a, st, false));
  } else {
    TB_TRY(tb::rmsnorm(m->xn, nullptr, m->last, nullptr, m->final_norm, m->B, m->d, m->c.eps, st));
    TB_TRY(tb::gemm_f32_nt(m->logits, m->xn, m->lm_head, (int)m->B, (int)m->V, (int)m->d, st));
    TB_TRY(tb::argmax_keys(m->keys, m->logits, m->B, m->V, m->v0, st));
  }
  TB_TRY(tb::allreduce(m->comm, m->keys, (size_t)m->B, true, st, m->err_word));
  int64_t p = m->host_pos - 1;
  TB_CUDA(cudaMemcpyAsync(m->pos, &p, sizeof(int64_t), cudaMemcpyHostToDevice, st));
  TB_TRY(tb::finish_step(m->keys, m->tokens, m->history, m->step, m->pos, (int)m->B, m->hist_cap, st, false));
  m->host_step += 1;
  // cudaMemcpyAsync from pageable host memory is staged before returning, so
  // the stack values above may go out of scope; keep the stream ordered.
  TB_CUDA(cudaStreamSynchronize(st));
  return TB_SUCCESS;
}

// Prefill / generic forward of tokens already in m->ids [B, S].
tb_status_t forward_tokens(tb_model* m, int64_t S) {
  cudaStream_t st = m->stream;
  for (int64_t s0 = 0; s0 < S; s0 += m->chunk_s) {
    const int64_t sc = S - s0 < m->chunk_s ? S - s0 : m->chunk_s;
    // embed rows b * sc + s of this chunk
    for (int64_t b = 0; b < m->B; b++)
      TB_TRY(tb::embedding(m->h + b * sc * m->d, m->embed, m->ids + b * S + s0, sc, m->Vg, m->d, m->bad, st, false));
    TB_TRY(forward_layers(m, sc));
    m->host_pos += sc;
    if (s0 + sc >= S) TB_TRY(finish_logits(m, sc));
  }
  return TB_SUCCESS;
}

// One kernel of the fused decode step (kind as in tb_model_bench_kernel).
tb_status_t decode_kernel(tb_model* m, int kind, int64_t l, bool pdl) {
  cudaStream_t st = m->stream;
  const float scale = 1.0f / (float)sqrt((double)m->D);
  {
    int8_t *wq, *wo, *wg, *wu, *wd;
    float *sq, *so, *sg, *su, *sd;
    lin_ptr(m, (int)l, 0, &wq, &sq);
    lin_ptr(m, (int)l, 3, &wo, &so);
    lin_ptr(m, (int)l, 4, &wg, &sg);
    lin_ptr(m, (int)l, 5, &wu, &su);
    lin_ptr(m, (int)l, 6, &wd, &sd);
    void* kcl = kv_layer(m, m->kc, l);
    void* vcl = kv_layer(m, m->vc, l);
    tb::QkvArgs qa{};
    qa.h = m->h;
    qa.norm_w = m->attn_norm + l * m->d;
    qa.eps = m->c.eps;
    qa.q = wq;
    qa.scale = sq;
    qa.cos_t = m->cos_t;
    qa.sin_t = m->sin_t;
    qa.pos = m->pos;
    qa.qout = m->qbuf;
    qa.kcache = static_cast<float*>(kcl);  // the fused QKV kernels: fp32 caches only
    qa.vcache = static_cast<float*>(vcl);
    qa.M = (int)m->B;
    qa.d = (int)m->d;
    qa.H = (int)m->H;
    qa.Hkv = (int)m->Hkv;
    qa.D = (int)m->D;
    qa.max_seq = (int)m->Ms;
    const float* resid = m->tp_rank == 0 ? m->h : nullptr;
    if (m->gv && (kind == 0 || kind == 2 || kind == 3) && m->B > kDecodeGemmRows && !m->group) {
      // 33..64 sequences: the prefill GEMM (a 128-row tile of the sequences'
      // digit rows against 128 weight rows) reads each weight tile once and
      // needs no split-K reduction; the digit rows (with the RMSNorm) once
      // per input.  The down projection (K = F) stays on the split-K GEMV:
      // its 128-row output tiles are too few to cover the SMs over that K.
      const int B = (int)m->B, d = (int)m->d, HD = (int)(m->H * m->D), F = (int)m->F;
      if (kind == 0) {
        TB_TRY(tb::gemm_tc_digits(m->tcdig, m->tcs, m->h, B, d, kTcPlanes, m->attn_norm + l * m->d, m->c.eps, st));
        TB_TRY(tb::gemm_tc_run(m->qkv, m->tcdig, m->tcs, wq, sq, nullptr, B, (int)m->NQKV, d, kTcPlanes, st));
        return tb::qkv_rope_append(m->qbuf, kcl, vcl, m->qkv, m->cos_t, m->sin_t, m->pos, m->B, m->H, m->Hkv, m->D,
                                   m->Ms, st, m->kv16);
      }
      if (kind == 2) {
        TB_TRY(tb::gemm_tc_digits(m->tcdig, m->tcs, m->attn, B, HD, kTcPlanes, nullptr, 0.f, st));
        return tb::gemm_tc_run(m->h, m->tcdig, m->tcs, wo, so, resid, B, d, HD, kTcPlanes, st);
      }
      if (kind == 3) {
        // gate and up rows are one [2F, d] matrix: one GEMM, then SwiGLU
        TB_TRY(tb::gemm_tc_digits(m->tcdig, m->tcs, m->h, B, d, kTcPlanes, m->mlp_norm + l * m->d, m->c.eps, st));
        TB_TRY(tb::gemm_tc_run(m->gu, m->tcdig, m->tcs, wg, sg, nullptr, B, 2 * F, d, kTcPlanes, st));
        return tb::silu_mul_rows(m->g, m->gu, m->B, m->F, st);
      }
    }
    if (m->gv && kind != 1) {
      // 2..64 sequences: each projection streams its weights once (tcgen05
      // GEMV, RMSNorm fused into the digit split), RoPE / KV append and
      // SwiGLU as separate elementwise kernels
      const int B = (int)m->B, d = (int)m->d, HD = (int)(m->H * m->D), F = (int)m->F;
      if (kind == 0) {
        TB_TRY(tb::gemv_tc(m->qkv, m->h, wq, sq, nullptr, B, (int)m->NQKV, d, m->gv_zero, false, m->gv_scratch, st,
                           m->attn_norm + l * m->d, m->c.eps, (int)m->group));
        return tb::qkv_rope_append(m->qbuf, kcl, vcl, m->qkv, m->cos_t, m->sin_t, m->pos, m->B, m->H, m->Hkv, m->D,
                                   m->Ms, st, m->kv16);
      }
      if (kind == 2)
        return tb::gemv_tc(m->h, m->attn, wo, so, resid, B, d, HD, m->gv_zero, false, m->gv_scratch, st, nullptr, 0.f,
                           (int)m->group);
      if (kind == 3) {
        // gate and up rows are one [2F, d] matrix: one GEMV launch, then SwiGLU
        TB_TRY(tb::gemv_tc(m->gu, m->h, wg, sg, nullptr, B, 2 * F, d, m->gv_zero, false, m->gv_scratch, st,
                           m->mlp_norm + l * m->d, m->c.eps, (int)m->group));
        return tb::silu_mul_rows(m->g, m->gu, m->B, m->F, st);
      }
      if (kind == 4)
        return tb::gemv_tc(m->h, m->g, wd, sd, resid, B, d, F, m->gv_zero, false, m->gv_scratch, st, nullptr, 0.f,
                           (int)m->group);
    }
    if (kind == 0) {
      // the fused kernels take up to 8 sequences: larger batches run in groups
      for (int64_t b0 = 0; b0 < m->B; b0 += 8) {
        tb::QkvArgs g = qa;
        g.h = m->h + b0 * m->d;
        g.qout = m->qbuf + b0 * m->H * m->D;
        g.kcache = qa.kcache + b0 * m->Hkv * m->Ms * m->D;
        g.vcache = qa.vcache + b0 * m->Hkv * m->Ms * m->D;
        g.M = (int)(m->B - b0 < 8 ? m->B - b0 : 8);
        TB_TRY(tb::gemv_qkv_rope(g, st, pdl));
      }
      return TB_SUCCESS;
    }
    tb::AttnDecodeArgs aa{};
    aa.q = m->qbuf;
    aa.kcache = kcl;
    aa.vcache = vcl;
    aa.out = m->attn;
    aa.partial = m->partial;
    aa.pos = m->pos;
    aa.B = (int)m->B;
    aa.H = (int)m->H;
    aa.Hkv = (int)m->Hkv;
    aa.D = (int)m->D;
    aa.max_seq = (int)m->Ms;
    aa.nsplit = m->nsplit;
    aa.scale = scale;
    aa.kv_bf16 = m->kv16;
    if (kind == 1) return tb::attn_decode(aa, st, pdl);
    // row-parallel under tensor parallelism: the residual joins on rank 0 and
    // the step sums the ranks' partial products after the kernel
    if (kind == 2)
      return tb::gemv_plain(m->h, m->attn, wo, so, resid, (int)m->B, (int)m->d, (int)(m->H * m->D), nullptr, 0.f, st,
                            pdl);
    tb::GateUpArgs ga{};
    ga.h = m->h;
    ga.norm_w = m->mlp_norm + l * m->d;
    ga.eps = m->c.eps;
    ga.gate = wg;
    ga.up = wu;
    ga.gate_scale = sg;
    ga.up_scale = su;
    ga.act = m->g;
    ga.M = (int)m->B;
    ga.d = (int)m->d;
    ga.F = (int)m->F;
    if (kind == 3) {
      for (int64_t b0 = 0; b0 < m->B; b0 += 8) {
        tb::GateUpArgs g = ga;
        g.h = m->h + b0 * m->d;
        g.act = m->g + b0 * m->F;
        g.M = (int)(m->B - b0 < 8 ? m->B - b0 : 8);
        TB_TRY(tb::gemv_gateup(g, st, pdl));
      }
      return TB_SUCCESS;
    }
    if (kind == 4)
      return tb::gemv_plain(m->h, m->g, wd, sd, resid, (int)m->B, (int)m->d, (int)m->F, nullptr, 0.f, st, pdl);
  }
  tb::LmHeadArgs la{};
  la.h = m->h;
  la.norm_w = m->final_norm;
  la.eps = m->c.eps;
  la.w = m->lm_head;
  la.logits = m->logits;
  la.argmax_keys = m->keys;
  la.M = (int)m->B;
  la.d = (int)m->d;
  la.V = (int)m->V;
  la.v0 = (int)m->v0;
  la.l2_prefetch = tb::l2_prefetch_enabled();
  if (kind == 5 && !m->lm_rows) {
    // d too wide for the fused kernel's staged rows, or too many row groups:
    // norm, fp32 GEMM, keys
    TB_TRY(tb::rmsnorm(m->xn, nullptr, m->h, nullptr, m->final_norm, m->B, m->d, m->c.eps, st));
    TB_TRY(tb::gemm_f32_nt(m->logits, m->xn, m->lm_head, (int)m->B, (int)m->V, (int)m->d, st));
    return tb::argmax_keys(m->keys, m->logits, m->B, m->V, m->v0, st);
  }
  if (kind == 5) {
    // groups of as many sequences as the kernel can stage (8, or fewer for wide d)
    const int64_t gr = m->lm_rows;
    for (int64_t b0 = 0; b0 < m->B; b0 += gr) {
      tb::LmHeadArgs g = la;
      g.h = m->h + b0 * m->d;
      g.logits = m->logits + b0 * m->V;
      g.argmax_keys = m->keys + b0;
      g.M = (int)(m->B - b0 < gr ? m->B - b0 : gr);
      TB_TRY(tb::gemv_lmhead(g, st, pdl));
    }
    return TB_SUCCESS;
  }
  return TB_ERROR_INVALID_ARGUMENT;
}

// One fused decode step (graph body).
tb_status_t decode_step_fused(tb_model* m) {
  const bool pdl = m->pdl;
  TB_TRY(tb::embedding(m->h, m->embed, m->tokens, m->B, m->Vg, m->d, m->bad, m->stream, pdl));
  for (int64_t l = 0; l < m->L; l++)
    for (int kind = 0; kind < 5; kind++) {
      TB_TRY(decode_kernel(m, kind, l, pdl));
      // tensor parallelism: sum the row-parallel o / down partial products
      if (kind == 2 || kind == 4)
        TB_TRY(tb::allreduce(m->comm, m->h, (size_t)(m->B * m->d), false, m->stream, m->err_word));
    }
  TB_TRY(decode_kernel(m, 5, 0, pdl));
  TB_TRY(tb::allreduce(m->comm, m->keys, (size_t)m->B, true, m->stream, m->err_word));
  TB_TRY(tb::finish_step(m->keys, m->tokens, m->history, m->step, m->pos, (int)m->B, m->hist_cap, m->stream, pdl));
  return TB_SUCCESS;
}

// Arguments of the persistent decode kernel (decode_mk.cu).
tb::MkArgs mk_args(tb_model* m) {
  tb::MkArgs a{};
  a.L = (int)m->L;
  a.d = (int)m->d;
  a.H = (int)m->H;
  a.Hkv = (int)m->Hkv;
  a.D = (int)m->D;
  a.F = (int)m->F;
  a.V = (int)m->V;
  a.max_seq = (int)m->Ms;
  a.nsplit = m->mk_nsplit;
  a.eps = m->c.eps;
  a.attn_scale = 1.0f / (float)sqrt((double)m->D);
  a.wqkv = m->wqkv;
  a.sqkv = m->sqkv;
  a.wo = m->wo;
  a.so = m->so;
  a.wg = m->wgate;
  a.sg = m->sgate;
  a.wu = m->wup;
  a.su = m->sup;
  a.wd = m->wdown;
  a.sd = m->sdown;
  a.attn_norm = m->attn_norm;
  a.mlp_norm = m->mlp_norm;
  a.final_norm = m->final_norm;
  a.embed = m->embed;
  a.lm_head = m->lm_head;
  a.cos_t = m->cos_t;
  a.sin_t = m->sin_t;
  a.kc = static_cast<float*>(m->kc);  // the persistent kernel runs fp32 caches only
  a.vc = static_cast<float*>(m->vc);
  a.h = m->h;
  a.ll = m->mk_ll;
  a.epoch = m->mk_epoch;
  a.logits = m->logits;
  a.keys = m->keys;
  a.tokens = m->tokens;
  a.history = m->history;
  a.step = m->step;
  a.pos = m->pos;
  a.hist_cap = m->hist_cap;
  a.bar_counter = m->bar_counter;
  a.err = m->err_word;
  a.trace = m->trace;
  a.utrace = m->trace ? m->trace + m->trace_n : nullptr;
  return a;
}

tb_status_t build_graph(tb_model* m) {
  if (m->graph) return TB_SUCCESS;
  cudaGraph_t g = nullptr;
  TB_CUDA(cudaStreamBeginCapture(m->stream, cudaStreamCaptureModeThreadLocal));
  tb_status_t s = m->mk ? tb::megakernel_launch(mk_args(m), m->stream) : decode_step_fused(m);
  cudaError_t e = cudaStreamEndCapture(m->stream, &g);
  if (s != TB_SUCCESS) {
    if (g) cudaGraphDestroy(g);
    return s;
  }
  if (e != cudaSuccess) return tb::cuda_fail(e, "cudaStreamEndCapture");
  e = cudaGraphInstantiate(&m->graph, g, 0);
  cudaGraphDestroy(g);
  if (e != cudaSuccess) {
    m->graph = nullptr;
    return tb::cuda_fail(e, "cudaGraphInstantiate");
  }
  return TB_SUCCESS;
}

}  // namespace

namespace {

tb_status_t create_model(tb_model** out, const tb_model_config* cfg, int device, tb_comm* comm, uint32_t flags,
                         int64_t group = 0) {
  TB_REQUIRE(out && cfg && group >= 0);
  TB_REQUIRE((flags & ~(uint32_t)TB_MODEL_KV_BF16) == 0);
  *out = nullptr;
  TB_REQUIRE(cfg->vocab > 0 && cfg->dim > 0 && cfg->layers > 0 && cfg->heads > 0 && cfg->kv_heads > 0);
  TB_REQUIRE(cfg->dim % cfg->heads == 0 && cfg->heads % cfg->kv_heads == 0 && cfg->hidden > 0);
  TB_REQUIRE(cfg->max_seq > 0 && cfg->max_batch > 0);
  TB_REQUIRE((cfg->dim / cfg->heads) % 2 == 0);
  const int tp = tb::comm_size(comm), rank = tb::comm_rank(comm);
  TB_REQUIRE(cfg->heads % tp == 0 && cfg->kv_heads % tp == 0 && cfg->hidden % tp == 0 && cfg->vocab % tp == 0);
  DeviceGuard guard(device);
  TB_CUDA(cudaSetDevice(device));
  tb_model* m = new tb_model();
  m->c = *cfg;
  m->device = device;
  m->comm = comm;
  m->kv16 = (flags & TB_MODEL_KV_BF16) != 0;
  m->group = group;
  m->tp = tp;
  m->tp_rank = rank;
  m->Hg = cfg->heads;
  m->Hkvg = cfg->kv_heads;
  m->Fg = cfg->hidden;
  m->Vg = cfg->vocab;
  m->d = cfg->dim;
  m->H = cfg->heads / tp;
  m->Hkv = cfg->kv_heads / tp;
  m->D = cfg->dim / cfg->heads;
  m->F = cfg->hidden / tp;
  m->V = cfg->vocab / tp;
  m->v0 = (int64_t)rank * m->V;
  m->L = cfg->layers;
  m->Ms = cfg->max_seq;
  m->B = cfg->max_batch;
  m->NQKV = (m->H + 2 * m->Hkv) * m->D;
  // per-group scales: every Linear's input width (this rank's share of the
  // row-parallel ones) a whole number of groups
  if (group && (m->d % group || (m->H * m->D) % group || m->F % group)) {
    delete m;
    return TB_ERROR_NOT_SUPPORTED;
  }
  m->hist_cap = m->Ms;
  m->chunk_s = 4096 / m->B > 0 ? 4096 / m->B : 1;
  if (m->chunk_s > m->Ms) m->chunk_s = m->Ms;
  m->rows_max = m->B * m->chunk_s;
  const size_t fused_smem = tb::gemv_smem_bytes(m->B <= 1 ? 1 : (m->B <= 2 ? 2 : (m->B <= 4 ? 4 : 8)), (int)m->d);
  {
    // 2..64 sequences: the decode projections run on the tcgen05 GEMV (needs
    // K % 128 and an sm_100 device; probed with an aligned stand-in pointer)
    const void* al = reinterpret_cast<const void*>(static_cast<uintptr_t>(256));
    const int64_t HD = m->H * m->D;
    // (a bf16 cache takes this path at batch 1 too: its RoPE / append kernel
    // writes either cache type)
    m->gv = (m->B > 1 || m->kv16 || m->group) && m->B <= tb::kGemvTcMaxM &&
            tb::gemv_tc_ok(al, m->B, m->NQKV, m->d, m->group) && tb::gemv_tc_ok(al, m->B, m->d, HD, m->group) &&
            tb::gemv_tc_ok(al, m->B, 2 * m->F, m->d, m->group) && tb::gemv_tc_ok(al, m->B, m->d, m->F, m->group);
  }
  // the captured decode step: the attention kernel's head shapes, and either
  // the tcgen05 GEMV projections (2..64 sequences) or the fused CUDA-core /
  // IMMA kernels, which stage up to 8 rows of x in shared memory
  m->lm_rows = 0;
  for (int r = 8; r >= 1 && !m->lm_rows; r /= 2)
    if (tb::gemv_smem_bytes(r, (int)m->d) <= 200 * 1024) m->lm_rows = r;
  // each row group re-reads the whole fp32 lm_head: past four groups one
  // fp32 GEMM over all rows is faster (7B shape, 64 sequences: 0.81 ms
  // against 1.44 ms per step; 32 sequences: 0.81 against 0.72)
  if (m->lm_rows && m->B > 4 * m->lm_rows) m->lm_rows = 0;
  m->fused = m->d % 16 == 0 && (m->H * m->D) % 16 == 0 && m->F % 16 == 0 && (m->D == 64 || m->D == 128) &&
             (m->H / m->Hkv == 1 || m->H / m->Hkv == 2 || m->H / m->Hkv == 4 || m->H / m->Hkv == 8) &&
             (m->gv ? m->B <= 64 : (m->B <= 16 && fused_smem <= 200 * 1024 && !m->kv16 && !m->group));
  const char* nopdl = getenv("TENDO_B200_NO_PDL");
  m->pdl = !(nopdl && *nopdl == '1');
  m->nsplit = tb::attn_decode_splits((int)m->B, (int)m->H, (int)m->Hkv, (int)m->D, m->Ms, m->kv16);
  {
    const char* e = getenv("TENDO_B200_MEGAKERNEL");
    m->mk = !(e && e[0] == '0') && tp == 1 && !m->kv16 && m->group == 0 &&
            tb::megakernel_supported((int)m->d, (int)m->H, (int)m->Hkv, (int)m->D, (int)m->F, (int)m->V, (int)m->B);
    m->mk_nsplit = tb::megakernel_splits((int)m->Hkv);
  }
  tb_status_t s = TB_SUCCESS;
  auto A = [&](tb_status_t r) {
    if (s == TB_SUCCESS) s = r;
  };
  const size_t L = m->L;
  const size_t gd = m->group ? (size_t)(m->d / m->group) : 1;
  A(dalloc(m, &m->wqkv, L * m->NQKV * m->d));
  A(dalloc(m, &m->sqkv, L * m->NQKV * gd));
  A(dalloc(m, &m->wo, L * m->d * m->H * m->D));
  A(dalloc(m, &m->so, L * m->d * lin_ng(m, 3)));
  // per layer the gate rows, then the up rows: one [2F, d] matrix, so a
  // single GEMV launch computes both
  A(dalloc(m, &m->wgate, L * 2 * m->F * m->d));
  A(dalloc(m, &m->sgate, L * 2 * m->F * gd));
  if (s == TB_SUCCESS) {
    m->wup = m->wgate + m->F * m->d;
    m->sup = m->sgate + m->F * gd;
  }
  A(dalloc(m, &m->wdown, L * m->d * m->F));
  A(dalloc(m, &m->sdown, L * m->d * lin_ng(m, 6)));
  A(dalloc(m, &m->attn_norm, L * m->d));
  A(dalloc(m, &m->mlp_norm, L * m->d));
  A(dalloc(m, &m->final_norm, (size_t)m->d));
  A(dalloc(m, &m->embed, (size_t)m->Vg * m->d));
  A(dalloc(m, &m->lm_head, (size_t)m->V * m->d));
  A(dalloc(m, &m->cos_t, (size_t)m->Ms * (m->D / 2)));
  A(dalloc(m, &m->sin_t, (size_t)m->Ms * (m->D / 2)));
  const size_t kv = L * m->B * m->Hkv * m->Ms * m->D * (m->kv16 ? 2 : 4);  // bytes
  {
    unsigned char *kc = nullptr, *vc = nullptr;
    A(dalloc(m, &kc, kv));
    A(dalloc(m, &vc, kv));
    m->kc = kc;
    m->vc = vc;
  }
  const size_t R = (size_t)m->rows_max;
  A(dalloc(m, &m->h, R * m->d));
  A(dalloc(m, &m->xn, R * m->d));
  A(dalloc(m, &m->qkv, R * m->NQKV));
  A(dalloc(m, &m->attn, R * m->H * m->D));
  const size_t gw = R * (m->F > m->H * m->D ? m->F : m->H * m->D);
  A(dalloc(m, &m->g, gw));
  A(dalloc(m, &m->u, R * m->F));
  if (m->gv) A(dalloc(m, &m->gu, (size_t)m->B * 2 * m->F));
  A(dalloc(m, &m->qbuf, (size_t)m->B * m->H * m->D));
  {
    // split partials of the decode attention: the per-step kernels' layout
    // and, at batch 1, the persistent kernel's (its rows are D + 4 floats)
    size_t pb = tb::attn_decode_workspace((int)m->B, (int)m->H, (int)m->D, m->nsplit);
    A(dalloc(m, &m->partial, pb / sizeof(float)));
  }
  if (m->mk) {
    const size_t w = tb::megakernel_ll_words((int)m->d, (int)m->H, (int)m->Hkv, (int)m->D, (int)m->F, m->mk_nsplit);
    A(dalloc(m, &m->mk_ll, w));
    A(dalloc(m, &m->mk_epoch, 1));
  }
  A(dalloc(m, &m->logits, (size_t)m->B * m->V));
  A(dalloc(m, &m->last, (size_t)m->B * m->d));
  A(dalloc(m, &m->keys, (size_t)m->B));
  A(dalloc(m, &m->tokens, (size_t)m->B));
  A(dalloc(m, &m->ids, (size_t)m->B * m->Ms));
  A(dalloc(m, &m->history, (size_t)m->hist_cap * m->B));
  A(dalloc(m, &m->pos, 1));
  A(dalloc(m, &m->step, 1));
  A(dalloc(m, &m->bad, 1));
  A(dalloc(m, &m->bar_counter, 1));
  m->trace_n = tb::megakernel_trace_stamps((int)m->L);
  A(dalloc(m, &m->trace, (size_t)m->trace_n + 2 * (size_t)tb::kMkUnitTrace));
  A(dalloc(m, &m->err_word, 1));
  A(dalloc(m, &m->samp_u, (size_t)m->B));
  if (m->gv) {
    int64_t nmax = m->NQKV > m->d ? m->NQKV : m->d;
    if (2 * m->F > nmax) nmax = 2 * m->F;
    int64_t kmax = m->d > m->H * m->D ? m->d : m->H * m->D;
    if (m->F > kmax) kmax = m->F;
    unsigned char* z = nullptr;
    unsigned char* sc = nullptr;
    A(dalloc(m, &z, tb::gemv_tc_zeroed_bytes(m->B, nmax, kmax)));
    A(dalloc(m, &sc, tb::gemv_tc_scratch_bytes(m->B, nmax, kmax, m->group)));
    m->gv_zero = z;
    m->gv_scratch = sc;
    if (z) {
      const cudaError_t ez = cudaMemset(z, 0, tb::gemv_tc_zeroed_bytes(m->B, nmax, kmax));
      if (ez != cudaSuccess) A(tb::cuda_fail(ez, "cudaMemset"));
    }
  }
  {
    int64_t kmax = m->d > m->H * m->D ? m->d : m->H * m->D;
    if (m->F > kmax) kmax = m->F;
    A(dalloc(m, &m->tcdig, (size_t)kTcPlanes * R * kmax));
    A(dalloc(m, &m->tcs, R));
  }
  if (s == TB_SUCCESS) {
    cudaError_t e = cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking);
    if (e != cudaSuccess) s = tb::cuda_fail(e, "cudaStreamCreate");
  }
  if (s == TB_SUCCESS) {
    std::vector<float> ct((size_t)m->Ms * (m->D / 2)), sn(ct.size());
    tb_rope_tables_host(ct.data(), sn.data(), (int)m->D, (int)m->Ms, cfg->rope_base);
    cudaError_t e = cudaMemcpy(m->cos_t, ct.data(), ct.size() * sizeof(float), cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(m->sin_t, sn.data(), sn.size() * sizeof(float), cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemset(m->keys, 0, sizeof(unsigned long long) * m->B);
    if (e == cudaSuccess) e = cudaMemset(m->kc, 0, kv);
    if (e == cudaSuccess) e = cudaMemset(m->vc, 0, kv);
    if (e == cudaSuccess) e = cudaMemset(m->pos, 0, sizeof(int64_t));
    if (e == cudaSuccess) e = cudaMemset(m->step, 0, sizeof(int64_t));
    if (e == cudaSuccess) e = cudaMemset(m->bad, 0, sizeof(int32_t));
    if (e == cudaSuccess) e = cudaMemset(m->bar_counter, 0, sizeof(unsigned int));
    if (e == cudaSuccess && m->mk) {
      const size_t w = tb::megakernel_ll_words((int)m->d, (int)m->H, (int)m->Hkv, (int)m->D, (int)m->F, m->mk_nsplit);
      e = cudaMemset(m->mk_ll, 0, w * sizeof(unsigned long long));
      if (e == cudaSuccess) e = cudaMemset(m->mk_epoch, 0, sizeof(unsigned int));
    }
    if (e == cudaSuccess) e = cudaMemset(m->err_word, 0, sizeof(int));
    if (e != cudaSuccess) s = tb::cuda_fail(e, "engine init");
  }
  if (s != TB_SUCCESS) {
    tb_model_destroy(m);
    return s;
  }
  *out = m;
  return TB_SUCCESS;
}

}  // namespace

extern "C" tb_status_t tb_model_create(tb_model** out, const tb_model_config* cfg, int device) {
  TB_INJECT("tb_model_create");
  return create_model(out, cfg, device, nullptr, 0);
}

extern "C" tb_status_t tb_model_create_tp(tb_model** out, const tb_model_config* cfg, int device, tb_comm* comm) {
  TB_INJECT("tb_model_create");
  TB_REQUIRE(comm);
  return create_model(out, cfg, device, comm, 0);
}

extern "C" tb_status_t tb_model_create_ex(tb_model** out, const tb_model_config* cfg, int device, tb_comm* comm,
                                          uint32_t flags) {
  TB_INJECT("tb_model_create");
  return create_model(out, cfg, device, comm, flags);
}

extern "C" tb_status_t tb_model_create_grouped(tb_model** out, const tb_model_config* cfg, int device, tb_comm* comm,
                                               uint32_t flags, int64_t group_size) {
  TB_INJECT("tb_model_create");
  return create_model(out, cfg, device, comm, flags, group_size);
}

extern "C" tb_status_t tb_model_destroy(tb_model* m) {
  if (!m) return TB_SUCCESS;
  DeviceGuard guard(m->device);
  if (m->graph) cudaGraphExecDestroy(m->graph);
  if (m->stream) {
    cudaStreamSynchronize(m->stream);
    cudaStreamDestroy(m->stream);
  }
  for (void* p : m->allocs) cudaFree(p);
  delete m;
  return TB_SUCCESS;
}

extern "C" tb_status_t tb_model_init_synthetic(tb_model* m, uint64_t seed) {
  TB_INJECT("tb_model_init_synthetic");
  TB_REQUIRE(m);
  DeviceGuard guard(m->device);
  tb_stream_t st = (tb_stream_t)m->stream;
  // every rank draws its shard with the unsharded element indices, so the
  // sharded model is the same model (column-parallel: rows row0..; row-
  // parallel: columns col0.. of full rows, scales over the full row)
  const int64_t r = m->tp_rank;
  for (int l = 0; l < m->L; l++) {
    for (int mat = 0; mat < 7; mat++) {
      int8_t* q;
      float* s;
      lin_ptr(m, l, mat, &q, &s);
      const int64_t rows = (int64_t)lin_rows(m, mat), cols = (int64_t)lin_cols(m, mat);
      int64_t row0 = 0, col0 = 0, K = cols;
      switch (mat) {
        case 0: row0 = r * m->H * m->D; break;
        case 1:
        case 2: row0 = r * m->Hkv * m->D; break;
        case 3: col0 = r * m->H * m->D; K = m->Hg * m->D; break;
        case 4:
        case 5: row0 = r * m->F; break;
        default: col0 = r * m->F; K = m->Fg; break;
      }
      if (m->group)
        TB_TRY(tb::synth_quant_shard_grp(q, s, rows, K, row0, col0, cols, m->group, seed,
                                         (uint64_t)l * TS_MATS + (uint64_t)mat, 0.02, m->stream));
      else
        TB_TRY(tb::synth_quant_shard(q, s, rows, K, row0, col0, cols, seed, (uint64_t)l * TS_MATS + (uint64_t)mat,
                                     0.02, m->stream));
    }
  }
  TB_TRY(tb_synth_normal_f32(m->embed, m->Vg, m->d, seed, 0x7fff0001ull, 0.02, st));
  TB_TRY(tb::synth_normal_rows(m->lm_head, m->V, m->d, m->v0, seed, 0x7fff0002ull, 0.02, m->stream));
  fill_kernel<<<256, 256, 0, m->stream>>>(m->attn_norm, m->L * m->d, 1.0f);
  fill_kernel<<<256, 256, 0, m->stream>>>(m->mlp_norm, m->L * m->d, 1.0f);
  fill_kernel<<<16, 256, 0, m->stream>>>(m->final_norm, m->d, 1.0f);
  TB_TRY(tb::check_launch("fill_kernel"));
  TB_CUDA(cudaStreamSynchronize(m->stream));
  return TB_SUCCESS;
}

extern "C" tb_status_t tb_model_set_linear(tb_model* m, int layer, int mat, const int8_t* q_host,
                                           const float* scale_host) {
  TB_REQUIRE(m && q_host && scale_host && layer >= 0 && layer < m->L && mat >= 0 && mat < 7);
  DeviceGuard guard(m->device);
  int8_t* q;
  float* s;
  lin_ptr(m, layer, mat, &q, &s);
  TB_CUDA(cudaMemcpy(q, q_host, lin_rows(m, mat) * lin_cols(m, mat), cudaMemcpyHostToDevice));
  TB_CUDA(cudaMemcpy(s, scale_host, lin_rows(m, mat) * lin_ng(m, mat) * sizeof(float), cudaMemcpyHostToDevice));
  return TB_SUCCESS;
}

extern "C" tb_status_t tb_model_get_linear(tb_model* m, int layer, int mat, int8_t* q_host, float* scale_host) {
  TB_REQUIRE(m && layer >= 0 && layer < m->L && mat >= 0 && mat < 7);
  DeviceGuard guard(m->device);
  int8_t* q;
  float* s;
  lin_ptr(m, layer, mat, &q, &s);
  TB_CUDA(cudaStreamSynchronize(m->stream));
  if (q_host) TB_CUDA(cudaMemcpy(q_host, q, lin_rows(m, mat) * lin_cols(m, mat), cudaMemcpyDeviceToHost));
  if (scale_host)
    TB_CUDA(cudaMemcpy(scale_host, s, lin_rows(m, mat) * lin_ng(m, mat) * sizeof(float), cudaMemcpyDeviceToHost));
  return TB_SUCCESS;
}

extern "C" tb_status_t tb_model_set_tensor(tb_model* m, int which, int layer, const float* host) {
  TB_REQUIRE(m && host && which >= 0 && which <= 4);
  DeviceGuard guard(m->device);
  float* dst = nullptr;
  size_t n = 0;
  switch (which) {
    case 0: dst = m->embed; n = (size_t)m->Vg * m->d; break;
    case 1: dst = m->lm_head; n = (size_t)m->V * m->d; break;
    case 2: dst = m->final_norm; n = (size_t)m->d; break;
    case 3: TB_REQUIRE(layer >= 0 && layer < m->L); dst = m->attn_norm + (size_t)layer * m->d; n = (size_t)m->d; break;
    default: TB_REQUIRE(layer >= 0 && layer < m->L); dst = m->mlp_norm + (size_t)layer * m->d; n = (size_t)m->d; break;
  }
  TB_CUDA(cudaMemcpy(dst, host, n * sizeof(float), cudaMemcpyHostToDevice));
  return TB_SUCCESS;
}

extern "C" tb_status_t tb_model_get_tensor(tb_model* m, int which, int layer, float* host) {
  TB_REQUIRE(m && host && which >= 0 && which <= 4);
  DeviceGuard guard(m->device);
  const float* src = nullptr;
  size_t n = 0;
  switch (which) {
    case 0: src = m->embed; n = (size_t)m->Vg * m->d; break;
    case 1: src = m->lm_head; n = (size_t)m->V * m->d; break;
    case 2: src = m->final_norm; n = (size_t)m->d; break;
    case 3: TB_REQUIRE(layer >= 0 && layer < m->L); src = m->attn_norm + (size_t)layer * m->d; n = (size_t)m->d; break;
    default: TB_REQUIRE(layer >= 0 && layer < m->L); src = m->mlp_norm + (size_t)layer * m->d; n = (size_t)m->d; break;
  }
  TB_CUDA(cudaStreamSynchronize(m->stream));
  TB_CUDA(cudaMemcpy(host, src, n * sizeof(float), cudaMemcpyDeviceToHost));
  return TB_SUCCESS;
}

extern "C" tb_status_t tb_model_bench_kernel(tb_model* m, int kind, int layer) {
  TB_REQUIRE(m && kind >= 0 && kind <= 5 && layer >= 0 && layer < m->L);
  TB_REQUIRE(m->fused && m->host_pos < m->Ms);
  DeviceGuard guard(m->device);
  return decode_kernel(m, kind, layer, false);
}

extern "C" tb_status_t tb_model_time_kernel(tb_model* m, int kind, int reps, float* us_per_launch) {
  TB_REQUIRE(m && us_per_launch && kind >= 0 && kind <= 5 && reps >= 1);
  TB_REQUIRE(m->fused && m->host_pos < m->Ms);
  DeviceGuard guard(m->device);
  // reps rounds over every layer's weights (so they stream from HBM), in one
  // CUDA graph, so the host launch cost is not part of the time
  cudaGraph_t g = nullptr;
  cudaGraphExec_t ge = nullptr;
  TB_CUDA(cudaStreamSynchronize(m->stream));
  TB_CUDA(cudaStreamBeginCapture(m->stream, cudaStreamCaptureModeThreadLocal));
  tb_status_t s = TB_SUCCESS;
  int64_t launches = 0;
  for (int r = 0; r < reps && s == TB_SUCCESS; r++)
    for (int64_t l = 0; l < m->L && s == TB_SUCCESS; l++, launches++) s = decode_kernel(m, kind, kind == 5 ? 0 : l, false);
  cudaError_t e = cudaStreamEndCapture(m->stream, &g);
  if (s != TB_SUCCESS) {
    if (g) cudaGraphDestroy(g);
    return s;
  }
  if (e != cudaSuccess) return tb::cuda_fail(e, "cudaStreamEndCapture");
  e = cudaGraphInstantiate(&ge, g, 0);
  cudaGraphDestroy(g);
  if (e != cudaSuccess) return tb::cuda_fail(e, "cudaGraphInstantiate");
  cudaEvent_t a = nullptr, b = nullptr;
  float ms = 0.f;
  e = cudaEventCreate(&a);
  if (e == cudaSuccess) e = cudaEventCreate(&b);
  if (e == cudaSuccess) e = cudaGraphLaunch(ge, m->stream);  // warm
  if (e == cudaSuccess) e = cudaEventRecord(a, m->stream);
  if (e == cudaSuccess) e = cudaGraphLaunch(ge, m->stream);
  if (e == cudaSuccess) e = cudaEventRecord(b, m->stream);
  if (e == cudaSuccess) e = cudaEventSynchronize(b);
  if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, a, b);
  if (a) cudaEventDestroy(a);
  if (b) cudaEventDestroy(b);
  cudaGraphExecDestroy(ge);
  if (e != cudaSuccess) return tb::cuda_fail(e, "tb_model_time_kernel");
  *us_per_launch = ms * 1000.0f / (float)launches;
  return TB_SUCCESS;
}

extern "C" tb_status_t tb_model_phase_times(tb_model* m, double* us, int max_entries, int* n_out) {
  TB_REQUIRE(m && us && n_out && max_entries >= 0);
  DeviceGuard guard(m->device);
  *n_out = 0;
  if (!m->mk) return TB_ERROR_NOT_SUPPORTED;
  TB_CUDA(cudaStreamSynchronize(m->stream));
  std::vector<uint64_t> t((size_t)m->trace_n);
  TB_CUDA(cudaMemcpy(t.data(), m->trace, sizeof(uint64_t) * t.size(), cudaMemcpyDeviceToHost));
  int n = 0;
  for (int i = 1; i < m->trace_n && n < max_entries; i++, n++) us[n] = (double)(t[i] - t[i - 1]) * 1e-3;
  *n_out = n;
  return TB_SUCCESS;
}

extern "C" tb_status_t tb_model_unit_times(tb_model* m, uint64_t* ns, int max_entries, int* n_out) {
  TB_REQUIRE(m && ns && n_out && max_entries >= 0);
  DeviceGuard guard(m->device);
  *n_out = 0;
  if (!m->mk) return TB_ERROR_NOT_SUPPORTED;
  TB_CUDA(cudaStreamSynchronize(m->stream));
  int n = 2 * tb::kMkUnitTrace;
  if (n > max_entries) n = max_entries;
  TB_CUDA(cudaMemcpy(ns, m->trace + m->trace_n, sizeof(uint64_t) * n, cudaMemcpyDeviceToHost));
  *n_out = n;
  return TB_SUCCESS;
}

extern "C" tb_status_t tb_model_last_logits(tb_model* m, float* logits_host) {
  TB_INJECT("tb_model_last_logits");
  TB_REQUIRE(m && logits_host);
  DeviceGuard guard(m->device);
  TB_CUDA(cudaStreamSynchronize(m->stream));
  TB_CUDA(cudaMemcpy(logits_host, m->logits, sizeof(float) * m->B * m->V, cudaMemcpyDeviceToHost));
  return TB_SUCCESS;
}

extern "C" tb_status_t tb_model_reset(tb_model* m) {
  TB_REQUIRE(m);
  DeviceGuard guard(m->device);
  TB_CUDA(cudaStreamSynchronize(m->stream));
  m->host_pos = 0;
  m->host_step = 0;
  TB_CUDA(cudaMemset(m->pos, 0, sizeof(int64_t)));
  TB_CUDA(cudaMemset(m->step, 0, sizeof(int64_t)));
  TB_CUDA(cudaMemset(m->keys, 0, sizeof(unsigned long long) * m->B));
  return TB_SUCCESS;
}

extern "C" int64_t tb_model_position(const tb_model* m) { return m ? m->host_pos : -1; }

extern "C" tb_status_t tb_model_set_position(tb_model* m, int64_t pos) {
  TB_REQUIRE(m && pos >= 0 && pos <= m->Ms);
  DeviceGuard guard(m->device);
  TB_CUDA(cudaStreamSynchronize(m->stream));
  m->host_pos = pos;
  TB_CUDA(cudaMemcpy(m->pos, &pos, sizeof(int64_t), cudaMemcpyHostToDevice));
  return TB_SUCCESS;
}

extern "C" tb_status_t tb_model_forward(tb_model* m, const int64_t* tokens_host, int64_t B, int64_t S,
                                        float* last_logits_host, int64_t* next_host) {
  TB_INJECT("tb_model_forward");
  TB_REQUIRE(m && tokens_host && B == m->B && S >= 1);
  TB_REQUIRE(m->host_pos + S <= m->Ms);  // nn/rope.go:109-111
  DeviceGuard guard(m->device);
  for (int64_t i = 0; i < B * S; i++) TB_REQUIRE(tokens_host[i] >= 0 && tokens_host[i] < m->Vg);
  TB_CUDA(cudaMemcpyAsync(m->ids, tokens_host, sizeof(int64_t) * B * S, cudaMemcpyHostToDevice, m->stream));
  TB_TRY(forward_tokens(m, S));
  if (last_logits_host)
    TB_CUDA(cudaMemcpyAsync(last_logits_host, m->logits, sizeof(float) * m->B * m->V, cudaMemcpyDeviceToHost, m->stream));
  if (next_host)
    TB_CUDA(cudaMemcpyAsync(next_host, m->tokens, sizeof(int64_t) * m->B, cudaMemcpyDeviceToHost, m->stream));
  TB_CUDA(cudaStreamSynchronize(m->stream));
  return TB_SUCCESS;
}

extern "C" tb_status_t tb_model_decode(tb_model* m, const int64_t* start_tokens_host, int64_t n_steps) {
  TB_INJECT("tb_model_decode");
  TB_REQUIRE(m && n_steps >= 0);
  TB_REQUIRE(m->host_pos + n_steps <= m->Ms);
  DeviceGuard guard(m->device);
  if (start_tokens_host) {
    for (int64_t i = 0; i < m->B; i++) TB_REQUIRE(start_tokens_host[i] >= 0 && start_tokens_host[i] < m->Vg);
    TB_CUDA(cudaMemcpyAsync(m->tokens, start_tokens_host, sizeof(int64_t) * m->B, cudaMemcpyHostToDevice, m->stream));
    TB_CUDA(cudaStreamSynchronize(m->stream));
  }
  if (m->fused) {
    TB_TRY(build_graph(m));
    for (int64_t i = 0; i < n_steps; i++) TB_CUDA(cudaGraphLaunch(m->graph, m->stream));
  } else {
    for (int64_t i = 0; i < n_steps; i++) {
      TB_CUDA(cudaMemcpyAsync(m->ids, m->tokens, sizeof(int64_t) * m->B, cudaMemcpyDeviceToDevice, m->stream));
      TB_TRY(forward_tokens(m, 1));  // advances host_pos and the history
    }
    return TB_SUCCESS;
  }
  m->host_pos += n_steps;
  m->host_step += n_steps;
  return TB_SUCCESS;
}

static tb_status_t check_waits(tb_model* m);

extern "C" tb_status_t tb_model_tokens(tb_model* m, int64_t* out_host, int64_t count) {
  TB_REQUIRE(m && out_host && count >= 0 && count <= m->hist_cap);
  DeviceGuard guard(m->device);
  TB_CUDA(cudaStreamSynchronize(m->stream));
  if (count) TB_CUDA(cudaMemcpy(out_host, m->history, sizeof(int64_t) * count * m->B, cudaMemcpyDeviceToHost));
  return check_waits(m);
}

// Device-side bounded waits that expired since the last check.
static tb_status_t check_waits(tb_model* m) {
  int v = 0, zero = 0;
  TB_CUDA(cudaMemcpy(&v, m->err_word, sizeof(int), cudaMemcpyDeviceToHost));
  if (tb::take_wait_timeouts() > 0) v = 1;  // the per-op kernels' bounded waits
  if (v) {
    TB_CUDA(cudaMemcpy(m->err_word, &zero, sizeof(int), cudaMemcpyHostToDevice));
    return TB_ERROR_TIMEOUT;
  }
  return TB_SUCCESS;
}

extern "C" tb_status_t tb_model_sync(tb_model* m) {
  TB_REQUIRE(m);
  DeviceGuard guard(m->device);
  TB_CUDA(cudaStreamSynchronize(m->stream));
  return check_waits(m);
}

extern "C" tb_stream_t tb_model_stream(tb_model* m) { return m ? (tb_stream_t)m->stream : nullptr; }

extern "C" int64_t tb_model_launches_per_step(const tb_model* m) {
  if (!m) return 0;
  if (!m->fused) return -1;
  // embedding + per layer (qkv, attention, combine, o, gate/up, down) + lm_head + tail
  if (m->mk) return 1;
  return 1 + m->L * 6 + 2;
}

namespace {

// After a step (greedy tail included): sample the step's logits instead and
// make the sampled tokens the step's output (tokens feed the next step).
tb_status_t sample_tail(tb_model* m, float temperature, int64_t top_k, float top_p, uint64_t seed, float* u) {
  cudaStream_t st = m->stream;
  TB_TRY(tb::sample_uniforms(u, m->step, m->B, seed, st));
  TB_TRY(tb_sample_f32(m->tokens, m->logits, u, m->B, m->V, temperature, top_k, top_p, (tb_stream_t)st));
  return tb::history_set(m->history, m->tokens, m->step, m->B, m->hist_cap, st);
}

}  // namespace

extern "C" tb_status_t tb_model_generate_sample(tb_model* m, const int64_t* prompt_host, int64_t B, int64_t S,
                                                int64_t n_new, float temperature, int64_t top_k, float top_p,
                                                uint64_t seed, int64_t* out_tokens_host) {
  TB_INJECT("tb_model_generate_sample");
  TB_REQUIRE(m && prompt_host && out_tokens_host && B == m->B && S >= 1 && n_new >= 1 && top_k >= 0);
  TB_REQUIRE(S + n_new - 1 <= m->Ms && n_new <= m->hist_cap);
  if (m->tp > 1) return TB_ERROR_NOT_SUPPORTED;  // the logits are sharded over the ranks
  DeviceGuard guard(m->device);
  float* u = m->samp_u;
  tb_status_t s = tb_model_reset(m);
  if (s == TB_SUCCESS) s = tb_model_forward(m, prompt_host, B, S, nullptr, nullptr);
  if (s == TB_SUCCESS) s = sample_tail(m, temperature, top_k, top_p, seed, u);
  for (int64_t i = 1; i < n_new && s == TB_SUCCESS; i++) {
    s = tb_model_decode(m, nullptr, 1);  // the step's logits (and its greedy choice, replaced below)
    if (s == TB_SUCCESS) s = sample_tail(m, temperature, top_k, top_p, seed, u);
  }
  TB_TRY(s);
  std::vector<int64_t> hist((size_t)(n_new * B));
  TB_TRY(tb_model_tokens(m, hist.data(), n_new));
  for (int64_t t = 0; t < n_new; t++)
    for (int64_t b = 0; b < B; b++) out_tokens_host[b * n_new + t] = hist[(size_t)(t * B + b)];
  return TB_SUCCESS;
}

extern "C" tb_status_t tb_model_generate_greedy(tb_model* m, const int64_t* prompt_host, int64_t B, int64_t S,
                                                int64_t n_new, int64_t* out_tokens_host) {
  TB_INJECT("tb_model_generate_greedy");
  TB_REQUIRE(m && prompt_host && out_tokens_host && B == m->B && S >= 1 && n_new >= 1);
  TB_REQUIRE(S + n_new - 1 <= m->Ms && n_new <= m->hist_cap);
  TB_TRY(tb_model_reset(m));
  TB_TRY(tb_model_forward(m, prompt_host, B, S, nullptr, nullptr));
  if (n_new > 1) TB_TRY(tb_model_decode(m, nullptr, n_new - 1));
  std::vector<int64_t> hist((size_t)(n_new * B));
  TB_TRY(tb_model_tokens(m, hist.data(), n_new));
  for (int64_t t = 0; t < n_new; t++)
    for (int64_t b = 0; b < B; b++) out_tokens_host[b * n_new + t] = hist[(size_t)(t * B + b)];
  return TB_SUCCESS;
}
