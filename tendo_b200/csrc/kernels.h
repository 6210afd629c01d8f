// kernels.h — internal launchers shared by the C ABI and the model engine.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/tendo_b200.h"

namespace tb {

struct QkvArgs {
  const float* h;       // residual stream [M, d]
  const float* norm_w;  // attn_norm [d]
  float eps;
  const int8_t* q;      // [(H + 2 Hkv) * D, d] = [Wq; Wk; Wv]
  const float* scale;   // [(H + 2 Hkv) * D]
  const float* cos_t;   // [max_seq, D/2]
  const float* sin_t;
  const int64_t* pos;   // device: current position
  float* qout;          // [M, H * D] post-RoPE
  float* kcache;        // [M, Hkv, max_seq, D] of this layer
  float* vcache;
  int M, d, H, Hkv, D, max_seq;
};

struct GateUpArgs {
  const float* h;
  const float* norm_w;
  float eps;
  const int8_t* gate;  // [F, d]
  const int8_t* up;    // [F, d]
  const float* gate_scale;
  const float* up_scale;
  float* act;  // [M, F]
  int M, d, F;
};

struct LmHeadArgs {
  const float* h;
  const float* norm_w;
  float eps;
  const float* w;  // [V, d] fp32
  float* logits;   // [M, V] (may be null)
  unsigned long long* argmax_keys;  // [M] (may be null)
  int M, d, V;
  int v0;  // vocabulary index of row 0 (tensor-parallel shards)
  bool l2_prefetch;
};

struct AttnDecodeArgs {
  const float* q;       // [B, H, D]
  const void* kcache;   // [B, Hkv, max_seq, D] fp32 (bf16 with kv_bf16)
  const void* vcache;
  float* out;           // [B, H, D]
  float* partial;       // [B, H, nsplit, D + 2] workspace
  const int64_t* pos;   // device position of the newest key (Sk = *pos + 1); null: use sk
  int64_t sk;
  int B, H, Hkv, D, max_seq, nsplit;
  float scale;
  bool l2_prefetch;  // set by the launcher
  bool kv_bf16;
};

// decode_mk.cu: the whole batch-1 decode step as one persistent kernel.
struct MkArgs {
  int L, d, H, Hkv, D, F, V, max_seq, nsplit;
  float eps, attn_scale;
  const int8_t* wqkv;  // [L][(H + 2 Hkv) D][d]
  const float* sqkv;
  const int8_t* wo;  // [L][d][H D]
  const float* so;
  const int8_t* wg;  // [L][F][d]
  const float* sg;
  const int8_t* wu;
  const float* su;
  const int8_t* wd;  // [L][d][F]
  const float* sd;
  const float* attn_norm;  // [L][d]
  const float* mlp_norm;
  const float* final_norm;
  const float* embed;    // [V][d]
  const float* lm_head;  // [V][d]
  const float* cos_t;
  const float* sin_t;
  float* kc;  // [L][Hkv][max_seq][D]
  float* vc;
  float* h;  // [d] residual stream after the last layer
  // Tagged exchange words (megakernel_ll_words of them, zeroed at creation):
  // each holds an fp32 value in its low half and the epoch tag of the phase
  // that wrote it in its high half, so a reader polls the data itself.
  unsigned long long* ll;
  unsigned int* epoch;  // decode steps run so far (tags of step e are unique to it)
  float* logits;  // [V]
  unsigned long long* keys;
  int64_t* tokens;
  int64_t* history;
  int64_t* step;
  int64_t* pos;
  int64_t hist_cap;
  unsigned int* bar_counter;  // arrivals at the step's final barrier (zeroed by the launch)
  int* err;                   // bounded waits that expired
  uint64_t* trace;            // optional: CTA 0 phase stamps (ns)
  uint64_t* utrace;           // optional: CTA 0 weight-stream units: [2 u] issued, [2 u + 1] landed (ns)
  // filled by megakernel_launch: sizes, and the shared-memory layout and
  // exchange-buffer offsets (kept in the parameter bank, not in registers)
  int kmax_bytes, xbuf_floats, tiles_max, tiles_res, RSX;
  size_t merge_bytes;
  uint32_t sm_dig, sm_xbuf, sm_ssc, sm_res, sm_rope, sm_red, sm_bar;
  uint32_t ll_q, ll_kv, ll_part, ll_attn, ll_h, ll_act;
};
// weight-stream units of CTA 0 whose issue and landing times the unit trace keeps
constexpr int kMkUnitTrace = 4096;
// phase stamps of one persistent decode step: start, 13 per layer, 3 for the
// lm_head (norm, tiles up to the final barrier, barrier)
inline int megakernel_trace_stamps(int L) { return 1 + 13 * L + 3; }
bool megakernel_supported(int d, int H, int Hkv, int D, int F, int V, int batch);
// attention splits per kv head of the persistent kernel (one split per CTA)
int megakernel_splits(int Hkv);
// tagged exchange words MkArgs::ll holds
size_t megakernel_ll_words(int d, int H, int Hkv, int D, int F, int nsplit);
tb_status_t megakernel_launch(MkArgs a, cudaStream_t st);

// gemv.cu
bool gemv_fast_ok(const float* x, const int8_t* q, int64_t K);
tb_status_t gemv_plain(float* out, const float* x, const int8_t* q, const float* scale, const float* resid, int M,
                       int N, int K, const float* norm_w, float eps, cudaStream_t st, bool pdl);
tb_status_t gemv_generic(float* out, const float* x, const int8_t* q, const float* scale, int M, int N, int K, int g,
                         cudaStream_t st);
tb_status_t gemv_qkv_rope(const QkvArgs& a, cudaStream_t st, bool pdl);
tb_status_t gemv_gateup(const GateUpArgs& a, cudaStream_t st, bool pdl);
tb_status_t gemv_lmhead(const LmHeadArgs& a, cudaStream_t st, bool pdl);

// gemv_mma.cu: the same GEMVs on the tensor cores (M <= 8, K % 64 == 0)
bool gemv_mma_ok(const float* x, const int8_t* q, int64_t M, int64_t K);
tb_status_t gemv_mma_plain(float* out, const float* x, const int8_t* q, const float* scale, const float* resid, int M,
                           int N, int K, const float* norm_w, float eps, cudaStream_t st, bool pdl);
tb_status_t gemv_mma_qkv(const QkvArgs& a, cudaStream_t st, bool pdl);
tb_status_t gemv_mma_gateup(const GateUpArgs& a, cudaStream_t st, bool pdl);
// TMA-fed tensor-core GEMVs (weights streamed to shared memory by cp.async.bulk).
bool gemv_tma_ok(const float* x, const int8_t* q, int64_t M, int64_t K);
tb_status_t gemv_tma_plain(float* out, const float* x, const int8_t* q, const float* scale, const float* resid, int M,
                           int N, int K, const float* norm_w, float eps, cudaStream_t st, bool pdl);
tb_status_t gemv_tma_qkv(const QkvArgs& a, cudaStream_t st, bool pdl);
tb_status_t gemv_tma_gateup(const GateUpArgs& a, cudaStream_t st, bool pdl);
// Bounded device waits that expired since the last call (and resets the count).
int take_wait_timeouts();
// Device address of that count, for kernels in other files.
int* wait_timeout_word();
// Kernel family of the decode GEMVs (TENDO_B200_GEMV = tma | mma | simt; default tma).
enum class GemvKind { kTma, kMma, kSimt };
GemvKind gemv_kind();
inline bool gemv_use_mma() { return gemv_kind() == GemvKind::kMma; }
bool l2_prefetch_enabled();

// attention.cu
// Split count of the decode attention: about four CTAs per SM; for grids of
// several waves, the count whose last wave of resident CTAs is fullest.
int attn_decode_splits(int B, int H, int Hkv, int D, int64_t max_seq, bool kv_bf16 = false);
size_t attn_decode_workspace(int B, int H, int D, int nsplit);
tb_status_t attn_decode(const AttnDecodeArgs& a, cudaStream_t st, bool pdl);
tb_status_t attn_prefill(float* out, const float* q, const void* kcache, const void* vcache, int B, int H,
                         int Hkv, int Sq, int64_t Sk, int D, int max_seq, float scale, cudaStream_t st,
                         bool kv_bf16 = false);

// gemm_tc.cu: the prefill-regime quantized Linear on the 5th-generation
// tensor cores.  x rows are split into `planes` int8 digit rows
// (x = s_m (d0 + d1 / 128 [+ d2 / 128^2]), optionally of RMSNorm(x) * norm_w),
// then out[M, N] = s_m scale[n] sum_p 128^-p (d_p . q_n) (+ resid) with the
// digit products summed exactly in s32 by tcgen05.mma kind::i8.
size_t gemm_tc_workspace(int64_t M, int64_t K, int planes);
bool gemm_tc_ok(const void* q, int64_t M, int64_t N, int64_t K);
tb_status_t gemm_tc_digits(int8_t* dig, float* srow, const float* x, int M, int K, int planes, const float* norm_w,
                           float eps, cudaStream_t st);
tb_status_t gemm_tc_run(float* out, const int8_t* dig, const float* srow, const int8_t* q, const float* scale,
                        const float* resid, int M, int N, int K, int planes, cudaStream_t st);
// digits + GEMM with the digit rows in `ws` (gemm_tc_workspace bytes).
tb_status_t gemm_tc(float* out, const float* x, const int8_t* q, const float* scale, const float* resid, int M, int N,
                    int K, int planes, void* ws, cudaStream_t st);
// per-group scales [N, K / group] (group a multiple of 128, K / group <= 128):
// digits + the grouped GEMM, digit rows in `ws` (gemm_tc_workspace bytes).
bool gemm_tc_grp_ok(const void* q, int64_t M, int64_t N, int64_t K, int64_t group);
tb_status_t gemm_tc_grp(float* out, const float* x, const int8_t* q, const float* scale, const float* resid, int M,
                        int N, int K, int group, int planes, void* ws, cudaStream_t st);

// gemv_tc.cu: the same product for 1 <= M <= kGemvTcMaxM on tcgen05 with the
// weights as the 128-row MMA operand and the work split evenly over the SMs
// by K blocks (split tiles finished by the last CTA to arrive).
// `zeroed` (gemv_tc_zeroed_bytes) holds counters and split-tile sums and is
// zero before and after each launch (zero_first: clear it first); `scratch`
// (gemv_tc_scratch_bytes) holds the digit rows (and, for per-group scales,
// the split tiles' fp32 partial rows).  group > 0: scale is [N, K / group],
// group a multiple of 128.
constexpr int kGemvTcMaxM = 64;
size_t gemv_tc_zeroed_bytes(int64_t M, int64_t N, int64_t K);
size_t gemv_tc_scratch_bytes(int64_t M, int64_t N, int64_t K, int64_t group = 0);
bool gemv_tc_ok(const void* q, int64_t M, int64_t N, int64_t K, int64_t group = 0);

// gemv_ring.cu: the quantized Linear for 1 <= M <= 5 rows, per-channel scales,
// K a multiple of 64, x and q 16-byte aligned; no workspace.
bool gemv_ring_ok(const float* x, const int8_t* q, int64_t M, int64_t N, int64_t K);
tb_status_t gemv_ring(float* out, const float* x, const int8_t* q, const float* scale, const float* resid, int M,
                      int N, int K, cudaStream_t st);
// norm_w != null: the product is of RMSNorm(x) * norm_w (the digit kernel applies it).
// digits_ready: `scratch` already holds the digit rows of this x (and norm)
// from the previous call with the same M and K (digit-kernel path only).
tb_status_t gemv_tc(float* out, const float* x, const int8_t* q, const float* scale, const float* resid, int M, int N,
                    int K, void* zeroed, bool zero_first, void* scratch, cudaStream_t st,
                    const float* norm_w = nullptr, float eps = 0.f, int group = 0, bool digits_ready = false);

// comm.cu: in-place NCCL allreduce on `st` (fp32 sum, or uint64 max for the
// packed greedy keys); a no-op without a communicator or with one rank.
// In-place sum (fp32) or max (uint64) over the communicator's ranks: the
// peer-memory kernel up to the exchange capacity, NCCL past it.  Expired
// device waits count in *err (the global wait-timeout word when null).
tb_status_t allreduce(tb_comm* c, void* buf, size_t count, bool u64_max, cudaStream_t st, int* err = nullptr);
bool peer_allreduce_active(const tb_comm* c);
int comm_rank(const tb_comm* c);
int comm_size(const tb_comm* c);

// gemm.cu: out[M, N] = x[M, K] @ (q * scale)^T (+ resid) on CUDA cores.
tb_status_t gemm_simt_i8(float* out, const float* x, const int8_t* q, const float* scale, const float* resid,
                         int M, int N, int K, int group, cudaStream_t st);
tb_status_t gemm_f32_nt(float* out, const float* a, const float* b, int M, int N, int K, cudaStream_t st);

// quant.cu: shards of the synthetic weights (tensor parallelism): rows
// row0.. of a K-column matrix (scales over the full row), columns col0..col0+cols.
tb_status_t synth_quant_shard(int8_t* q, float* scale, int64_t rows, int64_t K, int64_t row0, int64_t col0,
                              int64_t cols, uint64_t seed, uint64_t stream_id, double std_, cudaStream_t st);
// The same draw quantized per group of `group` kept columns: scale [rows][cols / group].
tb_status_t synth_quant_shard_grp(int8_t* q, float* scale, int64_t rows, int64_t K, int64_t row0, int64_t col0,
                                  int64_t cols, int64_t group, uint64_t seed, uint64_t stream_id, double std_,
                                  cudaStream_t st);
tb_status_t synth_normal_rows(float* w, int64_t rows, int64_t K, int64_t row0, uint64_t seed, uint64_t stream_id,
                              double std_, cudaStream_t st);

// ops.cu
tb_status_t embedding(float* out, const float* table, const int64_t* ids, int64_t n, int64_t vocab, int64_t dim,
                      int32_t* bad, cudaStream_t st, bool pdl);
tb_status_t rmsnorm(float* out, float* resid_out, const float* in, const float* resid, const float* w, int64_t rows,
                    int64_t d, float eps, cudaStream_t st);
// kc, vc: fp32 caches, or bf16 ones with kv_bf16
tb_status_t kv_append_rope(void* kc, void* vc, const float* k, const float* v, const float* cos_t,
                           const float* sin_t, int64_t B, int64_t Hkv, int64_t S, int64_t D, int64_t pos,
                           int64_t max_seq, int64_t ld, cudaStream_t st, bool kv_bf16 = false);
tb_status_t rope_rows(float* x, const float* cos_t, const float* sin_t, int64_t B, int64_t S, int64_t Hx, int64_t D,
                      int64_t pos, int64_t ld, cudaStream_t st);
tb_status_t silu_mul(float* out, const float* gate, const float* up, int64_t n, cudaStream_t st);
// out[m, j] = silu(gu[m, j]) * gu[m, F + j] for B rows of 2F values
tb_status_t silu_mul_rows(float* out, const float* gu, int64_t B, int64_t F, cudaStream_t st);
// Decode step, B rows of qkv [B][(H + 2 Hkv) D]: RoPE on the q and k heads at
// the device position *pos; q heads to q [B][H][D], k and v heads to the
// caches [B][Hkv][max_seq][D] at *pos (v unrotated; fp32, or bf16 with kv_bf16).
tb_status_t qkv_rope_append(float* q, void* kc, void* vc, const float* qkv, const float* cos_t, const float* sin_t,
                            const int64_t* pos, int64_t B, int64_t H, int64_t Hkv, int64_t D, int64_t max_seq,
                            cudaStream_t st, bool kv_bf16 = false);
tb_status_t argmax_rows(int64_t* out, const float* x, int64_t rows, int64_t n, cudaStream_t st);
// The sampler's uniforms for the token the last step generated, and the
// history entry of that step set to the (sampled) tokens.
tb_status_t sample_uniforms(float* u, const int64_t* step, int64_t B, uint64_t seed, cudaStream_t st);
tb_status_t history_set(int64_t* history, const int64_t* tokens, const int64_t* step, int64_t B, int64_t hist_cap,
                        cudaStream_t st);
// keys[r] = max(keys[r], packed (x[r][j], v0 + j)) over the row: the greedy
// choice as one orderable word (larger logit first, lower index on ties).
tb_status_t argmax_keys(unsigned long long* keys, const float* x, int64_t rows, int64_t n, int64_t v0,
                        cudaStream_t st);
// Decode-step tail: token[m] from the argmax key, history append, key reset, position + 1.
tb_status_t finish_step(unsigned long long* keys, int64_t* tokens, int64_t* history, int64_t* step, int64_t* pos,
                        int M, int64_t hist_cap, cudaStream_t st, bool pdl);

}  // namespace tb
