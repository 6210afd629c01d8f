/*
 * tendo_b200.h — C ABI of libtendo_b200.so, the B200 (sm_100a) kernels for
 * tendo's int8-quantized Llama inference path.
 *
 * Conventions (those of tendo's popcorn binding, cuda/popcorn.go:21-37):
 *  - every entry point returns a tb_status_t, TB_SUCCESS == 0;
 *  - tb_get_error_string(status) names a status; after TB_ERROR_CUDA,
 *    tb_get_last_cuda_error_string() holds the CUDA error text;
 *  - all tensor arguments are device pointers to contiguous row-major
 *    arrays, unless a parameter says "host";
 *  - kernels run on the stream passed in (NULL = legacy default stream) and
 *    on the device that is current on the calling thread;
 *  - the op entry points allocate nothing: output and workspace buffers come
 *    from the caller, who owns every buffer.
 * Only the tb_model_* engine allocates, once, at creation.
 */
#ifndef TENDO_B200_H
#define TENDO_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(TB_BUILDING_LIBRARY)
#define TB_API __attribute__((visibility("default")))
#else
#define TB_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* tb_stream_t; /* == cudaStream_t */

typedef enum {
  TB_SUCCESS = 0,
  TB_ERROR_INVALID_ARGUMENT = 1, /* bad size, null pointer, misaligned buffer */
  TB_ERROR_CUDA = 2,             /* a CUDA runtime call or launch failed */
  TB_ERROR_NOT_SUPPORTED = 3,    /* valid request this build does not handle */
  TB_ERROR_OUT_OF_MEMORY = 4,    /* engine allocation failed */
  TB_ERROR_TIMEOUT = 5,          /* a bounded device-side wait gave up */
  TB_ERROR_INJECTED = 6          /* host-side fault injection (TENDO_B200_INJECT) */
} tb_status_t;

/* popcornGetErrorString (cuda/popcorn.go:25). */
TB_API const char* tb_get_error_string(tb_status_t status);
/* popcornGetLastCudaErrorString (cuda/popcorn.go:28); per calling thread. */
TB_API const char* tb_get_last_cuda_error_string(void);
/* Library version, major * 10000 + minor * 100 + patch. */
TB_API int tb_version(void);

/* ---------------------------------------------------------------------------
 * Quantization (nn/quantize.go)
 * ------------------------------------------------------------------------- */

/* Symmetric absmax int8 quantization of w[N, K] (fp32): replaces the host
 * loops of nn.Quantize -> quantizePerChannel (nn/quantize.go:42-124) and
 * quantizePerGroup (nn/quantize.go:126-187).  group_size 0 = per output
 * channel (scale[N]); otherwise scale[N, K / group_size].  q and scale are
 * bit-identical to the reference: scale = maxAbs / 127 (1 when 0),
 * q = clamp(round_half_away(w / scale), -128, 127). */
TB_API tb_status_t tb_quantize_i8_f32(int8_t* q, float* scale, const float* w, int64_t N, int64_t K,
                               int64_t group_size, tb_stream_t stream);

/* Packs the reference's float32-coded q values ("stored as float32 but values
 * are int8 range", nn/quantize.go:68) into int8.  Values must be integers in
 * [-128, 127]; anything else sets *bad_count (device int32, may be NULL). */
TB_API tb_status_t tb_pack_q_f32_to_i8(int8_t* q, const float* q_f32, int64_t n, int32_t* bad_count,
                                tb_stream_t stream);

/* QuantizedTensor.Dequantize (nn/quantize.go:191-229): w = q * scale. */
TB_API tb_status_t tb_dequantize_i8_f32(float* w, const int8_t* q, const float* scale, int64_t N, int64_t K,
                                 int64_t group_size, tb_stream_t stream);

/* ---------------------------------------------------------------------------
 * Quantized Linear (nn/quantize.go:251-312)
 * ------------------------------------------------------------------------- */

/* out[M, N] = x[M, K] @ dequantize(q[N, K], scale)^T, fp32 in and out.
 * Replaces popcornDequantizeMatmul_i8f32 (cuda/popcorn.go:1306-1315, per
 * channel) and popcornDequantizeMatmulGrouped_i8f32 (cuda/popcorn.go:1353-1363,
 * group_size > 0), reached from cuda.Backend.DequantizeMatmul
 * (cuda/backend.go:676-721).  Every tensor-core path splits each row of x
 * into three int8 digit rows (x = s (d0 + d1/128 + d2/128^2), s = max|x|/127)
 * and sums every digit row times the raw int8 weights exactly in s32, so the
 * result is within 2^-21 s sum|w| of the fp32 product.  Routing:
 *   M <= 5, per-channel scales, K % 64 == 0: one weight stream through a
 *     shared-memory ring per SM, integer mma.sync (no workspace);
 *   M <= 32 otherwise: tcgen05.mma kind::i8 with the weights as the 128-row
 *     operand and the (tile, K block) work split evenly over the SMs
 *     (K % 128 == 0; other K run the CUDA-core GEMV);
 *   M > 32: tcgen05 128 x 128 output tiles.
 * Per-group scales (group_size > 0) take the tcgen05 paths when the group is
 * a multiple of 128 (M > 32: at most 128 groups per row): the exact s32 sum
 * of each group is scaled by scale[n, group] and added in fp32 in a fixed
 * order; other group sizes run the CUDA-core kernels.
 * Scratch: this entry point keeps library-owned buffers per device,
 * allocated on first use and grown on demand (calls that overlap in time on
 * one device must use tb_dequant_matmul_i8f32_ws). */
TB_API tb_status_t tb_dequant_matmul_i8f32(float* out, const float* x, const int8_t* q, const float* scale,
                                    int64_t M, int64_t N, int64_t K, int64_t group_size,
                                    tb_stream_t stream);

/* Quantized-Linear kernel modes. */
typedef enum {
  TB_GEMM_I8X3 = 0, /* tcgen05 kind::i8, three digit rows of x: within 2^-21 s sum|w| (default) */
  TB_GEMM_I8X2 = 1, /* M > 32: two digit rows, within 2^-14 s sum|w|, 1.5x fewer MMAs (M <= 32: as I8X3) */
  TB_GEMM_SIMT = 2  /* fp32 CUDA-core kernels (no tensor cores) */
} tb_gemm_mode_t;

/* tb_dequant_matmul_i8f32 with the GEMM mode chosen by the caller (used for
 * M > 32; M <= 32 always takes the GEMV). */
TB_API tb_status_t tb_dequant_matmul_i8f32_mode(float* out, const float* x, const int8_t* q, const float* scale,
                                         int64_t M, int64_t N, int64_t K, int64_t group_size,
                                         tb_gemm_mode_t mode, tb_stream_t stream);

/* Scratch bytes tb_dequant_matmul_i8f32_ws needs for these sizes and mode
 * (0 when no scratch is used: TB_GEMM_SIMT, M <= 32 with K not a multiple
 * of 128, per-group scales with a group that is not a multiple of 128 or,
 * for M > 32, more than 128 groups per row). */
TB_API size_t tb_dequant_matmul_workspace_size(int64_t M, int64_t N, int64_t K, int64_t group_size,
                                               tb_gemm_mode_t mode);

/* tb_dequant_matmul_i8f32_mode with caller-owned scratch (the Go backend's
 * pool): allocates nothing; any contents on entry.  workspace_bytes below the
 * size above returns TB_ERROR_INVALID_ARGUMENT. */
TB_API tb_status_t tb_dequant_matmul_i8f32_ws(float* out, const float* x, const int8_t* q, const float* scale,
                                              int64_t M, int64_t N, int64_t K, int64_t group_size,
                                              tb_gemm_mode_t mode, void* workspace, size_t workspace_bytes,
                                              tb_stream_t stream);

/* out[M, N] = a[M, K] @ b[N, K]^T in fp32: the fp32 lm_head projection
 * (models/llama/quantized.go:164-172, cuBLAS SGEMM in cuda/ops.go:182-330). */
TB_API tb_status_t tb_matmul_nt_f32(float* out, const float* a, const float* b, int64_t M, int64_t N, int64_t K,
                             tb_stream_t stream);

/* ---------------------------------------------------------------------------
 * Norm, activation, elementwise (cpu/backend.go; cuda/popcorn.go; cuDNN)
 * ------------------------------------------------------------------------- */

/* popcornRMSNorm_f32 (cuda/popcorn.go:615-623): out = x / sqrt(mean(x^2) + eps)
 * * weight over the last norm_size elements of n rows; weight may be NULL.
 * residual != NULL fuses the residual add first: x = in + residual, and x is
 * also written to residual_out (may alias residual). */
TB_API tb_status_t tb_rmsnorm_f32(float* out, const float* in, const float* weight, int64_t n, int64_t norm_size,
                           float eps, tb_stream_t stream);
TB_API tb_status_t tb_add_rmsnorm_f32(float* out, float* residual_out, const float* in, const float* residual,
                               const float* weight, int64_t n, int64_t norm_size, float eps,
                               tb_stream_t stream);

/* SiLU (cuDNN swish, cuda/ops.go:14-86; cpu/backend.go:193-198). */
TB_API tb_status_t tb_silu_f32(float* out, const float* in, int64_t n, tb_stream_t stream);
/* SwiGLU glue: out = silu(gate) * up (models/llama/quantized.go:392-404). */
TB_API tb_status_t tb_silu_mul_f32(float* out, const float* gate, const float* up, int64_t n, tb_stream_t stream);
/* Residual Add (models/llama/quantized.go:199, :219; cudnnOpTensor). */
TB_API tb_status_t tb_add_f32(float* out, const float* a, const float* b, int64_t n, tb_stream_t stream);

/* ---------------------------------------------------------------------------
 * Generic fp32 tensor ops of llama.Backend (models/llama/forward.go:13-27)
 *
 * The ops unchanged models/llama attention issues between its projections
 * (quantized.go:282-372): Q.K^T and P.V on strided views, the scale Mul, the
 * causal mask (Ones, Tril, Full, Where), Softmax and the KV-cache Cat.  Each
 * takes views as (rank, shape, element strides per dimension; a stride of 0
 * broadcasts or expands) and writes a new contiguous tensor of the output
 * shape, as the reference backends return new tensors.  NULL strides mean
 * contiguous.  Shape and stride arrays are HOST memory; data pointers are
 * device memory.  Arithmetic in the reference CPU backend's order
 * (cpu/backend.go).
 * ------------------------------------------------------------------------- */

#define TB_MAX_RANK 6

typedef enum { TB_BINARY_ADD = 0, TB_BINARY_SUB = 1, TB_BINARY_MUL = 2, TB_BINARY_DIV = 3 } tb_binary_op_t;

/* Full / Ones / Zeros (cpu/backend.go:60-86; cuda/backend.go:88-96): n
 * elements set to value. */
TB_API tb_status_t tb_fill_f32(float* out, float value, int64_t n, tb_stream_t stream);
/* Add / Sub / Mul / Div with broadcasting (cpu/backend.go:257-271,
 * binaryElementwise :1511-1560; cuda/backend.go:244-266): out[i] =
 * a[i] op b[i] in float32 over `shape`; a broadcast operand has stride 0. */
TB_API tb_status_t tb_binary_f32(float* out, const float* a, const float* b, int op, int rank, const int64_t* shape,
                          const int64_t* a_strides, const int64_t* b_strides, tb_stream_t stream);
/* Where (cpu/backend.go:1191-1255; cuda/backend.go:644): out = cond > 0 ? x : y. */
TB_API tb_status_t tb_where_f32(float* out, const float* cond, const float* x, const float* y, int rank,
                         const int64_t* shape, const int64_t* cond_strides, const int64_t* x_strides,
                         const int64_t* y_strides, tb_stream_t stream);
/* Tril (cpu/backend.go:1257-1285; cuda/backend.go:650) of a contiguous 2-D
 * tensor: keeps [r, c] where c <= r + k, else 0. */
TB_API tb_status_t tb_tril_f32(float* out, const float* in, int64_t rows, int64_t cols, int64_t k, tb_stream_t stream);
/* Softmax along dim (cpu/backend.go:1690-1744; cuDNN in cuda/ops.go:88-180):
 * per slice the max seeded at -MaxFloat32, exp(x - max) in double precision
 * rounded to float, a sequential float32 sum, then x / sum. */
TB_API tb_status_t tb_softmax_f32(float* out, const float* in, int rank, const int64_t* shape,
                           const int64_t* in_strides, int dim, tb_stream_t stream);
/* MatMul (cpu/backend.go:281-308 via gonum Gemm; cuBLAS in cuda/backend.go:268)
 * over batch dimensions: out[batch..., M, N] = sum_k a[batch..., m, k] *
 * b[batch..., k, n], with a's element (m, k) at a_rs m + a_cs k plus its batch
 * offset and b's (k, n) at b_rs k + b_cs n (a transposed view is a stride
 * swap; a broadcast batch dimension has stride 0).  Products rounded, then
 * summed in k order. */
TB_API tb_status_t tb_matmul_f32(float* out, const float* a, const float* b, int batch_rank,
                          const int64_t* batch_shape, const int64_t* a_batch_strides,
                          const int64_t* b_batch_strides, int64_t M, int64_t N, int64_t K, int64_t a_rs,
                          int64_t a_cs, int64_t b_rs, int64_t b_cs, tb_stream_t stream);
/* Cat of two tensors along dim (cpu/backend.go:1343-1407; popcornCat_f32,
 * cuda/popcorn.go:1077-1085): out has a's shape with a_shape[dim] +
 * b_shape[dim] along dim. */
TB_API tb_status_t tb_cat_f32(float* out, const float* a, const float* b, int rank, const int64_t* a_shape,
                       const int64_t* a_strides, const int64_t* b_shape, const int64_t* b_strides, int dim,
                       tb_stream_t stream);

/* ---------------------------------------------------------------------------
 * RoPE and attention (nn/rope.go; models/llama/quantized.go:229-382)
 * ------------------------------------------------------------------------- */

/* NewRoPE tables (nn/rope.go:22-52), computed on the HOST into host arrays
 * cos_t/sin_t [max_seq, dim / 2] with fp64 pow/cos/sin as the reference does. */
TB_API tb_status_t tb_rope_tables_host(float* cos_t, float* sin_t, int dim, int max_seq, float base);

/* RoPE.Apply / rotateHalf (nn/rope.go:102-197) on x[B, Hx, S, D] (contiguous),
 * positions pos_offset .. pos_offset + S - 1; out may alias x. */
TB_API tb_status_t tb_rope_apply_f32(float* out, const float* x, const float* cos_t, const float* sin_t, int64_t B,
                              int64_t Hx, int64_t S, int64_t D, int64_t pos_offset, int64_t max_seq,
                              tb_stream_t stream);

/* KV-cache append (the Cat along dim 2 of models/llama/quantized.go:282-299,
 * popcornCat_f32 cuda/popcorn.go:1077-1085) done in place, with RoPE fused on
 * k.  k, v: [B, S, Hkv, D] projections (the layout the Linear writes);
 * kcache, vcache: [B, Hkv, max_seq, D]; positions pos .. pos + S - 1. */
TB_API tb_status_t tb_kv_append_rope_f32(float* kcache, float* vcache, const float* k, const float* v,
                                  const float* cos_t, const float* sin_t, int64_t B, int64_t Hkv, int64_t S,
                                  int64_t D, int64_t pos, int64_t max_seq, tb_stream_t stream);

/* Scaled-dot-product attention over the cache: scores = (q . k) * scale,
 * causal mask keeps key j for query i when j <= i + (Sk - Sq), softmax over
 * keys, then P . V (models/llama/quantized.go:319-372, forward.go:345-417).
 * q: [B, Sq, H, D] (post-RoPE, the projection layout), caches
 * [B, Hkv, max_seq, D] holding Sk valid positions; GQA maps query head h to
 * kv head h / (H / Hkv).  out: [B, Sq, H, D].  Sq == 1 runs the split-K
 * decode kernel, which needs `workspace` of tb_attention_workspace_size()
 * bytes (device memory owned by the caller; its contents need not be zero).
 * Calls that share a workspace must not overlap on the GPU. */
TB_API size_t tb_attention_workspace_size(int64_t B, int64_t H, int64_t Sq, int64_t D, int64_t max_seq);
TB_API tb_status_t tb_attention_f32(float* out, const float* q, const float* kcache, const float* vcache, int64_t B,
                             int64_t H, int64_t Hkv, int64_t Sq, int64_t Sk, int64_t D, int64_t max_seq,
                             float scale, void* workspace, size_t workspace_bytes, tb_stream_t stream);

/* Decode attention (Sq == 1) that allocates nothing and takes no workspace.
 * No counterpart in the reference: tendo allocates every buffer through its
 * backend.  It exists for callers that cannot call cudaMalloc at all, such as
 * a host that reserves the whole GPU into its own pools at start-up, or a
 * foreign-language binding whose only device allocator is its own tensor
 * pool and cannot lend a per-call scratch buffer.  Same math and result
 * layout as tb_attention_f32 with Sq == 1.  Its split-K partials live in one
 * library-owned device array of TB_ATTENTION_NOALLOC_SCRATCH_BYTES per GPU
 * (kept until the process exits); sizes whose partials do not fit are
 * rejected with TB_ERROR_INVALID_ARGUMENT.  Each call looks up that array's
 * address on the current device (cudaGetSymbolAddress); the first call on a
 * device also loads the library's device code there, so make that first call
 * before any stream capture.  Every call on a device shares the
 * array, so calls that overlap on the GPU (different streams, or host
 * threads without ordering) race and corrupt each other's partials. */
#define TB_ATTENTION_NOALLOC_SCRATCH_BYTES (2u * 1024u * 1024u)
TB_API tb_status_t tb_attention_decode_noalloc_f32(float* out, const float* q, const float* kcache,
                                                   const float* vcache, int64_t B, int64_t H, int64_t Hkv,
                                                   int64_t Sk, int64_t D, int64_t max_seq, float scale,
                                                   tb_stream_t stream);

/* ---------------------------------------------------------------------------
 * Embedding and sampling
 * ------------------------------------------------------------------------- */

/* popcornEmbedding_f32 (cuda/popcorn.go:980-988): out[i, :] = table[ids[i], :].
 * Out-of-range ids produce zero rows and set *bad_count (device int32, may be
 * NULL) — the Go CPU path panics there. */
TB_API tb_status_t tb_embedding_f32(float* out, const float* table, const int64_t* ids, int64_t n, int64_t vocab,
                             int64_t dim, int32_t* bad_count, tb_stream_t stream);

/* popcornArgMax_f32 (cuda/popcorn.go:458-464) with models.Greedy's tie rule
 * (models/sampling.go:73-83, first index of the maximum): out_idx[r] for each
 * of `rows` rows of length n. */
TB_API tb_status_t tb_argmax_f32(int64_t* out_idx, const float* x, int64_t rows, int64_t n, tb_stream_t stream);

/* ---------------------------------------------------------------------------
 * Synthetic workload generator (include/tendo_synth.h), on the device
 * ------------------------------------------------------------------------- */

/* w[N, K] with w[n, k] = N(0, std) draw n*K + k of (seed, stream), fp32. */
TB_API tb_status_t tb_synth_normal_f32(float* w, int64_t N, int64_t K, uint64_t seed, uint64_t stream_id, double std_,
                                tb_stream_t stream);
/* Generates and quantizes per channel in one pass (no fp32 copy kept):
 * the device form of nn.Quantize applied to tb_synth_normal_f32's matrix. */
TB_API tb_status_t tb_synth_quantized_i8(int8_t* q, float* scale, int64_t N, int64_t K, uint64_t seed,
                                  uint64_t stream_id, double std_, tb_stream_t stream);
/* Host: n uniform token ids in [0, vocab) of (seed, TS_STREAM_PROMPT). */
TB_API tb_status_t tb_synth_tokens_host(int64_t* ids, int64_t n, int64_t vocab, uint64_t seed);

/* ---------------------------------------------------------------------------
 * Model engine: QuantizedModel (models/llama/quantized.go:13-477)
 * ------------------------------------------------------------------------- */

typedef struct {
  int32_t vocab, dim, layers, heads, kv_heads, hidden, max_seq;
  float rope_base, eps;
  int32_t max_batch; /* sequences decoded in lockstep */
} tb_model_config;

typedef struct tb_model tb_model;

/* Allocates weights, KV cache and work buffers on `device`. */
TB_API tb_status_t tb_model_create(tb_model** out, const tb_model_config* cfg, int device);

/* Sampler.Sample (models/sampling.go:47-70) on the device for B rows of
 * [V] logits: temperature (x / T when T != 1 and T > 0), top-k by value (0 or
 * >= V: off), top-p (0 or >= 1: off), then the first index whose fp32
 * cumulative probability exceeds uniforms[b] (the caller's draw in [0, 1),
 * the reference's rng.Float32()), in the reference's arithmetic and order;
 * top-p orders every remaining candidate, as applyTopP (:99-124) does.
 * V <= 40000.  Greedy is tb_argmax_f32. */
TB_API tb_status_t tb_sample_f32(int64_t* tokens, const float* logits, const float* uniforms, int64_t B, int64_t V,
                                 float temperature, int64_t top_k, float top_p, tb_stream_t stream);

/* ---------------------------------------------------------------------------
 * Tensor parallelism (the 70B shape over 2/4/8 GPUs)
 * ------------------------------------------------------------------------- */

/* A communicator over the ranks of one tensor-parallel group, one process (or
 * thread) per GPU: NCCL, loaded at run time (libnccl.so.2).  Rank 0 makes the
 * unique id, the caller distributes its bytes to every rank (any channel),
 * and each rank creates its communicator with it (collective: every rank
 * calls it).  Creation also maps every rank's peer-exchange region (8 MB per
 * rank of the group) into every other rank (CUDA IPC; up to 8 ranks on one
 * node); allreduces of up to 2 MB then run as one kernel over peer memory,
 * larger ones through NCCL.  If
 * any rank cannot map a peer, or TENDO_B200_ALLREDUCE=nccl is set, every
 * rank uses NCCL throughout.  The tb_comm_init / tb_allreduce_sum_f32 pair
 * planned for the reference's cgo layer. */
typedef struct tb_comm tb_comm;
TB_API size_t tb_comm_unique_id_bytes(void);
TB_API tb_status_t tb_comm_unique_id(void* id_out, size_t bytes);
TB_API tb_status_t tb_comm_create(tb_comm** out, const void* id, size_t bytes, int rank, int nranks, int device);
TB_API tb_status_t tb_comm_destroy(tb_comm* comm);
/* 1 when the communicator's allreduces run over peer memory, 0 when NCCL. */
TB_API int tb_comm_peer_active(const tb_comm* comm);
/* In-place fp32 sum over the ranks on `stream`.  Every rank gets the same
 * bits: the peer kernel adds the ranks' values in rank order. */
TB_API tb_status_t tb_allreduce_sum_f32(tb_comm* comm, float* buf, int64_t n, tb_stream_t stream);

/* The model's share on rank r of a tensor-parallel group of `nranks` GPUs
 * (models/llama/quantized.go layers, sharded Megatron-style): column-parallel
 * Wq/Wk/Wv (heads r H/n .. (r+1) H/n, kv heads likewise), Wgate/Wup (rows
 * r F/n ..) and the fp32 lm_head (vocabulary rows r V/n ..); row-parallel Wo
 * and Wdown (their input columns), followed by an allreduce of the residual
 * stream; embedding and norms replicated.  Greedy tokens come from an
 * allreduce (max) of packed (logit, index) keys, lowest index on ties as
 * models/sampling.go:73-83.  Needs heads, kv_heads, hidden and vocab
 * divisible by nranks.  Every rank calls the same model functions in the
 * same order. */
TB_API tb_status_t tb_model_create_tp(tb_model** out, const tb_model_config* cfg, int device, tb_comm* comm);

/* Model options for tb_model_create_ex. */
#define TB_MODEL_KV_BF16 1u /* KV cache in bf16 (rounded to nearest even when
                             * appended): half the cache bytes; a numerics
                             * change against the reference's fp32 cache.
                             * Decodes through the tcgen05 GEMV path (batch
                             * <= 64) or the per-step kernels. */

/* tb_model_create / tb_model_create_tp (comm may be null) with options. */
TB_API tb_status_t tb_model_create_ex(tb_model** out, const tb_model_config* cfg, int device, tb_comm* comm,
                                      uint32_t flags);
/* The model with every Linear quantized per group of group_size input
 * columns (QuantizeModel(m, groupSize), models/llama/quantized.go:52-73;
 * nn/quantize.go:126-187): scales [rows][K / group_size] in
 * tb_model_set_linear / tb_model_get_linear and in the synthetic weights.
 * group_size 0 is tb_model_create_ex.  Every Linear's input width (on a
 * tensor-parallel rank, its share of Wo and Wdown) must be a multiple of
 * group_size (TB_ERROR_NOT_SUPPORTED otherwise).  Decode runs the tcgen05
 * GEMV with per-group scales (group_size a multiple of 128, up to 64
 * sequences; other sizes run the per-step DequantizeMatmul); prefill runs
 * the grouped DequantizeMatmul; the batch-1 persistent kernel and the fused
 * per-channel kernels are not used. */
TB_API tb_status_t tb_model_create_grouped(tb_model** out, const tb_model_config* cfg, int device, tb_comm* comm,
                                           uint32_t flags, int64_t group_size);
TB_API tb_status_t tb_model_destroy(tb_model* m);
/* Synthetic weights: N(0, 0.02) from (seed, stream = layer * 8 + matrix),
 * quantized per channel (per group for tb_model_create_grouped) on the
 * device; gains 1.0; embedding and lm_head fp32. */
TB_API tb_status_t tb_model_init_synthetic(tb_model* m, uint64_t seed);
/* Loads one quantized Linear (mat 0..6 = q, k, v, o, gate, up, down) from
 * HOST arrays q[N, K] int8 and scale[N]; which = 0 embedding [V, d],
 * 1 lm_head [V, d], 2 final norm [d], 3 attn norm of `layer`, 4 mlp norm. */
TB_API tb_status_t tb_model_set_linear(tb_model* m, int layer, int mat, const int8_t* q_host, const float* scale_host);
TB_API tb_status_t tb_model_set_tensor(tb_model* m, int which, int layer, const float* host);
/* Copies a tensor set by tb_model_set_tensor back to a host array. */
TB_API tb_status_t tb_model_get_tensor(tb_model* m, int which, int layer, float* host);
/* Copies one quantized Linear back to host arrays. */
TB_API tb_status_t tb_model_get_linear(tb_model* m, int layer, int mat, int8_t* q_host, float* scale_host);
/* ExtractLastLogits (models/sampling.go:214-243): the logits [B, V] of the
 * last forward or decode step (this rank's vocabulary rows under tensor
 * parallelism) copied to a host array, after the engine stream drains. */
TB_API tb_status_t tb_model_last_logits(tb_model* m, float* logits_host);
/* Empties the KV cache (position 0). */
TB_API tb_status_t tb_model_reset(tb_model* m);
TB_API int64_t tb_model_position(const tb_model* m);

/* QuantizedModel.Forward (models/llama/quantized.go:125-178) over tokens
 * [B, S] (HOST int64) appended at the current position.  last_logits_host
 * [B, vocab] (may be NULL) receives the last position's logits and
 * next_host[B] (may be NULL) their greedy argmax. */
TB_API tb_status_t tb_model_forward(tb_model* m, const int64_t* tokens_host, int64_t B, int64_t S,
                             float* last_logits_host, int64_t* next_host);

/* QuantizedModel.Generate with the Sampler (models/llama/quantized.go:422-477,
 * models/sampling.go:47-70): the prompt, then n_new tokens per sequence, each
 * drawn on the device (tb_sample_f32) from the step's logits with the uniform
 * draw (seed, step * B + row) of the library's counter generator, so no
 * logits leave the GPU.  One GPU (not tensor parallel). */
TB_API tb_status_t tb_model_generate_sample(tb_model* m, const int64_t* prompt_host, int64_t B, int64_t S,
                                            int64_t n_new, float temperature, int64_t top_k, float top_p,
                                            uint64_t seed, int64_t* out_tokens_host);

/* GenerateGreedy (models/llama/generate.go:99-150): reset, prefill with
 * prompt[B, S] (HOST), then n_new greedy tokens into out_tokens_host[B, n_new].
 * Each decode step is one CUDA-graph launch that reads the token and position
 * from device memory, so only the token ids cross back to the host. */
TB_API tb_status_t tb_model_generate_greedy(tb_model* m, const int64_t* prompt_host, int64_t B, int64_t S,
                                     int64_t n_new, int64_t* out_tokens_host);

/* Device-resident decode: runs n_steps greedy steps from the current
 * position, feeding each argmax back as the next token, and keeps the tokens
 * on the device (fetch them with tb_model_tokens).  `start_tokens_host` [B]
 * (may be NULL = continue from the last token).  Asynchronous on the engine
 * stream; tb_model_sync waits. */
TB_API tb_status_t tb_model_decode(tb_model* m, const int64_t* start_tokens_host, int64_t n_steps);
TB_API tb_status_t tb_model_tokens(tb_model* m, int64_t* out_host, int64_t count);
TB_API tb_status_t tb_model_set_position(tb_model* m, int64_t pos);
TB_API tb_status_t tb_model_sync(tb_model* m);
/* The engine's CUDA stream (for events). */
TB_API tb_stream_t tb_model_stream(tb_model* m);
/* Launches one kernel of the fused decode step for `layer` on the engine
 * stream, without graph or programmatic launch, for timing it alone: kind
 * 0 = RMSNorm+QKV+RoPE+append GEMV, 1 = split-K attention + combine,
 * 2 = O GEMV + residual, 3 = RMSNorm+gate/up+SwiGLU GEMV, 4 = down GEMV +
 * residual, 5 = final RMSNorm + lm_head GEMV + argmax.  Reads and writes
 * the engine's own buffers at the current position. */
TB_API tb_status_t tb_model_bench_kernel(tb_model* m, int kind, int layer);
/* Times one kernel kind of the decode step: `reps` rounds over all layers'
 * weights launched from one CUDA graph (no host launch cost in the time),
 * timed with CUDA events on the engine stream; *us_per_launch = average. */
TB_API tb_status_t tb_model_time_kernel(tb_model* m, int kind, int reps, float* us_per_launch);
/* Phase timeline of the last persistent decode step (batch-1 engines): us[i]
 * = time between consecutive stamps taken by CTA 0: per layer 13 intervals
 * (qkv staging, tiles, epilogue; attention; then staging, tiles and epilogue
 * of o, gate/up and down; a staging interval includes the wait for the
 * previous phase's results), then the lm_head's norm, its tiles up to the
 * step's final barrier, and that barrier.
 * TB_ERROR_NOT_SUPPORTED when the engine decodes with separate kernels. */
TB_API tb_status_t tb_model_phase_times(tb_model* m, double* us, int max_entries, int* n_out);
/* Weight-stream trace of the last persistent decode step (batch-1 engines):
 * for the first 4096 stream units of CTA 0 (a unit = 8 weight rows x one
 * chunk of at most 4 KB), ns[2 u] = globaltimer when the producer issued its
 * copies and ns[2 u + 1] = when the consumers found it landed.
 * TB_ERROR_NOT_SUPPORTED when the engine decodes with separate kernels. */
TB_API tb_status_t tb_model_unit_times(tb_model* m, uint64_t* ns, int max_entries, int* n_out);
/* Kernel launches one decode step issues. */
TB_API int64_t tb_model_launches_per_step(const tb_model* m);

#ifdef __cplusplus
}
#endif
#endif /* TENDO_B200_H */
