// gemv.cu — decode-regime (M <= 32) dequant GEMV kernels: the plain
// tb_dequant_matmul path and the fused variants the model engine chains
// (RMSNorm prologue; RoPE + KV append, residual and SwiGLU epilogues; the
// fp32 lm_head with a fused greedy argmax).
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include "gemv.cuh"
#include "kernels.h"

namespace tb {
namespace {

__device__ __forceinline__ int group_stride() { return gridDim.x * (blockDim.x >> 5); }
__device__ __forceinline__ int first_group() { return blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); }

// Loads in flight per lane: U chunks of each of ROWS rows.
template <int MT, int ROWS>
struct Unroll {
  static constexpr int U = (MT <= 2 ? 8 : 4) / ROWS;
};

// ---------------------------------------------------------------------------
// Plain GEMV: out[m, n] = scale[n] * x[m, :] . q[n, :] (+ resid[m, n]).
// ---------------------------------------------------------------------------
template <int MT>
__global__ void __launch_bounds__(kGemvThreads) gemv_plain_kernel(float* out, const float* __restrict__ x,
                                                                  const int8_t* __restrict__ q,
                                                                  const float* __restrict__ scale,
                                                                  const float* resid, int M, int N, int K,
                                                                  const float* __restrict__ norm_w, float eps) {
  constexpr int ROWS = 1;
  extern __shared__ __align__(16) float xs[];
  const int ngroups = (N + ROWS - 1) / ROWS;
  int g = first_group();
  const int8_t* rp[ROWS];
  if (g < ngroups) {
#pragma unroll
    for (int r = 0; r < ROWS; r++) rp[r] = q + (size_t)min(g * ROWS + r, N - 1) * K;
    prefetch_rows<ROWS>(rp, K);
  }
  pdl_wait();
  pdl_launch_dependents();
  stage_x<MT>(xs, x, K, M, K, norm_w, eps, xs + MT * K);
  for (; g < ngroups; g += group_stride()) {
#pragma unroll
    for (int r = 0; r < ROWS; r++) rp[r] = q + (size_t)min(g * ROWS + r, N - 1) * K;
    float acc[ROWS][MT];
    gemv_rows<MT, ROWS, Unroll<MT, ROWS>::U>(acc, rp, xs, K);
    if ((threadIdx.x & 31) == 0) {
#pragma unroll
      for (int r = 0; r < ROWS; r++) {
        const int n = g * ROWS + r;
        if (n < N) {
          const float s = scale[n];
#pragma unroll
          for (int m = 0; m < MT; m++) {
            if (m < M) {
              float v = acc[r][m] * s;
              if (resid) v += resid[(size_t)m * N + n];
              out[(size_t)m * N + n] = v;
            }
          }
        }
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Fused Q/K/V projection of the decode step: x = RMSNorm(h) * attn_norm,
// rows of the concatenated [Wq; Wk; Wv] processed in rotate-half pairs
// (i, i + D/2) of one head, RoPE applied to q and k at position *pos, k and
// v written straight into the KV cache (the in-place form of the Cat append).
// ---------------------------------------------------------------------------
template <int MT>
__global__ void __launch_bounds__(kGemvThreads) gemv_qkv_rope_kernel(QkvArgs a) {
  constexpr int ROWS = 2;  // one rotate-half pair
  extern __shared__ __align__(16) float xs[];
  const int half = a.D / 2;
  const int npairs = (a.H + 2 * a.Hkv) * half;
  const int ngroups = npairs;
  const int K = a.d;
  int g = first_group();
  const int8_t* rp[ROWS];
  int rows[ROWS];
  auto map = [&](int gg) {
    const int t = gg / half, i = gg - t * half;
    rows[0] = t * a.D + i;
    rows[1] = t * a.D + i + half;
#pragma unroll
    for (int r = 0; r < ROWS; r++) rp[r] = a.q + (size_t)rows[r] * K;
  };
  if (g < ngroups) {
    map(g);
    prefetch_rows<ROWS>(rp, K);
  }
  pdl_wait();
  pdl_launch_dependents();
  stage_x<MT>(xs, a.h, K, a.M, K, a.norm_w, a.eps, xs + MT * K);
  const int64_t pos = *a.pos;
  for (; g < ngroups; g += group_stride()) {
    map(g);
    float acc[ROWS][MT];
    gemv_rows<MT, ROWS, Unroll<MT, ROWS>::U>(acc, rp, xs, K);
    const int lane = threadIdx.x & 31;
    {
      constexpr int p = 0;
      const int t = g / half, i = g - t * half;
      const float s0 = a.scale[rows[2 * p]], s1 = a.scale[rows[2 * p + 1]];
      const float c = a.cos_t[pos * half + i], sn = a.sin_t[pos * half + i];
#pragma unroll
      for (int m = 0; m < MT; m++) {
        if (m >= a.M || lane != m) continue;  // lane m stores sequence m
        const float x0 = acc[2 * p][m] * s0, x1 = acc[2 * p + 1][m] * s1;
        if (t < a.H) {
          float* o = a.qout + (size_t)m * a.H * a.D + (size_t)t * a.D;
          o[i] = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, sn));
          o[i + half] = __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, c));
        } else if (t < a.H + a.Hkv) {
          float* o = a.kcache + (((size_t)m * a.Hkv + (t - a.H)) * a.max_seq + pos) * a.D;
          o[i] = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, sn));
          o[i + half] = __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, c));
        } else {
          float* o = a.vcache + (((size_t)m * a.Hkv + (t - a.H - a.Hkv)) * a.max_seq + pos) * a.D;
          o[i] = x0;
          o[i + half] = x1;
        }
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Fused gate/up projection + SwiGLU: x = RMSNorm(h) * mlp_norm, rows
// (gate j, up j, gate j+1, up j+1), act[m, j] = silu(gate) * up with
// silu(g) = g * (1 / (1 + exp(-g))) (cpu/backend.go:193-198).
// ---------------------------------------------------------------------------
template <int MT>
__global__ void __launch_bounds__(kGemvThreads) gemv_gateup_kernel(GateUpArgs a) {
  constexpr int ROWS = 2;
  extern __shared__ __align__(16) float xs[];
  const int K = a.d, F = a.F;
  const int ngroups = F;
  int g = first_group();
  const int8_t* rp[ROWS];
  auto map = [&](int gg) {
    rp[0] = a.gate + (size_t)gg * K;
    rp[1] = a.up + (size_t)gg * K;
  };
  if (g < ngroups) {
    map(g);
    prefetch_rows<ROWS>(rp, K);
  }
  pdl_wait();
  pdl_launch_dependents();
  stage_x<MT>(xs, a.h, K, a.M, K, a.norm_w, a.eps, xs + MT * K);
  for (; g < ngroups; g += group_stride()) {
    map(g);
    float acc[ROWS][MT];
    gemv_rows<MT, ROWS, Unroll<MT, ROWS>::U>(acc, rp, xs, K);
    const int lane = threadIdx.x & 31;
    {
      constexpr int p = 0;
      const int j = g;
      const float sg = a.gate_scale[j], su = a.up_scale[j];
#pragma unroll
      for (int m = 0; m < MT; m++) {
        if (m >= a.M || lane != m) continue;
        const float gv = acc[2 * p][m] * sg, uv = acc[2 * p + 1][m] * su;
        const float sig = 1.0f / (1.0f + expf(-gv));
        a.act[(size_t)m * F + j] = (gv * sig) * uv;
      }
    }
  }
}

// ---------------------------------------------------------------------------
// fp32-weight GEMV for the lm_head: logits[m, n] = x[m, :] . W[n, :] with
// x = RMSNorm(h) * final_norm, and a greedy argmax folded in: each warp keeps
// the best (value, lowest index) per sequence and merges it into a 64-bit key
// with atomicMax (value made order-preserving in the high word, the index
// complemented in the low word so that ties keep the first index,
// models/sampling.go:73-83).
// ---------------------------------------------------------------------------
__device__ __forceinline__ unsigned long long argmax_key(float v, int idx) {
  uint32_t u = __float_as_uint(v);
  u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return ((unsigned long long)u << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)idx);
}

template <int MT>
__global__ void __launch_bounds__(kGemvThreads) gemv_lmhead_kernel(LmHeadArgs a) {
  constexpr int ROWS = 2;
  extern __shared__ __align__(16) float xs[];  // plain layout: x[m][k]
  float* red = xs + MT * a.d;
  const int K = a.d, N = a.V;
  const int ngroups = (N + ROWS - 1) / ROWS;
  const int lane = threadIdx.x & 31;
  int g = first_group();
  // TMA bulk prefetch of this warp's next kAhead row pairs into L2.
  constexpr int kAhead = 4;
  auto prefetch_task = [&](int task) {
    if (task < ngroups) {
      const int r0 = task * ROWS, rows = min(ROWS, N - r0);
      if (rows > 0 && (K * 4) % 16 == 0) prefetch_l2_bulk(a.w + (size_t)r0 * K, (uint32_t)(rows * K * 4));
    }
  };
  const bool l2pf = a.l2_prefetch;
  if (l2pf && lane == 0)
    for (int i = 0; i < kAhead; i++) prefetch_task(g + i * group_stride());
  pdl_wait();
  pdl_launch_dependents();
  // RMSNorm prologue in the plain layout.
  {
    float ss[MT];
#pragma unroll
    for (int m = 0; m < MT; m++) ss[m] = 0.f;
    for (int v = threadIdx.x; v < K / 4; v += blockDim.x)
#pragma unroll
      for (int m = 0; m < MT; m++)
        if (m < a.M) {
          float4 t = reinterpret_cast<const float4*>(a.h + (size_t)m * K)[v];
          ss[m] += t.x * t.x + t.y * t.y + t.z * t.z + t.w * t.w;
        }
    const int warp = threadIdx.x >> 5;
#pragma unroll
    for (int m = 0; m < MT; m++) {
      float s = warp_sum(ss[m]);
      if (lane == 0) red[m * kGemvWarps + warp] = s;
    }
    __syncthreads();
    float rms[MT];
#pragma unroll
    for (int m = 0; m < MT; m++) {
      float s = 0.f;
      for (int w = 0; w < (int)(blockDim.x >> 5); w++) s += red[m * kGemvWarps + w];
      rms[m] = __fsqrt_rn(__fadd_rn(__fdiv_rn(s, (float)K), a.eps));
    }
    for (int v = threadIdx.x; v < K / 4; v += blockDim.x) {
      float4 w = reinterpret_cast<const float4*>(a.norm_w)[v];
#pragma unroll
      for (int m = 0; m < MT; m++) {
        float4 t = make_float4(0.f, 0.f, 0.f, 0.f);
        if (m < a.M) {
          t = reinterpret_cast<const float4*>(a.h + (size_t)m * K)[v];
          t.x = __fmul_rn(__fdiv_rn(t.x, rms[m]), w.x);
          t.y = __fmul_rn(__fdiv_rn(t.y, rms[m]), w.y);
          t.z = __fmul_rn(__fdiv_rn(t.z, rms[m]), w.z);
          t.w = __fmul_rn(__fdiv_rn(t.w, rms[m]), w.w);
        }
        reinterpret_cast<float4*>(xs + (size_t)m * K)[v] = t;
      }
    }
    __syncthreads();
  }
  unsigned long long best[MT];
#pragma unroll
  for (int m = 0; m < MT; m++) best[m] = 0ull;
  const float4* xv = reinterpret_cast<const float4*>(xs);
  const int nv = K / 4;
  for (; g < ngroups; g += group_stride()) {
    if (l2pf && lane == 0) prefetch_task(g + kAhead * group_stride());
    const float4* rp[ROWS];
#pragma unroll
    for (int r = 0; r < ROWS; r++) rp[r] = reinterpret_cast<const float4*>(a.w + (size_t)min(g * ROWS + r, N - 1) * K);
    float acc[ROWS][MT];
#pragma unroll
    for (int r = 0; r < ROWS; r++)
#pragma unroll
      for (int m = 0; m < MT; m++) acc[r][m] = 0.f;
    int v = lane;
    for (; v + 96 < nv; v += 128) {
      int4 w[ROWS][4];
#pragma unroll
      for (int r = 0; r < ROWS; r++)
#pragma unroll
        for (int u = 0; u < 4; u++) w[r][u] = ld_stream_v4(rp[r] + v + 32 * u);
#pragma unroll
      for (int u = 0; u < 4; u++)
#pragma unroll
        for (int m = 0; m < MT; m++) {
          const float4 xx = xv[(size_t)m * nv + v + 32 * u];
#pragma unroll
          for (int r = 0; r < ROWS; r++) {
            float s = acc[r][m];
            s = fmaf(xx.x, __int_as_float(w[r][u].x), s);
            s = fmaf(xx.y, __int_as_float(w[r][u].y), s);
            s = fmaf(xx.z, __int_as_float(w[r][u].z), s);
            s = fmaf(xx.w, __int_as_float(w[r][u].w), s);
            acc[r][m] = s;
          }
        }
    }
    for (; v < nv; v += 32) {
#pragma unroll
      for (int r = 0; r < ROWS; r++) {
        const int4 w = ld_stream_v4(rp[r] + v);
#pragma unroll
        for (int m = 0; m < MT; m++) {
          const float4 xx = xv[(size_t)m * nv + v];
          float s = acc[r][m];
          s = fmaf(xx.x, __int_as_float(w.x), s);
          s = fmaf(xx.y, __int_as_float(w.y), s);
          s = fmaf(xx.z, __int_as_float(w.z), s);
          s = fmaf(xx.w, __int_as_float(w.w), s);
          acc[r][m] = s;
        }
      }
    }
#pragma unroll
    for (int r = 0; r < ROWS; r++)
#pragma unroll
      for (int m = 0; m < MT; m++) acc[r][m] = warp_sum(acc[r][m]);
#pragma unroll
    for (int r = 0; r < ROWS; r++) {
      const int n = g * ROWS + r;
      if (n >= N) continue;
#pragma unroll
      for (int m = 0; m < MT; m++) {
        if (m >= a.M) continue;
        if (lane == m && a.logits) a.logits[(size_t)m * N + n] = acc[r][m];
        const unsigned long long k = argmax_key(acc[r][m], n + a.v0);
        best[m] = k > best[m] ? k : best[m];
      }
    }
  }
  if (a.argmax_keys && lane == 0) {
#pragma unroll
    for (int m = 0; m < MT; m++)
      if (m < a.M && best[m] != 0ull) atomicMax(a.argmax_keys + m, best[m]);
  }
}

// ---------------------------------------------------------------------------
// Generic fallback: any K, any alignment, per-channel or per-group scales.
// One warp per (row, block of 8 x rows); the weight is dequantized to fp32
// first (q * scale, as QuantizedTensor.Dequantize does) and multiplied in.
// ---------------------------------------------------------------------------
__global__ void gemv_generic_kernel(float* out, const float* __restrict__ x, const int8_t* __restrict__ q,
                                    const float* __restrict__ scale, int M, int N, int K, int g) {
  const int lane = threadIdx.x & 31;
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int nwarps = (gridDim.x * blockDim.x) >> 5;
  const int ng = K / g;
  const int mblocks = (M + 7) / 8;
  for (int task = warp; task < N * mblocks; task += nwarps) {
    const int n = task / mblocks, m0 = (task % mblocks) * 8;
    float acc[8];
#pragma unroll
    for (int i = 0; i < 8; i++) acc[i] = 0.f;
    for (int k = lane; k < K; k += 32) {
      const float w = __fmul_rn((float)q[(size_t)n * K + k], scale[(size_t)n * ng + k / g]);
#pragma unroll
      for (int i = 0; i < 8; i++)
        if (m0 + i < M) acc[i] = fmaf(x[(size_t)(m0 + i) * K + k], w, acc[i]);
    }
#pragma unroll
    for (int i = 0; i < 8; i++) {
      float s = warp_sum(acc[i]);
      if (lane == 0 && m0 + i < M) out[(size_t)(m0 + i) * N + n] = s;
    }
  }
}

template <typename Kern, typename... Args>
tb_status_t launch(Kern kern, GemvPlan plan, size_t smem, cudaStream_t st, bool pdl, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(plan.grid);
  cfg.blockDim = dim3(plan.warps * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, args...);
  if (e != cudaSuccess) return cuda_fail(e, "cudaLaunchKernelEx(gemv)");
  return TB_SUCCESS;
}

template <typename Kern>
tb_status_t set_smem(Kern kern, size_t smem) {
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(smem)");
  }
  return TB_SUCCESS;
}

// One CTA per SM, warps chosen so the tasks divide evenly (gemv.cuh).
GemvPlan gemv_grid(int64_t tasks, size_t smem) {
  (void)smem;
  return gemv_plan(tasks, sm_count(), kGemvWarps);
}

int mt_for(int M) { return M <= 1 ? 1 : (M <= 2 ? 2 : (M <= 4 ? 4 : 8)); }

template <template <int> class K_, typename... Args>
struct MtDispatch;

}  // namespace

// Largest x rows one staged pass holds for this K (shared-memory bound).
static int max_mt_for_k(int K) {
  const size_t cap = 200 * 1024;
  int mt = 8;
  while (mt > 1 && gemv_smem_bytes(mt, K) > cap) mt >>= 1;
  return mt;
}

bool gemv_fast_ok(const float* x, const int8_t* q, int64_t K) {
  return K % 16 == 0 && aligned(x, 16) && aligned(q, 16) && gemv_smem_bytes(1, (int)K) <= 200 * 1024;
}

tb_status_t gemv_plain(float* out, const float* x, const int8_t* q, const float* scale, const float* resid,
                       int M, int N, int K, const float* norm_w, float eps, cudaStream_t st, bool pdl) {
  const GemvKind kind = gemv_kind();
  const bool tma = kind == GemvKind::kTma && gemv_tma_ok(x, q, M < 8 ? M : 8, K);
  const bool mma = kind == GemvKind::kMma && gemv_mma_ok(x, q, M < 8 ? M : 8, K);
  if (tma || mma) {
    for (int m0 = 0; m0 < M; m0 += 8) {
      const int mm = M - m0 < 8 ? M - m0 : 8;
      float* o = out + (size_t)m0 * N;
      const float* xx = x + (size_t)m0 * K;
      const float* rr = resid ? resid + (size_t)m0 * N : nullptr;
      if (tma)
        TB_TRY(gemv_tma_plain(o, xx, q, scale, rr, mm, N, K, norm_w, eps, st, pdl));
      else
        TB_TRY(gemv_mma_plain(o, xx, q, scale, rr, mm, N, K, norm_w, eps, st, pdl));
    }
    return TB_SUCCESS;
  }
  const int mt_cap = max_mt_for_k(K);
  for (int m0 = 0; m0 < M; m0 += mt_cap) {
    const int mm = M - m0 < mt_cap ? M - m0 : mt_cap;
    const int MT = mt_for(mm);
    const size_t smem = gemv_smem_bytes(MT, K);
    const GemvPlan grid = gemv_grid(N, smem);
    float* o = out + (size_t)m0 * N;
    const float* xx = x + (size_t)m0 * K;
    const float* rr = resid ? resid + (size_t)m0 * N : nullptr;
    switch (MT) {
      case 1:
        TB_TRY(set_smem(gemv_plain_kernel<1>, smem));
        TB_TRY(launch(gemv_plain_kernel<1>, grid, smem, st, pdl, o, xx, q, scale, rr, mm, N, K, norm_w, eps));
        break;
      case 2:
        TB_TRY(set_smem(gemv_plain_kernel<2>, smem));
        TB_TRY(launch(gemv_plain_kernel<2>, grid, smem, st, pdl, o, xx, q, scale, rr, mm, N, K, norm_w, eps));
        break;
      case 4:
        TB_TRY(set_smem(gemv_plain_kernel<4>, smem));
        TB_TRY(launch(gemv_plain_kernel<4>, grid, smem, st, pdl, o, xx, q, scale, rr, mm, N, K, norm_w, eps));
        break;
      default:
        TB_TRY(set_smem(gemv_plain_kernel<8>, smem));
        TB_TRY(launch(gemv_plain_kernel<8>, grid, smem, st, pdl, o, xx, q, scale, rr, mm, N, K, norm_w, eps));
        break;
    }
  }
  return TB_SUCCESS;
}

tb_status_t gemv_generic(float* out, const float* x, const int8_t* q, const float* scale, int M, int N, int K,
                         int g, cudaStream_t st) {
  const int64_t tasks = (int64_t)N * ((M + 7) / 8);
  int64_t blocks = (tasks + 7) / 8;
  const int64_t cap = (int64_t)sm_count() * 8;
  if (blocks > cap) blocks = cap;
  gemv_generic_kernel<<<(unsigned)blocks, 256, 0, st>>>(out, x, q, scale, M, N, K, g);
  return check_launch("gemv_generic_kernel");
}

tb_status_t gemv_qkv_rope(const QkvArgs& a, cudaStream_t st, bool pdl) {
  TB_REQUIRE(a.M >= 1 && a.M <= 8 && a.d % 16 == 0 && a.D % 2 == 0);
  if (gemv_kind() == GemvKind::kTma && a.D % 8 == 0 && gemv_tma_ok(a.h, a.q, a.M, a.d)) return gemv_tma_qkv(a, st, pdl);
  if (gemv_use_mma() && a.D % 8 == 0 && gemv_mma_ok(a.h, a.q, a.M, a.d)) return gemv_mma_qkv(a, st, pdl);
  const int MT = mt_for(a.M);
  const size_t smem = gemv_smem_bytes(MT, a.d);
  const int64_t groups = (int64_t)(a.H + 2 * a.Hkv) * (a.D / 2);
  const GemvPlan grid = gemv_grid(groups, smem);
  switch (MT) {
    case 1: TB_TRY(set_smem(gemv_qkv_rope_kernel<1>, smem)); return launch(gemv_qkv_rope_kernel<1>, grid, smem, st, pdl, a);
    case 2: TB_TRY(set_smem(gemv_qkv_rope_kernel<2>, smem)); return launch(gemv_qkv_rope_kernel<2>, grid, smem, st, pdl, a);
    case 4: TB_TRY(set_smem(gemv_qkv_rope_kernel<4>, smem)); return launch(gemv_qkv_rope_kernel<4>, grid, smem, st, pdl, a);
    default: TB_TRY(set_smem(gemv_qkv_rope_kernel<8>, smem)); return launch(gemv_qkv_rope_kernel<8>, grid, smem, st, pdl, a);
  }
}

tb_status_t gemv_gateup(const GateUpArgs& a, cudaStream_t st, bool pdl) {
  TB_REQUIRE(a.M >= 1 && a.M <= 8 && a.d % 16 == 0);
  if (gemv_kind() == GemvKind::kTma && gemv_tma_ok(a.h, a.gate, a.M, a.d) && tb::aligned(a.up, 16))
    return gemv_tma_gateup(a, st, pdl);
  if (gemv_use_mma() && gemv_mma_ok(a.h, a.gate, a.M, a.d) && tb::aligned(a.up, 16)) return gemv_mma_gateup(a, st, pdl);
  const int MT = mt_for(a.M);
  const size_t smem = gemv_smem_bytes(MT, a.d);
  const GemvPlan grid = gemv_grid(a.F, smem);
  switch (MT) {
    case 1: TB_TRY(set_smem(gemv_gateup_kernel<1>, smem)); return launch(gemv_gateup_kernel<1>, grid, smem, st, pdl, a);
    case 2: TB_TRY(set_smem(gemv_gateup_kernel<2>, smem)); return launch(gemv_gateup_kernel<2>, grid, smem, st, pdl, a);
    case 4: TB_TRY(set_smem(gemv_gateup_kernel<4>, smem)); return launch(gemv_gateup_kernel<4>, grid, smem, st, pdl, a);
    default: TB_TRY(set_smem(gemv_gateup_kernel<8>, smem)); return launch(gemv_gateup_kernel<8>, grid, smem, st, pdl, a);
  }
}

tb_status_t gemv_lmhead(const LmHeadArgs& a, cudaStream_t st, bool pdl) {
  TB_REQUIRE(a.M >= 1 && a.M <= 8 && a.d % 4 == 0);
  const int MT = mt_for(a.M);
  const size_t smem = (size_t)MT * a.d * sizeof(float) + 8 * kGemvWarps * sizeof(float);
  const GemvPlan grid = gemv_grid((a.V + 1) / 2, smem);
  switch (MT) {
    case 1: TB_TRY(set_smem(gemv_lmhead_kernel<1>, smem)); return launch(gemv_lmhead_kernel<1>, grid, smem, st, pdl, a);
    case 2: TB_TRY(set_smem(gemv_lmhead_kernel<2>, smem)); return launch(gemv_lmhead_kernel<2>, grid, smem, st, pdl, a);
    case 4: TB_TRY(set_smem(gemv_lmhead_kernel<4>, smem)); return launch(gemv_lmhead_kernel<4>, grid, smem, st, pdl, a);
    default: TB_TRY(set_smem(gemv_lmhead_kernel<8>, smem)); return launch(gemv_lmhead_kernel<8>, grid, smem, st, pdl, a);
  }
}

}  // namespace tb
