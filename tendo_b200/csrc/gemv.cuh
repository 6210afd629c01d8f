// gemv.cuh — the fused-dequant int8 GEMV used for decode (M <= 32).
//
// y[m, n] = scale[n] * sum_k x[m, k] * q[n, k]   (per-channel int8 weights)
//
// Layout and schedule (HBM-bound: each weight byte is read once per call):
//  - a CTA of kThreads threads stages x (MT rows) in shared memory, in a
//    permuted order: float4 j of 16-element chunk c lives at index
//    j * (K / 16) + c, so lanes reading consecutive chunks hit consecutive
//    float4s (no bank conflicts);
//  - each warp owns a group of ROWS weight rows at a time and streams them
//    with 16-byte ld.global.nc.L1::no_allocate loads, lane l taking chunks
//    l, l + 32, ... (a warp load covers 512 contiguous bytes of a row);
//  - int8 -> fp32 by byte permute + one FADD (exact), fp32 FMA against x;
//  - warp-shuffle reduction per (row, m); the per-channel scale is applied
//    once after the K sum (it factors out of the sum);
//  - persistent grid (a few CTAs per SM) striding over row groups.
// Variants differ only in how row groups map to weight rows (Plan) and what
// the epilogue writes; RMSNorm can be fused into the x staging.
#pragma once

#include "common.cuh"

namespace tb {

constexpr int kGemvThreads = 512;  // upper bound of the block size
constexpr int kGemvWarps = kGemvThreads / 32;

// Stage x rows into shared memory (permuted float4 layout).  With `norm`
// set, x is RMSNorm(x) * w first: sum of squares in fp32, rms =
// sqrt(ms + eps) correctly rounded (equal to the reference's float32(
// math.Sqrt(float64(.)))), x / rms * w with IEEE division.
template <int MT>
__device__ __forceinline__ void stage_x(float* xs, const float* __restrict__ x, int64_t ldx, int M, int K,
                                        const float* __restrict__ norm_w, float eps, float* red) {
  const int chunks = K >> 4;
  const int nv = K >> 2;  // float4 per row
  float inv[MT];
  if (norm_w != nullptr) {
    float ss[MT];
#pragma unroll
    for (int m = 0; m < MT; m++) ss[m] = 0.f;
    for (int v = threadIdx.x; v < nv; v += blockDim.x) {
#pragma unroll
      for (int m = 0; m < MT; m++) {
        if (m < M) {
          float4 t = *reinterpret_cast<const float4*>(x + m * ldx + 4 * v);
          ss[m] += t.x * t.x + t.y * t.y + t.z * t.z + t.w * t.w;
        }
      }
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
    for (int m = 0; m < MT; m++) {
      float s = warp_sum(ss[m]);
      if (lane == 0) red[m * kGemvWarps + warp] = s;
    }
    __syncthreads();
#pragma unroll
    for (int m = 0; m < MT; m++) {
      float s = 0.f;
      for (int w = 0; w < (int)(blockDim.x >> 5); w++) s += red[m * kGemvWarps + w];
      float ms = __fdiv_rn(s, (float)K);
      inv[m] = __fsqrt_rn(__fadd_rn(ms, eps));  // the rms itself; divided below
    }
  }
  for (int v = threadIdx.x; v < nv; v += blockDim.x) {
    const int c = v >> 2, j = v & 3;
#pragma unroll
    for (int m = 0; m < MT; m++) {
      float4 t = make_float4(0.f, 0.f, 0.f, 0.f);
      if (m < M) {
        t = *reinterpret_cast<const float4*>(x + m * ldx + 4 * v);
        if (norm_w != nullptr) {
          float4 w = *reinterpret_cast<const float4*>(norm_w + 4 * v);
          t.x = __fmul_rn(__fdiv_rn(t.x, inv[m]), w.x);
          t.y = __fmul_rn(__fdiv_rn(t.y, inv[m]), w.y);
          t.z = __fmul_rn(__fdiv_rn(t.z, inv[m]), w.z);
          t.w = __fmul_rn(__fdiv_rn(t.w, inv[m]), w.w);
        }
      }
      reinterpret_cast<float4*>(xs)[(m * 4 + j) * chunks + c] = t;
    }
  }
  __syncthreads();
}

// Dot products of ROWS weight rows with MT staged x rows.  row_ptr[r] points
// at row r's first byte.  Each lane walks chunks lane, lane + 32, ...; every
// iteration issues U chunks of every row (U * ROWS 16-byte loads in flight
// per lane) before consuming them.
template <int MT, int ROWS, int U>
__device__ __forceinline__ void gemv_rows(float (&acc)[ROWS][MT], const int8_t* const (&row_ptr)[ROWS],
                                          const float* xs, int K) {
  const int lane = threadIdx.x & 31;
  const int chunks = K >> 4;
  const float4* xv = reinterpret_cast<const float4*>(xs);
#pragma unroll
  for (int r = 0; r < ROWS; r++)
#pragma unroll
    for (int m = 0; m < MT; m++) acc[r][m] = 0.f;

  for (int c0 = lane; c0 < chunks; c0 += 32 * U) {
    int4 w[U][ROWS];
#pragma unroll
    for (int u = 0; u < U; u++) {
      const int c = c0 + 32 * u;
#pragma unroll
      for (int r = 0; r < ROWS; r++) w[u][r] = c < chunks ? ld_stream_v4(row_ptr[r] + 16 * c) : make_int4(0, 0, 0, 0);
    }
#pragma unroll
    for (int u = 0; u < U; u++) {
      const int c = c0 + 32 * u;
      if (c >= chunks) break;
#pragma unroll
      for (int m = 0; m < MT; m++) {
        const float4 x0 = xv[(m * 4 + 0) * chunks + c];
        const float4 x1 = xv[(m * 4 + 1) * chunks + c];
        const float4 x2 = xv[(m * 4 + 2) * chunks + c];
        const float4 x3 = xv[(m * 4 + 3) * chunks + c];
#pragma unroll
        for (int r = 0; r < ROWS; r++) {
          float a, b, cf, d;
          float s = acc[r][m];
          i8x4_to_f32((uint32_t)w[u][r].x, a, b, cf, d);
          s = fmaf(x0.x, a, s); s = fmaf(x0.y, b, s); s = fmaf(x0.z, cf, s); s = fmaf(x0.w, d, s);
          i8x4_to_f32((uint32_t)w[u][r].y, a, b, cf, d);
          s = fmaf(x1.x, a, s); s = fmaf(x1.y, b, s); s = fmaf(x1.z, cf, s); s = fmaf(x1.w, d, s);
          i8x4_to_f32((uint32_t)w[u][r].z, a, b, cf, d);
          s = fmaf(x2.x, a, s); s = fmaf(x2.y, b, s); s = fmaf(x2.z, cf, s); s = fmaf(x2.w, d, s);
          i8x4_to_f32((uint32_t)w[u][r].w, a, b, cf, d);
          s = fmaf(x3.x, a, s); s = fmaf(x3.y, b, s); s = fmaf(x3.z, cf, s); s = fmaf(x3.w, d, s);
          acc[r][m] = s;
        }
      }
    }
  }
#pragma unroll
  for (int r = 0; r < ROWS; r++)
#pragma unroll
    for (int m = 0; m < MT; m++) acc[r][m] = warp_sum(acc[r][m]);
}

// Balanced persistent schedule: one CTA per SM, `tasks` spread over
// gridDim.x * warps warps in rounds, so every SM gets the same number of
// tasks to within one.
struct GemvPlan {
  unsigned grid;
  unsigned warps;
};

inline GemvPlan gemv_plan(int64_t tasks, int sms, int max_warps) {
  if (tasks < 1) tasks = 1;
  const int64_t grid = tasks < sms ? tasks : sms;
  const int64_t slots = grid * max_warps;
  const int64_t rounds = (tasks + slots - 1) / slots;
  int64_t warps = (tasks + grid * rounds - 1) / (grid * rounds);
  if (warps < 1) warps = 1;
  return GemvPlan{(unsigned)grid, (unsigned)warps};
}

// L2 prefetch of a row group (issued before waiting on the previous kernel:
// the weights do not depend on it).
template <int ROWS>
__device__ __forceinline__ void prefetch_rows(const int8_t* const (&row_ptr)[ROWS], int K) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int r = 0; r < ROWS; r++)
    for (int off = lane * 128; off < K; off += 32 * 128)
      asm volatile("prefetch.global.L2 [%0];" ::"l"(row_ptr[r] + off));
}

// Shared-memory bytes of the staged x.
inline size_t gemv_smem_bytes(int MT, int K) { return (size_t)MT * K * sizeof(float) + 64 * sizeof(float) * 8; }

}  // namespace tb
