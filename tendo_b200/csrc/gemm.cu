// gemm.cu — CUDA-core fp32 GEMM tiles: the quantized Linear for per-group
// scales and shapes the tcgen05 path (gemm_tc.cu) does not take, and the fp32
// lm_head of the multi-row paths.
//
// out[M, N] = x[M, K] @ W^T (+ resid) with W = q * scale dequantized to fp32
// while the tile is staged in shared memory (the same rounding as
// QuantizedTensor.Dequantize, nn/quantize.go:204-222), or W fp32 directly
// (the lm_head).  64 x 64 output tiles, K steps of 32, 4 x 4 outputs per
// thread.
#include "common.cuh"
#include "kernels.h"

namespace tb {
namespace {

constexpr int GBM = 64, GBN = 64, GBK = 32, kGemmThreads = 256;

template <typename WT>
__device__ __forceinline__ float load_w(const WT* w, const float* scale, int64_t n, int64_t k, int64_t K, int64_t g) {
  if constexpr (sizeof(WT) == 1) {
    return __fmul_rn((float)w[n * K + k], scale[n * (K / g) + k / g]);
  } else {
    return w[n * K + k];
  }
}

template <typename WT>
__global__ void __launch_bounds__(kGemmThreads) gemm_simt_kernel(float* out, const float* __restrict__ x,
                                                                 const WT* __restrict__ w,
                                                                 const float* __restrict__ scale, const float* resid,
                                                                 int M, int N, int K, int g) {
  __shared__ float Xs[GBK][GBM + 4];
  __shared__ float Ws[GBK][GBN + 4];
  const int m0 = blockIdx.y * GBM, n0 = blockIdx.x * GBN;
  const int t = threadIdx.x;
  const int tm = t / 16, tn = t % 16;  // 16 x 16 threads, 4 x 4 outputs each
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; i++)
#pragma unroll
    for (int j = 0; j < 4; j++) acc[i][j] = 0.f;
  for (int k0 = 0; k0 < K; k0 += GBK) {
    // stage: 64 rows x 32 k of x and of W (8 elements per thread each)
#pragma unroll
    for (int i = 0; i < (GBM * GBK) / kGemmThreads; i++) {
      const int idx = t + i * kGemmThreads;
      const int r = idx / GBK, c = idx % GBK;
      const int gm = m0 + r, gk = k0 + c;
      Xs[c][r] = (gm < M && gk < K) ? x[(size_t)gm * K + gk] : 0.f;
      const int gn = n0 + r;
      Ws[c][r] = (gn < N && gk < K) ? load_w<WT>(w, scale, gn, gk, K, g) : 0.f;
    }
    __syncthreads();
#pragma unroll 8
    for (int kk = 0; kk < GBK; kk++) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; i++) a[i] = Xs[kk][tm * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; j++) b[j] = Ws[kk][tn + 16 * j];
#pragma unroll
      for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const int gm = m0 + tm * 4 + i;
    if (gm >= M) continue;
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const int gn = n0 + tn + 16 * j;
      if (gn >= N) continue;
      float v = acc[i][j];
      if (resid) v += resid[(size_t)gm * N + gn];
      out[(size_t)gm * N + gn] = v;
    }
  }
}

}  // namespace

tb_status_t gemm_simt_i8(float* out, const float* x, const int8_t* q, const float* scale, const float* resid,
                         int M, int N, int K, int group, cudaStream_t st) {
  const int g = group > 0 ? group : K;
  dim3 grid((N + GBN - 1) / GBN, (M + GBM - 1) / GBM);
  gemm_simt_kernel<int8_t><<<grid, kGemmThreads, 0, st>>>(out, x, q, scale, resid, M, N, K, g);
  return check_launch("gemm_simt_kernel<i8>");
}

tb_status_t gemm_f32_nt(float* out, const float* a, const float* b, int M, int N, int K, cudaStream_t st) {
  dim3 grid((N + GBN - 1) / GBN, (M + GBM - 1) / GBM);
  gemm_simt_kernel<float><<<grid, kGemmThreads, 0, st>>>(out, a, b, nullptr, nullptr, M, N, K, K);
  return check_launch("gemm_simt_kernel<f32>");
}

}  // namespace tb
