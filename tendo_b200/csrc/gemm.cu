// gemm.cu — CUDA-core fp32 GEMM tiles: the quantized Linear for per-group
// scales and shapes the tcgen05 path (gemm_tc.cu) does not take, and the fp32
// lm_head of the multi-row paths.
//
// out[M, N] = x[M, K] @ W^T (+ resid) with W = q * scale dequantized to fp32
// while the tile is staged in shared memory (the same rounding as
// QuantizedTensor.Dequantize, nn/quantize.go:204-222), or W fp32 directly
// (the lm_head).  64 x 64 output tiles, K steps of 32, 4 x 4 outputs per
// thread; the fp32 NT product of aligned operands has its own 64 x 128 tiles.
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

// fp32 NT product for K % 32 == 0 and 16-byte aligned rows (the lm_head):
// 64 x 128 output tiles, 4 x 8 outputs per thread read from shared memory as
// one 16-byte row of x and two of W per k, tiles staged with 16-byte loads.
// Each output is one fmaf chain over k in ascending order, as in
// gemm_simt_kernel, so both give the same bits.
constexpr int FBM = 64, FBN = 128, FBK = 32;

__global__ void __launch_bounds__(kGemmThreads) gemm_f32_nt_kernel(float* out, const float* __restrict__ x,
                                                                   const float* __restrict__ w, int M, int N, int K) {
  __shared__ __align__(16) float Xs[FBK][FBM + 4];
  __shared__ __align__(16) float Ws[FBK][FBN + 4];
  const int m0 = blockIdx.y * FBM, n0 = blockIdx.x * FBN;
  const int t = threadIdx.x;
  const int tm = t / 16, tn = t % 16;  // rows 4 tm .. 4 tm + 3; columns 4 tn .. and 64 + 4 tn ..
  float acc[4][8];
#pragma unroll
  for (int i = 0; i < 4; i++)
#pragma unroll
    for (int j = 0; j < 8; j++) acc[i][j] = 0.f;
  for (int k0 = 0; k0 < K; k0 += FBK) {
#pragma unroll
    for (int i = 0; i < (FBM * FBK / 4) / kGemmThreads; i++) {
      const int idx = t + i * kGemmThreads;
      const int r = idx / (FBK / 4), c = (idx % (FBK / 4)) * 4;
      const int gm = m0 + r;
      const float4 v = gm < M ? *reinterpret_cast<const float4*>(x + (size_t)gm * K + k0 + c)
                              : make_float4(0.f, 0.f, 0.f, 0.f);
      Xs[c][r] = v.x;
      Xs[c + 1][r] = v.y;
      Xs[c + 2][r] = v.z;
      Xs[c + 3][r] = v.w;
    }
#pragma unroll
    for (int i = 0; i < (FBN * FBK / 4) / kGemmThreads; i++) {
      const int idx = t + i * kGemmThreads;
      const int r = idx / (FBK / 4), c = (idx % (FBK / 4)) * 4;
      const int gn = n0 + r;
      const float4 v = gn < N ? *reinterpret_cast<const float4*>(w + (size_t)gn * K + k0 + c)
                              : make_float4(0.f, 0.f, 0.f, 0.f);
      Ws[c][r] = v.x;
      Ws[c + 1][r] = v.y;
      Ws[c + 2][r] = v.z;
      Ws[c + 3][r] = v.w;
    }
    __syncthreads();
#pragma unroll 8
    for (int kk = 0; kk < FBK; kk++) {
      const float4 a = *reinterpret_cast<const float4*>(&Xs[kk][tm * 4]);
      const float4 b0 = *reinterpret_cast<const float4*>(&Ws[kk][tn * 4]);
      const float4 b1 = *reinterpret_cast<const float4*>(&Ws[kk][64 + tn * 4]);
      const float av[4] = {a.x, a.y, a.z, a.w};
      const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
      for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 8; j++) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const int gm = m0 + tm * 4 + i;
    if (gm >= M) continue;
#pragma unroll
    for (int j = 0; j < 8; j++) {
      const int gn = n0 + (j < 4 ? tn * 4 + j : 64 + tn * 4 + (j - 4));
      if (gn < N) out[(size_t)gm * N + gn] = acc[i][j];
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
  if (K % FBK == 0 && aligned(a, 16) && aligned(b, 16)) {
    dim3 grid((N + FBN - 1) / FBN, (M + FBM - 1) / FBM);
    gemm_f32_nt_kernel<<<grid, kGemmThreads, 0, st>>>(out, a, b, M, N, K);
    return check_launch("gemm_f32_nt_kernel");
  }
  dim3 grid((N + GBN - 1) / GBN, (M + GBM - 1) / GBM);
  gemm_simt_kernel<float><<<grid, kGemmThreads, 0, st>>>(out, a, b, nullptr, nullptr, M, N, K, K);
  return check_launch("gemm_simt_kernel<f32>");
}

}  // namespace tb
