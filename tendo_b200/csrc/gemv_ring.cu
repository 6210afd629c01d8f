// gemv_ring.cu — the decode-regime quantized Linear for 1 <= M <= 5 rows
// (nn.QuantizedLinear.Forward -> Backend.DequantizeMatmul,
// cuda/backend.go:676-721 over cuda/popcorn.go:1306-1315), as one weight
// stream through a shared-memory ring.
//
// out[m, n] = scale[n] * sum_k x[m, k] * q[n, k]  (+ resid[m, n])
//
// One CTA per SM: 8 consumer warps and one producer warp.  The CTA owns the
// 8-row weight tiles blockIdx.x, + gridDim.x, ...; each tile's rows move in
// chunks of Kc bytes (Kc divides K, at most 4096) through the ring's stages
// with cp.async.bulk (mbarrier completion, L2 evict-first), eight lanes of
// the producer issuing one row each.  The producer starts at launch, before
// the programmatic-launch wait — the weights never depend on the preceding
// kernel — so the stream is in flight while the consumers turn x into digit
// rows:
//   x[m] = s_m (d0 + d1 / 128 + d2 / 128^2),  s_m = max_k |x[m, k]| / 127,
// digit j of row m in digit row j M + m.  The integer tensor cores
// (mma.sync m16n8k32 s8) multiply the digit rows (A, rows 3M <= 15) by the
// raw weight bytes of a chunk (B, 8 weight rows), four independent
// accumulators per warp; a tile's exact s32 sums are gathered over the warps
// with shared-memory integer atomics (order-free), and a single epilogue after
// the last tile scales and writes.  Nothing outside the inputs and outputs is
// written: the call needs no workspace.
#include <mutex>

#include "common.cuh"
#include "kernels.h"
#include "tma_common.cuh"

namespace tb {
namespace {

constexpr int kRgWarps = 8;
constexpr int kRgConsumers = kRgWarps * 32;
constexpr int kRgThreads = kRgConsumers + 32;
constexpr int kRgMaxStages = 5;
constexpr int kRgMaxM = 5;
constexpr int kRgSmemMax = 227 * 1024;
constexpr int kRgXr = 4;  // float4 of each x row per thread kept in registers (K <= 4096 read once)

struct RingArgs {
  float* out;
  const float* x;
  const int8_t* q;
  const float* scale;
  const float* resid;
  int M, N, K, Kc, nch, RS, RSX, stages, tiles_cta;
  uint32_t dig_off, part_off, xs_off, ssc_off, red_off, bar_off;
  int* err;
};

struct RingLayout {
  uint32_t dig_off, part_off, xs_off, ssc_off, red_off, bar_off, total;
  int RS, RSX, stage_bytes;
  // stages as many as fit (at most kRgMaxStages); 0 when not even two do
  int stages;
  void init(int M, int K, int Kc, int tiles_cta) {
    RS = bank_stride(Kc);
    RSX = bank_stride(K);
    stage_bytes = 8 * RS;
    const size_t rest = (size_t)3 * M * RSX + 128 + (size_t)tiles_cta * 16 * 8 * 4 + 16 * 4 + (size_t)tiles_cta * 8 * 4 +
                        kRgWarps * kRgMaxM * 4 + (size_t)2 * kRgMaxStages * 8 + 64;
    stages = 0;
    for (int s = kRgMaxStages; s >= 2; s--)
      if ((size_t)s * stage_bytes + rest <= (size_t)kRgSmemMax) {
        stages = s;
        break;
      }
    dig_off = (uint32_t)(stages * stage_bytes);
    part_off = (uint32_t)((dig_off + (size_t)3 * M * RSX + 127) & ~(size_t)127);
    xs_off = part_off + (uint32_t)(tiles_cta * 16 * 8 * 4);
    ssc_off = xs_off + 16 * 4;
    red_off = ssc_off + (uint32_t)(tiles_cta * 8 * 4);
    bar_off = (red_off + kRgWarps * kRgMaxM * 4 + 15) & ~15u;
    total = bar_off + 2 * kRgMaxStages * 8;
  }
};

// Elements 4 v .. 4 v + 3 of row m as digits: u = x c (|u| <= 127) rounded to
// a multiple of 2^-14, U = round(u 2^14), split exactly into balanced digits
// U = d0 2^14 + d1 2^7 + d2, digit j of row m to digit row j M + m.
__device__ __forceinline__ void put_digits(int8_t* dig, int RSX, int M, int m, int v, float4 t, float c) {
  const float vals[4] = {t.x * c, t.y * c, t.z * c, t.w * c};
  int b0[4], b1[4], b2[4];
#pragma unroll
  for (int j = 0; j < 4; j++) {
    int U = __float2int_rn(vals[j] * 16384.0f);
    U = min(max(U, -127 * 16384), 127 * 16384);
    const int d0 = (U + 8192) >> 14;
    const int r = U - (d0 << 14);
    const int d1 = (r + 64) >> 7;
    b0[j] = d0;
    b1[j] = d1;
    b2[j] = r - (d1 << 7);
  }
  reinterpret_cast<uint32_t*>(dig + (size_t)m * RSX)[v] =
      __byte_perm(__byte_perm(b0[0], b0[1], 0x0040), __byte_perm(b0[2], b0[3], 0x0040), 0x5410);
  reinterpret_cast<uint32_t*>(dig + (size_t)(M + m) * RSX)[v] =
      __byte_perm(__byte_perm(b1[0], b1[1], 0x0040), __byte_perm(b1[2], b1[3], 0x0040), 0x5410);
  reinterpret_cast<uint32_t*>(dig + (size_t)(2 * M + m) * RSX)[v] =
      __byte_perm(__byte_perm(b2[0], b2[1], 0x0040), __byte_perm(b2[2], b2[3], 0x0040), 0x5410);
}

// MM: the rows the kernel's registers hold (M <= MM).
template <int MM>
__global__ void __launch_bounds__(kRgThreads, 1) gemv_ring_kernel(RingArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  unsigned char* stages = smem;
  int8_t* dig = reinterpret_cast<int8_t*>(smem + a.dig_off);
  int* part = reinterpret_cast<int*>(smem + a.part_off);  // [tiles_cta][16 digit rows][8 columns]
  float* xs = reinterpret_cast<float*>(smem + a.xs_off);  // [M] row scales
  float* ssc = reinterpret_cast<float*>(smem + a.ssc_off);  // [tiles_cta * 8] channel scales
  float* red = reinterpret_cast<float*>(smem + a.red_off);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + a.bar_off);
  uint64_t* empty = full + kRgMaxStages;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = a.stages, M = a.M, K = a.K, N = a.N, Kc = a.Kc, nch = a.nch;
  const int ntiles = (N + 7) / 8;
  const int my = ntiles > (int)blockIdx.x ? (ntiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x : 0;
  const int units = my * nch;
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; s++) {
      mbarrier_init(&full[s], 1);
      mbarrier_init(&empty[s], kRgConsumers);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  for (int i = threadIdx.x; i < my * 16 * 8; i += kRgThreads) part[i] = 0;
  __syncthreads();

  if (warp == kRgWarps) {
    // producer: lane 0 posts a chunk's bytes, lanes 0..7 copy one row each
    uint64_t policy;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
    for (int u = 0; u < units; u++) {
      const int st = u % S, use = u / S;
      if (use > 0) mbarrier_wait(&empty[st], (uint32_t)((use - 1) & 1), a.err);
      const int tile = (int)blockIdx.x + (u / nch) * (int)gridDim.x, ch = u - (u / nch) * nch;
      if (lane == 0) mbarrier_expect_tx(&full[st], (uint32_t)(8 * Kc));
      __syncwarp();
      if (lane < 8) {
        int row = tile * 8 + lane;
        if (row >= N) row = N - 1;  // a ragged last tile repeats the last row; its columns are not written
        bulk_copy_g2s_hint(stages + (size_t)st * (8 * a.RS) + (size_t)lane * a.RS,
                           a.q + (size_t)row * K + (size_t)ch * Kc, (uint32_t)Kc, &full[st], policy);
      }
    }
    pdl_launch_dependents();
    // every copy lands before the consumers release its stage, so the CTA
    // never exits with a copy in flight
    return;
  }
  // the channel scales of this CTA's tiles do not depend on the preceding
  // kernel: fetched before the programmatic-launch wait
  for (int i = threadIdx.x; i < my * 8; i += kRgConsumers) {
    int row = ((int)blockIdx.x + (i >> 3) * (int)gridDim.x) * 8 + (i & 7);
    if (row >= N) row = N - 1;
    ssc[i] = __ldg(a.scale + row);
  }
  pdl_wait();
  pdl_launch_dependents();

  // ---- digit rows of x: the first kRgXr float4 of each row per thread stay
  // in registers between the row maxima and the digits (the rest is re-read)
  const int nv = K >> 2;
  float4 xr[MM][kRgXr];
  float mx[MM];
#pragma unroll
  for (int m = 0; m < MM; m++) {
    mx[m] = 0.f;
#pragma unroll
    for (int i = 0; i < kRgXr; i++) {
      const int v = threadIdx.x + i * kRgConsumers;
      xr[m][i] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (m < M && v < nv) xr[m][i] = __ldg(reinterpret_cast<const float4*>(a.x + (size_t)m * K) + v);
    }
  }
#pragma unroll
  for (int m = 0; m < MM; m++) {
#pragma unroll
    for (int i = 0; i < kRgXr; i++) {
      const float4 t = xr[m][i];
      mx[m] = fmaxf(mx[m], fmaxf(fmaxf(fabsf(t.x), fabsf(t.y)), fmaxf(fabsf(t.z), fabsf(t.w))));
    }
  }
  for (int v = threadIdx.x + kRgXr * kRgConsumers; v < nv; v += kRgConsumers) {
#pragma unroll
    for (int m = 0; m < MM; m++) {
      if (m < M) {
        const float4 t = __ldg(reinterpret_cast<const float4*>(a.x + (size_t)m * K) + v);
        mx[m] = fmaxf(mx[m], fmaxf(fmaxf(fabsf(t.x), fabsf(t.y)), fmaxf(fabsf(t.z), fabsf(t.w))));
      }
    }
  }
#pragma unroll
  for (int m = 0; m < MM; m++) {
    const float w = warp_max(mx[m]);
    if (lane == 0) red[warp * kRgMaxM + m] = w;
  }
  named_sync(kRgConsumers);
  float c[MM];
#pragma unroll
  for (int m = 0; m < MM; m++) {
    float am = 0.f;
    for (int w = 0; w < kRgWarps; w++) am = fmaxf(am, red[w * kRgMaxM + m]);
    const float sc = (am > 0.f && isfinite(am)) ? am / 127.0f : 1.0f;
    c[m] = 1.0f / sc;
    if (threadIdx.x == 0 && m < M) xs[m] = sc;
  }
  // u = x / s (|u| <= 127) rounded to a multiple of 2^-14, U = round(u 2^14),
  // split exactly into balanced digits U = d0 2^14 + d1 2^7 + d2
#pragma unroll
  for (int i = 0; i < kRgXr; i++) {
    const int v = threadIdx.x + i * kRgConsumers;
    if (v < nv) {
#pragma unroll
      for (int m = 0; m < MM; m++)
        if (m < M) put_digits(dig, a.RSX, M, m, v, xr[m][i], c[m]);
    }
  }
  for (int v = threadIdx.x + kRgXr * kRgConsumers; v < nv; v += kRgConsumers) {
#pragma unroll
    for (int m = 0; m < MM; m++)
      if (m < M) put_digits(dig, a.RSX, M, m, v, __ldg(reinterpret_cast<const float4*>(a.x + (size_t)m * K) + v), c[m]);
  }
  named_sync(kRgConsumers);

  // ---- the CTA's tiles through the ring ----
  const int g = lane >> 2, t = lane & 3, R = 3 * M;
  const bool has0 = g < R, has1 = g + 8 < R;
  const int RS = a.RS, kbc = Kc / 64;
  const int8_t* xr0 = dig + (size_t)(has0 ? g : 0) * a.RSX + 16 * t;
  const int8_t* xr1 = dig + (size_t)(has1 ? g + 8 : 0) * a.RSX + 16 * t;
  const uint4 z4 = make_uint4(0u, 0u, 0u, 0u);
  int u = 0;
  for (int it = 0; it < my; it++) {
    // four independent accumulators (integer sums: the split is exact)
    int d0[4] = {0, 0, 0, 0}, d1[4] = {0, 0, 0, 0}, d2[4] = {0, 0, 0, 0}, d3[4] = {0, 0, 0, 0};
    for (int ch = 0; ch < nch; ch++, u++) {
      const int st = u % S, use = u / S;
      mbarrier_wait(&full[st], (uint32_t)(use & 1), a.err);
      const unsigned char* sp = stages + (size_t)st * (8 * RS) + (size_t)g * RS + 16 * t;
      const int8_t* x0 = xr0 + ch * Kc;
      const int8_t* x1 = xr1 + ch * Kc;
      int kb = warp;
      for (; kb + kRgWarps < kbc; kb += 2 * kRgWarps) {
        const uint4 wa = *reinterpret_cast<const uint4*>(sp + kb * 64);
        const uint4 wb = *reinterpret_cast<const uint4*>(sp + (kb + kRgWarps) * 64);
        const uint4 xa0 = has0 ? *reinterpret_cast<const uint4*>(x0 + kb * 64) : z4;
        const uint4 xa1 = has1 ? *reinterpret_cast<const uint4*>(x1 + kb * 64) : z4;
        const uint4 xb0 = has0 ? *reinterpret_cast<const uint4*>(x0 + (kb + kRgWarps) * 64) : z4;
        const uint4 xb1 = has1 ? *reinterpret_cast<const uint4*>(x1 + (kb + kRgWarps) * 64) : z4;
        mma_s8_16832(d0, xa0.x, xa1.x, xa0.y, xa1.y, wa.x, wa.y);
        mma_s8_16832(d1, xa0.z, xa1.z, xa0.w, xa1.w, wa.z, wa.w);
        mma_s8_16832(d2, xb0.x, xb1.x, xb0.y, xb1.y, wb.x, wb.y);
        mma_s8_16832(d3, xb0.z, xb1.z, xb0.w, xb1.w, wb.z, wb.w);
      }
      if (kb < kbc) {
        const uint4 wa = *reinterpret_cast<const uint4*>(sp + kb * 64);
        const uint4 xa0 = has0 ? *reinterpret_cast<const uint4*>(x0 + kb * 64) : z4;
        const uint4 xa1 = has1 ? *reinterpret_cast<const uint4*>(x1 + kb * 64) : z4;
        mma_s8_16832(d0, xa0.x, xa1.x, xa0.y, xa1.y, wa.x, wa.y);
        mma_s8_16832(d1, xa0.z, xa1.z, xa0.w, xa1.w, wa.z, wa.w);
      }
      mbarrier_arrive(&empty[st]);
    }
    // D rows g (and g + 8) are digit rows, columns 2t, 2t + 1 the tile's rows
    int* p = part + it * 128;
    if (has0) {
      atomicAdd(&p[g * 8 + 2 * t], d0[0] + d1[0] + d2[0] + d3[0]);
      atomicAdd(&p[g * 8 + 2 * t + 1], d0[1] + d1[1] + d2[1] + d3[1]);
    }
    if (has1) {
      atomicAdd(&p[(g + 8) * 8 + 2 * t], d0[2] + d1[2] + d2[2] + d3[2]);
      atomicAdd(&p[(g + 8) * 8 + 2 * t + 1], d0[3] + d1[3] + d2[3] + d3[3]);
    }
  }
  named_sync(kRgConsumers);

  // ---- epilogue: y = s_m (S0 + S1 / 128 + S2 / 128^2), out = y scale[n] (+ resid) ----
  for (int i = threadIdx.x; i < my * M * 8; i += kRgConsumers) {
    const int it = i / (M * 8), r = i - it * M * 8, m = r >> 3, n = r & 7;
    const int row = ((int)blockIdx.x + it * (int)gridDim.x) * 8 + n;
    if (row >= N) continue;
    const int* p = part + it * 128;
    const int s0 = p[m * 8 + n], s1 = p[(M + m) * 8 + n], s2 = p[(2 * M + m) * 8 + n];
    const float y = xs[m] * ((float)s0 + (float)s1 * (1.0f / 128.0f) + (float)s2 * (1.0f / 16384.0f));
    float v = y * ssc[it * 8 + n];
    if (a.resid) v += a.resid[(size_t)m * N + row];
    a.out[(size_t)m * N + row] = v;
  }
}

int ring_tiles_cta(int64_t N) {
  const int64_t tiles = (N + 7) / 8;
  const int64_t grid = sm_count();
  return (int)((tiles + grid - 1) / grid);
}

bool ring_layout(RingLayout& Ly, int64_t M, int64_t N, int64_t K) {
  Ly.init((int)M, (int)K, chunk_bytes((int)K), ring_tiles_cta(N));
  return Ly.stages >= 3;  // shallower rings cannot cover the latency: the tcgen05 GEMV takes those
}

}  // namespace

bool gemv_ring_ok(const float* x, const int8_t* q, int64_t M, int64_t N, int64_t K) {
  if (M < 1 || M > kRgMaxM || N < 1 || K < 64 || K % 64 != 0) return false;
  if (N > (1 << 24) || K > (1 << 20)) return false;
  if (!aligned(x, 16) || !aligned(q, 16)) return false;
  RingLayout Ly;
  return ring_layout(Ly, M, N, K);
}

tb_status_t gemv_ring(float* out, const float* x, const int8_t* q, const float* scale, const float* resid, int M,
                      int N, int K, cudaStream_t st) {
  if (!gemv_ring_ok(x, q, M, N, K)) return TB_ERROR_NOT_SUPPORTED;
  static std::once_flag once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(once, [] {
    attr_err = cudaFuncSetAttribute(gemv_ring_kernel<kRgMaxM>, cudaFuncAttributeMaxDynamicSharedMemorySize, kRgSmemMax);
  });
  if (attr_err != cudaSuccess) return cuda_fail(attr_err, "cudaFuncSetAttribute(gemv_ring_kernel)");
  RingLayout Ly;
  ring_layout(Ly, M, N, K);
  RingArgs a{};
  a.out = out;
  a.x = x;
  a.q = q;
  a.scale = scale;
  a.resid = resid;
  a.M = M;
  a.N = N;
  a.K = K;
  a.Kc = chunk_bytes(K);
  a.nch = K / a.Kc;
  a.tiles_cta = ring_tiles_cta(N);
  a.RS = Ly.RS;
  a.RSX = Ly.RSX;
  a.stages = Ly.stages;
  a.dig_off = Ly.dig_off;
  a.part_off = Ly.part_off;
  a.xs_off = Ly.xs_off;
  a.ssc_off = Ly.ssc_off;
  a.red_off = Ly.red_off;
  a.bar_off = Ly.bar_off;
  a.err = wait_timeout_word();
  const int64_t tiles = ((int64_t)N + 7) / 8;
  int64_t grid = sm_count();
  if (grid > tiles) grid = tiles;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(kRgThreads);
  cfg.dynamicSmemBytes = Ly.total;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, gemv_ring_kernel<kRgMaxM>, a);
  if (e != cudaSuccess) return cuda_fail(e, "cudaLaunchKernelEx(gemv_ring_kernel)");
  return TB_SUCCESS;
}

}  // namespace tb
