// gemm_tc.cu — the prefill-regime quantized Linear (M > 32) on the
// 5th-generation tensor cores.
//
// out[M, N] = x[M, K] @ (q * scale)^T (+ resid), q int8 [N, K] as stored.
//
// The fp32 activations are split per row into int8 digit planes:
//   x[m, k] / s_m = d0 + d1 / 128 (+ d2 / 128^2),   s_m = max_k |x[m, k]| / 127,
// (tc_digits_kernel; optionally of RMSNorm(x) * norm_w, so the norm costs no
// extra pass).  Every plane times the raw weight bytes is an exact s32 sum on
// tcgen05.mma kind::i8, so the only approximation is the digit truncation:
// below 2^-21 (three planes) or 2^-14 (two planes) of s_m per element.
//
// gemm_tc_kernel: one 128 x 128 output tile per CTA, 4 warps.
//   warp 0 lane 0: TMA producer — per 128-byte K block, the NP digit-plane
//     tiles and the weight tile (128 rows x 128 bytes each, 128-byte
//     swizzle) into a ring of shared-memory stages (mbarrier completion);
//   warp 1 lane 0: MMA issuer — per K block 4 x NP tcgen05.mma (M 128,
//     N 128, K 32), plane p accumulating in TMEM columns [128 p, 128 p + 128);
//     tcgen05.commit releases the stage when its MMAs are done;
//   all 4 warps: epilogue — each thread owns one output row (its TMEM lane),
//     reads the plane accumulators with tcgen05.ld and writes
//     s_m * scale[n] * (D0 + D1 / 128 + D2 / 128^2) (+ resid).
// Consecutive CTAs share a weight tile (blockIdx.x walks M first), so a
// weight tile streams from HBM once and the other M tiles read it from L2.
// Every wait is bounded (counted in the library's timeout word).
#include <cuda.h>  // CUtensorMap and the tensor-map encoder's types (resolved through the runtime)

#include <cooperative_groups.h>

#include <mutex>

#include "common.cuh"
#include "kernels.h"
#include "tc_common.cuh"
#include "tma_common.cuh"

namespace tb {
namespace {

namespace cg = cooperative_groups;

constexpr int kTcBM = 128, kTcBN = 128, kTcBK = 128;  // kTcBK in bytes = int8 elements
constexpr int kTcTile = kTcBM * kTcBK;                 // 16 KB: one operand tile
constexpr int kTcThreads = 128;
constexpr int kTcMaxK = 65536;  // |sum of K products| < 2^31 for every plane

template <int NP>
struct TcCfg {
  static constexpr int kStageBytes = (NP + 1) * kTcTile;
  static constexpr int kStages = NP == 3 ? 3 : 4;
  static constexpr int kTmemCols = NP == 3 ? 512 : 256;  // NP x 128 accumulator columns, power of two
  static constexpr size_t kSmem = (size_t)kStages * kStageBytes + 1024 + 256;
};

// ---------------------------------------------------------------------------
// digit planes
// ---------------------------------------------------------------------------
// One row per thread-block cluster of C CTAs (grid C x M); CTA r of the
// cluster holds K / (4 C) float4 of the row in registers (VPT per thread),
// the row's sum of squares and max |x| are combined over the cluster through
// distributed shared memory in rank order (the same bits in every CTA), and
// each CTA writes the digits of its own slice.
template <int NP, int VPT>
__global__ void __launch_bounds__(256) tc_digits_kernel(int8_t* __restrict__ dig, float* __restrict__ srow,
                                                        const float* __restrict__ x, int M, int K,
                                                        const float* __restrict__ norm_w, float eps) {
  __shared__ float red[2][8];
  __shared__ float part[2];
  cg::cluster_group cl = cg::this_cluster();
  const int C = (int)cl.num_blocks(), r = (int)cl.block_rank();
  pdl_launch_dependents();  // the GEMV that consumes the digits may start streaming weights
  pdl_wait();               // x may come from the preceding kernel
  const int m = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nvc = (K >> 2) / C, v0 = r * nvc;  // this CTA's float4 of the row
  const float4* xr = reinterpret_cast<const float4*>(x + (size_t)m * K) + v0;
  const float4* wr = norm_w ? reinterpret_cast<const float4*>(norm_w) + v0 : nullptr;
  float4 t[VPT];
  float ss = 0.f, mx = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; i++) {
    const int v = threadIdx.x + i * 256;
    t[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (v < nvc) {
      t[i] = xr[v];
      ss += t[i].x * t[i].x + t[i].y * t[i].y + t[i].z * t[i].z + t[i].w * t[i].w;
      const float4 w = wr ? wr[v] : make_float4(1.f, 1.f, 1.f, 1.f);
      mx = fmaxf(mx, fmaxf(fmaxf(fabsf(t[i].x * w.x), fabsf(t[i].y * w.y)),
                           fmaxf(fabsf(t[i].z * w.z), fabsf(t[i].w * w.w))));
    }
  }
  ss = warp_sum(ss);
  mx = warp_max(mx);
  if (lane == 0) {
    red[0][warp] = ss;
    red[1][warp] = mx;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float s0 = 0.f, a0 = 0.f;
#pragma unroll
    for (int w = 0; w < 8; w++) {
      s0 += red[0][w];
      a0 = fmaxf(a0, red[1][w]);
    }
    part[0] = s0;
    part[1] = a0;
  }
  cl.sync();
  float tot = 0.f, a = 0.f;
  for (int q = 0; q < C; q++) {
    const float* pq = cl.map_shared_rank(part, q);
    tot += pq[0];
    a = fmaxf(a, pq[1]);
  }
  cl.sync();  // no CTA leaves while another still reads its partial sums
  // RMSNorm as cpu/backend.go:606-652: rms = sqrt(sumSq / d + eps), out = (x / rms) * w
  const float rms = norm_w ? __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)K), eps)) : 1.0f;
  if (norm_w) a = a / rms * 1.0001f;  // covers the rounding of (x / rms) * w against (x * w) / rms
  const float sc = (a > 0.f && isfinite(a)) ? a / 127.0f : 1.0f;
  const float inv = 1.0f / sc;
  if (threadIdx.x == 0 && r == 0) srow[m] = sc;
  uint32_t* d0 = reinterpret_cast<uint32_t*>(dig + (size_t)m * K) + v0;
  const size_t plane = (size_t)M * K / 4;  // uint32 per plane
#pragma unroll
  for (int i = 0; i < VPT; i++) {
    const int v = threadIdx.x + i * 256;
    if (v >= nvc) continue;
    float4 u4 = t[i];
    if (norm_w) {
      const float4 w = wr[v];
      u4.x = __fmul_rn(__fdiv_rn(u4.x, rms), w.x);
      u4.y = __fmul_rn(__fdiv_rn(u4.y, rms), w.y);
      u4.z = __fmul_rn(__fdiv_rn(u4.z, rms), w.z);
      u4.w = __fmul_rn(__fdiv_rn(u4.w, rms), w.w);
    }
    const float vals[4] = {u4.x, u4.y, u4.z, u4.w};
    uint32_t p[3] = {0u, 0u, 0u};
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const float u = fminf(fmaxf(vals[j] * inv, -127.0f), 127.0f);
      const float e0 = rintf(u);
      const float r1 = (u - e0) * 128.0f;
      const float e1 = rintf(r1);
      const float e2 = rintf((r1 - e1) * 128.0f);
      p[0] |= ((uint32_t)__float2int_rn(e0) & 0xffu) << (8 * j);
      p[1] |= ((uint32_t)__float2int_rn(e1) & 0xffu) << (8 * j);
      p[2] |= ((uint32_t)__float2int_rn(e2) & 0xffu) << (8 * j);
    }
#pragma unroll
    for (int q = 0; q < NP; q++) d0[q * plane + v] = p[q];
  }
}

template <int NP>
__global__ void __launch_bounds__(kTcThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   float* out, const float* __restrict__ srow, const float* __restrict__ scale,
                   const float* resid, int M, int N, int K, int vec_ok, int* err) {
  using C = TcCfg<NP>;
  extern __shared__ unsigned char smem_raw[];
  // 1024-byte alignment of the swizzled tiles (in the shared address space)
  unsigned char* smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)C::kStages * C::kStageBytes);
  uint64_t* empty = full + C::kStages;
  uint64_t* done = empty + C::kStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.x * kTcBM, n0 = blockIdx.y * kTcBN;
  const int nk = (K + kTcBK - 1) / kTcBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; s++) {
      mbarrier_init(&full[s], 1);
      mbarrier_init(&empty[s], 1);
    }
    mbarrier_init(done, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmA)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmB)) : "memory");
  }
  if (warp == 0) tmem_alloc(tmem_slot, C::kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0 && lane == 0) {
    // producer
    for (int kb = 0; kb < nk; kb++) {
      const int s = kb % C::kStages, use = kb / C::kStages;
      if (use > 0) mbarrier_wait(&empty[s], (uint32_t)((use - 1) & 1), err);
      unsigned char* st = smem + (size_t)s * C::kStageBytes;
      mbarrier_expect_tx(&full[s], (uint32_t)C::kStageBytes);
#pragma unroll
      for (int p = 0; p < NP; p++) tma_load_3d(st + p * kTcTile, &tmA, kb * kTcBK, m0, p, &full[s]);
      tma_load_2d(st + NP * kTcTile, &tmB, kb * kTcBK, n0, &full[s]);
    }
  } else if (warp == 1 && lane == 0) {
    // MMA issuer
    for (int kb = 0; kb < nk; kb++) {
      const int s = kb % C::kStages, use = kb / C::kStages;
      mbarrier_wait(&full[s], (uint32_t)(use & 1), err);
      tc_fence_after();
      const uint32_t a0 = smem_addr(smem + (size_t)s * C::kStageBytes);
      const uint32_t b0 = a0 + NP * kTcTile;
#pragma unroll
      for (int kk = 0; kk < kTcBK / 32; kk++) {
#pragma unroll
        for (int p = 0; p < NP; p++)
          tc_mma_i8(tmem + p * kTcBN, sw128_desc(a0 + p * kTcTile + kk * 32), sw128_desc(b0 + kk * 32),
                    idesc_i8(kTcBM, kTcBN), (kb | kk) != 0);
      }
      tc_commit(&empty[s]);  // the stage is free once these MMAs have read it
    }
    tc_commit(done);
  }
  __syncwarp();

  // epilogue: thread = output row m0 + 32 warp + lane = TMEM lane 32 warp + lane
  mbarrier_wait(done, 0u, err);
  __syncwarp();  // tcgen05.ld is warp-collective
  tc_fence_after();
  const int row = m0 + warp * 32 + lane;
  const bool live = row < M;
  const float sr = live ? srow[row] : 0.f;
  const uint32_t lane_base = tmem + ((uint32_t)(warp * 32) << 16);
  for (int c = 0; c < kTcBN; c += 32) {
    uint32_t acc[NP][32];
#pragma unroll
    for (int p = 0; p < NP; p++) tmem_ld32(lane_base + p * kTcBN + c, acc[p]);
    tmem_wait_ld();
#pragma unroll
    for (int p = 0; p < NP; p++) pin32(acc[p]);
    if (!live) continue;
    float* orow = out + (size_t)row * N;
    const float* rrow = resid ? resid + (size_t)row * N : nullptr;
#pragma unroll
    for (int j = 0; j < 32; j += 4) {
      const int n = n0 + c + j;
      float y[4];
#pragma unroll
      for (int e = 0; e < 4; e++) {
        float t = (float)(int)acc[0][j + e] + (float)(int)acc[1][j + e] * (1.0f / 128.0f);
        if (NP == 3) t += (float)(int)acc[NP - 1][j + e] * (1.0f / 16384.0f);
        y[e] = t;
      }
      if (vec_ok && n + 3 < N) {
        const float4 sc = *reinterpret_cast<const float4*>(scale + n);
        float4 o = make_float4(sr * sc.x * y[0], sr * sc.y * y[1], sr * sc.z * y[2], sr * sc.w * y[3]);
        if (rrow) {
          const float4 r = *reinterpret_cast<const float4*>(rrow + n);
          o.x += r.x;
          o.y += r.y;
          o.z += r.z;
          o.w += r.w;
        }
        *reinterpret_cast<float4*>(orow + n) = o;
      } else {
#pragma unroll
        for (int e = 0; e < 4; e++) {
          if (n + e < N) {
            float o = sr * scale[n + e] * y[e];
            if (rrow) o += rrow[n + e];
            orow[n + e] = o;
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, C::kTmemCols);
}

// ---------------------------------------------------------------------------
// per-group scales [N, K / group] (group a multiple of 128): the same digit
// planes and MMAs on a 128 x 64 tile, with an accumulator hand-off per group.
//   warp 0 lane 0: TMA producer (NP digit tiles + a 64-row weight tile per
//     128-byte K block);
//   warp 1 lane 0: MMA issuer — a group's NP plane accumulators (NP x 64
//     columns) go to one of two TMEM buffers, committed to the epilogue at
//     the group's last K block;
//   warps 2..5: epilogue — thread = output row (its TMEM lane); per group,
//     y = D0 + D1 / 128 (+ D2 / 128^2) per column, times scale[n, group]
//     (staged in shared memory for the tile's 64 rows), added into 64 fp32
//     registers; out = s_m * sum (+ resid) at the end.
// ---------------------------------------------------------------------------
constexpr int kGgBN = 64;                          // weight rows per tile (MMA N)
constexpr int kGgWTile = kGgBN * kTcBK;            // 8 KB
constexpr int kGgStages = 3;
constexpr int kGgThreads = 192;
constexpr int kGgMaxScales = 8192;                 // 64 rows x up to 128 groups
template <int NP>
struct GgCfg {
  static constexpr int kStageBytes = NP * kTcTile + kGgWTile;
  static constexpr size_t kSmem = (size_t)kGgStages * kStageBytes + 1024 + 256 + kGgMaxScales * 4;
};

template <int NP>
__global__ void __launch_bounds__(kGgThreads, 1)
    gemm_tc_grp_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                       float* out, const float* __restrict__ srow, const float* __restrict__ scale,
                       const float* resid, int M, int N, int K, int gs, int ng, int vec_ok, int* err) {
  using C = GgCfg<NP>;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)kGgStages * C::kStageBytes);
  uint64_t* empty = full + kGgStages;
  uint64_t* tfull = empty + kGgStages;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  float* sc_s = reinterpret_cast<float*>(smem + (size_t)kGgStages * C::kStageBytes + 256);  // [64][ng]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.x * kTcBM, n0 = blockIdx.y * kGgBN;
  const int nk = K / kTcBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kGgStages; s++) {
      mbarrier_init(&full[s], 1);
      mbarrier_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; b++) {
      mbarrier_init(&tfull[b], 1);
      mbarrier_init(&tempty[b], 4);  // one arrival per epilogue warp
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmA)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmB)) : "memory");
  }
  if (warp == 0) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      for (int kb = 0; kb < nk; kb++) {
        const int s = kb % kGgStages, use = kb / kGgStages;
        if (use > 0) mbarrier_wait(&empty[s], (uint32_t)((use - 1) & 1), err);
        unsigned char* st = smem + (size_t)s * C::kStageBytes;
        mbarrier_expect_tx(&full[s], (uint32_t)C::kStageBytes);
#pragma unroll
        for (int p = 0; p < NP; p++) tma_load_3d(st + p * kTcTile, &tmA, kb * kTcBK, m0, p, &full[s]);
        tma_load_2d(st + NP * kTcTile, &tmB, kb * kTcBK, n0, &full[s]);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = idesc_i8(kTcBM, kGgBN);
      int h = 0;
      uint32_t d = tmem;
      for (int kb = 0; kb < nk; kb++) {
        const int s = kb % kGgStages, use = kb / kGgStages;
        const bool first = kb % gs == 0;
        if (first) {
          const int buf = h & 1;
          if (h >= 2) mbarrier_wait(&tempty[buf], (uint32_t)(((h - 2) >> 1) & 1), err);
          d = tmem + (uint32_t)(buf * 256);
        }
        mbarrier_wait(&full[s], (uint32_t)(use & 1), err);
        tc_fence_after();
        const uint32_t a0 = smem_addr(smem + (size_t)s * C::kStageBytes);
        const uint32_t b0 = a0 + NP * kTcTile;
#pragma unroll
        for (int kk = 0; kk < kTcBK / 32; kk++) {
#pragma unroll
          for (int p = 0; p < NP; p++)
            tc_mma_i8(d + p * kGgBN, sw128_desc(a0 + p * kTcTile + kk * 32), sw128_desc(b0 + kk * 32), idesc,
                      !(first && kk == 0));
        }
        tc_commit(&empty[s]);
        if ((kb + 1) % gs == 0) {
          tc_commit(&tfull[h & 1]);
          h++;
        }
      }
    }
  } else {
    const int q = warp & 3;
    const int et = threadIdx.x - 64;  // 0..127
    // the tile's scales, [64 rows][ng groups]
    for (int i = et; i < kGgBN * ng; i += 128) {
      const int j = i / ng, n = n0 + j;
      sc_s[i] = n < N ? __ldg(scale + (size_t)n * ng + (i - j * ng)) : 0.f;
    }
    asm volatile("bar.sync 1, 128;" ::: "memory");
    float acc[kGgBN];
#pragma unroll
    for (int j = 0; j < kGgBN; j++) acc[j] = 0.f;
    const uint32_t lane_base = tmem + ((uint32_t)(q * 32) << 16);
    for (int g = 0; g < ng; g++) {
      const int buf = g & 1;
      mbarrier_wait(&tfull[buf], (uint32_t)((g >> 1) & 1), err);
      __syncwarp();
      tc_fence_after();
#pragma unroll
      for (int c = 0; c < kGgBN; c += 32) {
        uint32_t v[NP][32];
#pragma unroll
        for (int p = 0; p < NP; p++) tmem_ld32(lane_base + (uint32_t)(buf * 256 + p * kGgBN + c), v[p]);
        tmem_wait_ld();
#pragma unroll
        for (int p = 0; p < NP; p++) pin32(v[p]);
#pragma unroll
        for (int e = 0; e < 32; e++) {
          float y = (float)(int)v[0][e] + (float)(int)v[1][e] * (1.0f / 128.0f);
          if (NP == 3) y += (float)(int)v[NP - 1][e] * (1.0f / 16384.0f);
          acc[c + e] = __fmaf_rn(y, sc_s[(c + e) * ng + g], acc[c + e]);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbarrier_arrive(&tempty[buf]);
    }
    const int row = m0 + q * 32 + lane;
    if (row < M) {
      const float sr = srow[row];
      float* orow = out + (size_t)row * N;
      const float* rrow = resid ? resid + (size_t)row * N : nullptr;
#pragma unroll
      for (int j = 0; j < kGgBN; j += 4) {
        const int n = n0 + j;
        if (vec_ok && n + 3 < N) {
          float4 o = make_float4(sr * acc[j], sr * acc[j + 1], sr * acc[j + 2], sr * acc[j + 3]);
          if (rrow) {
            const float4 r = *reinterpret_cast<const float4*>(rrow + n);
            o.x += r.x;
            o.y += r.y;
            o.z += r.z;
            o.w += r.w;
          }
          *reinterpret_cast<float4*>(orow + n) = o;
        } else {
#pragma unroll
          for (int e = 0; e < 4; e++)
            if (n + e < N) orow[n + e] = rrow ? sr * acc[j + e] + rrow[n + e] : sr * acc[j + e];
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 512);
}

template <int NP>
tb_status_t launch_tc(float* out, const int8_t* dig, const float* srow, const int8_t* q, const float* scale,
                      const float* resid, int M, int N, int K, cudaStream_t st) {
  using C = TcCfg<NP>;
  EncodeTiledFn enc = encode_tiled();
  if (!enc) return TB_ERROR_NOT_SUPPORTED;
  CUtensorMap ta, tbm;
  {
    const cuuint64_t dims[3] = {(cuuint64_t)K, (cuuint64_t)M, (cuuint64_t)NP};
    const cuuint64_t strides[2] = {(cuuint64_t)K, (cuuint64_t)M * (cuuint64_t)K};
    const cuuint32_t box[3] = {kTcBK, kTcBM, 1};
    const cuuint32_t es[3] = {1, 1, 1};
    const CUresult r = enc(&ta, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<int8_t*>(dig), dims, strides, box, es,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return TB_ERROR_NOT_SUPPORTED;
  }
  {
    const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)N};
    const cuuint64_t strides[1] = {(cuuint64_t)K};
    const cuuint32_t box[2] = {kTcBK, kTcBN};
    const cuuint32_t es[2] = {1, 1};
    const CUresult r = enc(&tbm, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<int8_t*>(q), dims, strides, box, es,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return TB_ERROR_NOT_SUPPORTED;
  }
  static std::once_flag once[2];
  static cudaError_t attr_err[2];
  std::call_once(once[NP - 2], [] {
    attr_err[NP - 2] =
        cudaFuncSetAttribute(gemm_tc_kernel<NP>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)C::kSmem);
  });
  if (attr_err[NP - 2] != cudaSuccess) return cuda_fail(attr_err[NP - 2], "cudaFuncSetAttribute(gemm_tc)");
  const int vec_ok = (N % 4 == 0) && ((uintptr_t)out % 16 == 0) && ((uintptr_t)scale % 16 == 0) &&
                     (!resid || (uintptr_t)resid % 16 == 0);
  int* err = wait_timeout_word();
  const dim3 grid((M + kTcBM - 1) / kTcBM, (N + kTcBN - 1) / kTcBN);
  gemm_tc_kernel<NP><<<grid, kTcThreads, C::kSmem, st>>>(ta, tbm, out, srow, scale, resid, M, N, K, vec_ok, err);
  return check_launch("gemm_tc_kernel");
}

template <int NP>
tb_status_t launch_tc_grp(float* out, const int8_t* dig, const float* srow, const int8_t* q, const float* scale,
                          const float* resid, int M, int N, int K, int group, cudaStream_t st) {
  using C = GgCfg<NP>;
  EncodeTiledFn enc = encode_tiled();
  if (!enc) return TB_ERROR_NOT_SUPPORTED;
  CUtensorMap ta, tbm;
  {
    const cuuint64_t dims[3] = {(cuuint64_t)K, (cuuint64_t)M, (cuuint64_t)NP};
    const cuuint64_t strides[2] = {(cuuint64_t)K, (cuuint64_t)M * (cuuint64_t)K};
    const cuuint32_t box[3] = {kTcBK, kTcBM, 1};
    const cuuint32_t es[3] = {1, 1, 1};
    if (enc(&ta, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<int8_t*>(dig), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return TB_ERROR_NOT_SUPPORTED;
  }
  {
    const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)N};
    const cuuint64_t strides[1] = {(cuuint64_t)K};
    const cuuint32_t box[2] = {kTcBK, kGgBN};
    const cuuint32_t es[2] = {1, 1};
    if (enc(&tbm, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<int8_t*>(q), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return TB_ERROR_NOT_SUPPORTED;
  }
  static std::once_flag once[2];
  static cudaError_t attr_err[2];
  std::call_once(once[NP - 2], [] {
    attr_err[NP - 2] =
        cudaFuncSetAttribute(gemm_tc_grp_kernel<NP>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)C::kSmem);
  });
  if (attr_err[NP - 2] != cudaSuccess) return cuda_fail(attr_err[NP - 2], "cudaFuncSetAttribute(gemm_tc_grp)");
  const int vec_ok = (N % 4 == 0) && ((uintptr_t)out % 16 == 0) && (!resid || (uintptr_t)resid % 16 == 0);
  const dim3 grid((M + kTcBM - 1) / kTcBM, (N + kGgBN - 1) / kGgBN);
  gemm_tc_grp_kernel<NP><<<grid, kGgThreads, C::kSmem, st>>>(ta, tbm, out, srow, scale, resid, M, N, K,
                                                             group / kTcBK, K / group, vec_ok, wait_timeout_word());
  return check_launch("gemm_tc_grp_kernel");
}

}  // namespace

size_t gemm_tc_workspace(int64_t M, int64_t K, int planes) {
  const size_t dig = ((size_t)planes * (size_t)M * (size_t)K + 255) & ~(size_t)255;
  return dig + (size_t)M * sizeof(float);
}

bool gemm_tc_ok(const void* q, int64_t M, int64_t N, int64_t K) {
  static const bool sm100 = device_is_sm100();
  return sm100 && M >= 1 && N >= 1 && K >= 16 && K % 16 == 0 && K <= kTcMaxK && M <= 0x7fffffff / 4 &&
         N <= 65535 * kTcBN && ((uintptr_t)q % 16 == 0) && encode_tiled() != nullptr;
}

tb_status_t gemm_tc_digits(int8_t* dig, float* srow, const float* x, int M, int K, int planes, const float* norm_w,
                           float eps, cudaStream_t st) {
  if (M <= 0) return TB_SUCCESS;
  if (K % 4 != 0 || (uintptr_t)x % 16 != 0 || (norm_w && (uintptr_t)norm_w % 16 != 0))
    return TB_ERROR_NOT_SUPPORTED;
  // a cluster of C CTAs per row, each holding K / (4 C) float4 in registers:
  // 8 for the few rows of a decode step, down to 1 once the rows alone give
  // about two CTAs per SM (the prefill's hundreds of rows)
  int C = 8;
  while (C > 1 && ((K / 4) % C != 0 || (K / 4) / C < 64 || (int64_t)M * C / 2 >= 2 * sm_count())) C >>= 1;
  const int nvc = (K / 4) / C;
  const int vpt = (nvc + 255) / 256;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)C, (unsigned)M);
  cfg.blockDim = dim3(256);
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)C;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  cudaError_t e;
#define TB_DIGITS(NP_, VPT_) e = cudaLaunchKernelEx(&cfg, tc_digits_kernel<NP_, VPT_>, dig, srow, x, M, K, norm_w, eps)
  if (vpt > 16) return TB_ERROR_NOT_SUPPORTED;
  if (planes == 3) {
    if (vpt <= 1) TB_DIGITS(3, 1);
    else if (vpt <= 2) TB_DIGITS(3, 2);
    else if (vpt <= 4) TB_DIGITS(3, 4);
    else if (vpt <= 8) TB_DIGITS(3, 8);
    else TB_DIGITS(3, 16);
  } else {
    if (vpt <= 1) TB_DIGITS(2, 1);
    else if (vpt <= 2) TB_DIGITS(2, 2);
    else if (vpt <= 4) TB_DIGITS(2, 4);
    else if (vpt <= 8) TB_DIGITS(2, 8);
    else TB_DIGITS(2, 16);
  }
#undef TB_DIGITS
  if (e != cudaSuccess) return cuda_fail(e, "cudaLaunchKernelEx(tc_digits_kernel)");
  return TB_SUCCESS;
}

tb_status_t gemm_tc_run(float* out, const int8_t* dig, const float* srow, const int8_t* q, const float* scale,
                        const float* resid, int M, int N, int K, int planes, cudaStream_t st) {
  if (M <= 0 || N <= 0) return TB_SUCCESS;
  if (planes == 3) return launch_tc<3>(out, dig, srow, q, scale, resid, M, N, K, st);
  return launch_tc<2>(out, dig, srow, q, scale, resid, M, N, K, st);
}

bool gemm_tc_grp_ok(const void* q, int64_t M, int64_t N, int64_t K, int64_t group) {
  return group > 0 && group % kTcBK == 0 && K % group == 0 && (K / group) * kGgBN <= kGgMaxScales &&
         gemm_tc_ok(q, M, N, K) && N <= 65535 * kGgBN;
}

tb_status_t gemm_tc_grp(float* out, const float* x, const int8_t* q, const float* scale, const float* resid, int M,
                        int N, int K, int group, int planes, void* ws, cudaStream_t st) {
  int8_t* dig = static_cast<int8_t*>(ws);
  float* srow = reinterpret_cast<float*>(static_cast<unsigned char*>(ws) + gemm_tc_workspace(M, K, planes) -
                                         (size_t)M * sizeof(float));
  if (M <= 0 || N <= 0) return TB_SUCCESS;
  TB_TRY(gemm_tc_digits(dig, srow, x, M, K, planes, nullptr, 0.f, st));
  if (planes == 3) return launch_tc_grp<3>(out, dig, srow, q, scale, resid, M, N, K, group, st);
  return launch_tc_grp<2>(out, dig, srow, q, scale, resid, M, N, K, group, st);
}

tb_status_t gemm_tc(float* out, const float* x, const int8_t* q, const float* scale, const float* resid, int M, int N,
                    int K, int planes, void* ws, cudaStream_t st) {
  int8_t* dig = static_cast<int8_t*>(ws);
  float* srow = reinterpret_cast<float*>(static_cast<unsigned char*>(ws) + gemm_tc_workspace(M, K, planes) -
                                         (size_t)M * sizeof(float));
  TB_TRY(gemm_tc_digits(dig, srow, x, M, K, planes, nullptr, 0.f, st));
  return gemm_tc_run(out, dig, srow, q, scale, resid, M, N, K, planes, st);
}

}  // namespace tb
