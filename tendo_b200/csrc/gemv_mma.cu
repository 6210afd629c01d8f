// gemv_mma.cu — decode-regime dequant GEMV on the tensor cores.
//
// y[m, n] = scale[n] * sum_k x[m, k] * q[n, k] for M <= 8 batch rows.
//
// Why the tensor cores for a bandwidth-bound GEMV: on the CUDA cores every
// int8 weight costs a byte permute, a convert-add and an FMA (3+ issue slots
// per byte), which left the streaming kernel issue-bound at 45% DRAM
// throughput.  Here 16 weight bytes of one lane become 8 f16x2 operands
// (xor + byte permute + HSUB2, exact: int8 values are exact in f16) and four
// mma.m16n8k16 instructions do the 2 * 16 * 8 * 16 multiply-adds, about 1.6
// issue slots per weight byte.
//
// Operand layout.  A (16 x 16) = x: rows 0..7 are the f16 "hi" parts of the
// batch rows, rows 8..15 the "lo" parts (x = hi + lo exactly to ~22 bits),
// so y = D[m] + D[m + 8].  B (16 x 8) = W^T: column n is weight row row(n) of
// an 8-row tile.  The k order inside an mma is free as long as A and B agree:
// lane (g = lane / 4, t = lane % 4) loads 16 contiguous bytes of row row(g)
// at k = 64 kb + 16 t, and mma j of the k-block uses its bytes 4j .. 4j+3 as
// k-slots {2t, 2t+1} and {2t+8, 2t+9}; the lane's A registers hold x at the
// same 16 k.  Each x row is kept as fp32 scaled by a power of two so its
// largest value fits f16 comfortably; the scale is undone on the result.
//
// Schedule.  A CTA owns 8-row tiles (tile, tile + grid, ...); its W warps split
// K (warp w takes k-blocks w, w + W, ...), each lane keeping KPW 16-byte loads
// in flight per tile.  Partial tiles are summed across warps in shared memory
// (double-buffered, one barrier per tile) and the epilogue (scale, residual,
// RoPE + KV append, SwiGLU) runs on the reduced values.  The first tile's
// weights are requested before griddepcontrol.wait, so under programmatic
// dependent launch they stream while the previous kernel finishes.
#include <cuda_fp16.h>
#include <math.h>
#include <stdlib.h>

#include "common.cuh"
#include "kernels.h"

namespace tb {
namespace {

constexpr int kPad = 8;  // halves of padding per staged x row (bank spread)

__device__ __forceinline__ void mma_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Two signed bytes (positions lo, lo+1 of u ^ 0x80808080) as an exact f16x2.
__device__ __forceinline__ uint32_t i8pair_to_f16x2(uint32_t ux, uint32_t sel) {
  const uint32_t raw = __byte_perm(ux, 0x64646464u, sel);  // 1024 + (b + 128) per half
  const __half2 h = __hsub2(*reinterpret_cast<const __half2*>(&raw), __halves2half2(__ushort_as_half(0x6480),
                                                                                     __ushort_as_half(0x6480)));
  return *reinterpret_cast<const uint32_t*>(&h);
}

struct MmaSmem {
  // hi[MT][K + kPad], lo[MT][K + kPad] halves; then per-row scales; then the
  // double-buffered partial tiles red[2][W][8 m][8 n].
  static __host__ __device__ size_t x_halves(int MT, int K) { return (size_t)MT * (K + kPad); }
  static __host__ __device__ size_t bytes(int MT, int K, int W) {
    return 2 * x_halves(MT, K) * 2 + 16 * sizeof(float) + (size_t)2 * W * 64 * sizeof(float) +
           (size_t)2 * 8 * 32 * sizeof(float);
  }
};

// Stage x (optionally RMSNorm(x) * w) as f16 hi/lo rows scaled by 2^-e_m.
template <int MT>
__device__ void stage_x_f16(__half* hi, __half* lo, float* xscale, const float* __restrict__ x, int M, int K,
                            const float* __restrict__ norm_w, float eps, float* red) {
  const int nthreads = blockDim.x, warps = nthreads >> 5;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nv = K >> 2;
  // pass 1: sum of squares (RMSNorm) and max |x| per row
  float ss[MT], mx[MT];
#pragma unroll
  for (int m = 0; m < MT; m++) ss[m] = mx[m] = 0.f;
  for (int v = threadIdx.x; v < nv; v += nthreads) {
#pragma unroll
    for (int m = 0; m < MT; m++) {
      if (m < M) {
        const float4 t = reinterpret_cast<const float4*>(x + (size_t)m * K)[v];
        ss[m] += t.x * t.x + t.y * t.y + t.z * t.z + t.w * t.w;
        float a = fmaxf(fmaxf(fabsf(t.x), fabsf(t.y)), fmaxf(fabsf(t.z), fabsf(t.w)));
        if (norm_w) {
          const float4 w = reinterpret_cast<const float4*>(norm_w)[v];
          a = fmaxf(fmaxf(fabsf(t.x * w.x), fabsf(t.y * w.y)), fmaxf(fabsf(t.z * w.z), fabsf(t.w * w.w)));
        }
        mx[m] = fmaxf(mx[m], a);
      }
    }
  }
#pragma unroll
  for (int m = 0; m < MT; m++) {
    float s = warp_sum(ss[m]), a = warp_max(mx[m]);
    if (lane == 0) {
      red[(2 * m) * 32 + warp] = s;
      red[(2 * m + 1) * 32 + warp] = a;
    }
  }
  __syncthreads();
  float rms[MT], inv_sc[MT];
#pragma unroll
  for (int m = 0; m < MT; m++) {
    float s = 0.f, a = 0.f;
    for (int w = 0; w < warps; w++) {
      s += red[(2 * m) * 32 + w];
      a = fmaxf(a, red[(2 * m + 1) * 32 + w]);
    }
    rms[m] = norm_w ? __fsqrt_rn(__fadd_rn(__fdiv_rn(s, (float)K), eps)) : 1.0f;
    if (norm_w) a = a / rms[m] * 1.0001f;
    // power of two that brings max |x| to [2^13, 2^14): exact rescaling
    int e = 0;
    if (a > 0.f && isfinite(a)) {
      frexpf(a, &e);  // a = f * 2^e, f in [0.5, 1)
      e -= 14;
    }
    inv_sc[m] = ldexpf(1.0f, -e);
    if (threadIdx.x == 0) xscale[m] = ldexpf(1.0f, e);
  }
  // pass 2: values -> hi/lo halves
  for (int v = threadIdx.x; v < nv; v += nthreads) {
    float4 w4 = make_float4(1.f, 1.f, 1.f, 1.f);
    if (norm_w) w4 = reinterpret_cast<const float4*>(norm_w)[v];
#pragma unroll
    for (int m = 0; m < MT; m++) {
      float4 t = make_float4(0.f, 0.f, 0.f, 0.f);
      if (m < M) {
        t = reinterpret_cast<const float4*>(x + (size_t)m * K)[v];
        if (norm_w) {
          t.x = __fmul_rn(__fdiv_rn(t.x, rms[m]), w4.x);
          t.y = __fmul_rn(__fdiv_rn(t.y, rms[m]), w4.y);
          t.z = __fmul_rn(__fdiv_rn(t.z, rms[m]), w4.z);
          t.w = __fmul_rn(__fdiv_rn(t.w, rms[m]), w4.w);
        }
        t.x *= inv_sc[m];
        t.y *= inv_sc[m];
        t.z *= inv_sc[m];
        t.w *= inv_sc[m];
      }
      const float vals[4] = {t.x, t.y, t.z, t.w};
      __half h[4], l[4];
#pragma unroll
      for (int i = 0; i < 4; i++) {
        h[i] = __float2half_rn(vals[i]);
        l[i] = __float2half_rn(vals[i] - __half2float(h[i]));
      }
      __half* hp = hi + (size_t)m * (K + kPad) + 4 * v;
      __half* lp = lo + (size_t)m * (K + kPad) + 4 * v;
      *reinterpret_cast<__half2*>(hp) = __halves2half2(h[0], h[1]);
      *reinterpret_cast<__half2*>(hp + 2) = __halves2half2(h[2], h[3]);
      *reinterpret_cast<__half2*>(lp) = __halves2half2(l[0], l[1]);
      *reinterpret_cast<__half2*>(lp + 2) = __halves2half2(l[2], l[3]);
    }
  }
  __syncthreads();
}

// Row-tile plans: which 8 weight rows (one per B column) a tile covers.
struct PlainTiles {
  const int8_t* q;
  int N, K;
  __device__ int tiles() const { return (N + 7) / 8; }
  __device__ const int8_t* row(int tile, int n) const { return q + (size_t)min(tile * 8 + n, N - 1) * K; }
  __device__ void prefetch(int tile) const {
    const int r0 = tile * 8, rows = min(8, N - r0);
    if (rows > 0) prefetch_l2_bulk(q + (size_t)r0 * K, (uint32_t)(rows * K));
  }
};
struct QkvTiles {  // 4 rotate-half pairs: columns n and n + 4 are rows i and i + D/2 of one head
  const int8_t* q;
  int heads, D, K;
  __device__ int tiles() const { return heads * (D / 8); }
  __device__ int head(int tile) const { return tile / (D / 8); }
  __device__ int i0(int tile) const { return (tile % (D / 8)) * 4; }
  __device__ const int8_t* row(int tile, int n) const {
    const int r = head(tile) * D + i0(tile) + (n & 3) + (n >> 2) * (D / 2);
    return q + (size_t)r * K;
  }
  __device__ void prefetch(int tile) const {
    const int r = head(tile) * D + i0(tile);
    prefetch_l2_bulk(q + (size_t)r * K, (uint32_t)(4 * K));
    prefetch_l2_bulk(q + (size_t)(r + D / 2) * K, (uint32_t)(4 * K));
  }
};
struct GateUpTiles {  // columns 0..3: gate rows j0..j0+3; 4..7: the same up rows
  const int8_t* gate;
  const int8_t* up;
  int F, K;
  __device__ int tiles() const { return (F + 3) / 4; }
  __device__ const int8_t* row(int tile, int n) const {
    const int j = min(tile * 4 + (n & 3), F - 1);
    return ((n >> 2) ? up : gate) + (size_t)j * K;
  }
  __device__ void prefetch(int tile) const {
    const int j0 = tile * 4, rows = min(4, F - j0);
    if (rows > 0) {
      prefetch_l2_bulk(gate + (size_t)j0 * K, (uint32_t)(rows * K));
      prefetch_l2_bulk(up + (size_t)j0 * K, (uint32_t)(rows * K));
    }
  }
};

// One warp's share of one tile: k-blocks warp, warp + W, ... (KPW at most).
template <int KPW>
__device__ __forceinline__ void load_tile(int4 (&w)[KPW], const int8_t* rowp, int KB, int W, int warp, int t,
                                          int i0) {
#pragma unroll
  for (int i = 0; i < KPW; i++) {
    const int kb = warp + W * (i0 + i);
    w[i] = kb < KB ? ld_stream_v4(rowp + (size_t)kb * 64 + 16 * t) : make_int4(0, 0, 0, 0);
  }
}

template <int MT, int KPW>
__device__ __forceinline__ void mma_tile(float (&d)[4], const int4 (&w)[KPW], const __half* hi, const __half* lo,
                                         int K, int KB, int W, int warp, int g, int t, int i0) {
#pragma unroll
  for (int i = 0; i < KPW; i++) {
    const int kb = warp + W * (i0 + i);
    if (kb >= KB) break;
    uint32_t xh[8], xl[8];
    if (g < MT) {
      const uint4* ph = reinterpret_cast<const uint4*>(hi + (size_t)g * (K + kPad) + kb * 64 + 16 * t);
      const uint4* pl = reinterpret_cast<const uint4*>(lo + (size_t)g * (K + kPad) + kb * 64 + 16 * t);
      const uint4 h0 = ph[0], h1 = ph[1], l0 = pl[0], l1 = pl[1];
      xh[0] = h0.x; xh[1] = h0.y; xh[2] = h0.z; xh[3] = h0.w;
      xh[4] = h1.x; xh[5] = h1.y; xh[6] = h1.z; xh[7] = h1.w;
      xl[0] = l0.x; xl[1] = l0.y; xl[2] = l0.z; xl[3] = l0.w;
      xl[4] = l1.x; xl[5] = l1.y; xl[6] = l1.z; xl[7] = l1.w;
    } else {
#pragma unroll
      for (int p = 0; p < 8; p++) xh[p] = xl[p] = 0u;
    }
    const uint32_t words[4] = {(uint32_t)w[i].x, (uint32_t)w[i].y, (uint32_t)w[i].z, (uint32_t)w[i].w};
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const uint32_t ux = words[j] ^ 0x80808080u;
      const uint32_t b0 = i8pair_to_f16x2(ux, 0x4140);
      const uint32_t b1 = i8pair_to_f16x2(ux, 0x4342);
      const uint32_t a[4] = {xh[2 * j], xl[2 * j], xh[2 * j + 1], xl[2 * j + 1]};
      mma_16816(d, a, b0, b1);
    }
  }
}

// Partial tile of this warp -> red[buf][warp][m][n] (m < MT): y = D[m] + D[m + 8].
template <int MT>
__device__ __forceinline__ void store_partial(float* red, const float (&d)[4], int warp, int g, int t) {
  if (g < MT) {
    float* r = red + (size_t)warp * 64 + g * 8 + 2 * t;
    r[0] = d[0] + d[2];
    r[1] = d[1] + d[3];
  }
}

template <int MT>
__device__ __forceinline__ float reduce_partial(const float* red, int W, int m, int n) {
  float s = 0.f;
  for (int w = 0; w < W; w++) s += red[(size_t)w * 64 + m * 8 + n];
  return s;
}

// ---------------------------------------------------------------------------
// Generic driver.  Tiles maps tiles to rows; Epi(tile, m, n, y, valid) is
// called by whole warps (threads m * 8 + n), so partner columns n and n ^ 4
// can meet through __shfl_xor_sync(.., 4); y already carries the x scale.
// ---------------------------------------------------------------------------
template <int MT, int KPW, typename Tiles, typename Epi>
__device__ __forceinline__ void gemv_mma_body(const Tiles& tiles, const Epi& epi, const float* __restrict__ x,
                                              int M, int K, const float* __restrict__ norm_w, float eps,
                                              bool l2_prefetch) {
  extern __shared__ __align__(16) unsigned char smem[];
  __half* hi = reinterpret_cast<__half*>(smem);
  __half* lo = hi + MmaSmem::x_halves(MT, K);
  float* xscale = reinterpret_cast<float*>(lo + MmaSmem::x_halves(MT, K));
  const int W = blockDim.x >> 5;
  float* red = xscale + 16;  // [2][W][64]
  float* scratch = red + 2 * W * 64;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int KB = K >> 6;
  const int ntiles = tiles.tiles();
  const int nrounds = ((KB + W - 1) / W + KPW - 1) / KPW;
  int tile = blockIdx.x;
  // The TMA unit streams this CTA's next kPrefetch tiles into L2 ahead of the
  // register loads (weights never depend on the preceding kernel).
  constexpr int kPrefetch = 4;
  if (l2_prefetch && threadIdx.x == 0)
    for (int i = 0; i < kPrefetch; i++)
      if (tile + i * (int)gridDim.x < ntiles) tiles.prefetch(tile + i * gridDim.x);
  int4 w[KPW];
  if (tile < ntiles) load_tile<KPW>(w, tiles.row(tile, g), KB, W, warp, t, 0);
  pdl_wait();
  pdl_launch_dependents();
  stage_x_f16<MT>(hi, lo, xscale, x, M, K, norm_w, eps, scratch);
  constexpr int kEpiThreads = ((MT * 8 + 31) / 32) * 32;
  int buf = 0;
  for (; tile < ntiles; tile += gridDim.x) {
    float d[4] = {0.f, 0.f, 0.f, 0.f};
    if (l2_prefetch && threadIdx.x == 0 && tile + kPrefetch * (int)gridDim.x < ntiles)
      tiles.prefetch(tile + kPrefetch * gridDim.x);
    const int8_t* rowp = tiles.row(tile, g);
    for (int r = 0; r < nrounds; r++) {
      if (r > 0) load_tile<KPW>(w, rowp, KB, W, warp, t, r * KPW);
      mma_tile<MT, KPW>(d, w, hi, lo, K, KB, W, warp, g, t, r * KPW);
    }
    const int next = tile + gridDim.x;
    if (next < ntiles) load_tile<KPW>(w, tiles.row(next, g), KB, W, warp, t, 0);
    float* rb = red + (size_t)buf * W * 64;
    store_partial<MT>(rb, d, warp, g, t);
    __syncthreads();
    if (threadIdx.x < kEpiThreads) {
      const int m = threadIdx.x >> 3, n = threadIdx.x & 7;
      const bool valid = m < M && m < MT;
      const float y = valid ? reduce_partial<MT>(rb, W, m, n) * xscale[m] : 0.f;
      epi(tile, m, n, y, valid);
    }
    buf ^= 1;
  }
}

struct PlainEpi {
  float* out;
  const float* scale;
  const float* resid;
  int N;
  __device__ __forceinline__ void operator()(int tile, int m, int n, float y, bool valid) const {
    const int r = tile * 8 + n;
    if (!valid || r >= N) return;
    float v = y * scale[r];
    if (resid) v += resid[(size_t)m * N + r];
    out[(size_t)m * N + r] = v;
  }
  // Split form for the TMA kernel: pre() issues the global loads early.
  __device__ __forceinline__ float4 pre(int tile, int m, int n, bool valid) const {
    const int r = tile * 8 + n;
    float4 c = make_float4(0.f, 0.f, 0.f, 0.f);
    if (valid && r < N) {
      c.x = scale[r];
      if (resid) c.y = resid[(size_t)m * N + r];
    }
    return c;
  }
  __device__ __forceinline__ void post(int tile, int m, int n, float y, bool valid, float4 c) const {
    const int r = tile * 8 + n;
    if (!valid || r >= N) return;
    out[(size_t)m * N + r] = resid ? y * c.x + c.y : y * c.x;
  }
};

// Column n < 4 holds row i of a head, column n + 4 row i + D/2: rotate-half
// at position pos (nn/rope.go:141-197), then q -> qout, k -> cache (post-RoPE),
// v -> cache (raw).
struct QkvEpi {
  QkvArgs a;
  QkvTiles tiles;
  int64_t pos;
  __device__ __forceinline__ void operator()(int tile, int m, int n, float y, bool valid) const {
    const int half = a.D / 2;
    const int head = tiles.head(tile), i = tiles.i0(tile) + (n & 3);
    const int r = head * a.D + i + (n >> 2) * half;
    const float v = valid ? y * a.scale[r] : 0.f;
    const float partner = __shfl_xor_sync(0xffffffffu, v, 4);
    if (!valid || n >= 4) return;
    const float x0 = v, x1 = partner;
    if (head < a.H + a.Hkv) {
      const float c = a.cos_t[pos * half + i], sn = a.sin_t[pos * half + i];
      const float o0 = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, sn));
      const float o1 = __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, c));
      float* o = head < a.H ? a.qout + ((size_t)m * a.H + head) * a.D
                            : a.kcache + (((size_t)m * a.Hkv + (head - a.H)) * a.max_seq + pos) * a.D;
      o[i] = o0;
      o[i + half] = o1;
    } else {
      float* o = a.vcache + (((size_t)m * a.Hkv + (head - a.H - a.Hkv)) * a.max_seq + pos) * a.D;
      o[i] = x0;
      o[i + half] = x1;
    }
  }
  __device__ __forceinline__ float4 pre(int tile, int m, int n, bool valid) const {
    const int half = a.D / 2;
    const int head = tiles.head(tile), i = tiles.i0(tile) + (n & 3);
    const int r = head * a.D + i + (n >> 2) * half;
    float4 c = make_float4(0.f, 0.f, 0.f, 0.f);
    if (valid) {
      c.x = a.scale[r];
      c.y = a.cos_t[pos * half + i];
      c.z = a.sin_t[pos * half + i];
    }
    return c;
  }
  __device__ __forceinline__ void post(int tile, int m, int n, float y, bool valid, float4 c) const {
    const int half = a.D / 2;
    const int head = tiles.head(tile), i = tiles.i0(tile) + (n & 3);
    const float v = valid ? y * c.x : 0.f;
    const float partner = __shfl_xor_sync(0xffffffffu, v, 4);
    if (!valid || n >= 4) return;
    const float x0 = v, x1 = partner;
    if (head < a.H + a.Hkv) {
      const float o0 = __fsub_rn(__fmul_rn(x0, c.y), __fmul_rn(x1, c.z));
      const float o1 = __fadd_rn(__fmul_rn(x0, c.z), __fmul_rn(x1, c.y));
      float* o = head < a.H ? a.qout + ((size_t)m * a.H + head) * a.D
                            : a.kcache + (((size_t)m * a.Hkv + (head - a.H)) * a.max_seq + pos) * a.D;
      o[i] = o0;
      o[i + half] = o1;
    } else {
      float* o = a.vcache + (((size_t)m * a.Hkv + (head - a.H - a.Hkv)) * a.max_seq + pos) * a.D;
      o[i] = x0;
      o[i + half] = x1;
    }
  }
};

// Columns 0..3 gate rows j0.., 4..7 the same up rows: act = silu(gate) * up.
struct GateUpEpi {
  GateUpArgs a;
  __device__ __forceinline__ void operator()(int tile, int m, int n, float y, bool valid) const {
    const int j = tile * 4 + (n & 3);
    const bool in = valid && j < a.F;
    const float v = in ? y * ((n >> 2) ? a.up_scale[j] : a.gate_scale[j]) : 0.f;
    const float partner = __shfl_xor_sync(0xffffffffu, v, 4);
    if (!in || n >= 4) return;
    const float sig = 1.0f / (1.0f + expf(-v));
    a.act[(size_t)m * a.F + j] = (v * sig) * partner;
  }
  __device__ __forceinline__ float4 pre(int tile, int m, int n, bool valid) const {
    const int j = tile * 4 + (n & 3);
    float4 c = make_float4(0.f, 0.f, 0.f, 0.f);
    if (valid && j < a.F) c.x = (n >> 2) ? a.up_scale[j] : a.gate_scale[j];
    return c;
  }
  __device__ __forceinline__ void post(int tile, int m, int n, float y, bool valid, float4 c) const {
    const int j = tile * 4 + (n & 3);
    const bool in = valid && j < a.F;
    const float v = in ? y * c.x : 0.f;
    const float partner = __shfl_xor_sync(0xffffffffu, v, 4);
    if (!in || n >= 4) return;
    const float sig = 1.0f / (1.0f + expf(-v));
    a.act[(size_t)m * a.F + j] = (v * sig) * partner;
  }
};

template <int MT, int KPW>
__global__ void __launch_bounds__(512) gemv_mma_plain_kernel(float* out, const float* __restrict__ x,
                                                              const int8_t* __restrict__ q,
                                                              const float* __restrict__ scale, const float* resid,
                                                              int M, int N, int K, const float* __restrict__ norm_w,
                                                              float eps, bool l2_prefetch) {
  const PlainTiles tiles{q, N, K};
  const PlainEpi epi{out, scale, resid, N};
  gemv_mma_body<MT, KPW>(tiles, epi, x, M, K, norm_w, eps, l2_prefetch);
}

template <int MT, int KPW>
__global__ void __launch_bounds__(512) gemv_mma_qkv_kernel(QkvArgs a, bool l2_prefetch) {
  const QkvTiles tiles{a.q, a.H + 2 * a.Hkv, a.D, a.d};
  // The position was written by an earlier step's tail kernel, complete before
  // the preceding kernel could launch this one (programmatic launch chain).
  const QkvEpi epi{a, tiles, *a.pos};
  gemv_mma_body<MT, KPW>(tiles, epi, a.h, a.M, a.d, a.norm_w, a.eps, l2_prefetch);
}

template <int MT, int KPW>
__global__ void __launch_bounds__(512) gemv_mma_gateup_kernel(GateUpArgs a, bool l2_prefetch) {
  const GateUpTiles tiles{a.gate, a.up, a.F, a.d};
  const GateUpEpi epi{a};
  gemv_mma_body<MT, KPW>(tiles, epi, a.h, a.M, a.d, a.norm_w, a.eps, l2_prefetch);
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
// ---------------------------------------------------------------------------
// TMA-fed variant: the weight stream goes global -> shared memory through the
// TMA unit (cp.async.bulk, mbarrier completion) instead of register loads, so
// the bytes in flight per SM are set by the stage count, not by the L1 miss
// machinery.  One producer warp (one elected thread) runs up to `stages`
// chunks ahead, starting before griddepcontrol.wait; W consumer warps convert
// and multiply from shared memory.  A chunk is 8 rows x Kc bytes (Kc divides
// K, at most 4096); each row lands at stride RS = Kc (+64 when Kc is a
// multiple of 128) so the lanes of a 16-byte shared load hit distinct banks.
// Every wait is bounded: on expiry the kernel counts the event in
// g_wait_timeouts and carries on, so the host sees an error instead of a hang.
// ---------------------------------------------------------------------------
__device__ int g_wait_timeouts;

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// Waits for the phase of parity `parity`; gives up after a bounded number of
// polls (seconds at most) and records the timeout.
__device__ __forceinline__ void mbar_wait(uint64_t* bar, uint32_t parity) {
  const uint32_t a = smem_u32(bar);
  for (uint32_t it = 0; it < (1u << 24); it++) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
        : "=r"(done)
        : "r"(a), "r"(parity)
        : "memory");
    if (done) return;
  }
  atomicAdd(&g_wait_timeouts, 1);
}
__device__ __forceinline__ void tma_load_1d(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void consumer_sync(int nthreads) {
  asm volatile("bar.sync 1, %0;" ::"r"(nthreads) : "memory");
}

// Stage x (optionally RMSNorm(x) * w) as three int8 digit rows per batch row:
// u = v / s with s = max|v| / 127, d0 = rint(u), d1 = rint((u - d0) * 128),
// d2 = rint(((u - d0) * 128 - d1) * 128); u = d0 + d1 / 128 + d2 / 128^2 to
// within 2^-15 (every remainder step is exact in fp32).  Digit p of row m goes
// to digit row p * M + m (stride RSX bytes); rows 3M .. 16 RG - 1 are zero.
template <int RG>
__device__ void stage_x_digits(int8_t* dig, int RSX, float* xscale, const float* __restrict__ x, int M, int K,
                               const float* __restrict__ norm_w, float eps, float* red, int nthreads) {
  const int warps = nthreads >> 5;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nv = K >> 2;
  constexpr int MX = 16 * RG / 3 + 1;  // batch rows this layout can hold (5 or 10)
  float ss[MX], mx[MX];
#pragma unroll
  for (int m = 0; m < MX; m++) ss[m] = mx[m] = 0.f;
  for (int v = threadIdx.x; v < nv; v += nthreads) {
    float4 w4 = make_float4(1.f, 1.f, 1.f, 1.f);
    if (norm_w) w4 = reinterpret_cast<const float4*>(norm_w)[v];
#pragma unroll
    for (int m = 0; m < MX; m++) {
      if (m < M) {
        const float4 t = reinterpret_cast<const float4*>(x + (size_t)m * K)[v];
        ss[m] += t.x * t.x + t.y * t.y + t.z * t.z + t.w * t.w;
        mx[m] = fmaxf(mx[m], fmaxf(fmaxf(fabsf(t.x * w4.x), fabsf(t.y * w4.y)),
                                   fmaxf(fabsf(t.z * w4.z), fabsf(t.w * w4.w))));
      }
    }
  }
#pragma unroll
  for (int m = 0; m < MX; m++) {
    const float s = warp_sum(ss[m]), a = warp_max(mx[m]);
    if (lane == 0) {
      red[(2 * m) * 32 + warp] = s;
      red[(2 * m + 1) * 32 + warp] = a;
    }
  }
  consumer_sync(nthreads);
  float rms[MX], inv[MX];
#pragma unroll
  for (int m = 0; m < MX; m++) {
    float s = 0.f, a = 0.f;
    for (int w = 0; w < warps; w++) {
      s += red[(2 * m) * 32 + w];
      a = fmaxf(a, red[(2 * m + 1) * 32 + w]);
    }
    rms[m] = norm_w ? __fsqrt_rn(__fadd_rn(__fdiv_rn(s, (float)K), eps)) : 1.0f;
    if (norm_w) a = a / rms[m] * 1.0001f;  // bound of max |x / rms * w|
    const float sc = (a > 0.f && isfinite(a)) ? a / 127.0f : 1.0f;
    inv[m] = 1.0f / sc;
    if (threadIdx.x == 0 && m < M) xscale[m] = sc;
  }
  for (int v = threadIdx.x; v < nv; v += nthreads) {
    float4 w4 = make_float4(1.f, 1.f, 1.f, 1.f);
    if (norm_w) w4 = reinterpret_cast<const float4*>(norm_w)[v];
#pragma unroll
    for (int m = 0; m < MX; m++) {
      if (m >= M) continue;
      float4 t = reinterpret_cast<const float4*>(x + (size_t)m * K)[v];
      if (norm_w) {
        t.x = __fmul_rn(__fdiv_rn(t.x, rms[m]), w4.x);
        t.y = __fmul_rn(__fdiv_rn(t.y, rms[m]), w4.y);
        t.z = __fmul_rn(__fdiv_rn(t.z, rms[m]), w4.z);
        t.w = __fmul_rn(__fdiv_rn(t.w, rms[m]), w4.w);
      }
      const float vals[4] = {t.x, t.y, t.z, t.w};
      uint32_t p0 = 0, p1 = 0, p2 = 0;
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const float u = fminf(fmaxf(vals[i] * inv[m], -127.0f), 127.0f);
        const float d0 = rintf(u);
        const float r1 = (u - d0) * 128.0f;
        const float d1 = rintf(r1);
        const float d2 = rintf((r1 - d1) * 128.0f);
        p0 |= ((uint32_t)(int)d0 & 0xffu) << (8 * i);
        p1 |= ((uint32_t)(int)d1 & 0xffu) << (8 * i);
        p2 |= ((uint32_t)(int)d2 & 0xffu) << (8 * i);
      }
      *reinterpret_cast<uint32_t*>(dig + (size_t)(0 * M + m) * RSX + 4 * v) = p0;
      *reinterpret_cast<uint32_t*>(dig + (size_t)(1 * M + m) * RSX + 4 * v) = p1;
      *reinterpret_cast<uint32_t*>(dig + (size_t)(2 * M + m) * RSX + 4 * v) = p2;
    }
  }
  // zero the unused digit rows
  for (int i = threadIdx.x; i < (16 * RG - 3 * M) * (K / 4); i += nthreads) {
    const int r = 3 * M + i / (K / 4), c = i % (K / 4);
    *reinterpret_cast<uint32_t*>(dig + (size_t)r * RSX + 4 * c) = 0u;
  }
  consumer_sync(nthreads);
}

__device__ __forceinline__ void imma_16832(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                           uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

struct TmaLayout {
  int Kc, RS, RSX, stages, W;
  size_t stage_bytes, x_off, xs_off, red_off, scr_off, bar_off, total;
  __host__ __device__ static int stride(int bytes) { return (bytes % 128 == 0) ? bytes + 64 : bytes; }
  __host__ __device__ void init(int RG, int K, int Kc_, int stages_, int W_) {
    Kc = Kc_;
    RS = stride(Kc);
    RSX = stride(K);
    stages = stages_;
    W = W_;
    stage_bytes = (size_t)8 * RS;
    x_off = (size_t)stages * stage_bytes;
    xs_off = x_off + (size_t)16 * RG * RSX;
    red_off = (xs_off + 16 * sizeof(float) + 15) & ~(size_t)15;
    scr_off = red_off + (size_t)2 * W * 16 * RG * 8 * sizeof(int);
    bar_off = (scr_off + 2 * 16 * 32 * sizeof(float) + 15) & ~(size_t)15;
    total = bar_off + (size_t)2 * stages * sizeof(uint64_t);
  }
};

// RG row groups of 16 digit rows: RG = 1 serves M <= 5, RG = 2 serves M <= 8.
template <int RG, typename Tiles, typename Epi>
__device__ __forceinline__ void gemv_tma_body(const Tiles& tiles, const Epi& epi, const float* __restrict__ x, int M,
                                              int K, const float* __restrict__ norm_w, float eps, int Kc,
                                              int stages) {
  extern __shared__ __align__(128) unsigned char smem[];
  const int W = (int)(blockDim.x >> 5) - 1;  // consumer warps; warp W produces
  TmaLayout L;
  L.init(RG, K, Kc, stages, W);
  unsigned char* stage_base = smem;
  int8_t* dig = reinterpret_cast<int8_t*>(smem + L.x_off);
  float* xscale = reinterpret_cast<float*>(smem + L.xs_off);
  int* red = reinterpret_cast<int*>(smem + L.red_off);
  float* scratch = reinterpret_cast<float*>(smem + L.scr_off);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bar_off);
  uint64_t* empty = full + stages;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nch = K / Kc, kbc = Kc / 64;
  const int ntiles = tiles.tiles();
  const int my_tiles = ntiles > (int)blockIdx.x ? (ntiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
  const int units = my_tiles * nch;
  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], (uint32_t)(W * 32));
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if (warp == W) {
    // producer: weights never depend on the preceding kernel, so no wait here
    if (lane == 0) {
      for (int u = 0; u < units; u++) {
        const int s = u % stages, use = u / stages;
        if (use > 0) mbar_wait(&empty[s], (uint32_t)((use - 1) & 1));
        const int tile = (int)blockIdx.x + (u / nch) * (int)gridDim.x, ch = u % nch;
        unsigned char* dst = stage_base + (size_t)s * L.stage_bytes;
        mbar_expect_tx(&full[s], (uint32_t)(8 * Kc));
#pragma unroll
        for (int n = 0; n < 8; n++)
          tma_load_1d(dst + (size_t)n * L.RS, tiles.row(tile, n) + (size_t)ch * Kc, (uint32_t)Kc, &full[s]);
      }
      // every copy completes before the consumers release its stage, so the
      // CTA never exits with a copy in flight
    }
    pdl_launch_dependents();
    return;
  }
  pdl_wait();
  pdl_launch_dependents();
  const int nthreads = W * 32;
  stage_x_digits<RG>(dig, L.RSX, xscale, x, M, K, norm_w, eps, scratch, nthreads);
  const int g = lane >> 2, t = lane & 3;
  constexpr int MXT = RG == 1 ? 5 : 8;           // batch rows per launch
  constexpr int kEpiThreads = ((MXT * 8 + 31) / 32) * 32;
  constexpr int kEpiWarps = kEpiThreads / 32;
  const int epi_groups = W / kEpiWarps;
  const int R = 3 * M;
  int d[RG][4];
  int buf = 0;
  for (int u = 0; u < units; u++) {
    const int s = u % stages, use = u / stages, ch = u % nch, it = u / nch;
    const int tile = (int)blockIdx.x + it * (int)gridDim.x;
    // the epilogue of tile `it` runs on warps [ew0, ew0 + kEpiWarps), rotating
    const int ew0 = (it % epi_groups) * kEpiWarps;
    const bool is_epi = ch == nch - 1 && warp >= ew0 && warp < ew0 + kEpiWarps;
    const int et = (int)threadIdx.x - ew0 * 32, em = et >> 3, en = et & 7;
    const bool evalid = em < M;
    float4 ec = make_float4(0.f, 0.f, 0.f, 0.f);
    if (is_epi) ec = epi.pre(tile, em, en, evalid);  // global loads overlap the MMA work below
    if (ch == 0) {
#pragma unroll
      for (int rg = 0; rg < RG; rg++) d[rg][0] = d[rg][1] = d[rg][2] = d[rg][3] = 0;
    }
    mbar_wait(&full[s], (uint32_t)(use & 1));
    const unsigned char* st = stage_base + (size_t)s * L.stage_bytes + (size_t)g * L.RS + 16 * t;
    const int8_t* xr = dig + (size_t)g * L.RSX + ch * Kc + 16 * t;
#pragma unroll 4
    for (int kb = warp; kb < kbc; kb += W) {
      const uint4 wv = *reinterpret_cast<const uint4*>(st + kb * 64);
#pragma unroll
      for (int rg = 0; rg < RG; rg++) {
        const uint4 xa = *reinterpret_cast<const uint4*>(xr + (size_t)(16 * rg) * L.RSX + kb * 64);
        const uint4 xb = *reinterpret_cast<const uint4*>(xr + (size_t)(16 * rg + 8) * L.RSX + kb * 64);
        imma_16832(d[rg], xa.x, xb.x, xa.y, xb.y, wv.x, wv.y);
        imma_16832(d[rg], xa.z, xb.z, xa.w, xb.w, wv.z, wv.w);
      }
    }
    mbar_arrive(&empty[s]);
    if (ch == nch - 1) {
      // partial tile of this warp: red[buf][warp][row][n], rows < 3M
      int* rb = red + (size_t)buf * W * (16 * RG * 8);
      int* rw = rb + (size_t)warp * (16 * RG * 8);
#pragma unroll
      for (int rg = 0; rg < RG; rg++) {
        const int r0 = 16 * rg + g, r1 = r0 + 8;
        if (r0 < R) {
          rw[r0 * 8 + 2 * t] = d[rg][0];
          rw[r0 * 8 + 2 * t + 1] = d[rg][1];
        }
        if (r1 < R) {
          rw[r1 * 8 + 2 * t] = d[rg][2];
          rw[r1 * 8 + 2 * t + 1] = d[rg][3];
        }
      }
      consumer_sync(nthreads);
      if (warp >= ew0 && warp < ew0 + kEpiWarps) {
        float y = 0.f;
        if (evalid) {
          int s0 = 0, s1 = 0, s2 = 0;
          for (int w = 0; w < W; w++) {
            const int* p = rb + (size_t)w * (16 * RG * 8);
            s0 += p[(0 * M + em) * 8 + en];
            s1 += p[(1 * M + em) * 8 + en];
            s2 += p[(2 * M + em) * 8 + en];
          }
          y = xscale[em] * ((float)s0 + (float)s1 * (1.0f / 128.0f) + (float)s2 * (1.0f / 16384.0f));
        }
        epi.post(tile, em, en, y, evalid, ec);
      }
      buf ^= 1;
    }
  }
}

template <int RG>
__global__ void __launch_bounds__(288) gemv_tma_plain_kernel(float* out, const float* __restrict__ x,
                                                             const int8_t* __restrict__ q,
                                                             const float* __restrict__ scale, const float* resid,
                                                             int M, int N, int K, const float* __restrict__ norm_w,
                                                             float eps, int Kc, int stages) {
  const PlainTiles tiles{q, N, K};
  const PlainEpi epi{out, scale, resid, N};
  gemv_tma_body<RG>(tiles, epi, x, M, K, norm_w, eps, Kc, stages);
}

template <int RG>
__global__ void __launch_bounds__(288) gemv_tma_qkv_kernel(QkvArgs a, int Kc, int stages) {
  const QkvTiles tiles{a.q, a.H + 2 * a.Hkv, a.D, a.d};
  // The position was written by an earlier step's tail kernel, complete before
  // the preceding kernel could launch this one (programmatic launch chain).
  const QkvEpi epi{a, tiles, *a.pos};
  gemv_tma_body<RG>(tiles, epi, a.h, a.M, a.d, a.norm_w, a.eps, Kc, stages);
}

template <int RG>
__global__ void __launch_bounds__(288) gemv_tma_gateup_kernel(GateUpArgs a, int Kc, int stages) {
  const GateUpTiles tiles{a.gate, a.up, a.F, a.d};
  const GateUpEpi epi{a};
  gemv_tma_body<RG>(tiles, epi, a.h, a.M, a.d, a.norm_w, a.eps, Kc, stages);
}

struct MmaShape {
  int kpw, warps;
};

// At most 16 warps (the 512-thread launch bound keeps 128 registers per
// thread); KPW loads per lane per round; more k-blocks than 16 * 16 run in
// several rounds per tile.  Enough warps for the epilogue (MT * 8 threads).
MmaShape mma_shape(int K, int MT) {
  const int KB = K / 64;
  MmaShape s;
  s.kpw = KB <= 128 ? 8 : (KB <= 192 ? 12 : 16);
  s.warps = (KB + s.kpw - 1) / s.kpw;
  if (s.warps > 16) s.warps = 16;
  const int min_w = (MT * 8 + 31) / 32;
  if (s.warps < min_w) s.warps = min_w;
  return s;
}

template <typename Kern, typename... Args>
tb_status_t launch_mma(Kern kern, int64_t tiles, int warps, size_t smem, cudaStream_t st, bool pdl, Args... args) {
  if (smem > 48 * 1024) {
    cudaError_t e0 = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e0 != cudaSuccess) return cuda_fail(e0, "cudaFuncSetAttribute(gemv_mma)");
  }
  int occ = 0;
  cudaError_t e = cudaSuccess;
  {
    // occupancy per (kernel, block, smem), cached: the query costs microseconds of host time
    static thread_local const void* ck[16];
    static thread_local int cw[16], co[16];
    static thread_local size_t cs[16];
    static thread_local int cn = 0;
    int hit = -1;
    for (int i = 0; i < cn; i++)
      if (ck[i] == (const void*)kern && cw[i] == warps && cs[i] == smem) hit = i;
    if (hit >= 0) {
      occ = co[hit];
    } else {
      e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, warps * 32, smem);
      if (e != cudaSuccess) return cuda_fail(e, "cudaOccupancyMaxActiveBlocksPerMultiprocessor");
      const int slot = cn < 16 ? cn++ : 15;
      ck[slot] = (const void*)kern;
      cw[slot] = warps;
      cs[slot] = smem;
      co[slot] = occ;
    }
  }
  if (occ < 1) return TB_ERROR_NOT_SUPPORTED;
  if (occ > 4) occ = 4;
  int64_t grid = (int64_t)sm_count() * occ;
  if (grid > tiles) grid = tiles;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(warps * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  e = cudaLaunchKernelEx(&cfg, kern, args...);
  if (e != cudaSuccess) return cuda_fail(e, "cudaLaunchKernelEx(gemv_mma)");
  return TB_SUCCESS;
}

int mt_of(int M) { return M <= 1 ? 1 : (M <= 2 ? 2 : (M <= 4 ? 4 : 8)); }


#define TB_MMA_DISPATCH(KERN, MT_, KPW_, ...)                                               \
  do {                                                                                      \
    if (KPW_ == 12) {                                                                       \
      switch (MT_) {                                                                        \
        case 1: return launch_mma(KERN<1, 12>, __VA_ARGS__);                                \
        case 2: return launch_mma(KERN<2, 12>, __VA_ARGS__);                                \
        case 4: return launch_mma(KERN<4, 12>, __VA_ARGS__);                                \
        default: return launch_mma(KERN<8, 12>, __VA_ARGS__);                               \
      }                                                                                     \
    } else if (KPW_ == 8) {                                                                 \
      switch (MT_) {                                                                        \
        case 1: return launch_mma(KERN<1, 8>, __VA_ARGS__);                                 \
        case 2: return launch_mma(KERN<2, 8>, __VA_ARGS__);                                 \
        case 4: return launch_mma(KERN<4, 8>, __VA_ARGS__);                                 \
        default: return launch_mma(KERN<8, 8>, __VA_ARGS__);                                \
      }                                                                                     \
    } else {                                                                                \
      switch (MT_) {                                                                        \
        case 1: return launch_mma(KERN<1, 16>, __VA_ARGS__);                                \
        case 2: return launch_mma(KERN<2, 16>, __VA_ARGS__);                                \
        case 4: return launch_mma(KERN<4, 16>, __VA_ARGS__);                                \
        default: return launch_mma(KERN<8, 16>, __VA_ARGS__);                               \
      }                                                                                     \
    }                                                                                       \
  } while (0)

}  // namespace

// TMA bulk L2 prefetch of upcoming tiles (TENDO_B200_L2PF=1); off by default:
// measured slower than plain streaming loads on the decode shapes.
bool l2_prefetch_enabled() {
  static const bool on = [] {
    const char* e = getenv("TENDO_B200_L2PF");
    return e && e[0] == '1';
  }();
  return on;
}

bool gemv_mma_ok(const float* x, const int8_t* q, int64_t M, int64_t K) {
  if (M < 1 || M > 8 || K % 64 != 0 || K > 65536) return false;
  if (!aligned(x, 16) || !aligned(q, 16)) return false;
  const MmaShape s = mma_shape((int)K, mt_of((int)M));
  return MmaSmem::bytes(mt_of((int)M), (int)K, s.warps) <= 200 * 1024;
}

tb_status_t gemv_mma_plain(float* out, const float* x, const int8_t* q, const float* scale, const float* resid, int M,
                           int N, int K, const float* norm_w, float eps, cudaStream_t st, bool pdl) {
  const int MT = mt_of(M);
  const MmaShape s = mma_shape(K, MT);
  const size_t smem = MmaSmem::bytes(MT, K, s.warps);
  const int64_t tiles = (N + 7) / 8;
  TB_MMA_DISPATCH(gemv_mma_plain_kernel, MT, s.kpw, tiles, s.warps, smem, st, pdl, out, x, q, scale, resid, M, N, K,
                  norm_w, eps, l2_prefetch_enabled());
}

tb_status_t gemv_mma_qkv(const QkvArgs& a, cudaStream_t st, bool pdl) {
  const int MT = mt_of(a.M);
  const MmaShape s = mma_shape(a.d, MT);
  const size_t smem = MmaSmem::bytes(MT, a.d, s.warps);
  const int64_t tiles = (int64_t)(a.H + 2 * a.Hkv) * (a.D / 8);
  TB_MMA_DISPATCH(gemv_mma_qkv_kernel, MT, s.kpw, tiles, s.warps, smem, st, pdl, a, l2_prefetch_enabled());
}

tb_status_t gemv_mma_gateup(const GateUpArgs& a, cudaStream_t st, bool pdl) {
  const int MT = mt_of(a.M);
  const MmaShape s = mma_shape(a.d, MT);
  const size_t smem = MmaSmem::bytes(MT, a.d, s.warps);
  const int64_t tiles = (a.F + 3) / 4;
  TB_MMA_DISPATCH(gemv_mma_gateup_kernel, MT, s.kpw, tiles, s.warps, smem, st, pdl, a, l2_prefetch_enabled());
}

}  // namespace tb

// ---------------------------------------------------------------------------
// TMA-fed launchers
// ---------------------------------------------------------------------------
namespace tb {
namespace {

struct TmaPlan {
  int Kc, stages, W, ctas_per_sm;
  size_t smem;
};

// Chunk width: the largest divisor of K/64 k-blocks that keeps Kc <= 4096
// bytes; as many stages as fit (2..4) next to the staged x.
bool tma_plan(int RG, int K, TmaPlan* p) {
  if (K % 64 != 0) return false;
  const int KB = K / 64;
  int d = 1;
  while (KB / d > 64 || KB % d != 0) d++;
  p->Kc = 64 * (KB / d);
  const int kbc = KB / d;
  p->W = kbc < 8 ? kbc : 8;
  const int min_w = RG == 1 ? 2 : 2;  // the epilogue takes up to two warps
  if (p->W < min_w) p->W = min_w;
  // two CTAs per SM when two stages each fit in half the shared memory, so
  // one CTA's tile barrier and epilogue overlap the other's streaming
  for (int s = 3; s >= 2; s--) {
    TmaLayout L;
    L.init(RG, K, p->Kc, s, p->W);
    if (L.total <= 110 * 1024) {
      p->stages = s;
      p->smem = L.total;
      p->ctas_per_sm = 2;
      return true;
    }
  }
  for (int s = 4; s >= 2; s--) {
    TmaLayout L;
    L.init(RG, K, p->Kc, s, p->W);
    if (L.total <= 220 * 1024) {
      p->stages = s;
      p->smem = L.total;
      p->ctas_per_sm = 1;
      return true;
    }
  }
  return false;
}

template <typename Kern, typename... Args>
tb_status_t launch_tma(Kern kern, int64_t tiles, const TmaPlan& p, cudaStream_t st, bool pdl, Args... args) {
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)p.smem);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(gemv_tma)");
  int64_t grid = (int64_t)sm_count() * p.ctas_per_sm;
  if (grid > tiles) grid = tiles;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3((p.W + 1) * 32);
  cfg.dynamicSmemBytes = p.smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  e = cudaLaunchKernelEx(&cfg, kern, args...);
  if (e != cudaSuccess) return cuda_fail(e, "cudaLaunchKernelEx(gemv_tma)");
  return TB_SUCCESS;
}

#define TB_TMA_DISPATCH(KERN, RG_, ...)                                  \
  do {                                                                   \
    if (RG_ == 1) return launch_tma(KERN<1>, __VA_ARGS__);               \
    return launch_tma(KERN<2>, __VA_ARGS__);                             \
  } while (0)

int rg_of(int M) { return M <= 5 ? 1 : 2; }

}  // namespace

bool gemv_tma_ok(const float* x, const int8_t* q, int64_t M, int64_t K) {
  if (M < 1 || M > 8 || K % 64 != 0 || K > 65536) return false;
  if (!aligned(x, 16) || !aligned(q, 16)) return false;
  TmaPlan p;
  return tma_plan(rg_of((int)M), (int)K, &p);
}

tb_status_t gemv_tma_plain(float* out, const float* x, const int8_t* q, const float* scale, const float* resid, int M,
                           int N, int K, const float* norm_w, float eps, cudaStream_t st, bool pdl) {
  const int RG = rg_of(M);
  TmaPlan p;
  if (!tma_plan(RG, K, &p)) return TB_ERROR_NOT_SUPPORTED;
  const int64_t tiles = (N + 7) / 8;
  TB_TMA_DISPATCH(gemv_tma_plain_kernel, RG, tiles, p, st, pdl, out, x, q, scale, resid, M, N, K, norm_w, eps, p.Kc,
                  p.stages);
}

tb_status_t gemv_tma_qkv(const QkvArgs& a, cudaStream_t st, bool pdl) {
  const int RG = rg_of(a.M);
  TmaPlan p;
  if (!tma_plan(RG, a.d, &p)) return TB_ERROR_NOT_SUPPORTED;
  const int64_t tiles = (int64_t)(a.H + 2 * a.Hkv) * (a.D / 8);
  TB_TMA_DISPATCH(gemv_tma_qkv_kernel, RG, tiles, p, st, pdl, a, p.Kc, p.stages);
}

tb_status_t gemv_tma_gateup(const GateUpArgs& a, cudaStream_t st, bool pdl) {
  const int RG = rg_of(a.M);
  TmaPlan p;
  if (!tma_plan(RG, a.d, &p)) return TB_ERROR_NOT_SUPPORTED;
  const int64_t tiles = (a.F + 3) / 4;
  TB_TMA_DISPATCH(gemv_tma_gateup_kernel, RG, tiles, p, st, pdl, a, p.Kc, p.stages);
}

int* wait_timeout_word() {
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, g_wait_timeouts) != cudaSuccess) return nullptr;
  return static_cast<int*>(p);
}

int take_wait_timeouts() {
  int v = 0, zero = 0;
  if (cudaMemcpyFromSymbol(&v, g_wait_timeouts, sizeof(int)) != cudaSuccess) return -1;
  if (v) cudaMemcpyToSymbol(g_wait_timeouts, &zero, sizeof(int));
  return v;
}

GemvKind gemv_kind() {
  static const GemvKind k = [] {
    const char* e = getenv("TENDO_B200_GEMV");
    if (e && strcmp(e, "simt") == 0) return GemvKind::kSimt;
    if (e && strcmp(e, "mma") == 0) return GemvKind::kMma;
    return GemvKind::kTma;
  }();
  return k;
}

}  // namespace tb
