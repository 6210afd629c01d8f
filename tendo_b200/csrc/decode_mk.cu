// decode_mk.cu — the whole batch-1 decode step as one persistent kernel.
//
// One CTA per SM (cooperative launch: all co-resident), 8 consumer warps and
// one producer warp.  The producer walks the step's weight tiles in order —
// per layer the Q/K/V, O, gate/up and down projections, then the fp32
// lm_head — and streams them through a ring of kMkStages shared-memory
// stages with cp.async.bulk (mbarrier completion).  Weights never depend on
// activations, so the stream never waits for a phase to finish: while the
// consumers run attention or sit in a grid barrier, the next projection's
// tiles are already landing.  The consumers run the phases in order,
// separated by a grid barrier:
//   embed | per layer: RMSNorm + QKV + RoPE + KV append | split-K attention |
//   combine + O + residual | RMSNorm + gate/up + SwiGLU | down + residual |
//   final RMSNorm + lm_head + argmax | token, position, history update.
// Int8 projections use the integer tensor cores: the raw weight bytes are
// the B operand, the activation row is three int8 digit rows
// (x / s = d0 + d1 / 128 + d2 / 128^2), accumulation is exact in s32.  A
// projection phase keeps every tile's per-warp partial sums in shared memory
// and runs all of its epilogues after one barrier at the end, so the tile
// loop itself never synchronises the warps.
// Every wait (mbarrier or grid barrier) is bounded and counts a timeout in
// an error word instead of hanging.
#include <math.h>

#include "common.cuh"
#include "kernels.h"
#include "tma_common.cuh"

namespace tb {
namespace {

constexpr int kMkWarps = 8;  // consumer warps
constexpr int kMkConsumers = kMkWarps * 32;
constexpr int kMkThreads = kMkConsumers + 32;  // + producer warp
constexpr int kMkStages = 5;
constexpr int kMkChunkMax = 4096;
constexpr int kMkStageBytes = 8 * (kMkChunkMax + 64);
constexpr int kMkXRegs = 12;  // float4 of x per consumer thread: K <= 12288
constexpr int kMkPart = kMkWarps * 24;  // ints of partial sums per tile
constexpr int kMkMaxSplit = 8;          // attention splits per kv head

struct MkLayout {
  size_t stage_off, dig_off, xbuf_off, red_off, bar_off, total;
  int RSX;
  // xbuf (fp32 activations, O input and lm_head input) and the per-tile
  // partial sums share a region: the O phase is done with xbuf once its
  // digits are staged, and the lm_head phase keeps no partials.
  __host__ __device__ void init(int kmax_bytes, int xbuf_floats, size_t merge_bytes, int tiles_max) {
    RSX = bank_stride(kmax_bytes);
    stage_off = 0;
    dig_off = (size_t)kMkStages * kMkStageBytes;
    size_t dig_bytes = (size_t)3 * RSX;
    if (dig_bytes < merge_bytes) dig_bytes = merge_bytes;  // the attention merge reuses this region
    xbuf_off = (dig_off + dig_bytes + 127) & ~(size_t)127;
    size_t xb = (size_t)xbuf_floats * sizeof(float);
    const size_t pb = (size_t)tiles_max * kMkPart * sizeof(int);
    if (xb < pb) xb = pb;
    red_off = (xbuf_off + xb + 15) & ~(size_t)15;
    bar_off = (red_off + 64 * sizeof(float) + 15) & ~(size_t)15;
    total = bar_off + (size_t)2 * kMkStages * sizeof(uint64_t);
  }
};

// Weight stream of one phase: p = 4 l + {0 qkv, 1 o, 2 gate/up, 3 down}; p = 4 L: lm_head.
struct Stream {
  const int8_t* base;
  const int8_t* base2;
  int row_bytes, ntiles, kind, D, rows;
};

__device__ __forceinline__ Stream stream_of(const MkArgs& a, int p) {
  Stream s{};
  const int HD = a.H * a.D, NQKV = (a.H + 2 * a.Hkv) * a.D;
  if (p == 4 * a.L) {
    s.base = reinterpret_cast<const int8_t*>(a.lm_head);
    s.row_bytes = a.d * 4;
    s.ntiles = (a.V + 7) / 8;
    s.kind = 3;
    s.rows = a.V;
    return s;
  }
  const int l = p >> 2, k = p & 3;
  if (k == 0) {
    s.base = a.wqkv + (size_t)l * NQKV * a.d;
    s.row_bytes = a.d;
    s.ntiles = (a.H + 2 * a.Hkv) * (a.D / 8);
    s.kind = 1;
    s.D = a.D;
  } else if (k == 1) {
    s.base = a.wo + (size_t)l * a.d * HD;
    s.row_bytes = HD;
    s.ntiles = a.d / 8;
    s.kind = 0;
  } else if (k == 2) {
    s.base = a.wg + (size_t)l * a.F * a.d;
    s.base2 = a.wu + (size_t)l * a.F * a.d;
    s.row_bytes = a.d;
    s.ntiles = a.F / 4;
    s.kind = 2;
  } else {
    s.base = a.wd + (size_t)l * a.d * a.F;
    s.row_bytes = a.F;
    s.ntiles = a.d / 8;
    s.kind = 0;
  }
  return s;
}

// Row of column n (0..7) of a tile: plain rows 8 t + n; QKV rotate-half pairs
// (columns n and n + 4 are rows i and i + D/2 of one head); gate rows 4 t +
// n and the same up rows; lm_head rows 8 t + n (clamped).
__device__ __forceinline__ const int8_t* row_of(const Stream& s, int tile, int n) {
  if (s.kind == 1) {
    const int per = s.D / 8, head = tile / per, i0 = (tile % per) * 4;
    const int r = head * s.D + i0 + (n & 3) + (n >> 2) * (s.D / 2);
    return s.base + (size_t)r * s.row_bytes;
  }
  if (s.kind == 2) return ((n >> 2) ? s.base2 : s.base) + (size_t)(tile * 4 + (n & 3)) * s.row_bytes;
  int r = tile * 8 + n;
  if (s.kind == 3 && r >= s.rows) r = s.rows - 1;
  return s.base + (size_t)r * s.row_bytes;
}

// Walks this CTA's weight-stream units (phase p, tile, chunk) in consumption order.
struct UnitCursor {
  Stream s;
  int p, tile, ch, Kc, nch;
  bool done;
  __device__ __forceinline__ void load(const MkArgs& a) {
    for (; p <= 4 * a.L; p++) {
      s = stream_of(a, p);
      Kc = chunk_bytes(s.row_bytes);
      nch = s.row_bytes / Kc;
      tile = blockIdx.x;
      ch = 0;
      if (tile < s.ntiles) return;
    }
    done = true;
  }
  __device__ __forceinline__ void start(const MkArgs& a) {
    p = 0;
    done = false;
    load(a);
  }
  __device__ __forceinline__ void advance(const MkArgs& a) {
    if (++ch < nch) return;
    ch = 0;
    tile += gridDim.x;
    if (tile < s.ntiles) return;
    p++;
    load(a);
  }
};

struct Pipe {
  unsigned char* stages;
  uint64_t* full;
  uint64_t* empty;
  int* err;
  int u;  // next unit
};

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Optional phase trace (CTA 0): arrival and departure time of every barrier.
struct Trace {
  uint64_t* buf;
  int n;
  __device__ __forceinline__ void stamp() {
    if (buf && blockIdx.x == 0 && threadIdx.x == 0) buf[n] = global_ns();
    n++;
  }
};

__device__ __forceinline__ void grid_sync(unsigned int* counter, unsigned int& target, int* err, Trace& tr) {
  named_sync(kMkConsumers);
  tr.stamp();
  target += gridDim.x;
  if (threadIdx.x == 0) {
    __threadfence();
    atomicAdd(counter, 1u);
    for (uint32_t it = 0;; it++) {
      unsigned int v;
      asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(counter) : "memory");
      if (v >= target) break;
      if (it > (1u << 22)) {
        atomicAdd(err, 1);
        break;
      }
      __nanosleep(32);
    }
    // no fence here: the acquire load above already orders this thread's
    // later accesses after every CTA's release, and the CTA barrier below
    // carries that order to the other threads
  }
  named_sync(kMkConsumers);
  tr.stamp();
}

// x (global, optionally RMSNorm(x) * w, or shared) -> three int8 digit rows,
// one pass: each thread keeps its NV float4s in registers between the
// reduction and the digit step (NV * 4 * 256 >= K).  Returns the row scale s
// (x = s * (d0 + d1 / 128 + d2 / 128^2)).
template <int NV>
__device__ float stage_digits_n(int8_t* dig, int RSX, const float* src, bool src_smem, int K, const float* norm_w,
                                float eps, float* red) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nv = K >> 2;
  float4 xv[NV];
#pragma unroll
  for (int i = 0; i < NV; i++) {
    const int v = threadIdx.x + i * kMkConsumers;
    xv[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (v < nv) xv[i] = src_smem ? reinterpret_cast<const float4*>(src)[v] : ldcg4(src + 4 * v);
  }
  float ss = 0.f, mx = 0.f;
#pragma unroll
  for (int i = 0; i < NV; i++) {
    const int v = threadIdx.x + i * kMkConsumers;
    const float4 t = xv[i];
    ss += t.x * t.x + t.y * t.y + t.z * t.z + t.w * t.w;
    float4 w4 = make_float4(1.f, 1.f, 1.f, 1.f);
    if (norm_w && v < nv) w4 = reinterpret_cast<const float4*>(norm_w)[v];
    mx = fmaxf(mx, fmaxf(fmaxf(fabsf(t.x * w4.x), fabsf(t.y * w4.y)), fmaxf(fabsf(t.z * w4.z), fabsf(t.w * w4.w))));
  }
  ss = warp_sum(ss);
  mx = warp_max(mx);
  if (lane == 0) {
    red[warp] = ss;
    red[kMkWarps + warp] = mx;
  }
  named_sync(kMkConsumers);
  float s = 0.f, a = 0.f;
#pragma unroll
  for (int w = 0; w < kMkWarps; w++) {
    s += red[w];
    a = fmaxf(a, red[kMkWarps + w]);
  }
  const float rms = norm_w ? __fsqrt_rn(__fadd_rn(__fdiv_rn(s, (float)K), eps)) : 1.0f;
  if (norm_w) a = a / rms * 1.0001f;
  const float sc = (a > 0.f && isfinite(a)) ? a / 127.0f : 1.0f;
  const float inv = 1.0f / sc;
#pragma unroll
  for (int i = 0; i < NV; i++) {
    const int v = threadIdx.x + i * kMkConsumers;
    if (v >= nv) continue;
    float4 t = xv[i];
    if (norm_w) {
      const float4 w4 = reinterpret_cast<const float4*>(norm_w)[v];
      t.x = __fmul_rn(__fdiv_rn(t.x, rms), w4.x);
      t.y = __fmul_rn(__fdiv_rn(t.y, rms), w4.y);
      t.z = __fmul_rn(__fdiv_rn(t.z, rms), w4.z);
      t.w = __fmul_rn(__fdiv_rn(t.w, rms), w4.w);
    }
    const float vals[4] = {t.x, t.y, t.z, t.w};
    uint32_t p0 = 0, p1 = 0, p2 = 0;
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const float uu = fminf(fmaxf(vals[j] * inv, -127.0f), 127.0f);
      const float d0 = rintf(uu);
      const float r1 = (uu - d0) * 128.0f;
      const float d1 = rintf(r1);
      const float d2 = rintf((r1 - d1) * 128.0f);
      p0 |= ((uint32_t)__float2int_rn(d0) & 0xffu) << (8 * j);
      p1 |= ((uint32_t)__float2int_rn(d1) & 0xffu) << (8 * j);
      p2 |= ((uint32_t)__float2int_rn(d2) & 0xffu) << (8 * j);
    }
    reinterpret_cast<uint32_t*>(dig)[v] = p0;
    reinterpret_cast<uint32_t*>(dig + RSX)[v] = p1;
    reinterpret_cast<uint32_t*>(dig + 2 * RSX)[v] = p2;
  }
  named_sync(kMkConsumers);
  return sc;
}

__device__ __forceinline__ float stage_digits(int8_t* dig, int RSX, const float* src, bool src_smem, int K,
                                              const float* norm_w, float eps, float* red) {
  if (K <= 4 * 4 * kMkConsumers) return stage_digits_n<4>(dig, RSX, src, src_smem, K, norm_w, eps, red);
  return stage_digits_n<kMkXRegs>(dig, RSX, src, src_smem, K, norm_w, eps, red);
}

// One int8 tile through the pipe; this warp's partial sums of digit rows 0..2
// go to part[warp * 24 + row * 8 + column] (lanes g < 3 hold row g).
__device__ __forceinline__ void int8_tile(int* part, Pipe& pp, const int8_t* dig, int RSX, int Kc, int nch) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int RS = bank_stride(Kc), kbc = Kc / 64;
  int d[4] = {0, 0, 0, 0};
  for (int ch = 0; ch < nch; ch++, pp.u++) {
    const int st = pp.u % kMkStages, use = pp.u / kMkStages;
    mbarrier_wait(&pp.full[st], (uint32_t)(use & 1), pp.err);
    const unsigned char* sp = pp.stages + (size_t)st * kMkStageBytes + (size_t)g * RS + 16 * t;
    const int8_t* xr = dig + (size_t)(g < 3 ? g : 0) * RSX + ch * Kc + 16 * t;
#pragma unroll 4
    for (int kb = warp; kb < kbc; kb += kMkWarps) {
      const uint4 wv = *reinterpret_cast<const uint4*>(sp + kb * 64);
      uint4 xa = make_uint4(0u, 0u, 0u, 0u);
      if (g < 3) xa = *reinterpret_cast<const uint4*>(xr + kb * 64);
      mma_s8_16832(d, xa.x, 0u, xa.y, 0u, wv.x, wv.y);
      mma_s8_16832(d, xa.z, 0u, xa.w, 0u, wv.z, wv.w);
    }
    mbarrier_arrive(&pp.empty[st]);
  }
  if (g < 3) {
    part[warp * 24 + g * 8 + 2 * t] = d[0];
    part[warp * 24 + g * 8 + 2 * t + 1] = d[1];
  }
}

// After the phase barrier: y of column `lane` (< 8) of tile `it`.
__device__ __forceinline__ float tile_value(const int* part_all, int it, float sc) {
  const int lane = threadIdx.x & 31;
  if (lane >= 8) return 0.f;
  const int* p = part_all + it * kMkPart;
  int s0 = 0, s1 = 0, s2 = 0;
#pragma unroll
  for (int w = 0; w < kMkWarps; w++) {
    s0 += p[w * 24 + lane];
    s1 += p[w * 24 + 8 + lane];
    s2 += p[w * 24 + 16 + lane];
  }
  return sc * ((float)s0 + (float)s1 * (1.0f / 128.0f) + (float)s2 * (1.0f / 16384.0f));
}

// L2-only load whose line is marked evict-first: the KV rows of a layer are
// read once per token.
__device__ __forceinline__ float4 ld_evict_first4(const float* p, uint64_t pol) {
  float4 v;
  asm volatile("ld.global.cg.L2::cache_hint.v4.f32 {%0, %1, %2, %3}, [%4], %5;"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "l"(p), "l"(pol));
  return v;
}

template <int VEC, int G>
__device__ void attention_unit(const MkArgs& a, int l, int unit, int64_t sk, float* merge) {
  constexpr int D = VEC * 32, U = 8;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kvh = unit / a.nsplit, split = unit % a.nsplit;
  int64_t chunk = (sk + a.nsplit - 1) / a.nsplit;
  chunk = (chunk + U - 1) / U * U;
  const int64_t start = (int64_t)split * chunk, end = min(start + chunk, sk);
  const float* kb = a.kc + (((size_t)l * a.Hkv + kvh) * a.max_seq) * D;
  const float* vb = a.vc + (((size_t)l * a.Hkv + kvh) * a.max_seq) * D;
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  float qr[G][VEC];
#pragma unroll
  for (int gi = 0; gi < G; gi++)
#pragma unroll
    for (int e = 0; e < VEC; e++) qr[gi][e] = ldcg(a.q + (size_t)(kvh * G + gi) * D + lane * VEC + e);
  float mx[G], lsum[G], o[G][VEC];
#pragma unroll
  for (int gi = 0; gi < G; gi++) {
    mx[gi] = -INFINITY;
    lsum[gi] = 0.f;
#pragma unroll
    for (int e = 0; e < VEC; e++) o[gi][e] = 0.f;
  }
  for (int64_t j0 = start + (int64_t)warp * U; j0 < end; j0 += (int64_t)kMkWarps * U) {
    float kr[U][VEC], vr[U][VEC];
#pragma unroll
    for (int u = 0; u < U; u++) {
      const int64_t j = j0 + u;
#pragma unroll
      for (int e = 0; e < VEC; e++) kr[u][e] = vr[u][e] = 0.f;
      if (j < end) {
        if constexpr (VEC == 4) {
          const float4 k4 = ld_evict_first4(kb + j * D + lane * 4, pol), v4 = ld_evict_first4(vb + j * D + lane * 4, pol);
          kr[u][0] = k4.x; kr[u][1] = k4.y; kr[u][2] = k4.z; kr[u][3] = k4.w;
          vr[u][0] = v4.x; vr[u][1] = v4.y; vr[u][2] = v4.z; vr[u][3] = v4.w;
        } else {
#pragma unroll
          for (int e = 0; e < VEC; e++) {
            kr[u][e] = ldcg(kb + j * D + lane * VEC + e);
            vr[u][e] = ldcg(vb + j * D + lane * VEC + e);
          }
        }
      }
    }
#pragma unroll
    for (int gi = 0; gi < G; gi++) {
      float s[U];
#pragma unroll
      for (int u = 0; u < U; u++) {
        float dd = 0.f;
#pragma unroll
        for (int e = 0; e < VEC; e++) dd = fmaf(qr[gi][e], kr[u][e], dd);
        s[u] = dd;
      }
#pragma unroll
      for (int o2 = 16; o2 > 0; o2 >>= 1)
#pragma unroll
        for (int u = 0; u < U; u++) s[u] += __shfl_xor_sync(0xffffffffu, s[u], o2);
      float tmax = -INFINITY;
#pragma unroll
      for (int u = 0; u < U; u++) {
        s[u] = (j0 + u < end) ? s[u] * a.attn_scale : -INFINITY;
        tmax = fmaxf(tmax, s[u]);
      }
      const float mn = fmaxf(mx[gi], tmax);
      const float corr = expf(mx[gi] - mn);
      float psum = 0.f;
#pragma unroll
      for (int e = 0; e < VEC; e++) o[gi][e] *= corr;
#pragma unroll
      for (int u = 0; u < U; u++) {
        const float p = expf(s[u] - mn);
        psum += p;
#pragma unroll
        for (int e = 0; e < VEC; e++) o[gi][e] = fmaf(p, vr[u][e], o[gi][e]);
      }
      lsum[gi] = lsum[gi] * corr + psum;
      mx[gi] = mn;
    }
  }
  // merge the warps: merge[warp][gi][D + 2]
#pragma unroll
  for (int gi = 0; gi < G; gi++) {
    float* mw = merge + ((size_t)warp * G + gi) * (D + 2);
#pragma unroll
    for (int e = 0; e < VEC; e++) mw[lane * VEC + e] = o[gi][e];
    if (lane == 0) {
      mw[D] = mx[gi];
      mw[D + 1] = lsum[gi];
    }
  }
  named_sync(kMkConsumers);
  for (int idx = threadIdx.x; idx < G * D; idx += kMkConsumers) {
    const int gi = idx / D, e = idx - gi * D;
    float m = -INFINITY;
#pragma unroll
    for (int w = 0; w < kMkWarps; w++) m = fmaxf(m, merge[((size_t)w * G + gi) * (D + 2) + D]);
    float L = 0.f, O = 0.f;
    if (m != -INFINITY) {
#pragma unroll
      for (int w = 0; w < kMkWarps; w++) {
        const float* mw = merge + ((size_t)w * G + gi) * (D + 2);
        const float c = expf(mw[D] - m);
        L = fmaf(mw[D + 1], c, L);
        O = fmaf(mw[e], c, O);
      }
    }
    float* part = a.partial + ((size_t)(kvh * G + gi) * a.nsplit + split) * (D + 4);
    part[e] = O;
    if (e == 0) {
      part[D] = m;
      part[D + 1] = L;
    }
  }
  // the last split of this kv head to finish combines all its splits
  __threadfence();
  named_sync(kMkConsumers);
  int* flag = reinterpret_cast<int*>(merge);
  if (threadIdx.x == 0) {
    const unsigned int ticket = atomicAdd(a.head_done + kvh, 1u);
    flag[0] = ticket == (unsigned int)(a.nsplit - 1);
  }
  named_sync(kMkConsumers);
  const bool last = flag[0] != 0;
  named_sync(kMkConsumers);
  if (last) {
    __threadfence();
    for (int idx = threadIdx.x; idx < G * D; idx += kMkConsumers) {
      const int gi = idx / D, e = idx - gi * D;
      const float* p = a.partial + (size_t)(kvh * G + gi) * a.nsplit * (D + 4);
      float ms[kMkMaxSplit], ls[kMkMaxSplit], os[kMkMaxSplit];
#pragma unroll
      for (int s = 0; s < kMkMaxSplit; s++) {
        ms[s] = -INFINITY;
        ls[s] = os[s] = 0.f;
        if (s < a.nsplit) {
          ms[s] = ldcg(p + (size_t)s * (D + 4) + D);
          ls[s] = ldcg(p + (size_t)s * (D + 4) + D + 1);
          os[s] = ldcg(p + (size_t)s * (D + 4) + e);
        }
      }
      float m = -INFINITY;
#pragma unroll
      for (int s = 0; s < kMkMaxSplit; s++) m = fmaxf(m, ms[s]);
      float L = 0.f, O = 0.f;
#pragma unroll
      for (int s = 0; s < kMkMaxSplit; s++) {
        const float c = ms[s] == -INFINITY ? 0.f : expf(ms[s] - m);
        L = fmaf(ls[s], c, L);
        O = fmaf(os[s], c, O);
      }
      a.attn[(size_t)(kvh * G + gi) * D + e] = O / L;
    }
    if (threadIdx.x == 0) a.head_done[kvh] = 0u;  // ready for the next step
  }
  named_sync(kMkConsumers);  // merge is reused by the next unit
}

__device__ __forceinline__ unsigned long long greedy_key(float v, int idx) {
  uint32_t b = __float_as_uint(v);
  b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return ((unsigned long long)b << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)idx);
}

__global__ void __launch_bounds__(kMkThreads, 1) decode_megakernel(MkArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  MkLayout Ly;
  Ly.init(a.kmax_bytes, a.xbuf_floats, a.merge_bytes, a.tiles_max);
  unsigned char* stages = smem + Ly.stage_off;
  int8_t* dig = reinterpret_cast<int8_t*>(smem + Ly.dig_off);
  float* merge = reinterpret_cast<float*>(smem + Ly.dig_off);
  float* xbuf = reinterpret_cast<float*>(smem + Ly.xbuf_off);
  int* part = reinterpret_cast<int*>(smem + Ly.xbuf_off);  // shares the region with xbuf
  float* redf = reinterpret_cast<float*>(smem + Ly.red_off);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + Ly.bar_off);
  uint64_t* empty = full + kMkStages;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kMkStages; s++) {
      mbarrier_init(&full[s], 1);
      mbarrier_init(&empty[s], kMkConsumers);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();

  if (warp == kMkWarps) {
    // producer: the step's weight tiles in consumption order
    if (lane == 0) {
      // weights are read once per token: evict them first, so the activations,
      // norm weights, channel scales and KV rows the consumers touch stay in L2
      uint64_t policy;
      asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
      UnitCursor c;
      c.start(a);
      for (int u = 0; !c.done; u++) {
        const int st = u % kMkStages, use = u / kMkStages;
        if (use > 0) mbarrier_wait(&empty[st], (uint32_t)((use - 1) & 1), a.err);
        unsigned char* dst = stages + (size_t)st * kMkStageBytes;
        const int RS = bank_stride(c.Kc);
        mbarrier_expect_tx(&full[st], (uint32_t)(8 * c.Kc));
#pragma unroll
        for (int n = 0; n < 8; n++)
          bulk_copy_g2s_hint(dst + (size_t)n * RS, row_of(c.s, c.tile, n) + (size_t)c.ch * c.Kc, (uint32_t)c.Kc,
                             &full[st], policy);
        c.advance(a);
      }
      // every copy lands before the consumers release its stage, so the CTA
      // never exits with a copy in flight
    }
    return;
  }
  // consumers
  unsigned int target = 0;
  Trace tr{a.trace, 0};
  tr.stamp();
  Pipe pp{stages, full, empty, a.err, 0};
  const int64_t pos = *a.pos;
  const int64_t sk = pos + 1;
  const int64_t token = __ldcg(a.tokens);
  const int half = a.D / 2;
  const int HD = a.H * a.D;
  // embedding (cpu/backend.go:1289-1339): h = embed[token]
  for (int i = blockIdx.x * kMkConsumers + threadIdx.x; i < a.d; i += gridDim.x * kMkConsumers)
    a.h[i] = a.embed[(size_t)token * a.d + i];
  grid_sync(a.bar_counter, target, a.err, tr);

  for (int l = 0; l < a.L; l++) {
    // ---- RMSNorm + Q/K/V + RoPE + KV append ----
    {
      const Stream s = stream_of(a, 4 * l + 0);
      const int Kc = chunk_bytes(s.row_bytes), nch = s.row_bytes / Kc;
      const float sc = stage_digits(dig, Ly.RSX, a.h, false, a.d, a.attn_norm + (size_t)l * a.d, a.eps, redf);
      tr.stamp();
      int nt = 0;
      for (int tile = blockIdx.x; tile < s.ntiles; tile += gridDim.x, nt++)
        int8_tile(part + nt * kMkPart, pp, dig, Ly.RSX, Kc, nch);
      named_sync(kMkConsumers);
      tr.stamp();
      const float* sqkv = a.sqkv + (size_t)l * (a.H + 2 * a.Hkv) * a.D;
      float* kcl = a.kc + (size_t)l * a.Hkv * a.max_seq * a.D;
      float* vcl = a.vc + (size_t)l * a.Hkv * a.max_seq * a.D;
      for (int it = warp; it < nt; it += kMkWarps) {
        const int tile = blockIdx.x + it * gridDim.x;
        const int per = a.D / 8, head = tile / per, i = (tile % per) * 4 + (lane & 3);
        const int r = head * a.D + i + ((lane >> 2) & 1) * half;
        const float y = tile_value(part, it, sc);
        const float v = lane < 8 ? y * sqkv[r] : 0.f;
        const float partner = __shfl_xor_sync(0xffffffffu, v, 4);
        if (lane < 4) {
          if (head < a.H + a.Hkv) {
            const float c = a.cos_t[pos * half + i], sn = a.sin_t[pos * half + i];
            const float o0 = __fsub_rn(__fmul_rn(v, c), __fmul_rn(partner, sn));
            const float o1 = __fadd_rn(__fmul_rn(v, sn), __fmul_rn(partner, c));
            float* o = head < a.H ? a.q + (size_t)head * a.D : kcl + ((size_t)(head - a.H) * a.max_seq + pos) * a.D;
            o[i] = o0;
            o[i + half] = o1;
          } else {
            float* o = vcl + ((size_t)(head - a.H - a.Hkv) * a.max_seq + pos) * a.D;
            o[i] = v;
            o[i + half] = partner;
          }
        }
      }
    }
    grid_sync(a.bar_counter, target, a.err, tr);
    // ---- split-K attention over the cache ----
    {
      const int units = a.Hkv * a.nsplit;
      const int G = a.H / a.Hkv;
      for (int unit = blockIdx.x; unit < units; unit += gridDim.x) {
        if (a.D == 128) {
          if (G == 1) attention_unit<4, 1>(a, l, unit, sk, merge);
          else if (G == 2) attention_unit<4, 2>(a, l, unit, sk, merge);
          else if (G == 4) attention_unit<4, 4>(a, l, unit, sk, merge);
          else attention_unit<4, 8>(a, l, unit, sk, merge);
        } else {
          if (G == 1) attention_unit<2, 1>(a, l, unit, sk, merge);
          else if (G == 2) attention_unit<2, 2>(a, l, unit, sk, merge);
          else if (G == 4) attention_unit<2, 4>(a, l, unit, sk, merge);
          else attention_unit<2, 8>(a, l, unit, sk, merge);
        }
      }
    }
    grid_sync(a.bar_counter, target, a.err, tr);
    // ---- O projection + residual (the attention phase left the combined heads in a.attn) ----
    {
      tr.stamp();
      const Stream s = stream_of(a, 4 * l + 1);
      const int Kc = chunk_bytes(s.row_bytes), nch = s.row_bytes / Kc;
      const float sc = stage_digits(dig, Ly.RSX, a.attn, false, HD, nullptr, 0.f, redf);
      tr.stamp();
      int nt = 0;
      for (int tile = blockIdx.x; tile < s.ntiles; tile += gridDim.x, nt++)
        int8_tile(part + nt * kMkPart, pp, dig, Ly.RSX, Kc, nch);
      named_sync(kMkConsumers);
      tr.stamp();
      const float* so = a.so + (size_t)l * a.d;
      for (int it = warp; it < nt; it += kMkWarps) {
        const int r = (blockIdx.x + it * gridDim.x) * 8 + lane;
        const float y = tile_value(part, it, sc);
        if (lane < 8) a.h[r] = ldcg(a.h + r) + y * so[r];
      }
    }
    grid_sync(a.bar_counter, target, a.err, tr);
    // ---- RMSNorm + gate/up + SwiGLU ----
    {
      const Stream s = stream_of(a, 4 * l + 2);
      const int Kc = chunk_bytes(s.row_bytes), nch = s.row_bytes / Kc;
      const float sc = stage_digits(dig, Ly.RSX, a.h, false, a.d, a.mlp_norm + (size_t)l * a.d, a.eps, redf);
      tr.stamp();
      int nt = 0;
      for (int tile = blockIdx.x; tile < s.ntiles; tile += gridDim.x, nt++)
        int8_tile(part + nt * kMkPart, pp, dig, Ly.RSX, Kc, nch);
      named_sync(kMkConsumers);
      tr.stamp();
      const float* sg = a.sg + (size_t)l * a.F;
      const float* su = a.su + (size_t)l * a.F;
      for (int it = warp; it < nt; it += kMkWarps) {
        const int j = (blockIdx.x + it * gridDim.x) * 4 + (lane & 3);
        const float y = tile_value(part, it, sc);
        const float v = lane < 8 ? y * ((lane >> 2) ? su[j] : sg[j]) : 0.f;
        const float partner = __shfl_xor_sync(0xffffffffu, v, 4);
        if (lane < 4) {
          const float sig = 1.0f / (1.0f + expf(-v));
          a.act[j] = (v * sig) * partner;
        }
      }
    }
    grid_sync(a.bar_counter, target, a.err, tr);
    // ---- down projection + residual ----
    {
      const Stream s = stream_of(a, 4 * l + 3);
      const int Kc = chunk_bytes(s.row_bytes), nch = s.row_bytes / Kc;
      const float sc = stage_digits(dig, Ly.RSX, a.act, false, a.F, nullptr, 0.f, redf);
      tr.stamp();
      int nt = 0;
      for (int tile = blockIdx.x; tile < s.ntiles; tile += gridDim.x, nt++)
        int8_tile(part + nt * kMkPart, pp, dig, Ly.RSX, Kc, nch);
      named_sync(kMkConsumers);
      tr.stamp();
      const float* sd = a.sd + (size_t)l * a.d;
      for (int it = warp; it < nt; it += kMkWarps) {
        const int r = (blockIdx.x + it * gridDim.x) * 8 + lane;
        const float y = tile_value(part, it, sc);
        if (lane < 8) a.h[r] = ldcg(a.h + r) + y * sd[r];
      }
    }
    grid_sync(a.bar_counter, target, a.err, tr);
  }

  // ---- final RMSNorm + fp32 lm_head + greedy argmax ----
  {
    // xbuf = RMSNorm(h) * final_norm in fp32 (quantized.go:154-172)
    float ss = 0.f;
    for (int v = threadIdx.x; v < a.d / 4; v += kMkConsumers) {
      const float4 t = ldcg4(a.h + 4 * v);
      ss += t.x * t.x + t.y * t.y + t.z * t.z + t.w * t.w;
    }
    ss = warp_sum(ss);
    if (lane == 0) redf[warp] = ss;
    named_sync(kMkConsumers);
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < kMkWarps; w++) tot += redf[w];
    const float rms = __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)a.d), a.eps));
    for (int i = threadIdx.x; i < a.d; i += kMkConsumers)
      xbuf[i] = __fmul_rn(__fdiv_rn(ldcg(a.h + i), rms), a.final_norm[i]);
    named_sync(kMkConsumers);
    tr.stamp();
    const Stream s = stream_of(a, 4 * a.L);
    const int Kc = chunk_bytes(s.row_bytes), nch = s.row_bytes / Kc, RS = bank_stride(Kc);
    const int fpc = Kc / 4;  // floats per chunk
    unsigned long long best = 0ull;
    for (int tile = blockIdx.x; tile < s.ntiles; tile += gridDim.x) {
      float acc = 0.f;
      for (int ch = 0; ch < nch; ch++, pp.u++) {
        const int st = pp.u % kMkStages, use = pp.u / kMkStages;
        mbarrier_wait(&full[st], (uint32_t)(use & 1), a.err);
        const float* wr = reinterpret_cast<const float*>(stages + (size_t)st * kMkStageBytes + (size_t)warp * RS);
        const float* xr = xbuf + ch * fpc;
        for (int v = lane; v < fpc / 4; v += 32) {
          const float4 w4 = reinterpret_cast<const float4*>(wr)[v];
          const float4 x4 = reinterpret_cast<const float4*>(xr)[v];
          acc = fmaf(x4.x, w4.x, acc);
          acc = fmaf(x4.y, w4.y, acc);
          acc = fmaf(x4.z, w4.z, acc);
          acc = fmaf(x4.w, w4.w, acc);
        }
        mbarrier_arrive(&empty[st]);
      }
      acc = warp_sum(acc);
      const int r = tile * 8 + warp;
      if (r < a.V) {
        if (lane == 0) a.logits[r] = acc;
        const unsigned long long k = greedy_key(acc, r);
        best = k > best ? k : best;
      }
    }
    if (lane == 0 && best) atomicMax(a.keys, best);
  }
  grid_sync(a.bar_counter, target, a.err, tr);
  // ---- token, history and position (models/sampling.go:73-83) ----
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    const unsigned long long k = atomicAdd(a.keys, 0ull);
    const int64_t tok = (int64_t)(0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull));
    *a.tokens = tok;
    const int64_t st = *a.step;
    if (st < a.hist_cap) a.history[st] = tok;
    *a.step = st + 1;
    *a.pos = pos + 1;
    *a.keys = 0ull;
  }
}

int max_tiles_per_cta(const MkArgs& a, int grid) {
  int t = (a.H + 2 * a.Hkv) * (a.D / 8);
  if (a.d / 8 > t) t = a.d / 8;
  if (a.F / 4 > t) t = a.F / 4;
  return (t + grid - 1) / grid;
}

void fill_sizes(MkArgs& a, int grid) {
  int kmax = a.d > a.H * a.D ? a.d : a.H * a.D;
  if (a.F > kmax) kmax = a.F;
  a.kmax_bytes = kmax;
  a.xbuf_floats = a.H * a.D > a.d ? a.H * a.D : a.d;
  a.merge_bytes = (size_t)kMkWarps * (a.H / a.Hkv) * (a.D + 2) * sizeof(float);
  a.tiles_max = max_tiles_per_cta(a, grid);
}

}  // namespace

size_t megakernel_partial_bytes(int H, int D, int nsplit) { return (size_t)H * nsplit * (D + 4) * sizeof(float); }

bool megakernel_supported(int d, int H, int Hkv, int D, int F, int V, int batch) {
  if (batch != 1) return false;
  if (d % 64 || (H * D) % 64 || F % 64 || (4 * d) % 64) return false;
  if (d % 8 || F % 4 || D % 8 || (D != 64 && D != 128)) return false;
  const int G = H / Hkv;
  if (H % Hkv || (G != 1 && G != 2 && G != 4 && G != 8)) return false;
  int kmax = d > H * D ? d : H * D;
  if (F > kmax) kmax = F;
  if (kmax > 4 * kMkConsumers * kMkXRegs) return false;  // digits staged from registers
  MkArgs a{};
  a.d = d;
  a.H = H;
  a.Hkv = Hkv;
  a.D = D;
  a.F = F;
  a.V = V;
  fill_sizes(a, sm_count());
  MkLayout Ly;
  Ly.init(a.kmax_bytes, a.xbuf_floats, a.merge_bytes, a.tiles_max);
  return Ly.total <= 227 * 1024;
}

tb_status_t megakernel_launch(MkArgs a, cudaStream_t st) {
  const int grid = sm_count();
  fill_sizes(a, grid);
  MkLayout Ly;
  Ly.init(a.kmax_bytes, a.xbuf_floats, a.merge_bytes, a.tiles_max);
  const size_t smem = Ly.total;
  cudaError_t e = cudaFuncSetAttribute(decode_megakernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(decode_megakernel)");
  e = cudaMemsetAsync(a.bar_counter, 0, sizeof(unsigned int), st);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(barrier)");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kMkThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, decode_megakernel, a);
  if (e != cudaSuccess) return cuda_fail(e, "cudaLaunchKernelEx(decode_megakernel)");
  return TB_SUCCESS;
}

}  // namespace tb
