// decode_mk.cu — the whole batch-1 decode step as one persistent kernel.
//
// One CTA per SM (cooperative launch: all co-resident), 8 consumer warps and
// one producer warp.  The producer walks the step's input stream in the order
// the consumers use it — per layer the Q/K/V weight tiles, this CTA's slice
// of the KV cache, the O, gate/up and down weight tiles, then the fp32
// lm_head — and moves it through a ring of kMkStages shared-memory stages
// with cp.async.bulk (mbarrier completion).  None of it depends on this
// step's activations (the cache rows it streams were written by earlier
// steps), so the stream never waits for a phase to finish.
//
// Phases hand their results to the next phase through tagged exchange words:
// a 64-bit store of (fp32 value, epoch tag of the writing phase).  A reader
// polls the words it needs until every tag matches, so one L2 round trip both
// synchronises and moves the data — there is no grid barrier between phases,
// only one at the end of the step for the greedy token.  Per layer:
//   RMSNorm + QKV + RoPE (q, new k/v tagged; k/v also appended to the cache) |
//   split-K attention over the streamed cache rows, split 0 of each kv head
//   combining the others' tagged partials | O + residual | RMSNorm + gate/up
//   + SwiGLU | down + residual;
// then final RMSNorm + lm_head + greedy argmax | token, position, history.
// Each CTA keeps the residual rows its O and down tiles own in shared memory,
// and fetches each phase's channel scales with cp.async during the tile loop.
// Int8 projections use the integer tensor cores: the raw weight bytes are the
// B operand, the activation row is three int8 digit rows
// (x / s = d0 + d1 / 128 + d2 / 128^2), accumulation is exact in s32.
// Every wait (mbarrier, tagged word, barrier) is bounded and counts a timeout
// in an error word instead of hanging.
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
constexpr int kMkKvBytes = 16384;  // K (or V) bytes of one cache unit: 32 rows of D 128, 64 of D 64
constexpr int kMkXRegs = 12;       // float4 of x per consumer thread: K <= 12288
constexpr int kMkPart = kMkWarps * 24;  // ints of partial sums per tile
constexpr int kMkMaxSplit = 8;          // attention splits per kv head
constexpr int kMkTagKinds = 8;          // tags per layer
constexpr uint32_t kMkSpin = 1u << 18;  // polls of a tagged word before it counts as a timeout

// tag kinds of a layer's exchange words
constexpr int kTagQkv = 0, kTagPart = 1, kTagAttn = 2, kTagH1 = 3, kTagAct = 4, kTagH2 = 5;

__device__ __forceinline__ uint32_t tag_of(uint32_t e, int L, int l, int k) {
  return e * (uint32_t)(kMkTagKinds * (L + 1)) + (uint32_t)(kMkTagKinds * l + k);
}

// Offsets (in words) of the exchange buffers inside MkArgs::ll.
struct LLOff {
  size_t q, kv, part, attn, h, act, total;
  __host__ __device__ void init(int d, int H, int Hkv, int D, int F, int nsplit) {
    q = 0;
    kv = q + (size_t)H * D;
    part = kv + (size_t)2 * Hkv * D;
    attn = part + (size_t)H * nsplit * (D + 2);
    h = attn + (size_t)H * D;
    act = h + (size_t)d;
    total = act + (size_t)F;
  }
};

__device__ __forceinline__ void ll_store(unsigned long long* p, float v, uint32_t tag) {
  const unsigned long long w = ((unsigned long long)tag << 32) | (unsigned long long)__float_as_uint(v);
  asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ unsigned long long ll_load(const unsigned long long* p) {
  unsigned long long w;
  asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
  return w;
}
// Two consecutive words (16-byte aligned); each 8-byte word is read atomically.
__device__ __forceinline__ ulonglong2 ll_load2(const unsigned long long* p) {
  ulonglong2 w;
  asm volatile("ld.relaxed.gpu.global.v2.b64 {%0, %1}, [%2];" : "=l"(w.x), "=l"(w.y) : "l"(p) : "memory");
  return w;
}
// A poll loop gives up after kMkSpin polls, or at once when another wait of
// the launch has already timed out: a broken exchange ends the step within a
// fraction of a second instead of a wait per word.  The caller counts it.
__device__ __forceinline__ bool spin_expired(uint32_t it, const int* err) {
  if (it >= kMkSpin) return true;
  return (it & 255u) == 255u && *reinterpret_cast<const volatile int*>(err) != 0;
}
__device__ __forceinline__ uint32_t ll_tag(unsigned long long w) { return (uint32_t)(w >> 32); }
__device__ __forceinline__ float ll_val(unsigned long long w) { return __uint_as_float((uint32_t)w); }

__device__ __forceinline__ void cp_async16(void* smem_dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(smem_dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

struct MkLayout {
  size_t stage_off, dig_off, xbuf_off, ssc_off, res_off, rope_off, red_off, bar_off, total;
  int RSX;
  // xbuf (the lm_head's fp32 input) and the per-tile partial sums share a
  // region: the lm_head phase keeps no partials.  The digit rows and the
  // attention's warp merge share another.
  __host__ __device__ void init(int kmax_bytes, int xbuf_floats, size_t merge_bytes, int tiles_max, int tiles_res,
                                int D) {
    RSX = bank_stride(kmax_bytes);
    stage_off = 0;
    dig_off = (size_t)kMkStages * kMkStageBytes;
    size_t dig_bytes = (size_t)3 * RSX;
    if (dig_bytes < merge_bytes) dig_bytes = merge_bytes;
    xbuf_off = (dig_off + dig_bytes + 127) & ~(size_t)127;
    size_t xb = (size_t)xbuf_floats * sizeof(float);
    const size_t pb = (size_t)tiles_max * kMkPart * sizeof(int);
    if (xb < pb) xb = pb;
    ssc_off = (xbuf_off + xb + 15) & ~(size_t)15;
    res_off = ssc_off + (size_t)tiles_max * 8 * sizeof(float);
    rope_off = (res_off + (size_t)tiles_res * 8 * sizeof(float) + 15) & ~(size_t)15;
    red_off = (rope_off + (size_t)D * sizeof(float) + 15) & ~(size_t)15;
    bar_off = (red_off + 64 * sizeof(float) + 15) & ~(size_t)15;
    total = bar_off + (size_t)2 * kMkStages * sizeof(uint64_t);
  }
};

// This CTA's attention split: kv head kvh, cache rows [j0, j1) of the rows
// before the step's position, in nunits units of kMkKvBytes / (4 D) rows.
struct AttnSplit {
  int kvh, split, nunits;
  int64_t j0, j1;
};

__device__ __forceinline__ AttnSplit attn_split_of(const MkArgs& a, int64_t pos) {
  AttnSplit s{};
  s.kvh = -1;
  const int b = blockIdx.x;
  if (b >= a.Hkv * a.nsplit) return s;
  s.kvh = b / a.nsplit;
  s.split = b % a.nsplit;
  const int pu = kMkKvBytes / (a.D * 4);
  int64_t chunk = (pos + a.nsplit - 1) / a.nsplit;
  chunk = (chunk + pu - 1) / pu * pu;
  s.j0 = (int64_t)s.split * chunk;
  s.j1 = s.j0 + chunk < pos ? s.j0 + chunk : pos;
  s.nunits = s.j1 > s.j0 ? (int)((s.j1 - s.j0 + pu - 1) / pu) : 0;
  return s;
}

// Input stream of one phase: p = 5 l + {0 qkv, 1 cache slice, 2 o, 3 gate/up, 4 down}; p = 5 L: lm_head.
struct Stream {
  const int8_t* base;
  const int8_t* base2;
  int row_bytes, ntiles, kind, D, rows, layer;
};
constexpr int kKindPlain = 0, kKindQkv = 1, kKindGateUp = 2, kKindLmHead = 3, kKindKv = 4;

__device__ __forceinline__ Stream stream_of(const MkArgs& a, int p, const AttnSplit& at) {
  Stream s{};
  const int HD = a.H * a.D, NQKV = (a.H + 2 * a.Hkv) * a.D;
  if (p == 5 * a.L) {
    s.base = reinterpret_cast<const int8_t*>(a.lm_head);
    s.row_bytes = a.d * 4;
    s.ntiles = (a.V + 7) / 8;
    s.kind = kKindLmHead;
    s.rows = a.V;
    return s;
  }
  const int l = p / 5, k = p - 5 * l;
  s.layer = l;
  if (k == 0) {
    s.base = a.wqkv + (size_t)l * NQKV * a.d;
    s.row_bytes = a.d;
    s.ntiles = (a.H + 2 * a.Hkv) * (a.D / 8);
    s.kind = kKindQkv;
    s.D = a.D;
  } else if (k == 1) {
    s.ntiles = at.nunits;
    s.kind = kKindKv;
    s.D = a.D;
  } else if (k == 2) {
    s.base = a.wo + (size_t)l * a.d * HD;
    s.row_bytes = HD;
    s.ntiles = a.d / 8;
    s.kind = kKindPlain;
  } else if (k == 3) {
    s.base = a.wg + (size_t)l * 2 * a.F * a.d;  // a layer's gate rows, then its up rows
    s.base2 = a.wu + (size_t)l * 2 * a.F * a.d;
    s.row_bytes = a.d;
    s.ntiles = a.F / 4;
    s.kind = kKindGateUp;
  } else {
    s.base = a.wd + (size_t)l * a.d * a.F;
    s.row_bytes = a.F;
    s.ntiles = a.d / 8;
    s.kind = kKindPlain;
  }
  return s;
}

// Row of column n (0..7) of a weight tile: plain rows 8 t + n; QKV rotate-half
// pairs (columns n and n + 4 are rows i and i + D/2 of one head); gate rows
// 4 t + n and the same up rows; lm_head rows 8 t + n (clamped).
__device__ __forceinline__ const int8_t* row_of(const Stream& s, int tile, int n) {
  if (s.kind == kKindQkv) {
    const int per = s.D / 8, head = tile / per, i0 = (tile % per) * 4;
    const int r = head * s.D + i0 + (n & 3) + (n >> 2) * (s.D / 2);
    return s.base + (size_t)r * s.row_bytes;
  }
  if (s.kind == kKindGateUp) return ((n >> 2) ? s.base2 : s.base) + (size_t)(tile * 4 + (n & 3)) * s.row_bytes;
  int r = tile * 8 + n;
  if (s.kind == kKindLmHead && r >= s.rows) r = s.rows - 1;
  return s.base + (size_t)r * s.row_bytes;
}

// Walks this CTA's stream units (phase p, tile, chunk) in consumption order.
// Weight phases visit tiles blockIdx.x, + gridDim.x, ...; the cache slice
// visits its units 0, 1, ...
struct UnitCursor {
  Stream s;
  int p, tile, ch, Kc, nch;
  bool done;
  __device__ __forceinline__ void load(const MkArgs& a, const AttnSplit& at) {
    for (; p <= 5 * a.L; p++) {
      s = stream_of(a, p, at);
      if (s.kind == kKindKv) {
        Kc = 0;
        nch = 1;
        tile = 0;
      } else {
        Kc = chunk_bytes(s.row_bytes);
        nch = s.row_bytes / Kc;
        tile = blockIdx.x;
      }
      ch = 0;
      if (tile < s.ntiles) return;
    }
    done = true;
  }
  __device__ __forceinline__ void start(const MkArgs& a, const AttnSplit& at) {
    p = 0;
    done = false;
    load(a, at);
  }
  __device__ __forceinline__ void advance(const MkArgs& a, const AttnSplit& at) {
    if (++ch < nch) return;
    ch = 0;
    tile += s.kind == kKindKv ? 1 : (int)gridDim.x;
    if (tile < s.ntiles) return;
    p++;
    load(a, at);
  }
};

struct Pipe {
  unsigned char* stages;
  uint64_t* full;
  uint64_t* empty;
  int* err;
  int u;  // next unit
  uint64_t* utrace;
};

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Unit trace (CTA 0): when the consumers find unit u landed.
__device__ __forceinline__ void unit_landed(const Pipe& pp) {
  if (pp.utrace && blockIdx.x == 0 && threadIdx.x == 0 && pp.u < kMkUnitTrace) pp.utrace[2 * pp.u + 1] = global_ns();
}

// Optional phase trace (CTA 0): a stamp at the end of every phase step.
struct Trace {
  uint64_t* buf;
  int n;
  __device__ __forceinline__ void stamp() {
    if (buf && blockIdx.x == 0 && threadIdx.x == 0) buf[n] = global_ns();
    n++;
  }
};

// The step's one grid barrier (before the greedy token is read).
__device__ __forceinline__ void grid_sync(unsigned int* counter, int* err, Trace& tr) {
  named_sync(kMkConsumers);
  tr.stamp();
  if (threadIdx.x == 0) {
    __threadfence();
    atomicAdd(counter, 1u);
    for (uint32_t it = 0;; it++) {
      unsigned int v;
      asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(counter) : "memory");
      if (v >= gridDim.x) break;
      if (it > (1u << 22)) {
        atomicAdd(err, 1);
        break;
      }
      __nanosleep(32);
    }
  }
  named_sync(kMkConsumers);
  tr.stamp();
}

// x -> registers: element 4 v + j of thread v = threadIdx.x + i * 256.
// From tagged words (polled until every tag is `tag`) or from plain memory.
template <int NV>
__device__ __forceinline__ void gather_x(float4 (&xv)[NV], const float* plain, const unsigned long long* ll,
                                         uint32_t tag, int K, int* err) {
  const int nv = K >> 2;
  if (ll) {
    ulonglong2 ra[NV], rb[NV];
#pragma unroll
    for (int i = 0; i < NV; i++) {
      const int v = threadIdx.x + i * kMkConsumers;
      ra[i] = rb[i] = make_ulonglong2(0ull, 0ull);
      if (v < nv) {
        ra[i] = ll_load2(ll + 4 * v);
        rb[i] = ll_load2(ll + 4 * v + 2);
      }
    }
    for (uint32_t it = 0;; it++) {
      bool ok = true;
#pragma unroll
      for (int i = 0; i < NV; i++) {
        const int v = threadIdx.x + i * kMkConsumers;
        if (v >= nv) continue;
        if (ll_tag(ra[i].x) != tag || ll_tag(ra[i].y) != tag) {
          ok = false;
          ra[i] = ll_load2(ll + 4 * v);
        }
        if (ll_tag(rb[i].x) != tag || ll_tag(rb[i].y) != tag) {
          ok = false;
          rb[i] = ll_load2(ll + 4 * v + 2);
        }
      }
      if (ok) break;
      if (spin_expired(it, err)) {
        atomicAdd(err, 1);
        break;
      }
      __nanosleep(100);
    }
#pragma unroll
    for (int i = 0; i < NV; i++)
      xv[i] = make_float4(ll_val(ra[i].x), ll_val(ra[i].y), ll_val(rb[i].x), ll_val(rb[i].y));
  } else {
#pragma unroll
    for (int i = 0; i < NV; i++) {
      const int v = threadIdx.x + i * kMkConsumers;
      xv[i] = v < nv ? __ldg(reinterpret_cast<const float4*>(plain) + v) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
}

// x (optionally RMSNorm(x) * w) -> three int8 digit rows in shared memory,
// one pass: each thread keeps its NV float4s in registers between the
// reduction and the digit step.  Returns the row scale s
// (x = s * (d0 + d1 / 128 + d2 / 128^2)).
template <int NV>
__device__ float stage_digits_n(int8_t* dig, int RSX, const float* plain, const unsigned long long* ll, uint32_t tag,
                                int K, const float* norm_w, float eps, float* red, int* err) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nv = K >> 2;
  // the norm weights do not depend on the step: their loads go out before
  // the poll of x, so both round trips overlap
  float4 w4[NV];
#pragma unroll
  for (int i = 0; i < NV; i++) {
    const int v = threadIdx.x + i * kMkConsumers;
    w4[i] = make_float4(1.f, 1.f, 1.f, 1.f);
    if (norm_w && v < nv) w4[i] = __ldg(reinterpret_cast<const float4*>(norm_w) + v);
  }
  float4 xv[NV];
  gather_x<NV>(xv, plain, ll, tag, K, err);
  float ss = 0.f, mx = 0.f;
#pragma unroll
  for (int i = 0; i < NV; i++) {
    const float4 t = xv[i];
    ss += t.x * t.x + t.y * t.y + t.z * t.z + t.w * t.w;
    const float4 w = w4[i];
    mx = fmaxf(mx, fmaxf(fmaxf(fabsf(t.x * w.x), fabsf(t.y * w.y)), fmaxf(fabsf(t.z * w.z), fabsf(t.w * w.w))));
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
  // one multiplier per element: u = x * w / (rms * sc), |u| < 127; then u is
  // rounded to a multiple of 2^-14 (U = round(u 2^14)) and U is split exactly
  // into balanced digits U = d0 2^14 + d1 2^7 + d2 (d0 in [-127, 127], d1
  // and d2 in [-64, 63]) with integer shifts
  const float c = __fdiv_rn(1.0f, rms) * (1.0f / sc);
#pragma unroll
  for (int i = 0; i < NV; i++) {
    const int v = threadIdx.x + i * kMkConsumers;
    if (v >= nv) continue;
    const float4 t = xv[i];
    const float4 w = w4[i];  // ones without a norm
    const float vals[4] = {t.x * (w.x * c), t.y * (w.y * c), t.z * (w.z * c), t.w * (w.w * c)};
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
    // low bytes of four ints -> one word
    const uint32_t p0 = __byte_perm(__byte_perm(b0[0], b0[1], 0x0040), __byte_perm(b0[2], b0[3], 0x0040), 0x5410);
    const uint32_t p1 = __byte_perm(__byte_perm(b1[0], b1[1], 0x0040), __byte_perm(b1[2], b1[3], 0x0040), 0x5410);
    const uint32_t p2 = __byte_perm(__byte_perm(b2[0], b2[1], 0x0040), __byte_perm(b2[2], b2[3], 0x0040), 0x5410);
    reinterpret_cast<uint32_t*>(dig)[v] = p0;
    reinterpret_cast<uint32_t*>(dig + RSX)[v] = p1;
    reinterpret_cast<uint32_t*>(dig + 2 * RSX)[v] = p2;
  }
  named_sync(kMkConsumers);
  return sc;
}

__device__ __forceinline__ float stage_digits(int8_t* dig, int RSX, const float* plain, const unsigned long long* ll,
                                              uint32_t tag, int K, const float* norm_w, float eps, float* red,
                                              int* err) {
  if (K <= 4 * 4 * kMkConsumers) return stage_digits_n<4>(dig, RSX, plain, ll, tag, K, norm_w, eps, red, err);
  return stage_digits_n<kMkXRegs>(dig, RSX, plain, ll, tag, K, norm_w, eps, red, err);
}

// Channel scales of this CTA's nt tiles of a phase -> ssc[it * 8 + column]
// (two 16-byte cp.async per tile; waited for before the epilogue).
__device__ __forceinline__ void prefetch_scales(float* ssc, const MkArgs& a, int l, int kind, int nt) {
  const int t = threadIdx.x;
  if (t < 2 * nt) {
    const int it = t >> 1, hf = t & 1;
    const int tile = blockIdx.x + it * gridDim.x;
    const float* src;
    if (kind == 0) {  // qkv: rows i0..i0+3 and i0+D/2..i0+D/2+3 of a head
      const int per = a.D / 8, head = tile / per, i0 = (tile % per) * 4;
      src = a.sqkv + (size_t)l * (a.H + 2 * a.Hkv) * a.D + head * a.D + i0 + hf * (a.D / 2);
    } else if (kind == 2) {  // gate rows 4 t.., up rows 4 t..
      src = (hf ? a.su : a.sg) + (size_t)l * 2 * a.F + tile * 4;
    } else {  // o (1) / down (3): rows 8 t .. 8 t + 7
      src = (kind == 1 ? a.so : a.sd) + (size_t)l * a.d + tile * 8 + hf * 4;
    }
    cp_async16(ssc + it * 8 + hf * 4, src);
  }
  cp_async_commit();
}

// One int8 tile through the pipe; this warp's partial sums of digit rows 0..2
// go to part[warp * 24 + row * 8 + column] (lanes g < 3 hold row g).
__device__ __forceinline__ void int8_tile(int* part, Pipe& pp, const int8_t* dig, int RSX, int Kc, int nch) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int RS = bank_stride(Kc), kbc = Kc / 64;
  // four independent accumulators: a stage's MMAs form four short dependency
  // chains instead of one long one (integer sums, so the split is exact)
  int d0[4] = {0, 0, 0, 0}, d1[4] = {0, 0, 0, 0}, d2[4] = {0, 0, 0, 0}, d3[4] = {0, 0, 0, 0};
  for (int ch = 0; ch < nch; ch++, pp.u++) {
    const int st = pp.u % kMkStages, use = pp.u / kMkStages;
    mbarrier_wait(&pp.full[st], (uint32_t)(use & 1), pp.err);
    unit_landed(pp);
    const unsigned char* sp = pp.stages + (size_t)st * kMkStageBytes + (size_t)g * RS + 16 * t;
    const int8_t* xr = dig + (size_t)(g < 3 ? g : 0) * RSX + ch * Kc + 16 * t;
    int kb = warp;
    for (; kb + kMkWarps < kbc; kb += 2 * kMkWarps) {
      const uint4 wa = *reinterpret_cast<const uint4*>(sp + kb * 64);
      const uint4 wb = *reinterpret_cast<const uint4*>(sp + (kb + kMkWarps) * 64);
      uint4 xa = make_uint4(0u, 0u, 0u, 0u), xb = make_uint4(0u, 0u, 0u, 0u);
      if (g < 3) {
        xa = *reinterpret_cast<const uint4*>(xr + kb * 64);
        xb = *reinterpret_cast<const uint4*>(xr + (kb + kMkWarps) * 64);
      }
      mma_s8_16832(d0, xa.x, 0u, xa.y, 0u, wa.x, wa.y);
      mma_s8_16832(d1, xa.z, 0u, xa.w, 0u, wa.z, wa.w);
      mma_s8_16832(d2, xb.x, 0u, xb.y, 0u, wb.x, wb.y);
      mma_s8_16832(d3, xb.z, 0u, xb.w, 0u, wb.z, wb.w);
    }
    if (kb < kbc) {
      const uint4 wa = *reinterpret_cast<const uint4*>(sp + kb * 64);
      uint4 xa = make_uint4(0u, 0u, 0u, 0u);
      if (g < 3) xa = *reinterpret_cast<const uint4*>(xr + kb * 64);
      mma_s8_16832(d0, xa.x, 0u, xa.y, 0u, wa.x, wa.y);
      mma_s8_16832(d1, xa.z, 0u, xa.w, 0u, wa.z, wa.w);
    }
    mbarrier_arrive(&pp.empty[st]);
  }
  if (g < 3) {
    part[warp * 24 + g * 8 + 2 * t] = d0[0] + d1[0] + d2[0] + d3[0];
    part[warp * 24 + g * 8 + 2 * t + 1] = d0[1] + d1[1] + d2[1] + d3[1];
  }
}

// After the phase's tile loop: y of column `lane` (< 8) of tile `it`.
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

// Online-softmax update of one query head with R key/value rows (the
// reference's scale after Q.K^T; masked rows carry -inf).
template <int VEC, int R>
__device__ __forceinline__ void softmax_rows(const float (&qv)[VEC], const float (&kr)[R][VEC], const float (&vr)[R][VEC],
                                             const bool (&valid)[R], float scale, float& mx, float& ls,
                                             float (&o)[VEC]) {
  float s[R];
#pragma unroll
  for (int u = 0; u < R; u++) {
    float dd = 0.f;
#pragma unroll
    for (int e = 0; e < VEC; e++) dd = fmaf(qv[e], kr[u][e], dd);
    s[u] = dd;
  }
#pragma unroll
  for (int o2 = 16; o2 > 0; o2 >>= 1)
#pragma unroll
    for (int u = 0; u < R; u++) s[u] += __shfl_xor_sync(0xffffffffu, s[u], o2);
  float tmax = -INFINITY;
#pragma unroll
  for (int u = 0; u < R; u++) {
    s[u] = valid[u] ? s[u] * scale : -INFINITY;
    tmax = fmaxf(tmax, s[u]);
  }
  const float mn = fmaxf(mx, tmax);
  const float corr = expf(mx - mn);
  float psum = 0.f;
#pragma unroll
  for (int e = 0; e < VEC; e++) o[e] *= corr;
#pragma unroll
  for (int u = 0; u < R; u++) {
    const float p = expf(s[u] - mn);
    psum += p;
#pragma unroll
    for (int e = 0; e < VEC; e++) o[e] = fmaf(p, vr[u][e], o[e]);
  }
  ls = ls * corr + psum;
  mx = mn;
}

// This CTA's attention split of kv head at.kvh: the cache rows [j0, j1)
// arrive through the ring; split 0 adds the step's own row (tagged new k/v)
// and combines the other splits' tagged partials into the heads' outputs.
// The G query heads of the kv head each get 8 / G warps, and each of those
// warps a fixed range of every unit's rows, so the registers one warp holds
// do not grow with G.
template <int VEC>
__device__ void attention_split(const MkArgs& a, const LLOff& lo, const AttnSplit& at, Pipe& pp, float* merge,
                                uint32_t tag_qkv, uint32_t tag_part, uint32_t tag_attn) {
  constexpr int D = VEC * 32;
  constexpr int PU = kMkKvBytes / (D * 4);  // cache rows per unit
  constexpr int R = 4;                       // rows per softmax update
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kvh = at.kvh, G = a.H / a.Hkv, WPH = kMkWarps / G;
  const int gi = warp / WPH, wr = warp - gi * WPH;  // query head of the group, row range
  const int RW = PU / WPH;                          // rows per warp per unit (a multiple of R)
  const int hq = kvh * G + gi;
  unsigned long long* ll = a.ll;
  // q of this warp's query head
  float qr[VEC];
  {
    unsigned long long w[VEC];
#pragma unroll
    for (int e = 0; e < VEC; e++) w[e] = ll_load(ll + lo.q + (size_t)hq * D + lane * VEC + e);
    for (uint32_t it = 0;; it++) {
      bool ok = true;
#pragma unroll
      for (int e = 0; e < VEC; e++)
        if (ll_tag(w[e]) != tag_qkv) {
          ok = false;
          w[e] = ll_load(ll + lo.q + (size_t)hq * D + lane * VEC + e);
        }
      if (ok) break;
      if (spin_expired(it, pp.err)) {
        atomicAdd(pp.err, 1);
        break;
      }
      __nanosleep(64);
    }
#pragma unroll
    for (int e = 0; e < VEC; e++) qr[e] = ll_val(w[e]);
  }
  float mx = -INFINITY, lsum = 0.f, o[VEC];
#pragma unroll
  for (int e = 0; e < VEC; e++) o[e] = 0.f;
  for (int u = 0; u < at.nunits; u++, pp.u++) {
    const int st = pp.u % kMkStages, use = pp.u / kMkStages;
    mbarrier_wait(&pp.full[st], (uint32_t)(use & 1), pp.err);
    unit_landed(pp);
    const int64_t js = at.j0 + (int64_t)u * PU;
    const int rows = (int)((at.j1 - js) < PU ? (at.j1 - js) : PU);
    const float* ks = reinterpret_cast<const float*>(pp.stages + (size_t)st * kMkStageBytes);
    const float* vs = ks + kMkKvBytes / 4;
    for (int r0 = wr * RW; r0 < wr * RW + RW && r0 < rows; r0 += R) {
      float kr[R][VEC], vr[R][VEC];
      bool valid[R];
#pragma unroll
      for (int i = 0; i < R; i++) {
        valid[i] = r0 + i < rows;
        const int rr = valid[i] ? r0 + i : r0;
        if constexpr (VEC == 4) {
          const float4 k4 = *reinterpret_cast<const float4*>(ks + rr * D + lane * 4);
          const float4 v4 = *reinterpret_cast<const float4*>(vs + rr * D + lane * 4);
          kr[i][0] = k4.x; kr[i][1] = k4.y; kr[i][2] = k4.z; kr[i][3] = k4.w;
          vr[i][0] = v4.x; vr[i][1] = v4.y; vr[i][2] = v4.z; vr[i][3] = v4.w;
        } else {
          const float2 k2 = *reinterpret_cast<const float2*>(ks + rr * D + lane * 2);
          const float2 v2 = *reinterpret_cast<const float2*>(vs + rr * D + lane * 2);
          kr[i][0] = k2.x; kr[i][1] = k2.y;
          vr[i][0] = v2.x; vr[i][1] = v2.y;
        }
      }
      softmax_rows<VEC, R>(qr, kr, vr, valid, a.attn_scale, mx, lsum, o);
    }
    mbarrier_arrive(&pp.empty[st]);
  }
  if (at.split == 0 && wr == 0) {
    // the step's own key/value row, written tagged by the QKV epilogues
    float kr[1][VEC], vr[1][VEC];
    const bool valid[1] = {true};
    unsigned long long wk[VEC], wv[VEC];
#pragma unroll
    for (int e = 0; e < VEC; e++) {
      wk[e] = ll_load(ll + lo.kv + (size_t)kvh * D + lane * VEC + e);
      wv[e] = ll_load(ll + lo.kv + (size_t)(a.Hkv + kvh) * D + lane * VEC + e);
    }
    for (uint32_t it = 0;; it++) {
      bool ok = true;
#pragma unroll
      for (int e = 0; e < VEC; e++) {
        if (ll_tag(wk[e]) != tag_qkv) {
          ok = false;
          wk[e] = ll_load(ll + lo.kv + (size_t)kvh * D + lane * VEC + e);
        }
        if (ll_tag(wv[e]) != tag_qkv) {
          ok = false;
          wv[e] = ll_load(ll + lo.kv + (size_t)(a.Hkv + kvh) * D + lane * VEC + e);
        }
      }
      if (ok) break;
      if (spin_expired(it, pp.err)) {
        atomicAdd(pp.err, 1);
        break;
      }
      __nanosleep(64);
    }
#pragma unroll
    for (int e = 0; e < VEC; e++) {
      kr[0][e] = ll_val(wk[e]);
      vr[0][e] = ll_val(wv[e]);
    }
    softmax_rows<VEC, 1>(qr, kr, vr, valid, a.attn_scale, mx, lsum, o);
  }
  // merge the warps of each query head: merge[warp][D + 2]
  {
    float* mw = merge + (size_t)warp * (D + 2);
#pragma unroll
    for (int e = 0; e < VEC; e++) mw[lane * VEC + e] = o[e];
    if (lane == 0) {
      mw[D] = mx;
      mw[D + 1] = lsum;
    }
  }
  named_sync(kMkConsumers);
  const int ns = a.nsplit;
  for (int idx = threadIdx.x; idx < G * D; idx += kMkConsumers) {
    const int g = idx / D, e = idx - g * D;
    const float* mg = merge + (size_t)g * WPH * (D + 2);
    float m = -INFINITY;
    for (int w = 0; w < WPH; w++) m = fmaxf(m, mg[(size_t)w * (D + 2) + D]);
    float L = 0.f, O = 0.f;
    if (m != -INFINITY) {
      for (int w = 0; w < WPH; w++) {
        const float* mw = mg + (size_t)w * (D + 2);
        const float c = expf(mw[D] - m);
        L = fmaf(mw[D + 1], c, L);
        O = fmaf(mw[e], c, O);
      }
    }
    const int hqo = kvh * G + g;
    if (at.split != 0) {
      unsigned long long* p = ll + lo.part + ((size_t)hqo * ns + at.split) * (D + 2);
      ll_store(p + e, O, tag_part);
      if (e == 0) {
        ll_store(p + D, m, tag_part);
        ll_store(p + D + 1, L, tag_part);
      }
      continue;
    }
    // split 0 combines: its own (m, L, O) and the other splits' tagged partials
    unsigned long long pm[kMkMaxSplit], pl[kMkMaxSplit], po[kMkMaxSplit];
    const unsigned long long* pb = ll + lo.part + (size_t)hqo * ns * (D + 2);
#pragma unroll
    for (int s = 1; s < kMkMaxSplit; s++) {
      pm[s] = pl[s] = po[s] = 0ull;
      if (s < ns) {
        pm[s] = ll_load(pb + (size_t)s * (D + 2) + D);
        pl[s] = ll_load(pb + (size_t)s * (D + 2) + D + 1);
        po[s] = ll_load(pb + (size_t)s * (D + 2) + e);
      }
    }
    for (uint32_t it = 0;; it++) {
      bool ok = true;
#pragma unroll
      for (int s = 1; s < kMkMaxSplit; s++) {
        if (s >= ns) continue;
        if (ll_tag(pm[s]) != tag_part) {
          ok = false;
          pm[s] = ll_load(pb + (size_t)s * (D + 2) + D);
        }
        if (ll_tag(pl[s]) != tag_part) {
          ok = false;
          pl[s] = ll_load(pb + (size_t)s * (D + 2) + D + 1);
        }
        if (ll_tag(po[s]) != tag_part) {
          ok = false;
          po[s] = ll_load(pb + (size_t)s * (D + 2) + e);
        }
      }
      if (ok) break;
      if (spin_expired(it, pp.err)) {
        atomicAdd(pp.err, 1);
        break;
      }
      __nanosleep(64);
    }
    float M = m;
#pragma unroll
    for (int s = 1; s < kMkMaxSplit; s++)
      if (s < ns) M = fmaxf(M, ll_val(pm[s]));
    float Lc = 0.f, Oc = 0.f;
    if (m != -INFINITY) {
      const float c = expf(m - M);
      Lc = L * c;
      Oc = O * c;
    }
#pragma unroll
    for (int s = 1; s < kMkMaxSplit; s++) {
      if (s >= ns) continue;
      const float ms = ll_val(pm[s]);
      if (ms == -INFINITY) continue;
      const float c = expf(ms - M);
      Lc = fmaf(ll_val(pl[s]), c, Lc);
      Oc = fmaf(ll_val(po[s]), c, Oc);
    }
    ll_store(ll + lo.attn + (size_t)hqo * D + e, Oc / Lc, tag_attn);
  }
  named_sync(kMkConsumers);  // merge is reused by the next phase's digits
}

__device__ __forceinline__ unsigned long long greedy_key(float v, int idx) {
  uint32_t b = __float_as_uint(v);
  b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return ((unsigned long long)b << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)idx);
}

__global__ void __launch_bounds__(kMkThreads, 1) decode_megakernel(MkArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  const LLOff lo{a.ll_q, a.ll_kv, a.ll_part, a.ll_attn, a.ll_h, a.ll_act, 0};
  unsigned char* stages = smem;
  int8_t* dig = reinterpret_cast<int8_t*>(smem + a.sm_dig);
  float* merge = reinterpret_cast<float*>(smem + a.sm_dig);
  float* xbuf = reinterpret_cast<float*>(smem + a.sm_xbuf);
  int* part = reinterpret_cast<int*>(smem + a.sm_xbuf);  // shares the region with xbuf
  float* ssc = reinterpret_cast<float*>(smem + a.sm_ssc);
  float* hres = reinterpret_cast<float*>(smem + a.sm_res);
  float* srope = reinterpret_cast<float*>(smem + a.sm_rope);
  float* redf = reinterpret_cast<float*>(smem + a.sm_red);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + a.sm_bar);
  uint64_t* empty = full + kMkStages;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t pos = *a.pos;
  const AttnSplit at = attn_split_of(a, pos);
  if (threadIdx.x == 0) {
    for (int s = 0; s < kMkStages; s++) {
      mbarrier_init(&full[s], 1);
      mbarrier_init(&empty[s], kMkConsumers);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();

  if (warp == kMkWarps) {
    // producer warp: the step's stream in consumption order.  All lanes walk
    // the units; lane 0 posts a unit's byte count and lanes 0..7 each issue
    // one row's copy (one thread issuing all of them cannot keep up with HBM)
    // weights and cache rows are read once per step: evict them first, so
    // the exchange words, norm weights and scales stay in L2
    uint64_t policy;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
    const int pu = kMkKvBytes / (a.D * 4);
    UnitCursor c;
    c.start(a, at);
    for (int u = 0; !c.done; u++) {
      const int st = u % kMkStages, use = u / kMkStages;
      if (use > 0) mbarrier_wait(&empty[st], (uint32_t)((use - 1) & 1), a.err);
      unsigned char* dst = stages + (size_t)st * kMkStageBytes;
      if (c.s.kind == kKindKv) {
        const int64_t js = at.j0 + (int64_t)c.tile * pu;
        const int rows = (int)((at.j1 - js) < pu ? (at.j1 - js) : pu);
        const uint32_t bytes = (uint32_t)rows * (uint32_t)a.D * 4u;
        if (lane == 0) mbarrier_expect_tx(&full[st], 2u * bytes);
        __syncwarp();
        if (lane < 2) {
          const size_t off = (((size_t)c.s.layer * a.Hkv + at.kvh) * a.max_seq + (size_t)js) * a.D;
          bulk_copy_g2s_hint(dst + lane * kMkKvBytes, (lane ? a.vc : a.kc) + off, bytes, &full[st], policy);
        }
      } else {
        if (lane == 0) mbarrier_expect_tx(&full[st], (uint32_t)(8 * c.Kc));
        __syncwarp();
        if (lane < 8)
          bulk_copy_g2s_hint(dst + (size_t)lane * bank_stride(c.Kc), row_of(c.s, c.tile, lane) + (size_t)c.ch * c.Kc,
                             (uint32_t)c.Kc, &full[st], policy);
      }
      if (lane == 0 && a.utrace && blockIdx.x == 0 && u < kMkUnitTrace) a.utrace[2 * u] = global_ns();
      c.advance(a, at);
    }
    // every copy lands before the consumers release its stage, so the CTA
    // never exits with a copy in flight
    return;
  }
  // consumers
  Trace tr{a.trace, 0};
  tr.stamp();
  Pipe pp{stages, full, empty, a.err, 0, a.utrace};
  const int64_t token = __ldcg(a.tokens);
  const uint32_t e = *a.epoch + 1u;
  const int half = a.D / 2;
  const int HD = a.H * a.D;
  const int L = a.L;
  unsigned long long* ll = a.ll;
  const float* emb = a.embed + (size_t)token * a.d;
  // residual rows this CTA's O / down tiles own, from the embedding
  // (cpu/backend.go:1289-1339); the rotary table row of the position
  for (int j = threadIdx.x; j < a.tiles_res * 8; j += kMkConsumers) {
    const int tile = blockIdx.x + (j >> 3) * gridDim.x;
    hres[j] = tile < a.d / 8 ? __ldg(emb + tile * 8 + (j & 7)) : 0.f;
  }
  for (int i = threadIdx.x; i < half; i += kMkConsumers) {
    srope[i] = __ldg(a.cos_t + (size_t)pos * half + i);
    srope[half + i] = __ldg(a.sin_t + (size_t)pos * half + i);
  }
  // (the first staging's CTA barriers order these before their readers)

  for (int l = 0; l < L; l++) {
    // ---- RMSNorm + Q/K/V + RoPE + KV append ----
    {
      const Stream s = stream_of(a, 5 * l, at);
      const int Kc = chunk_bytes(s.row_bytes), nch = s.row_bytes / Kc;
      const float sc = l == 0 ? stage_digits(dig, a.RSX, emb, nullptr, 0u, a.d, a.attn_norm, a.eps, redf, a.err)
                              : stage_digits(dig, a.RSX, nullptr, ll + lo.h, tag_of(e, L, l - 1, kTagH2), a.d,
                                             a.attn_norm + (size_t)l * a.d, a.eps, redf, a.err);
      tr.stamp();
      const int nt = s.ntiles > (int)blockIdx.x ? (s.ntiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x : 0;
      prefetch_scales(ssc, a, l, 0, nt);
      for (int it = 0; it < nt; it++) int8_tile(part + it * kMkPart, pp, dig, a.RSX, Kc, nch);
      cp_async_wait_all();
      named_sync(kMkConsumers);
      tr.stamp();
      const uint32_t tg = tag_of(e, L, l, kTagQkv);
      float* kcl = a.kc + (size_t)l * a.Hkv * a.max_seq * a.D;
      float* vcl = a.vc + (size_t)l * a.Hkv * a.max_seq * a.D;
      for (int it = warp; it < nt; it += kMkWarps) {
        const int tile = blockIdx.x + it * gridDim.x;
        const int per = a.D / 8, head = tile / per, i = (tile % per) * 4 + (lane & 3);
        const float y = tile_value(part, it, sc);
        const float v = lane < 8 ? y * ssc[it * 8 + lane] : 0.f;
        const float partner = __shfl_xor_sync(0xffffffffu, v, 4);
        if (lane < 4) {
          if (head < a.H + a.Hkv) {
            const float c = srope[i], sn = srope[half + i];
            const float o0 = __fsub_rn(__fmul_rn(v, c), __fmul_rn(partner, sn));
            const float o1 = __fadd_rn(__fmul_rn(v, sn), __fmul_rn(partner, c));
            if (head < a.H) {
              ll_store(ll + lo.q + (size_t)head * a.D + i, o0, tg);
              ll_store(ll + lo.q + (size_t)head * a.D + i + half, o1, tg);
            } else {
              const int kh = head - a.H;
              float* o = kcl + ((size_t)kh * a.max_seq + pos) * a.D;
              o[i] = o0;
              o[i + half] = o1;
              ll_store(ll + lo.kv + (size_t)kh * a.D + i, o0, tg);
              ll_store(ll + lo.kv + (size_t)kh * a.D + i + half, o1, tg);
            }
          } else {
            const int vh = head - a.H - a.Hkv;
            float* o = vcl + ((size_t)vh * a.max_seq + pos) * a.D;
            o[i] = v;
            o[i + half] = partner;
            ll_store(ll + lo.kv + (size_t)(a.Hkv + vh) * a.D + i, v, tg);
            ll_store(ll + lo.kv + (size_t)(a.Hkv + vh) * a.D + i + half, partner, tg);
          }
        }
      }
      tr.stamp();
    }
    // ---- split-K attention over the cache (quantized.go:319-372) ----
    if (at.kvh >= 0) {
      const uint32_t tq = tag_of(e, L, l, kTagQkv), tp = tag_of(e, L, l, kTagPart), ta = tag_of(e, L, l, kTagAttn);
      if (a.D == 128) attention_split<4>(a, lo, at, pp, merge, tq, tp, ta);
      else attention_split<2>(a, lo, at, pp, merge, tq, tp, ta);
    }
    tr.stamp();
    // ---- O projection + residual ----
    {
      const Stream s = stream_of(a, 5 * l + 2, at);
      const int Kc = chunk_bytes(s.row_bytes), nch = s.row_bytes / Kc;
      const float sc = stage_digits(dig, a.RSX, nullptr, ll + lo.attn, tag_of(e, L, l, kTagAttn), HD, nullptr, 0.f,
                                    redf, a.err);
      tr.stamp();
      const int nt = s.ntiles > (int)blockIdx.x ? (s.ntiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x : 0;
      prefetch_scales(ssc, a, l, 1, nt);
      for (int it = 0; it < nt; it++) int8_tile(part + it * kMkPart, pp, dig, a.RSX, Kc, nch);
      cp_async_wait_all();
      named_sync(kMkConsumers);
      tr.stamp();
      const uint32_t tg = tag_of(e, L, l, kTagH1);
      for (int it = warp; it < nt; it += kMkWarps) {
        const int r = (blockIdx.x + it * gridDim.x) * 8 + lane;
        const float y = tile_value(part, it, sc);
        if (lane < 8) {
          const float hv = hres[it * 8 + lane] + y * ssc[it * 8 + lane];
          hres[it * 8 + lane] = hv;
          ll_store(ll + lo.h + r, hv, tg);
        }
      }
      tr.stamp();
    }
    // ---- RMSNorm + gate/up + SwiGLU ----
    {
      const Stream s = stream_of(a, 5 * l + 3, at);
      const int Kc = chunk_bytes(s.row_bytes), nch = s.row_bytes / Kc;
      const float sc = stage_digits(dig, a.RSX, nullptr, ll + lo.h, tag_of(e, L, l, kTagH1), a.d,
                                    a.mlp_norm + (size_t)l * a.d, a.eps, redf, a.err);
      tr.stamp();
      const int nt = s.ntiles > (int)blockIdx.x ? (s.ntiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x : 0;
      prefetch_scales(ssc, a, l, 2, nt);
      for (int it = 0; it < nt; it++) int8_tile(part + it * kMkPart, pp, dig, a.RSX, Kc, nch);
      cp_async_wait_all();
      named_sync(kMkConsumers);
      tr.stamp();
      const uint32_t tg = tag_of(e, L, l, kTagAct);
      for (int it = warp; it < nt; it += kMkWarps) {
        const int j = (blockIdx.x + it * gridDim.x) * 4 + (lane & 3);
        const float y = tile_value(part, it, sc);
        const float v = lane < 8 ? y * ssc[it * 8 + lane] : 0.f;
        const float partner = __shfl_xor_sync(0xffffffffu, v, 4);
        if (lane < 4) {
          const float sig = 1.0f / (1.0f + expf(-v));
          ll_store(ll + lo.act + j, (v * sig) * partner, tg);
        }
      }
      tr.stamp();
    }
    // ---- down projection + residual ----
    {
      const Stream s = stream_of(a, 5 * l + 4, at);
      const int Kc = chunk_bytes(s.row_bytes), nch = s.row_bytes / Kc;
      const float sc = stage_digits(dig, a.RSX, nullptr, ll + lo.act, tag_of(e, L, l, kTagAct), a.F, nullptr, 0.f,
                                    redf, a.err);
      tr.stamp();
      const int nt = s.ntiles > (int)blockIdx.x ? (s.ntiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x : 0;
      prefetch_scales(ssc, a, l, 3, nt);
      for (int it = 0; it < nt; it++) int8_tile(part + it * kMkPart, pp, dig, a.RSX, Kc, nch);
      cp_async_wait_all();
      named_sync(kMkConsumers);
      tr.stamp();
      const uint32_t tg = tag_of(e, L, l, kTagH2);
      for (int it = warp; it < nt; it += kMkWarps) {
        const int r = (blockIdx.x + it * gridDim.x) * 8 + lane;
        const float y = tile_value(part, it, sc);
        if (lane < 8) {
          const float hv = hres[it * 8 + lane] + y * ssc[it * 8 + lane];
          hres[it * 8 + lane] = hv;
          ll_store(ll + lo.h + r, hv, tg);
          if (l == L - 1) a.h[r] = hv;
        }
      }
      tr.stamp();
    }
  }

  // ---- final RMSNorm + fp32 lm_head + greedy argmax ----
  {
    // xbuf = RMSNorm(h) * final_norm in fp32 (quantized.go:154-172)
    float ss = 0.f;
    const uint32_t th = tag_of(e, L, L - 1, kTagH2);
    if (a.d <= 4 * 4 * kMkConsumers) {
      float4 xv[4];
      gather_x<4>(xv, nullptr, ll + lo.h, th, a.d, a.err);
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const int v = threadIdx.x + i * kMkConsumers;
        if (v < a.d / 4) {
          reinterpret_cast<float4*>(xbuf)[v] = xv[i];
          ss += xv[i].x * xv[i].x + xv[i].y * xv[i].y + xv[i].z * xv[i].z + xv[i].w * xv[i].w;
        }
      }
    } else {
      float4 xv[kMkXRegs];
      gather_x<kMkXRegs>(xv, nullptr, ll + lo.h, th, a.d, a.err);
#pragma unroll
      for (int i = 0; i < kMkXRegs; i++) {
        const int v = threadIdx.x + i * kMkConsumers;
        if (v < a.d / 4) {
          reinterpret_cast<float4*>(xbuf)[v] = xv[i];
          ss += xv[i].x * xv[i].x + xv[i].y * xv[i].y + xv[i].z * xv[i].z + xv[i].w * xv[i].w;
        }
      }
    }
    ss = warp_sum(ss);
    if (lane == 0) redf[warp] = ss;
    named_sync(kMkConsumers);
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < kMkWarps; w++) tot += redf[w];
    const float rms = __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)a.d), a.eps));
    for (int i = threadIdx.x; i < a.d; i += kMkConsumers) xbuf[i] = __fmul_rn(__fdiv_rn(xbuf[i], rms), a.final_norm[i]);
    named_sync(kMkConsumers);
    tr.stamp();
    const Stream s = stream_of(a, 5 * L, at);
    const int Kc = chunk_bytes(s.row_bytes), nch = s.row_bytes / Kc, RS = bank_stride(Kc);
    const int fpc = Kc / 4;  // floats per chunk
    unsigned long long best = 0ull;
    for (int tile = blockIdx.x; tile < s.ntiles; tile += gridDim.x) {
      float acc = 0.f;
      for (int ch = 0; ch < nch; ch++, pp.u++) {
        const int st = pp.u % kMkStages, use = pp.u / kMkStages;
        mbarrier_wait(&full[st], (uint32_t)(use & 1), a.err);
        unit_landed(pp);
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
  grid_sync(a.bar_counter, a.err, tr);
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
    *a.epoch = e;
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
  a.xbuf_floats = a.d;
  a.merge_bytes = (size_t)kMkWarps * (a.D + 2) * sizeof(float);
  a.tiles_max = max_tiles_per_cta(a, grid);
  a.tiles_res = (a.d / 8 + grid - 1) / grid;
  MkLayout Ly;
  Ly.init(a.kmax_bytes, a.xbuf_floats, a.merge_bytes, a.tiles_max, a.tiles_res, a.D);
  a.RSX = Ly.RSX;
  a.sm_dig = (uint32_t)Ly.dig_off;
  a.sm_xbuf = (uint32_t)Ly.xbuf_off;
  a.sm_ssc = (uint32_t)Ly.ssc_off;
  a.sm_res = (uint32_t)Ly.res_off;
  a.sm_rope = (uint32_t)Ly.rope_off;
  a.sm_red = (uint32_t)Ly.red_off;
  a.sm_bar = (uint32_t)Ly.bar_off;
  LLOff lo;
  lo.init(a.d, a.H, a.Hkv, a.D, a.F, a.nsplit);
  a.ll_q = (uint32_t)lo.q;
  a.ll_kv = (uint32_t)lo.kv;
  a.ll_part = (uint32_t)lo.part;
  a.ll_attn = (uint32_t)lo.attn;
  a.ll_h = (uint32_t)lo.h;
  a.ll_act = (uint32_t)lo.act;
}

}  // namespace

int megakernel_splits(int Hkv) {
  int ns = Hkv > 0 ? sm_count() / Hkv : 1;  // one split per CTA
  if (ns < 1) ns = 1;
  if (ns > kMkMaxSplit) ns = kMkMaxSplit;
  return ns;
}

size_t megakernel_ll_words(int d, int H, int Hkv, int D, int F, int nsplit) {
  LLOff lo;
  lo.init(d, H, Hkv, D, F, nsplit);
  return lo.total;
}

bool megakernel_supported(int d, int H, int Hkv, int D, int F, int V, int batch) {
  if (batch != 1) return false;
  if (d % 64 || (H * D) % 64 || F % 64 || (4 * d) % 64) return false;
  if (d % 8 || F % 4 || D % 8 || (D != 64 && D != 128)) return false;
  const int G = H / Hkv;
  if (H % Hkv || (G != 1 && G != 2 && G != 4 && G != 8)) return false;
  if (Hkv > sm_count()) return false;  // one attention split per CTA
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
  if (a.tiles_max * 2 > kMkConsumers) return false;  // scale prefetch: one cp.async per thread
  MkLayout Ly;
  Ly.init(a.kmax_bytes, a.xbuf_floats, a.merge_bytes, a.tiles_max, a.tiles_res, a.D);
  return Ly.total <= 227 * 1024;
}

tb_status_t megakernel_launch(MkArgs a, cudaStream_t st) {
  const int grid = sm_count();
  fill_sizes(a, grid);
  MkLayout Ly;
  Ly.init(a.kmax_bytes, a.xbuf_floats, a.merge_bytes, a.tiles_max, a.tiles_res, a.D);
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
