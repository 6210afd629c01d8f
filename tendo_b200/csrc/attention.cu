// attention.cu — KV-cache attention for the quantized Llama path
// (models/llama/quantized.go:319-372): scores = (q . k) * (1/sqrt(D)),
// causal mask j <= i + (Sk - Sq) (models/llama/forward.go:372-417), softmax
// over keys, P . V; GQA reads kv head h / (H / Hkv) directly
// (models/llama/forward.go:345-370) instead of materialising the repeat.
//
// Decode (Sq = 1) is HBM-bound on the cache (fp32 as the reference stores
// it, or bf16 as a model option, read with its own 16-byte-load kernel): split-K over positions,
// one CTA per (split, kv head, sequence) serving all H / Hkv query heads of
// that kv head (each K/V row is read once), online softmax per warp, then a
// combine kernel merges the splits.  Prefill is a tiled (flash-style) fp32
// kernel with the online softmax, so no [S, S] score matrix is stored.
#include <math.h>

#include "common.cuh"
#include "kernels.h"

namespace tb {
namespace {

template <int VEC>
struct VecT;
template <>
struct VecT<2> {
  using T = float2;
};
template <>
struct VecT<4> {
  using T = float4;
};
template <>
struct VecT<1> {
  using T = float;
};

template <int VEC>
__device__ __forceinline__ void load_vec(float (&r)[VEC], const float* p) {
  if constexpr (VEC == 4) {
    float4 t = *reinterpret_cast<const float4*>(p);
    r[0] = t.x; r[1] = t.y; r[2] = t.z; r[3] = t.w;
  } else if constexpr (VEC == 1) {
    r[0] = *p;
  } else {
    float2 t = *reinterpret_cast<const float2*>(p);
    r[0] = t.x; r[1] = t.y;
  }
}
// One tile of U cached rows for G >= 32 / U query heads sharing them (the
// online softmax of each head, the reference's scale after Q.K^T, rows at or
// past `end` masked).  The G U partial dot products of a lane are summed over
// the warp in one butterfly: each round a lane keeps half of its values and
// adds the partner's copy of them, so after five rounds (NV = G U values,
// 62 shuffles for 64) lane l holds the finished scores v = (l << log2(NV/32)) + i,
// i.e. 32 / G consecutive lanes hold one head's U scores.  Those lanes find
// the head's tile max and its exponentials once (not in every lane), and
// the probabilities are then broadcast to every lane for P.V.
template <int VEC, int G, int U>
__device__ __forceinline__ void tile_grouped(const float (&qr)[G][VEC], const float (&kr)[U][VEC],
                                             const float (&vr)[U][VEC], int64_t j0, int64_t end, float scale,
                                             float (&mx)[G], float (&l)[G], float (&o)[G][VEC]) {
  constexpr int NV = G * U;      // scores of the tile
  constexpr int PL = NV / 32;    // finished scores per lane
  constexpr int LG = 32 / G;     // lanes holding one head's scores
  const int lane = threadIdx.x & 31;
  float s[NV];
#pragma unroll
  for (int gi = 0; gi < G; gi++)
#pragma unroll
    for (int u = 0; u < U; u++) {
      float d = 0.f;
#pragma unroll
      for (int e = 0; e < VEC; e++) d = fmaf(qr[gi][e], kr[u][e], d);
      s[gi * U + u] = d;
    }
  // butterfly: offsets 16, 8, 4, 2, 1, halving the values a lane keeps
#pragma unroll
  for (int r = 0; r < 5; r++) {
    const int off = 16 >> r;
    const int half = NV >> (r + 1);
    const bool up = (lane & off) != 0;
#pragma unroll
    for (int i = 0; i < half; i++) {
      const float keep = up ? s[i + half] : s[i];
      const float send = up ? s[i] : s[i + half];
      s[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
    }
  }
  // this lane's scores: head gi = lane / LG, rows u0 .. u0 + PL - 1
  const int gi_own = lane / LG, u0 = (lane % LG) * PL;
  float tmax = -INFINITY;
#pragma unroll
  for (int i = 0; i < PL; i++) {
    s[i] = (j0 + u0 + i < end) ? s[i] * scale : -INFINITY;
    tmax = fmaxf(tmax, s[i]);
  }
#pragma unroll
  for (int o2 = LG / 2; o2 > 0; o2 >>= 1) tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, o2));
  float mown = mx[0];
#pragma unroll
  for (int gi = 1; gi < G; gi++)
    if (gi == gi_own) mown = mx[gi];
  const float mn_own = fmaxf(mown, tmax);  // finite: position j0 < end is valid
  float p[PL], psum = 0.f;
#pragma unroll
  for (int i = 0; i < PL; i++) {
    p[i] = expf(s[i] - mn_own);
    psum += p[i];
  }
#pragma unroll
  for (int o2 = LG / 2; o2 > 0; o2 >>= 1) psum += __shfl_xor_sync(0xffffffffu, psum, o2);
#pragma unroll
  for (int gi = 0; gi < G; gi++) {
    const float mn = __shfl_sync(0xffffffffu, mn_own, gi * LG);
    const float ps = __shfl_sync(0xffffffffu, psum, gi * LG);
    const float corr = expf(mx[gi] - mn);
#pragma unroll
    for (int e = 0; e < VEC; e++) o[gi][e] *= corr;
#pragma unroll
    for (int u = 0; u < U; u++) {
      const float pu = __shfl_sync(0xffffffffu, p[u % PL], gi * LG + u / PL);
#pragma unroll
      for (int e = 0; e < VEC; e++) o[gi][e] = fmaf(pu, vr[u][e], o[gi][e]);
    }
    l[gi] = l[gi] * corr + ps;
    mx[gi] = mn;
  }
}

// grid (nsplit, Hkv, B); VEC = D / 32 values per lane; G query heads per kv
// head; W warps (8 when G >= 4: the G running softmaxes take registers, so
// fewer CTAs fit per SM and each needs more rows in flight).  Each warp takes
// tiles of U consecutive positions: U K rows and U V rows are loaded at once
// (2 U 16-byte loads in flight per lane for D = 128), the U scores reduced
// together, and the running softmax updated once per tile.
template <int VEC, int G, int W>
__global__ void __launch_bounds__(W * 32) attn_decode_kernel(AttnDecodeArgs a) {
  constexpr int D = VEC * 32;
  constexpr int U = 8;
  constexpr int kAttnWarps = W;
  constexpr int kAttnThreads = W * 32;
  __shared__ float sm_o[kAttnWarps][G][D];
  __shared__ float sm_ml[kAttnWarps][G][2];
  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // The position and every cached row before it were written by earlier
  // decode steps, complete before the preceding kernel could launch this one;
  // only row *pos comes from that kernel, so the older rows are prefetched
  // into L2 before waiting on it.
  const int64_t sk = a.pos ? (*a.pos + 1) : a.sk;
  int64_t chunk = (sk + a.nsplit - 1) / a.nsplit;
  chunk = (chunk + U - 1) / U * U;
  const int64_t start = (int64_t)split * chunk;
  const int64_t end = min(start + chunk, sk);
  const float* kb = static_cast<const float*>(a.kcache) + ((size_t)b * a.Hkv + kvh) * a.max_seq * D;
  const float* vb = static_cast<const float*>(a.vcache) + ((size_t)b * a.Hkv + kvh) * a.max_seq * D;
  if (threadIdx.x == 0 && a.l2_prefetch) {
    const int64_t pend = min(end, sk - 1);  // row sk - 1 comes from the preceding kernel
    if (pend > start) {
      prefetch_l2_bulk(kb + start * D, (uint32_t)((pend - start) * D * sizeof(float)));
      prefetch_l2_bulk(vb + start * D, (uint32_t)((pend - start) * D * sizeof(float)));
    }
  }
  pdl_wait();
  pdl_launch_dependents();

  float qr[G][VEC];
#pragma unroll
  for (int gi = 0; gi < G; gi++) load_vec<VEC>(qr[gi], a.q + ((size_t)b * a.H + kvh * G + gi) * D + lane * VEC);

  float mx[G], l[G], o[G][VEC];
#pragma unroll
  for (int gi = 0; gi < G; gi++) {
    mx[gi] = -INFINITY;
    l[gi] = 0.f;
#pragma unroll
    for (int e = 0; e < VEC; e++) o[gi][e] = 0.f;
  }
  for (int64_t j0 = start + (int64_t)warp * U; j0 < end; j0 += (int64_t)kAttnWarps * U) {
    float kr[U][VEC], vr[U][VEC];
#pragma unroll
    for (int u = 0; u < U; u++) {
      const int64_t j = j0 + u;
      if (j < end) {
        load_vec<VEC>(kr[u], kb + j * D + lane * VEC);
        load_vec<VEC>(vr[u], vb + j * D + lane * VEC);
      } else {
#pragma unroll
        for (int e = 0; e < VEC; e++) kr[u][e] = vr[u][e] = 0.f;
      }
    }
    if constexpr (G * U >= 32) {
      tile_grouped<VEC, G, U>(qr, kr, vr, j0, end, a.scale, mx, l, o);
    } else {
#pragma unroll
      for (int gi = 0; gi < G; gi++) {
        float s[U];
#pragma unroll
        for (int u = 0; u < U; u++) {
          float d = 0.f;
#pragma unroll
          for (int e = 0; e < VEC; e++) d = fmaf(qr[gi][e], kr[u][e], d);
          s[u] = d;
        }
#pragma unroll
        for (int o2 = 16; o2 > 0; o2 >>= 1)
#pragma unroll
          for (int u = 0; u < U; u++) s[u] += __shfl_xor_sync(0xffffffffu, s[u], o2);
        float tmax = -INFINITY;
#pragma unroll
        for (int u = 0; u < U; u++) {
          s[u] = (j0 + u < end) ? s[u] * a.scale : -INFINITY;
          tmax = fmaxf(tmax, s[u]);
        }
        const float mn = fmaxf(mx[gi], tmax);  // finite: position j0 < end is valid
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
        l[gi] = l[gi] * corr + psum;
        mx[gi] = mn;
      }
    }
  }
  // merge the warps of this CTA
#pragma unroll
  for (int gi = 0; gi < G; gi++) {
#pragma unroll
    for (int e = 0; e < VEC; e++) sm_o[warp][gi][lane * VEC + e] = o[gi][e];
    if (lane == 0) {
      sm_ml[warp][gi][0] = mx[gi];
      sm_ml[warp][gi][1] = l[gi];
    }
  }
  __syncthreads();
  for (int t = threadIdx.x; t < G * D; t += kAttnThreads) {
    const int gi = t / D, e = t - gi * D;
    float m = -INFINITY;
#pragma unroll
    for (int w = 0; w < kAttnWarps; w++) m = fmaxf(m, sm_ml[w][gi][0]);
    float L = 0.f, O = 0.f;
    if (m != -INFINITY) {
#pragma unroll
      for (int w = 0; w < kAttnWarps; w++) {
        const float c = expf(sm_ml[w][gi][0] - m);
        L = fmaf(sm_ml[w][gi][1], c, L);
        O = fmaf(sm_o[w][gi][e], c, O);
      }
    }
    float* part = a.partial + (((size_t)b * a.H + kvh * G + gi) * a.nsplit + split) * (D + 2);
    part[e] = O;
    if (e == 0) {
      part[D] = m;
      part[D + 1] = L;
    }
  }
}

// bf16 cache (D = 32, 64 or 128): each lane loads 16 bytes (8 elements) of a row,
// so LR = D / 8 lanes cover a row and a warp load covers RW = 32 / LR rows.
// A tile is UU such loads per lane (U = UU RW rows) of K and of V; a lane
// keeps the scores and P V products of its own rows, the row groups agree on
// the tile's max and sum through shuffles, and the partial outputs of the row
// groups are added once at the end (they share every rescaling).  Same grid,
// split and partial-output format as attn_decode_kernel.
template <int D, int G, int W, int UU>
__global__ void __launch_bounds__(W * 32) attn_decode_b16_kernel(AttnDecodeArgs a) {
  constexpr int LR = D / 8, RW = 32 / LR, U = UU * RW;
  __shared__ float sm_o[W][G][D];
  __shared__ float sm_ml[W][G][2];
  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rl = lane / LR, el = (lane % LR) * 8;
  const int64_t sk = a.pos ? (*a.pos + 1) : a.sk;
  int64_t chunk = (sk + a.nsplit - 1) / a.nsplit;
  chunk = (chunk + U - 1) / U * U;
  const int64_t start = (int64_t)split * chunk;
  const int64_t end = min(start + chunk, sk);
  const __nv_bfloat16* kb = static_cast<const __nv_bfloat16*>(a.kcache) + ((size_t)b * a.Hkv + kvh) * a.max_seq * D;
  const __nv_bfloat16* vb = static_cast<const __nv_bfloat16*>(a.vcache) + ((size_t)b * a.Hkv + kvh) * a.max_seq * D;
  if (threadIdx.x == 0 && a.l2_prefetch) {
    const int64_t pend = min(end, sk - 1);  // row sk - 1 comes from the preceding kernel
    if (pend > start) {
      prefetch_l2_bulk(kb + start * D, (uint32_t)((pend - start) * D * 2));
      prefetch_l2_bulk(vb + start * D, (uint32_t)((pend - start) * D * 2));
    }
  }
  pdl_wait();
  pdl_launch_dependents();

  float qr[G][8];
#pragma unroll
  for (int gi = 0; gi < G; gi++) {
    const float* qp = a.q + ((size_t)b * a.H + kvh * G + gi) * D + el;
    const float4 q0 = *reinterpret_cast<const float4*>(qp), q1 = *reinterpret_cast<const float4*>(qp + 4);
    qr[gi][0] = q0.x; qr[gi][1] = q0.y; qr[gi][2] = q0.z; qr[gi][3] = q0.w;
    qr[gi][4] = q1.x; qr[gi][5] = q1.y; qr[gi][6] = q1.z; qr[gi][7] = q1.w;
  }
  float mx[G], l[G], o[G][8];
#pragma unroll
  for (int gi = 0; gi < G; gi++) {
    mx[gi] = -INFINITY;
    l[gi] = 0.f;
#pragma unroll
    for (int e = 0; e < 8; e++) o[gi][e] = 0.f;
  }
  for (int64_t j0 = start + (int64_t)warp * U; j0 < end; j0 += (int64_t)W * U) {
    uint4 kr[UU], vr[UU];
#pragma unroll
    for (int u = 0; u < UU; u++) {
      const int64_t j = j0 + u * RW + rl;
      if (j < end) {
        kr[u] = *reinterpret_cast<const uint4*>(kb + j * D + el);
        vr[u] = *reinterpret_cast<const uint4*>(vb + j * D + el);
      } else {
        kr[u] = make_uint4(0u, 0u, 0u, 0u);
        vr[u] = make_uint4(0u, 0u, 0u, 0u);
      }
    }
#pragma unroll
    for (int gi = 0; gi < G; gi++) {
      float s[UU];
#pragma unroll
      for (int u = 0; u < UU; u++) {
        const uint32_t w[4] = {kr[u].x, kr[u].y, kr[u].z, kr[u].w};
        float d = 0.f;
#pragma unroll
        for (int h = 0; h < 4; h++) {
          d = fmaf(qr[gi][2 * h], __uint_as_float(w[h] << 16), d);
          d = fmaf(qr[gi][2 * h + 1], __uint_as_float(w[h] & 0xffff0000u), d);
        }
        s[u] = d;
      }
      // the row's dot product over its LR lanes
#pragma unroll
      for (int o2 = LR / 2; o2 > 0; o2 >>= 1)
#pragma unroll
        for (int u = 0; u < UU; u++) s[u] += __shfl_xor_sync(0xffffffffu, s[u], o2);
      float tmax = -INFINITY;
#pragma unroll
      for (int u = 0; u < UU; u++) {
        s[u] = (j0 + u * RW + rl < end) ? s[u] * a.scale : -INFINITY;
        tmax = fmaxf(tmax, s[u]);
      }
      // the tile's max over the row groups
#pragma unroll
      for (int o2 = LR; o2 < 32; o2 <<= 1) tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, o2));
      const float mn = fmaxf(mx[gi], tmax);  // finite: row j0 < end is valid
      const float corr = expf(mx[gi] - mn);
      float psum = 0.f;
#pragma unroll
      for (int e = 0; e < 8; e++) o[gi][e] *= corr;
#pragma unroll
      for (int u = 0; u < UU; u++) {
        const float p = expf(s[u] - mn);
        psum += p;
        const uint32_t w[4] = {vr[u].x, vr[u].y, vr[u].z, vr[u].w};
#pragma unroll
        for (int h = 0; h < 4; h++) {
          o[gi][2 * h] = fmaf(p, __uint_as_float(w[h] << 16), o[gi][2 * h]);
          o[gi][2 * h + 1] = fmaf(p, __uint_as_float(w[h] & 0xffff0000u), o[gi][2 * h + 1]);
        }
      }
#pragma unroll
      for (int o2 = LR; o2 < 32; o2 <<= 1) psum += __shfl_xor_sync(0xffffffffu, psum, o2);
      l[gi] = l[gi] * corr + psum;
      mx[gi] = mn;
    }
  }
  // add the row groups' partial outputs, then merge the warps of this CTA
#pragma unroll
  for (int gi = 0; gi < G; gi++) {
#pragma unroll
    for (int e = 0; e < 8; e++) {
      float v = o[gi][e];
#pragma unroll
      for (int o2 = LR; o2 < 32; o2 <<= 1) v += __shfl_xor_sync(0xffffffffu, v, o2);
      o[gi][e] = v;
    }
    if (rl == 0) {
#pragma unroll
      for (int e = 0; e < 8; e++) sm_o[warp][gi][el + e] = o[gi][e];
    }
    if (lane == 0) {
      sm_ml[warp][gi][0] = mx[gi];
      sm_ml[warp][gi][1] = l[gi];
    }
  }
  __syncthreads();
  for (int t = threadIdx.x; t < G * D; t += W * 32) {
    const int gi = t / D, e = t - gi * D;
    float m = -INFINITY;
#pragma unroll
    for (int w = 0; w < W; w++) m = fmaxf(m, sm_ml[w][gi][0]);
    float L = 0.f, O = 0.f;
    if (m != -INFINITY) {
#pragma unroll
      for (int w = 0; w < W; w++) {
        const float c = expf(sm_ml[w][gi][0] - m);
        L = fmaf(sm_ml[w][gi][1], c, L);
        O = fmaf(sm_o[w][gi][e], c, O);
      }
    }
    float* part = a.partial + (((size_t)b * a.H + kvh * G + gi) * a.nsplit + split) * (D + 2);
    part[e] = O;
    if (e == 0) {
      part[D] = m;
      part[D + 1] = L;
    }
  }
}

// One warp per (sequence, head): out = sum_s o_s e^(m_s - M) / sum_s l_s e^(m_s - M).
// Lane s holds split s's (m, l) (nsplit <= 64: two per lane), so the max and
// the weighted sum of l are warp reductions; each lane then sums its D / 32
// output elements over the splits with independent loads.
template <int VEC>
__global__ void attn_combine_kernel(float* out, const float* partial, int B, int H, int nsplit) {
  constexpr int D = VEC * 32;
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  pdl_wait();
  pdl_launch_dependents();
  if (gw >= B * H) return;
  const float* p = partial + (size_t)gw * nsplit * (D + 2);
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  if (lane < nsplit) {
    m0 = p[(size_t)lane * (D + 2) + D];
    l0 = p[(size_t)lane * (D + 2) + D + 1];
  }
  if (lane + 32 < nsplit) {
    m1 = p[(size_t)(lane + 32) * (D + 2) + D];
    l1 = p[(size_t)(lane + 32) * (D + 2) + D + 1];
  }
  const float M = warp_max(fmaxf(m0, m1));
  const float c0 = m0 == -INFINITY ? 0.f : expf(m0 - M);
  const float c1 = m1 == -INFINITY ? 0.f : expf(m1 - M);
  const float L = warp_sum(l0 * c0 + l1 * c1);
  float acc[VEC];
#pragma unroll
  for (int e = 0; e < VEC; e++) acc[e] = 0.f;
  for (int s = 0; s < nsplit; s++) {
    const float c = __shfl_sync(0xffffffffu, s < 32 ? c0 : c1, s & 31);
    if (c == 0.f) continue;
    const float* ps = p + (size_t)s * (D + 2) + lane * VEC;
#pragma unroll
    for (int e = 0; e < VEC; e++) acc[e] = fmaf(ps[e], c, acc[e]);
  }
  float* o = out + (size_t)gw * D + lane * VEC;
#pragma unroll
  for (int e = 0; e < VEC; e++) o[e] = acc[e] / L;
}

// ---------------------------------------------------------------------------
// Prefill: grid (ceil(Sq / BQ), H, B), 256 threads; q/out [B, Sq, H, D].
// ---------------------------------------------------------------------------
constexpr int BQ = 32, BK = 16, KU = BK / 8, kPfThreads = 256;

template <int D, typename KT>
__global__ void __launch_bounds__(kPfThreads) attn_prefill_kernel(float* out, const float* __restrict__ q,
                                                                   const KT* __restrict__ kc,
                                                                   const KT* __restrict__ vc, int H, int Hkv,
                                                                   int Sq, int64_t Sk, int max_seq, float scale) {
  __shared__ float Qs[BQ][D + 1];
  __shared__ float Ks[BK][D + 1];
  __shared__ float Vs[BK][D];
  __shared__ float Ps[BQ][BK];
  const int qt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int kvh = h / (H / Hkv);
  const int t = threadIdx.x;
  const int qi = t >> 3, sub = t & 7;
  const int64_t offset = Sk - Sq;
  const int q0 = qt * BQ;
  for (int i = t; i < BQ * D; i += kPfThreads) {
    const int r = i / D, e = i - r * D;
    const int qq = q0 + r;
    Qs[r][e] = qq < Sq ? q[(((size_t)b * Sq + qq) * H + h) * D + e] : 0.f;
  }
  const KT* kb = kc + ((size_t)b * Hkv + kvh) * max_seq * D;
  const KT* vb = vc + ((size_t)b * Hkv + kvh) * max_seq * D;
  constexpr int OV = D / 8;
  float o[OV];
#pragma unroll
  for (int v = 0; v < OV; v++) o[v] = 0.f;
  float mrow = -INFINITY, lrow = 0.f;
  const int64_t qpos = q0 + qi;
  const int64_t last_key = min((int64_t)(q0 + BQ - 1) + offset, Sk - 1);
  for (int64_t k0 = 0; k0 <= last_key; k0 += BK) {
    __syncthreads();
    for (int i = t; i < BK * D; i += kPfThreads) {
      const int r = i / D, e = i - r * D;
      const int64_t kk = k0 + r;
      const bool ok = kk < Sk;
      Ks[r][e] = ok ? kv_get(kb + kk * D + e) : 0.f;
      Vs[r][e] = ok ? kv_get(vb + kk * D + e) : 0.f;
    }
    __syncthreads();
    float s[KU];
#pragma unroll
    for (int u = 0; u < KU; u++) {
      const int kj = sub + 8 * u;
      float acc = 0.f;
#pragma unroll 8
      for (int e = 0; e < D; e++) acc = fmaf(Qs[qi][e], Ks[kj][e], acc);
      const int64_t kpos = k0 + kj;
      const bool valid = kpos < Sk && kpos <= qpos + offset && qpos < Sq;
      s[u] = valid ? acc * scale : -INFINITY;
    }
    float tm = s[0];
#pragma unroll
    for (int u = 1; u < KU; u++) tm = fmaxf(tm, s[u]);
    tm = fmaxf(tm, __shfl_xor_sync(0xffffffffu, tm, 1));
    tm = fmaxf(tm, __shfl_xor_sync(0xffffffffu, tm, 2));
    tm = fmaxf(tm, __shfl_xor_sync(0xffffffffu, tm, 4));
    const float mn = fmaxf(mrow, tm);
    float ps = 0.f;
#pragma unroll
    for (int u = 0; u < KU; u++) {
      const float p = mn == -INFINITY ? 0.f : expf(s[u] - mn);
      Ps[qi][sub + 8 * u] = p;
      ps += p;
    }
    ps += __shfl_xor_sync(0xffffffffu, ps, 1);
    ps += __shfl_xor_sync(0xffffffffu, ps, 2);
    ps += __shfl_xor_sync(0xffffffffu, ps, 4);
    const float corr = (mrow == -INFINITY) ? 0.f : expf(mrow - mn);
    lrow = lrow * corr + ps;
    mrow = mn;
    __syncwarp();
#pragma unroll
    for (int v = 0; v < OV; v++) o[v] *= corr;
#pragma unroll 4
    for (int kj = 0; kj < BK; kj++) {
      const float p = Ps[qi][kj];
#pragma unroll
      for (int v = 0; v < OV; v++) o[v] = fmaf(p, Vs[kj][sub + 8 * v], o[v]);
    }
  }
  if (qpos < Sq) {
    float* dst = out + (((size_t)b * Sq + qpos) * H + h) * D;
    const float inv = 1.0f / lrow;
#pragma unroll
    for (int v = 0; v < OV; v++) dst[sub + 8 * v] = o[v] * inv;
  }
}

// a bf16 cache: 16-byte loads of 8 elements (attn_decode_b16_kernel); loads
// per lane per tile, fewer where the G softmaxes take the registers
template <int G>
constexpr int b16_loads() {
  return G <= 2 ? 8 : (G == 4 ? 4 : 2);
}

// Resident CTAs per SM of the decode kernel for these shapes (0: none).
template <int VEC, int G>
int decode_occupancy_g(bool kv16) {
  constexpr int W = G >= 4 ? 8 : 4;
  int n = 0;
  const cudaError_t e =
      kv16 ? cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, attn_decode_b16_kernel<VEC * 32, G, W, b16_loads<G>()>,
                                                           W * 32, 0)
           : cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, attn_decode_kernel<VEC, G, W>, W * 32, 0);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return n;
}

template <int VEC>
int decode_occupancy_v(int G, bool kv16) {
  switch (G) {
    case 1: return decode_occupancy_g<VEC, 1>(kv16);
    case 2: return decode_occupancy_g<VEC, 2>(kv16);
    case 4: return decode_occupancy_g<VEC, 4>(kv16);
    case 8: return VEC == 1 && !kv16 ? 0 : decode_occupancy_g<VEC, 8>(kv16);
    default: return 0;
  }
}

int decode_occupancy(int D, int G, bool kv16) {
  if (D == 128) return decode_occupancy_v<4>(G, kv16);
  if (D == 64) return decode_occupancy_v<2>(G, kv16);
  if (D == 32) return decode_occupancy_v<1>(G, kv16);
  return 0;
}

template <int VEC, int G>
tb_status_t launch_decode(AttnDecodeArgs a, cudaStream_t st, bool pdl) {
  // the older rows are prefetched into L2 only while a layer's whole cache
  // fits in it comfortably (a batch-1 step); larger caches stream directly
  a.l2_prefetch = (double)a.B * a.Hkv * a.max_seq * (a.D * (a.kv_bf16 ? 4.0 : 8.0)) <= 96e6;
  constexpr int W = G >= 4 ? 8 : 4;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.nsplit, a.Hkv, a.B);
  cfg.blockDim = dim3(W * 32);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  constexpr int UU = b16_loads<G>();
  cudaError_t e = a.kv_bf16 ? cudaLaunchKernelEx(&cfg, attn_decode_b16_kernel<VEC * 32, G, W, UU>, a)
                            : cudaLaunchKernelEx(&cfg, attn_decode_kernel<VEC, G, W>, a);
  if (e != cudaSuccess) return cuda_fail(e, "attn_decode_kernel");
  const int warps = a.B * a.H;
  cfg.gridDim = dim3((warps + 3) / 4);
  cfg.blockDim = dim3(128);
  e = cudaLaunchKernelEx(&cfg, attn_combine_kernel<VEC>, a.out, (const float*)a.partial, a.B, a.H, a.nsplit);
  if (e != cudaSuccess) return cuda_fail(e, "attn_combine_kernel");
  return TB_SUCCESS;
}

template <int VEC>
tb_status_t launch_decode_g(const AttnDecodeArgs& a, cudaStream_t st, bool pdl) {
  if (VEC == 1 && a.H / a.Hkv > 4) return TB_ERROR_NOT_SUPPORTED;
  switch (a.H / a.Hkv) {
    case 1: return launch_decode<VEC, 1>(a, st, pdl);
    case 2: return launch_decode<VEC, 2>(a, st, pdl);
    case 4: return launch_decode<VEC, 4>(a, st, pdl);
    case 8: return launch_decode<VEC, 8>(a, st, pdl);
    default: return TB_ERROR_NOT_SUPPORTED;
  }
}

}  // namespace

int attn_decode_splits(int B, int H, int Hkv, int D, int64_t max_seq, bool kv_bf16) {
  // About four CTAs per SM, never a split shorter than 16 keys, at most 64.
  const int sm = sm_count();
  const int64_t units = (int64_t)B * Hkv;
  int64_t cap = (max_seq + 15) / 16;
  if (cap > 64) cap = 64;
  auto clampv = [&](int64_t v) { return v > cap ? cap : (v < 1 ? 1 : v); };
  const int64_t base = clampv((4LL * sm + units - 1) / units);
  // never above the count for Hkv = 1, which sizes the C ABI's workspace
  const int64_t bound = clampv((4LL * sm + B - 1) / B);
  // A grid of more than one wave of resident CTAs: the count in
  // [base, 2 base + 2] whose last wave is fullest (ties: fewer splits).
  const int occ = Hkv > 0 && H % Hkv == 0 ? decode_occupancy(D, H / Hkv, kv_bf16) : 0;
  const double slots = (double)sm * occ;
  if (occ <= 0 || (double)(units * base) < slots) return (int)base;
  int64_t best = base;
  double best_eff = 0.0;
  for (int64_t ns = base; ns <= 2 * base + 2 && ns <= bound; ns++) {
    const double x = (double)(units * ns) / slots;
    const double eff = x / ceil(x);
    if (eff > best_eff + 1e-9) {
      best_eff = eff;
      best = ns;
    }
  }
  return (int)best;
}

size_t attn_decode_workspace(int B, int H, int D, int nsplit) {
  return (size_t)B * H * nsplit * (D + 2) * sizeof(float);
}

tb_status_t attn_decode(const AttnDecodeArgs& a, cudaStream_t st, bool pdl) {
  TB_REQUIRE(a.Hkv > 0 && a.H % a.Hkv == 0);
  if (a.D == 128) return launch_decode_g<4>(a, st, pdl);
  if (a.D == 64) return launch_decode_g<2>(a, st, pdl);
  if (a.D == 32) return launch_decode_g<1>(a, st, pdl);
  return TB_ERROR_NOT_SUPPORTED;
}

template <typename KT>
tb_status_t launch_prefill(float* out, const float* q, const KT* kc, const KT* vc, int B, int H, int Hkv, int Sq,
                           int64_t Sk, int D, int max_seq, float scale, cudaStream_t st) {
  dim3 grid((Sq + BQ - 1) / BQ, H, B);
  if (D == 128)
    attn_prefill_kernel<128, KT><<<grid, kPfThreads, 0, st>>>(out, q, kc, vc, H, Hkv, Sq, Sk, max_seq, scale);
  else if (D == 64)
    attn_prefill_kernel<64, KT><<<grid, kPfThreads, 0, st>>>(out, q, kc, vc, H, Hkv, Sq, Sk, max_seq, scale);
  else if (D == 32)
    attn_prefill_kernel<32, KT><<<grid, kPfThreads, 0, st>>>(out, q, kc, vc, H, Hkv, Sq, Sk, max_seq, scale);
  else
    return TB_ERROR_NOT_SUPPORTED;
  return check_launch("attn_prefill_kernel");
}

tb_status_t attn_prefill(float* out, const float* q, const void* kcache, const void* vcache, int B, int H,
                         int Hkv, int Sq, int64_t Sk, int D, int max_seq, float scale, cudaStream_t st,
                         bool kv_bf16) {
  TB_REQUIRE(Hkv > 0 && H % Hkv == 0 && Sq >= 1 && Sk >= Sq);
  if (kv_bf16)
    return launch_prefill(out, q, static_cast<const __nv_bfloat16*>(kcache), static_cast<const __nv_bfloat16*>(vcache),
                          B, H, Hkv, Sq, Sk, D, max_seq, scale, st);
  return launch_prefill(out, q, static_cast<const float*>(kcache), static_cast<const float*>(vcache), B, H, Hkv, Sq,
                        Sk, D, max_seq, scale, st);
}

}  // namespace tb

// ---------------------------------------------------------------------------
// C ABI
// ---------------------------------------------------------------------------
extern "C" size_t tb_attention_workspace_size(int64_t B, int64_t H, int64_t Sq, int64_t D, int64_t max_seq) {
  if (B <= 0 || H <= 0 || D <= 0 || Sq != 1) return 0;
  const int ns = tb::attn_decode_splits((int)B, (int)H, 1, (int)D, max_seq, false);
  // sized for the largest split count any Hkv can pick (Hkv = 1 maximises it)
  return tb::attn_decode_workspace((int)B, (int)H, (int)D, ns);
}

extern "C" tb_status_t tb_attention_f32(float* out, const float* q, const float* kcache, const float* vcache,
                                        int64_t B, int64_t H, int64_t Hkv, int64_t Sq, int64_t Sk, int64_t D,
                                        int64_t max_seq, float scale, void* workspace, size_t workspace_bytes,
                                        tb_stream_t stream) {
  TB_INJECT("tb_attention_f32");
  TB_REQUIRE(B >= 0 && H > 0 && Hkv > 0 && H % Hkv == 0 && Sq >= 0 && D > 0);
  TB_REQUIRE(Sk >= Sq && Sk <= max_seq);
  if (B == 0 || Sq == 0) return TB_SUCCESS;
  TB_REQUIRE(out && q && kcache && vcache);
  TB_REQUIRE(Sk >= 1);
  TB_REQUIRE(tb::aligned(q, 16) && tb::aligned(kcache, 16) && tb::aligned(vcache, 16));
  cudaStream_t st = (cudaStream_t)stream;
  if (Sq == 1) {
    tb::AttnDecodeArgs a{};
    a.q = q;
    a.kcache = kcache;
    a.vcache = vcache;
    a.out = out;
    a.pos = nullptr;
    a.sk = Sk;
    a.B = (int)B;
    a.H = (int)H;
    a.Hkv = (int)Hkv;
    a.D = (int)D;
    a.max_seq = (int)max_seq;
    a.scale = scale;
    a.nsplit = tb::attn_decode_splits((int)B, (int)H, (int)Hkv, (int)D, max_seq, false);
    TB_REQUIRE(workspace && workspace_bytes >= tb::attn_decode_workspace(a.B, a.H, a.D, a.nsplit));
    a.partial = (float*)workspace;
    return tb::attn_decode(a, st, false);
  }
  return tb::attn_prefill(out, q, kcache, vcache, (int)B, (int)H, (int)Hkv, (int)Sq, Sk, (int)D, (int)max_seq, scale,
                          st);
}

// ---------------------------------------------------------------------------
// Decode attention without a caller workspace: the split-K partials go to a
// library-owned device array instead of a buffer the caller allocates.  The
// array is shared by every call on a GPU and keeps the previous call's
// contents; nothing in it needs to start at zero (every split writes its
// whole partial, empty splits included), but calls that overlap on the GPU
// race on it.
// ---------------------------------------------------------------------------
namespace {

static __device__ __align__(256) unsigned char g_noalloc_attn_scratch[TB_ATTENTION_NOALLOC_SCRATCH_BYTES];

// Device address of the scratch array on the current device.  The host-side
// symbol is only a stand-in for it; the address is looked up on every call
// (a cheap host query), so it stays right after a device reset reloads the
// library's device code at a new address.
tb_status_t noalloc_scratch(void** out) {
  void* p = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_attn_scratch);
  if (e != cudaSuccess) return tb::cuda_fail(e, "cudaGetSymbolAddress(g_noalloc_attn_scratch)");
  *out = p;
  return TB_SUCCESS;
}

}  // namespace

extern "C" tb_status_t tb_attention_decode_noalloc_f32(float* out, const float* q, const float* kcache,
                                                       const float* vcache, int64_t B, int64_t H, int64_t Hkv,
                                                       int64_t Sk, int64_t D, int64_t max_seq, float scale,
                                                       tb_stream_t stream) {
  TB_INJECT("tb_attention_decode_noalloc_f32");
  TB_REQUIRE(B >= 0 && H > 0 && Hkv > 0 && H % Hkv == 0 && D > 0);
  TB_REQUIRE(Sk >= 1 && Sk <= max_seq);
  TB_REQUIRE(B <= 0x7fffffff && H <= 0x7fffffff && max_seq <= 0x7fffffff);
  if (B == 0) return TB_SUCCESS;
  TB_REQUIRE(out && q && kcache && vcache);
  TB_REQUIRE(tb::aligned(q, 16) && tb::aligned(kcache, 16) && tb::aligned(vcache, 16));
  // As many splits as the caller-workspace path would use, capped by what
  // fits in the scratch array; a single split that does not fit is rejected.
  const size_t per_split = (size_t)B * H * (D + 2) * sizeof(float);
  TB_REQUIRE(per_split <= TB_ATTENTION_NOALLOC_SCRATCH_BYTES);
  int nsplit = tb::attn_decode_splits((int)B, (int)H, (int)Hkv, (int)D, max_seq, false);
  const int fit = (int)(TB_ATTENTION_NOALLOC_SCRATCH_BYTES / per_split);
  if (nsplit > fit) nsplit = fit;
  void* scratch = nullptr;
  TB_TRY(noalloc_scratch(&scratch));
  tb::AttnDecodeArgs a{};
  a.q = q;
  a.kcache = kcache;
  a.vcache = vcache;
  a.out = out;
  a.partial = (float*)scratch;
  a.pos = nullptr;
  a.sk = Sk;
  a.B = (int)B;
  a.H = (int)H;
  a.Hkv = (int)Hkv;
  a.D = (int)D;
  a.max_seq = (int)max_seq;
  a.nsplit = nsplit;
  a.scale = scale;
  return tb::attn_decode(a, (cudaStream_t)stream, false);
}
