// sample.cu — temperature / top-k / top-p sampling on the device, so a
// generation loop never copies a [V] logit row to the host per token.
//
// One CTA per row restates Sampler.Sample (models/sampling.go:47-70) step by
// step, in the reference's arithmetic:
//   temperature   x /= T when T != 1 and T > 0 (fp32 division);
//   top-k         the k-th largest value by value (findKthLargest, :163-186)
//                 — an exact 4-pass 8-bit radix select on order-preserving
//                 keys — and x < threshold -> -inf (ties at the threshold stay);
//   top-p         softmax (max, float32(exp(float64(x - max))), fp32 sum in
//                 index order, division), candidates sorted by probability
//                 descending with ties in index order (sortIndicesByValue's
//                 stable insertion sort, :188-197), fp32 cumulative sum in that
//                 order up to the first value >= P; the rest -> -inf;
//   sample        softmax again, then the first index whose fp32 cumulative
//                 sum (index order) exceeds the caller's uniform r, else V - 1
//                 (sampleFromProbs, :124-134).
// The sums that the reference accumulates sequentially are accumulated by
// one thread over the finite entries in index order (the -inf entries add
// exact zeros), so they round exactly as the reference's loops do.
// Limits: V <= 40000; top-p needs at most 4096 finite candidates after top-k
// (otherwise the row reports unsupported in *unsupported and returns V - 1).
#include <math.h>
#include <stdint.h>

#include <mutex>

#include "common.cuh"
#include "kernels.h"

namespace tb {
namespace {

constexpr int kSmpThreads = 1024;
constexpr int kSmpMaxV = 40000;
constexpr int kSmpMaxCand = 4096;

__device__ __forceinline__ uint32_t ord_key(float v) {
  const uint32_t b = __float_as_uint(v);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

__device__ float block_max(float v, float* red) {
  v = warp_max(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float m = -INFINITY;
  for (int w = 0; w < kSmpThreads / 32; w++) m = fmaxf(m, red[w]);
  return m;
}

// Ordered compaction of the finite entries of x into idx (index order);
// returns their count (all threads).
__device__ int compact_finite(const float* x, int V, int* idx, int cap, int* scan) {
  const int t = threadIdx.x;
  const int per = (V + kSmpThreads - 1) / kSmpThreads;
  const int i0 = t * per, i1 = min(V, i0 + per);
  int c = 0;
  for (int i = i0; i < i1; i++) c += x[i] != -INFINITY;
  __syncthreads();
  scan[t] = c;
  __syncthreads();
  if (t == 0) {
    int run = 0;
    for (int k = 0; k < kSmpThreads; k++) {
      const int v = scan[k];
      scan[k] = run;
      run += v;
    }
    scan[kSmpThreads] = run;
  }
  __syncthreads();
  int o = scan[t];
  for (int i = i0; i < i1; i++)
    if (x[i] != -INFINITY) {
      if (o < cap) idx[o] = i;
      o++;
    }
  __syncthreads();
  return scan[kSmpThreads];
}

__global__ void __launch_bounds__(kSmpThreads) sample_kernel(int64_t* tokens, const float* __restrict__ logits,
                                                              const float* __restrict__ uniforms, int V, float T,
                                                              int K, float P, int* unsupported) {
  extern __shared__ float x[];                               // [V]
  int* idx = reinterpret_cast<int*>(x + V);                  // [kSmpMaxCand]
  float* e = reinterpret_cast<float*>(idx + kSmpMaxCand);    // [kSmpMaxCand]
  unsigned long long* keys = reinterpret_cast<unsigned long long*>(e + kSmpMaxCand);  // [kSmpMaxCand]
  __shared__ int scan[kSmpThreads + 1];
  __shared__ float red[kSmpThreads / 32];
  __shared__ unsigned int hist[256];
  __shared__ uint32_t sel[2];
  __shared__ int cutoff_s, bad_s;
  const int b = blockIdx.x, t = threadIdx.x;
  const float* row = logits + (size_t)b * V;
  const bool temp = T != 1.0f && T > 0.0f;
  for (int i = t; i < V; i += kSmpThreads) x[i] = temp ? __fdiv_rn(row[i], T) : row[i];
  if (t == 0) bad_s = 0;
  __syncthreads();

  // top-k: exact k-th largest value, 8 bits of the order-preserving key at a time
  if (K > 0 && K < V) {
    uint32_t prefix = 0, mask = 0;
    int k = K;
    for (int shift = 24; shift >= 0; shift -= 8) {
      for (int i = t; i < 256; i += kSmpThreads) hist[i] = 0u;
      __syncthreads();
      for (int i = t; i < V; i += kSmpThreads) {
        const uint32_t key = ord_key(x[i]);
        if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 255u], 1u);
      }
      __syncthreads();
      if (t == 0) {
        int digit = 255;
        for (; digit > 0; digit--) {
          if ((int)hist[digit] >= k) break;
          k -= (int)hist[digit];
        }
        sel[0] = prefix | ((uint32_t)digit << shift);
        sel[1] = (uint32_t)k;
      }
      __syncthreads();
      prefix = sel[0];
      k = (int)sel[1];
      mask |= 255u << shift;
      __syncthreads();
    }
    // prefix is now the key of the k-th largest value; compare as floats, as
    // the reference does (-0 and +0 are equal there)
    const float thr = __uint_as_float((prefix & 0x80000000u) ? (prefix & 0x7FFFFFFFu) : ~prefix);
    for (int i = t; i < V; i += kSmpThreads)
      if (x[i] < thr) x[i] = -INFINITY;
    __syncthreads();
  }

  // top-p
  if (P > 0.0f && P < 1.0f) {
    float m = -INFINITY;
    for (int i = t; i < V; i += kSmpThreads) m = fmaxf(m, x[i]);
    m = block_max(m, red);
    const int n = compact_finite(x, V, idx, kSmpMaxCand, scan);
    if (n > kSmpMaxCand) {
      if (t == 0) bad_s = 1;
    } else {
      for (int c = t; c < n; c += kSmpThreads) e[c] = (float)exp((double)(x[idx[c]] - m));
      __syncthreads();
      if (t == 0) {  // fp32 sum in index order (the -inf entries add zeros)
        float s = 0.f;
        for (int c = 0; c < n; c++) s = __fadd_rn(s, e[c]);
        red[0] = s;
      }
      __syncthreads();
      const float sum = red[0];
      int np2 = 1;
      while (np2 < n) np2 <<= 1;
      for (int c = t; c < np2; c += kSmpThreads) {
        if (c < n) {
          const float p = __fdiv_rn(e[c], sum);
          // candidates are in index order: a lower position is a lower index
          keys[c] = ((unsigned long long)ord_key(p) << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)c);
        } else {
          keys[c] = 0ull;
        }
      }
      __syncthreads();
      // bitonic sort, descending: probability first, then lower index first
      for (int size = 2; size <= np2; size <<= 1)
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
          for (int c = t; c < np2; c += kSmpThreads) {
            const int o = c ^ stride;
            if (o > c) {
              const bool desc = (c & size) == 0;
              const unsigned long long a = keys[c], bb = keys[o];
              if (desc ? (a < bb) : (a > bb)) {
                keys[c] = bb;
                keys[o] = a;
              }
            }
          }
          __syncthreads();
        }
      if (t == 0) {
        float cs = 0.f;
        int cut = 0;
        for (int c = 0; c < n; c++) {
          const int pc = (int)(0xFFFFFFFFu - (uint32_t)(keys[c] & 0xFFFFFFFFull));
          cs = __fadd_rn(cs, __fdiv_rn(e[pc], sum));
          if (cs >= P) {
            cut = c + 1;
            break;
          }
        }
        cutoff_s = cut;
      }
      __syncthreads();
      for (int c = cutoff_s + t; c < n; c += kSmpThreads) {
        const int pc = (int)(0xFFFFFFFFu - (uint32_t)(keys[c] & 0xFFFFFFFFull));
        x[idx[pc]] = -INFINITY;
      }
      if (cutoff_s == 0)  // the reference masks every token when the sum never reaches P
        for (int i = t; i < V; i += kSmpThreads) x[i] = -INFINITY;
      __syncthreads();
    }
  }

  // softmax + inverse CDF in index order: the exponentials in parallel (x
  // becomes e, zero where masked), the reference's two sequential sums on one
  // thread over the non-zero terms (a zero term changes neither the sum nor
  // the comparison with r)
  float m = -INFINITY;
  for (int i = t; i < V; i += kSmpThreads) m = fmaxf(m, x[i]);
  m = block_max(m, red);
  __syncthreads();
  if (m != -INFINITY)
    for (int i = t; i < V; i += kSmpThreads) x[i] = x[i] == -INFINITY ? 0.f : (float)exp((double)(x[i] - m));
  __syncthreads();
  if (t == 0) {
    int64_t tok = V - 1;
    if (bad_s) {
      atomicAdd(unsupported, 1);
    } else if (m != -INFINITY) {
      float s = 0.f;
      for (int i = 0; i < V; i++)
        if (x[i] != 0.f) s = __fadd_rn(s, x[i]);
      const float r = uniforms[b];
      float cs = 0.f;
      for (int i = 0; i < V; i++) {
        if (x[i] == 0.f) continue;
        cs = __fadd_rn(cs, __fdiv_rn(x[i], s));
        if (r < cs) {
          tok = i;
          break;
        }
      }
    }
    tokens[b] = tok;
  }
}

size_t sample_smem(int V) { return (size_t)V * 4 + (size_t)kSmpMaxCand * (4 + 4 + 8); }

}  // namespace
}  // namespace tb

extern "C" tb_status_t tb_sample_f32(int64_t* tokens, const float* logits, const float* uniforms, int64_t B, int64_t V,
                                     float temperature, int64_t top_k, float top_p, int32_t* unsupported,
                                     tb_stream_t stream) {
  TB_INJECT("tb_sample_f32");
  TB_REQUIRE(B >= 0 && V >= 1 && V <= tb::kSmpMaxV && top_k >= 0 && B <= 0x7fffffff);
  if (B == 0) return TB_SUCCESS;
  TB_REQUIRE(tokens && logits && uniforms && unsupported);
  const size_t smem = tb::sample_smem((int)V);
  static std::once_flag once;
  static cudaError_t attr = cudaSuccess;
  std::call_once(once, [] {
    attr = cudaFuncSetAttribute(tb::sample_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)tb::sample_smem(tb::kSmpMaxV));
  });
  if (attr != cudaSuccess) return tb::cuda_fail(attr, "cudaFuncSetAttribute(sample_kernel)");
  const int K = top_k > V ? (int)V : (int)top_k;
  tb::sample_kernel<<<(unsigned)B, tb::kSmpThreads, smem, (cudaStream_t)stream>>>(tokens, logits, uniforms, (int)V,
                                                                                   temperature, K, top_p, unsupported);
  return tb::check_launch("sample_kernel");
}
