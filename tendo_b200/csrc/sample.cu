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
//                 index order, division), every candidate in order of
//                 probability descending with ties in index order
//                 (sortIndicesByValue's stable insertion sort, :188-197),
//                 fp32 cumulative sum in that order up to the first value
//                 >= P; the rest -> -inf.  The order is produced kSmpBatch
//                 candidates at a time: an exact radix select finds the
//                 batch's smallest key among the candidates below the previous
//                 batch, a bitonic sort orders the batch, and the running sum
//                 continues through it, so any number of candidates is served;
//   sample        softmax again, then the first index whose fp32 cumulative
//                 sum (index order) exceeds the caller's uniform r, else V - 1
//                 (sampleFromProbs, :124-134).
// The sums that the reference accumulates sequentially are accumulated by
// one thread over the finite entries in index order (the -inf entries add
// exact zeros), so they round exactly as the reference's loops do.
// Limit: V <= 40000 (the row lives in shared memory; the candidate keys carry
// the index in 16 bits).
#include <math.h>
#include <stdint.h>

#include <mutex>

#include "common.cuh"
#include "kernels.h"

namespace tb {
namespace {

constexpr int kSmpThreads = 1024;
constexpr int kSmpMaxV = 40000;  // 16-bit index field of the candidate keys
constexpr int kSmpBatch = 4096;  // candidates sorted at a time by top-p

__device__ __forceinline__ uint32_t ord_key(float v) {
  const uint32_t b = __float_as_uint(v);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float ord_value(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k);
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

// Candidate key of token i whose probability has order key pk (> 0): larger
// keys come first in sortIndicesByValue's order (probability descending,
// ties in index order).
__device__ __forceinline__ unsigned long long cand_key(uint32_t pk, int i) {
  return ((unsigned long long)pk << 16) | (unsigned long long)(0xFFFFu - (uint32_t)i);
}

__global__ void __launch_bounds__(kSmpThreads) sample_kernel(int64_t* tokens, const float* __restrict__ logits,
                                                              const float* __restrict__ uniforms, int V, float T,
                                                              int K, float P) {
  // x[V]: the row (temperature, top-k); during top-p the probabilities' order
  // keys (0 for a zero probability), afterwards the masked row again
  extern __shared__ float x[];
  unsigned long long* batch = reinterpret_cast<unsigned long long*>(x + ((V + 1) & ~1));  // [kSmpBatch]
  uint32_t* xk = reinterpret_cast<uint32_t*>(x);
  __shared__ float red[kSmpThreads / 32];
  __shared__ unsigned int hist[256];
  __shared__ unsigned long long sel_s;
  __shared__ int k_s, cnt_s, done_s;
  __shared__ float thr_k_s, sum_s;
  __shared__ unsigned long long cut_s;
  const int b = blockIdx.x, t = threadIdx.x;
  const float* row = logits + (size_t)b * V;
  const bool temp = T != 1.0f && T > 0.0f;
  for (int i = t; i < V; i += kSmpThreads) x[i] = temp ? __fdiv_rn(row[i], T) : row[i];
  if (t == 0) thr_k_s = -INFINITY;
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
        sel_s = prefix | ((uint32_t)digit << shift);
        k_s = k;
      }
      __syncthreads();
      prefix = (uint32_t)sel_s;
      k = k_s;
      mask |= 255u << shift;
      __syncthreads();
    }
    // prefix is now the key of the k-th largest value; compare as floats, as
    // the reference does (-0 and +0 are equal there)
    const float thr = ord_value(prefix);
    for (int i = t; i < V; i += kSmpThreads)
      if (x[i] < thr) x[i] = -INFINITY;
    if (t == 0) thr_k_s = thr;
    __syncthreads();
  }

  // top-p over every candidate: probabilities as the reference's softmax
  // computes them, then the candidates in sortIndicesByValue's order, kSmpBatch
  // at a time (an exact radix select of the batch's smallest key, a bitonic
  // sort of the batch), with the fp32 cumulative sum carried on one thread
  // across batches until it first reaches P
  const bool topp = P > 0.0f && P < 1.0f;
  if (topp) {
    float m = -INFINITY;
    for (int i = t; i < V; i += kSmpThreads) m = fmaxf(m, x[i]);
    m = block_max(m, red);
    // exponentials in parallel; the -inf entries become exact zeros
    for (int i = t; i < V; i += kSmpThreads) x[i] = x[i] == -INFINITY ? 0.f : (float)exp((double)(x[i] - m));
    __syncthreads();
    if (t == 0) {  // fp32 sum in index order (a zero term changes nothing)
      float s = 0.f;
      for (int i = 0; i < V; i++)
        if (x[i] != 0.f) s = __fadd_rn(s, x[i]);
      sum_s = s;
    }
    __syncthreads();
    const float sum = sum_s;
    int npos = 0;
    for (int i = t; i < V; i += kSmpThreads) {
      const float p = x[i] != 0.f ? __fdiv_rn(x[i], sum) : 0.f;
      xk[i] = p > 0.f ? ord_key(p) : 0u;
      npos += p > 0.f;
    }
    if (t == 0) cnt_s = 0;
    __syncthreads();
    atomicAdd(&cnt_s, npos);
    if (t == 0) {
      done_s = 0;
      cut_s = ~0ull;  // keeps nothing unless the sum reaches P
    }
    __syncthreads();
    int remaining = cnt_s;
    unsigned long long prev = 1ull << 48;  // every candidate key is below it
    float cs = 0.f;                        // thread 0's running sum
    while (remaining > 0) {
      const int nb = remaining < kSmpBatch ? remaining : kSmpBatch;
      // the nb-th largest key below prev (all of them when they fit a batch)
      unsigned long long lo = 0ull;
      if (nb < remaining) {
        unsigned long long prefix = 0ull, mask = 0ull;
        int k = nb;
        for (int shift = 40; shift >= 0; shift -= 8) {
          for (int i = t; i < 256; i += kSmpThreads) hist[i] = 0u;
          __syncthreads();
          for (int i = t; i < V; i += kSmpThreads) {
            if (xk[i] == 0u) continue;
            const unsigned long long key = cand_key(xk[i], i);
            if (key < prev && (key & mask) == prefix) atomicAdd(&hist[(unsigned)(key >> shift) & 255u], 1u);
          }
          __syncthreads();
          if (t == 0) {
            int digit = 255;
            for (; digit > 0; digit--) {
              if ((int)hist[digit] >= k) break;
              k -= (int)hist[digit];
            }
            sel_s = prefix | ((unsigned long long)digit << shift);
            k_s = k;
          }
          __syncthreads();
          prefix = sel_s;
          k = k_s;
          mask |= 255ull << shift;
          __syncthreads();
        }
        lo = prefix;  // keys are distinct: exactly nb candidates lie in [lo, prev)
      }
      if (t == 0) cnt_s = 0;
      __syncthreads();
      for (int i = t; i < V; i += kSmpThreads) {
        if (xk[i] == 0u) continue;
        const unsigned long long key = cand_key(xk[i], i);
        if (key < prev && key >= lo) batch[atomicAdd(&cnt_s, 1)] = key;
      }
      int np2 = 1;
      while (np2 < nb) np2 <<= 1;
      __syncthreads();
      for (int c = nb + t; c < np2; c += kSmpThreads) batch[c] = 0ull;
      __syncthreads();
      // bitonic sort, descending
      for (int size = 2; size <= np2; size <<= 1)
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
          for (int c = t; c < np2; c += kSmpThreads) {
            const int o = c ^ stride;
            if (o > c) {
              const bool desc = (c & size) == 0;
              const unsigned long long a = batch[c], bb = batch[o];
              if (desc ? (a < bb) : (a > bb)) {
                batch[c] = bb;
                batch[o] = a;
              }
            }
          }
          __syncthreads();
        }
      if (t == 0) {
        for (int c = 0; c < nb; c++) {
          cs = __fadd_rn(cs, ord_value((uint32_t)(batch[c] >> 16)));
          if (cs >= P) {
            cut_s = batch[c];
            done_s = 1;
            break;
          }
        }
      }
      __syncthreads();
      if (done_s) break;
      remaining -= nb;
      prev = batch[nb - 1];
      __syncthreads();  // the next batch overwrites batch[]
    }
    // the row again, masked by top-k and top-p: a token stays when its key is
    // at or above the cutoff's (the reference masks every token when the sum
    // never reaches P)
    const unsigned long long cut = cut_s;
    const float thr_k = thr_k_s;
    for (int i = t; i < V; i += kSmpThreads) {
      const uint32_t pk = xk[i];
      float v = temp ? __fdiv_rn(row[i], T) : row[i];
      if (v < thr_k || pk == 0u || cand_key(pk, i) < cut) v = -INFINITY;
      x[i] = v;
    }
    __syncthreads();
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
    if (m != -INFINITY) {
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

size_t sample_smem(int V) { return (size_t)((V + 1) & ~1) * 4 + (size_t)kSmpBatch * 8; }

}  // namespace
}  // namespace tb

extern "C" tb_status_t tb_sample_f32(int64_t* tokens, const float* logits, const float* uniforms, int64_t B, int64_t V,
                                     float temperature, int64_t top_k, float top_p, tb_stream_t stream) {
  TB_INJECT("tb_sample_f32");
  TB_REQUIRE(B >= 0 && V >= 1 && V <= tb::kSmpMaxV && top_k >= 0 && B <= 0x7fffffff);
  if (B == 0) return TB_SUCCESS;
  TB_REQUIRE(tokens && logits && uniforms);
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
                                                                                   temperature, K, top_p);
  return tb::check_launch("sample_kernel");
}
