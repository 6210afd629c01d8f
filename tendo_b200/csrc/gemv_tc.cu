// gemv_tc.cu — the decode-regime quantized Linear (1 <= M <= 64) on the
// 5th-generation tensor cores, for the microbench and C-ABI callers.
//
// out[M, N] = x[M, K] @ (q * scale)^T (+ resid), q int8 [N, K] as stored.
//
// x is split into three int8 digit rows per batch row,
//   x[m] = s_m (d0 + d1 / 128 + d2 / 128^2),   s_m = max_k |x[m, k]| / 127,
// and every digit row times the raw weight bytes is an exact s32 sum
// (tcgen05.mma kind::i8).  The MMA runs "swapped": the weights are the
// 128-row A operand and the 3M digit rows (padded to ND, a multiple of 16)
// the N side, so a tile is 128 weight rows x ND digit columns in TMEM and the
// weight stream — the only large operand — moves in 16 KB TMA boxes.
//
// Work split ("stream-K"): the tile-major space of (weight tile, 128-byte
// K block) iterations is cut into gridDim.x equal contiguous ranges, one per
// CTA (one CTA per SM), so every SM streams the same number of weight bytes
// whatever N and K are.  A tile whose K blocks span several CTAs is summed in
// the workspace with integer reductions (red.add: exact, order-free); the
// last CTA to count itself in finishes the tile and zeroes its slots again.
//
// Warps: 0 = TMA producer, 1 = MMA issuer (4 x tcgen05.mma per 128-byte K
// block into one of two TMEM accumulators), 2..5 = epilogue (one weight row
// per thread: its TMEM lane).  A digit kernel writes the digit rows (with the
// RMSNorm when the caller fuses one) and the producer loads them with TMA.
// The producer starts the weight stream before the programmatic-launch wait:
// weights never depend on the preceding kernel.
#include <string.h>

#include <mutex>

#include "common.cuh"
#include "kernels.h"
#include "tc_common.cuh"
#include "tma_common.cuh"

namespace tb {
namespace {

constexpr int kGvRows = 128;               // weight rows per tile (MMA M)
constexpr int kGvSub = 128;                // K bytes of one 128-byte-swizzled sub-tile
constexpr int kGvWSub = kGvRows * kGvSub;  // 16 KB: 128 weight rows x 128 bytes
constexpr int kGvTmemCols = 512;           // two accumulators of up to 256 columns (ND <= 192)

struct GvArgs {
  float* out;
  const float* srow;    // TMA digits: row scales written by the digit kernel
  const float* scale;
  const float* resid;
  int* acc;             // [tiles][ND][128] s32 sums of split tiles (zero between launches)
  unsigned int* count;  // [tiles] CTAs done with a split tile (zero between launches)
  float* part;          // per-group scales: [grid][2][M][128] fp32 partial rows of split tiles
  int M, N, K, ND, KB, total, stages;
  int gs, ngroups;      // per-group scales: 128-byte sub-tiles per group, groups per row
  int* err;
};

// CTA whose iteration range holds iteration `it` (ranges: floor(b T / G)).
__device__ __forceinline__ int owner_of(long long it, long long total, long long grid) {
  return (int)(((it + 1) * grid + total - 1) / total) - 1;
}
__device__ __forceinline__ int range_begin(long long b, long long total, long long grid) {
  return (int)(b * total / grid);
}

__device__ __forceinline__ void epi_sync() { asm volatile("bar.sync 2, 128;" ::: "memory"); }

// GKB 128-byte K sub-tiles per stage (one 3-D TMA box of 128 rows x GKB x 128
// bytes for the weights: longer runs per row, fewer copies).
//
// GRP: per-group scales [N, K / group] (group a multiple of 128).  The MMA
// hands an accumulator to the epilogue at every group boundary (and at the
// end of a tile segment, which may cut a group: the scale is linear), the
// epilogue scales each group's exact s32 sums by scale[n, group] and adds them
// into fp32 rows in shared memory.  A split tile's fp32 partial rows go to the
// CTA's own workspace slots; the last CTA to count in adds them in CTA order,
// so the sum does not depend on arrival order.
template <int GKB, bool GRP>
__global__ void __launch_bounds__(192, 1)
    gemv_tc_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX, GvArgs a) {
  constexpr int kGvBK = kGvSub * GKB;     // K bytes per stage
  constexpr int kGvWTile = kGvWSub * GKB;  // weight bytes per stage
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
  const int S = a.stages;
  const int stage_bytes = kGvWTile + a.ND * kGvBK;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)S * stage_bytes);
  uint64_t* empty = full + S;
  uint64_t* tfull = empty + S;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* last_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* accs = reinterpret_cast<float*>(smem + (size_t)S * stage_bytes + 512);  // GRP: [ND][128]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long T = a.total, G = gridDim.x;
  const int b0 = range_begin(blockIdx.x, T, G), b1 = range_begin(blockIdx.x + 1, T, G);
  const int KB = a.KB, M = a.M, ND = a.ND;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; s++) {
      mbarrier_init(&full[s], 1);
      mbarrier_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; b++) {
      mbarrier_init(&tfull[b], 1);
      mbarrier_init(&tempty[b], 4);  // one arrival per epilogue warp
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmW)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmX)) : "memory");
  }
  if (warp == 0) tmem_alloc(tmem_slot, kGvTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_launch_dependents();

  if (warp == 0) {
    if (lane == 0) {
      // producer; with TMA digits, the digit boxes of the first stages go out
      // after the programmatic-launch wait, behind the weight boxes
      const int n = b1 - b0;
      const int pre = n < S ? n : S;
      for (int i = 0; i < pre; i++) {
        const int it = b0 + i;
        mbarrier_expect_tx(&full[i], (uint32_t)stage_bytes);
        tma_load_3d(smem + (size_t)i * stage_bytes, &tmW, 0, (it / KB) * kGvRows, (it % KB) * GKB, &full[i]);
      }
      {
        pdl_wait();
        for (int i = 0; i < pre; i++)
          for (int g = 0; g < GKB; g++)
            tma_load_2d(smem + (size_t)i * stage_bytes + kGvWTile + g * ND * kGvSub, &tmX,
                        ((b0 + i) % KB) * kGvBK + g * kGvSub, 0, &full[i]);
      }
      for (int i = pre; i < n; i++) {
        const int s = i % S, use = i / S;
        const int it = b0 + i, kb = it % KB;
        mbarrier_wait(&empty[s], (uint32_t)((use - 1) & 1), a.err);
        unsigned char* st = smem + (size_t)s * stage_bytes;
        mbarrier_expect_tx(&full[s], (uint32_t)stage_bytes);
        tma_load_3d(st, &tmW, 0, (it / KB) * kGvRows, kb * GKB, &full[s]);
        for (int g = 0; g < GKB; g++)
            tma_load_2d(st + kGvWTile + g * ND * kGvSub, &tmX, kb * kGvBK + g * kGvSub, 0, &full[s]);
      }
    }
  } else if (warp == 1) {
    if (GRP && lane == 0) {
      // MMA issuer, per-group scales: one accumulator per (group, segment)
      // piece, alternating buffers; h counts the hand-offs
      const uint32_t idesc = idesc_i8(kGvRows, ND);
      int i = 0, h = 0;
      for (int it = b0; it < b1;) {
        const int tstart = (it / KB) * KB;
        const int seg_end = min(b1, tstart + KB);
        int j = (it - tstart) * GKB;  // 128-byte sub-tile within the tile
        bool open = false;
        uint32_t d = tmem;
        for (; it < seg_end; it++, i++) {
          const int s = i % S, use = i / S;
          mbarrier_wait(&full[s], (uint32_t)(use & 1), a.err);
          tc_fence_after();
          const uint32_t w0 = smem_addr(smem + (size_t)s * stage_bytes), x0 = w0 + kGvWTile;
#pragma unroll
          for (int g = 0; g < GKB; g++, j++) {
            const bool first = !open;
            if (!open) {
              const int buf = h & 1;
              if (h >= 2) mbarrier_wait(&tempty[buf], (uint32_t)(((h - 2) >> 1) & 1), a.err);
              tc_fence_after();
              d = tmem + (uint32_t)(buf * 256);
              open = true;
            }
#pragma unroll
            for (int kk = 0; kk < kGvSub / 32; kk++)
              tc_mma_i8(d, sw128_desc(w0 + g * kGvRows * kGvSub + kk * 32), sw128_desc(x0 + g * ND * kGvSub + kk * 32),
                        idesc, !(first && kk == 0));
            if ((j + 1) % a.gs == 0 || (it + 1 == seg_end && g == GKB - 1)) {
              tc_commit(&tfull[h & 1]);
              h++;
              open = false;
            }
          }
          tc_commit(&empty[s]);
        }
      }
    } else if (lane == 0) {
      // MMA issuer: one accumulator per tile segment, alternating buffers
      const uint32_t idesc = idesc_i8(kGvRows, ND);
      int i = 0, seg = 0;
      for (int it = b0; it < b1; seg++) {
        const int seg_end = min(b1, (it / KB + 1) * KB);
        const int buf = seg & 1;
        if (seg >= 2) mbarrier_wait(&tempty[buf], (uint32_t)(((seg - 2) >> 1) & 1), a.err);
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(buf * 256);
        for (int first = 1; it < seg_end; it++, i++, first = 0) {
          const int s = i % S, use = i / S;
          mbarrier_wait(&full[s], (uint32_t)(use & 1), a.err);
          tc_fence_after();
          const uint32_t w0 = smem_addr(smem + (size_t)s * stage_bytes), x0 = w0 + kGvWTile;
#pragma unroll
          for (int g = 0; g < GKB; g++)
#pragma unroll
            for (int kk = 0; kk < kGvSub / 32; kk++)
              tc_mma_i8(d, sw128_desc(w0 + g * kGvRows * kGvSub + kk * 32), sw128_desc(x0 + g * ND * kGvSub + kk * 32),
                        idesc, !(first && g == 0 && kk == 0));
          tc_commit(&empty[s]);
        }
        tc_commit(&tfull[buf]);
      }
    }
  } else if (warp < 6) {
    // epilogue: thread = weight row (tile row 32 q + lane = its TMEM lane)
    const int q = warp & 3;
    const int rowt = q * 32 + lane;
    const float* srow = a.srow;
    if (GRP) {
      // fp32 sums per accumulator column (digit row p M + m) of this thread's
      // weight row; distinct columns, so a 16-column chunk is read, updated
      // and written back as a batch
      float* acc_r = accs + rowt;  // [ND][128]
      for (int c = 0; c < ND; c++) acc_r[c * kGvRows] = 0.f;
      const int nd3 = 3 * M, ncol = (nd3 + 15) & ~15;
      // the scale of each hand-off is loaded one hand-off ahead
      auto scale_of = [&](int tile_, int grp_) {
        const int nn = tile_ * kGvRows + rowt;
        return nn < a.N ? __ldg(a.scale + (size_t)nn * a.ngroups + grp_) : 0.f;
      };
      // out[m, n] = srow[m] y[m] (+ resid) for rows m0 .. m0 + 7
      auto emit = [&](int m0, const float* y, int n) {
        float sr[8], rs[8];
#pragma unroll
        for (int mm = 0; mm < 8; mm++) {
          const int m = m0 + mm < M ? m0 + mm : M - 1;
          sr[mm] = __ldcg(srow + m);
          rs[mm] = a.resid ? __ldcg(a.resid + (size_t)m * a.N + n) : 0.f;
        }
#pragma unroll
        for (int mm = 0; mm < 8; mm++)
          if (m0 + mm < M) a.out[(size_t)(m0 + mm) * a.N + n] = a.resid ? sr[mm] * y[mm] + rs[mm] : sr[mm] * y[mm];
      };
      float sg_next = scale_of(b0 / KB, ((b0 % KB) * GKB) / a.gs);
      int h = 0;
      for (int it = b0; it < b1;) {
        const int tile = it / KB;
        const int tstart = tile * KB, tend = tstart + KB;
        const int seg_end = min(b1, tend);
        const int n = tile * kGvRows + rowt;
        const bool live = n < a.N;
        for (int j = (it - tstart) * GKB, je = (seg_end - tstart) * GKB; j < je; h++) {
          const int grp = j / a.gs;
          const int jn = min(je, (grp + 1) * a.gs);
          const int buf = h & 1;
          const float sg = sg_next;
          if (jn < je)
            sg_next = scale_of(tile, jn / a.gs);
          else if (seg_end < b1)
            sg_next = scale_of(tile + 1, 0);
          mbarrier_wait(&tfull[buf], (uint32_t)((h >> 1) & 1), a.err);
          __syncwarp();
          tc_fence_after();
          const uint32_t tb = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * 256);
          for (int j0 = 0; j0 < ncol; j0 += 16) {
            uint32_t v[16];
            tmem_ld16(tb + j0, v);
            tmem_wait_ld();
            pin16(v);
            float* ac = acc_r + j0 * kGvRows;
            float t[16];
#pragma unroll
            for (int c = 0; c < 16; c++) t[c] = ac[c * kGvRows];
#pragma unroll
            for (int c = 0; c < 16; c++) ac[c * kGvRows] = __fmaf_rn((float)(int)v[c], sg, t[c]);
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbarrier_arrive(&tempty[buf]);
          j = jn;
        }
        // y[m] = a0 + a1 / 128 + a2 / 128^2 over this segment; columns re-zeroed
        auto seg_sum = [&](int m) {
          const float y = acc_r[m * kGvRows] + acc_r[(M + m) * kGvRows] * (1.0f / 128.0f) +
                          acc_r[(2 * M + m) * kGvRows] * (1.0f / 16384.0f);
          return y;
        };
        const int c0 = owner_of(tstart, T, G), c1 = owner_of(tend - 1, T, G);
        if (c0 == c1) {
          for (int m0 = 0; m0 < M; m0 += 8) {
            float y[8];
#pragma unroll
            for (int mm = 0; mm < 8; mm++) y[mm] = m0 + mm < M ? seg_sum(m0 + mm) : 0.f;
            if (live) emit(m0, y, n);
          }
        } else {
          // split tile: this CTA's slot 0 is its first segment, slot 1 its last
          const int slot = tile == b0 / KB ? 0 : 1;
          float* ps = a.part + ((size_t)(blockIdx.x * 2 + slot) * M) * kGvRows + rowt;
          for (int m = 0; m < M; m++) ps[(size_t)m * kGvRows] = seg_sum(m);
          epi_sync();
          if (threadIdx.x == 64) {
            unsigned int prev;
            asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(prev) : "l"(a.count + tile) : "memory");
            *last_flag = prev == (unsigned int)(c1 - c0) ? 1 : 0;
          }
          epi_sync();
          if (*last_flag) {
            // the contributors' partial rows, added in CTA order
            for (int m0 = 0; m0 < M; m0 += 8) {
              float y[8];
#pragma unroll
              for (int mm = 0; mm < 8; mm++) y[mm] = 0.f;
#pragma unroll 4
              for (int c = c0; c <= c1; c++) {
                const int sl = tile == range_begin(c, T, G) / KB ? 0 : 1;
                const float* pc = a.part + ((size_t)(c * 2 + sl) * M + m0) * kGvRows + rowt;
                float v[8];
#pragma unroll
                for (int mm = 0; mm < 8; mm++) v[mm] = m0 + mm < M ? __ldcg(pc + (size_t)mm * kGvRows) : 0.f;
#pragma unroll
                for (int mm = 0; mm < 8; mm++) y[mm] += v[mm];
              }
              if (live) emit(m0, y, n);
            }
            if (threadIdx.x == 64) a.count[tile] = 0u;
          }
          epi_sync();
        }
        for (int c = 0; c < ncol; c++) acc_r[c * kGvRows] = 0.f;
        it = seg_end;
      }
    } else {
    int seg = 0;
    for (int it = b0; it < b1; seg++) {
      const int tile = it / KB;
      const int tstart = tile * KB, tend = tstart + KB;
      const int seg_end = min(b1, tend);
      const int buf = seg & 1;
      mbarrier_wait(&tfull[buf], (uint32_t)((seg >> 1) & 1), a.err);
      __syncwarp();
      tc_fence_after();
      const uint32_t tb = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * 256);
      const int n = tile * kGvRows + rowt;
      const bool live = n < a.N;
      const float sc = live ? a.scale[n] : 0.f;
      if (owner_of(tstart, T, G) == owner_of(tend - 1, T, G)) {
        // the whole tile is this CTA's: finish it from TMEM
        for (int m = 0; m < M; m++) {
          uint32_t c0 = tmem_ld1(tb + m), c1 = tmem_ld1(tb + M + m), c2 = tmem_ld1(tb + 2 * M + m);
          tmem_wait_ld();
          pin1(c0);
          pin1(c1);
          pin1(c2);
          if (live) {
            const float y = (__ldcg(srow + m)) *
                            ((float)(int)c0 + (float)(int)c1 * (1.0f / 128.0f) + (float)(int)c2 * (1.0f / 16384.0f));
            float o = y * sc;
            if (a.resid) o += __ldcg(a.resid + (size_t)m * a.N + n);
            a.out[(size_t)m * a.N + n] = o;
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbarrier_arrive(&tempty[buf]);
      } else {
        // split tile: add this CTA's sums into the tile's slots, count in; the
        // last CTA to count finishes the tile and zeroes the slots again
        const int nc = owner_of(tend - 1, T, G) - owner_of(tstart, T, G) + 1;
        int* acc = a.acc + (size_t)tile * ND * kGvRows + rowt;
        for (int j0 = 0; j0 < ND; j0 += 16) {
          uint32_t v[16];
          tmem_ld16(tb + j0, v);
          tmem_wait_ld();
          pin16(v);
#pragma unroll
          for (int j = 0; j < 16; j++)
            if (j0 + j < 3 * M) atomicAdd(acc + (size_t)(j0 + j) * kGvRows, (int)v[j]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbarrier_arrive(&tempty[buf]);
        // the CTA barrier orders every thread's reductions before the counter's
        // release; its acquire (and the barrier after it) orders the last
        // CTA's reads after every other CTA's reductions
        epi_sync();
        if (threadIdx.x == 64) {
          unsigned int prev;
          asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(prev) : "l"(a.count + tile) : "memory");
          *last_flag = prev == (unsigned int)(nc - 1) ? 1 : 0;
        }
        epi_sync();
        if (*last_flag) {
          for (int m0 = 0; m0 < M; m0 += 8) {
            int d[3][8];
#pragma unroll
            for (int p = 0; p < 3; p++)
#pragma unroll
              for (int mm = 0; mm < 8; mm++)
                d[p][mm] = (m0 + mm < M) ? __ldcg(acc + (size_t)(p * M + m0 + mm) * kGvRows) : 0;
#pragma unroll
            for (int p = 0; p < 3; p++)
#pragma unroll
              for (int mm = 0; mm < 8; mm++)
                if (m0 + mm < M) acc[(size_t)(p * M + m0 + mm) * kGvRows] = 0;
            // row scales and residuals of the chunk before its first store
            float sr[8], rs[8];
#pragma unroll
            for (int mm = 0; mm < 8; mm++) {
              const int m = m0 + mm < M ? m0 + mm : M - 1;
              sr[mm] = __ldcg(srow + m);
              rs[mm] = (a.resid && live) ? __ldcg(a.resid + (size_t)m * a.N + n) : 0.f;
            }
#pragma unroll
            for (int mm = 0; mm < 8; mm++) {
              const int m = m0 + mm;
              if (m < M && live) {
                const float y = sr[mm] * ((float)d[0][mm] + (float)d[1][mm] * (1.0f / 128.0f) +
                                          (float)d[2][mm] * (1.0f / 16384.0f));
                float o = y * sc;
                if (a.resid) o += rs[mm];
                a.out[(size_t)m * a.N + n] = o;
              }
            }
          }
          if (threadIdx.x == 64) a.count[tile] = 0u;
        }
        epi_sync();
      }
      it = seg_end;
    }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, kGvTmemCols);
}

// Workspace: a zero-maintained part (per-tile counters and split-tile sums:
// zero before a launch, zero again after it) and a scratch part for the
// digit rows and row scales.
struct GvLayout {
  size_t count, acc, zeroed, dig, srow, part, scratch;
};

// per-group scales add the split tiles' fp32 partial rows: two slots of
// M x 128 per CTA (at most one CTA per SM)
GvLayout gv_layout(int64_t M, int64_t N, int64_t K, int64_t group = 0) {
  const int64_t ND = ((3 * M + 15) / 16) * 16;
  const int64_t tiles = (N + kGvRows - 1) / kGvRows;
  GvLayout L;
  L.count = 0;
  L.acc = ((size_t)tiles * 4 + 255) & ~(size_t)255;
  L.zeroed = L.acc + (((size_t)tiles * ND * kGvRows * 4 + 255) & ~(size_t)255);
  L.dig = 0;
  L.srow = (((size_t)(3 * M * K) + 255) & ~(size_t)255);
  L.part = (L.srow + (size_t)M * 4 + 255) & ~(size_t)255;
  L.scratch = group > 0 ? L.part + (size_t)sm_count() * 2 * M * kGvRows * 4 : L.srow + (size_t)M * 4;
  return L;
}

template <int GKB, bool GRP>
tb_status_t set_gv_smem() {
  static std::once_flag once;
  static cudaError_t err = cudaSuccess;
  std::call_once(once, [] {
    err = cudaFuncSetAttribute(gemv_tc_kernel<GKB, GRP>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
  });
  if (err != cudaSuccess) return cuda_fail(err, "cudaFuncSetAttribute(gemv_tc)");
  return TB_SUCCESS;
}

}  // namespace

size_t gemv_tc_zeroed_bytes(int64_t M, int64_t N, int64_t K) { return gv_layout(M, N, K).zeroed; }
size_t gemv_tc_scratch_bytes(int64_t M, int64_t N, int64_t K, int64_t group) {
  return gv_layout(M, N, K, group).scratch;
}

bool gemv_tc_ok(const void* q, int64_t M, int64_t N, int64_t K, int64_t group) {
  return M >= 1 && M <= kGemvTcMaxM && gemm_tc_ok(q, M, N, K) && K % kGvSub == 0 &&
         (group == 0 || (group > 0 && group % kGvSub == 0 && K % group == 0));
}

namespace {
template <bool GRP>
tb_status_t launch_gv(const cudaLaunchConfig_t& cfg, int G, const CUtensorMap& tw, const CUtensorMap& tx,
                      const GvArgs& a) {
  if (G == 2) {
    TB_TRY((set_gv_smem<2, GRP>()));
    TB_CUDA(cudaLaunchKernelEx(&cfg, gemv_tc_kernel<2, GRP>, tw, tx, a));
  } else {
    TB_TRY((set_gv_smem<1, GRP>()));
    TB_CUDA(cudaLaunchKernelEx(&cfg, gemv_tc_kernel<1, GRP>, tw, tx, a));
  }
  return TB_SUCCESS;
}
}  // namespace

tb_status_t gemv_tc(float* out, const float* x, const int8_t* q, const float* scale, const float* resid, int M, int N,
                    int K, void* zeroed, bool zero_first, void* scratch, cudaStream_t st, const float* norm_w,
                    float eps, int group, bool digits_ready) {
  const GvLayout L = gv_layout(M, N, K, group);
  unsigned char* z = static_cast<unsigned char*>(zeroed);
  unsigned char* w = static_cast<unsigned char*>(scratch);
  // the digit kernel (which also applies the RMSNorm) writes the digit rows
  // for TMA: measured faster at every M than converter warps inside this
  // kernel (M = 8, N = 28672, K = 8192: 49.0 against 88.3 us)
  const int ND = ((3 * M + 15) / 16) * 16;
  const int acc_bytes = group > 0 ? ND * kGvRows * 4 : 0;  // per-group: fp32 column sums
  // two 128-byte sub-tiles per stage where K allows (halves the copies and
  // doubles the contiguous run per weight row), unless the per-group column
  // sums would leave fewer than three such stages
  int G = K % (2 * kGvSub) == 0 ? 2 : 1;
  if (G == 2 && group > 0 && (200 * 1024 - acc_bytes) / (2 * (kGvWSub + ND * kGvSub)) < 3) G = 1;
  const int kGvBK = kGvSub * G;
  const int kGvWTile = kGvWSub * G;
  const int KB = K / kGvBK;
  const int tiles = (N + kGvRows - 1) / kGvRows;
  const int total = tiles * KB;
  int grid = sm_count();
  if (grid > total) grid = total;
  const int stage_bytes = kGvWTile + ND * kGvBK;
  int stages = (200 * 1024 - acc_bytes) / stage_bytes;  // as many weight boxes in flight as fit
  if (stages > 16) stages = 16;
  const size_t smem = (size_t)stages * stage_bytes + 1024 + 512 + acc_bytes;

  EncodeTiledFn enc = encode_tiled();
  if (!enc) return TB_ERROR_NOT_SUPPORTED;
  CUtensorMap tw, tx;
  memset(&tx, 0, sizeof(tx));
  {
    const cuuint64_t dims[3] = {(cuuint64_t)kGvSub, (cuuint64_t)N, (cuuint64_t)(K / kGvSub)};
    const cuuint64_t strides[2] = {(cuuint64_t)K, (cuuint64_t)kGvSub};
    const cuuint32_t box[3] = {kGvSub, kGvRows, (cuuint32_t)G};
    const cuuint32_t es[3] = {1, 1, 1};
    if (enc(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<int8_t*>(q), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return TB_ERROR_NOT_SUPPORTED;
  }
  int8_t* dig = reinterpret_cast<int8_t*>(w + L.dig);
  float* srow = reinterpret_cast<float*>(w + L.srow);
  if (zero_first) TB_CUDA(cudaMemsetAsync(z, 0, L.zeroed, st));
  {
    const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)(3 * M)};
    const cuuint64_t strides[1] = {(cuuint64_t)K};
    const cuuint32_t box[2] = {kGvSub, (cuuint32_t)ND};
    const cuuint32_t es[2] = {1, 1};
    if (enc(&tx, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, dig, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return TB_ERROR_NOT_SUPPORTED;
    if (!digits_ready) TB_TRY(gemm_tc_digits(dig, srow, x, M, K, 3, norm_w, eps, st));
  }

  GvArgs a{};
  a.out = out;
  a.srow = srow;
  a.scale = scale;
  a.resid = resid;
  a.acc = reinterpret_cast<int*>(z + L.acc);
  a.count = reinterpret_cast<unsigned int*>(z + L.count);
  a.M = M;
  a.N = N;
  a.K = K;
  a.ND = ND;
  a.KB = KB;
  a.total = total;
  a.stages = stages;
  a.part = group > 0 ? reinterpret_cast<float*>(w + L.part) : nullptr;
  a.gs = group > 0 ? group / kGvSub : 0;
  a.ngroups = group > 0 ? K / group : 0;
  a.err = wait_timeout_word();
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(192);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return group > 0 ? launch_gv<true>(cfg, G, tw, tx, a) : launch_gv<false>(cfg, G, tw, tx, a);
}

}  // namespace tb
