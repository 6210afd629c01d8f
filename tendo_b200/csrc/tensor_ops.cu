// tensor_ops.cu — the generic fp32 tensor ops that tendo's unchanged Llama
// attention issues through llama.Backend (models/llama/forward.go:13-27,
// models/llama/quantized.go:282-372): strided batched MatMul (Q.K^T on a
// transposed view, P.V on the GQA-expanded view), broadcast Add / Sub / Mul /
// Div, Softmax along one dimension, Where, Tril, Cat and Full.
//
// Every op takes strided views — per dimension an element stride, 0 for a
// broadcast or expanded dimension — and writes a new contiguous tensor, as
// the reference backends do.  The arithmetic follows the reference CPU
// backend's order (cpu/backend.go): elementwise float32 operations, a
// softmax with the max seeded at -MaxFloat32, exp in double precision and a
// sequential float32 sum, and matmul sums of separately rounded products in k
// order (the order the oracle restates for gonum's Gemm).  These are the
// compatibility path; tb_attention_f32 is the fused one.
#include <math.h>
#include <float.h>

#include "common.cuh"
#include "kernels.h"

namespace tb {
namespace {

constexpr int kRank = TB_MAX_RANK;

struct View {
  int64_t shape[kRank];
  int64_t stride[kRank];
  int rank;
};

// Offset of flat (contiguous, row-major over `shape`) index i in a view with
// `strides` over the same shape.
__device__ __forceinline__ int64_t view_offset(int64_t i, const int64_t* shape, const int64_t* strides, int rank) {
  int64_t off = 0;
  for (int d = rank - 1; d >= 0; d--) {
    const int64_t c = i % shape[d];
    i /= shape[d];
    off += c * strides[d];
  }
  return off;
}

__global__ void fill_kernel(float* out, float v, int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    out[i] = v;
}

__global__ void binary_kernel(float* out, const float* a, const float* b, int op, View va, View vb, int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const float x = a[view_offset(i, va.shape, va.stride, va.rank)];
    const float y = b[view_offset(i, va.shape, vb.stride, va.rank)];
    float r;
    switch (op) {
      case TB_BINARY_ADD: r = __fadd_rn(x, y); break;
      case TB_BINARY_SUB: r = __fsub_rn(x, y); break;
      case TB_BINARY_MUL: r = __fmul_rn(x, y); break;
      default: r = __fdiv_rn(x, y); break;
    }
    out[i] = r;
  }
}

__global__ void where_kernel(float* out, const float* c, const float* x, const float* y, View vc, View vx, View vy,
                             int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const float cv = c[view_offset(i, vc.shape, vc.stride, vc.rank)];
    out[i] = cv > 0.f ? x[view_offset(i, vc.shape, vx.stride, vc.rank)] : y[view_offset(i, vc.shape, vy.stride, vc.rank)];
  }
}

__global__ void tril_kernel(float* out, const float* in, int64_t rows, int64_t cols, int64_t k) {
  const int64_t n = rows * cols;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / cols, c = i - r * cols;
    out[i] = c <= r + k ? in[i] : 0.f;
  }
}

// One warp per slice along `dim`: the exponentials in parallel, the max and
// the sum in the reference's order (max over the slice, then a sequential
// float32 sum by lane 0).
__global__ void softmax_kernel(float* out, const float* in, View vin, int dim, int64_t nslices) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t slice = blockIdx.x * (int64_t)(blockDim.x >> 5) + warp;
  if (slice >= nslices) return;
  const int64_t len = vin.shape[dim];
  // the slice's first element: coordinates of every other dimension from `slice`
  int64_t rem = slice, in_base = 0, out_base = 0, out_stride = 1, ostride = 1;
  for (int d = vin.rank - 1; d >= 0; d--) {
    if (d == dim) {
      out_stride = ostride;
    } else {
      const int64_t c = rem % vin.shape[d];
      rem /= vin.shape[d];
      in_base += c * vin.stride[d];
      out_base += c * ostride;
    }
    ostride *= vin.shape[d];
  }
  const int64_t is = vin.stride[dim];
  float mx = -FLT_MAX;
  for (int64_t j = lane; j < len; j += 32) mx = fmaxf(mx, in[in_base + j * is]);
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  for (int64_t j = lane; j < len; j += 32)
    out[out_base + j * out_stride] = (float)exp((double)__fsub_rn(in[in_base + j * is], mx));
  __syncwarp();
  float sum = 0.f;
  if (lane == 0)
    for (int64_t j = 0; j < len; j++) sum = __fadd_rn(sum, out[out_base + j * out_stride]);
  sum = __shfl_sync(0xffffffffu, sum, 0);
  for (int64_t j = lane; j < len; j += 32) out[out_base + j * out_stride] = __fdiv_rn(out[out_base + j * out_stride], sum);
}

constexpr int kMmTile = 16;

struct MmArgs {
  float* out;
  const float* a;
  const float* b;
  View batch;             // batch dimensions (shape) with a's strides
  int64_t b_stride[kRank];  // b's batch strides
  int64_t M, N, K, a_rs, a_cs, b_rs, b_cs;
};

// out[batch, m, n] = sum_k a[batch, m, k] * b[batch, k, n], each product
// rounded, then added in k order.  16 x 16 output tile per block, k in
// 16-wide slabs staged in shared memory.
__global__ void matmul_kernel(MmArgs p) {
  __shared__ float as[kMmTile][kMmTile + 1];
  __shared__ float bs[kMmTile][kMmTile + 1];
  const int64_t bi = blockIdx.z;
  int64_t aoff = 0, boff = 0, rem = bi;
  for (int d = p.batch.rank - 1; d >= 0; d--) {
    const int64_t c = rem % p.batch.shape[d];
    rem /= p.batch.shape[d];
    aoff += c * p.batch.stride[d];
    boff += c * p.b_stride[d];
  }
  const int tx = threadIdx.x, ty = threadIdx.y;
  const int64_t m = blockIdx.y * (int64_t)kMmTile + ty, n = blockIdx.x * (int64_t)kMmTile + tx;
  float acc = 0.f;
  for (int64_t k0 = 0; k0 < p.K; k0 += kMmTile) {
    const int64_t ka = k0 + tx, kb = k0 + ty;
    as[ty][tx] = (m < p.M && ka < p.K) ? p.a[aoff + m * p.a_rs + ka * p.a_cs] : 0.f;
    bs[ty][tx] = (kb < p.K && n < p.N) ? p.b[boff + kb * p.b_rs + n * p.b_cs] : 0.f;
    __syncthreads();
    const int kmax = (p.K - k0) < kMmTile ? (int)(p.K - k0) : kMmTile;
    for (int k = 0; k < kmax; k++) acc = __fadd_rn(acc, __fmul_rn(as[ty][k], bs[k][tx]));
    __syncthreads();
  }
  if (m < p.M && n < p.N) p.out[(bi * p.M + m) * p.N + n] = acc;
}

__global__ void cat_kernel(float* out, const float* a, const float* b, View vo, View va, View vb, int dim, int64_t n) {
  const int64_t asz = va.shape[dim];
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    int64_t rem = i, oa = 0, ob = 0;
    bool from_a = true;
    for (int d = vo.rank - 1; d >= 0; d--) {
      int64_t c = rem % vo.shape[d];
      rem /= vo.shape[d];
      if (d == dim && c >= asz) {
        from_a = false;
        c -= asz;
      }
      oa += c * va.stride[d];
      ob += c * vb.stride[d];
    }
    out[i] = from_a ? a[oa] : b[ob];
  }
}

unsigned grid_for(int64_t n) {
  int64_t g = (n + 255) / 256;
  const int64_t cap = (int64_t)sm_count() * 16;
  return (unsigned)(g < 1 ? 1 : (g > cap ? cap : g));
}

// Copies a host shape / stride pair into a View; rank and sizes checked.
bool make_view(View& v, int rank, const int64_t* shape, const int64_t* strides) {
  if (rank < 1 || rank > kRank || !shape) return false;
  v.rank = rank;
  for (int d = 0; d < rank; d++) {
    if (shape[d] < 0) return false;
    v.shape[d] = shape[d];
    v.stride[d] = strides ? strides[d] : 0;
  }
  if (!strides) {  // contiguous
    int64_t s = 1;
    for (int d = rank - 1; d >= 0; d--) {
      v.stride[d] = s;
      s *= shape[d];
    }
  }
  return true;
}

int64_t numel(const View& v) {
  int64_t n = 1;
  for (int d = 0; d < v.rank; d++) n *= v.shape[d];
  return n;
}

}  // namespace
}  // namespace tb

using tb::View;

extern "C" tb_status_t tb_fill_f32(float* out, float value, int64_t n, tb_stream_t stream) {
  TB_INJECT("tb_fill_f32");
  TB_REQUIRE(n >= 0);
  if (n == 0) return TB_SUCCESS;
  TB_REQUIRE(out);
  tb::fill_kernel<<<tb::grid_for(n), 256, 0, (cudaStream_t)stream>>>(out, value, n);
  return tb::check_launch("fill_kernel");
}

extern "C" tb_status_t tb_binary_f32(float* out, const float* a, const float* b, int op, int rank, const int64_t* shape,
                                     const int64_t* a_strides, const int64_t* b_strides, tb_stream_t stream) {
  TB_INJECT("tb_binary_f32");
  TB_REQUIRE(op >= TB_BINARY_ADD && op <= TB_BINARY_DIV);
  View va, vb;
  TB_REQUIRE(tb::make_view(va, rank, shape, a_strides) && tb::make_view(vb, rank, shape, b_strides));
  const int64_t n = tb::numel(va);
  if (n == 0) return TB_SUCCESS;
  TB_REQUIRE(out && a && b);
  tb::binary_kernel<<<tb::grid_for(n), 256, 0, (cudaStream_t)stream>>>(out, a, b, op, va, vb, n);
  return tb::check_launch("binary_kernel");
}

extern "C" tb_status_t tb_where_f32(float* out, const float* cond, const float* x, const float* y, int rank,
                                    const int64_t* shape, const int64_t* cond_strides, const int64_t* x_strides,
                                    const int64_t* y_strides, tb_stream_t stream) {
  TB_INJECT("tb_where_f32");
  View vc, vx, vy;
  TB_REQUIRE(tb::make_view(vc, rank, shape, cond_strides) && tb::make_view(vx, rank, shape, x_strides) &&
             tb::make_view(vy, rank, shape, y_strides));
  const int64_t n = tb::numel(vc);
  if (n == 0) return TB_SUCCESS;
  TB_REQUIRE(out && cond && x && y);
  tb::where_kernel<<<tb::grid_for(n), 256, 0, (cudaStream_t)stream>>>(out, cond, x, y, vc, vx, vy, n);
  return tb::check_launch("where_kernel");
}

extern "C" tb_status_t tb_tril_f32(float* out, const float* in, int64_t rows, int64_t cols, int64_t k,
                                   tb_stream_t stream) {
  TB_INJECT("tb_tril_f32");
  TB_REQUIRE(rows >= 0 && cols >= 0);
  if (rows == 0 || cols == 0) return TB_SUCCESS;
  TB_REQUIRE(out && in);
  tb::tril_kernel<<<tb::grid_for(rows * cols), 256, 0, (cudaStream_t)stream>>>(out, in, rows, cols, k);
  return tb::check_launch("tril_kernel");
}

extern "C" tb_status_t tb_softmax_f32(float* out, const float* in, int rank, const int64_t* shape,
                                      const int64_t* in_strides, int dim, tb_stream_t stream) {
  TB_INJECT("tb_softmax_f32");
  View v;
  TB_REQUIRE(tb::make_view(v, rank, shape, in_strides));
  if (dim < 0) dim += rank;
  TB_REQUIRE(dim >= 0 && dim < rank);
  const int64_t n = tb::numel(v);
  if (n == 0) return TB_SUCCESS;
  TB_REQUIRE(out && in);
  const int64_t slices = n / v.shape[dim];
  const int per_block = 8;
  const int64_t blocks = (slices + per_block - 1) / per_block;
  TB_REQUIRE(blocks <= 0x7fffffff);
  tb::softmax_kernel<<<(unsigned)blocks, 32 * per_block, 0, (cudaStream_t)stream>>>(out, in, v, dim, slices);
  return tb::check_launch("softmax_kernel");
}

extern "C" tb_status_t tb_matmul_f32(float* out, const float* a, const float* b, int batch_rank,
                                     const int64_t* batch_shape, const int64_t* a_batch_strides,
                                     const int64_t* b_batch_strides, int64_t M, int64_t N, int64_t K, int64_t a_rs,
                                     int64_t a_cs, int64_t b_rs, int64_t b_cs, tb_stream_t stream) {
  TB_INJECT("tb_matmul_f32");
  TB_REQUIRE(batch_rank >= 0 && batch_rank <= TB_MAX_RANK - 2 && M >= 0 && N >= 0 && K >= 0);
  tb::MmArgs p{};
  p.batch.rank = batch_rank;
  int64_t nb = 1;
  for (int d = 0; d < batch_rank; d++) {
    TB_REQUIRE(batch_shape && a_batch_strides && b_batch_strides && batch_shape[d] >= 0);
    p.batch.shape[d] = batch_shape[d];
    p.batch.stride[d] = a_batch_strides[d];
    p.b_stride[d] = b_batch_strides[d];
    nb *= batch_shape[d];
  }
  if (nb == 0 || M == 0 || N == 0) return TB_SUCCESS;
  TB_REQUIRE(out && a && b);
  TB_REQUIRE(nb <= 65535);
  p.out = out;
  p.a = a;
  p.b = b;
  p.M = M;
  p.N = N;
  p.K = K;
  p.a_rs = a_rs;
  p.a_cs = a_cs;
  p.b_rs = b_rs;
  p.b_cs = b_cs;
  const int64_t gx = (N + tb::kMmTile - 1) / tb::kMmTile, gy = (M + tb::kMmTile - 1) / tb::kMmTile;
  TB_REQUIRE(gx <= 0x7fffffff && gy <= 65535);
  tb::matmul_kernel<<<dim3((unsigned)gx, (unsigned)gy, (unsigned)nb), dim3(tb::kMmTile, tb::kMmTile), 0,
                      (cudaStream_t)stream>>>(p);
  return tb::check_launch("matmul_kernel");
}

extern "C" tb_status_t tb_cat_f32(float* out, const float* a, const float* b, int rank, const int64_t* a_shape,
                                  const int64_t* a_strides, const int64_t* b_shape, const int64_t* b_strides, int dim,
                                  tb_stream_t stream) {
  TB_INJECT("tb_cat_f32");
  View va, vb, vo;
  TB_REQUIRE(tb::make_view(va, rank, a_shape, a_strides) && tb::make_view(vb, rank, b_shape, b_strides));
  if (dim < 0) dim += rank;
  TB_REQUIRE(dim >= 0 && dim < rank);
  for (int d = 0; d < rank; d++) TB_REQUIRE(d == dim || a_shape[d] == b_shape[d]);
  vo = va;
  vo.shape[dim] = a_shape[dim] + b_shape[dim];
  const int64_t n = tb::numel(vo);
  if (n == 0) return TB_SUCCESS;
  TB_REQUIRE(out && (a || a_shape[dim] == 0) && (b || b_shape[dim] == 0));
  tb::cat_kernel<<<tb::grid_for(n), 256, 0, (cudaStream_t)stream>>>(out, a, b, vo, va, vb, dim, n);
  return tb::check_launch("cat_kernel");
}
