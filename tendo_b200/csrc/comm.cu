// comm.cu — the collective layer of tensor parallelism: an NCCL communicator
// behind the C ABI (the reference's planned tb_comm_init /
// tb_allreduce_sum_f32 pair).  libnccl.so.2 is resolved at run time, so the
// library loads in processes without NCCL and shares the NCCL that the host
// framework (PyTorch) already loaded.
//
// Allreduces up to the exchange capacity (2 MB by default) run as one kernel
// of our own over peer memory instead of NCCL: every rank maps the other
// ranks' exchange regions (CUDA IPC handles, swapped once with an NCCL
// all-gather when the communicator is made), and each CTA of the kernel
//   1. stores its slice of the local buffer into every peer's receive slot
//      for (this call's parity, this rank) over NVLink, each 32-bit value
//      in a 64-bit word tagged with the call's sequence number, then
//   2. reads the same slice from every peer's slot in its own memory,
//      polling each word until its tag matches (bounded; an expired wait
//      counts in the error word), and combines the ranks' values in rank
//      order 0, 1, ... (the same bits on every rank) into the local buffer.
// The sequence number lives in device memory and the kernel's last CTA
// advances it, so a captured graph replays with fresh tags; receive slots
// alternate by its parity, so a rank one call ahead never overwrites a slot a
// slower rank still reads.  Plain loads and stores only: no multicast and no
// bulk copies from peer memory.
#include <dlfcn.h>
#include <nccl.h>
#include <stdlib.h>
#include <string.h>

#include <mutex>
#include <string>

#include "common.cuh"
#include "kernels.h"

namespace tb {
namespace {
constexpr int kPxMaxRanks = 8;
constexpr int kPxMaxCtas = 64;
constexpr int kPxThreads = 512;
constexpr uint32_t kPxSpin = 1u << 22;        // flag polls before a wait counts as expired (about a second)
constexpr size_t kPxDefaultCap = 2u << 20;   // payload bytes per receive slot
}  // namespace
}  // namespace tb

struct tb_comm {
  ncclComm_t nccl = nullptr;
  int rank = 0, nranks = 1, device = 0;
  // peer exchange: this rank's region [2 parities][nranks][cap] receive
  // slots, then [2][nranks][kPxMaxCtas] flags, then the sequence number and
  // the CTA-done counter; region[r] is rank r's region as mapped here
  unsigned char* region[tb::kPxMaxRanks] = {};
  size_t cap = 0;
  bool peer = false;
};

namespace tb {
namespace {

struct NcclApi {
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                             cudaStream_t) = nullptr;
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  const char* (*get_error_string)(ncclResult_t) = nullptr;
  bool ok = false;
};

const NcclApi& nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return;
    api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
    api.comm_init_rank = reinterpret_cast<decltype(api.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
    api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
    api.all_reduce = reinterpret_cast<decltype(api.all_reduce)>(dlsym(h, "ncclAllReduce"));
    api.all_gather = reinterpret_cast<decltype(api.all_gather)>(dlsym(h, "ncclAllGather"));
    api.get_error_string = reinterpret_cast<decltype(api.get_error_string)>(dlsym(h, "ncclGetErrorString"));
    api.ok = api.get_unique_id && api.comm_init_rank && api.comm_destroy && api.all_reduce && api.all_gather &&
             api.get_error_string;
  });
  return api;
}

tb_status_t nccl_fail(ncclResult_t r, const char* where) {
  const NcclApi& api = nccl();
  const char* msg = api.get_error_string ? api.get_error_string(r) : "nccl error";
  return fail_message((std::string(where) + ": " + msg).c_str());
}

struct PeerArgs {
  void* buf;  // this rank's data, reduced in place
  unsigned char* region[kPxMaxRanks];
  size_t cap;  // payload bytes per receive slot (the slot holds 2 cap bytes of tagged words)
  int64_t n;   // elements (fp32 for a sum, uint64 for a max)
  int rank, nranks;
  int* err;
};

// Region: [2 parities][nranks] receive slots of 2 cap bytes, then the call
// sequence number and the CTA-done counter.
__host__ __device__ inline size_t px_slot_bytes(size_t cap) { return 2 * cap; }
__host__ __device__ inline size_t px_seq_off(size_t cap, int nranks) {
  return (size_t)2 * nranks * px_slot_bytes(cap);
}
inline size_t px_region_bytes(size_t cap, int nranks) { return px_seq_off(cap, nranks) + 64; }

__device__ __forceinline__ ulonglong2 ld_volatile_v2(const ulonglong2* p) {
  ulonglong2 v;
  asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(v.x), "=l"(v.y) : "l"(p) : "memory");
  return v;
}

// Tagged words: 32 payload bits in the low half of a 64-bit word, the call's
// sequence number in the high half.  A 64-bit store is single-copy atomic, so
// a reader that sees the tag sees the payload with it: no fence, no flag.
// One "pair" is two payload words (two fp32 values, or the halves of one
// uint64), moved as one 16-byte store of two tagged words.
template <bool MAXU64>
__global__ void __launch_bounds__(kPxThreads) peer_allreduce_kernel(PeerArgs a) {
  unsigned char* own = a.region[a.rank];
  uint32_t* seqp = reinterpret_cast<uint32_t*>(own + px_seq_off(a.cap, a.nranks));
  // every CTA reads the number before any CTA counts itself done below
  const uint32_t e = *reinterpret_cast<volatile uint32_t*>(seqp) + 1u;
  const unsigned long long tag = (unsigned long long)e << 32;
  const int par = (int)(e & 1u);
  const int64_t nw = MAXU64 ? 2 * a.n : a.n;  // payload words
  const int64_t np = (nw + 1) / 2;             // pairs
  const int64_t per = (np + gridDim.x - 1) / gridDim.x;
  const int64_t p0 = (int64_t)blockIdx.x * per, p1 = p0 + per < np ? p0 + per : np;
  uint32_t* words = static_cast<uint32_t*>(a.buf);
  // 1. this rank's pairs into every peer's slot (par, rank)
  for (int64_t p = p0 + threadIdx.x; p < p1; p += blockDim.x) {
    const uint32_t w0 = words[2 * p], w1 = 2 * p + 1 < nw ? words[2 * p + 1] : 0u;
    const ulonglong2 v = make_ulonglong2(tag | w0, tag | w1);
    for (int r = 0; r < a.nranks; r++) {
      if (r == a.rank) continue;
      ulonglong2* slot = reinterpret_cast<ulonglong2*>(a.region[r] + ((size_t)par * a.nranks + a.rank) *
                                                                           px_slot_bytes(a.cap));
      slot[p] = v;
    }
  }
  // 2. the peers' pairs (bounded polls on the tags), combined in rank order
  __shared__ int gave_up;
  if (threadIdx.x == 0) gave_up = 0;
  __syncthreads();
  for (int64_t p = p0 + threadIdx.x; p < p1; p += blockDim.x) {
    const uint32_t m0 = words[2 * p], m1 = 2 * p + 1 < nw ? words[2 * p + 1] : 0u;
    float s0 = 0.f, s1 = 0.f;
    unsigned long long mx = 0ull;
    for (int r = 0; r < a.nranks; r++) {
      uint32_t w0 = m0, w1 = m1;
      if (r != a.rank) {
        const ulonglong2* src = reinterpret_cast<const ulonglong2*>(own + ((size_t)par * a.nranks + r) *
                                                                                px_slot_bytes(a.cap)) + p;
        ulonglong2 v = ld_volatile_v2(src);
        uint32_t it = 0;
        while (((v.x >> 32) != e || (v.y >> 32) != e) && !*reinterpret_cast<volatile int*>(&gave_up)) {
          if (++it >= kPxSpin) {
            if (a.err) atomicAdd(a.err, 1);
            gave_up = 1;
            break;
          }
          v = ld_volatile_v2(src);
        }
        w0 = (uint32_t)v.x;
        w1 = (uint32_t)v.y;
      }
      if (MAXU64) {
        const unsigned long long x = ((unsigned long long)w1 << 32) | w0;
        mx = r == 0 || x > mx ? x : mx;
      } else if (r == 0) {
        s0 = __uint_as_float(w0);
        s1 = __uint_as_float(w1);
      } else {
        s0 += __uint_as_float(w0);
        s1 += __uint_as_float(w1);
      }
    }
    if (MAXU64) {
      words[2 * p] = (uint32_t)mx;
      words[2 * p + 1] = (uint32_t)(mx >> 32);
    } else {
      words[2 * p] = __float_as_uint(s0);
      if (2 * p + 1 < nw) words[2 * p + 1] = __float_as_uint(s1);
    }
  }
  // the last CTA to finish advances the sequence number for the next call
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned int* done = reinterpret_cast<unsigned int*>(seqp + 1);
    __threadfence();
    if (atomicAdd(done, 1u) == gridDim.x - 1) {
      *done = 0u;
      __threadfence();
      atomicExch(seqp, e);
    }
  }
}

// CTAs for `pairs` tagged pairs: two per thread, at most kPxMaxCtas.
int peer_grid(int64_t pairs) {
  int64_t g = (pairs + 2 * kPxThreads - 1) / (2 * kPxThreads);
  if (g < 1) g = 1;
  return (int)(g < kPxMaxCtas ? g : kPxMaxCtas);
}

bool peer_disabled() {
  static const bool off = [] {
    const char* e = getenv("TENDO_B200_ALLREDUCE");
    return e && strcmp(e, "nccl") == 0;
  }();
  return off;
}

// Maps every rank's exchange region (collective over the communicator; on
// any failure every rank keeps NCCL for all calls).
tb_status_t peer_setup(tb_comm* c, size_t cap) {
  if (c->nranks < 2 || c->nranks > kPxMaxRanks || peer_disabled()) return TB_SUCCESS;
  const NcclApi& api = nccl();
  const size_t bytes = px_region_bytes(cap, c->nranks);
  int ok = 1;
  unsigned char* mine = nullptr;
  cudaIpcMemHandle_t h{};
  if (cudaMalloc(&mine, bytes) != cudaSuccess || cudaMemset(mine, 0, bytes) != cudaSuccess ||
      cudaDeviceSynchronize() != cudaSuccess || cudaIpcGetMemHandle(&h, mine) != cudaSuccess) {
    cudaGetLastError();
    ok = 0;
  }
  // swap the handles (and whether each rank has one) with NCCL
  const size_t hb = sizeof(cudaIpcMemHandle_t);
  unsigned char* dev = nullptr;
  int* okd = nullptr;
  if (cudaMalloc(&dev, hb * (c->nranks + 1)) != cudaSuccess || cudaMalloc(&okd, sizeof(int)) != cudaSuccess) {
    if (dev) cudaFree(dev);
    if (mine) cudaFree(mine);
    return fail_message("peer exchange: cudaMalloc");
  }
  cudaMemcpy(dev + hb * c->nranks, &h, hb, cudaMemcpyHostToDevice);
  ncclResult_t r = api.all_gather(dev + hb * c->nranks, dev, hb, ncclUint8, c->nccl, 0);
  unsigned char hosts[kPxMaxRanks * sizeof(cudaIpcMemHandle_t)];
  if (r == ncclSuccess && cudaStreamSynchronize(0) == cudaSuccess)
    cudaMemcpy(hosts, dev, hb * c->nranks, cudaMemcpyDeviceToHost);
  else
    ok = 0;
  c->region[c->rank] = mine;
  for (int q = 0; q < c->nranks && ok; q++) {
    if (q == c->rank) continue;
    cudaIpcMemHandle_t ph;
    memcpy(&ph, hosts + hb * q, hb);
    void* p = nullptr;
    if (cudaIpcOpenMemHandle(&p, ph, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
      cudaGetLastError();
      ok = 0;
      break;
    }
    c->region[q] = static_cast<unsigned char*>(p);
  }
  // every rank takes the peer path only if every rank mapped every region
  cudaMemcpy(okd, &ok, sizeof(int), cudaMemcpyHostToDevice);
  r = api.all_reduce(okd, okd, 1, ncclInt32, ncclMin, c->nccl, 0);
  int all = 0;
  if (r == ncclSuccess && cudaStreamSynchronize(0) == cudaSuccess)
    cudaMemcpy(&all, okd, sizeof(int), cudaMemcpyDeviceToHost);
  cudaFree(dev);
  cudaFree(okd);
  if (r != ncclSuccess) return nccl_fail(r, "peer exchange: ncclAllReduce");
  if (!all) {
    for (int q = 0; q < c->nranks; q++)
      if (q != c->rank && c->region[q]) cudaIpcCloseMemHandle(c->region[q]);
    for (int q = 0; q < c->nranks; q++) c->region[q] = nullptr;
    if (mine) cudaFree(mine);
    cudaGetLastError();
    return TB_SUCCESS;
  }
  c->cap = cap;
  c->peer = true;
  return TB_SUCCESS;
}

void peer_teardown(tb_comm* c) {
  if (!c->peer) return;
  for (int q = 0; q < c->nranks; q++)
    if (q != c->rank && c->region[q]) cudaIpcCloseMemHandle(c->region[q]);
  cudaFree(c->region[c->rank]);
  for (int q = 0; q < c->nranks; q++) c->region[q] = nullptr;
  c->peer = false;
}

}  // namespace

bool peer_allreduce_active(const tb_comm* c) { return c && c->peer; }

tb_status_t allreduce(tb_comm* c, void* buf, size_t count, bool u64_max, cudaStream_t st, int* err) {
  if (!c || c->nranks == 1 || count == 0) return TB_SUCCESS;
  const size_t bytes = count * (u64_max ? 8 : 4);
  if (c->peer && bytes <= c->cap && aligned(buf, 16)) {
    PeerArgs a{};
    a.buf = buf;
    for (int q = 0; q < c->nranks; q++) a.region[q] = c->region[q];
    a.cap = c->cap;
    a.n = (int64_t)count;
    a.rank = c->rank;
    a.nranks = c->nranks;
    a.err = err ? err : wait_timeout_word();
    const int g = peer_grid((int64_t)((bytes / 4 + 1) / 2));
    if (u64_max)
      peer_allreduce_kernel<true><<<g, kPxThreads, 0, st>>>(a);
    else
      peer_allreduce_kernel<false><<<g, kPxThreads, 0, st>>>(a);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "peer_allreduce_kernel");
    return TB_SUCCESS;
  }
  const NcclApi& api = nccl();
  const ncclResult_t r = api.all_reduce(buf, buf, count, u64_max ? ncclUint64 : ncclFloat32,
                                        u64_max ? ncclMax : ncclSum, c->nccl, st);
  if (r != ncclSuccess) return nccl_fail(r, "ncclAllReduce");
  return TB_SUCCESS;
}

int comm_rank(const tb_comm* c) { return c ? c->rank : 0; }
int comm_size(const tb_comm* c) { return c ? c->nranks : 1; }

}  // namespace tb

extern "C" size_t tb_comm_unique_id_bytes(void) { return sizeof(ncclUniqueId); }

extern "C" tb_status_t tb_comm_unique_id(void* id_out, size_t bytes) {
  TB_INJECT("tb_comm_unique_id");
  TB_REQUIRE(id_out && bytes >= sizeof(ncclUniqueId));
  const tb::NcclApi& api = tb::nccl();
  if (!api.ok) return TB_ERROR_NOT_SUPPORTED;
  ncclUniqueId id;
  const ncclResult_t r = api.get_unique_id(&id);
  if (r != ncclSuccess) return tb::nccl_fail(r, "ncclGetUniqueId");
  memcpy(id_out, &id, sizeof(id));
  return TB_SUCCESS;
}

extern "C" tb_status_t tb_comm_create(tb_comm** out, const void* id, size_t bytes, int rank, int nranks,
                                      int device) {
  TB_INJECT("tb_comm_create");
  TB_REQUIRE(out && nranks >= 1 && rank >= 0 && rank < nranks && device >= 0);
  *out = nullptr;
  tb_comm* c = new tb_comm();
  c->rank = rank;
  c->nranks = nranks;
  c->device = device;
  if (nranks > 1) {
    TB_REQUIRE(id && bytes >= sizeof(ncclUniqueId));
    const tb::NcclApi& api = tb::nccl();
    if (!api.ok) {
      delete c;
      return TB_ERROR_NOT_SUPPORTED;
    }
    int prev = 0;
    cudaGetDevice(&prev);
    cudaError_t e = cudaSetDevice(device);
    if (e != cudaSuccess) {
      delete c;
      return tb::cuda_fail(e, "cudaSetDevice");
    }
    ncclUniqueId uid;
    memcpy(&uid, id, sizeof(uid));
    const ncclResult_t r = api.comm_init_rank(&c->nccl, nranks, uid, rank);
    if (r != ncclSuccess) {
      cudaSetDevice(prev);
      delete c;
      return tb::nccl_fail(r, "ncclCommInitRank");
    }
    const tb_status_t ps = tb::peer_setup(c, tb::kPxDefaultCap);
    cudaSetDevice(prev);
    if (ps != TB_SUCCESS) {
      api.comm_destroy(c->nccl);
      delete c;
      return ps;
    }
  }
  *out = c;
  return TB_SUCCESS;
}

extern "C" tb_status_t tb_comm_destroy(tb_comm* c) {
  if (!c) return TB_SUCCESS;
  if (c->nranks > 1) {
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(c->device);
    tb::peer_teardown(c);
    cudaSetDevice(prev);
  }
  if (c->nccl) tb::nccl().comm_destroy(c->nccl);
  delete c;
  return TB_SUCCESS;
}

extern "C" tb_status_t tb_allreduce_sum_f32(tb_comm* c, float* buf, int64_t n, tb_stream_t stream) {
  TB_INJECT("tb_allreduce_sum_f32");
  TB_REQUIRE(c && n >= 0 && (n == 0 || buf));
  return tb::allreduce(c, buf, (size_t)n, false, (cudaStream_t)stream);
}

extern "C" int tb_comm_peer_active(const tb_comm* c) { return tb::peer_allreduce_active(c) ? 1 : 0; }
