// comm.cu — the collective layer of tensor parallelism: an NCCL communicator
// behind the C ABI (the reference's planned tb_comm_init /
// tb_allreduce_sum_f32 pair).  libnccl.so.2 is resolved at run time, so the
// library loads in processes without NCCL and shares the NCCL that the host
// framework (PyTorch) already loaded.
#include <dlfcn.h>
#include <nccl.h>
#include <string.h>

#include <mutex>
#include <string>

#include "common.cuh"
#include "kernels.h"

struct tb_comm {
  ncclComm_t nccl = nullptr;
  int rank = 0, nranks = 1, device = 0;
};

namespace tb {
namespace {

struct NcclApi {
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                             cudaStream_t) = nullptr;
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
    api.get_error_string = reinterpret_cast<decltype(api.get_error_string)>(dlsym(h, "ncclGetErrorString"));
    api.ok = api.get_unique_id && api.comm_init_rank && api.comm_destroy && api.all_reduce && api.get_error_string;
  });
  return api;
}

tb_status_t nccl_fail(ncclResult_t r, const char* where) {
  const NcclApi& api = nccl();
  const char* msg = api.get_error_string ? api.get_error_string(r) : "nccl error";
  return fail_message((std::string(where) + ": " + msg).c_str());
}

}  // namespace

tb_status_t allreduce(tb_comm* c, void* buf, size_t count, bool u64_max, cudaStream_t st) {
  if (!c || c->nranks == 1 || count == 0) return TB_SUCCESS;
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
    cudaSetDevice(prev);
    if (r != ncclSuccess) {
      delete c;
      return tb::nccl_fail(r, "ncclCommInitRank");
    }
  }
  *out = c;
  return TB_SUCCESS;
}

extern "C" tb_status_t tb_comm_destroy(tb_comm* c) {
  if (!c) return TB_SUCCESS;
  if (c->nccl) tb::nccl().comm_destroy(c->nccl);
  delete c;
  return TB_SUCCESS;
}

extern "C" tb_status_t tb_allreduce_sum_f32(tb_comm* c, float* buf, int64_t n, tb_stream_t stream) {
  TB_INJECT("tb_allreduce_sum_f32");
  TB_REQUIRE(c && n >= 0 && (n == 0 || buf));
  return tb::allreduce(c, buf, (size_t)n, false, (cudaStream_t)stream);
}
