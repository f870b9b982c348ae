// Tensor-parallel collectives of the model: the NCCL all-reduce that follows the row-parallel
// projections (attn_output and ffn_down) when a model's weights are sharded over several GPUs.
//
// NCCL is loaded at run time (dlopen of libnccl.so.2, normally already mapped into the process by
// PyTorch) so that libzllm_cuda.so carries no link-time dependency: a single-GPU user never needs
// it.  One communicator per model; every rank enqueues the same collectives in the same order on
// the model's stream, also inside captured CUDA graphs (NCCL supports graph capture), and the
// graphs are released before the communicator.
#include <dlfcn.h>
#include <cstring>
#include <mutex>
#include <nccl.h>

#include "internal.h"

namespace zllm {

namespace {

struct NcclApi {
  decltype(&ncclGetUniqueId) get_unique_id = nullptr;
  decltype(&ncclCommInitRank) comm_init_rank = nullptr;
  decltype(&ncclAllReduce) all_reduce = nullptr;
  decltype(&ncclCommDestroy) comm_destroy = nullptr;
  decltype(&ncclGetErrorString) error_string = nullptr;
  bool ok = false;
  const char *why = "";
};

const NcclApi &nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) { api.why = "libnccl.so.2 not found (import torch first, or put NCCL on the library path)"; return; }
    api.get_unique_id = reinterpret_cast<decltype(&ncclGetUniqueId)>(dlsym(h, "ncclGetUniqueId"));
    api.comm_init_rank = reinterpret_cast<decltype(&ncclCommInitRank)>(dlsym(h, "ncclCommInitRank"));
    api.all_reduce = reinterpret_cast<decltype(&ncclAllReduce)>(dlsym(h, "ncclAllReduce"));
    api.comm_destroy = reinterpret_cast<decltype(&ncclCommDestroy)>(dlsym(h, "ncclCommDestroy"));
    api.error_string = reinterpret_cast<decltype(&ncclGetErrorString)>(dlsym(h, "ncclGetErrorString"));
    api.ok = api.get_unique_id && api.comm_init_rank && api.all_reduce && api.comm_destroy && api.error_string;
    if (!api.ok) api.why = "libnccl.so.2 lacks a needed symbol";
  });
  return api;
}

const char *nccl_err(ncclResult_t r) {
  const NcclApi &a = nccl();
  return a.ok ? a.error_string(r) : a.why;
}

}  // namespace

int tp_unique_id(void *out, size_t bytes, const char **why) {
  const NcclApi &a = nccl();
  if (!a.ok) { *why = a.why; return -1; }
  if (bytes < sizeof(ncclUniqueId)) { *why = "unique id buffer smaller than NCCL_UNIQUE_ID_BYTES"; return -1; }
  ncclUniqueId id;
  const ncclResult_t r = a.get_unique_id(&id);
  if (r != ncclSuccess) { *why = nccl_err(r); return -1; }
  memcpy(out, &id, sizeof(id));
  return 0;
}

int tp_comm_init(void **comm, int rank, int size, const void *unique_id, const char **why) {
  const NcclApi &a = nccl();
  if (!a.ok) { *why = a.why; return -1; }
  ncclUniqueId id;
  memcpy(&id, unique_id, sizeof(id));
  ncclComm_t c = nullptr;
  const ncclResult_t r = a.comm_init_rank(&c, size, id, rank);   // blocks until every rank has joined
  if (r != ncclSuccess) { *why = nccl_err(r); return -1; }
  *comm = c;
  return 0;
}

void tp_comm_destroy(void *comm) {
  const NcclApi &a = nccl();
  if (a.ok && comm) a.comm_destroy(static_cast<ncclComm_t>(comm));
}

// in-place sum of `count` f32 over the communicator's ranks, enqueued on `s`
cudaError_t tp_allreduce_sum(void *comm, float *buf, size_t count, cudaStream_t s, const char **why) {
  const NcclApi &a = nccl();
  if (!a.ok) { *why = a.why; return cudaErrorUnknown; }
  const ncclResult_t r = a.all_reduce(buf, buf, count, ncclFloat32, ncclSum, static_cast<ncclComm_t>(comm), s);
  if (r != ncclSuccess) { *why = nccl_err(r); return cudaErrorUnknown; }
  return cudaSuccess;
}

size_t tp_unique_id_bytes() { return sizeof(ncclUniqueId); }

}  // namespace zllm
