// Tensor-parallel collectives of the model: the all-reduce that follows the row-parallel
// projections (attn_output and ffn_down) when a model's weights are sharded over several GPUs.
//
// Two implementations of the same sum:
//  * NCCL (ncclAllReduce), always available;
//  * a one-shot all-reduce over NVLink peer memory (tp_ar_*), used when every rank is its own
//    process and CUDA IPC maps the peers' buffers: each rank publishes its partial vector in its
//    own buffer, stamps a per-slice epoch flag (release, system scope), waits for the peers' flags
//    of the same slice (bounded: 2 s, then ST_PEER_TIMEOUT and no wait), and sums the W partials of
//    the slice from the peers' memory in rank order -- so every rank gets the same bits.  Decode
//    vectors are a few KB to a few hundred KB: one kernel of a few CTAs, no NCCL launch overhead.
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

#include "common.cuh"
#include "internal.h"

namespace zllm {

namespace {

struct NcclApi {
  decltype(&ncclGetUniqueId) get_unique_id = nullptr;
  decltype(&ncclCommInitRank) comm_init_rank = nullptr;
  decltype(&ncclAllReduce) all_reduce = nullptr;
  decltype(&ncclAllGather) all_gather = nullptr;
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
    api.all_gather = reinterpret_cast<decltype(&ncclAllGather)>(dlsym(h, "ncclAllGather"));
    api.comm_destroy = reinterpret_cast<decltype(&ncclCommDestroy)>(dlsym(h, "ncclCommDestroy"));
    api.error_string = reinterpret_cast<decltype(&ncclGetErrorString)>(dlsym(h, "ncclGetErrorString"));
    api.ok = api.get_unique_id && api.comm_init_rank && api.all_reduce && api.all_gather && api.comm_destroy &&
             api.error_string;
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

// every rank's `count` floats, in rank order, on every rank
cudaError_t tp_allgather(void *comm, const float *send, float *recv, size_t count, cudaStream_t s, const char **why) {
  const NcclApi &a = nccl();
  if (!a.ok) { *why = a.why; return cudaErrorUnknown; }
  const ncclResult_t r = a.all_gather(send, recv, count, ncclFloat32, static_cast<ncclComm_t>(comm), s);
  if (r != ncclSuccess) { *why = nccl_err(r); return cudaErrorUnknown; }
  return cudaSuccess;
}

namespace {
// rank r's slice of a vocab split evenly over `size` ranks starts at r * V / size
__device__ __forceinline__ int64_t vocab_start(int r, int64_t V, int size) { return (int64_t)r * V / size; }

// logits [nl][V] from the gathered slices recv [size][nl][vpad]
__global__ void vocab_gather_kernel(const float *__restrict__ recv, int nl, int64_t vpad, int64_t V, int size,
                                    float *__restrict__ logits) {
  const int64_t total = (int64_t)nl * V;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    const int t = (int)(e / V);
    const int64_t v = e - (int64_t)t * V;
    int r = (int)(v * size / V);
    while (r + 1 < size && vocab_start(r + 1, V, size) <= v) r++;
    while (r > 0 && vocab_start(r, V, size) > v) r--;
    logits[e] = recv[((int64_t)r * nl + t) * vpad + (v - vocab_start(r, V, size))];
  }
}
}  // namespace

cudaError_t launch_vocab_gather(const float *recv, int nl, int64_t vpad, int64_t V, int size, float *logits,
                                cudaStream_t s) {
  const int64_t total = (int64_t)nl * V;
  const int64_t grid = (total + 255) / 256 < 4096 ? (total + 255) / 256 : 4096;
  vocab_gather_kernel<<<(unsigned)grid, 256, 0, s>>>(recv, nl, vpad, V, size, logits);
  return cudaGetLastError();
}

// ============================================================================ one-shot all-reduce
namespace {

constexpr int kArMaxRanks = 8, kArMaxCtas = 32, kArThreads = 256;

struct ArArgs {
  float *x;                         // in: this rank's partial, out: the sum (n floats)
  uint8_t *peer[kArMaxRanks];       // every rank's allocation (own included), see ar_layout
  uint8_t *mine;                    // this rank's allocation
  unsigned *status;
  int64_t n, cap;
  int rank, size;
};

// Layout of a rank's allocation: recv [2 parities][kArMaxRanks senders][cap] floats, then the
// stamps [kArMaxRanks senders][kArMaxCtas slices] (epochs), then its epoch and done counters.
__host__ __device__ inline int64_t ar_recv_off(int64_t cap, int par, int sender) {
  return ((int64_t)par * kArMaxRanks + sender) * cap * 4;
}
__host__ __device__ inline int64_t ar_flag_off(int64_t cap) { return (int64_t)2 * kArMaxRanks * cap * 4; }

__device__ __forceinline__ void st_release_sys(int *p, int v) {
  asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire_sys(const int *p) {
  int v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// CTA c owns slice c of the vector.  It stores its partial slice into every rank's receive slot for
// this sender (peer stores over NVLink), then, after a CTA barrier, one release store per rank
// stamps the slice with the epoch -- the release orders the CTA's earlier stores (they happen
// before it through the barrier).  Each rank then polls its own stamps, and sums the senders'
// slices from its own memory in rank order.  The epoch is read before any CTA can have moved it:
// the last CTA of a launch advances it after every CTA has counted itself done.  The receive slots
// alternate by epoch parity: a sender writes parity p again only two epochs later, after it has
// seen this rank's stamp of the epoch in between, which this rank writes after its reads of p.
__global__ void __launch_bounds__(kArThreads) tp_ar_kernel(const ArArgs a) {
  const int c = blockIdx.x, tid = threadIdx.x;
  // under programmatic dependent launch the next GEMV may become resident now and stream its
  // weights; x (and the epoch, which the previous all-reduce advanced before any later kernel ran)
  // are read only after the producing kernel has completed
  pdl_launch_dependents();
  pdl_wait();
  int *myflags = reinterpret_cast<int *>(a.mine + ar_flag_off(a.cap));
  int *epoch = myflags + kArMaxRanks * kArMaxCtas, *done = epoch + 1;
  const int e = *reinterpret_cast<volatile int *>(epoch) + 1;
  const int par = e & 1;
  const int64_t chunk = (a.n + gridDim.x - 1) / gridDim.x;
  const int64_t i0 = c * chunk, i1 = min(a.n, i0 + chunk);
  for (int64_t i = i0 + tid; i < i1; i += kArThreads) {
    const float v = a.x[i];
    for (int r = 0; r < a.size; r++)
      reinterpret_cast<float *>(a.peer[r] + ar_recv_off(a.cap, par, a.rank))[i] = v;
  }
  __syncthreads();
  if (tid < a.size)
    st_release_sys(reinterpret_cast<int *>(a.peer[tid] + ar_flag_off(a.cap)) + a.rank * kArMaxCtas + c, e);
  if (tid < a.size) {
    const uint64_t deadline = globaltimer_ns() + WAIT_DEADLINE_NS;
    while (ld_acquire_sys(myflags + tid * kArMaxCtas + c) < e) {
      if (globaltimer_ns() > deadline) { atomicOr(a.status, ST_PEER_TIMEOUT); break; }
    }
  }
  __syncthreads();
  for (int64_t i = i0 + tid; i < i1; i += kArThreads) {
    float acc = 0.f;
    for (int r = 0; r < a.size; r++)
      acc = __fadd_rn(acc, __ldcv(reinterpret_cast<const float *>(a.mine + ar_recv_off(a.cap, par, r)) + i));
    a.x[i] = acc;
  }
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    if (atomicAdd(done, 1) == (int)gridDim.x - 1) {
      *done = 0;
      *reinterpret_cast<volatile int *>(epoch) = e;
    }
  }
}

}  // namespace

struct TpAr {
  void *base = nullptr;                 // own allocation (ar_layout)
  void *peer[kArMaxRanks] = {};         // the peers' allocations, mapped by CUDA IPC (own: base)
  int64_t cap = 0;
  int rank = 0, size = 1;
};

static size_t ar_bytes(int64_t cap) { return (size_t)ar_flag_off(cap) + (kArMaxRanks * kArMaxCtas + 2) * 4; }

int tp_ar_setup(void *comm, int rank, int size, int64_t cap, cudaStream_t s, TpAr **out, const char **why) {
  *out = nullptr;
  const NcclApi &api = nccl();
  if (!api.ok) { *why = api.why; return -1; }
  if (size < 2 || size > kArMaxRanks) { *why = "one-shot all-reduce: 2..8 ranks"; return -1; }
  TpAr *ar = new TpAr;
  ar->cap = (cap + 3) / 4 * 4;
  ar->rank = rank;
  ar->size = size;
  void *ids = nullptr;
  cudaIpcMemHandle_t hs[kArMaxRanks];
  cudaError_t e = cudaMalloc(&ar->base, ar_bytes(ar->cap));
  if (e == cudaSuccess) e = cudaMemsetAsync(ar->base, 0, ar_bytes(ar->cap), s);
  if (e == cudaSuccess) e = cudaMalloc(&ids, sizeof(cudaIpcMemHandle_t) * (size + 1));
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&hs[0], ar->base);
  if (e == cudaSuccess) e = cudaMemcpyAsync(ids, &hs[0], sizeof(cudaIpcMemHandle_t), cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) {
    *why = cudaGetErrorString(e);
    if (ids) cudaFree(ids);
    if (ar->base) cudaFree(ar->base);
    delete ar;
    cudaGetLastError();
    return -1;
  }
  // every rank's handle to every rank (also a barrier: all buffers are zeroed before any use)
  uint8_t *gathered = reinterpret_cast<uint8_t *>(ids) + sizeof(cudaIpcMemHandle_t);
  ncclResult_t r = api.all_gather(ids, gathered, sizeof(cudaIpcMemHandle_t), ncclUint8, static_cast<ncclComm_t>(comm), s);
  if (r == ncclSuccess) {
    e = cudaMemcpyAsync(hs, gathered, sizeof(cudaIpcMemHandle_t) * size, cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  }
  cudaFree(ids);
  bool ok = r == ncclSuccess && e == cudaSuccess;
  for (int p = 0; ok && p < size; p++) {
    if (p == rank) { ar->peer[p] = ar->base; continue; }
    e = cudaIpcOpenMemHandle(&ar->peer[p], hs[p], cudaIpcMemLazyEnablePeerAccess);
    ok = e == cudaSuccess;
  }
  if (!ok) cudaGetLastError();
  // the ranks agree on using it: a rank that could not map a peer makes everyone keep NCCL
  float *flag = nullptr;
  float hflag = ok ? 0.f : 1.f;
  if (cudaMalloc(&flag, sizeof(float)) == cudaSuccess &&
      cudaMemcpyAsync(flag, &hflag, sizeof(float), cudaMemcpyHostToDevice, s) == cudaSuccess &&
      api.all_reduce(flag, flag, 1, ncclFloat32, ncclSum, static_cast<ncclComm_t>(comm), s) == ncclSuccess &&
      cudaMemcpyAsync(&hflag, flag, sizeof(float), cudaMemcpyDeviceToHost, s) == cudaSuccess &&
      cudaStreamSynchronize(s) == cudaSuccess && hflag == 0.f) {
    cudaFree(flag);
    *out = ar;
    return 0;
  }
  if (flag) cudaFree(flag);
  *why = r != ncclSuccess ? nccl_err(r) : e != cudaSuccess ? cudaGetErrorString(e) : "a peer could not map this rank's buffer";
  for (int p = 0; p < size; p++)
    if (p != rank && ar->peer[p]) cudaIpcCloseMemHandle(ar->peer[p]);
  cudaFree(ar->base);
  delete ar;
  cudaGetLastError();
  return -1;
}

cudaError_t tp_ar_sum(TpAr *ar, float *x, int64_t n, unsigned *status, cudaStream_t s, bool pdl) {
  if (n > ar->cap) return cudaErrorInvalidValue;
  ArArgs a{};
  a.x = x;
  for (int p = 0; p < ar->size; p++) a.peer[p] = reinterpret_cast<uint8_t *>(ar->peer[p]);
  a.mine = reinterpret_cast<uint8_t *>(ar->base);
  a.status = status;
  a.n = n;
  a.cap = ar->cap;
  a.rank = ar->rank;
  a.size = ar->size;
  // slices of 256 values: a one-token hidden state (5120) spreads over 20 CTAs, each with its own
  // peer stores and stamp polls in flight
  int64_t ctas = (n + kArThreads - 1) / kArThreads;
  if (ctas > kArMaxCtas) ctas = kArMaxCtas;
  if (ctas < 1) ctas = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)ctas);
  cfg.blockDim = dim3(kArThreads);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, tp_ar_kernel, a);
}

// Failure detection without a fault: the all-reduce kernel on this GPU against a phantom second
// rank whose stamps never come.  The kernel's bounded wait expires (2 s), it sets ST_PEER_TIMEOUT in
// `status`, finishes and returns; the caller reads the status word as after any pass.
int tp_ar_phantom_wait(unsigned *status, cudaStream_t s, const char **why) {
  const int64_t cap = 1024;
  void *b0 = nullptr, *b1 = nullptr, *x = nullptr;
  cudaError_t e = cudaMalloc(&b0, ar_bytes(cap));
  if (e == cudaSuccess) e = cudaMalloc(&b1, ar_bytes(cap));
  if (e == cudaSuccess) e = cudaMalloc(&x, cap * sizeof(float));
  if (e == cudaSuccess) e = cudaMemsetAsync(b0, 0, ar_bytes(cap), s);
  if (e == cudaSuccess) e = cudaMemsetAsync(b1, 0, ar_bytes(cap), s);
  if (e == cudaSuccess) e = cudaMemsetAsync(x, 0, cap * sizeof(float), s);
  if (e == cudaSuccess) {
    ArArgs a{};
    a.x = reinterpret_cast<float *>(x);
    a.peer[0] = reinterpret_cast<uint8_t *>(b0);     // this rank
    a.peer[1] = reinterpret_cast<uint8_t *>(b1);     // the phantom: it never stamps b0's slots
    a.mine = a.peer[0];
    a.status = status;
    a.n = cap;
    a.cap = cap;
    a.rank = 0;
    a.size = 2;
    tp_ar_kernel<<<1, kArThreads, 0, s>>>(a);
    e = cudaGetLastError();
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  }
  for (void *p : {b0, b1, x})
    if (p) cudaFree(p);
  if (e != cudaSuccess) { *why = cudaGetErrorString(e); return -1; }
  return 0;
}

// Every rank calls this after its last pass; the NCCL all-reduce is the barrier that keeps a rank
// from freeing its buffer while a peer may still read it.
void tp_ar_destroy(TpAr *ar, void *comm, cudaStream_t s) {
  if (!ar) return;
  const NcclApi &api = nccl();
  float *flag = nullptr;
  if (api.ok && comm && cudaMalloc(&flag, sizeof(float)) == cudaSuccess) {
    if (cudaMemsetAsync(flag, 0, sizeof(float), s) == cudaSuccess &&
        api.all_reduce(flag, flag, 1, ncclFloat32, ncclSum, static_cast<ncclComm_t>(comm), s) == ncclSuccess)
      cudaStreamSynchronize(s);
    cudaFree(flag);
  }
  for (int p = 0; p < ar->size; p++)
    if (p != ar->rank && ar->peer[p]) cudaIpcCloseMemHandle(ar->peer[p]);
  cudaFree(ar->base);
  delete ar;
  cudaGetLastError();
}

}  // namespace zllm
