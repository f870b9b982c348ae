// zllm_attn_decode_noalloc: decode attention whose scratch is a fixed array compiled into the
// library, so the call itself allocates no device memory (declared in include/zllm.h).
//
// zllm_attn_decode takes the split-context partial results and the merge counters from the
// context's scratch, which grows with cudaMalloc / cudaFree the first time a larger launch comes
// along.  Some callers cannot let that happen inside a step: a server that has handed all free HBM
// to its KV pool before it starts decoding (a cudaMalloc there fails with out-of-memory in the
// middle of a request), and a host that owns the device memory through its own allocator, where a
// cudaFree behind its back synchronizes the whole device and stalls every other stream.  This
// variant runs the same kernel with the same split of the context (so results are identical) but
// keeps its scratch in `g_attn_scratch` below.
//
// Limits: the partial results of one call must fit in kPartialBytes (4 MiB) and the call may cover
// at most kMaxGroups (4096) (sequence, KV head) pairs; larger requests are rejected with ZLLM_E_ARG
// before anything is launched.  All calls on one device share the array: two calls that overlap in
// time (different streams, contexts or threads on the same device) race on it, so callers order
// them (one stream, or events).
//
// When the array comes into being: this file is its own CUDA module, and under lazy module loading
// (the CUDA default) a module's device variables are allocated when the module is first touched.
// zllm_init touches it -- zllm_noalloc_setup looks the array's address up with cudaGetSymbolAddress,
// the context's device current -- so the 4 MiB + 16 KiB are taken when the first context on a
// device is created (an out-of-memory there fails zllm_init, not a decode step), every later call
// of zllm_attn_decode_noalloc reuses the cached address and allocates nothing, and the device holds
// the array until the process exits.
#include <mutex>

#include "../../include/zllm.h"
#include "capi_internal.h"
#include "internal.h"

namespace {

constexpr size_t kPartialBytes = 4u << 20;
constexpr int kMaxGroups = 4096;
constexpr int kMaxDevices = 64;

// [partials: kPartialBytes][merge counters: kMaxGroups int32]
__device__ __align__(256) unsigned char g_attn_scratch[kPartialBytes + kMaxGroups * sizeof(int32_t)];

std::mutex g_addr_mu;
void *g_addr[kMaxDevices] = {};

// the array's device address on `device`, looked up once per device with that device current
int lookup(zllm_ctx *c, int device, void **out) {
  if (device < 0 || device >= kMaxDevices) {
    zllm_set_error(c, "fixed attention scratch: device %d out of range (max %d)", device, kMaxDevices - 1);
    return ZLLM_E_ARG;
  }
  std::lock_guard<std::mutex> lock(g_addr_mu);
  if (!g_addr[device]) {
    int prev = 0;
    cudaError_t e = cudaGetDevice(&prev);
    if (e == cudaSuccess && prev != device) e = cudaSetDevice(device);
    void *p = nullptr;
    if (e == cudaSuccess) e = cudaGetSymbolAddress(&p, g_attn_scratch);
    if (prev != device) cudaSetDevice(prev);
    if (e != cudaSuccess) return zllm_cuda_fail(c, e, "cudaGetSymbolAddress(fixed attention scratch)");
    g_addr[device] = p;
  }
  *out = g_addr[device];
  return ZLLM_OK;
}

}  // namespace

int zllm_noalloc_setup(zllm_ctx *c) {
  void *p = nullptr;
  return lookup(c, c->device, &p);
}

extern "C" int zllm_attn_decode_noalloc(zllm_ctx *c, const zllm_attn_geom *g, const float *q, const void *kcache,
                                        const void *vcache, const int32_t *npos, int nseq, int max_pos, float *out,
                                        void *stream) {
  if (!c) return ZLLM_E_ARG;
  if (!g || g->n_head <= 0 || g->n_head_kv <= 0 || g->n_head % g->n_head_kv || g->head_dim <= 0 || g->ctx <= 0 ||
      g->n_rot <= 0 || g->n_rot > g->head_dim || g->n_rot % 2) {
    zllm_set_error(c, "bad attention geometry");
    return ZLLM_E_ARG;
  }
  if (!q || !kcache || !vcache || !npos || !out || nseq < 1 || max_pos < 0 || max_pos > g->ctx) {
    zllm_set_error(c, "zllm_attn_decode_noalloc: bad argument");
    return ZLLM_E_ARG;
  }
  const int group = g->n_head / g->n_head_kv;
  if (!zllm::attn_supported(g->head_dim, group)) {
    zllm_set_error(c, "zllm_attn_decode_noalloc: head_dim %d / group %d not supported (head_dim 64 or 128, group 1, "
                      "2, 4 or 8)", g->head_dim, group);
    return ZLLM_E_UNSUPPORTED;
  }
  const int64_t groups = (int64_t)nseq * g->n_head_kv;
  if (groups > kMaxGroups) {
    zllm_set_error(c, "zllm_attn_decode_noalloc: %lld (sequence, KV head) pairs exceed the fixed scratch (max %d)",
                   (long long)groups, kMaxGroups);
    return ZLLM_E_ARG;
  }
  const int nsplit = zllm_attn_splits(c, g, nseq, max_pos);     // the same split as zllm_attn_decode
  const size_t part_bytes = (size_t)groups * nsplit * group * (g->head_dim + 2) * sizeof(float);
  if (part_bytes > kPartialBytes) {
    zllm_set_error(c, "zllm_attn_decode_noalloc: %zu bytes of partial results exceed the fixed scratch (max %zu)",
                   part_bytes, kPartialBytes);
    return ZLLM_E_ARG;
  }
  void *base = nullptr;
  int rc = lookup(c, c->device, &base);        // cached by zllm_init: no allocation, no module load here
  if (rc) return rc;
  float *partial = (float *)base;
  int32_t *counters = (int32_t *)((unsigned char *)base + kPartialBytes);
  cudaStream_t s = stream ? (cudaStream_t)stream : c->stream;
  // the merge counters must start at zero; clear the ones this launch uses
  cudaError_t e = cudaMemsetAsync(counters, 0, (size_t)groups * sizeof(int32_t), s);
  if (e != cudaSuccess) return zllm_cuda_fail(c, e, "zllm_attn_decode_noalloc: counter clear");
  return zllm_attn_launch(c, g, q, kcache, vcache, npos, nseq, nsplit, out, partial, counters, s, nullptr, nullptr);
}
