// Definitions of the opaque C-ABI handles (shared by the capi*.cu files).
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <set>

#include "../../include/zllm.h"
#include "internal.h"

constexpr int kScratchSlots = 16;

struct zllm_ctx {
  int device = 0;
  int num_sms = 148;
  cudaStream_t stream = nullptr;
  unsigned *status_dev = nullptr;    // device word the kernels report timeouts into (atomicOr)
  unsigned *status_host = nullptr;   // pinned host copy of it, read back on the stream (zllm_finish)
  void *scratch[kScratchSlots] = {};
  size_t scratch_bytes[kScratchSlots] = {};
  char err[512] = {0};
  std::set<struct zllm_weight *> weights;   // live uploads: zllm_destroy releases their device memory
};

struct zllm_weight {
  zllm_ctx *ctx = nullptr;
  zllm::DevMatrix m{};
  size_t bytes = 0;
  bool owns = true;
  int gemm_ok = -1;      // k-quant: the tensor-core GEMM may take it (1), not (0), not yet known (-1)
  float gemm_wscale = 1.f;   // power of two applied to its dequantized values in f16
  bool gemm_kx = false;      // it takes the exact-A GEMM (launch_gemm_kx) rather than the hi / lo one
  float gemm_mscale = 1.f;   // the exact-A GEMM's power of two for the min values
  // zllm_matvec's call on this weight recorded as a CUDA graph (copy in, GEMV, copies out), replayed
  // while the host buffers and the context scratch it used stay the same
  cudaGraphExec_t mv_exec = nullptr;
  const void *mv_key[11] = {};
  const void *mv_seen[11] = {};   // the previous call's addresses
};

// Whether the tensor-core GEMM may take this k-quant weight (computed once, synchronously).
int zllm_weight_gemm_ok(zllm_ctx *c, zllm_weight *w);
size_t gemm_act_bytes(const zllm_weight *w, int ntok);
cudaError_t gemm_run(const zllm_weight *w, const zllm::ActView &a, int ntok, void *bbuf, float *y, int64_t y_stride,
                     const float *y_add, unsigned *status, cudaStream_t st, bool swiglu);

void zllm_set_error(zllm_ctx *c, const char *fmt, ...);
int zllm_cuda_fail(zllm_ctx *c, cudaError_t e, const char *what);
int zllm_scratch(zllm_ctx *c, int slot, size_t bytes, void **out);
int zllm_check_status(zllm_ctx *c);
// Enqueue the status word's copy into pinned host memory on `s`, synchronize `s` once and report a
// timeout bit: the end of a host-buffer call without a second, blocking copy.
int zllm_finish(zllm_ctx *c, cudaStream_t s);
// Loads the fixed attention scratch of zllm_attn_decode_noalloc on the context's device and caches
// its address (capi_noalloc.cu); zllm_init calls it, so no later call of that entry point allocates.
int zllm_noalloc_setup(zllm_ctx *c);
int zllm_attn_splits(const zllm_ctx *c, const zllm_attn_geom *g, int nseq, int max_pos);
int zllm_attn_launch(zllm_ctx *c, const zllm_attn_geom *g, const float *q, const void *kcache, const void *vcache,
                     const int32_t *npos, int nseq, int nsplit, float *out, float *partial, int32_t *counters,
                     cudaStream_t s, const int32_t *seq, const zllm::KvPages *pages);
