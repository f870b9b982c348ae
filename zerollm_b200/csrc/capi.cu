// extern "C" entry points of libzllm_cuda.so (declared in include/zllm.h).
#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <new>

#include "../../include/zllm.h"
#include "capi_internal.h"
#include "common.cuh"
#include "internal.h"

using namespace zllm;

// ------------------------------------------------------------------------------------ helpers
void zllm_set_error(zllm_ctx *c, const char *fmt, ...) {
  if (!c) return;
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(c->err, sizeof(c->err), fmt, ap);
  va_end(ap);
}

int zllm_cuda_fail(zllm_ctx *c, cudaError_t e, const char *what) {
  zllm_set_error(c, "%s: %s", what, cudaGetErrorString(e));
  return e == cudaErrorMemoryAllocation ? ZLLM_E_OOM : ZLLM_E_CUDA;
}

// Grow-only device scratch buffer.
int zllm_scratch(zllm_ctx *c, int slot, size_t bytes, void **out) {
  if (slot < 0 || slot >= kScratchSlots) return ZLLM_E_ARG;
  if (c->scratch_bytes[slot] < bytes) {
    if (c->scratch[slot]) {
      cudaStreamSynchronize(c->stream);
      cudaFree(c->scratch[slot]);
      c->scratch[slot] = nullptr;
      c->scratch_bytes[slot] = 0;
    }
    size_t want = bytes < 4096 ? 4096 : bytes;
    cudaError_t e = cudaMalloc(&c->scratch[slot], want);
    if (e != cudaSuccess) return zllm_cuda_fail(c, e, "cudaMalloc(scratch)");
    c->scratch_bytes[slot] = want;
  }
  *out = c->scratch[slot];
  return ZLLM_OK;
}

static cudaStream_t pick(zllm_ctx *c, void *stream) { return stream ? (cudaStream_t)stream : c->stream; }
// Programmatic dependent launch is used on real streams only: the legacy default stream (handle 0,
// passed through `zllm_stream`-less callers) keeps plain stream ordering.
static bool pdl_ok(cudaStream_t s) { return s != nullptr && s != cudaStreamLegacy && s != cudaStreamPerThread; }

namespace {
// zllm_matvec's recorded call on mapped pinned buffers: the GPU fetches x itself (the product is
// launched programmatically behind it and prefetches its weights meanwhile), and the status word is
// stored into the mapped pinned host word once the product has finished
__global__ void mv_fetch_kernel(const float *__restrict__ src, float *__restrict__ dst, int64_t n) {
  zllm::pdl_launch_dependents();
  const int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x, step = (int64_t)gridDim.x * blockDim.x;
  if (((uintptr_t)src | (uintptr_t)dst) % 16 == 0) {
    for (int64_t i = t; i < n / 4; i += step)
      reinterpret_cast<float4 *>(dst)[i] = reinterpret_cast<const float4 *>(src)[i];
    for (int64_t i = n / 4 * 4 + t; i < n; i += step) dst[i] = src[i];
  } else {
    for (int64_t i = t; i < n; i += step) dst[i] = src[i];
  }
}
__global__ void mv_status_kernel(const unsigned *st, unsigned *out) {
  zllm::pdl_wait();
  *out = *reinterpret_cast<const volatile unsigned *>(st);
}
}  // namespace

// ------------------------------------------------------------------------------------ context
extern "C" const char *zllm_version(void) { return "zllm-b200 0.1 (sm_100a)"; }

extern "C" int zllm_init(int device, zllm_ctx **out) {
  if (!out) return ZLLM_E_ARG;
  *out = nullptr;
  zllm_ctx *c = new (std::nothrow) zllm_ctx();
  if (!c) return ZLLM_E_OOM;
  c->device = device;
  cudaError_t e = cudaSetDevice(device);
  if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&c->num_sms, cudaDevAttrMultiProcessorCount, device);
  // the status word lives in device memory: device atomics on mapped host memory are not atomic
  // (and may be lost) on PCIe hosts
  if (e == cudaSuccess) e = cudaMalloc((void **)&c->status_dev, sizeof(unsigned));
  if (e == cudaSuccess) e = cudaMallocHost((void **)&c->status_host, sizeof(unsigned));
  if (e == cudaSuccess) e = cudaMemsetAsync(c->status_dev, 0, sizeof(unsigned), c->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
  if (e != cudaSuccess) {
    fprintf(stderr, "zllm_init: %s\n", cudaGetErrorString(e));
    int rc = e == cudaErrorMemoryAllocation ? ZLLM_E_OOM : ZLLM_E_CUDA;
    zllm_destroy(c);
    return rc;
  }
  // the fixed scratch of zllm_attn_decode_noalloc comes into being here, not inside a decode step
  if (int rc = zllm_noalloc_setup(c)) {
    fprintf(stderr, "zllm_init: %s\n", c->err);
    zllm_destroy(c);
    return rc;
  }
  *out = c;
  return ZLLM_OK;
}

static void mv_forget(zllm_weight *w);

extern "C" void zllm_destroy(zllm_ctx *c) {
  if (!c) return;
  cudaSetDevice(c->device);
  if (c->stream) cudaStreamSynchronize(c->stream);
  // weights may outlive their context: free their device memory now and detach them, so a later
  // zllm_weight_free only releases the handle
  for (zllm_weight *w : c->weights) {
    mv_forget(w);
    if (w->m.data && w->owns) cudaFree(w->m.data);
    w->m.data = nullptr;
    w->ctx = nullptr;
  }
  c->weights.clear();
  for (int i = 0; i < kScratchSlots; i++)
    if (c->scratch[i]) cudaFree(c->scratch[i]);
  if (c->status_dev) cudaFree(c->status_dev);
  if (c->status_host) cudaFreeHost(c->status_host);
  if (c->stream) cudaStreamDestroy(c->stream);
  delete c;
}

extern "C" const char *zllm_last_error(const zllm_ctx *c) { return c ? c->err : "no context"; }
extern "C" void *zllm_stream(zllm_ctx *c) { return c ? (void *)c->stream : nullptr; }

int zllm_check_status(zllm_ctx *c) {
  unsigned st = 0;
  cudaError_t e = cudaMemcpy(&st, c->status_dev, sizeof(unsigned), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return zllm_cuda_fail(c, e, "reading the device status word");
  if (st) {
    cudaMemset(c->status_dev, 0, sizeof(unsigned));
    if (st == ST_BAD_ARGS) {
      zllm_set_error(c, "a kernel found an index out of range in device data (status 0x%x: a paged-KV table entry or a "
                        "position past its table row) and read page 0 instead", st);
      return ZLLM_E_ARG;
    }
    zllm_set_error(c, "device wait timed out (status 0x%x): a bulk copy, a stage hand-off or a peer GPU's all-reduce "
                      "slice did not complete within 2 s; the kernel drained its copies and returned", st);
    return ZLLM_E_TIMEOUT;
  }
  return ZLLM_OK;
}

int zllm_finish(zllm_ctx *c, cudaStream_t s) {
  *c->status_host = 0;
  cudaError_t e = cudaMemcpyAsync(c->status_host, c->status_dev, sizeof(unsigned), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return zllm_cuda_fail(c, e, "reading the device status word");
  if (*c->status_host) return zllm_check_status(c);     // rare: clear the word and report, as zllm_sync does
  return ZLLM_OK;
}

extern "C" int zllm_peer_wait_selftest(zllm_ctx *c) {
  if (!c) return ZLLM_E_ARG;
  cudaSetDevice(c->device);
  const char *why = "";
  if (tp_ar_phantom_wait(c->status_dev, c->stream, &why)) {
    zllm_set_error(c, "zllm_peer_wait_selftest: %s", why);
    return ZLLM_E_CUDA;
  }
  return zllm_check_status(c);
}

extern "C" int zllm_sync(zllm_ctx *c) {
  if (!c) return ZLLM_E_ARG;
  cudaError_t e = cudaStreamSynchronize(c->stream);
  if (e != cudaSuccess) return zllm_cuda_fail(c, e, "cudaStreamSynchronize");
  return zllm_check_status(c);
}

// ------------------------------------------------------------------------------------ weights
extern "C" int zllm_weight_upload(zllm_ctx *c, int type, int64_t rows, int64_t cols, const void *host, size_t nbytes,
                                  zllm_weight **out) {
  if (!c || !out || !host || rows <= 0 || cols <= 0) { zllm_set_error(c, "zllm_weight_upload: bad argument"); return ZLLM_E_ARG; }
  *out = nullptr;
  if (!type_supported(type)) {
    zllm_set_error(c, "reference kernels: unsupported tensor type %d (supported: F32, F16, BF16, Q4_0, Q5_0, Q8_0, Q4_K, Q5_K, Q6_K)", type);
    return ZLLM_E_UNSUPPORTED;
  }
  const int64_t rb = raw_row_bytes(type, cols);
  if (rb < 0) { zllm_set_error(c, "row length %lld is not a multiple of the block size of type %d", (long long)cols, type); return ZLLM_E_ARG; }
  if ((size_t)(rb * rows) != nbytes) {
    zllm_set_error(c, "zllm_weight_upload: %zu bytes given, %lld expected", nbytes, (long long)(rb * rows));
    return ZLLM_E_ARG;
  }
  zllm_weight *w = new (std::nothrow) zllm_weight();
  if (!w) return ZLLM_E_OOM;
  w->ctx = c;
  w->m.type = type;
  w->m.rows = rows;
  w->m.cols = cols;
  w->m.row_stride = dev_row_stride(type, cols);
  w->bytes = (size_t)dev_matrix_bytes(type, rows, cols);
  cudaSetDevice(c->device);
  cudaError_t e = cudaMalloc((void **)&w->m.data, w->bytes);
  if (e != cudaSuccess) { delete w; return zllm_cuda_fail(c, e, "cudaMalloc(weight)"); }
  void *staging = nullptr;
  const bool direct = w->m.row_stride == rb && (type == T_F16 || type == T_BF16 || type == T_F32);
  if (direct) {
    e = cudaMemcpyAsync(w->m.data, host, nbytes, cudaMemcpyHostToDevice, c->stream);
  } else {
    e = cudaMalloc(&staging, nbytes);
    if (e == cudaSuccess) e = cudaMemcpyAsync(staging, host, nbytes, cudaMemcpyHostToDevice, c->stream);
    if (e == cudaSuccess) e = repack_upload(w->m, staging, c->stream);
  }
  if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
  if (staging) cudaFree(staging);
  if (e != cudaSuccess) {
    cudaFree(w->m.data);
    delete w;
    return zllm_cuda_fail(c, e, "zllm_weight_upload");
  }
  c->weights.insert(w);
  *out = w;
  return ZLLM_OK;
}

// Drop zllm_matvec's recorded call on this weight (the weight or its context is going away).
static void mv_forget(zllm_weight *w) {
  if (w->mv_exec) cudaGraphExecDestroy(w->mv_exec);
  w->mv_exec = nullptr;
  memset(w->mv_key, 0, sizeof w->mv_key);
  memset(w->mv_seen, 0, sizeof w->mv_seen);
}

extern "C" void zllm_weight_free(zllm_weight *w) {
  if (!w) return;
  if (w->ctx) {
    cudaSetDevice(w->ctx->device);
    cudaStreamSynchronize(w->ctx->stream);
    mv_forget(w);
    if (w->m.data && w->owns) cudaFree(w->m.data);
    w->ctx->weights.erase(w);
  }
  delete w;
}

extern "C" int zllm_weight_info(const zllm_weight *w, int *type, int64_t *rows, int64_t *cols, size_t *bytes) {
  if (!w) return ZLLM_E_ARG;
  if (type) *type = w->m.type;
  if (rows) *rows = w->m.rows;
  if (cols) *cols = w->m.cols;
  if (bytes) *bytes = w->bytes;
  return ZLLM_OK;
}

// ------------------------------------------------------------------------------------ kernels
extern "C" int zllm_quantize_act(zllm_ctx *c, const float *x, int64_t k, int ntok, int8_t *xq, float *xd, int32_t *xs,
                                 void *stream) {
  if (!c || !x || !xq || !xd || !xs || k <= 0 || k % 32 || ntok < 1) {
    zllm_set_error(c, "zllm_quantize_act: bad argument (k must be a positive multiple of 32)");
    return ZLLM_E_ARG;
  }
  cudaStream_t st = pick(c, stream);
  cudaError_t e = launch_quantize(x, k, ntok, xq, xd, xs, c->status_dev, st, pdl_ok(st));
  return e == cudaSuccess ? ZLLM_OK : zllm_cuda_fail(c, e, "quantize_act launch");
}

int zllm_weight_gemm_ok(zllm_ctx *c, zllm_weight *w) {
  if (w->gemm_ok >= 0) return w->gemm_ok;
  if (!gemm_kq_supported(w->m)) return w->gemm_ok = 0;
  void *buf = nullptr;
  if (zllm_scratch(c, 13, 16, &buf)) return 0;
  unsigned bits[3] = {0, 0, 0};
  unsigned *d = reinterpret_cast<unsigned *>(buf);
  cudaError_t e = launch_kq_bound(w->m, d, c->stream);
  if (e == cudaSuccess) e = launch_kx_info(w->m, d + 1, c->stream);
  if (e == cudaSuccess) e = cudaMemcpyAsync(bits, buf, 12, cudaMemcpyDeviceToHost, c->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
  if (e != cudaSuccess) { cudaGetLastError(); return 0; }
  float bound, mbound;
  memcpy(&bound, &bits[0], 4);
  memcpy(&mbound, &bits[1], 4);
  w->gemm_wscale = gemm_weight_scale(bound);
  w->gemm_mscale = gemm_weight_scale(mbound);
  // exact A: Q4_K / Q5_K always (sc * q <= 63 * 31), Q6_K while (q - 32) * scale stays within 2048
  w->gemm_kx = w->m.type == zllm::T_Q6_K ? bits[2] <= 64 : true;
  return w->gemm_ok = bound < 3.0e38f ? 1 : 0;          // NaN or infinite scales: the exact kernel
}

// The tensor-core GEMM of a qualifying weight on ntok >= kGemmMinTokens tokens of (xq, xd, xs):
// activation tiles in bbuf (gemm_act_bytes), then the product.
size_t gemm_act_bytes(const zllm_weight *w, int ntok) {
  return w->gemm_kx ? gemm_bx_bytes(w->m.cols, ntok, w->m.type, w->m.rows) : gemm_b_bytes(w->m.cols, ntok);
}
cudaError_t gemm_run(const zllm_weight *w, const ActView &a, int ntok, void *bbuf, float *y, int64_t y_stride,
                     const float *y_add, unsigned *status, cudaStream_t st, bool swiglu) {
  if (w->gemm_kx) {
    cudaError_t e = launch_gemm_prep_kx(a, ntok, w->m.type, w->m.rows, bbuf, st);
    return e == cudaSuccess ? launch_gemm_kx(w->m, bbuf, ntok, y, y_stride, y_add, w->gemm_mscale, status, st, swiglu) : e;
  }
  cudaError_t e = launch_gemm_prep(a, ntok, bbuf, st);
  return e == cudaSuccess ? launch_gemm_kq(w->m, bbuf, ntok, y, y_stride, y_add, w->gemm_wscale, status, st, swiglu) : e;
}

extern "C" int zllm_mm(zllm_ctx *c, const zllm_weight *w, const int8_t *xq, const float *xd, const int32_t *xs,
                       const float *x, int ntok, float *y, int64_t y_stride, const float *y_add, void *stream) {
  if (!c || !w || !y || ntok < 1) { zllm_set_error(c, "zllm_mm: bad argument"); return ZLLM_E_ARG; }
  if (!w->m.data) { zllm_set_error(c, "zllm_mm: the weight's context was destroyed"); return ZLLM_E_STATE; }
  const bool q = type_quantized(w->m.type);
  // quantized weights read (xq, xd, xs); a one-token k-quant product may pass x alone instead and
  // the GEMV quantizes it
  const bool fused = q && !xq && x && ntok == 1 && kq_type(w->m.type);
  if (q ? (!fused && (!xq || !xd || !xs)) : !x) {
    zllm_set_error(c, "zllm_mm: missing activation for this weight type");
    return ZLLM_E_ARG;
  }
  if (ntok > 1 && y_stride < w->m.rows) { zllm_set_error(c, "zllm_mm: y_stride < rows"); return ZLLM_E_ARG; }
  ActView a{fused ? nullptr : xq, xd, xs, x, w->m.cols};
  const char *why = "";
  cudaStream_t st = pick(c, stream);
  if (ntok >= kGemmMinTokens && xq && (uintptr_t)xq % 8 == 0 && kq_type(w->m.type) &&
      zllm_weight_gemm_ok(c, const_cast<zllm_weight *>(w))) {
    // kGemmMinTokens or more tokens: the tensor-core GEMM on f16 tiles of the activation
    void *bbuf = nullptr;
    int rc = zllm_scratch(c, 14, gemm_act_bytes(w, ntok), &bbuf);
    if (rc) return rc;
    cudaError_t e = gemm_run(w, a, ntok, bbuf, y, y_stride, y_add, c->status_dev, st, false);
    return e == cudaSuccess ? ZLLM_OK : zllm_cuda_fail(c, e, "gemm launch");
  }
  cudaError_t e = launch_gemv(w->m, a, ntok, y, y_stride, y_add, c->status_dev, c->num_sms, st, pdl_ok(st), &why);
  if (e == cudaErrorInvalidValue && why[0]) { zllm_set_error(c, "zllm_mm: %s", why); return ZLLM_E_UNSUPPORTED; }
  return e == cudaSuccess ? ZLLM_OK : zllm_cuda_fail(c, e, "gemv launch");
}

extern "C" int zllm_mm_fused(zllm_ctx *c, const zllm_weight *w, const float *x, const float *norm_w, double eps,
                             int swiglu, float *y, const float *y_add, void *stream) {
  if (!c || !w || !x || !y) { zllm_set_error(c, "zllm_mm_fused: bad argument"); return ZLLM_E_ARG; }
  if (!w->m.data) { zllm_set_error(c, "zllm_mm_fused: the weight's context was destroyed"); return ZLLM_E_STATE; }
  if (!kq_type(w->m.type)) { zllm_set_error(c, "zllm_mm_fused: Q4_K, Q5_K or Q6_K weights only"); return ZLLM_E_UNSUPPORTED; }
  GemvFuse fz;
  fz.norm_w = norm_w;
  fz.eps = eps;
  fz.swiglu = swiglu != 0;
  ActView a{nullptr, nullptr, nullptr, x, w->m.cols};
  const char *why = "";
  cudaStream_t st = pick(c, stream);
  cudaError_t e = launch_gemv_kq_ex(w->m, a, 1, y, w->m.rows, y_add, fz, c->status_dev, c->num_sms, st, pdl_ok(st), &why);
  if (e == cudaErrorInvalidValue && why[0]) { zllm_set_error(c, "zllm_mm_fused: %s", why); return ZLLM_E_ARG; }
  return e == cudaSuccess ? ZLLM_OK : zllm_cuda_fail(c, e, "zllm_mm_fused launch");
}

extern "C" int zllm_rmsnorm_quant(zllm_ctx *c, const float *x, const float *w, int n, int ntok, double eps, float *xb,
                                  int8_t *xq, float *xd, int32_t *xs, void *stream) {
  const bool q = xq || xd || xs;
  if (!c || !x || !w || n < 1 || ntok < 1 || (!xb && !q) || (q && (!xq || !xd || !xs || n % 32))) {
    zllm_set_error(c, "zllm_rmsnorm_quant: bad argument");
    return ZLLM_E_ARG;
  }
  cudaStream_t st = pick(c, stream);
  cudaError_t e = launch_rmsnorm_quant(x, w, n, ntok, eps, xb, xq, xd, xs, st, pdl_ok(st));
  return e == cudaSuccess ? ZLLM_OK : zllm_cuda_fail(c, e, "zllm_rmsnorm_quant launch");
}

extern "C" int zllm_swiglu_quant(zllm_ctx *c, const float *gate, const float *up, int n, int ntok, int64_t stride,
                                 float *hb, int8_t *xq, float *xd, int32_t *xs, void *stream) {
  const bool q = xq || xd || xs;
  if (!c || !gate || !up || n < 32 || n % 32 || ntok < 1 || stride < n || (!hb && !q) || (q && (!xq || !xd || !xs))) {
    zllm_set_error(c, "zllm_swiglu_quant: bad argument (n a positive multiple of 32, stride >= n)");
    return ZLLM_E_ARG;
  }
  cudaStream_t st = pick(c, stream);
  cudaError_t e = launch_swiglu_quant(gate, up, n, ntok, stride, hb, xq, xd, xs, st, pdl_ok(st));
  return e == cudaSuccess ? ZLLM_OK : zllm_cuda_fail(c, e, "zllm_swiglu_quant launch");
}

extern "C" int zllm_gemm_f16(zllm_ctx *c, const void *A, const void *B, int64_t m, int64_t n, int64_t k, float *D,
                             void *stream) {
  if (!c || !A || !B || !D || m < 1 || n < 1 || k < 64 || k % 64) {
    zllm_set_error(c, "zllm_gemm_f16: bad argument (k must be a positive multiple of 64)");
    return ZLLM_E_ARG;
  }
  if (((uintptr_t)A | (uintptr_t)B) % 16) { zllm_set_error(c, "zllm_gemm_f16: A and B must be 16-byte aligned"); return ZLLM_E_ARG; }
  void *scr = nullptr;
  int rc = zllm_scratch(c, 15, gemm_f16_scratch_bytes(m, n, k), &scr);
  if (rc) return rc;
  cudaError_t e = launch_gemm_f16(reinterpret_cast<const uint16_t *>(A), reinterpret_cast<const uint16_t *>(B), m, n, k, D, scr,
                                  c->status_dev, pick(c, stream));
  return e == cudaSuccess ? ZLLM_OK : zllm_cuda_fail(c, e, "gemm_f16 launch");
}

extern "C" int zllm_matvec(zllm_ctx *c, const zllm_weight *w, const float *x_host, int ntok, float *y_host) {
  if (!c || !w || !x_host || !y_host || ntok < 1) { zllm_set_error(c, "zllm_matvec: bad argument"); return ZLLM_E_ARG; }
  cudaSetDevice(c->device);
  const int64_t K = w->m.cols, R = w->m.rows;
  void *xs_, *xq_, *xd_, *xsum_, *y_;
  int rc;
  if ((rc = zllm_scratch(c, 0, sizeof(float) * K * ntok, &xs_))) return rc;
  if ((rc = zllm_scratch(c, 1, (size_t)K * ntok, &xq_))) return rc;
  if ((rc = zllm_scratch(c, 2, sizeof(float) * (K / 32 + 1) * ntok, &xd_))) return rc;
  if ((rc = zllm_scratch(c, 3, sizeof(int32_t) * (K / 32 + 1) * ntok, &xsum_))) return rc;
  if ((rc = zllm_scratch(c, 4, sizeof(float) * R * ntok, &y_))) return rc;
  // one token on a k-quant: the GEMV quantizes x itself
  const bool q = type_quantized(w->m.type), fused = q && ntok == 1 && kq_type(w->m.type);
  // the whole call: x in, (quantization,) the product, y and the status word out; y_dev: y_host's
  // device address when the recorded call writes it straight into the mapped pinned buffer
  float *y_dev = nullptr;
  const float *x_dev = nullptr;
  unsigned *status_map = nullptr;
  auto enqueue = [&]() -> int {
    cudaError_t e;
    if (x_dev) {
      const int64_t n = K * ntok;
      mv_fetch_kernel<<<(unsigned)std::min<int64_t>((n / 4 + 255) / 256 + 1, 64), 256, 0, c->stream>>>(x_dev, (float *)xs_, n);
      e = cudaGetLastError();
    } else {
      e = cudaMemcpyAsync(xs_, x_host, sizeof(float) * K * ntok, cudaMemcpyHostToDevice, c->stream);
    }
    if (e != cudaSuccess) return zllm_cuda_fail(c, e, "zllm_matvec: x in");
    int r;
    if (q && !fused &&
        (r = zllm_quantize_act(c, (const float *)xs_, K, ntok, (int8_t *)xq_, (float *)xd_, (int32_t *)xsum_, c->stream)))
      return r;
    if ((r = zllm_mm(c, w, fused ? nullptr : (const int8_t *)xq_, (const float *)xd_, (const int32_t *)xsum_,
                     (const float *)xs_, ntok, y_dev ? y_dev : (float *)y_, R, nullptr, c->stream)))
      return r;
    if (!y_dev) e = cudaMemcpyAsync(y_host, y_, sizeof(float) * R * ntok, cudaMemcpyDeviceToHost, c->stream);
    if (e == cudaSuccess && status_map) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(1);
      cfg.blockDim = dim3(1);
      cfg.stream = c->stream;
      cudaLaunchAttribute at[1];
      at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
      at[0].val.programmaticStreamSerializationAllowed = 1;
      cfg.attrs = at;
      cfg.numAttrs = 1;
      e = cudaLaunchKernelEx(&cfg, mv_status_kernel, (const unsigned *)c->status_dev, status_map);
    } else if (e == cudaSuccess) {
      e = cudaMemcpyAsync(c->status_host, c->status_dev, sizeof(unsigned), cudaMemcpyDeviceToHost, c->stream);
    }
    return e == cudaSuccess ? ZLLM_OK : zllm_cuda_fail(c, e, "zllm_matvec: y / status out");
  };
  // Below the GEMM's token count nothing in the call allocates or synchronizes, so it is recorded
  // once as a CUDA graph and replayed: one launch and one synchronization per call.
  // Pinned host buffers only (a pageable copy cannot be recorded), and only for a call seen twice in
  // a row, so one-off buffers do not pay for a recording.
  auto pinned = [](const void *p, void **dev) {
    cudaPointerAttributes at;
    const bool ok = cudaPointerGetAttributes(&at, p) == cudaSuccess && at.type == cudaMemoryTypeHost;
    cudaGetLastError();
    if (dev) *dev = ok ? at.devicePointer : nullptr;
    return ok;
  };
  // every address the recording holds: host buffers or a scratch slot regrown (zllm_topk shares
  // slots 0-4) record the call again
  const void *key[11] = {w->m.data, x_host, y_host, xs_, xq_, xd_, xsum_, y_, reinterpret_cast<const void *>((intptr_t)ntok),
                         nullptr, nullptr};
  zllm_weight *wm = const_cast<zllm_weight *>(w);
  // the buffers are checked on every call, replays included: a recording must never run on a
  // buffer that was unpinned since, even at the same address
  void *xmap = nullptr, *ymap = nullptr;
  const bool eligible = !(ntok >= kGemmMinTokens && kq_type(w->m.type)) && pinned(x_host, &xmap) && pinned(y_host, &ymap);
  key[9] = xmap;
  key[10] = ymap;
  const bool hit = eligible && wm->mv_exec && memcmp(key, wm->mv_key, sizeof key) == 0;
  const bool graph = hit || (eligible && memcmp(key, wm->mv_seen, sizeof key) == 0);
  memcpy(wm->mv_seen, key, sizeof key);
  if (graph && !hit) {
    // the recorded call reads x and writes y and the status word over PCIe through the mapped
    // buffers: no copy nodes, and the product's launch overlaps the fetch of x
    void *smap = nullptr;
    if (xmap && ymap && pinned(c->status_host, &smap) && smap) {
      y_dev = static_cast<float *>(ymap);
      x_dev = static_cast<const float *>(xmap);
      status_map = static_cast<unsigned *>(smap);
    }
    if (wm->mv_exec) cudaGraphExecDestroy(wm->mv_exec);
    wm->mv_exec = nullptr;
    cudaGraph_t g = nullptr;
    cudaError_t e = cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal);
    if (e != cudaSuccess) return zllm_cuda_fail(c, e, "zllm_matvec: begin capture");
    rc = enqueue();
    e = cudaStreamEndCapture(c->stream, &g);
    if (rc == ZLLM_OK && e != cudaSuccess) rc = zllm_cuda_fail(c, e, "zllm_matvec: end capture");
    if (rc == ZLLM_OK) {
      e = cudaGraphInstantiate(&wm->mv_exec, g, 0);
      if (e != cudaSuccess) {
        wm->mv_exec = nullptr;
        rc = zllm_cuda_fail(c, e, "zllm_matvec: graph instantiate");
      }
    }
    if (g) cudaGraphDestroy(g);
    if (rc) return rc;
    memcpy(wm->mv_key, key, sizeof key);
  }
  *c->status_host = 0;
  if (graph) {
    cudaError_t e = cudaGraphLaunch(wm->mv_exec, c->stream);
    if (e != cudaSuccess) return zllm_cuda_fail(c, e, "zllm_matvec: graph launch");
  } else if ((rc = enqueue())) {
    return rc;
  }
  cudaError_t e = cudaStreamSynchronize(c->stream);
  if (e != cudaSuccess) return zllm_cuda_fail(c, e, "zllm_matvec: synchronize");
  if (*c->status_host) return zllm_check_status(c);     // rare: clear the word and report, as zllm_sync does
  return ZLLM_OK;
}
