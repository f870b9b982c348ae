/*
 * zllm.h -- C ABI of libzllm_cuda.so, the B200 (sm_100a) backend for zerollm's decode/prefill
 * hot path: k-quant dequant-dot matmuls, the f16 KV-cache append, GQA decode attention and
 * prefix-cache restore.
 *
 * Everything is plain C: opaque handles, plain pointers and sizes.  Host buffers stay owned by
 * the caller (the library copies); device memory allocated by the library is owned by the
 * context.  Every function returns ZLLM_OK (0) or a negative ZLLM_E_* code; the message of the
 * last failure is zllm_last_error(ctx).  One context per host thread; calls are serialised on
 * the context's CUDA stream and the host-buffer entry points block until their results are in
 * host memory (the reference's pool awaits its workers the same way, src/compute/pool.js:201-219).
 *
 * Each entry point names the reference interface it replaces (file:line in the zerollm tree).
 */
#ifndef ZLLM_H
#define ZLLM_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------------------------ errors */
enum {
  ZLLM_OK = 0,
  ZLLM_E_ARG = -1,          /* bad argument (size, type, pointer) */
  ZLLM_E_OOM = -2,          /* device allocation failed */
  ZLLM_E_CUDA = -3,         /* a CUDA runtime call failed */
  ZLLM_E_CTX_FULL = -4,     /* "context full (N tokens)"   (src/compute/pool.js:151) */
  ZLLM_E_TIMEOUT = -5,      /* a bounded device wait expired; the kernel drained and returned */
  ZLLM_E_STATE = -6,        /* "model is closed" / a latched earlier failure (pool.js:123-127, :146-147) */
  ZLLM_E_UNSUPPORTED = -7,  /* tensor type or shape the kernels do not handle */
  ZLLM_E_TOKEN = -8,        /* "token id X out of range"   (pool.js:152) */
  ZLLM_E_BATCH = -9         /* "batch of B tokens (max M)" (pool.js:149) */
};

/* ggml tensor type ids (src/gguf/types.js:10-15) accepted by the kernels
 * (the set of src/model/config.js:12-15). */
enum {
  ZLLM_F32 = 0, ZLLM_F16 = 1, ZLLM_Q4_0 = 2, ZLLM_Q5_0 = 6, ZLLM_Q8_0 = 8,
  ZLLM_Q4_K = 12, ZLLM_Q5_K = 13, ZLLM_Q6_K = 14, ZLLM_BF16 = 30
};

typedef struct zllm_ctx zllm_ctx;
typedef struct zllm_weight zllm_weight;

/* ------------------------------------------------------------------------------------ context */
/* Library version string. */
const char *zllm_version(void);
/* Open a context on CUDA device `device` (one CUDA stream, a device status word, scratch).
 * Replaces the worker-pool start-up (PoolModel.create, src/compute/pool.js:33-121). */
int zllm_init(int device, zllm_ctx **out);
/* Release everything the context owns.  Safe on NULL.  (PoolModel.close, pool.js:302-316) */
void zllm_destroy(zllm_ctx *ctx);
/* Message of the last failure on this context ("" if none). */
const char *zllm_last_error(const zllm_ctx *ctx);
/* The cudaStream_t the context issues on, as void*. */
void *zllm_stream(zllm_ctx *ctx);
/* Wait for the context stream and report a device-side timeout as ZLLM_E_TIMEOUT. */
int zllm_sync(zllm_ctx *ctx);

/* ------------------------------------------------------------------------------------ weights */
/* Upload one matrix of `rows` x `cols` (cols = GGUF ne0, the row length) given as the raw GGUF
 * bytes of its rows (rows * rowBytes(type, cols) bytes; src/compute/ref-kernels.js:65-77).
 * The device copy is repacked for the kernels.  Replaces the worker's read of its row slice into
 * WebAssembly memory (src/compute/worker.js:129-148, src/model/loader.js:8-16). */
int zllm_weight_upload(zllm_ctx *ctx, int ggml_type, int64_t rows, int64_t cols, const void *host_bytes,
                       size_t nbytes, zllm_weight **out);
void zllm_weight_free(zllm_weight *w);
/* Shape and device footprint of an uploaded matrix. */
int zllm_weight_info(const zllm_weight *w, int *ggml_type, int64_t *rows, int64_t *cols, size_t *device_bytes);

/* ------------------------------------------------------------------------------------ kernels
 * Device-pointer entry points, enqueued on `stream` (a cudaStream_t; NULL = the context stream,
 * (void *)1 = cudaStreamLegacy, the legacy default stream).  They do not synchronise.  On a real
 * stream consecutive kernels are chained with programmatic dependent launch (the next kernel starts
 * streaming its weights while the previous one finishes); on the legacy stream they are not. */

/* xq[t][k] int8, xd[t][k/32] f32 scales, xs[t][k/32] int32 block sums of x[t][k] for t < ntok;
 * bit-exact with quantizeAct (src/compute/ref-kernels.js:44-62; worker `prep` worker.js:238-249). */
int zllm_quantize_act(zllm_ctx *ctx, const float *x, int64_t k, int ntok, int8_t *xq, float *xd, int32_t *xs,
                      void *stream);

/* y[t*y_stride + r] = (y_add ? y_add[t*y_stride + r] : 0) + dot(W[r], act_t) for r < rows, t < ntok.
 * Quantized W reads the quantized activation (xq, xd, xs); F16/BF16/F32 W reads x.
 * Replaces the per-type kernels matvec_* / mm_* (src/compute/wasm/kernels.js:30-240,
 * src/compute/wasm/kquant-kernels.js:337-504) and the dispatch in src/compute/worker.js:251-270.
 * y_add == y gives the in-place residual add of worker.js:346 / :432. */
int zllm_mm(zllm_ctx *ctx, const zllm_weight *w, const int8_t *xq, const float *xd, const int32_t *xs, const float *x,
            int ntok, float *y, int64_t y_stride, const float *y_add, void *stream);

/* Host-buffer convenience: y_host[t][rows] = W . x_host[t][cols] (quantizing x on the device first),
 * blocking.  The CUDA counterpart of `matvec(w, new Act(x), y)` (src/compute/ref-kernels.js:127). */
int zllm_matvec(zllm_ctx *ctx, const zllm_weight *w, const float *x_host, int ntok, float *y_host);

#ifdef __cplusplus
}
#endif
#endif /* ZLLM_H */
