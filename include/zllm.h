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
/* Failure-detection check with no fault: runs the tensor-parallel all-reduce kernel on this GPU
 * against a phantom second rank that never publishes its slice.  The kernel's bounded wait gives up
 * after 2 s, the kernel returns, and the call reports ZLLM_E_TIMEOUT (status bit 0x10) like any pass
 * whose peer died; the context stays usable.  Allocates two small buffers for the call.  No
 * reference counterpart (the reference runs in one process). */
int zllm_peer_wait_selftest(zllm_ctx *ctx);

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
 * Quantized W reads the quantized activation (xq, xd, xs); F16/BF16/F32 W reads x.  A one-token
 * product on a k-quant W (Q4_K, Q5_K, Q6_K) may pass xq = NULL and the f32 x: the GEMV quantizes it
 * itself, bit-exactly as zllm_quantize_act.
 * Replaces the per-type kernels matvec_* / mm_* (src/compute/wasm/kernels.js:30-240,
 * src/compute/wasm/kquant-kernels.js:337-504) and the dispatch in src/compute/worker.js:251-270.
 * y_add == y gives the in-place residual add of worker.js:346 / :432.
 * 64 or more tokens on a k-quant W run the tensor-core GEMM (sub-block scale x quant dequantized
 * exactly into f16, the quantized activation as an f16 hi/lo pair, two MMAs per K slice, f32
 * accumulation with the super-block scales applied in f32: within ~1e-6 of the largest output of the
 * per-token arithmetic, not bit-identical to it; Q6_K matrices with a sub-block scale above 64 split
 * the weights into hi/lo too, three MMAs, ~1e-5); 1..63 tokens keep the per-token
 * arithmetic, so batches below 64 reproduce single tokens bit for bit
 * (test/kquant-kernels.test.js:65-97).  The GEMM's activation tiles live in a context scratch
 * buffer that grows on demand (a cudaMalloc on first use). */
int zllm_mm(zllm_ctx *ctx, const zllm_weight *w, const int8_t *xq, const float *xd, const int32_t *xs, const float *x,
            int ntok, float *y, int64_t y_stride, const float *y_add, void *stream);

/* D[j*m + i] = sum_k A[i*k + kk] * B[j*k + kk] for i < m, j < n: f16 A [m][k] and B [n][k] (row-major,
 * 16-byte aligned, k a multiple of 64), f32 D [n][m], on the same tcgen05 kernel as the k-quant GEMM
 * (the reference has no f16 GEMM entry; this one exposes the dense core of its batched mm_* path,
 * src/compute/worker.js:251-270, for tests and f16 callers).  Scratch for the tiled operands is a
 * context buffer that grows on demand. */
int zllm_gemm_f16(zllm_ctx *ctx, const void *A, const void *B, int64_t m, int64_t n, int64_t k, float *D, void *stream);

/* One-token k-quant (Q4_K / Q5_K / Q6_K) product with the fusions of the decode pass, on device
 * buffers: x f32 [cols] is RMSNormed with norm_w first when norm_w is given (src/compute/ref-kernels.js:
 * 305-310, eps as the model's) and quantized inside the kernel (quantizeAct, :44-62); then
 *   swiglu == 0: y[r] = (y_add ? y_add[r] : 0) + W[r] . x      (residual: src/compute/worker.js:346, :432)
 *   swiglu != 0: the rows are (gate, up) pairs 2i, 2i + 1 and y[i] = f32(silu(gate_i) * up_i)
 *                (worker.js:426, silu ref-kernels.js:322, in double), rows / 2 outputs.
 * Exposes the fused kernels the model's decode pass launches, for parity tests and hosts that run a
 * layer op by op. */
int zllm_mm_fused(zllm_ctx *ctx, const zllm_weight *w, const float *x, const float *norm_w, double eps, int swiglu,
                  float *y, const float *y_add, void *stream);

/* Layer glue on device buffers, each fused with the quantization its consumer needs (any of xb /
 * xq+xd+xs may be NULL; quantizing needs n % 32 == 0):
 *   zllm_rmsnorm_quant: xb[t] = rmsnorm(x[t], w, eps) for ntok vectors of n (src/compute/ref-kernels.js:
 *     305-310: double sum of squares, s = 1/sqrt(ss/n + eps), f32(x * s * w)), then quantizeAct of xb;
 *   zllm_swiglu_quant: hb[t][i] = f32(silu(gate[t*stride + i]) * up[t*stride + i]) in double
 *     (src/compute/worker.js:426, ref-kernels.js:322), then quantizeAct of hb. */
int zllm_rmsnorm_quant(zllm_ctx *ctx, const float *x, const float *w, int n, int ntok, double eps, float *xb,
                       int8_t *xq, float *xd, int32_t *xs, void *stream);
int zllm_swiglu_quant(zllm_ctx *ctx, const float *gate, const float *up, int n, int ntok, int64_t stride, float *hb,
                      int8_t *xq, float *xd, int32_t *xs, void *stream);

/* Host-buffer convenience: y_host[t][rows] = W . x_host[t][cols] (quantizing x on the device first),
 * blocking.  The CUDA counterpart of `matvec(w, new Act(x), y)` (src/compute/ref-kernels.js:127).
 * With pinned (page-locked, device-mapped) host buffers, a call repeated on the same weight and
 * buffers is recorded once as a CUDA graph and replayed: one launch and one synchronization per call,
 * x read and y written by the GPU through the mapped buffers.  Below the GEMM's 64 tokens only; the
 * recording is dropped with the weight, and the buffers are re-checked on every call. */
int zllm_matvec(zllm_ctx *ctx, const zllm_weight *w, const float *x_host, int ntok, float *y_host);

/* ------------------------------------------------------------------------------------ attention
 * Geometry of one attention layer's KV cache.  A sequence's cache holds, per layer, K then V, each
 * [n_head_kv][ctx][head_dim] (head-major, so one head's positions are contiguous); elements are f16
 * (kv_f16 = 1, the reference's --kv f16) or f32.  seq_stride / head_stride are in elements between
 * consecutive sequences / KV heads of the same K (or V) block. */
typedef struct {
  int n_head, n_head_kv, head_dim, n_rot;
  int neox;          /* 1: rotate pairs (i, i + n_rot/2) (qwen2/qwen3); 0: (2i, 2i+1) (llama) */
  int kv_f16;
  int ctx;           /* positions per sequence */
  double rms_eps;    /* as read from GGUF metadata (an f32 value) */
  int64_t seq_stride, head_stride;
} zllm_attn_geom;

/* RoPE tables cos/sin [ctx_len][n_rot/2] computed on the host in double (Math.cos / Math.sin of
 * p * base^(-2i/n_rot) / freq_factors[i]) and copied to device memory.  src/compute/ref-kernels.js:329-342.
 * freq_factors_host may be NULL. */
int zllm_rope_tables(zllm_ctx *ctx, int n_rot, double base, int ctx_len, const float *freq_factors_host,
                     float *cos_dev, float *sin_dev);

/* For ntok tokens: optional biases, per-head q-norm / k-norm, RoPE at pos[t], then the append of k and
 * v at position pos[t] of sequence seq[t] (f32 -> f16 round-to-nearest-even when kv_f16); q_out gets the
 * roped queries [ntok][n_head*head_dim].  Replaces src/compute/worker.js:290-309 and :313-315 (the
 * append and the q preparation of the attention phase) and src/model/forward.js:113-121. */
int zllm_qkv_append(zllm_ctx *ctx, const zllm_attn_geom *g, int ntok, const float *q, int64_t q_stride, const float *k,
                    const float *v, int64_t kv_stride, const float *bq, const float *bk, const float *bv,
                    const float *q_norm, const float *k_norm, const float *rope_cos, const float *rope_sin,
                    const int32_t *pos, const int32_t *seq, float *q_out, void *kcache, void *vcache, void *stream);

/* out[s][h][:] = softmax(q[s][h] . K[s][h/group][0..npos[s]) / sqrt(head_dim)) . V[...] for nseq
 * sequences (npos device array, every value <= max_pos <= ctx).  Context-split ("flash decoding")
 * with the merge done by the last CTA; scratch comes from the context.  Replaces the attention loop
 * of src/compute/worker.js:310-337 (WASM attn_scores / attn_av, src/compute/wasm/attn-kernels.js:26-194)
 * and src/model/forward.js:123-140. */
int zllm_attn_decode(zllm_ctx *ctx, const zllm_attn_geom *g, const float *q, const void *kcache, const void *vcache,
                     const int32_t *npos, int nseq, int max_pos, float *out, void *stream);

/* zllm_attn_decode with the same arguments and results, but the call allocates no device memory:
 * its scratch (split-context partials and merge counters) is a fixed array compiled into the
 * library, 4 MiB of partials + 4096 counters, held by every GPU on which a context was created
 * until the process exits.  For callers that may not allocate during a step (all free HBM already handed to
 * a KV pool; device memory owned by another allocator, where a cudaFree would synchronize the
 * device).  A call needing more than 4 MiB of partials (nseq * n_head_kv * splits * group *
 * (head_dim + 2) floats) or more than 4096 (sequence, KV head) pairs returns ZLLM_E_ARG without
 * launching.  All calls on one device share the array: calls that overlap in time race, so order
 * them (one stream, or events).  zllm_init loads the array on its device and looks up its address
 * (cudaGetSymbolAddress), so the memory is taken when the first context on a device is created and
 * no call of this function allocates, the first one included.  No counterpart in the reference. */
int zllm_attn_decode_noalloc(zllm_ctx *ctx, const zllm_attn_geom *g, const float *q, const void *kcache,
                             const void *vcache, const int32_t *npos, int nseq, int max_pos, float *out, void *stream);

/* ------------------------------------------------------------------------ paged KV caches
 * A layer's K cache and V cache as pools of fixed-size pages instead of one contiguous run per
 * sequence: each pool holds num_pages pages of [n_head_kv][page_size][head_dim] elements (f16 or f32
 * as g->kv_f16), and row s of block_table lists sequence s's pages in position order, so position p
 * of sequence s is row p % page_size of page block_table[s * max_pages + p / page_size].  Memory then
 * follows the positions in use (a server pages 64 sequences of up to 32k positions without reserving
 * 64 x 32k per layer up front) and sequences that share a prefix can point at the same pages.  The
 * reference keeps one contiguous cache per worker (src/compute/worker.js:121-125); it has no paging.
 * page_size is a power of two from 16 to 4096; block_table is device memory.  A position past a row's
 * max_pages pages, or a table entry outside [0, num_pages), reads page 0 and makes the next
 * synchronizing call (zllm_sync) return ZLLM_E_ARG. */
typedef struct {
  const int32_t *block_table;  /* device [rows][max_pages] page indices */
  int max_pages;               /* entries per row */
  int num_pages;               /* pages in each pool */
  int page_size;               /* positions per page */
} zllm_kv_pages;

/* zllm_qkv_append into paged pools: token t goes to position pos[t] of sequence seq[t] (table row
 * seq[t]); the arithmetic and the stored bits are zllm_qkv_append's. */
int zllm_qkv_append_paged(zllm_ctx *ctx, const zllm_attn_geom *g, const zllm_kv_pages *pages, int ntok, const float *q,
                          int64_t q_stride, const float *k, const float *v, int64_t kv_stride, const float *bq,
                          const float *bk, const float *bv, const float *q_norm, const float *k_norm,
                          const float *rope_cos, const float *rope_sin, const int32_t *pos, const int32_t *seq,
                          float *q_out, void *kpool, void *vpool, void *stream);
/* zllm_attn_decode over paged pools: query s attends to positions [0, npos[s]) of table row s
 * (max_pos <= max_pages * page_size).  The same context split and arithmetic as zllm_attn_decode, so
 * the outputs are the same bits as over a contiguous cache holding the same rows. */
int zllm_attn_decode_paged(zllm_ctx *ctx, const zllm_attn_geom *g, const zllm_kv_pages *pages, const float *q,
                           const void *kpool, const void *vpool, const int32_t *npos, int nseq, int max_pos, float *out,
                           void *stream);

/* kvSet: n positions of one layer's K or V block of one sequence from f32 [n][n_head_kv*head_dim]
 * (device) -- cast to f16 when kv_f16.  kvGet: the reverse (f16 -> f32 exact).
 * src/compute/worker.js:457-472, src/compute/pool.js:225-238. */
int zllm_kv_import(zllm_ctx *ctx, const zllm_attn_geom *g, void *cache_block, int n, const float *stage, void *stream);
int zllm_kv_export(zllm_ctx *ctx, const zllm_attn_geom *g, const void *cache_block, int n, float *stage, void *stream);

/* Byte copy of positions [0, n) of every KV head between two K (or V) blocks with the given head
 * strides (elements): a prefix-cache slot restore or save (src/model/prefix-cache.js:50-96 restores
 * through kvSet; a device-resident slot makes it a copy).  Bit-exact by construction. */
int zllm_kv_copy(zllm_ctx *ctx, const zllm_attn_geom *g, void *dst_block, int64_t dst_head_stride,
                 const void *src_block, int64_t src_head_stride, int n, void *stream);

/* ------------------------------------------------------------------------------------ model
 * A whole llama / qwen2 / qwen3 model on one GPU: the CUDA counterpart of the worker pool's model
 * interface (PoolModel, src/compute/pool.js:24-317; RefModel, src/model/forward.js:10-168).  It holds
 * n_seq independent sequences (1 = the reference's single-sequence model), each with its own KV
 * cache of ctx positions. */
typedef struct zllm_model zllm_model;

typedef struct {
  int n_embd, n_layer, n_ff, n_head, n_head_kv, head_dim, n_rot, vocab;   /* src/model/config.js:73-123 */
  int neox;          /* RoPE pairing: 1 split-half (qwen2/qwen3), 0 adjacent (llama) */
  int kv_f16;        /* --kv f16 (1) or f32 (0) */
  int ctx;           /* positions per sequence */
  int n_seq;         /* independent sequences */
  int max_batch;     /* most tokens one call carries (the pool's maxBatch, <= 64; pool.js:63) */
  int logits_batch;  /* most positions one call returns logits for with want = 2 (pool.js:65) */
  double rms_eps, rope_base;
} zllm_model_config;

/* tensor kinds for zllm_model_set_matrix / zllm_model_set_vector (GGUF tensor names) */
enum {
  ZLLM_T_TOK_EMBD = 0,    /* token_embd.weight   [vocab][n_embd] */
  ZLLM_T_OUTPUT = 1,      /* output.weight       [vocab][n_embd] (absent: tied to token_embd) */
  ZLLM_T_OUTPUT_NORM = 2, /* output_norm.weight  [n_embd] */
  ZLLM_T_ROPE_FREQS = 3,  /* rope_freqs.weight   [n_rot/2] */
  ZLLM_T_ATTN_NORM = 10,  /* blk.L.attn_norm.weight */
  ZLLM_T_WQ = 11, ZLLM_T_WK = 12, ZLLM_T_WV = 13, ZLLM_T_WO = 14,  /* blk.L.attn_{q,k,v,output}.weight */
  ZLLM_T_BQ = 15, ZLLM_T_BK = 16, ZLLM_T_BV = 17,                  /* blk.L.attn_{q,k,v}.bias (qwen2) */
  ZLLM_T_Q_NORM = 18, ZLLM_T_K_NORM = 19,                          /* blk.L.attn_{q,k}_norm.weight (qwen3) */
  ZLLM_T_FFN_NORM = 20,
  ZLLM_T_GATE = 21, ZLLM_T_UP = 22, ZLLM_T_DOWN = 23               /* blk.L.ffn_{gate,up,down}.weight */
};

int zllm_model_create(zllm_ctx *ctx, const zllm_model_config *cfg, zllm_model **out);
/* Raw GGUF bytes of one matrix (the worker's weight plan, src/compute/worker.js:49-97). */
int zllm_model_set_matrix(zllm_model *m, int kind, int layer, int ggml_type, int64_t rows, int64_t cols,
                          const void *host_bytes, size_t nbytes);
/* An f32 vector (norm weights, biases, RoPE frequency factors). */
int zllm_model_set_vector(zllm_model *m, int kind, int layer, const float *host, int64_t n);
/* ------------------------------------------------------------------------ tensor parallelism
 * A model too large for one GPU runs with its weights sharded over `size` GPUs, one process (one
 * context, one model) per GPU: each rank's model is created with its local configuration (its
 * query / KV heads and its slice of the FFN; the host cuts the shards) and joins the group before
 * its first pass.  attn_output and ffn_down are row-parallel: after each, the ranks' partial sums
 * are added with an NCCL all-reduce over NVLink (the reference has one process and no such step;
 * BASELINE config 4).  NCCL is opened at run time (libnccl.so.2).
 * zllm_tp_unique_id: rank 0 creates the group's id (out: NCCL_UNIQUE_ID_BYTES = 128 bytes), which the
 * host hands to every rank; zllm_model_set_tp blocks until all `size` ranks have joined. */
int zllm_tp_unique_id(zllm_ctx *ctx, void *out, size_t bytes);
/* The model's own stream (a cudaStream_t): every pass runs on it; a caller may record CUDA events
 * on it to time passes on the device (no reference counterpart). */
void *zllm_model_stream(zllm_model *m);
/* Which collective sums the row-parallel partials once the model is ready: 0 none (one GPU), 1 NCCL
 * all-reduce, 2 the library's one-shot all-reduce over NVLink peer memory (every rank its own
 * process, the peers' buffers mapped by CUDA IPC).  No reference counterpart. */
int zllm_model_tp_collective(zllm_model *m);
int zllm_model_set_tp(zllm_model *m, int rank, int size, const void *unique_id);
/* Tensor parallel: this rank holds only rows [v0, v0 + n) of the output head, the even split
 * v0 = rank * vocab / size (call after zllm_model_set_tp, before setting the output matrix, which
 * then has n rows).  Each pass computes the rank's logits slice and gathers every rank's slice
 * (NCCL all-gather), so every rank ends with the full logits and the same argmax, while reading
 * 1/size of the head.  Needs a separate output matrix (not the tied token embedding).  The reference
 * has one process and no such split (its output head is read by every worker thread). */
int zllm_model_set_vocab_shard(zllm_model *m, int64_t v0, int64_t n);

/* Allocate the KV caches and activations once every tensor is set (called by the first pass). */
int zllm_model_ready(zllm_model *m);
/* n tokens of sequence `seq` at its next positions in one pass (forwardBatch, pool.js:145-160;
 * forward = n 1).  want: 0 no logits, 1 the last token's, 2 every token's ([n][vocab], n <=
 * logits_batch).  logits_host / argmax_host may be NULL.  Errors as the pool: ZLLM_E_CTX_FULL
 * "context full (N tokens)", ZLLM_E_TOKEN "token id X out of range", ZLLM_E_BATCH "batch of B tokens
 * (max M)"; a device failure latches and every later call returns ZLLM_E_STATE (pool.js:123-127). */
int zllm_model_forward(zllm_model *m, int seq, const int32_t *tokens, int n, int want, float *logits_host,
                       int32_t *argmax_host);
/* One token for each of n distinct sequences (batched decode); logits [n][vocab]. */
int zllm_model_decode(zllm_model *m, const int32_t *seqs, const int32_t *tokens, int n, float *logits_host,
                      int32_t *argmax_host);
/* Greedy generation on the device: `steps` passes, the first on `tokens`, each later one on the
 * argmax of the previous pass's logits (src/model/generate.js:4-10 with greedy sampling), with no
 * host round trip between passes.  seqs == NULL: one token (n == 1) continuing sequence `seq`;
 * else one token for each of n distinct sequences.  out_host[steps][n] receives each pass's argmax
 * (the next input).  The reference's generate() loop (src/model/generate.js:55-96) does the same
 * with a host round trip per token. */
int zllm_model_generate(zllm_model *m, int seq, const int32_t *seqs, const int32_t *tokens, int n, int steps,
                        int32_t *out_host);
/* Positions held by a sequence (PoolModel.pos). */
int zllm_model_pos(const zllm_model *m, int seq);
/* Roll back to n positions (truncate, pool.js:278-294: positional bookkeeping) / forget all. */
int zllm_model_truncate(zllm_model *m, int seq, int n);
int zllm_model_reset(zllm_model *m, int seq);
/* kvGet / kvSet on host buffers f32 [n][n_head_kv*head_dim] (pool.js:225-238). */
int zllm_model_kv_get(zllm_model *m, int seq, int layer, int is_v, int n, float *out);
int zllm_model_kv_set(zllm_model *m, int seq, int layer, int is_v, int n, const float *in);
/* After the KV regions were filled (kvSet): the sequence now holds n positions (restorePrefix, pool.js:244-247). */
int zllm_model_restore_prefix(zllm_model *m, int seq, int n);
/* Sampling candidates on the device (src/sampling/sampler.js:20-42 topKSelect, after the penalties of
 * :98-112): the k (<= 256) largest logits of each of the first `rows` rows of the last pass's logits,
 * sorted by value descending then index ascending, into ids_host / vals_host [rows][k]; entries past
 * the finite values of a row have id -1.  pen_tok / pen_cnt: the n_pen (<= 4096) distinct recent
 * tokens and their counts; each gets l/repeat_penalty (l > 0) or l*repeat_penalty, minus
 * count*frequency + presence, in double, stored as f32.  The softmax, min-p, top-p and the draw
 * (sampler.js:116-148) run on the k pairs in the caller.  A pass with want 0 and no logits_host
 * keeps the logits on the device for this call. */
int zllm_model_topk(zllm_model *m, int rows, int k, const int32_t *pen_tok, const int32_t *pen_cnt, int n_pen,
                    double repeat_penalty, double frequency, double presence, int32_t *ids_host, float *vals_host);
/* The same selection on host buffers (kernel-level, for tests): rows x n logits (n <= 327680). */
int zllm_topk(zllm_ctx *c, const float *logits_host, int rows, int64_t n, int k, const int32_t *pen_tok,
              const int32_t *pen_cnt, int n_pen, double repeat_penalty, double frequency, double presence,
              int32_t *ids_host, float *vals_host);
/* Device-resident prefix slot: save the first n positions of a sequence's KV, restore them (a byte
 * copy) into a sequence, which then holds those n positions. */
int zllm_model_slot_save(zllm_model *m, int seq, int n);
int zllm_model_slot_restore(zllm_model *m, int seq);
/* Record passes into CUDA graphs (default on). */
int zllm_model_set_graphs(zllm_model *m, int on);
/* Device pointer of the logits of the last pass ([rows][vocab] f32). */
void *zllm_model_logits(zllm_model *m);
void zllm_model_destroy(zllm_model *m);

#ifdef __cplusplus
}
#endif
#endif /* ZLLM_H */
