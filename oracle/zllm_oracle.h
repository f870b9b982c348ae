/*
 * zllm_oracle.h -- TEST INFRASTRUCTURE ONLY.
 *
 * CPU restatement of the zerollm reference's plain-JS oracle (src/compute/ref-kernels.js,
 * src/compute/quant.js, src/util/f16.js, src/model/forward.js and the f16-KV path of
 * src/compute/worker.js).  Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline
 * leg may load this library, and only as the checker / the timed CPU baseline; the product
 * path (libzllm_cuda.so) never links or calls it.
 *
 * Arithmetic contract: every scalar operation the JS performs on Numbers is done here in
 * IEEE double in the same order, every store into a Float32Array / Int8Array / Int32Array /
 * Uint16Array is reproduced as the same conversion.  The library is compiled with
 * -ffp-contract=off so no multiply-add is fused.
 */
#ifndef ZLLM_ORACLE_H
#define ZLLM_ORACLE_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ggml type ids (src/gguf/types.js:10-15) */
enum {
  ZO_F32 = 0, ZO_F16 = 1, ZO_Q4_0 = 2, ZO_Q5_0 = 6, ZO_Q8_0 = 8,
  ZO_Q4_K = 12, ZO_Q5_K = 13, ZO_Q6_K = 14, ZO_BF16 = 30
};

uint16_t zo_f32_to_f16(float x);                 /* f16.js:7-30  */
float    zo_f16_to_f32(uint16_t h);              /* f16.js:33-40 */
float    zo_bf16_to_f32(uint16_t h);             /* f16.js:56    */
int64_t  zo_row_bytes(int type, int64_t cols);   /* ref-kernels.js:65-77; -1 = unsupported */

void zo_unpack_scale_min_k4(const uint8_t *q, int32_t *sc, int32_t *mn); /* quant.js:109-118 */

/* ref-kernels.js:44-62.  s may be NULL. */
void zo_quantize_act(const float *x, int64_t n, int8_t *q, float *d, int32_t *s);

/* ref-kernels.js:80-120 (+ quant.js dequantizers).  Returns 0, or -1 on an unsupported type. */
int zo_dequant_row(int type, const uint8_t *w, int64_t cols, int64_t row, float *out);

/* ref-kernels.js:127-302: y[r] for r in [r0, r1).  For quantized types x is quantized first
 * (Act.quant).  nthreads > 1 splits rows over OpenMP threads (per-row arithmetic unchanged). */
int zo_matvec(int type, const uint8_t *w, int64_t rows, int64_t cols, const float *x,
              float *y, int64_t r0, int64_t r1, int nthreads);

/* Same, with the activation already quantized (q, d, s as written by zo_quantize_act). */
int zo_matvec_q(int type, const uint8_t *w, int64_t cols, const float *x, const int8_t *xq,
                const float *xd, const int32_t *xs, float *y, int64_t r0, int64_t r1, int nthreads);

void   zo_rmsnorm(float *out, const float *x, const float *weight, double eps, int n); /* :305-310 */
void   zo_softmax(float *x, int n);                                                   /* :313-320 */
double zo_silu(double z);                                                             /* :322     */
/* :329-342, tables[pos*half + i]; freq_factors may be NULL */
void   zo_rope_tables(int n_rot, double base, int ctx, const float *freq_factors, float *cos_t, float *sin_t);
/* :349-363; neox != 0 rotates (i, i+half), else (2i, 2i+1) */
void   zo_apply_rope(float *v, int n_heads, int head_dim, int n_rot, int neox,
                     const float *cos_t, const float *sin_t, int pos, int h0);

/* One query head over one KV head's cache (positions 0..npos-1, each hd values, contiguous).
 * f32 cache: forward.js:126-139.  f16 cache: worker.js:320-333.  scores needs npos floats. */
void zo_attn_head_f32(const float *qh, const float *k, const float *v, int npos, int hd,
                      int kv_stride, float *scores, float *out);
void zo_attn_head_f16(const float *qh, const uint16_t *k, const uint16_t *v, int npos, int hd,
                      int kv_stride, float *scores, float *out);

/* ------------------------------------------------------------------ whole model (forward.js) */
typedef struct {
  int n_embd, n_layer, n_ff, n_head, n_head_kv, head_dim, n_rot, vocab;
  int neox;            /* 1 = qwen2/qwen3 split-half RoPE, 0 = llama adjacent pairs */
  int kv_f16;          /* 0 = RefModel f32 cache, 1 = pool f16 cache (worker.js:303-306) */
  int ctx;
  double rms_eps, rope_base;
} zo_config;

typedef struct { int type; int64_t rows, cols; const uint8_t *data; } zo_weight;

typedef struct {
  const float *attn_norm, *ffn_norm;
  const float *bq, *bk, *bv;        /* may be NULL */
  const float *q_norm, *k_norm;     /* may be NULL */
  zo_weight wq, wk, wv, wo, gate, up, down;
} zo_layer;

typedef struct zo_model zo_model;

/* layers: n_layer entries; output == NULL means tied to tok_embd.  Pointers are borrowed. */
zo_model *zo_model_new(const zo_config *cfg, const zo_weight *tok_embd, const zo_weight *output,
                       const float *output_norm, const zo_layer *layers, const float *rope_freqs);
void zo_model_free(zo_model *m);
int  zo_model_pos(const zo_model *m);
int  zo_model_restore_prefix(zo_model *m, int n);
void zo_model_truncate(zo_model *m, int n);
/* forward.js:94-158.  logits may be NULL (logits:false).  Returns 0, -1 context full, -2 bad token. */
int  zo_model_forward(zo_model *m, int token, float *logits, int nthreads);
/* kvGet / kvSet: f32 [n][kvDim] (forward.js:72-75; pool f16 path: worker.js:457-472) */
int  zo_model_kv_get(zo_model *m, int layer, int is_v, int n, float *out);
int  zo_model_kv_set(zo_model *m, int layer, int is_v, int n, const float *in);

#ifdef __cplusplus
}
#endif
#endif
