// extern "C" entry points for the KV cache and decode attention (declared in include/zllm.h).
#include <cmath>
#include <vector>

#include "../../include/zllm.h"
#include "capi_internal.h"
#include "internal.h"

using namespace zllm;

static cudaStream_t pick_stream(zllm_ctx *c, void *stream) { return stream ? (cudaStream_t)stream : c->stream; }
static bool pdl_stream(cudaStream_t s) { return s != nullptr && s != cudaStreamLegacy && s != cudaStreamPerThread; }

static int check_geom(zllm_ctx *c, const zllm_attn_geom *g) {
  if (!g || g->n_head <= 0 || g->n_head_kv <= 0 || g->n_head % g->n_head_kv || g->head_dim <= 0 || g->ctx <= 0 ||
      g->n_rot <= 0 || g->n_rot > g->head_dim || g->n_rot % 2) {
    zllm_set_error(c, "bad attention geometry");
    return ZLLM_E_ARG;
  }
  return ZLLM_OK;
}

extern "C" int zllm_rope_tables(zllm_ctx *c, int n_rot, double base, int ctx_len, const float *ff, float *cos_dev,
                                float *sin_dev) {
  if (!c || n_rot <= 0 || n_rot % 2 || ctx_len <= 0 || !cos_dev || !sin_dev) {
    zllm_set_error(c, "zllm_rope_tables: bad argument");
    return ZLLM_E_ARG;
  }
  const int half = n_rot / 2;
  std::vector<float> cs((size_t)ctx_len * half), sn((size_t)ctx_len * half);
  for (int i = 0; i < half; i++) {
    double freq = std::pow(base, (-2.0 * i) / n_rot);         // ref-kernels.js:334
    if (ff) freq /= (double)ff[i];
    for (int p = 0; p < ctx_len; p++) {
      cs[(size_t)p * half + i] = (float)std::cos(p * freq);
      sn[(size_t)p * half + i] = (float)std::sin(p * freq);
    }
  }
  cudaError_t e = cudaMemcpyAsync(cos_dev, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice, c->stream);
  if (e == cudaSuccess) e = cudaMemcpyAsync(sin_dev, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice, c->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
  return e == cudaSuccess ? ZLLM_OK : zllm_cuda_fail(c, e, "zllm_rope_tables");
}

extern "C" int zllm_qkv_append(zllm_ctx *c, const zllm_attn_geom *g, int ntok, const float *q, int64_t q_stride,
                               const float *k, const float *v, int64_t kv_stride, const float *bq, const float *bk,
                               const float *bv, const float *q_norm, const float *k_norm, const float *rope_cos,
                               const float *rope_sin, const int32_t *pos, const int32_t *seq, float *q_out, void *kcache,
                               void *vcache, void *stream) {
  if (!c) return ZLLM_E_ARG;
  int rc = check_geom(c, g);
  if (rc) return rc;
  if (ntok < 1 || !q || !k || !v || !rope_cos || !rope_sin || !pos || !seq || !q_out || !kcache || !vcache) {
    zllm_set_error(c, "zllm_qkv_append: bad argument");
    return ZLLM_E_ARG;
  }
  QkvPostArgs a{};
  a.q = q; a.k = k; a.v = v; a.q_stride = q_stride; a.kv_stride = kv_stride;
  a.bq = bq; a.bk = bk; a.bv = bv; a.q_norm = q_norm; a.k_norm = k_norm;
  a.rope_cos = rope_cos; a.rope_sin = rope_sin; a.pos = pos; a.seq = seq;
  a.q_out = q_out; a.q_out_stride = (int64_t)g->n_head * g->head_dim;
  a.kcache = kcache; a.vcache = vcache; a.seq_stride = g->seq_stride; a.head_stride = g->head_stride;
  a.n_head = g->n_head; a.n_kv = g->n_head_kv; a.head_dim = g->head_dim; a.n_rot = g->n_rot; a.neox = g->neox;
  a.kv_f16 = g->kv_f16; a.ntok = ntok; a.eps = g->rms_eps;
  cudaStream_t s = pick_stream(c, stream);
  cudaError_t e = launch_qkv_post(a, s, pdl_stream(s));
  return e == cudaSuccess ? ZLLM_OK : zllm_cuda_fail(c, e, "qkv_append launch");
}

// context splits of a decode attention launch: those of the longest sequence (attn_nsplit is
// non-decreasing in the length)
int zllm_attn_splits(const zllm_ctx *c, const zllm_attn_geom *g, int nseq, int max_pos) {
  (void)c; (void)nseq;
  return attn_nsplit(max_pos, attn_warps(g->n_head_kv));
}

// the paging descriptor as the kernels take it; ZLLM_OK or ZLLM_E_ARG with the message set
static int kv_pages(zllm_ctx *c, const zllm_kv_pages *p, KvPages *out) {
  int log2 = 0;
  while (log2 < 13 && (1 << log2) < (p ? p->page_size : 0)) log2++;
  if (!p || !p->block_table || p->max_pages < 1 || p->num_pages < 1 || p->page_size < 16 || p->page_size > 4096 ||
      (1 << log2) != p->page_size) {
    zllm_set_error(c, "paged KV: a device block table, max_pages >= 1, num_pages >= 1 and a power-of-two page_size in [16, 4096]");
    return ZLLM_E_ARG;
  }
  out->table = p->block_table;
  out->max_pages = p->max_pages;
  out->num_pages = p->num_pages;
  out->page_log2 = log2;
  return ZLLM_OK;
}

int zllm_attn_launch(zllm_ctx *c, const zllm_attn_geom *g, const float *q, const void *kcache, const void *vcache,
                     const int32_t *npos, int nseq, int nsplit, float *out, float *partial, int32_t *counters,
                     cudaStream_t s, const int32_t *seq, const KvPages *pages) {
  // each lane reads head_dim / 32 elements of a row as one vector load: the caches and the
  // strides must keep that vector aligned
  const int64_t elt = g->kv_f16 ? 2 : 4, vec = (g->head_dim / 32) * elt;
  if ((uintptr_t)kcache % vec || (uintptr_t)vcache % vec || (g->seq_stride * elt) % vec || (g->head_stride * elt) % vec) {
    zllm_set_error(c, "zllm_attn_decode: caches and strides must be %lld-byte aligned", (long long)vec);
    return ZLLM_E_ARG;
  }
  AttnArgs a{};
  a.seq = seq;
  a.q = q; a.kcache = kcache; a.vcache = vcache; a.seq_stride = g->seq_stride; a.head_stride = g->head_stride;
  a.npos = npos; a.out = out; a.partial = partial; a.counters = counters; a.status = c->status_dev;
  a.scale = (float)(1.0 / std::sqrt((double)g->head_dim));
  a.n_head = g->n_head; a.n_kv = g->n_head_kv; a.head_dim = g->head_dim; a.nseq = nseq; a.nsplit = nsplit;
  if (pages) a.pages = *pages;
  cudaError_t e = launch_attn(a, g->kv_f16 != 0, s, pdl_stream(s));
  return e == cudaSuccess ? ZLLM_OK : zllm_cuda_fail(c, e, "attn_decode launch");
}

extern "C" int zllm_attn_decode(zllm_ctx *c, const zllm_attn_geom *g, const float *q, const void *kcache,
                                const void *vcache, const int32_t *npos, int nseq, int max_pos, float *out,
                                void *stream) {
  if (!c) return ZLLM_E_ARG;
  int rc = check_geom(c, g);
  if (rc) return rc;
  if (!q || !kcache || !vcache || !npos || !out || nseq < 1 || max_pos < 0 || max_pos > g->ctx) {
    zllm_set_error(c, "zllm_attn_decode: bad argument");
    return ZLLM_E_ARG;
  }
  if (!attn_supported(g->head_dim, g->n_head / g->n_head_kv)) {
    zllm_set_error(c, "zllm_attn_decode: head_dim %d / group %d not supported (head_dim 64 or 128, group 1, 2, 4 or 8)",
                   g->head_dim, g->n_head / g->n_head_kv);
    return ZLLM_E_UNSUPPORTED;
  }
  const int nsplit = zllm_attn_splits(c, g, nseq, max_pos);
  const int group = g->n_head / g->n_head_kv;
  const size_t part_bytes = (size_t)nseq * g->n_head_kv * nsplit * group * (g->head_dim + 2) * sizeof(float);
  const size_t cnt_bytes = (size_t)nseq * g->n_head_kv * sizeof(int32_t);
  void *part, *cnt;
  if ((rc = zllm_scratch(c, 8, part_bytes, &part))) return rc;
  if (c->scratch_bytes[9] < cnt_bytes) {
    // counters start at zero and every launch leaves them at zero
    if ((rc = zllm_scratch(c, 9, cnt_bytes, &cnt))) return rc;
    cudaError_t e = cudaMemsetAsync(c->scratch[9], 0, c->scratch_bytes[9], c->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
    if (e != cudaSuccess) return zllm_cuda_fail(c, e, "counter init");
  }
  cnt = c->scratch[9];
  return zllm_attn_launch(c, g, q, kcache, vcache, npos, nseq, nsplit, out, (float *)part, (int32_t *)cnt,
                          pick_stream(c, stream), nullptr, nullptr);
}

extern "C" int zllm_qkv_append_paged(zllm_ctx *c, const zllm_attn_geom *g, const zllm_kv_pages *pages, int ntok,
                                     const float *q, int64_t q_stride, const float *k, const float *v, int64_t kv_stride,
                                     const float *bq, const float *bk, const float *bv, const float *q_norm,
                                     const float *k_norm, const float *rope_cos, const float *rope_sin, const int32_t *pos,
                                     const int32_t *seq, float *q_out, void *kpool, void *vpool, void *stream) {
  if (!c) return ZLLM_E_ARG;
  int rc = check_geom(c, g);
  if (rc) return rc;
  KvPages pg{};
  if ((rc = kv_pages(c, pages, &pg))) return rc;
  if (ntok < 1 || !q || !k || !v || !rope_cos || !rope_sin || !pos || !seq || !q_out || !kpool || !vpool) {
    zllm_set_error(c, "zllm_qkv_append_paged: bad argument");
    return ZLLM_E_ARG;
  }
  QkvPostArgs a{};
  a.q = q; a.k = k; a.v = v; a.q_stride = q_stride; a.kv_stride = kv_stride;
  a.bq = bq; a.bk = bk; a.bv = bv; a.q_norm = q_norm; a.k_norm = k_norm;
  a.rope_cos = rope_cos; a.rope_sin = rope_sin; a.pos = pos; a.seq = seq;
  a.q_out = q_out; a.q_out_stride = (int64_t)g->n_head * g->head_dim;
  a.kcache = kpool; a.vcache = vpool;
  a.n_head = g->n_head; a.n_kv = g->n_head_kv; a.head_dim = g->head_dim; a.n_rot = g->n_rot; a.neox = g->neox;
  a.kv_f16 = g->kv_f16; a.ntok = ntok; a.eps = g->rms_eps;
  a.pages = pg;
  a.status = c->status_dev;
  cudaStream_t s = pick_stream(c, stream);
  cudaError_t e = launch_qkv_post(a, s, pdl_stream(s));
  return e == cudaSuccess ? ZLLM_OK : zllm_cuda_fail(c, e, "qkv_append_paged launch");
}

extern "C" int zllm_attn_decode_paged(zllm_ctx *c, const zllm_attn_geom *g, const zllm_kv_pages *pages, const float *q,
                                      const void *kpool, const void *vpool, const int32_t *npos, int nseq, int max_pos,
                                      float *out, void *stream) {
  if (!c) return ZLLM_E_ARG;
  int rc = check_geom(c, g);
  if (rc) return rc;
  KvPages pg{};
  if ((rc = kv_pages(c, pages, &pg))) return rc;
  if (!q || !kpool || !vpool || !npos || !out || nseq < 1 || max_pos < 0 ||
      (int64_t)max_pos > (int64_t)pages->max_pages * pages->page_size) {
    zllm_set_error(c, "zllm_attn_decode_paged: bad argument (max_pos <= max_pages * page_size)");
    return ZLLM_E_ARG;
  }
  if (!attn_supported(g->head_dim, g->n_head / g->n_head_kv)) {
    zllm_set_error(c, "zllm_attn_decode_paged: head_dim %d / group %d not supported (head_dim 64 or 128, group 1, 2, 4 or 8)",
                   g->head_dim, g->n_head / g->n_head_kv);
    return ZLLM_E_UNSUPPORTED;
  }
  const int nsplit = zllm_attn_splits(c, g, nseq, max_pos);
  const int group = g->n_head / g->n_head_kv;
  const size_t part_bytes = (size_t)nseq * g->n_head_kv * nsplit * group * (g->head_dim + 2) * sizeof(float);
  const size_t cnt_bytes = (size_t)nseq * g->n_head_kv * sizeof(int32_t);
  void *part, *cnt;
  if ((rc = zllm_scratch(c, 8, part_bytes, &part))) return rc;
  if (c->scratch_bytes[9] < cnt_bytes) {
    if ((rc = zllm_scratch(c, 9, cnt_bytes, &cnt))) return rc;
    cudaError_t e = cudaMemsetAsync(c->scratch[9], 0, c->scratch_bytes[9], c->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
    if (e != cudaSuccess) return zllm_cuda_fail(c, e, "counter init");
  }
  cnt = c->scratch[9];
  return zllm_attn_launch(c, g, q, kpool, vpool, npos, nseq, nsplit, out, (float *)part, (int32_t *)cnt,
                          pick_stream(c, stream), nullptr, &pg);
}

extern "C" int zllm_kv_import(zllm_ctx *c, const zllm_attn_geom *g, void *block, int n, const float *stage, void *stream) {
  if (!c) return ZLLM_E_ARG;
  int rc = check_geom(c, g);
  if (rc) return rc;
  if (!block || !stage || n < 0 || n > g->ctx) { zllm_set_error(c, "zllm_kv_import: bad argument"); return ZLLM_E_ARG; }
  cudaError_t e = launch_kv_convert(const_cast<float *>(stage), block, n, g->n_head_kv, g->head_dim, g->head_stride,
                                    g->kv_f16 != 0, 0, pick_stream(c, stream));
  return e == cudaSuccess ? ZLLM_OK : zllm_cuda_fail(c, e, "kv_import");
}

extern "C" int zllm_kv_export(zllm_ctx *c, const zllm_attn_geom *g, const void *block, int n, float *stage, void *stream) {
  if (!c) return ZLLM_E_ARG;
  int rc = check_geom(c, g);
  if (rc) return rc;
  if (!block || !stage || n < 0 || n > g->ctx) { zllm_set_error(c, "zllm_kv_export: bad argument"); return ZLLM_E_ARG; }
  cudaError_t e = launch_kv_convert(stage, const_cast<void *>(block), n, g->n_head_kv, g->head_dim, g->head_stride,
                                    g->kv_f16 != 0, 1, pick_stream(c, stream));
  return e == cudaSuccess ? ZLLM_OK : zllm_cuda_fail(c, e, "kv_export");
}

extern "C" int zllm_kv_copy(zllm_ctx *c, const zllm_attn_geom *g, void *dst, int64_t dst_hs, const void *src,
                            int64_t src_hs, int n, void *stream) {
  if (!c) return ZLLM_E_ARG;
  int rc = check_geom(c, g);
  if (rc) return rc;
  if (!dst || !src || n < 0 || dst_hs < (int64_t)n * g->head_dim || src_hs < (int64_t)n * g->head_dim) {
    zllm_set_error(c, "zllm_kv_copy: bad argument");
    return ZLLM_E_ARG;
  }
  if (n == 0) return ZLLM_OK;
  const size_t el = g->kv_f16 ? 2 : 4;
  if (((uintptr_t)dst | (uintptr_t)src | (uintptr_t)(dst_hs * el) | (uintptr_t)(src_hs * el) |
       (uintptr_t)((size_t)n * g->head_dim * el)) % 16) {
    zllm_set_error(c, "zllm_kv_copy: blocks, head strides and the copied rows must be multiples of 16 bytes");
    return ZLLM_E_ARG;
  }
  cudaError_t e = launch_kv_block_copy(dst, dst_hs * el, 0, src, src_hs * el, 0, (int64_t)n * g->head_dim * el,
                                       g->n_head_kv, 1, c->num_sms, pick_stream(c, stream));
  return e == cudaSuccess ? ZLLM_OK : zllm_cuda_fail(c, e, "zllm_kv_copy");
}
