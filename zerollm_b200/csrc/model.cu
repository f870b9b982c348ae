// Model runtime: the whole forward pass of a llama / qwen2 / qwen3 model on one GPU, built from the
// kernels of gemv.cu, quant.cu, kv.cu and ops.cu, behind the extern "C" model entry points of
// include/zllm.h.
//
// One pass runs n tokens, each token t belonging to sequence seq[t] at position pos[t]: either B
// consecutive tokens of one sequence (the reference's forwardBatch, src/compute/pool.js:145-160 /
// the worker's runBatch, src/compute/worker.js:410-445) or one token of each of n independent
// sequences (batched serving).  The phase order is the reference worker's: embedding; per layer
// RMSNorm -> q,k,v -> norms/RoPE/KV append -> attention -> wo + residual -> RMSNorm -> gate, up ->
// SwiGLU -> down + residual; output RMSNorm -> output head (src/compute/worker.js:278-348, :410-445;
// src/model/forward.js:94-158).  Every matmul input is quantized per 32 values exactly like the
// reference's quantizeAct, fused into the kernel that produces it.
//
// Steady-state decode passes of the same shape are recorded once into a CUDA graph and replayed
// (kernels chained with programmatic dependent launch inside the graph).
#include <algorithm>
#include <initializer_list>
#include <cmath>
#include <cstring>
#include <new>
#include <string>
#include <vector>

#include "../../include/zllm.h"
#include "capi_internal.h"
#include "internal.h"

using namespace zllm;

namespace {

struct Layer {
  zllm_weight *w[7] = {};                 // wq wk wv wo gate up down
  zllm_weight *qkv = nullptr, *gu = nullptr;   // [wq; wk; wv] and [gate; up] row-concatenated (when types agree)
  float *attn_norm = nullptr, *ffn_norm = nullptr, *q_norm = nullptr, *k_norm = nullptr;
  float *bq = nullptr, *bk = nullptr, *bv = nullptr;
};

enum { WQ = 0, WK, WV, WO, GATE, UP, DOWN };

template <typename T>
cudaError_t dalloc(T **p, size_t n) { return cudaMalloc((void **)p, (n ? n : 1) * sizeof(T)); }

}  // namespace

struct zllm_model {
  zllm_ctx *ctx = nullptr;
  zllm_model_config c{};
  cudaStream_t stream = nullptr;
  std::vector<Layer> L;
  zllm_weight *tok = nullptr, *out = nullptr;           // out == nullptr: tied to tok
  float *out_norm = nullptr, *rope_freqs_host_dev = nullptr;
  std::vector<float> rope_freqs_host;
  bool ready = false, failed = false, closed = false;
  // device state
  float *rope_cos = nullptr, *rope_sin = nullptr;
  void *kv = nullptr;                                    // [seq][layer][2][n_kv][ctx][hd]
  size_t kv_bytes = 0;
  void *slot = nullptr;                                  // prefix slot: [layer][2][n_kv][slot_n][hd]
  int slot_cap = 0, slot_n = 0;
  float *x = nullptr, *xb = nullptr, *q = nullptr, *k = nullptr, *v = nullptr, *qr = nullptr, *att = nullptr;
  float *g = nullptr, *u = nullptr, *hb = nullptr, *logits = nullptr, *part = nullptr;
  float *qkv = nullptr, *gu = nullptr;                   // outputs of the row-concatenated projections
  void *gemm_b = nullptr;                                // f16 activation tiles of the tensor-core GEMM (max_batch >= 64)
  void *head_tiles = nullptr, *head_b = nullptr;         // F16 output head tiled for the GEMM, and its activation tiles
  void *tp_comm = nullptr;                               // NCCL communicator when the weights are sharded
  TpAr *tp_ar = nullptr;                                 // one-shot NVLink all-reduce (NULL: NCCL's)
  int64_t vocab0 = 0, vocab_n = 0;                       // vocab-split output head: this rank's rows (n 0: whole)
  int64_t vpad = 0;                                      // columns of a rank's padded logits slice
  float *lsend = nullptr, *lrecv = nullptr;              // this rank's slice [LB][vpad], all slices [size][LB][vpad]
  float *arg_v = nullptr;                                // argmax chunk results [LB][kArgmaxChunks]
  int32_t *arg_i = nullptr;
  int lb = 0;                                            // rows of the logits buffer
  float *topk_pv = nullptr;                              // top-k chunk candidates [LB][kTopkChunks][kTopkMax]
  int32_t *topk_pi = nullptr;
  float *topk_v = nullptr;                               // top-k results [LB][kTopkMax]
  int32_t *topk_i = nullptr;
  int32_t *pen = nullptr;                                // penalised tokens and their counts [2][kTopkMaxPen]
  int tp_rank = 0, tp_size = 1;
  int8_t *xq = nullptr;
  float *xd = nullptr;
  int32_t *xs = nullptr, *d_tok = nullptr, *d_pos = nullptr, *d_seq = nullptr, *d_npos = nullptr, *d_arg = nullptr;
  int32_t *counters = nullptr, *h_io = nullptr;          // h_io: pinned [4][max_batch] staging of the int arrays
  int nsplit = 1;
  std::vector<int> pos;                                   // positions held per sequence
  // decode graph cache: one graph per token count
  struct Graph { int n = 0; int want = 0; int adv = 0; int distinct = 0; cudaGraphExec_t exec = nullptr; };
  std::vector<Graph> graphs;
  std::vector<std::pair<int, int>> eager_seen;           // shapes (n, want | adv << 2) run once eagerly before being recorded
  int32_t *d_gen = nullptr, *d_step = nullptr;           // greedy generation: tokens [steps][n], step counter
  int64_t gen_cap = 0;
  bool use_graphs = true;

  int64_t qdim() const { return (int64_t)c.n_head * c.head_dim; }
  int64_t kvdim() const { return (int64_t)c.n_head_kv * c.head_dim; }
  int64_t seq_elems() const { return (int64_t)c.n_layer * 2 * kvdim() * c.ctx; }
  size_t el() const { return c.kv_f16 ? 2 : 4; }
  zllm_attn_geom geom() const {
    zllm_attn_geom g{};
    g.n_head = c.n_head; g.n_head_kv = c.n_head_kv; g.head_dim = c.head_dim; g.n_rot = c.n_rot; g.neox = c.neox;
    g.kv_f16 = c.kv_f16; g.ctx = c.ctx; g.rms_eps = c.rms_eps;
    g.seq_stride = seq_elems(); g.head_stride = (int64_t)c.ctx * c.head_dim;
    return g;
  }
  uint8_t *kv_block(int seq, int layer, int is_v) const {
    return (uint8_t *)kv + ((int64_t)seq * seq_elems() + ((int64_t)layer * 2 + is_v) * kvdim() * c.ctx) * el();
  }
};

static int fail(zllm_model *m, int rc) {
  if (rc == ZLLM_E_CUDA || rc == ZLLM_E_TIMEOUT || rc == ZLLM_E_OOM) m->failed = true;   // latched like pool.js:123-127
  return rc;
}

#define CK(expr, what)                                                   \
  do {                                                                   \
    cudaError_t e_ = (expr);                                             \
    if (e_ != cudaSuccess) return fail(m, zllm_cuda_fail(m->ctx, e_, what)); \
  } while (0)

extern "C" int zllm_model_create(zllm_ctx *ctx, const zllm_model_config *cfg, zllm_model **out) {
  if (!ctx || !cfg || !out) return ZLLM_E_ARG;
  *out = nullptr;
  const zllm_model_config &c = *cfg;
  if (c.n_embd <= 0 || c.n_layer <= 0 || c.n_ff <= 0 || c.n_head <= 0 || c.n_head_kv <= 0 || c.n_head % c.n_head_kv ||
      c.head_dim <= 0 || c.vocab <= 0 || c.ctx <= 0 || c.n_seq <= 0 || c.max_batch <= 0 || c.max_batch > 64 ||
      c.n_rot <= 0 || c.n_rot > c.head_dim || c.n_rot % 2 || c.n_embd % 32 || c.n_ff % 32 || (c.n_head * c.head_dim) % 32) {
    zllm_set_error(ctx, "zllm_model_create: bad configuration");
    return ZLLM_E_ARG;
  }
  if (!attn_supported(c.head_dim, c.n_head / c.n_head_kv)) {
    zllm_set_error(ctx, "zllm_model_create: head_dim %d with %d query heads per KV head is not supported", c.head_dim,
                   c.n_head / c.n_head_kv);
    return ZLLM_E_UNSUPPORTED;
  }
  zllm_model *m = new (std::nothrow) zllm_model();
  if (!m) return ZLLM_E_OOM;
  m->ctx = ctx;
  m->c = c;
  if (m->c.logits_batch < 1) m->c.logits_batch = 1;
  if (m->c.logits_batch > m->c.max_batch) m->c.logits_batch = m->c.max_batch;
  m->L.resize(c.n_layer);
  m->pos.assign(c.n_seq, 0);
  cudaSetDevice(ctx->device);
  if (cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking) != cudaSuccess) { delete m; return ZLLM_E_CUDA; }
  *out = m;
  return ZLLM_OK;
}

extern "C" int zllm_model_set_matrix(zllm_model *m, int kind, int layer, int ggml_type, int64_t rows, int64_t cols,
                                     const void *host, size_t nbytes) {
  if (!m || m->ready) return ZLLM_E_STATE;
  const zllm_model_config &c = m->c;
  int64_t er = 0, ec = 0;
  switch (kind) {
    case ZLLM_T_TOK_EMBD: er = c.vocab; ec = c.n_embd; break;
    case ZLLM_T_OUTPUT: er = m->vocab_n ? m->vocab_n : c.vocab; ec = c.n_embd; break;
    case ZLLM_T_WQ: er = m->qdim(); ec = c.n_embd; break;
    case ZLLM_T_WK: case ZLLM_T_WV: er = m->kvdim(); ec = c.n_embd; break;
    case ZLLM_T_WO: er = c.n_embd; ec = m->qdim(); break;
    case ZLLM_T_GATE: case ZLLM_T_UP: er = c.n_ff; ec = c.n_embd; break;
    case ZLLM_T_DOWN: er = c.n_embd; ec = c.n_ff; break;
    default: zllm_set_error(m->ctx, "zllm_model_set_matrix: unknown tensor kind %d", kind); return ZLLM_E_ARG;
  }
  const bool per_layer = kind >= ZLLM_T_WQ;
  if (per_layer && (layer < 0 || layer >= c.n_layer)) { zllm_set_error(m->ctx, "layer %d out of range", layer); return ZLLM_E_ARG; }
  if (rows != er || cols != ec) {
    zllm_set_error(m->ctx, "tensor kind %d: shape %lld x %lld, expected %lld x %lld", kind, (long long)rows, (long long)cols,
                   (long long)er, (long long)ec);
    return ZLLM_E_ARG;
  }
  zllm_weight *w = nullptr;
  int rc = zllm_weight_upload(m->ctx, ggml_type, rows, cols, host, nbytes, &w);
  if (rc) return rc;
  zllm_weight **slotp = nullptr;
  switch (kind) {
    case ZLLM_T_TOK_EMBD: slotp = &m->tok; break;
    case ZLLM_T_OUTPUT: slotp = &m->out; break;
    case ZLLM_T_WQ: slotp = &m->L[layer].w[WQ]; break;
    case ZLLM_T_WK: slotp = &m->L[layer].w[WK]; break;
    case ZLLM_T_WV: slotp = &m->L[layer].w[WV]; break;
    case ZLLM_T_WO: slotp = &m->L[layer].w[WO]; break;
    case ZLLM_T_GATE: slotp = &m->L[layer].w[GATE]; break;
    case ZLLM_T_UP: slotp = &m->L[layer].w[UP]; break;
    case ZLLM_T_DOWN: slotp = &m->L[layer].w[DOWN]; break;
  }
  if (*slotp) zllm_weight_free(*slotp);
  *slotp = w;
  return ZLLM_OK;
}

extern "C" int zllm_model_set_vector(zllm_model *m, int kind, int layer, const float *host, int64_t n) {
  if (!m || m->ready) return ZLLM_E_STATE;
  const zllm_model_config &c = m->c;
  int64_t en = 0;
  float **dst = nullptr;
  const bool per_layer = kind >= ZLLM_T_ATTN_NORM;
  if (per_layer && (layer < 0 || layer >= c.n_layer)) { zllm_set_error(m->ctx, "layer %d out of range", layer); return ZLLM_E_ARG; }
  switch (kind) {
    case ZLLM_T_OUTPUT_NORM: en = c.n_embd; dst = &m->out_norm; break;
    case ZLLM_T_ROPE_FREQS:
      if (n != c.n_rot / 2 || !host) { zllm_set_error(m->ctx, "rope_freqs: %lld values, expected %d", (long long)n, c.n_rot / 2); return ZLLM_E_ARG; }
      m->rope_freqs_host.assign(host, host + n);
      return ZLLM_OK;
    case ZLLM_T_ATTN_NORM: en = c.n_embd; dst = &m->L[layer].attn_norm; break;
    case ZLLM_T_FFN_NORM: en = c.n_embd; dst = &m->L[layer].ffn_norm; break;
    case ZLLM_T_Q_NORM: en = c.head_dim; dst = &m->L[layer].q_norm; break;
    case ZLLM_T_K_NORM: en = c.head_dim; dst = &m->L[layer].k_norm; break;
    case ZLLM_T_BQ: en = m->qdim(); dst = &m->L[layer].bq; break;
    case ZLLM_T_BK: en = m->kvdim(); dst = &m->L[layer].bk; break;
    case ZLLM_T_BV: en = m->kvdim(); dst = &m->L[layer].bv; break;
    default: zllm_set_error(m->ctx, "zllm_model_set_vector: unknown tensor kind %d", kind); return ZLLM_E_ARG;
  }
  if (n != en || !host) { zllm_set_error(m->ctx, "vector kind %d: %lld values, expected %lld", kind, (long long)n, (long long)en); return ZLLM_E_ARG; }
  if (!*dst) CK(dalloc(dst, (size_t)n), "cudaMalloc(vector)");
  CK(cudaMemcpyAsync(*dst, host, sizeof(float) * n, cudaMemcpyHostToDevice, m->stream), "vector upload");
  CK(cudaStreamSynchronize(m->stream), "vector upload");
  return ZLLM_OK;
}

// The rows of several matrices of one type and row length as one weight (the projections that read
// the same activation: q, k, v; gate, up), so one GEMV launch streams them all.  Every row's
// bytes are copied unchanged (for the k-quants to their place in the 16-row units), so every
// output row keeps its bits.  NULL when types or widths differ.  With `interleave` (equal row
// counts) row i of matrix j lands at row i * count + j instead: the gate / up pairs of the SwiGLU
// epilogue.
static zllm_weight *concat_rows(zllm_model *m, std::initializer_list<zllm_weight *> ws, bool interleave = false) {
  const zllm_weight *w0 = *ws.begin();
  int64_t rows = 0;
  for (const zllm_weight *w : ws) {
    if (!w || w->m.type != w0->m.type || w->m.cols != w0->m.cols || w->m.row_stride != w0->m.row_stride) return nullptr;
    if (interleave && w->m.rows != w0->m.rows) return nullptr;
    rows += w->m.rows;
  }
  zllm_weight *f = new (std::nothrow) zllm_weight();
  if (!f) return nullptr;
  f->ctx = m->ctx;
  f->m = w0->m;
  f->m.rows = rows;
  f->bytes = (size_t)dev_matrix_bytes(f->m.type, rows, f->m.cols);
  if (cudaMalloc((void **)&f->m.data, f->bytes) != cudaSuccess) { delete f; cudaGetLastError(); return nullptr; }
  size_t off = 0;
  cudaError_t e = cudaSuccess;
  const size_t rs = (size_t)w0->m.row_stride, count = ws.size();
  int j = 0;
  const bool kq = kq_type(w0->m.type);
  if (kq && rows % 16) e = cudaMemsetAsync(f->m.data, 0, f->bytes, m->stream);   // padding rows
  int64_t row0 = 0;
  for (const zllm_weight *w : ws) {
    if (e != cudaSuccess) break;
    if (kq) {
      e = interleave ? launch_kq_copy_rows(f->m, j, (int64_t)count, w->m, m->stream)
                     : launch_kq_copy_rows(f->m, row0, 1, w->m, m->stream);
      row0 += w->m.rows;
    } else if (interleave)
      e = cudaMemcpy2DAsync(f->m.data + j * rs, count * rs, w->m.data, rs, rs, (size_t)w->m.rows, cudaMemcpyDeviceToDevice,
                            m->stream);
    else
      e = cudaMemcpyAsync(f->m.data + off, w->m.data, w->bytes, cudaMemcpyDeviceToDevice, m->stream);
    off += w->bytes;
    j++;
  }
  if (e == cudaSuccess) e = cudaStreamSynchronize(m->stream);
  if (e != cudaSuccess) { cudaFree(f->m.data); delete f; cudaGetLastError(); return nullptr; }
  m->ctx->weights.insert(f);
  return f;
}

extern "C" void *zllm_model_stream(zllm_model *m) { return m ? (void *)m->stream : nullptr; }

extern "C" int zllm_tp_unique_id(zllm_ctx *ctx, void *out, size_t bytes) {
  if (!ctx || !out) return ZLLM_E_ARG;
  const char *why = "";
  if (tp_unique_id(out, bytes, &why)) { zllm_set_error(ctx, "zllm_tp_unique_id: %s", why); return ZLLM_E_UNSUPPORTED; }
  return ZLLM_OK;
}

extern "C" int zllm_model_set_tp(zllm_model *m, int rank, int size, const void *unique_id) {
  if (!m || !unique_id || size < 1 || rank < 0 || rank >= size) return ZLLM_E_ARG;
  if (m->ready || m->tp_comm) { zllm_set_error(m->ctx, "zllm_model_set_tp: call it once, before the first pass"); return ZLLM_E_STATE; }
  if (size == 1) return ZLLM_OK;
  cudaSetDevice(m->ctx->device);
  const char *why = "";
  if (tp_comm_init(&m->tp_comm, rank, size, unique_id, &why)) {
    zllm_set_error(m->ctx, "zllm_model_set_tp: %s", why);
    return ZLLM_E_CUDA;
  }
  m->tp_rank = rank;
  m->tp_size = size;
  return ZLLM_OK;
}

extern "C" int zllm_model_set_vocab_shard(zllm_model *m, int64_t v0, int64_t n) {
  if (!m) return ZLLM_E_ARG;
  if (m->ready || m->out || m->tp_size <= 1) {
    zllm_set_error(m->ctx, "zllm_model_set_vocab_shard: call it after zllm_model_set_tp, before the output matrix and the first pass");
    return ZLLM_E_STATE;
  }
  const int64_t V = m->c.vocab, a = (int64_t)m->tp_rank * V / m->tp_size, b = (int64_t)(m->tp_rank + 1) * V / m->tp_size;
  if (v0 != a || n != b - a) {
    zllm_set_error(m->ctx, "zllm_model_set_vocab_shard: rank %d of %d holds rows [%lld, %lld) of the output head", m->tp_rank,
                   m->tp_size, (long long)a, (long long)b);
    return ZLLM_E_ARG;
  }
  m->vocab0 = v0;
  m->vocab_n = n;
  return ZLLM_OK;
}

extern "C" int zllm_model_ready(zllm_model *m) {
  if (!m) return ZLLM_E_ARG;
  if (m->ready) return ZLLM_OK;
  const zllm_model_config &c = m->c;
  if (!m->tok || !m->out_norm) { zllm_set_error(m->ctx, "model: token_embd / output_norm missing"); return ZLLM_E_ARG; }
  for (int l = 0; l < c.n_layer; l++) {
    for (int i = 0; i < 7; i++)
      if (!m->L[l].w[i]) { zllm_set_error(m->ctx, "model: layer %d matrix %d missing", l, i); return ZLLM_E_ARG; }
    if (!m->L[l].attn_norm || !m->L[l].ffn_norm) { zllm_set_error(m->ctx, "model: layer %d norms missing", l); return ZLLM_E_ARG; }
  }
  // one launch per group of projections that read the same activation
  for (auto &L : m->L) {
    if ((L.qkv = concat_rows(m, {L.w[WQ], L.w[WK], L.w[WV]})))
      for (int i : {WQ, WK, WV}) { zllm_weight_free(L.w[i]); L.w[i] = nullptr; }
    // gate / up interleaved for the SwiGLU epilogue, which only the k-quant GEMV has
    if (kq_type(L.w[GATE]->m.type) && (L.gu = concat_rows(m, {L.w[GATE], L.w[UP]}, true)))
      for (int i : {GATE, UP}) { zllm_weight_free(L.w[i]); L.w[i] = nullptr; }
  }
  const int MB = c.max_batch;
  const int64_t E = c.n_embd, F = c.n_ff, Q = m->qdim(), KV = m->kvdim();
  const int64_t KX = std::max(E, std::max(F, Q));
  const int LB = std::max(c.logits_batch, c.n_seq < MB ? c.n_seq : MB);
  CK(dalloc(&m->rope_cos, (size_t)c.ctx * c.n_rot / 2), "rope");
  CK(dalloc(&m->rope_sin, (size_t)c.ctx * c.n_rot / 2), "rope");
  int rc = zllm_rope_tables(m->ctx, c.n_rot, c.rope_base, c.ctx, m->rope_freqs_host.empty() ? nullptr : m->rope_freqs_host.data(),
                            m->rope_cos, m->rope_sin);
  if (rc) return fail(m, rc);
  m->kv_bytes = (size_t)c.n_seq * m->seq_elems() * m->el();
  CK(cudaMalloc(&m->kv, m->kv_bytes), "cudaMalloc(KV cache)");
  CK(cudaMemsetAsync(m->kv, 0, m->kv_bytes, m->stream), "KV clear");
  CK(dalloc(&m->x, MB * E), "act");
  CK(dalloc(&m->xb, MB * KX), "act");
  CK(dalloc(&m->xq, MB * KX), "act");
  CK(dalloc(&m->xd, MB * KX / 32), "act");
  CK(dalloc(&m->xs, MB * KX / 32), "act");
  CK(dalloc(&m->q, MB * Q), "act");
  CK(dalloc(&m->qkv, MB * (Q + 2 * KV)), "act");
  CK(dalloc(&m->gu, MB * 2 * F), "act");
  CK(dalloc(&m->k, MB * KV), "act");
  CK(dalloc(&m->v, MB * KV), "act");
  CK(dalloc(&m->qr, MB * Q), "act");
  CK(dalloc(&m->att, MB * Q), "act");
  CK(dalloc(&m->g, MB * F), "act");
  CK(dalloc(&m->u, MB * F), "act");
  CK(dalloc(&m->hb, MB * F), "act");
  if (MB >= kGemmMinTokens) {
    // passes of kGemmMinTokens or more tokens run the k-quant projections as tensor-core GEMMs
    size_t gb = gemm_b_bytes(KX, MB);
    for (auto &L : m->L)
      for (zllm_weight *w : {L.w[0], L.w[1], L.w[2], L.w[3], L.w[4], L.w[5], L.w[6], L.qkv, L.gu})
        if (w && kq_type(w->m.type) && zllm_weight_gemm_ok(m->ctx, w))
          for (int n = kGemmMinTokens; n <= MB; n++) gb = std::max(gb, gemm_act_bytes(w, n));   // split-K varies with n
    CK(cudaMalloc(&m->gemm_b, gb), "GEMM activation tiles");
  }
  CK(dalloc(&m->logits, (size_t)LB * c.vocab), "logits");
  CK(dalloc(&m->arg_v, (size_t)LB * kArgmaxChunks), "argmax scratch");
  CK(dalloc(&m->arg_i, (size_t)LB * kArgmaxChunks), "argmax scratch");
  m->lb = LB;
  CK(dalloc(&m->topk_pv, (size_t)LB * kTopkChunks * kTopkMax), "top-k scratch");
  CK(dalloc(&m->topk_pi, (size_t)LB * kTopkChunks * kTopkMax), "top-k scratch");
  CK(dalloc(&m->topk_v, (size_t)LB * kTopkMax), "top-k scratch");
  CK(dalloc(&m->topk_i, (size_t)LB * kTopkMax), "top-k scratch");
  CK(dalloc(&m->pen, (size_t)2 * kTopkMaxPen), "top-k scratch");
  if (m->vocab_n) {
    if (!m->out) { zllm_set_error(m->ctx, "model: a vocab-split head needs its own output matrix"); return fail(m, ZLLM_E_ARG); }
    m->vpad = (c.vocab + m->tp_size - 1) / m->tp_size;
    CK(dalloc(&m->lsend, (size_t)LB * m->vpad), "logits slice");
    CK(dalloc(&m->lrecv, (size_t)m->tp_size * LB * m->vpad), "gathered logits");
  }
  {
    // an F16 output head that passes of kHeadGemmMinRows or more logit rows will use (batched decode,
    // all-position logits) is also kept tiled for the tensor-core GEMM
    const zllm_weight *ow = m->out ? m->out : m->tok;
    if (LB >= kHeadGemmMinRows && ow->m.type == T_F16 && E % 64 == 0) {
      CK(cudaMalloc(&m->head_tiles, gemm_f16_tiles_bytes(ow->m.rows, E)), "output head tiles");
      CK(launch_gemm_tile_f16(ow->m, m->head_tiles, m->stream), "output head tiling");
      CK(cudaMalloc(&m->head_b, gemm_b_bytes(E, LB)), "output head activation tiles");
    }
  }
  CK(dalloc(&m->d_tok, MB), "ids");
  CK(dalloc(&m->d_pos, MB), "ids");
  CK(dalloc(&m->d_seq, MB), "ids");
  CK(dalloc(&m->d_npos, MB), "ids");
  CK(dalloc(&m->d_arg, MB), "ids");
  CK(cudaHostAlloc((void **)&m->h_io, sizeof(int32_t) * 4 * MB, cudaHostAllocDefault), "pinned ids");
  const zllm_attn_geom g = m->geom();
  m->nsplit = zllm_attn_splits(m->ctx, &g, 1, c.ctx);     // the most splits any pass uses (one query)
  const int group = c.n_head / c.n_head_kv;
  CK(dalloc(&m->part, (size_t)MB * c.n_head_kv * m->nsplit * group * (c.head_dim + 2)), "attention scratch");
  CK(dalloc(&m->counters, (size_t)MB * c.n_head_kv), "attention counters");
  CK(cudaMemsetAsync(m->counters, 0, sizeof(int32_t) * MB * c.n_head_kv, m->stream), "counters");
  if (m->tp_size > 1) {
    // the one-shot all-reduce when every peer's buffer maps (collective over the ranks); else NCCL
    const char *why = "";
    if (tp_ar_setup(m->tp_comm, m->tp_rank, m->tp_size, (int64_t)MB * E, m->stream, &m->tp_ar, &why)) m->tp_ar = nullptr;
  }
  CK(cudaStreamSynchronize(m->stream), "model ready");
  m->ready = true;
  return ZLLM_OK;
}

// ------------------------------------------------------------------------------------ the pass
// 64 or more tokens (a prefill chunk) on a k-quant weight that qualifies: the tensor-core GEMM on
// f16 hi / lo tiles of the quantized activation (~1e-5 of the largest output from the exact
// per-token arithmetic).  Smaller batches (batched decode) keep the per-token kernel, which streams
// the weights faster at that size and stays bit-identical to single-token passes.
static bool use_gemm(const zllm_model *m, const zllm_weight *w, int n) {
  return n >= kGemmMinTokens && m->gemm_b && w->gemm_ok == 1;
}
static cudaError_t gemm(zllm_model *m, const zllm_weight *w, int n, float *y, int64_t ys, const float *y_add, int64_t k,
                        bool swiglu) {
  const ActView a{m->xq, m->xd, m->xs, nullptr, k};
  return gemm_run(w, a, n, m->gemm_b, y, ys, y_add, m->ctx->status_dev, m->stream, swiglu);
}

static cudaError_t gemv(zllm_model *m, const zllm_weight *w, int n, float *y, int64_t ys, const float *y_add, const float *xf,
                        int64_t k, bool pdl = false) {
  if (use_gemm(m, w, n)) return gemm(m, w, n, y, ys, y_add, k, false);
  ActView a{m->xq, m->xd, m->xs, xf, k};
  const char *why = "";
  return launch_gemv(w->m, a, n, y, ys, y_add, m->ctx->status_dev, m->ctx->num_sms, m->stream, pdl, &why);
}

// A k-quant GEMV with fused work: `act` may carry the f32 activation alone (one token).
static cudaError_t gemv_ex(zllm_model *m, const zllm_weight *w, int n, float *y, int64_t ys, const float *y_add,
                           const ActView &act, const GemvFuse &fz, bool pdl = false) {
  if (act.xq && !fz.norm_w && use_gemm(m, w, n)) return gemm(m, w, n, y, ys, y_add, act.k, fz.swiglu);
  const char *why = "";
  return launch_gemv_kq_ex(w->m, act, n, y, ys, y_add, fz, m->ctx->status_dev, m->ctx->num_sms, m->stream, pdl, &why);
}

// Sum the ranks' x (n tokens x n_embd) in place: the all-reduce after a row-parallel projection.
static cudaError_t tp_reduce(zllm_model *m, int n) {
  if (m->tp_size <= 1) return cudaSuccess;
  // chained with programmatic dependent launch: the all-reduce waits for the GEMV in hardware and the
  // next GEMV streams its weights in while the ranks exchange their partial sums
  if (m->tp_ar) return tp_ar_sum(m->tp_ar, m->x, (int64_t)n * m->c.n_embd, m->ctx->status_dev, m->stream, true);
  const char *why = "";
  return tp_allreduce_sum(m->tp_comm, m->x, (size_t)n * m->c.n_embd, m->stream, &why);
}

// Enqueue the pass for n tokens whose ids / positions / sequences are already in d_tok / d_pos /
// d_seq / d_npos.  want: 0 no logits, 1 the last token's, 2 every token's.  distinct: every token
// belongs to a different sequence (decode), so the attention kernel can do the q/k/v
// post-processing and the KV append of its own query (no token reads another token's new row).
static cudaError_t enqueue_pass(zllm_model *m, int n, int want, bool distinct) {
  const zllm_model_config &c = m->c;
  const int64_t E = c.n_embd, F = c.n_ff, Q = m->qdim(), KV = m->kvdim();
  cudaStream_t s = m->stream;
  cudaError_t e;
  // Programmatic dependent launch (a kernel streams its weights or cache rows in before it waits
  // for its input): in single-token passes for the GEMVs, the attention and the o projection after
  // it; and for every k-quant GEMV of a multi-token pass (measured: +2 % at 32 sequences).
#define RUN(x) do { if ((e = (x)) != cudaSuccess) return e; } while (0)
  RUN(launch_embed(m->tok->m, m->d_tok, n, m->x, s, false));
  const zllm_attn_geom g = m->geom();
  for (int l = 0; l < c.n_layer; l++) {
    const Layer &L = m->L[l];
    // a single-token pass folds the norms, the activation quantization and SwiGLU into the k-quant
    // GEMVs (the same arithmetic as the separate kernels, so the same bits)
    const bool one = n == 1;
    const bool fuse_qkv = one && L.qkv && kq_type(L.qkv->m.type);
    if (!fuse_qkv) RUN(launch_rmsnorm_quant(m->x, L.attn_norm, (int)E, n, c.rms_eps, m->xb, m->xq, m->xd, m->xs, s, false));
    QkvPostArgs pa{};
    if (L.qkv) {
      if (fuse_qkv) {
        GemvFuse fz;
        fz.norm_w = L.attn_norm;
        fz.eps = c.rms_eps;
        RUN(gemv_ex(m, L.qkv, 1, m->qkv, Q + 2 * KV, nullptr, ActView{nullptr, nullptr, nullptr, m->x, E}, fz, l > 0));
      } else {
        RUN(gemv(m, L.qkv, n, m->qkv, Q + 2 * KV, nullptr, m->xb, E, true));
      }
      pa.q = m->qkv; pa.k = m->qkv + Q; pa.v = m->qkv + Q + KV; pa.q_stride = Q + 2 * KV; pa.kv_stride = Q + 2 * KV;
    } else {
      RUN(gemv(m, L.w[WQ], n, m->q, Q, nullptr, m->xb, E));
      RUN(gemv(m, L.w[WK], n, m->k, KV, nullptr, m->xb, E));
      RUN(gemv(m, L.w[WV], n, m->v, KV, nullptr, m->xb, E));
      pa.q = m->q; pa.k = m->k; pa.v = m->v; pa.q_stride = Q; pa.kv_stride = KV;
    }
    pa.bq = L.bq; pa.bk = L.bk; pa.bv = L.bv; pa.q_norm = L.q_norm; pa.k_norm = L.k_norm;
    pa.rope_cos = m->rope_cos; pa.rope_sin = m->rope_sin; pa.pos = m->d_pos; pa.seq = m->d_seq;
    pa.q_out = m->qr; pa.q_out_stride = Q;
    pa.kcache = m->kv_block(0, l, 0); pa.vcache = m->kv_block(0, l, 1);
    pa.seq_stride = g.seq_stride; pa.head_stride = g.head_stride;
    pa.n_head = c.n_head; pa.n_kv = c.n_head_kv; pa.head_dim = c.head_dim; pa.n_rot = c.n_rot; pa.neox = c.neox;
    pa.kv_f16 = c.kv_f16; pa.ntok = n; pa.eps = c.rms_eps;
    if (!distinct) RUN(launch_qkv_post(pa, s, false));
    AttnArgs aa{};
    aa.fused = distinct ? 1 : 0;
    aa.post = pa;
    aa.q = m->qr; aa.seq = m->d_seq; aa.kcache = m->kv_block(0, l, 0); aa.vcache = m->kv_block(0, l, 1);
    aa.seq_stride = g.seq_stride; aa.head_stride = g.head_stride; aa.npos = m->d_npos; aa.out = m->att;
    aa.partial = m->part; aa.counters = m->counters; aa.status = m->ctx->status_dev;
    aa.scale = (float)(1.0 / std::sqrt((double)c.head_dim));
    // one split count for every pass: a query's context partition (and so its rounding) does not
    // depend on how many tokens share the pass, so batched passes equal token-by-token ones bit for bit
    aa.n_head = c.n_head; aa.n_kv = c.n_head_kv; aa.head_dim = c.head_dim; aa.nseq = n; aa.nsplit = m->nsplit;
    // single-token passes chain the attention and the o projection with programmatic dependent
    // launch: the attention streams its first K/V rows while the q/k/v GEMV finishes, and the o
    // GEMV's CTAs land on the SMs the attention leaves free and stream their weights meanwhile
    RUN(launch_attn(aa, c.kv_f16 != 0, s, one));
    // tensor parallel: attn_output and ffn_down are row-parallel, so each rank holds a partial sum;
    // rank 0 adds the residual, the others overwrite x, and one all-reduce gives every rank
    // x + sum of the partials
    const float *res = m->tp_size > 1 && m->tp_rank != 0 ? nullptr : m->x;
    if (one && kq_type(L.w[WO]->m.type)) {
      RUN(gemv_ex(m, L.w[WO], 1, m->x, E, res, ActView{nullptr, nullptr, nullptr, m->att, Q}, GemvFuse{}, true));
    } else {
      RUN(launch_quantize(m->att, Q, n, m->xq, m->xd, m->xs, m->ctx->status_dev, s, false));
      RUN(gemv(m, L.w[WO], n, m->x, E, res, m->att, Q, true));                      // x += wo . att
    }
    RUN(tp_reduce(m, n));
    if (L.gu) {
      // interleaved (gate, up) rows; the GEMV writes hb = silu(gate) * up
      GemvFuse fz;
      fz.swiglu = true;
      if (one) {
        fz.norm_w = L.ffn_norm;
        fz.eps = c.rms_eps;
        RUN(gemv_ex(m, L.gu, 1, m->hb, F, nullptr, ActView{nullptr, nullptr, nullptr, m->x, E}, fz, true));
      } else {
        RUN(launch_rmsnorm_quant(m->x, L.ffn_norm, (int)E, n, c.rms_eps, m->xb, m->xq, m->xd, m->xs, s, false));
        RUN(gemv_ex(m, L.gu, n, m->hb, F, nullptr, ActView{m->xq, m->xd, m->xs, m->xb, E}, fz, true));
      }
      if (one && kq_type(L.w[DOWN]->m.type)) {
        RUN(gemv_ex(m, L.w[DOWN], 1, m->x, E, res, ActView{nullptr, nullptr, nullptr, m->hb, F}, GemvFuse{}, true));
      } else {
        RUN(launch_quantize(m->hb, F, n, m->xq, m->xd, m->xs, m->ctx->status_dev, s, false));
        RUN(gemv(m, L.w[DOWN], n, m->x, E, res, m->hb, F, true));                   // x += down . hb
      }
      RUN(tp_reduce(m, n));
    } else {
      RUN(launch_rmsnorm_quant(m->x, L.ffn_norm, (int)E, n, c.rms_eps, m->xb, m->xq, m->xd, m->xs, s, false));
      RUN(gemv(m, L.w[GATE], n, m->g, F, nullptr, m->xb, E));
      RUN(gemv(m, L.w[UP], n, m->u, F, nullptr, m->xb, E));
      RUN(launch_swiglu_quant(m->g, m->u, (int)F, n, F, m->hb, m->xq, m->xd, m->xs, s, false));
      RUN(gemv(m, L.w[DOWN], n, m->x, E, res, m->hb, F));                     // x += down . hb
      RUN(tp_reduce(m, n));
    }
  }
  if (want) {
    const zllm_weight *ow = m->out ? m->out : m->tok;
    const int nl = want == 2 ? n : 1;
    const float *xl = want == 2 ? m->x : m->x + (int64_t)(n - 1) * E;
    RUN(launch_rmsnorm_quant(xl, m->out_norm, (int)E, nl, c.rms_eps, m->xb, m->xq, m->xd, m->xs, s, false));
    // a vocab-split head writes this rank's slice, and the ranks gather every slice into the logits
    float *lout = m->vocab_n ? m->lsend : m->logits;
    const int64_t lstride = m->vocab_n ? m->vpad : c.vocab;
    if (nl >= kHeadGemmMinRows && m->head_tiles) {
      RUN(launch_gemm_prep_f32(m->xb, E, E, nl, m->head_b, s));
      RUN(launch_gemm_f16_tiled(m->head_tiles, ow->m.rows, E, m->head_b, nl, lout, lstride, m->ctx->status_dev, s));
    } else {
      RUN(gemv(m, ow, nl, lout, lstride, nullptr, m->xb, E));
    }
    if (m->vocab_n) {
      const char *why = "";
      RUN(tp_allgather(m->tp_comm, m->lsend, m->lrecv, (size_t)nl * m->vpad, s, &why));
      RUN(launch_vocab_gather(m->lrecv, nl, m->vpad, c.vocab, m->tp_size, m->logits, s));
    }
    RUN(launch_argmax(m->logits, c.vocab, c.vocab, nl, m->d_arg, m->arg_v, m->arg_i, s, false));
  }
#undef RUN
  return cudaSuccess;
}

// Validate, stage the int arrays, run the pass (replaying a recorded graph when possible), copy out.
// One pass of n tokens (with `adv`: followed by the greedy advance of generate), replayed from a
// recorded graph when the shape was seen before.
static int launch_shape(zllm_model *m, int n, int want, bool adv, bool distinct) {
  cudaStream_t s = m->stream;
  const int key = want | (adv ? 4 : 0) | (distinct ? 8 : 0);
  auto enqueue = [&]() -> cudaError_t {
    cudaError_t e = enqueue_pass(m, n, want, distinct);
    if (e == cudaSuccess && adv) e = launch_advance(m->d_arg, n, m->d_tok, m->d_pos, m->d_npos, m->d_gen, m->d_step, s, false);
    return e;
  };
  cudaGraphExec_t exec = nullptr;
  bool eager = !m->use_graphs;
  if (!eager) {
    for (auto &gr : m->graphs)
      if (gr.n == n && gr.want == want && gr.adv == (adv ? 1 : 0) && gr.distinct == (distinct ? 1 : 0)) exec = gr.exec;
    // the first pass of a shape runs eagerly (kernel attributes are set outside any capture)
    if (!exec && std::find(m->eager_seen.begin(), m->eager_seen.end(), std::make_pair(n, key)) == m->eager_seen.end()) {
      m->eager_seen.push_back({n, key});
      eager = true;
    }
  }
  if (!eager) {
    if (!exec) {
      cudaGraph_t graph = nullptr;
      CK(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal), "graph capture");
      cudaError_t e = enqueue();
      cudaError_t e2 = cudaStreamEndCapture(s, &graph);
      if (e != cudaSuccess || e2 != cudaSuccess) {
        if (graph) cudaGraphDestroy(graph);
        cudaGetLastError();
        return fail(m, zllm_cuda_fail(m->ctx, e != cudaSuccess ? e : e2, "recording the pass"));
      }
      e = cudaGraphInstantiate(&exec, graph, 0);
      cudaGraphDestroy(graph);
      if (e != cudaSuccess) return fail(m, zllm_cuda_fail(m->ctx, e, "cudaGraphInstantiate"));
      m->graphs.push_back({n, want, adv ? 1 : 0, distinct ? 1 : 0, exec});
    }
    CK(cudaGraphLaunch(exec, s), "cudaGraphLaunch");
  } else {
    CK(enqueue(), "pass launch");
  }
  return ZLLM_OK;
}

static int run(zllm_model *m, const int32_t *seqs, int single_seq, const int32_t *tokens, int n, int want, float *logits_host,
               int32_t *argmax_host) {
  if (!m) return ZLLM_E_ARG;
  if (m->closed) { zllm_set_error(m->ctx, "model is closed"); return ZLLM_E_STATE; }
  if (m->failed) return ZLLM_E_STATE;
  if (!m->ready) { int rc = zllm_model_ready(m); if (rc) return rc; }
  const zllm_model_config &c = m->c;
  if (n < 1 || n > c.max_batch) { zllm_set_error(m->ctx, "batch of %d tokens (max %d)", n, c.max_batch); return ZLLM_E_BATCH; }
  if (want == 2 && n > c.logits_batch && single_seq >= 0) {
    zllm_set_error(m->ctx, "logits for all positions of a batch of %d tokens (this pool supports %d; raise the logitsBatch option)",
                   n, c.logits_batch);
    return ZLLM_E_BATCH;
  }
  for (int i = 0; i < n; i++)
    if (!(tokens[i] >= 0 && tokens[i] < c.vocab)) { zllm_set_error(m->ctx, "token id %d out of range", tokens[i]); return ZLLM_E_TOKEN; }
  int32_t *ht = m->h_io, *hp = m->h_io + c.max_batch, *hs = m->h_io + 2 * c.max_batch, *hn = m->h_io + 3 * c.max_batch;
  std::vector<int> added(c.n_seq, 0);
  for (int i = 0; i < n; i++) {
    const int sq = single_seq >= 0 ? single_seq : seqs[i];
    if (sq < 0 || sq >= c.n_seq) { zllm_set_error(m->ctx, "sequence %d out of range", sq); return ZLLM_E_ARG; }
    const int p = m->pos[sq] + added[sq]++;
    if (p >= c.ctx) { zllm_set_error(m->ctx, "context full (%d tokens)", c.ctx); return ZLLM_E_CTX_FULL; }
    ht[i] = tokens[i]; hp[i] = p; hs[i] = sq; hn[i] = p + 1;
  }
  cudaStream_t s = m->stream;
  CK(cudaMemcpyAsync(m->d_tok, ht, sizeof(int32_t) * n, cudaMemcpyHostToDevice, s), "ids");
  CK(cudaMemcpyAsync(m->d_pos, hp, sizeof(int32_t) * n, cudaMemcpyHostToDevice, s), "ids");
  CK(cudaMemcpyAsync(m->d_seq, hs, sizeof(int32_t) * n, cudaMemcpyHostToDevice, s), "ids");
  CK(cudaMemcpyAsync(m->d_npos, hn, sizeof(int32_t) * n, cudaMemcpyHostToDevice, s), "ids");
  bool distinct = true;
  for (int sq = 0; sq < c.n_seq; sq++) distinct = distinct && added[sq] <= 1;
  int rc0 = launch_shape(m, n, want, false, distinct);
  if (rc0) return rc0;
  const int nl = want == 2 ? n : 1;
  if (want && logits_host)
    CK(cudaMemcpyAsync(logits_host, m->logits, sizeof(float) * nl * c.vocab, cudaMemcpyDeviceToHost, s), "logits");
  if (want && argmax_host) CK(cudaMemcpyAsync(argmax_host, m->d_arg, sizeof(int32_t) * nl, cudaMemcpyDeviceToHost, s), "argmax");
  int rc = zllm_finish(m->ctx, s);             // one synchronization; the status word comes back on the stream
  if (rc) return fail(m, rc);
  for (int sq = 0; sq < c.n_seq; sq++) m->pos[sq] += added[sq];
  return ZLLM_OK;
}

extern "C" int zllm_model_forward(zllm_model *m, int seq, const int32_t *tokens, int n, int want, float *logits_host,
                                  int32_t *argmax_host) {
  if (!m || !tokens || want < 0 || want > 2) return ZLLM_E_ARG;
  if (seq < 0 || seq >= m->c.n_seq) { zllm_set_error(m->ctx, "sequence %d out of range", seq); return ZLLM_E_ARG; }
  return run(m, nullptr, seq, tokens, n, want, logits_host, argmax_host);
}

extern "C" int zllm_model_decode(zllm_model *m, const int32_t *seqs, const int32_t *tokens, int n, float *logits_host,
                                 int32_t *argmax_host) {
  if (!m || !tokens || !seqs) return ZLLM_E_ARG;
  for (int i = 0; i < n; i++)
    for (int j = 0; j < i; j++)
      if (seqs[i] == seqs[j]) { zllm_set_error(m->ctx, "zllm_model_decode: sequence %d appears twice", seqs[i]); return ZLLM_E_ARG; }
  return run(m, seqs, -1, tokens, n, 2, logits_host, argmax_host);
}

// Greedy generation on the device: `steps` passes, the first on `tokens`, each later one on the
// argmax of the previous pass's logits (generate.js:4-10 with greedy sampling), with no host work
// between passes.  n == 1 with seqs == NULL continues sequence `seq`; otherwise one token for each
// of the n distinct sequences.  out_host[steps][n] receives every pass's argmax.
extern "C" int zllm_model_generate(zllm_model *m, int seq, const int32_t *seqs, const int32_t *tokens, int n, int steps,
                                   int32_t *out_host) {
  if (!m || !tokens || !out_host || steps < 1 || (!seqs && n != 1)) return ZLLM_E_ARG;
  if (m->closed) { zllm_set_error(m->ctx, "model is closed"); return ZLLM_E_STATE; }
  if (m->failed) return ZLLM_E_STATE;
  if (!m->ready) { int rc = zllm_model_ready(m); if (rc) return rc; }
  const zllm_model_config &c = m->c;
  if (n < 1 || n > c.max_batch) { zllm_set_error(m->ctx, "batch of %d tokens (max %d)", n, c.max_batch); return ZLLM_E_BATCH; }
  int32_t *ht = m->h_io, *hp = m->h_io + c.max_batch, *hs = m->h_io + 2 * c.max_batch, *hn = m->h_io + 3 * c.max_batch;
  for (int i = 0; i < n; i++) {
    const int sq = seqs ? seqs[i] : seq;
    if (sq < 0 || sq >= c.n_seq) { zllm_set_error(m->ctx, "sequence %d out of range", sq); return ZLLM_E_ARG; }
    for (int j = 0; j < i; j++)
      if (seqs[j] == sq) { zllm_set_error(m->ctx, "zllm_model_generate: sequence %d appears twice", sq); return ZLLM_E_ARG; }
    if (!(tokens[i] >= 0 && tokens[i] < c.vocab)) { zllm_set_error(m->ctx, "token id %d out of range", tokens[i]); return ZLLM_E_TOKEN; }
    if (m->pos[sq] + steps > c.ctx) { zllm_set_error(m->ctx, "context full (%d tokens)", c.ctx); return ZLLM_E_CTX_FULL; }
    ht[i] = tokens[i]; hp[i] = m->pos[sq]; hs[i] = sq; hn[i] = m->pos[sq] + 1;
  }
  cudaStream_t s = m->stream;
  if ((int64_t)steps * n > m->gen_cap) {
    CK(cudaStreamSynchronize(s), "generate");
    if (m->d_gen) cudaFree(m->d_gen);
    m->d_gen = nullptr;
    m->gen_cap = 0;
    CK(cudaMalloc(&m->d_gen, sizeof(int32_t) * (size_t)steps * n), "cudaMalloc(generated tokens)");
    m->gen_cap = (int64_t)steps * n;
    // recorded advance graphs hold the old buffer
    for (auto it = m->graphs.begin(); it != m->graphs.end();)
      if (it->adv) { cudaGraphExecDestroy(it->exec); it = m->graphs.erase(it); } else ++it;
  }
  if (!m->d_step) CK(cudaMalloc(&m->d_step, sizeof(int32_t)), "cudaMalloc(step)");
  CK(cudaMemsetAsync(m->d_step, 0, sizeof(int32_t), s), "step");
  CK(cudaMemcpyAsync(m->d_tok, ht, sizeof(int32_t) * n, cudaMemcpyHostToDevice, s), "ids");
  CK(cudaMemcpyAsync(m->d_pos, hp, sizeof(int32_t) * n, cudaMemcpyHostToDevice, s), "ids");
  CK(cudaMemcpyAsync(m->d_seq, hs, sizeof(int32_t) * n, cudaMemcpyHostToDevice, s), "ids");
  CK(cudaMemcpyAsync(m->d_npos, hn, sizeof(int32_t) * n, cudaMemcpyHostToDevice, s), "ids");
  const int want = n == 1 ? 1 : 2;
  for (int i = 0; i < steps; i++) {
    int rc = launch_shape(m, n, want, true, true);            // distinct sequences, checked above
    if (rc) return rc;
  }
  CK(cudaMemcpyAsync(out_host, m->d_gen, sizeof(int32_t) * (size_t)steps * n, cudaMemcpyDeviceToHost, s), "tokens");
  int rc = zllm_finish(m->ctx, s);
  if (rc) return fail(m, rc);
  for (int i = 0; i < n; i++) m->pos[seqs ? seqs[i] : seq] += steps;
  return ZLLM_OK;
}

extern "C" int zllm_model_pos(const zllm_model *m, int seq) {
  if (!m || seq < 0 || seq >= m->c.n_seq) return ZLLM_E_ARG;
  return m->pos[seq];
}

extern "C" int zllm_model_truncate(zllm_model *m, int seq, int n) {
  if (!m || seq < 0 || seq >= m->c.n_seq) return ZLLM_E_ARG;
  if (n < 0) n = 0;
  if (n < m->pos[seq]) m->pos[seq] = n;            // a KV cache is positional (src/compute/pool.js:278-281)
  return ZLLM_OK;
}

extern "C" int zllm_model_reset(zllm_model *m, int seq) { return zllm_model_truncate(m, seq, 0); }

extern "C" int zllm_model_set_graphs(zllm_model *m, int on) {
  if (!m) return ZLLM_E_ARG;
  m->use_graphs = on != 0;
  return ZLLM_OK;
}

extern "C" void *zllm_model_logits(zllm_model *m) { return m ? m->logits : nullptr; }

extern "C" int zllm_model_tp_collective(zllm_model *m) {
  if (!m || m->tp_size <= 1) return 0;
  return m->tp_ar ? 2 : 1;
}

static int kv_io(zllm_model *m, int seq, int layer, int is_v, int n, float *host, bool get) {
  if (!m || !host || seq < 0 || seq >= m->c.n_seq || layer < 0 || layer >= m->c.n_layer || (is_v != 0 && is_v != 1) ||
      n < 0 || n > m->c.ctx)
    return ZLLM_E_ARG;
  if (m->failed) return ZLLM_E_STATE;
  if (!m->ready) { int rc = zllm_model_ready(m); if (rc) return rc; }
  if (n == 0) return ZLLM_OK;
  const zllm_attn_geom g = m->geom();
  void *stage;
  int rc = zllm_scratch(m->ctx, 12, sizeof(float) * n * m->kvdim(), &stage);
  if (rc) return rc;
  cudaStream_t s = m->stream;
  if (get) {
    rc = zllm_kv_export(m->ctx, &g, m->kv_block(seq, layer, is_v), n, (float *)stage, s);
    if (rc) return rc;
    CK(cudaMemcpyAsync(host, stage, sizeof(float) * n * m->kvdim(), cudaMemcpyDeviceToHost, s), "kvGet");
  } else {
    CK(cudaMemcpyAsync(stage, host, sizeof(float) * n * m->kvdim(), cudaMemcpyHostToDevice, s), "kvSet");
    rc = zllm_kv_import(m->ctx, &g, m->kv_block(seq, layer, is_v), n, (const float *)stage, s);
    if (rc) return rc;
  }
  CK(cudaStreamSynchronize(s), get ? "kvGet" : "kvSet");
  return ZLLM_OK;
}

extern "C" int zllm_model_kv_get(zllm_model *m, int seq, int layer, int is_v, int n, float *out) {
  return kv_io(m, seq, layer, is_v, n, out, true);
}
extern "C" int zllm_model_kv_set(zllm_model *m, int seq, int layer, int is_v, int n, const float *in) {
  return kv_io(m, seq, layer, is_v, n, const_cast<float *>(in), false);
}

// The k best logits of each of the last pass's first `rows` rows, sorted (src/sampling/sampler.js:20-42), after the
// penalties of :98-112 for the n_pen distinct tokens pen_tok with counts pen_cnt; only the k pairs are copied out.
extern "C" int zllm_model_topk(zllm_model *m, int rows, int k, const int32_t *pen_tok, const int32_t *pen_cnt, int n_pen,
                               double repeat_penalty, double frequency, double presence, int32_t *ids_host,
                               float *vals_host) {
  if (!m || !ids_host || !vals_host || k <= 0 || k > kTopkMax || n_pen < 0 || n_pen > kTopkMaxPen ||
      (n_pen && (!pen_tok || !pen_cnt)))
    return ZLLM_E_ARG;
  if (m->closed) { zllm_set_error(m->ctx, "model is closed"); return ZLLM_E_STATE; }
  if (m->failed) return ZLLM_E_STATE;
  if (!m->ready) { int rc = zllm_model_ready(m); if (rc) return rc; }
  if (rows <= 0 || rows > m->lb || k > m->c.vocab ||
      ((int64_t)m->c.vocab + kTopkChunks - 1) / kTopkChunks * (int64_t)(sizeof(float) + sizeof(int)) > kTopkSmem)
    return ZLLM_E_ARG;
  for (int j = 0; j < n_pen; j++)
    if (pen_tok[j] < 0 || pen_tok[j] >= m->c.vocab) {
      zllm_set_error(m->ctx, "token id %d out of range", pen_tok[j]);
      return ZLLM_E_TOKEN;
    }
  cudaStream_t s = m->stream;
  if (n_pen) {
    CK(cudaMemcpyAsync(m->pen, pen_tok, sizeof(int32_t) * n_pen, cudaMemcpyHostToDevice, s), "penalties");
    CK(cudaMemcpyAsync(m->pen + kTopkMaxPen, pen_cnt, sizeof(int32_t) * n_pen, cudaMemcpyHostToDevice, s), "penalties");
  }
  CK(launch_topk(m->logits, m->c.vocab, m->c.vocab, rows, k, m->pen, m->pen + kTopkMaxPen, n_pen, repeat_penalty, frequency,
                 presence, m->topk_pv, m->topk_pi, m->topk_v, m->topk_i, s), "top-k");
  CK(cudaMemcpyAsync(ids_host, m->topk_i, sizeof(int32_t) * rows * k, cudaMemcpyDeviceToHost, s), "top-k");
  CK(cudaMemcpyAsync(vals_host, m->topk_v, sizeof(float) * rows * k, cudaMemcpyDeviceToHost, s), "top-k");
  CK(cudaStreamSynchronize(s), "top-k");
  return ZLLM_OK;
}

extern "C" int zllm_model_restore_prefix(zllm_model *m, int seq, int n) {
  if (!m || seq < 0 || seq >= m->c.n_seq || n < 0 || n > m->c.ctx) return ZLLM_E_ARG;
  m->pos[seq] = n;                                  // src/compute/pool.js:244-247: the model now holds n positions
  return ZLLM_OK;
}

extern "C" int zllm_model_slot_save(zllm_model *m, int seq, int n) {
  if (!m || seq < 0 || seq >= m->c.n_seq || n < 0 || n > m->pos[seq]) return ZLLM_E_ARG;
  if (!m->ready) { int rc = zllm_model_ready(m); if (rc) return rc; }
  if (n > m->slot_cap) {
    if (m->slot) cudaFree(m->slot);
    m->slot = nullptr;
    m->slot_cap = 0;
    CK(cudaMalloc(&m->slot, (size_t)m->c.n_layer * 2 * m->kvdim() * n * m->el()), "cudaMalloc(prefix slot)");
    m->slot_cap = n;
  }
  // every layer's K and V blocks in one launch: [layer][k|v][n_kv][n][hd] out of the cache
  const int64_t el = (int64_t)m->el(), hd = m->c.head_dim, KV = m->kvdim();
  CK(launch_kv_block_copy(m->slot, (int64_t)m->slot_cap * hd * el, KV * m->slot_cap * el, m->kv_block(seq, 0, 0),
                          (int64_t)m->c.ctx * hd * el, KV * m->c.ctx * el, (int64_t)n * hd * el, m->c.n_head_kv,
                          m->c.n_layer * 2, m->ctx->num_sms, m->stream), "slot save");
  CK(cudaStreamSynchronize(m->stream), "slot save");
  m->slot_n = n;
  return ZLLM_OK;
}

extern "C" int zllm_model_slot_restore(zllm_model *m, int seq) {
  if (!m || seq < 0 || seq >= m->c.n_seq) return ZLLM_E_ARG;
  if (!m->slot || m->slot_n == 0) { zllm_set_error(m->ctx, "no prefix slot saved"); return ZLLM_E_STATE; }
  const int64_t el = (int64_t)m->el(), hd = m->c.head_dim, KV = m->kvdim();
  CK(launch_kv_block_copy(m->kv_block(seq, 0, 0), (int64_t)m->c.ctx * hd * el, KV * m->c.ctx * el, m->slot,
                          (int64_t)m->slot_cap * hd * el, KV * m->slot_cap * el, (int64_t)m->slot_n * hd * el,
                          m->c.n_head_kv, m->c.n_layer * 2, m->ctx->num_sms, m->stream), "slot restore");
  CK(cudaStreamSynchronize(m->stream), "slot restore");
  m->pos[seq] = m->slot_n;
  return ZLLM_OK;
}

extern "C" void zllm_model_destroy(zllm_model *m) {
  if (!m) return;
  m->closed = true;
  cudaSetDevice(m->ctx->device);
  if (m->stream) cudaStreamSynchronize(m->stream);
  for (auto &gr : m->graphs)
    if (gr.exec) cudaGraphExecDestroy(gr.exec);
  for (auto &L : m->L) {
    for (auto *w : L.w) zllm_weight_free(w);
    zllm_weight_free(L.qkv);
    zllm_weight_free(L.gu);
    for (float *p : {L.attn_norm, L.ffn_norm, L.q_norm, L.k_norm, L.bq, L.bk, L.bv}) cudaFree(p);
  }
  zllm_weight_free(m->tok);
  zllm_weight_free(m->out);
  for (void *p : {(void *)m->out_norm, (void *)m->rope_cos, (void *)m->rope_sin, m->kv, m->slot, (void *)m->x, (void *)m->xb,
                  (void *)m->q, (void *)m->k, (void *)m->v, (void *)m->qr, (void *)m->att, (void *)m->g, (void *)m->u,
                  (void *)m->hb, (void *)m->qkv, (void *)m->gu, (void *)m->logits, (void *)m->part, (void *)m->xq, (void *)m->xd, (void *)m->xs,
                  (void *)m->d_tok, (void *)m->d_pos, (void *)m->d_seq, (void *)m->d_npos, (void *)m->d_arg,
                  (void *)m->counters, (void *)m->d_gen, (void *)m->d_step, m->gemm_b, m->head_tiles, m->head_b,
                  (void *)m->lsend, (void *)m->lrecv, (void *)m->arg_v, (void *)m->arg_i,
                  (void *)m->topk_pv, (void *)m->topk_pi, (void *)m->topk_v, (void *)m->topk_i, (void *)m->pen})
    if (p) cudaFree(p);
  if (m->h_io) cudaFreeHost(m->h_io);
  if (m->tp_ar) tp_ar_destroy(m->tp_ar, m->tp_comm, m->stream);   // after the graphs that use it
  if (m->tp_comm) tp_comm_destroy(m->tp_comm);          // after the graphs that hold its collectives
  if (m->stream) cudaStreamDestroy(m->stream);
  delete m;
}
