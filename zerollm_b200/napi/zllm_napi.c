/* zllm_napi.c -- the Node-API add-on that lets the reference's JavaScript host drive
 * libzllm_cuda.so: `--kernels cuda` loads it from src/compute/cuda.js (zerollm_b200/napi/cuda.js),
 * whose CudaModel stands in for PoolModel (src/compute/pool.js:24-317) wherever
 * src/cli/common.js:110-113 creates a model.
 *
 * Every call that runs a pass (forward, decode, generate) is an napi_async_work: the pass runs on a
 * libuv worker thread and the call returns a Promise, so the event loop stays free the way the
 * pool's Atomics.waitAsync keeps it free (pool.js:207-218).  The typed arrays a pass reads or fills
 * are held by references until it completes.  The other calls are synchronous and throw on error.
 * Errors carry the library's messages, which are the pool's ("context full (N tokens)", "token id X
 * out of range", "batch of B tokens (max M)", "model is closed"; pool.js:146-155).
 *
 * Exports (h is the handle create() returns):
 *   create({nEmbd, nLayer, nFf, nHead, nHeadKv, headDim, nRot, vocab, neox, kvF16, ctx, nSeq,
 *           maxBatch, logitsBatch, rmsEps, ropeBase, device}) -> h
 *   setMatrix(h, kind, layer, ggmlType, rows, cols, Uint8Array rawGgufBytes)
 *   setVector(h, kind, layer, Float32Array)
 *   ready(h)
 *   forward(h, seq, Int32Array tokens, want, Float32Array|null logits, Int32Array|null argmax) -> Promise
 *   decode(h, Int32Array seqs, Int32Array tokens, Float32Array|null logits, Int32Array|null argmax) -> Promise
 *   generate(h, seq, Int32Array|null seqs, Int32Array tokens, steps, Int32Array out) -> Promise
 *   kvGet(h, seq, layer, isV, n) -> Float32Array [n][kvDim];  kvSet(h, seq, layer, isV, n, Float32Array)
 *   restorePrefix(h, seq, n), truncate(h, seq, n), reset(h, seq), pos(h, seq) -> n
 *   slotSave(h, seq, n), slotRestore(h, seq), close(h) (idempotent)
 */
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "napi_decl.h"
#include "zllm.h"

typedef struct {
  zllm_ctx *ctx;
  zllm_model *m;
  int kv_dim;
} Handle;

/* ------------------------------------------------------------------------------- helpers */
static napi_value undef(napi_env env) {
  napi_value v;
  napi_get_undefined(env, &v);
  return v;
}

static napi_value throw_msg(napi_env env, const char *msg) {
  napi_throw_error(env, NULL, msg);
  return NULL;
}

static napi_value throw_rc(napi_env env, Handle *h, int rc) {
  char buf[600];
  snprintf(buf, sizeof buf, "%s", h && h->ctx ? zllm_last_error(h->ctx) : "zllm: no context");
  if (!buf[0]) snprintf(buf, sizeof buf, "zllm error %d", rc);
  return throw_msg(env, buf);
}

static Handle *handle_of(napi_env env, napi_value v) {
  void *p = NULL;
  if (napi_get_value_external(env, v, &p) != napi_ok || !p) return NULL;
  Handle *h = (Handle *)p;
  return h;
}

static int get_i32(napi_env env, napi_value v, int32_t *out) { return napi_get_value_int32(env, v, out) == napi_ok; }

/* data pointer and element count of a typed array of the given type; null / undefined give NULL */
static int typed(napi_env env, napi_value v, napi_typedarray_type want, void **data, size_t *n) {
  napi_typedarray_type t;
  napi_value ab;
  size_t off;
  *data = NULL;
  *n = 0;
  if (napi_get_typedarray_info(env, v, &t, n, data, &ab, &off) != napi_ok) return 0;
  return t == want;
}

static int field_i32(napi_env env, napi_value obj, const char *name, int32_t dflt, int32_t *out) {
  napi_value v;
  *out = dflt;
  if (napi_get_named_property(env, obj, name, &v) != napi_ok) return 0;
  int32_t x;
  if (napi_get_value_int32(env, v, &x) == napi_ok) *out = x;
  return 1;
}

static int field_f64(napi_env env, napi_value obj, const char *name, double dflt, double *out) {
  napi_value v;
  *out = dflt;
  if (napi_get_named_property(env, obj, name, &v) != napi_ok) return 0;
  double x;
  if (napi_get_value_double(env, v, &x) == napi_ok) *out = x;
  return 1;
}

#define ARGS(N)                                                             \
  size_t argc = (N);                                                        \
  napi_value a[(N) > 0 ? (N) : 1];                                          \
  if (napi_get_cb_info(env, info, &argc, a, NULL, NULL) != napi_ok || argc < (N)) \
    return throw_msg(env, "zllm: wrong number of arguments");

#define HANDLE(v)                                                           \
  Handle *h = handle_of(env, (v));                                          \
  if (!h) return throw_msg(env, "zllm: not a model handle");                \
  if (!h->m) return throw_msg(env, "model is closed");

/* ------------------------------------------------------------------------------- lifetime */
static void handle_finalize(napi_env env, void *data, void *hint) {
  (void)env;
  (void)hint;
  Handle *h = (Handle *)data;
  if (h->m) zllm_model_destroy(h->m);
  if (h->ctx) zllm_destroy(h->ctx);
  free(h);
}

static napi_value js_create(napi_env env, napi_callback_info info) {
  ARGS(1);
  zllm_model_config c;
  memset(&c, 0, sizeof c);
  int32_t device = 0;
  field_i32(env, a[0], "nEmbd", 0, &c.n_embd);
  field_i32(env, a[0], "nLayer", 0, &c.n_layer);
  field_i32(env, a[0], "nFf", 0, &c.n_ff);
  field_i32(env, a[0], "nHead", 0, &c.n_head);
  field_i32(env, a[0], "nHeadKv", 0, &c.n_head_kv);
  field_i32(env, a[0], "headDim", 0, &c.head_dim);
  field_i32(env, a[0], "nRot", c.head_dim, &c.n_rot);
  field_i32(env, a[0], "vocab", 0, &c.vocab);
  field_i32(env, a[0], "neox", 1, &c.neox);
  field_i32(env, a[0], "kvF16", 0, &c.kv_f16);
  field_i32(env, a[0], "ctx", 2048, &c.ctx);
  field_i32(env, a[0], "nSeq", 1, &c.n_seq);
  field_i32(env, a[0], "maxBatch", 16, &c.max_batch);
  field_i32(env, a[0], "logitsBatch", 16, &c.logits_batch);
  field_i32(env, a[0], "device", 0, &device);
  field_f64(env, a[0], "rmsEps", 1e-6, &c.rms_eps);
  field_f64(env, a[0], "ropeBase", 10000.0, &c.rope_base);
  Handle *h = (Handle *)calloc(1, sizeof(Handle));
  if (!h) return throw_msg(env, "zllm: out of host memory");
  int rc = zllm_init(device, &h->ctx);
  if (rc) {
    free(h);
    return throw_msg(env, "zllm_init failed (no usable CUDA device?)");
  }
  rc = zllm_model_create(h->ctx, &c, &h->m);
  if (rc) {
    napi_value err = throw_rc(env, h, rc);
    zllm_destroy(h->ctx);
    free(h);
    return err;
  }
  h->kv_dim = c.n_head_kv * c.head_dim;
  napi_value ext;
  if (napi_create_external(env, h, handle_finalize, NULL, &ext) != napi_ok) {
    handle_finalize(env, h, NULL);
    return throw_msg(env, "zllm: napi_create_external failed");
  }
  return ext;
}

static napi_value js_close(napi_env env, napi_callback_info info) {
  ARGS(1);
  Handle *h = handle_of(env, a[0]);
  if (h && h->m) {
    zllm_model_destroy(h->m);
    h->m = NULL;
  }
  return undef(env);
}

/* ------------------------------------------------------------------------------- weights */
static napi_value js_set_matrix(napi_env env, napi_callback_info info) {
  ARGS(7);
  HANDLE(a[0]);
  int32_t kind, layer, type;
  int64_t rows, cols;
  if (!get_i32(env, a[1], &kind) || !get_i32(env, a[2], &layer) || !get_i32(env, a[3], &type) ||
      napi_get_value_int64(env, a[4], &rows) != napi_ok || napi_get_value_int64(env, a[5], &cols) != napi_ok)
    return throw_msg(env, "setMatrix: bad argument");
  void *data;
  size_t n;
  if (!typed(env, a[6], napi_uint8_array, &data, &n)) return throw_msg(env, "setMatrix: bytes must be a Uint8Array");
  int rc = zllm_model_set_matrix(h->m, kind, layer, type, rows, cols, data, n);
  return rc ? throw_rc(env, h, rc) : undef(env);
}

static napi_value js_set_vector(napi_env env, napi_callback_info info) {
  ARGS(4);
  HANDLE(a[0]);
  int32_t kind, layer;
  if (!get_i32(env, a[1], &kind) || !get_i32(env, a[2], &layer)) return throw_msg(env, "setVector: bad argument");
  void *data;
  size_t n;
  if (!typed(env, a[3], napi_float32_array, &data, &n)) return throw_msg(env, "setVector: values must be a Float32Array");
  int rc = zllm_model_set_vector(h->m, kind, layer, (const float *)data, (int64_t)n);
  return rc ? throw_rc(env, h, rc) : undef(env);
}

static napi_value js_ready(napi_env env, napi_callback_info info) {
  ARGS(1);
  HANDLE(a[0]);
  int rc = zllm_model_ready(h->m);
  return rc ? throw_rc(env, h, rc) : undef(env);
}

/* ------------------------------------------------------------------------------- passes (async) */
enum { PASS_FORWARD, PASS_DECODE, PASS_GENERATE };

typedef struct {
  int kind;
  Handle *h;
  int seq, n, want, steps, rc;
  int32_t *seqs, *tokens, *out_i;
  float *logits;
  char err[512];
  napi_ref refs[5];
  int nrefs;
  napi_deferred deferred;
  napi_async_work work;
} Pass;

static void pass_exec(napi_env env, void *p_) {
  (void)env;
  Pass *p = (Pass *)p_;
  switch (p->kind) {
    case PASS_FORWARD:
      p->rc = zllm_model_forward(p->h->m, p->seq, p->tokens, p->n, p->want, p->logits, p->out_i);
      break;
    case PASS_DECODE:
      p->rc = zllm_model_decode(p->h->m, p->seqs, p->tokens, p->n, p->logits, p->out_i);
      break;
    default:
      p->rc = zllm_model_generate(p->h->m, p->seq, p->seqs, p->tokens, p->n, p->steps, p->out_i);
      break;
  }
  if (p->rc) snprintf(p->err, sizeof p->err, "%s", zllm_last_error(p->h->ctx));
}

static void pass_done(napi_env env, napi_status st, void *p_) {
  Pass *p = (Pass *)p_;
  napi_value v;
  if (p->rc || st != napi_ok) {
    napi_value msg;
    napi_create_string_utf8(env, p->rc ? p->err : "zllm: pass cancelled", NAPI_AUTO_LENGTH, &msg);
    napi_create_error(env, NULL, msg, &v);
    napi_reject_deferred(env, p->deferred, v);
  } else {
    napi_get_undefined(env, &v);
    napi_resolve_deferred(env, p->deferred, v);
  }
  for (int i = 0; i < p->nrefs; i++) napi_delete_reference(env, p->refs[i]);
  napi_delete_async_work(env, p->work);
  free(p);
}

/* keeps a typed array alive while the pass runs on the worker thread */
static void hold(napi_env env, Pass *p, napi_value v) {
  if (p->nrefs < 5 && napi_create_reference(env, v, 1, &p->refs[p->nrefs]) == napi_ok) p->nrefs++;
}

static napi_value queue_pass(napi_env env, Pass *p, const char *name) {
  napi_value promise, nm;
  if (napi_create_promise(env, &p->deferred, &promise) != napi_ok) {
    for (int i = 0; i < p->nrefs; i++) napi_delete_reference(env, p->refs[i]);
    free(p);
    return throw_msg(env, "zllm: napi_create_promise failed");
  }
  napi_create_string_utf8(env, name, NAPI_AUTO_LENGTH, &nm);
  napi_create_async_work(env, NULL, nm, pass_exec, pass_done, p, &p->work);
  napi_queue_async_work(env, p->work);
  return promise;
}

/* an optional typed array argument (null / undefined -> NULL) */
static int opt_typed(napi_env env, napi_value v, napi_typedarray_type t, void **data, size_t *n) {
  if (typed(env, v, t, data, n)) return 1;
  *data = NULL;
  *n = 0;
  napi_typedarray_type tt;
  napi_value ab;
  size_t off;
  void *d;
  size_t nn;
  return napi_get_typedarray_info(env, v, &tt, &nn, &d, &ab, &off) != napi_ok;   /* not a typed array: absent */
}

static napi_value js_forward(napi_env env, napi_callback_info info) {
  ARGS(6);
  HANDLE(a[0]);
  Pass *p = (Pass *)calloc(1, sizeof(Pass));
  if (!p) return throw_msg(env, "zllm: out of host memory");
  p->kind = PASS_FORWARD;
  p->h = h;
  void *tok, *lg, *am;
  size_t n, nl, na;
  if (!get_i32(env, a[1], &p->seq) || !typed(env, a[2], napi_int32_array, &tok, &n) || !get_i32(env, a[3], &p->want) ||
      !opt_typed(env, a[4], napi_float32_array, &lg, &nl) || !opt_typed(env, a[5], napi_int32_array, &am, &na)) {
    free(p);
    return throw_msg(env, "forward: bad argument");
  }
  p->tokens = (int32_t *)tok;
  p->n = (int)n;
  p->logits = (float *)lg;
  p->out_i = (int32_t *)am;
  hold(env, p, a[2]);
  if (lg) hold(env, p, a[4]);
  if (am) hold(env, p, a[5]);
  return queue_pass(env, p, "zllm_forward");
}

static napi_value js_decode(napi_env env, napi_callback_info info) {
  ARGS(5);
  HANDLE(a[0]);
  Pass *p = (Pass *)calloc(1, sizeof(Pass));
  if (!p) return throw_msg(env, "zllm: out of host memory");
  p->kind = PASS_DECODE;
  p->h = h;
  void *sq, *tok, *lg, *am;
  size_t ns, n, nl, na;
  if (!typed(env, a[1], napi_int32_array, &sq, &ns) || !typed(env, a[2], napi_int32_array, &tok, &n) || ns != n ||
      !opt_typed(env, a[3], napi_float32_array, &lg, &nl) || !opt_typed(env, a[4], napi_int32_array, &am, &na)) {
    free(p);
    return throw_msg(env, "decode: bad argument");
  }
  p->seqs = (int32_t *)sq;
  p->tokens = (int32_t *)tok;
  p->n = (int)n;
  p->logits = (float *)lg;
  p->out_i = (int32_t *)am;
  hold(env, p, a[1]);
  hold(env, p, a[2]);
  if (lg) hold(env, p, a[3]);
  if (am) hold(env, p, a[4]);
  return queue_pass(env, p, "zllm_decode");
}

static napi_value js_generate(napi_env env, napi_callback_info info) {
  ARGS(6);
  HANDLE(a[0]);
  Pass *p = (Pass *)calloc(1, sizeof(Pass));
  if (!p) return throw_msg(env, "zllm: out of host memory");
  p->kind = PASS_GENERATE;
  p->h = h;
  void *sq, *tok, *out;
  size_t ns, n, no;
  if (!get_i32(env, a[1], &p->seq) || !opt_typed(env, a[2], napi_int32_array, &sq, &ns) ||
      !typed(env, a[3], napi_int32_array, &tok, &n) || !get_i32(env, a[4], &p->steps) ||
      !typed(env, a[5], napi_int32_array, &out, &no) || (sq && ns != n) || p->steps < 1 ||
      no < (size_t)p->steps * n) {
    free(p);
    return throw_msg(env, "generate: bad argument");
  }
  p->seqs = (int32_t *)sq;
  p->tokens = (int32_t *)tok;
  p->n = (int)n;
  p->out_i = (int32_t *)out;
  if (sq) hold(env, p, a[2]);
  hold(env, p, a[3]);
  hold(env, p, a[5]);
  return queue_pass(env, p, "zllm_generate");
}

/* ------------------------------------------------------------------------------- KV and positions */
static napi_value js_kv_get(napi_env env, napi_callback_info info) {
  ARGS(5);
  HANDLE(a[0]);
  int32_t seq, layer, isv, n;
  if (!get_i32(env, a[1], &seq) || !get_i32(env, a[2], &layer) || !get_i32(env, a[3], &isv) || !get_i32(env, a[4], &n) ||
      n < 0)
    return throw_msg(env, "kvGet: bad argument");
  const size_t count = (size_t)n * (size_t)h->kv_dim;
  void *data = NULL;
  napi_value ab, arr;
  if (napi_create_arraybuffer(env, count * sizeof(float), &data, &ab) != napi_ok)
    return throw_msg(env, "kvGet: cannot allocate the result");
  if (count) {
    int rc = zllm_model_kv_get(h->m, seq, layer, isv, n, (float *)data);
    if (rc) return throw_rc(env, h, rc);
  }
  napi_create_typedarray(env, napi_float32_array, count, ab, 0, &arr);
  return arr;
}

static napi_value js_kv_set(napi_env env, napi_callback_info info) {
  ARGS(6);
  HANDLE(a[0]);
  int32_t seq, layer, isv, n;
  void *data;
  size_t cnt;
  if (!get_i32(env, a[1], &seq) || !get_i32(env, a[2], &layer) || !get_i32(env, a[3], &isv) || !get_i32(env, a[4], &n) ||
      n < 0 || !typed(env, a[5], napi_float32_array, &data, &cnt) || cnt < (size_t)n * (size_t)h->kv_dim)
    return throw_msg(env, "kvSet: bad argument");
  int rc = zllm_model_kv_set(h->m, seq, layer, isv, n, (const float *)data);
  return rc ? throw_rc(env, h, rc) : undef(env);
}

/* (h, seq, n) -> fn(m, seq, n) */
static napi_value seq_n_call(napi_env env, napi_callback_info info, int (*fn)(zllm_model *, int, int)) {
  ARGS(3);
  HANDLE(a[0]);
  int32_t seq, n;
  if (!get_i32(env, a[1], &seq) || !get_i32(env, a[2], &n)) return throw_msg(env, "zllm: bad argument");
  int rc = fn(h->m, seq, n);
  return rc ? throw_rc(env, h, rc) : undef(env);
}

static napi_value js_restore_prefix(napi_env env, napi_callback_info info) { return seq_n_call(env, info, zllm_model_restore_prefix); }
static napi_value js_truncate(napi_env env, napi_callback_info info) { return seq_n_call(env, info, zllm_model_truncate); }
static napi_value js_slot_save(napi_env env, napi_callback_info info) { return seq_n_call(env, info, zllm_model_slot_save); }

static napi_value js_reset(napi_env env, napi_callback_info info) {
  ARGS(2);
  HANDLE(a[0]);
  int32_t seq;
  if (!get_i32(env, a[1], &seq)) return throw_msg(env, "reset: bad argument");
  int rc = zllm_model_reset(h->m, seq);
  return rc ? throw_rc(env, h, rc) : undef(env);
}

static napi_value js_slot_restore(napi_env env, napi_callback_info info) {
  ARGS(2);
  HANDLE(a[0]);
  int32_t seq;
  if (!get_i32(env, a[1], &seq)) return throw_msg(env, "slotRestore: bad argument");
  int rc = zllm_model_slot_restore(h->m, seq);
  return rc ? throw_rc(env, h, rc) : undef(env);
}

static napi_value js_pos(napi_env env, napi_callback_info info) {
  ARGS(2);
  HANDLE(a[0]);
  int32_t seq;
  if (!get_i32(env, a[1], &seq)) return throw_msg(env, "pos: bad argument");
  napi_value v;
  napi_create_int32(env, zllm_model_pos(h->m, seq), &v);
  return v;
}

/* ------------------------------------------------------------------------------- registration */
__attribute__((visibility("default"))) napi_value napi_register_module_v1(napi_env env, napi_value exports) {
  static const struct { const char *name; napi_callback fn; } fns[] = {
      {"create", js_create},         {"close", js_close},
      {"setMatrix", js_set_matrix},  {"setVector", js_set_vector},
      {"ready", js_ready},           {"forward", js_forward},
      {"decode", js_decode},         {"generate", js_generate},
      {"kvGet", js_kv_get},          {"kvSet", js_kv_set},
      {"restorePrefix", js_restore_prefix}, {"truncate", js_truncate},
      {"reset", js_reset},           {"pos", js_pos},
      {"slotSave", js_slot_save},    {"slotRestore", js_slot_restore},
  };
  for (size_t i = 0; i < sizeof fns / sizeof fns[0]; i++) {
    napi_value f;
    if (napi_create_function(env, fns[i].name, NAPI_AUTO_LENGTH, fns[i].fn, NULL, &f) != napi_ok ||
        napi_set_named_property(env, exports, fns[i].name, f) != napi_ok)
      return NULL;
  }
  return exports;
}

/* The Node-API version the add-on needs (Node >= 22 provides 9 and later). */
__attribute__((visibility("default"))) int32_t node_api_module_get_api_version_v1(void) { return 8; }
