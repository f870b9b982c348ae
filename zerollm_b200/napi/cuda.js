// src/compute/cuda.js -- CudaModel: the B200 backend behind `--kernels cuda`.
//
// A drop-in for PoolModel (src/compute/pool.js:24-317) wherever the engine takes a model:
// createModel (src/cli/common.js:110-113), generate (src/model/generate.js:55-96), PrefixCache
// (src/model/prefix-cache.js:50-134) and generateSpeculative (src/model/speculative.js:100).  It
// drives libzllm_cuda.so through the zllm_napi.node add-on (zllm_napi.c beside this file); every pass
// is asynchronous on the add-on's side, so the event loop stays free as with the worker pool.
//
// In the reference checkout this file goes to src/compute/cuda.js, the add-on to build/zllm_napi.node
// (with libzllm_cuda.so beside it), and createModel gains
//   if (opts.kernels === 'cuda') return (await import('../compute/cuda.js')).CudaModel.create(g, {...});
import { createRequire } from 'node:module';
import fs from 'node:fs';
import { modelConfig, assertSupportedTensorTypes } from '../model/config.js';
import { readTensorBytes } from '../gguf/reader.js';

const zllm = createRequire(import.meta.url)('../../build/zllm_napi.node');

// tensor kinds of zllm_model_set_matrix / zllm_model_set_vector (include/zllm.h)
const KIND = { token_embd: 0, output: 1, output_norm: 2, rope_freqs: 3, attn_norm: 10, attn_q: 11, attn_k: 12, attn_v: 13,
  attn_output: 14, attn_q_bias: 15, attn_k_bias: 16, attn_v_bias: 17, attn_q_norm: 18, attn_k_norm: 19, ffn_norm: 20,
  ffn_gate: 21, ffn_up: 22, ffn_down: 23 };

// GGUF name -> [kind, layer]: token_embd.weight, output.weight, blk.L.attn_q.weight, blk.L.attn_q.bias ...
function kindOf(name) {
  const m = /^blk\.(\d+)\.(.+)\.(weight|bias)$/.exec(name);
  if (m) {
    const k = KIND[m[3] === 'bias' ? `${m[2]}_bias` : m[2]];
    return k === undefined ? null : [k, Number(m[1])];
  }
  const t = /^(.+)\.weight$/.exec(name);
  return t && KIND[t[1]] !== undefined ? [KIND[t[1]], 0] : null;
}

export class CudaModel {
  static async create(g, opts = {}) { const m = new CudaModel(); await m.#init(g, opts); return m; }

  get pos() { return this.tokens.length; }

  async #init(g, opts) {
    this.cfg = modelConfig(g);
    assertSupportedTensorTypes(g);
    const c = this.cfg;
    this.ctx = Math.min(opts.ctx ?? 2048, c.nCtxTrain);
    this.kv = opts.kv ?? 'f32';
    this.kernels = 'cuda';
    this.maxBatch = Math.max(1, Math.min(opts.maxBatch ?? 16, 64));                 // src/compute/layout.js:23
    this.logitsBatch = Math.max(1, Math.min(opts.logitsBatch ?? 16, this.maxBatch)); // layout.js:48
    this.h = zllm.create({ nEmbd: c.nEmbd, nLayer: c.nLayer, nFf: c.nFF, nHead: c.nHead, nHeadKv: c.nHeadKv,
      headDim: c.headDim, nRot: c.nRot ?? c.headDim, vocab: c.vocabSize, neox: c.ropeType === 'neox' ? 1 : 0,
      kvF16: this.kv === 'f16' ? 1 : 0, ctx: this.ctx, nSeq: 1, maxBatch: this.maxBatch, logitsBatch: this.logitsBatch,
      rmsEps: c.rmsEps, ropeBase: c.ropeBase, device: opts.device ?? 0 });
    const fd = fs.openSync(g.path, 'r');
    try {
      for (const t of g.tensors) {
        const kl = kindOf(t.name);
        if (!kl) continue;
        const bytes = readTensorBytes(fd, t, 0, new Uint8Array(t.nBytes));  // raw GGUF bytes (src/gguf/reader.js:201-214)
        if (t.dims.length === 1) zllm.setVector(this.h, kl[0], kl[1], new Float32Array(bytes.buffer, 0, t.dims[0]));
        else zllm.setMatrix(this.h, kl[0], kl[1], t.type, t.dims[1], t.dims[0], bytes);
        opts.onProgress?.(t.name);
      }
    } finally { fs.closeSync(fd); }
    zllm.ready(this.h);
    this.logits = new Float32Array(this.logitsBatch * c.vocabSize);
    this.tokens = [];
    this.failed = null;
    this.closed = false;
  }

  forward(token, opts = {}) { return this.forwardBatch([token], opts); }

  async forwardBatch(tokens, opts = {}) {
    if (this.failed) throw this.failed;                                     // pool.js:123-127
    if (this.closed) throw new Error('model is closed');
    const lg = opts.logits ?? true;
    const want = lg === false || lg === 'none' ? 0 : lg === 'all' ? 2 : 1;
    try {
      await zllm.forward(this.h, 0, Int32Array.from(tokens), want, want ? this.logits : null, null);
    } catch (e) {
      if (!/context full|out of range|batch of|logits for all positions/.test(e.message)) this.failed = e;
      throw e;
    }
    for (const t of tokens) this.tokens.push(t);
    const V = this.cfg.vocabSize;
    return want === 2 ? this.logits.subarray(0, tokens.length * V) : want ? this.logits.subarray(0, V) : null;
  }

  async kvGet(layer, isV, n) { return zllm.kvGet(this.h, 0, layer, isV, n); }          // Float32Array [n][kvDim]
  async kvSet(layer, isV, n, data) { zllm.kvSet(this.h, 0, layer, isV, n, data); }
  restorePrefix(ids) { this.tokens = Array.from(ids); zllm.restorePrefix(this.h, 0, ids.length); }
  async truncate(n) {
    if (n < this.tokens.length) { this.tokens.length = Math.max(0, n); zllm.truncate(this.h, 0, this.tokens.length); }
    return 0;
  }
  reset() { this.tokens.length = 0; zllm.reset(this.h, 0); }
  markRollback() {}                                                          // the KV cache is positional
  async close() { if (!this.closed) { this.closed = true; zllm.close(this.h); } }
}
