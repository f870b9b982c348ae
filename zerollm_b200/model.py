"""CudaModel: the B200 backend behind the reference's model interface.

Mirrors ``PoolModel`` (src/compute/pool.js:24-317) -- the object ``generate()``,
``PrefixCache`` and ``generateSpeculative`` drive -- over the ``zllm_model_*`` entry points of
libzllm_cuda.so: ``create``, ``pos`` / ``tokens`` / ``ctx`` / ``cfg`` / ``kernels`` / ``kv`` /
``maxBatch`` / ``logitsBatch``, ``forward(token, logits=...)``, ``forwardBatch(tokens, logits=...)``
returning a float32 view valid until the next call, ``kvGet`` / ``kvSet`` (f32 [n][kvDim]),
``restorePrefix(ids)``, ``truncate(n)``, ``reset()``, ``close()`` (idempotent) and
``markRollback()`` (a no-op: the KV cache is positional).  Errors carry the pool's messages
("context full (N tokens)", "token id X out of range", "batch of B tokens (max M)", "model is
closed"); a backend failure latches and is raised again on every later call (pool.js:123-127).

Beyond the reference (one sequence per model), ``n_seq`` > 1 holds independent sequences that
``decode`` steps together, one token each -- batched serving.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import ggml
from .kernels import Context
from .lib import (E_BATCH, E_CTX_FULL, E_STATE, E_TOKEN, ModelConfig, T_ATTN_NORM, T_BK, T_BQ, T_BV, T_DOWN, T_FFN_NORM,
                  T_GATE, T_K_NORM, T_OUTPUT, T_OUTPUT_NORM, T_Q_NORM, T_ROPE_FREQS, T_TOK_EMBD, T_UP, T_WK, T_WO, T_WQ,
                  T_WV, ZllmError, load)

MAX_BATCH = 64                 # src/compute/layout.js:23
DEFAULT_LOGITS_BATCH = 16      # src/compute/layout.js:48

_MATS = (("wq", T_WQ), ("wk", T_WK), ("wv", T_WV), ("wo", T_WO), ("gate", T_GATE), ("up", T_UP), ("down", T_DOWN))
_VECS = (("attn_norm", T_ATTN_NORM), ("ffn_norm", T_FFN_NORM), ("q_norm", T_Q_NORM), ("k_norm", T_K_NORM),
         ("bq", T_BQ), ("bk", T_BK), ("bv", T_BV))


class CudaModel:
    """A model resident on one GPU.  ``cfg`` is a model config dict (zerollm_b200.synth layout, the
    fields of src/model/config.js:73-123); ``weights`` the raw GGUF tensors of the model."""

    @classmethod
    def create(cls, cfg: dict, weights: dict, ctx: int = 2048, kv: str = "f32", max_batch: int = 16,
               logits_batch: int | None = None, device: int = 0, n_seq: int = 1, context: Context | None = None,
               tp: tuple | None = None):
        return cls(cfg, weights, ctx, kv, max_batch, logits_batch, device, n_seq, context, tp)

    def __init__(self, cfg, weights, ctx=2048, kv="f32", max_batch=16, logits_batch=None, device=0, n_seq=1, context=None,
                 tp=None):
        """``tp = (rank, size, unique_id)`` joins a tensor-parallel group: ``cfg`` / ``weights`` are
        then this rank's shard (zerollm_b200.tp.shard_model) and ``unique_id`` the group's id from
        rank 0's ``tp_unique_id``."""
        if kv not in ("f32", "f16"):
            raise ValueError(f'kv must be f32 or f16 (got "{kv}")')
        self.cfg = dict(cfg)
        self.ctx = min(int(ctx), int(cfg.get("n_ctx_train", ctx)))
        self.kv = kv
        self.kernels = "cuda"
        self.maxBatch = max(1, min(int(max_batch), MAX_BATCH))
        self.logitsBatch = max(1, min(DEFAULT_LOGITS_BATCH if logits_batch is None else int(logits_batch), self.maxBatch))
        self.n_seq = int(n_seq)
        self.lib = load()
        self.context = context or Context(device)
        self._own_context = context is None
        self.failed = None
        self.closed = False
        self._tokens = [[] for _ in range(self.n_seq)]
        self.vocab = int(cfg["vocab"])
        self.kv_dim = cfg["n_head_kv"] * cfg["head_dim"]
        mc = ModelConfig(n_embd=cfg["n_embd"], n_layer=cfg["n_layer"], n_ff=cfg["n_ff"], n_head=cfg["n_head"],
                         n_head_kv=cfg["n_head_kv"], head_dim=cfg["head_dim"], n_rot=cfg.get("n_rot", cfg["head_dim"]),
                         vocab=self.vocab, neox=1 if cfg.get("rope_type", "neox") == "neox" else 0,
                         kv_f16=1 if kv == "f16" else 0, ctx=self.ctx, n_seq=self.n_seq, max_batch=self.maxBatch,
                         logits_batch=self.logitsBatch, rms_eps=float(cfg["rms_eps"]), rope_base=float(cfg["rope_base"]))
        h = C.c_void_p()
        self._check(self.lib.zllm_model_create(self.context.h, C.byref(mc), C.byref(h)), "zllm_model_create")
        self.h = h
        if tp is not None:
            rank, size, uid = tp
            buf = C.create_string_buffer(bytes(uid), len(uid))
            self._check(self.lib.zllm_model_set_tp(self.h, int(rank), int(size), buf), "zllm_model_set_tp")
            if cfg.get("vocab_shard") is not None:
                v0, n = cfg["vocab_shard"]
                self._check(self.lib.zllm_model_set_vocab_shard(self.h, int(v0), int(n)), "zllm_model_set_vocab_shard")
        self._load(weights)
        self._check(self.lib.zllm_model_ready(self.h), "zllm_model_ready")
        self._logits = np.zeros((self.logitsBatch if self.n_seq == 1 else max(self.logitsBatch, self.n_seq), self.vocab),
                                np.float32)
        self._argmax = np.zeros(MAX_BATCH, np.int32)

    # ---------------------------------------------------------------------------------- set-up
    def _check(self, rc, what=""):
        if rc:
            msg = self.lib.zllm_last_error(self.context.h).decode()
            raise ZllmError(rc, msg if not what or rc in (E_CTX_FULL, E_TOKEN, E_BATCH) else f"{what}: {msg}")

    def _mat(self, kind, layer, t):
        buf = np.ascontiguousarray(t["data"], np.uint8)
        self._check(self.lib.zllm_model_set_matrix(self.h, kind, layer, t["type"], t["rows"], t["cols"],
                                                   buf.ctypes.data_as(C.c_void_p), buf.nbytes), "zllm_model_set_matrix")

    def _vec(self, kind, layer, v):
        a = np.ascontiguousarray(v, np.float32)
        self._check(self.lib.zllm_model_set_vector(self.h, kind, layer, a.ctypes.data_as(C.c_void_p), a.size),
                    "zllm_model_set_vector")

    def _load(self, w):
        self._mat(T_TOK_EMBD, 0, w["tok_embd"])
        if w.get("output") is not None:
            self._mat(T_OUTPUT, 0, w["output"])
        self._vec(T_OUTPUT_NORM, 0, w["output_norm"])
        if w.get("rope_freqs") is not None:
            self._vec(T_ROPE_FREQS, 0, w["rope_freqs"])
        for l, L in enumerate(w["layers"]):
            for name, kind in _MATS:
                self._mat(kind, l, L[name])
            for name, kind in _VECS:
                if L.get(name) is not None:
                    self._vec(kind, l, L[name])

    # ---------------------------------------------------------------------------------- interface
    @property
    def pos(self) -> int:
        return len(self._tokens[0])

    @property
    def tokens(self) -> list:
        return self._tokens[0]

    def _guard(self):
        if self.failed:
            raise self.failed
        if self.closed:
            raise ZllmError(E_STATE, "model is closed")

    def _run(self, rc, what):
        if rc:
            err = ZllmError(rc, self.lib.zllm_last_error(self.context.h).decode())
            if rc not in (E_CTX_FULL, E_TOKEN, E_BATCH, -1):
                self.failed = err
            raise err

    def forward(self, token: int, logits=True):
        return self.forwardBatch([token], logits=logits)

    def forwardBatch(self, tokens, logits=True, seq: int = 0):
        """B tokens at the next positions in one pass; logits True/'last' -> [vocab] of the last token,
        'all' -> [B][vocab], False/'none' -> None (pool.js:145-160).  'device' / 'device-all' compute
        the same logits but leave them on the GPU (for zerollm_b200.sampler) and return None."""
        self._guard()
        toks = np.ascontiguousarray(np.asarray(tokens, dtype=np.int64).astype(np.int32))
        B = toks.size
        want = 0 if logits is False or logits == "none" else 2 if logits in ("all", "device-all") else 1
        host = want and logits not in ("device", "device-all")
        rc = self.lib.zllm_model_forward(self.h, seq, toks.ctypes.data_as(C.c_void_p), B, want,
                                         self._logits.ctypes.data_as(C.c_void_p) if host else None,
                                         self._argmax.ctypes.data_as(C.c_void_p) if host else None)
        self._run(rc, "forward")
        self._tokens[seq].extend(int(t) for t in toks)
        if not host:
            return None
        if want == 2:
            return self._logits[:B]
        return self._logits[0] if want else None

    def decode(self, seqs, tokens):
        """One token for each of several distinct sequences; returns ([n][vocab] logits, [n] argmax)."""
        self._guard()
        s = np.ascontiguousarray(seqs, np.int32)
        t = np.ascontiguousarray(tokens, np.int32)
        rc = self.lib.zllm_model_decode(self.h, s.ctypes.data_as(C.c_void_p), t.ctypes.data_as(C.c_void_p), t.size,
                                        self._logits.ctypes.data_as(C.c_void_p), self._argmax.ctypes.data_as(C.c_void_p))
        self._run(rc, "decode")
        for sq, tk in zip(s, t):
            self._tokens[int(sq)].append(int(tk))
        return self._logits[:t.size], self._argmax[:t.size]

    def generate(self, tokens, steps: int, seqs=None) -> np.ndarray:
        """Greedy decoding on the device: ``steps`` passes starting from ``tokens`` (one per sequence
        of ``seqs``, or one token of sequence 0), each pass fed the previous pass's argmax.  Returns
        the argmax tokens [steps][n]."""
        self._guard()
        t = np.ascontiguousarray(np.atleast_1d(tokens), np.int32)
        n = t.size
        out = np.zeros((steps, n), np.int32)
        s = None if seqs is None else np.ascontiguousarray(seqs, np.int32)
        rc = self.lib.zllm_model_generate(self.h, 0, None if s is None else s.ctypes.data_as(C.c_void_p),
                                          t.ctypes.data_as(C.c_void_p), n, int(steps), out.ctypes.data_as(C.c_void_p))
        self._run(rc, "generate")
        for i in range(n):
            sq = 0 if s is None else int(s[i])
            self._tokens[sq].append(int(t[i]))
            self._tokens[sq].extend(int(v) for v in out[:-1, i])
        return out

    def tp_collective(self) -> int:
        """0 one GPU, 1 NCCL all-reduce, 2 the one-shot all-reduce over NVLink peer memory."""
        return int(self.lib.zllm_model_tp_collective(self.h))

    def kvGet(self, layer: int, isV: int, n: int, seq: int = 0) -> np.ndarray:
        self._guard()
        out = np.empty(n * self.kv_dim, np.float32)
        self._run(self.lib.zllm_model_kv_get(self.h, seq, layer, isV, n, out.ctypes.data_as(C.c_void_p)), "kvGet")
        return out

    def kvSet(self, layer: int, isV: int, n: int, data, seq: int = 0):
        self._guard()
        a = np.ascontiguousarray(np.asarray(data, np.float32)[: n * self.kv_dim])
        self._run(self.lib.zllm_model_kv_set(self.h, seq, layer, isV, n, a.ctypes.data_as(C.c_void_p)), "kvSet")

    def restorePrefix(self, ids, seq: int = 0):
        self._tokens[seq] = [int(i) for i in ids]
        self._run(self.lib.zllm_model_restore_prefix(self.h, seq, len(ids)), "restorePrefix")

    def saveSlot(self, n: int, seq: int = 0):
        """Keep the first n positions of a sequence in the device-resident prefix slot."""
        self._guard()
        self._run(self.lib.zllm_model_slot_save(self.h, seq, n), "slot save")
        self._slot_ids = list(self._tokens[seq][:n])

    def restoreSlot(self, seq: int = 0):
        """Byte-copy the prefix slot into a sequence, which then holds exactly those positions."""
        self._guard()
        self._run(self.lib.zllm_model_slot_restore(self.h, seq), "slot restore")
        self._tokens[seq] = list(getattr(self, "_slot_ids", []))

    def truncate(self, n: int, seq: int = 0) -> int:
        if n >= len(self._tokens[seq]):
            return 0
        n = max(0, n)
        self._tokens[seq] = self._tokens[seq][:n]
        self.lib.zllm_model_truncate(self.h, seq, n)
        return 0

    def reset(self, seq: int = 0):
        self._tokens[seq] = []
        self.lib.zllm_model_reset(self.h, seq)

    def markRollback(self):
        pass

    def close(self):
        if self.closed:
            return
        self.closed = True
        if getattr(self, "h", None):
            self.lib.zllm_model_destroy(self.h)
            self.h = None
        if self._own_context:
            self.context.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def tp_unique_id(context: Context) -> bytes:
    """A new tensor-parallel group id (rank 0 creates it; every rank passes it to CudaModel(tp=...))."""
    lib = load()
    buf = C.create_string_buffer(128)
    rc = lib.zllm_tp_unique_id(context.h, buf, 128)
    if rc:
        raise ZllmError(rc, lib.zllm_last_error(context.h).decode())
    return buf.raw
