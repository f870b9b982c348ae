"""ctypes bindings for liboracle.so (TEST INFRASTRUCTURE ONLY; see oracle/__init__.py)."""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
BUILD = os.path.join(HERE, "_build")

F32, F16, Q4_0, Q5_0, Q8_0, Q4_K, Q5_K, Q6_K, BF16 = 0, 1, 2, 6, 8, 12, 13, 14, 30

_lib = None


def build(native: bool = False) -> str:
    """Compile the oracle with make; returns the library path."""
    target = "native" if native else "all"
    subprocess.run(["make", "-s", "-C", HERE, target], check=True)
    return os.path.join(BUILD, "liboracle_native.so" if native else "liboracle.so")


def _p(a):
    return a.ctypes.data_as(C.c_void_p) if a is not None else None


def _setup(lib):
    vp, i64, i32, dbl = C.c_void_p, C.c_int64, C.c_int, C.c_double
    lib.zo_f32_to_f16.restype = C.c_uint16
    lib.zo_f32_to_f16.argtypes = [C.c_float]
    lib.zo_f16_to_f32.restype = C.c_float
    lib.zo_f16_to_f32.argtypes = [C.c_uint16]
    lib.zo_row_bytes.restype = i64
    lib.zo_row_bytes.argtypes = [i32, i64]
    lib.zo_unpack_scale_min_k4.argtypes = [vp, vp, vp]
    lib.zo_quantize_act.argtypes = [vp, i64, vp, vp, vp]
    lib.zo_dequant_row.restype = i32
    lib.zo_dequant_row.argtypes = [i32, vp, i64, i64, vp]
    lib.zo_matvec.restype = i32
    lib.zo_matvec.argtypes = [i32, vp, i64, i64, vp, vp, i64, i64, i32]
    lib.zo_matvec_q.restype = i32
    lib.zo_matvec_q.argtypes = [i32, vp, i64, vp, vp, vp, vp, vp, i64, i64, i32]
    lib.zo_rmsnorm.argtypes = [vp, vp, vp, dbl, i32]
    lib.zo_softmax.argtypes = [vp, i32]
    lib.zo_silu.restype = dbl
    lib.zo_silu.argtypes = [dbl]
    lib.zo_rope_tables.argtypes = [i32, dbl, i32, vp, vp, vp]
    lib.zo_apply_rope.argtypes = [vp, i32, i32, i32, i32, vp, vp, i32, i32]
    lib.zo_attn_head_f32.argtypes = [vp, vp, vp, i32, i32, i32, vp, vp]
    lib.zo_attn_head_f16.argtypes = [vp, vp, vp, i32, i32, i32, vp, vp]
    lib.zo_model_new.restype = vp
    lib.zo_model_new.argtypes = [vp, vp, vp, vp, vp, vp]
    lib.zo_model_free.argtypes = [vp]
    lib.zo_model_pos.restype = i32
    lib.zo_model_pos.argtypes = [vp]
    lib.zo_model_truncate.argtypes = [vp, i32]
    lib.zo_model_restore_prefix.restype = i32
    lib.zo_model_restore_prefix.argtypes = [vp, i32]
    lib.zo_model_forward.restype = i32
    lib.zo_model_forward.argtypes = [vp, i32, vp, i32]
    lib.zo_model_kv_get.restype = i32
    lib.zo_model_kv_get.argtypes = [vp, i32, i32, i32, vp]
    lib.zo_model_kv_set.restype = i32
    lib.zo_model_kv_set.argtypes = [vp, i32, i32, i32, vp]


def lib(path: str | None = None):
    """Load (building if needed) the oracle library."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    if path is None:
        path = os.path.join(BUILD, "liboracle.so")
        if not os.path.exists(path):
            build()
    L = C.CDLL(path)
    _setup(L)
    if path.endswith("liboracle.so"):
        _lib = L
    return L


# ------------------------------------------------------------------------------------- scalars
def f32_to_f16(x: float) -> int:
    return int(lib().zo_f32_to_f16(float(x)))


def f16_to_f32(h: int) -> float:
    return float(lib().zo_f16_to_f32(int(h)))


def row_bytes(t: int, cols: int) -> int:
    return int(lib().zo_row_bytes(t, cols))


def unpack_scale_min_k4(q12: bytes):
    q = np.frombuffer(bytes(q12), dtype=np.uint8).copy()
    sc = np.zeros(8, np.int32)
    mn = np.zeros(8, np.int32)
    lib().zo_unpack_scale_min_k4(_p(q), _p(sc), _p(mn))
    return sc.tolist(), mn.tolist()


# ------------------------------------------------------------------------------------- vectors
def quantize_act(x: np.ndarray):
    x = np.ascontiguousarray(x, dtype=np.float32)
    n = x.size
    q = np.zeros(n, np.int8)
    d = np.zeros(n // 32, np.float32)
    s = np.zeros(n // 32, np.int32)
    lib().zo_quantize_act(_p(x), n, _p(q), _p(d), _p(s))
    return q, d, s


def dequant(t: int, w: np.ndarray, rows: int, cols: int) -> np.ndarray:
    w = np.ascontiguousarray(w, dtype=np.uint8)
    out = np.zeros((rows, cols), np.float32)
    for r in range(rows):
        rc = lib().zo_dequant_row(t, _p(w), cols, r, _p(out[r]))
        if rc:
            raise ValueError(f"oracle: unsupported type {t}")
    return out


def matvec(t: int, w: np.ndarray, rows: int, cols: int, x: np.ndarray, nthreads: int = 1,
           r0: int = 0, r1: int | None = None, library=None) -> np.ndarray:
    """y = W x as ref-kernels.js:127-302 (x quantized per 32 for quantized types)."""
    w = np.ascontiguousarray(w, dtype=np.uint8)
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.zeros(rows, np.float32)
    r1 = rows if r1 is None else r1
    rc = (library or lib()).zo_matvec(t, _p(w), rows, cols, _p(x), _p(y), r0, r1, nthreads)
    if rc:
        raise ValueError(f"oracle: unsupported type {t} / cols {cols}")
    return y


def matvec_q(t: int, w: np.ndarray, rows: int, cols: int, xq, xd, xs, x=None, nthreads: int = 1):
    w = np.ascontiguousarray(w, dtype=np.uint8)
    y = np.zeros(rows, np.float32)
    xq = np.ascontiguousarray(xq, np.int8)
    xd = np.ascontiguousarray(xd, np.float32)
    xs = np.ascontiguousarray(xs, np.int32)
    x = None if x is None else np.ascontiguousarray(x, np.float32)
    rc = lib().zo_matvec_q(t, _p(w), cols, _p(x), _p(xq), _p(xd), _p(xs), _p(y), 0, rows, nthreads)
    if rc:
        raise ValueError("oracle: bad matvec_q call")
    return y


def rmsnorm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    out = np.zeros_like(x)
    lib().zo_rmsnorm(_p(out), _p(x), _p(w), float(eps), x.size)
    return out


def softmax(x: np.ndarray) -> np.ndarray:
    x = np.array(x, np.float32, copy=True)
    lib().zo_softmax(_p(x), x.size)
    return x


def silu(z: float) -> float:
    return float(lib().zo_silu(float(z)))


def rope_tables(n_rot: int, base: float, ctx: int, freq_factors=None):
    half = n_rot // 2
    c = np.zeros(ctx * half, np.float32)
    s = np.zeros(ctx * half, np.float32)
    ff = None if freq_factors is None else np.ascontiguousarray(freq_factors, np.float32)
    lib().zo_rope_tables(n_rot, float(base), ctx, _p(ff), _p(c), _p(s))
    return c, s


def apply_rope(v: np.ndarray, n_heads: int, head_dim: int, n_rot: int, neox: bool, cos_t, sin_t, pos: int):
    v = np.array(v, np.float32, copy=True)
    lib().zo_apply_rope(_p(v), n_heads, head_dim, n_rot, 1 if neox else 0, _p(cos_t), _p(sin_t), pos, 0)
    return v


def attn_head(q: np.ndarray, k: np.ndarray, v: np.ndarray, f16: bool) -> np.ndarray:
    """One query head over npos cached positions ([npos][hd] K and V; u16 bits when f16)."""
    q = np.ascontiguousarray(q, np.float32)
    hd = q.size
    npos = k.shape[0]
    out = np.zeros(hd, np.float32)
    sc = np.zeros(max(npos, 1), np.float32)
    if f16:
        k = np.ascontiguousarray(k, np.uint16)
        v = np.ascontiguousarray(v, np.uint16)
        lib().zo_attn_head_f16(_p(q), _p(k), _p(v), npos, hd, hd, _p(sc), _p(out))
    else:
        k = np.ascontiguousarray(k, np.float32)
        v = np.ascontiguousarray(v, np.float32)
        lib().zo_attn_head_f32(_p(q), _p(k), _p(v), npos, hd, hd, _p(sc), _p(out))
    return out


def f32_to_f16_array(x: np.ndarray) -> np.ndarray:
    """Vectorised f16.js:7-30 (round to nearest even) via the oracle's scalar routine."""
    L = lib()
    x = np.ascontiguousarray(x, np.float32).ravel()
    return np.fromiter((L.zo_f32_to_f16(float(v)) for v in x), dtype=np.uint16, count=x.size)


# ------------------------------------------------------------------------------------- model
class _Cfg(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("n_embd", "n_layer", "n_ff", "n_head", "n_head_kv", "head_dim",
                                      "n_rot", "vocab", "neox", "kv_f16", "ctx")] + \
               [("rms_eps", C.c_double), ("rope_base", C.c_double)]


class _W(C.Structure):
    _fields_ = [("type", C.c_int), ("rows", C.c_int64), ("cols", C.c_int64), ("data", C.c_void_p)]


class _Layer(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in ("attn_norm", "ffn_norm", "bq", "bk", "bv", "q_norm", "k_norm")] + \
               [(n, _W) for n in ("wq", "wk", "wv", "wo", "gate", "up", "down")]


class OracleModel:
    """forward.js RefModel (kv_f16=False) / 1-worker JS pool with --kv f16 (kv_f16=True).

    ``weights`` is a dict in the layout of ``zerollm_b200.synth`` models: numpy raw GGUF bytes
    per tensor plus their (type, rows, cols), f32 norm vectors.  Arrays are kept alive here.
    """

    def __init__(self, cfg: dict, weights: dict, ctx: int, kv_f16: bool, nthreads: int = 1):
        self.cfg = cfg
        self.nthreads = nthreads
        self._keep = []
        c = _Cfg(n_embd=cfg["n_embd"], n_layer=cfg["n_layer"], n_ff=cfg["n_ff"], n_head=cfg["n_head"],
                 n_head_kv=cfg["n_head_kv"], head_dim=cfg["head_dim"], n_rot=cfg.get("n_rot", cfg["head_dim"]),
                 vocab=cfg["vocab"], neox=1 if cfg.get("rope_type", "neox") == "neox" else 0,
                 kv_f16=1 if kv_f16 else 0, ctx=ctx, rms_eps=float(cfg["rms_eps"]), rope_base=float(cfg["rope_base"]))
        self._c = c

        def W(t):
            arr = np.ascontiguousarray(t["data"], np.uint8)
            self._keep.append(arr)
            return _W(type=t["type"], rows=t["rows"], cols=t["cols"], data=arr.ctypes.data)

        def V(a):
            if a is None:
                return None
            a = np.ascontiguousarray(a, np.float32)
            self._keep.append(a)
            return a.ctypes.data

        layers = (_Layer * cfg["n_layer"])()
        for l, Lw in enumerate(weights["layers"]):
            layers[l] = _Layer(attn_norm=V(Lw["attn_norm"]), ffn_norm=V(Lw["ffn_norm"]), bq=V(Lw.get("bq")),
                               bk=V(Lw.get("bk")), bv=V(Lw.get("bv")), q_norm=V(Lw.get("q_norm")),
                               k_norm=V(Lw.get("k_norm")), wq=W(Lw["wq"]), wk=W(Lw["wk"]), wv=W(Lw["wv"]),
                               wo=W(Lw["wo"]), gate=W(Lw["gate"]), up=W(Lw["up"]), down=W(Lw["down"]))
        self._layers = layers
        tok = W(weights["tok_embd"])
        out = W(weights["output"]) if weights.get("output") is not None else None
        self._tok, self._out = tok, out
        onorm = V(weights["output_norm"])
        rf = V(weights.get("rope_freqs"))
        self._m = lib().zo_model_new(C.byref(c), C.byref(tok), C.byref(out) if out is not None else None,
                                     onorm, layers, rf)
        self.vocab = cfg["vocab"]
        self.kv_dim = cfg["n_head_kv"] * cfg["head_dim"]

    def __del__(self):
        m = getattr(self, "_m", None)
        if m:
            lib().zo_model_free(m)
            self._m = None

    @property
    def pos(self) -> int:
        return int(lib().zo_model_pos(self._m))

    def truncate(self, n: int):
        lib().zo_model_truncate(self._m, n)

    def restore_prefix(self, n: int):
        """forward.js:78: after kv_set filled positions [0, n), the model holds n positions."""
        if lib().zo_model_restore_prefix(self._m, int(n)):
            raise ValueError(f"prefix of {n} positions does not fit the context ({self._c.ctx})")

    def forward(self, token: int, logits: bool = True):
        out = np.zeros(self.vocab, np.float32) if logits else None
        rc = lib().zo_model_forward(self._m, int(token), _p(out), self.nthreads)
        if rc == -1:
            raise RuntimeError(f"context full ({self._c.ctx} tokens)")
        if rc == -2:
            raise ValueError(f"token id {token} out of range")
        return out

    def kv_get(self, layer: int, is_v: int, n: int) -> np.ndarray:
        out = np.zeros(n * self.kv_dim, np.float32)
        lib().zo_model_kv_get(self._m, layer, is_v, n, _p(out))
        return out

    def kv_set(self, layer: int, is_v: int, n: int, data: np.ndarray):
        data = np.ascontiguousarray(data, np.float32)
        lib().zo_model_kv_set(self._m, layer, is_v, n, _p(data))


# ------------------------------------------------------------------------------------ sampling
# src/sampling/sampler.js, restated in numpy / Python doubles (the checker of the device top-k).
def penalize(logits: np.ndarray, history, repeat_penalty=1.0, frequency=0.0, presence=0.0, last_n=64) -> np.ndarray:
    """sampler.js:98-112: a copy of the f32 logits with each distinct token of the last ``last_n``
    of ``history`` penalised in double and stored back as f32."""
    out = np.array(logits, np.float32, copy=True)
    counts = {}
    for t in list(history)[max(0, len(history) - last_n):]:
        counts[int(t)] = counts.get(int(t), 0) + 1
    for t, c in counts.items():
        l = float(out[t])
        v = (l / repeat_penalty if l > 0 else l * repeat_penalty) if repeat_penalty != 1 else l
        v -= c * frequency + presence
        out[t] = np.float32(v)
    return out


def topk_select(logits: np.ndarray, k: int):
    """sampler.js:20-42: the k largest (ids, values), value descending then index ascending
    (the order the size-k heap plus its final sort produce); NaN values are left out."""
    l = np.asarray(logits, np.float32)
    idx = np.nonzero(~np.isnan(l))[0]
    order = idx[np.lexsort((idx, -l[idx].astype(np.float64)))][:k]
    return order.astype(np.int32), l[order]


def mulberry32(seed: int):
    """src/util/rng.js:4-13 (a second statement, in numpy uint32, of the published generator)."""
    a = np.uint32(seed & 0xFFFFFFFF)

    def rand():
        nonlocal a
        with np.errstate(over="ignore"):
            a = np.uint32(a + np.uint32(0x6D2B79F5))
            t = a
            t = np.uint32(np.uint32(t ^ (t >> np.uint32(15))) * np.uint32(t | np.uint32(1)))
            t = np.uint32(t ^ np.uint32(t + np.uint32(np.uint32(t ^ (t >> np.uint32(7))) * np.uint32(t | np.uint32(61)))))
            return float(np.uint32(t ^ (t >> np.uint32(14)))) / 4294967296.0

    return rand
