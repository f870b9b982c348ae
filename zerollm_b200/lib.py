"""ctypes binding of libzllm_cuda.so (include/zllm.h).

The library is the product: there is no CPU fallback.  Loading fails loudly when the shared
object has not been built, and every call that returns a negative code raises ``ZllmError``
with the library's message.
"""
from __future__ import annotations

import ctypes as C
import os
import re

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
LIB_PATH = os.path.join(PKG, "libzllm_cuda.so")
HEADER = os.path.join(ROOT, "include", "zllm.h")

OK, E_ARG, E_OOM, E_CUDA, E_CTX_FULL, E_TIMEOUT, E_STATE, E_UNSUPPORTED, E_TOKEN, E_BATCH = 0, -1, -2, -3, -4, -5, -6, -7, -8, -9


class ZllmError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(message)
        self.code = code


vp, i32, i64, sz = C.c_void_p, C.c_int, C.c_int64, C.c_size_t
PP = C.POINTER(C.c_void_p)

# name -> (restype, argtypes)
SIGNATURES = {
    "zllm_version": (C.c_char_p, []),
    "zllm_init": (i32, [i32, PP]),
    "zllm_destroy": (None, [vp]),
    "zllm_last_error": (C.c_char_p, [vp]),
    "zllm_stream": (vp, [vp]),
    "zllm_sync": (i32, [vp]),
    "zllm_peer_wait_selftest": (i32, [vp]),
    "zllm_weight_upload": (i32, [vp, i32, i64, i64, vp, sz, PP]),
    "zllm_weight_free": (None, [vp]),
    "zllm_weight_info": (i32, [vp, C.POINTER(i32), C.POINTER(i64), C.POINTER(i64), C.POINTER(sz)]),
    "zllm_quantize_act": (i32, [vp, vp, i64, i32, vp, vp, vp, vp]),
    "zllm_mm": (i32, [vp, vp, vp, vp, vp, vp, i32, vp, i64, vp, vp]),
    "zllm_gemm_f16": (i32, [vp, vp, vp, i64, i64, i64, vp, vp]),
    "zllm_mm_fused": (i32, [vp, vp, vp, vp, C.c_double, i32, vp, vp, vp]),
    "zllm_rmsnorm_quant": (i32, [vp, vp, vp, i32, i32, C.c_double, vp, vp, vp, vp, vp]),
    "zllm_swiglu_quant": (i32, [vp, vp, vp, i32, i32, i64, vp, vp, vp, vp, vp]),
    "zllm_tp_unique_id": (i32, [vp, vp, sz]),
    "zllm_model_stream": (vp, [vp]),
    "zllm_model_tp_collective": (i32, [vp]),
    "zllm_model_set_vocab_shard": (i32, [vp, i64, i64]),
    "zllm_model_set_tp": (i32, [vp, i32, i32, vp]),
    "zllm_matvec": (i32, [vp, vp, vp, i32, vp]),
    "zllm_rope_tables": (i32, [vp, i32, C.c_double, i32, vp, vp, vp]),
    "zllm_qkv_append": (i32, [vp, vp, i32, vp, i64, vp, vp, i64, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp]),
    "zllm_attn_decode": (i32, [vp, vp, vp, vp, vp, vp, i32, i32, vp, vp]),
    "zllm_attn_decode_noalloc": (i32, [vp, vp, vp, vp, vp, vp, i32, i32, vp, vp]),
    "zllm_qkv_append_paged": (i32, [vp, vp, vp, i32, vp, i64, vp, vp, i64, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp,
                                    vp]),
    "zllm_attn_decode_paged": (i32, [vp, vp, vp, vp, vp, vp, vp, i32, i32, vp, vp]),
    "zllm_kv_import": (i32, [vp, vp, vp, i32, vp, vp]),
    "zllm_kv_export": (i32, [vp, vp, vp, i32, vp, vp]),
    "zllm_kv_copy": (i32, [vp, vp, vp, i64, vp, i64, i32, vp]),
    "zllm_model_create": (i32, [vp, vp, PP]),
    "zllm_model_set_matrix": (i32, [vp, i32, i32, i32, i64, i64, vp, sz]),
    "zllm_model_set_vector": (i32, [vp, i32, i32, vp, i64]),
    "zllm_model_ready": (i32, [vp]),
    "zllm_model_forward": (i32, [vp, i32, vp, i32, i32, vp, vp]),
    "zllm_model_decode": (i32, [vp, vp, vp, i32, vp, vp]),
    "zllm_model_generate": (i32, [vp, i32, vp, vp, i32, i32, vp]),
    "zllm_model_pos": (i32, [vp, i32]),
    "zllm_model_truncate": (i32, [vp, i32, i32]),
    "zllm_model_reset": (i32, [vp, i32]),
    "zllm_model_kv_get": (i32, [vp, i32, i32, i32, i32, vp]),
    "zllm_model_kv_set": (i32, [vp, i32, i32, i32, i32, vp]),
    "zllm_model_restore_prefix": (i32, [vp, i32, i32]),
    "zllm_model_topk": (i32, [vp, i32, i32, vp, vp, i32, C.c_double, C.c_double, C.c_double, vp, vp]),
    "zllm_topk": (i32, [vp, vp, i32, C.c_int64, i32, vp, vp, i32, C.c_double, C.c_double, C.c_double, vp, vp]),
    "zllm_model_slot_save": (i32, [vp, i32, i32]),
    "zllm_model_slot_restore": (i32, [vp, i32]),
    "zllm_model_set_graphs": (i32, [vp, i32]),
    "zllm_model_logits": (vp, [vp]),
    "zllm_model_destroy": (None, [vp]),
}


class ModelConfig(C.Structure):
    """zllm_model_config (include/zllm.h)"""
    _fields_ = [(n, C.c_int) for n in ("n_embd", "n_layer", "n_ff", "n_head", "n_head_kv", "head_dim", "n_rot", "vocab",
                                      "neox", "kv_f16", "ctx", "n_seq", "max_batch", "logits_batch")] + \
               [("rms_eps", C.c_double), ("rope_base", C.c_double)]


# tensor kinds (include/zllm.h)
T_TOK_EMBD, T_OUTPUT, T_OUTPUT_NORM, T_ROPE_FREQS = 0, 1, 2, 3
T_ATTN_NORM, T_WQ, T_WK, T_WV, T_WO, T_BQ, T_BK, T_BV, T_Q_NORM, T_K_NORM, T_FFN_NORM, T_GATE, T_UP, T_DOWN = range(10, 24)


class AttnGeom(C.Structure):
    """zllm_attn_geom (include/zllm.h)"""
    _fields_ = [("n_head", C.c_int), ("n_head_kv", C.c_int), ("head_dim", C.c_int), ("n_rot", C.c_int),
                ("neox", C.c_int), ("kv_f16", C.c_int), ("ctx", C.c_int), ("rms_eps", C.c_double),
                ("seq_stride", C.c_int64), ("head_stride", C.c_int64)]

class KvPages(C.Structure):
    """zllm_kv_pages (include/zllm.h)"""
    _fields_ = [("block_table", C.c_void_p), ("max_pages", C.c_int), ("num_pages", C.c_int), ("page_size", C.c_int)]


_lib = None


def header_functions(path: str = HEADER) -> list[str]:
    """Names of the functions include/zllm.h declares."""
    text = open(path).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(zllm_[a-z0-9_]+)\s*\(", text)))


def load(path: str = LIB_PATH):
    """Load libzllm_cuda.so (once).  Raises if it is missing: build it with
    ``python -m zerollm_b200.build`` (or ``__graft_entry__.build()``)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise ZllmError(E_STATE, f"{path} is not built: run `python -m zerollm_b200.build`")
    L = C.CDLL(path)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def check(rc: int, ctx=None, what: str = ""):
    if rc != OK:
        msg = load().zllm_last_error(ctx).decode() if ctx else ""
        raise ZllmError(rc, f"{what}: {msg}" if what else msg)
    return rc
