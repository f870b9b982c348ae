"""Host mirror of the reference's kernel interface over libzllm_cuda.so.

Mirrors ``src/compute/ref-kernels.js``: a ``Weight`` is a matrix of raw GGUF rows (type, rows,
cols), an ``Act`` is an activation with a lazily built Q8_0-style quantization shared by every
matmul that consumes it (``Act.quant``, ref-kernels.js:24-37), and ``matvec(w, act, y)``
computes ``y[r] = dot(W[r], x)`` (ref-kernels.js:127).  Device memory is held in torch tensors
(plumbing only); every computation runs in libzllm_cuda.so.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import ggml
from .lib import check, load


def _torch():
    import torch
    return torch


def _ptr(t):
    return None if t is None else C.c_void_p(t.data_ptr())


# cudaStreamLegacy: the library reads a NULL stream as "the context's own stream", so torch's
# default stream (handle 0) must be passed as the explicit legacy-stream handle.
STREAM_LEGACY = 1


def _stream(st) -> C.c_void_p:
    st = int(st)
    return C.c_void_p(st if st else STREAM_LEGACY)


class Context:
    """One CUDA device, one stream, one status word (zllm_init)."""

    def __init__(self, device: int = 0):
        self.lib = load()
        h = C.c_void_p()
        rc = self.lib.zllm_init(device, C.byref(h))
        if rc:
            check(rc, None, f"zllm_init(device {device})")
        self.h = h
        self.device = device

    @property
    def stream(self) -> int:
        return self.lib.zllm_stream(self.h) or 0

    def torch_stream(self):
        torch = _torch()
        return torch.cuda.ExternalStream(self.stream, device=f"cuda:{self.device}")

    def sync(self):
        check(self.lib.zllm_sync(self.h), self.h, "zllm_sync")

    def close(self):
        if getattr(self, "h", None):
            self.lib.zllm_destroy(self.h)
            self.h = None

    def __del__(self):
        self.close()


class Weight:
    """A device-resident matrix uploaded from raw GGUF bytes (zllm_weight_upload)."""

    def __init__(self, ctx: Context, type: int, rows: int, cols: int, data):
        self.ctx, self.type, self.rows, self.cols = ctx, int(type), int(rows), int(cols)
        buf = np.ascontiguousarray(np.frombuffer(data, np.uint8) if isinstance(data, (bytes, bytearray)) else data, np.uint8)
        h = C.c_void_p()
        check(ctx.lib.zllm_weight_upload(ctx.h, self.type, self.rows, self.cols, buf.ctypes.data_as(C.c_void_p),
                                         buf.nbytes, C.byref(h)), ctx.h, "zllm_weight_upload")
        self.h = h

    @classmethod
    def from_tensor(cls, ctx: Context, t: dict) -> "Weight":
        return cls(ctx, t["type"], t["rows"], t["cols"], t["data"])

    @property
    def device_bytes(self) -> int:
        n = C.c_size_t()
        check(self.ctx.lib.zllm_weight_info(self.h, None, None, None, C.byref(n)), self.ctx.h)
        return n.value

    def free(self):
        if getattr(self, "h", None):
            self.ctx.lib.zllm_weight_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


class Act:
    """f32 activations x [ntok, K] on the device with a lazily built int8 quantization."""

    def __init__(self, ctx: Context, x):
        torch = _torch()
        if not isinstance(x, torch.Tensor):
            x = torch.as_tensor(np.ascontiguousarray(x, np.float32))
        if x.dim() == 1:
            x = x.view(1, -1)
        self.ctx = ctx
        self.x = x.to(device=f"cuda:{ctx.device}", dtype=torch.float32).contiguous()
        self.q = self.d = self.s = None

    @property
    def ntok(self) -> int:
        return self.x.shape[0]

    @property
    def k(self) -> int:
        return self.x.shape[1]

    def quant(self, stream=None) -> "Act":
        if self.q is None:
            torch = _torch()
            dev = self.x.device
            self.q = torch.empty((self.ntok, self.k), dtype=torch.int8, device=dev)
            self.d = torch.empty((self.ntok, self.k // 32), dtype=torch.float32, device=dev)
            self.s = torch.empty((self.ntok, self.k // 32), dtype=torch.int32, device=dev)
            st = stream if stream is not None else torch.cuda.current_stream(dev).cuda_stream
            check(self.ctx.lib.zllm_quantize_act(self.ctx.h, _ptr(self.x), self.k, self.ntok, _ptr(self.q), _ptr(self.d),
                                                 _ptr(self.s), _stream(st)), self.ctx.h, "zllm_quantize_act")
        return self


def matvec(w: Weight, a: Act, y=None, y_add=None, stream=None, fused_quant: bool = False):
    """y[t, r] = (y_add[t, r] +) dot(W[r], x[t]) on the device; returns y [ntok, rows].

    ``fused_quant`` (one token, k-quant weight) passes the f32 activation alone and lets the GEMV
    quantize it."""
    torch = _torch()
    if a.k != w.cols:
        raise ValueError(f"activation length {a.k} != weight cols {w.cols}")
    if y is None:
        y = torch.empty((a.ntok, w.rows), dtype=torch.float32, device=a.x.device)
    st = stream if stream is not None else torch.cuda.current_stream(a.x.device).cuda_stream
    if w.type in ggml.QUANTIZED and fused_quant:
        args = (None, None, None, _ptr(a.x))
    elif w.type in ggml.QUANTIZED:
        a.quant(st)
        args = (_ptr(a.q), _ptr(a.d), _ptr(a.s), None)
    else:
        args = (None, None, None, _ptr(a.x))
    check(w.ctx.lib.zllm_mm(w.ctx.h, w.h, *args, a.ntok, _ptr(y), y.stride(0), _ptr(y_add), _stream(st)),
          w.ctx.h, "zllm_mm")
    return y


def matvec_host(w: Weight, x: np.ndarray) -> np.ndarray:
    """Host buffers in and out (zllm_matvec): x [ntok, cols] or [cols] f32 -> y [ntok, rows]."""
    x = np.ascontiguousarray(x, np.float32)
    ntok = 1 if x.ndim == 1 else x.shape[0]
    y = np.empty((ntok, w.rows), np.float32)
    check(w.ctx.lib.zllm_matvec(w.ctx.h, w.h, x.ctypes.data_as(C.c_void_p), ntok, y.ctypes.data_as(C.c_void_p)),
          w.ctx.h, "zllm_matvec")
    return y
