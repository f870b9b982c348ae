"""GGUF reader feeding the device uploads straight from a memory mapping.

Follows the reference's reader (src/gguf/reader.js:132-193): the "GGUF" magic, version 2 or 3,
tensor and metadata counts, metadata key/value pairs (reader.js:66-92), the tensor infos (name,
dims in ggml order -- dims[0] is the row length --, type, offset relative to the data section),
and the data section starting at the next multiple of ``general.alignment`` (default 32).  The
same checks raise the same messages: a bad magic, an unsupported version, implausible counts or
lengths, and a tensor that extends past the end of the file (a truncated download).

Where the reference reads each tensor into a worker's WASM memory (readTensorBytes,
reader.js:205-214), ``GGUFFile.tensor_data`` hands out a read-only ``np.memmap`` view of the file:
``CudaModel`` passes that pointer to ``zllm_model_set_matrix``, whose host-to-device copy and
load-time repack into the unit layout read the page cache directly -- no host-side copy of the
weights.  ``model_config`` maps the metadata to the model config (src/model/config.js:73-123) and
``load_model`` names the tensors the way RefModel does (src/model/forward.js:26-41).
"""
from __future__ import annotations

import math
import os
import struct

import numpy as np

from . import ggml

MAX_STRING = 1 << 30          # reader.js:5-6
MAX_ARRAY = 1 << 28
SUPPORTED_ARCHS = ("llama", "qwen2", "qwen3")   # config.js:6, without the hybrid qwen35

# GGUF metadata value types (src/gguf/types.js: GGUF_TYPE)
(U8, I8, U16, I16, U32, I32, F32, BOOL, STRING, ARRAY, U64, I64, F64) = range(13)
_SCALAR = {U8: "<B", I8: "<b", U16: "<H", I16: "<h", U32: "<I", I32: "<i", F32: "<f", U64: "<Q", I64: "<q",
           F64: "<d"}
_NP = {U8: np.uint8, I8: np.int8, U16: np.uint16, I16: np.int16, U32: np.uint32, I32: np.int32, F32: np.float32,
       U64: np.uint64, I64: np.int64, F64: np.float64}


class _Cursor:
    """Sequential little-endian reads over the mapped file, with the reference's end-of-file check."""

    def __init__(self, buf: memoryview, size: int):
        self.buf, self.size, self.pos = buf, size, 0

    def need(self, n: int) -> int:
        if self.pos + n > self.size:
            raise ValueError(f"GGUF: unexpected end of file at byte {self.pos} (need {n} more, file is {self.size} bytes)")
        p = self.pos
        self.pos += n
        return p

    def scalar(self, t: int):
        fmt = _SCALAR[t]
        return struct.unpack_from(fmt, self.buf, self.need(struct.calcsize(fmt)))[0]

    def size_field(self, what: str) -> int:
        v = self.scalar(U64)
        if v > (1 << 53) - 1:
            raise ValueError(f"GGUF: {what} does not fit in a safe integer")
        return v

    def string(self) -> str:
        n = self.size_field("string length")
        if n > MAX_STRING:
            raise ValueError(f"GGUF: implausible string length {n}")
        p = self.need(n)
        return bytes(self.buf[p:p + n]).decode("utf-8", errors="replace")

    def value(self, t: int):
        """One metadata value (reader.js:66-92).  Numeric arrays come back as numpy arrays (the
        tokenizer's score and type arrays run to 150k entries), strings as a list."""
        if t in _SCALAR:
            return self.scalar(t)
        if t == BOOL:
            return self.buf[self.need(1)] != 0
        if t == STRING:
            return self.string()
        if t == ARRAY:
            et = self.scalar(U32)
            n = self.size_field("array length")
            if n > MAX_ARRAY:
                raise ValueError(f"GGUF: implausible array length {n}")
            if et in _NP:
                dt = np.dtype(_NP[et]).newbyteorder("<")
                p = self.need(n * dt.itemsize)
                return np.frombuffer(self.buf, dt, n, p).copy()
            return [self.value(et) for _ in range(n)]
        raise ValueError(f"GGUF: unknown metadata value type {t}")


class TensorInfo:
    __slots__ = ("name", "dims", "type", "offset", "abs_offset", "n_elements", "n_bytes")

    def __init__(self, name, dims, type_, offset, abs_offset, n_elements, n_bytes):
        self.name, self.dims, self.type, self.offset = name, dims, type_, offset
        self.abs_offset, self.n_elements, self.n_bytes = abs_offset, n_elements, n_bytes

    @property
    def rows(self) -> int:
        return self.n_elements // self.dims[0]

    @property
    def cols(self) -> int:
        return self.dims[0]


class GGUFFile:
    """A parsed GGUF file (reader.js:105-128): ``metadata``, ``tensors`` (in file order),
    ``alignment``, ``data_start``; the tensor bytes stay in the file mapping."""

    def __init__(self, path, size, version, metadata, tensors, alignment, data_start, mm):
        self.path, self.file_size, self.version = path, size, version
        self.metadata, self.tensors = metadata, tensors
        self.tensor_map = {t.name: t for t in tensors}
        self.alignment, self.data_start = alignment, data_start
        self._mm = mm

    def get(self, key, default=None):
        return self.metadata.get(key, default)

    def tensor(self, name):
        return self.tensor_map.get(name)

    def require_tensor(self, name) -> TensorInfo:
        t = self.tensor_map.get(name)
        if t is None:
            raise KeyError(f"tensor not found in GGUF: {name}")
        return t

    def tensor_data(self, name_or_info) -> np.ndarray:
        """The tensor's raw bytes as a read-only uint8 view of the file mapping."""
        t = name_or_info if isinstance(name_or_info, TensorInfo) else self.require_tensor(name_or_info)
        if t.n_bytes is None:
            raise ValueError(f"tensor {t.name}: unknown type {t.type}")
        return self._mm[t.abs_offset:t.abs_offset + t.n_bytes]


def read_gguf(path: str) -> GGUFFile:
    """Parse the header, metadata and tensor infos of a GGUF file (reader.js:132-193)."""
    size = os.path.getsize(path)
    if size < 4:
        raise ValueError(f"GGUF: unexpected end of file at byte 0 (need 4 more, file is {size} bytes)")
    mm = np.memmap(path, np.uint8, "r")
    c = _Cursor(memoryview(mm), size)
    magic = bytes(mm[:4])
    if magic != b"GGUF":
        raise ValueError(f'not a GGUF file (magic "{magic.decode("latin1")}")')
    c.pos = 4
    version = c.scalar(U32)
    if version < 2 or version > 3:
        raise ValueError(f"unsupported GGUF version {version} (expected 2 or 3)")
    n_tensors = c.size_field("tensor count")
    n_kv = c.size_field("metadata count")
    if n_tensors > 1e6 or n_kv > 1e6:
        raise ValueError("GGUF: implausible tensor/metadata count (corrupt file?)")
    meta = {}
    for _ in range(n_kv):
        key = c.string()
        meta[key] = c.value(c.scalar(U32))
    align = meta.get("general.alignment", 32)
    if not isinstance(align, int) or isinstance(align, bool) or align <= 0:
        raise ValueError(f"GGUF: bad general.alignment {align}")
    raw = []
    for _ in range(n_tensors):
        name = c.string()
        nd = c.scalar(U32)
        if nd < 1 or nd > 8:
            raise ValueError(f"GGUF: tensor {name} has {nd} dims")
        dims = [c.size_field("tensor dim") for _ in range(nd)]
        raw.append((name, dims, c.scalar(U32), c.size_field("tensor offset")))
    data_start = -(-c.pos // align) * align
    tensors = []
    for name, dims, t, off in raw:
        n_el = math.prod(int(d) for d in dims)   # Python ints: a corrupt header cannot wrap around
        if n_el > 1 << 53:
            raise ValueError(f"GGUF: tensor {name} has an implausible element count {n_el} (dims {dims})")
        n_bytes = None
        if t in ggml.TYPE_INFO:
            _, bs, ts = ggml.TYPE_INFO[t]
            n_bytes = (n_el // bs) * ts          # types.js tensorBytes: whole blocks
        abs_off = data_start + off
        if n_bytes is not None and abs_off + n_bytes > size:
            raise ValueError(f"GGUF: tensor {name} extends past end of file (truncated download?): needs bytes up to "
                             f"{abs_off + n_bytes}, file has {size}")
        tensors.append(TensorInfo(name, dims, t, off, abs_off, n_el, n_bytes))
    return GGUFFile(path, size, version, meta, tensors, align, data_start, mm)


def model_config(g: GGUFFile) -> dict:
    """Model config from the metadata (config.js:73-123), as the dict ``CudaModel`` takes."""
    arch = g.get("general.architecture")
    if not isinstance(arch, str):
        raise ValueError("GGUF has no general.architecture")
    if arch not in SUPPORTED_ARCHS:
        raise ValueError(f'architecture "{arch}" is not supported (supported: {", ".join(SUPPORTED_ARCHS)})')

    def need(k):
        v = g.get(f"{arch}.{k}")
        if v is None:
            raise ValueError(f"GGUF is missing metadata key {arch}.{k}")
        return v

    n_embd = int(need("embedding_length"))
    n_head = int(need("attention.head_count"))
    n_head_kv = int(g.get(f"{arch}.attention.head_count_kv", n_head))
    head_dim = g.get(f"{arch}.attention.key_length")
    if head_dim is None:
        if n_embd % n_head:
            raise ValueError(f"cannot determine integer head_dim (embd {n_embd} / heads {n_head})")
        head_dim = n_embd // n_head
    head_dim = int(head_dim)
    embd = g.tensor("token_embd.weight")
    toks = g.get("tokenizer.ggml.tokens")
    vocab = g.get(f"{arch}.vocab_size")
    if vocab is None:
        vocab = len(toks) if isinstance(toks, list) else (embd.dims[1] if embd is not None else None)
    if vocab is None:
        raise ValueError("cannot determine vocab size")
    return dict(arch=arch, n_ctx_train=int(need("context_length")), n_embd=n_embd, n_layer=int(need("block_count")),
                n_ff=int(need("feed_forward_length")), n_head=n_head, n_head_kv=n_head_kv, head_dim=head_dim,
                n_rot=int(g.get(f"{arch}.rope.dimension_count", head_dim)), vocab=int(vocab),
                rms_eps=float(g.get(f"{arch}.attention.layer_norm_rms_epsilon", 1e-5)),
                rope_base=float(g.get(f"{arch}.rope.freq_base", 10000)),
                rope_type="norm" if arch == "llama" else "neox",
                qk_norm=g.tensor("blk.0.attn_q_norm.weight") is not None,
                qkv_bias=g.tensor("blk.0.attn_q.bias") is not None,
                tied=g.tensor("output.weight") is None,
                has_rope_freqs=g.tensor("rope_freqs.weight") is not None)


def _vector(g: GGUFFile, t: TensorInfo) -> np.ndarray:
    """A norm / bias vector as f32 (forward.js loadVector): F32 as stored, F16 / BF16 widened."""
    raw = g.tensor_data(t)
    if t.type == ggml.F32:
        return raw.view("<f4").astype(np.float32)
    if t.type == ggml.F16:
        return raw.view("<f2").astype(np.float32)
    if t.type == ggml.BF16:
        return (raw.view("<u2").astype(np.uint32) << 16).view(np.float32)
    raise ValueError(f"tensor {t.name}: vector of type {ggml.type_name(t.type)} is not supported")


def _matrix(g: GGUFFile, t: TensorInfo) -> dict:
    if len(t.dims) != 2:
        raise ValueError(f"tensor {t.name}: expected a matrix, got dims {t.dims}")
    ggml.row_bytes(t.type, t.cols)            # raises like rowSize for unsupported types / ragged rows
    return {"type": t.type, "rows": t.rows, "cols": t.cols, "data": g.tensor_data(t)}


def load_model(path: str) -> tuple[dict, dict]:
    """``(cfg, weights)`` of a GGUF model for ``CudaModel.create``; the matrices are views of the
    file mapping (forward.js:26-41 names the tensors)."""
    g = read_gguf(path)
    cfg = model_config(g)
    W = lambda n: _matrix(g, g.require_tensor(n))       # noqa: E731
    V = lambda n: _vector(g, g.require_tensor(n))       # noqa: E731
    opt = lambda n: _vector(g, g.tensor(n)) if g.tensor(n) is not None else None   # noqa: E731
    w = {"tok_embd": W("token_embd.weight"), "output_norm": V("output_norm.weight"),
         "output": None if cfg["tied"] else W("output.weight"),
         "rope_freqs": V("rope_freqs.weight") if cfg["has_rope_freqs"] else None}
    layers = []
    for l in range(cfg["n_layer"]):
        p = f"blk.{l}."
        layers.append({"attn_norm": V(p + "attn_norm.weight"), "wq": W(p + "attn_q.weight"),
                       "wk": W(p + "attn_k.weight"), "wv": W(p + "attn_v.weight"), "wo": W(p + "attn_output.weight"),
                       "bq": opt(p + "attn_q.bias"), "bk": opt(p + "attn_k.bias"), "bv": opt(p + "attn_v.bias"),
                       "q_norm": opt(p + "attn_q_norm.weight"), "k_norm": opt(p + "attn_k_norm.weight"),
                       "ffn_norm": V(p + "ffn_norm.weight"), "gate": W(p + "ffn_gate.weight"),
                       "up": W(p + "ffn_up.weight"), "down": W(p + "ffn_down.weight")})
    w["layers"] = layers
    return cfg, w


# ------------------------------------------------------------------------------------- writer
_LAYER_NAMES = (("attn_norm", "attn_norm.weight"), ("wq", "attn_q.weight"), ("wk", "attn_k.weight"),
                ("wv", "attn_v.weight"), ("wo", "attn_output.weight"), ("bq", "attn_q.bias"), ("bk", "attn_k.bias"),
                ("bv", "attn_v.bias"), ("q_norm", "attn_q_norm.weight"), ("k_norm", "attn_k_norm.weight"),
                ("ffn_norm", "ffn_norm.weight"), ("gate", "ffn_gate.weight"), ("up", "ffn_up.weight"),
                ("down", "ffn_down.weight"))


def _put_str(out: list, s: str):
    b = s.encode()
    out.append(struct.pack("<Q", len(b)) + b)


def write_gguf(path: str, cfg: dict, weights: dict, alignment: int = 32):
    """Write a model as a GGUF v3 file (the metadata ``model_config`` reads; the layout of the
    reference's tiny-model tool, tools/make-tiny-gguf.js).  For synthetic models in tests and
    benches; the tensor bytes are written as given."""
    arch = cfg.get("arch", "qwen3")
    kv = [("general.architecture", STRING, arch), ("general.alignment", U32, alignment),
          (f"{arch}.context_length", U32, int(cfg.get("n_ctx_train", 40960))),
          (f"{arch}.embedding_length", U32, cfg["n_embd"]), (f"{arch}.block_count", U32, cfg["n_layer"]),
          (f"{arch}.feed_forward_length", U32, cfg["n_ff"]), (f"{arch}.attention.head_count", U32, cfg["n_head"]),
          (f"{arch}.attention.head_count_kv", U32, cfg["n_head_kv"]),
          (f"{arch}.attention.key_length", U32, cfg["head_dim"]),
          (f"{arch}.rope.dimension_count", U32, cfg.get("n_rot", cfg["head_dim"])),
          (f"{arch}.attention.layer_norm_rms_epsilon", F32, cfg["rms_eps"]),
          (f"{arch}.rope.freq_base", F32, cfg["rope_base"]), (f"{arch}.vocab_size", U32, cfg["vocab"])]
    tensors = []                       # (name, dims, type, bytes)

    def mat(name, t):
        tensors.append((name, [t["cols"], t["rows"]], t["type"], np.ascontiguousarray(t["data"], np.uint8)))

    def vec(name, v):
        a = np.ascontiguousarray(v, "<f4")
        tensors.append((name, [a.size], ggml.F32, a.view(np.uint8)))

    mat("token_embd.weight", weights["tok_embd"])
    vec("output_norm.weight", weights["output_norm"])
    if weights.get("output") is not None:
        mat("output.weight", weights["output"])
    if weights.get("rope_freqs") is not None:
        vec("rope_freqs.weight", weights["rope_freqs"])
    for l, L in enumerate(weights["layers"]):
        for key, name in _LAYER_NAMES:
            if L.get(key) is None:
                continue
            (mat if isinstance(L[key], dict) else vec)(f"blk.{l}.{name}", L[key])
    head = [b"GGUF", struct.pack("<IQQ", 3, len(tensors), len(kv))]
    for key, t, v in kv:
        _put_str(head, key)
        head.append(struct.pack("<I", t))
        if t == STRING:
            _put_str(head, v)
        else:
            head.append(struct.pack(_SCALAR[t], v))
    off = 0
    offs = []
    for name, dims, t, data in tensors:
        off = -(-off // alignment) * alignment
        offs.append(off)
        _put_str(head, name)
        head.append(struct.pack("<I", len(dims)) + struct.pack(f"<{len(dims)}Q", *dims))
        head.append(struct.pack("<IQ", t, off))
        off += data.nbytes
    hb = b"".join(head)
    start = -(-len(hb) // alignment) * alignment
    with open(path, "wb") as f:
        f.write(hb)
        f.write(b"\0" * (start - len(hb)))
        for (name, dims, t, data), o in zip(tensors, offs):
            f.seek(start + o)
            f.write(data.tobytes())
