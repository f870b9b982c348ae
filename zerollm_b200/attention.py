"""Host mirror of the attention side of the hot path (KV append, decode attention, KV import /
export, prefix-slot copies) over libzllm_cuda.so.

The per-sequence KV cache of one model is a device tensor [layer][k|v][n_head_kv][ctx][head_dim]
(f16 bits as int16 for ``--kv f16``, else f32), i.e. the reference worker's private cache layout
``[k|v][ownedHead][pos][hd]`` per layer (src/compute/worker.js:123, :303) for all KV heads.
"""
from __future__ import annotations

import ctypes as C

from .kernels import _ptr, _stream
from .lib import AttnGeom, KvPages, check


def _torch():
    import torch
    return torch


class KVCache:
    """Device KV cache of ``nseq`` sequences: [nseq][layer][2][n_kv][ctx][hd]."""

    def __init__(self, ctx, n_layer: int, n_kv: int, head_dim: int, max_ctx: int, kv_f16: bool, nseq: int = 1):
        torch = _torch()
        self.ctx, self.n_layer, self.n_kv, self.head_dim, self.max_ctx, self.kv_f16, self.nseq = \
            ctx, n_layer, n_kv, head_dim, max_ctx, kv_f16, nseq
        dt = torch.int16 if kv_f16 else torch.float32
        self.t = torch.zeros((nseq, n_layer, 2, n_kv, max_ctx, head_dim), dtype=dt, device=f"cuda:{ctx.device}")

    @property
    def head_stride(self) -> int:
        return self.max_ctx * self.head_dim

    @property
    def seq_stride(self) -> int:
        return self.n_layer * 2 * self.n_kv * self.max_ctx * self.head_dim

    def block(self, seq: int, layer: int, is_v: int):
        """The K (is_v=0) or V (is_v=1) block [n_kv][ctx][hd] of one layer of one sequence."""
        return self.t[seq, layer, is_v]

    def geom(self, n_head: int, n_rot: int | None = None, neox: bool = True, eps: float = 1e-6) -> AttnGeom:
        return AttnGeom(n_head=n_head, n_head_kv=self.n_kv, head_dim=self.head_dim,
                        n_rot=self.head_dim if n_rot is None else n_rot, neox=1 if neox else 0,
                        kv_f16=1 if self.kv_f16 else 0, ctx=self.max_ctx, rms_eps=float(eps),
                        seq_stride=self.seq_stride, head_stride=self.head_stride)


def rope_tables(ctx, n_rot: int, base: float, ctx_len: int, freq_factors=None):
    """(cos, sin) device tables [ctx_len][n_rot/2] (ref-kernels.js:329-342)."""
    import numpy as np
    torch = _torch()
    half = n_rot // 2
    cos = torch.empty((ctx_len, half), dtype=torch.float32, device=f"cuda:{ctx.device}")
    sin = torch.empty_like(cos)
    ff = None if freq_factors is None else np.ascontiguousarray(freq_factors, np.float32)
    check(ctx.lib.zllm_rope_tables(ctx.h, n_rot, float(base), ctx_len,
                                   None if ff is None else ff.ctypes.data_as(C.c_void_p), _ptr(cos), _ptr(sin)),
          ctx.h, "zllm_rope_tables")
    return cos, sin


def _cur_stream(dev, stream):
    torch = _torch()
    return stream if stream is not None else torch.cuda.current_stream(dev).cuda_stream


def qkv_append(ctx, geom: AttnGeom, cache: KVCache, layer: int, q, k, v, pos, seq, rope, q_norm=None, k_norm=None,
               bq=None, bk=None, bv=None, q_out=None, stream=None):
    """Norms, RoPE and the K/V append for ntok tokens; returns the roped queries [ntok][n_head*hd].
    ``pos`` / ``seq`` are int32 device tensors [ntok]; the cache blocks of ``layer`` are written."""
    torch = _torch()
    ntok = q.shape[0]
    if q_out is None:
        q_out = torch.empty((ntok, geom.n_head * geom.head_dim), dtype=torch.float32, device=q.device)
    kc = cache.block(0, layer, 0)
    vc = cache.block(0, layer, 1)
    st = _cur_stream(q.device, stream)
    check(ctx.lib.zllm_qkv_append(ctx.h, C.byref(geom), ntok, _ptr(q), q.stride(0), _ptr(k), _ptr(v), k.stride(0),
                                  _ptr(bq), _ptr(bk), _ptr(bv), _ptr(q_norm), _ptr(k_norm), _ptr(rope[0]), _ptr(rope[1]),
                                  _ptr(pos), _ptr(seq), _ptr(q_out), _ptr(kc), _ptr(vc), _stream(st)),
          ctx.h, "zllm_qkv_append")
    return q_out


def attn_decode(ctx, geom: AttnGeom, cache: KVCache, layer: int, q, npos, max_pos: int, out=None, stream=None):
    """Decode attention for nseq sequences: q [nseq][n_head*hd], npos int32 device [nseq]."""
    torch = _torch()
    nseq = q.shape[0]
    if out is None:
        out = torch.empty_like(q)
    st = _cur_stream(q.device, stream)
    check(ctx.lib.zllm_attn_decode(ctx.h, C.byref(geom), _ptr(q), _ptr(cache.block(0, layer, 0)),
                                   _ptr(cache.block(0, layer, 1)), _ptr(npos), nseq, int(max_pos), _ptr(out), _stream(st)),
          ctx.h, "zllm_attn_decode")
    return out


def kv_set(ctx, geom: AttnGeom, block, n: int, data, stream=None):
    """kvSet: f32 [n][n_kv*hd] (device tensor) into a K or V block."""
    st = _cur_stream(data.device, stream)
    check(ctx.lib.zllm_kv_import(ctx.h, C.byref(geom), _ptr(block), n, _ptr(data), _stream(st)), ctx.h, "zllm_kv_import")


def kv_get(ctx, geom: AttnGeom, block, n: int, stream=None):
    """kvGet: a K or V block's first n positions as f32 [n][n_kv*hd]."""
    torch = _torch()
    out = torch.empty((n, geom.n_head_kv * geom.head_dim), dtype=torch.float32, device=block.device)
    st = _cur_stream(block.device, stream)
    check(ctx.lib.zllm_kv_export(ctx.h, C.byref(geom), _ptr(block), n, _ptr(out), _stream(st)), ctx.h, "zllm_kv_export")
    return out


def kv_copy(ctx, geom: AttnGeom, dst, dst_head_stride: int, src, src_head_stride: int, n: int, stream=None):
    st = _cur_stream(dst.device, stream)
    check(ctx.lib.zllm_kv_copy(ctx.h, C.byref(geom), _ptr(dst), dst_head_stride, _ptr(src), src_head_stride, n,
                               _stream(st)), ctx.h, "zllm_kv_copy")


class PagedKV:
    """Paged K and V pools of one layer: [num_pages][n_kv][page_size][hd] each (f16 bits as int16 or
    f32), and a block table [rows][max_pages] int32 of page indices (zllm_kv_pages)."""

    def __init__(self, ctx, n_kv: int, head_dim: int, num_pages: int, page_size: int, kv_f16: bool, table):
        torch = _torch()
        self.ctx, self.n_kv, self.head_dim, self.num_pages, self.page_size, self.kv_f16 = \
            ctx, n_kv, head_dim, num_pages, page_size, kv_f16
        dt = torch.int16 if kv_f16 else torch.float32
        shape = (num_pages, n_kv, page_size, head_dim)
        self.k = torch.zeros(shape, dtype=dt, device=f"cuda:{ctx.device}")
        self.v = torch.zeros(shape, dtype=dt, device=f"cuda:{ctx.device}")
        self.table = torch.as_tensor(table, dtype=torch.int32).to(f"cuda:{ctx.device}").contiguous()
        self.max_pages = self.table.shape[1]

    def desc(self) -> KvPages:
        return KvPages(block_table=self.table.data_ptr(), max_pages=self.max_pages, num_pages=self.num_pages,
                       page_size=self.page_size)

    def geom(self, n_head: int, n_rot: int | None = None, neox: bool = True, eps: float = 1e-6) -> AttnGeom:
        return AttnGeom(n_head=n_head, n_head_kv=self.n_kv, head_dim=self.head_dim,
                        n_rot=self.head_dim if n_rot is None else n_rot, neox=1 if neox else 0,
                        kv_f16=1 if self.kv_f16 else 0, ctx=self.max_pages * self.page_size, rms_eps=float(eps),
                        seq_stride=0, head_stride=0)


def qkv_append_paged(ctx, geom: AttnGeom, kv: PagedKV, q, k, v, pos, seq, rope, q_norm=None, k_norm=None, bq=None,
                     bk=None, bv=None, q_out=None, stream=None):
    """qkv_append into the paged pools (token t at position pos[t] of table row seq[t])."""
    torch = _torch()
    ntok = q.shape[0]
    if q_out is None:
        q_out = torch.empty((ntok, geom.n_head * geom.head_dim), dtype=torch.float32, device=q.device)
    pg = kv.desc()
    st = _cur_stream(q.device, stream)
    check(ctx.lib.zllm_qkv_append_paged(ctx.h, C.byref(geom), C.byref(pg), ntok, _ptr(q), q.stride(0), _ptr(k), _ptr(v),
                                        k.stride(0), _ptr(bq), _ptr(bk), _ptr(bv), _ptr(q_norm), _ptr(k_norm),
                                        _ptr(rope[0]), _ptr(rope[1]), _ptr(pos), _ptr(seq), _ptr(q_out), _ptr(kv.k),
                                        _ptr(kv.v), _stream(st)), ctx.h, "zllm_qkv_append_paged")
    return q_out


def attn_decode_paged(ctx, geom: AttnGeom, kv: PagedKV, q, npos, max_pos: int, out=None, stream=None):
    """Decode attention over the paged pools: query s reads table row s."""
    torch = _torch()
    nseq = q.shape[0]
    if out is None:
        out = torch.empty_like(q)
    pg = kv.desc()
    st = _cur_stream(q.device, stream)
    check(ctx.lib.zllm_attn_decode_paged(ctx.h, C.byref(geom), C.byref(pg), _ptr(q), _ptr(kv.k), _ptr(kv.v), _ptr(npos),
                                         nseq, int(max_pos), _ptr(out), _stream(st)), ctx.h, "zllm_attn_decode_paged")
    return out
