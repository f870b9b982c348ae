"""zllm_attn_decode_noalloc: the decode attention entry point whose scratch is a fixed array in the
library.  Called through the C ABI and checked against zllm_attn_decode (same kernel, same split, so
the results agree well inside the attention tolerance) on two calls in a row with different
lengths, with no change in the device's free memory across those calls; oversized requests are
refused before anything runs."""
import ctypes as C
import gc

import numpy as np
import pytest

from zerollm_b200.attention import KVCache
from zerollm_b200.kernels import Context
from zerollm_b200.lib import E_ARG

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def _filled(ctx, rng, nkv, hd, max_ctx, nseq):
    cache = KVCache(ctx, 1, nkv, hd, max_ctx, True, nseq)
    cache.t.copy_(torch.as_tensor(rng.standard_normal(cache.t.shape).astype(np.float16).view(np.int16)))
    return cache


def _call(ctx, fn, g, q, cache, npos, max_pos, out):
    P = lambda t: C.c_void_p(t.data_ptr())
    return fn(ctx.h, C.byref(g), P(q), P(cache.block(0, 0, 0)), P(cache.block(0, 0, 1)), P(npos), q.shape[0],
              int(max_pos), P(out), C.c_void_p(1))          # (void*)1: the legacy default stream, torch's stream


def test_noalloc_matches_allocating_entry_point():
    ctx = Context(0)
    try:
        L = ctx.lib
        rng = np.random.default_rng(2026)
        nseq, nh, nkv, hd, max_ctx = 3, 32, 8, 128, 3000
        cache = _filled(ctx, rng, nkv, hd, max_ctx, nseq)
        g = cache.geom(nh)
        q = torch.as_tensor((rng.standard_normal((nseq, nh * hd)) * 2).astype(np.float32)).cuda()
        lens = [np.array([2900, 1, 777], np.int32), np.array([64, 2999, 130], np.int32)]
        want = []
        for n in lens:
            out = torch.empty_like(q)
            assert _call(ctx, L.zllm_attn_decode, g, q, cache, torch.as_tensor(n).cuda(), n.max(), out) == 0
            want.append(out)
        warm = torch.empty_like(q)
        npos0 = torch.as_tensor(lens[0]).cuda()
        assert _call(ctx, L.zllm_attn_decode_noalloc, g, q, cache, npos0, lens[0].max(), warm) == 0
        outs = [torch.empty_like(q) for _ in lens]
        npos = [torch.as_tensor(n).cuda() for n in lens]
        gc.collect()                                                # earlier tests' handles are freed now, not mid-check
        torch.cuda.synchronize()
        free0 = torch.cuda.mem_get_info()[0]
        for n, t, o in zip(lens, npos, outs):                       # two calls in a row, different lengths
            assert _call(ctx, L.zllm_attn_decode_noalloc, g, q, cache, t, n.max(), o) == 0, \
                L.zllm_last_error(ctx.h).decode()
        torch.cuda.synchronize()
        assert torch.cuda.mem_get_info()[0] >= free0                # nothing allocated (a late free elsewhere may add)
        assert ctx.lib.zllm_sync(ctx.h) == 0
        for got, ref in zip(outs, want):
            rel = float((got - ref).abs().max() / ref.abs().max())
            assert rel <= 2e-3, rel                                  # the f16-KV attention tolerance
            assert rel <= 1e-6, rel
        assert torch.equal(warm, want[0])
    finally:
        ctx.close()


def test_noalloc_rejects_requests_beyond_its_scratch():
    ctx = Context(0)
    try:
        L = ctx.lib
        rng = np.random.default_rng(7)
        cache = _filled(ctx, rng, 8, 128, 64, 1)
        g = cache.geom(64)                                           # group 8
        for nseq in (200, 513):                                      # 6.7 MB of partials; 4104 (seq, head) pairs
            q = torch.zeros((nseq, 64 * 128), dtype=torch.float32, device="cuda")
            npos = torch.ones(nseq, dtype=torch.int32, device="cuda")
            out = torch.full_like(q, 5.0)
            assert _call(ctx, L.zllm_attn_decode_noalloc, g, q, cache, npos, 1, out) == E_ARG
            assert b"fixed scratch" in L.zllm_last_error(ctx.h)
            torch.cuda.synchronize()
            assert bool((out == 5.0).all())                          # nothing was launched
    finally:
        ctx.close()
