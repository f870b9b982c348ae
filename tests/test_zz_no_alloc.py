"""zllm_attn_decode_noalloc: the decode attention entry point whose scratch is a fixed array in the
library, for callers that may not allocate device memory inside a decode step (a server whose KV
pool already holds all free HBM, a host whose own allocator owns the device memory).

Called through the C ABI and checked against zllm_attn_decode (same kernel, same split, so the
results agree well inside the attention tolerance) on two calls in a row with different lengths.
The device's free memory is read before the very first no-alloc call of the process and must not
drop across the calls: the library loads the array when the context is created, so not even the
first call allocates.  The same check also runs in a fresh process with lazy module loading forced
on (CUDA_MODULE_LOADING=LAZY), the case where a module's device arrays appear on first touch.
Oversized requests are refused before anything runs.  This file sorts last so that a run stopping
at the first failure has already run every other test."""
import ctypes as C
import gc
import os
import subprocess
import sys

import numpy as np
import pytest

from zerollm_b200.attention import KVCache
from zerollm_b200.kernels import Context
from zerollm_b200.lib import E_ARG

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _filled(ctx, rng, nkv, hd, max_ctx, nseq):
    cache = KVCache(ctx, 1, nkv, hd, max_ctx, True, nseq)
    cache.t.copy_(torch.as_tensor(rng.standard_normal(cache.t.shape).astype(np.float16).view(np.int16)))
    return cache


def _call(ctx, fn, g, q, cache, npos, max_pos, out):
    P = lambda t: C.c_void_p(t.data_ptr())
    return fn(ctx.h, C.byref(g), P(q), P(cache.block(0, 0, 0)), P(cache.block(0, 0, 1)), P(npos), q.shape[0],
              int(max_pos), P(out), C.c_void_p(1))          # (void*)1: the legacy default stream, torch's stream


def check_noalloc_against_allocating_entry_point():
    """Two no-alloc calls in a row (different lengths) equal the allocating entry point's results,
    and the device's free memory, read before the first no-alloc call, does not drop."""
    ctx = Context(0)
    try:
        L = ctx.lib
        rng = np.random.default_rng(2026)
        nseq, nh, nkv, hd, max_ctx = 3, 32, 8, 128, 3000
        cache = _filled(ctx, rng, nkv, hd, max_ctx, nseq)
        g = cache.geom(nh)
        q = torch.as_tensor((rng.standard_normal((nseq, nh * hd)) * 2).astype(np.float32)).cuda()
        lens = [np.array([2900, 1, 777], np.int32), np.array([64, 2999, 130], np.int32)]
        npos = [torch.as_tensor(n).cuda() for n in lens]
        want = []
        for n, t in zip(lens, npos):                                # the allocating entry point first
            out = torch.empty_like(q)
            assert _call(ctx, L.zllm_attn_decode, g, q, cache, t, n.max(), out) == 0
            want.append(out)
        outs = [torch.empty_like(q) for _ in lens]
        gc.collect()                                                # earlier handles are freed now, not mid-check
        torch.cuda.synchronize()
        free0 = torch.cuda.mem_get_info()[0]
        for n, t, o in zip(lens, npos, outs):                       # the first no-alloc calls of the process
            assert _call(ctx, L.zllm_attn_decode_noalloc, g, q, cache, t, n.max(), o) == 0, \
                L.zllm_last_error(ctx.h).decode()
        torch.cuda.synchronize()
        free1 = torch.cuda.mem_get_info()[0]
        assert free1 >= free0, (free0, free1)                       # nothing allocated (a late free elsewhere may add)
        assert ctx.lib.zllm_sync(ctx.h) == 0
        for got, ref in zip(outs, want):
            rel = float((got - ref).abs().max() / ref.abs().max())
            assert rel <= 2e-3, rel                                  # the f16-KV attention tolerance
            assert torch.equal(got, ref)                             # same kernel, same split: same bits
    finally:
        ctx.close()


def test_noalloc_matches_allocating_entry_point():
    check_noalloc_against_allocating_entry_point()


def test_noalloc_first_call_allocates_nothing_in_a_fresh_process():
    env = dict(os.environ, CUDA_MODULE_LOADING="LAZY")
    code = ("import sys; sys.path.insert(0, %r); sys.path.insert(0, %r); import test_zz_no_alloc as t; "
            "t.check_noalloc_against_allocating_entry_point(); print('fresh-process check passed')"
            % (ROOT, os.path.join(ROOT, "tests")))
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    assert "fresh-process check passed" in r.stdout


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
