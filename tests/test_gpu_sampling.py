"""Device candidate selection for sampling (zllm_topk / zllm_model_topk) against the oracle's
restatement of sampler.js's penalties and topKSelect: ids and values bit-exact, at the output
head's vocabulary, with ties, NaN and -inf, rows shorter than the chunking, and penalties; then the
whole seeded sampler over a model's device-resident logits against the same sampler fed from the
oracle's selection (test/sampler.test.js's properties hold through the device path).
"""
import ctypes as C

import numpy as np
import pytest

import oracle as O
from zerollm_b200 import ggml, synth
from zerollm_b200.kernels import Context
from zerollm_b200.lib import E_TOKEN, OK
from zerollm_b200.model import CudaModel
from zerollm_b200.sampler import Sampler

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def _ptr(a):
    return a.ctypes.data_as(C.c_void_p) if a is not None and a.size else None


def _topk(ctx, logits, k, hist=(), rp=1.0, freq=0.0, pres=0.0):
    logits = np.ascontiguousarray(np.atleast_2d(logits), np.float32)
    rows, n = logits.shape
    s = Sampler(repeat_penalty=rp, frequency_penalty=freq, presence_penalty=pres, repeat_last_n=64)
    pt, pc = (np.asarray(x, np.int32) for x in s.penalised(list(hist)))
    ids = np.empty((rows, k), np.int32)
    vals = np.empty((rows, k), np.float32)
    rc = ctx.lib.zllm_topk(ctx.h, _ptr(logits), rows, n, k, _ptr(pt), _ptr(pc), int(pt.size), rp, freq, pres, _ptr(ids),
                           _ptr(vals))
    assert rc == OK, ctx.lib.zllm_last_error(ctx.h)
    return ids, vals


def _want(row, k, hist=(), rp=1.0, freq=0.0, pres=0.0):
    ids, vals = O.topk_select(O.penalize(row, hist, rp, freq, pres, 64), k)
    pad = k - ids.size
    return np.concatenate([ids, np.full(pad, -1, np.int32)]), vals


def _check(ctx, logits, k, **kw):
    ids, vals = _topk(ctx, logits, k, **kw)
    for r, row in enumerate(np.atleast_2d(logits)):
        wi, wv = _want(row, k, **kw)
        assert np.array_equal(ids[r], wi), (r, k)
        assert np.array_equal(vals[r][: wv.size], wv), (r, k)


def test_topk_kernel_matches_oracle():
    ctx = Context(0)
    rng = np.random.default_rng(5)
    big = rng.standard_normal((3, 151936)).astype(np.float32)
    for k in (1, 40, 256):
        _check(ctx, big, k)
    ties = np.round(rng.standard_normal((2, 151936)) * 2).astype(np.float32) / 2     # a few dozen distinct values
    ties[0, ::1001] = np.nan
    ties[1, ::997] = -np.inf
    for k in (1, 40, 256):
        _check(ctx, ties, k)
    _check(ctx, rng.standard_normal((1, 10)).astype(np.float32), 10)          # most chunks empty
    _check(ctx, rng.standard_normal((2, 1000)).astype(np.float32), 256)       # k above a chunk's length
    nan_row = np.full((1, 64), np.nan, np.float32)
    nan_row[0, 7] = 1.0
    _check(ctx, nan_row, 4)                                                   # fewer finite values than k
    hist = [5, 9, 9, 151935, 0, 77, 9, 5] * 3
    _check(ctx, big, 40, hist=hist, rp=1.3, freq=0.1, pres=0.25)
    _check(ctx, -np.abs(big), 40, hist=hist, rp=1.3)
    pt = np.asarray([151936], np.int32)
    pc = np.asarray([1], np.int32)
    ids = np.empty(4, np.int32)
    vals = np.empty(4, np.float32)
    assert ctx.lib.zllm_topk(ctx.h, _ptr(big), 1, 151936, 4, _ptr(pt), _ptr(pc), 1, 1.1, 0.0, 0.0, _ptr(ids),
                             _ptr(vals)) == E_TOKEN
    ctx.close()


def test_sampler_over_device_logits():
    cfg = synth.tiny()
    w = synth.make_model(cfg, seed=13, quant="q4_k_m", dist="tame", output_type=ggml.F16)
    m = CudaModel.create(cfg, w, ctx=64, kv="f16")
    toks = [3, 17, 42, 5]
    host = m.forwardBatch(toks, logits="all").copy()
    hist = [3, 17, 3, 42, 5, 5, 5]
    s = Sampler(temperature=0.9, top_k=40, top_p=0.95, min_p=0.02, repeat_penalty=1.2, frequency_penalty=0.05,
                presence_penalty=0.1, seed=21)
    ids, vals = s.candidates(m, hist, rows=4)
    for r in range(4):
        wi, wv = _want(host[r], 40, hist, 1.2, 0.05, 0.1)
        assert np.array_equal(ids[r], wi) and np.array_equal(vals[r], wv)
    # the seeded draws through the device selection == the same sampler fed by the oracle
    ref = Sampler(temperature=0.9, top_k=40, top_p=0.95, min_p=0.02, repeat_penalty=1.2, frequency_penalty=0.05,
                  presence_penalty=0.1, seed=21)
    for _ in range(50):
        got = s.sample(m, hist, row=3)
        wi, wv = _want(host[3], 40, hist, 1.2, 0.05, 0.1)
        assert got == ref.draw(ref.from_candidates(wi, wv))
    greedy = Sampler(temperature=0)
    assert m.forwardBatch([9], logits="device") is None          # logits stay on the device
    t = greedy.sample(m)
    m.truncate(4)
    assert t == int(np.argmax(m.forward(9)))
    m.close()
