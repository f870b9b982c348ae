"""The on-disk formats through the CUDA backend:

* a model loaded from a GGUF file (device uploads read straight from the file mapping) computes
  the same logits, bit for bit, as the same weights uploaded from memory;
* the ZLLMKV01 prefix cache written from one CudaModel and loaded into a fresh one continues
  bit-identically (test/prefix-cache.test.js:28-48), with the f16 KV cache filled by the device
  cast of the file's f32 rows;
* a load that fails leaves the model at position 0 and usable (prefix-cache.test.js:84-98).
"""
import numpy as np
import pytest

from zerollm_b200 import ggml, gguf, synth
from zerollm_b200.model import CudaModel
from zerollm_b200.prefix_cache import PrefixCache, kernel_flavour, model_fingerprint

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

PREFIX = [(i * 17 + 5) % 250 for i in range(21)]
REST = [9, 33, 120, 7]


def _file(tmp_path, seed=6):
    cfg = synth.tiny()
    w = synth.make_model(cfg, seed=seed, quant="q4_k_m", dist="tame", output_type=ggml.F16)
    p = str(tmp_path / "m.gguf")
    gguf.write_gguf(p, cfg, w)
    return cfg, w, p


def test_model_from_gguf_matches_memory(tmp_path):
    cfg, w, p = _file(tmp_path)
    cfg2, w2 = gguf.load_model(p)
    a = CudaModel.create(cfg, w, ctx=64, kv="f16", max_batch=32)
    b = CudaModel.create(cfg2, w2, ctx=64, kv="f16")
    la = a.forwardBatch(PREFIX[:8], logits="all").copy()
    lb = b.forwardBatch(PREFIX[:8], logits="all").copy()
    assert np.array_equal(la, lb)
    for t in REST:
        assert np.array_equal(a.forward(t), b.forward(t))
    a.close()
    b.close()


def test_prefix_cache_through_the_device(tmp_path):
    cfg, w, p = _file(tmp_path, seed=11)
    cfg, w = gguf.load_model(p)
    a = CudaModel.create(cfg, w, ctx=64, kv="f16", max_batch=32)
    cache = PrefixCache(str(tmp_path / "kv"), model_fingerprint(p, kernel_flavour(a)))
    a.forwardBatch(PREFIX, logits=False)
    cache.save(a, PREFIX)
    for t in REST:
        want = a.forward(t).copy()
    b = CudaModel.create(cfg, w, ctx=64, kv="f16", max_batch=32)
    assert cache.load(b, PREFIX)
    assert b.pos == len(PREFIX) and b.tokens == PREFIX
    for l in range(cfg["n_layer"]):
        for v in (0, 1):
            assert np.array_equal(b.kvGet(l, v, len(PREFIX)), a.kvGet(l, v, len(PREFIX)))
    for t in REST:
        got = b.forward(t)
    assert np.array_equal(got, want)
    # a damaged file: refused, the model stays fresh and usable
    f = cache.file(PREFIX)
    good = open(f, "rb").read()
    open(f, "wb").write(good[:-1])
    c = CudaModel.create(cfg, w, ctx=64, kv="f16", max_batch=32)
    assert not cache.load(c, PREFIX)
    assert c.pos == 0
    fresh = CudaModel.create(cfg, w, ctx=64, kv="f16", max_batch=32)
    assert np.array_equal(c.forward(5), fresh.forward(5))
    for m in (a, b, c, fresh):
        m.close()
