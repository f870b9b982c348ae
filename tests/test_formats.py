"""The on-disk formats either side of the hot path, on the CPU: the GGUF reader that feeds the
device uploads (src/gguf/reader.js) and the ZLLMKV01 prefix-cache file (src/model/prefix-cache.js).

* a model written as GGUF reads back with the same config and the same tensor bytes, and an
  independent parser (gguf-py, in the image) agrees on every tensor; a file gguf-py wrote reads
  back too;
* the oracle's forward pass over the weights read from the file equals the pass over the
  in-memory weights, bit for bit;
* the reader's errors: bad magic, unsupported version, a truncated file (reader.js:139-186);
* the prefix cache: round trip, its file layout, and every refusal of
  test/prefix-cache.test.js:50-80 (different tokens, model identity, a used model, an empty
  prefix, truncated / extended / bad-magic / garbage files, a tampered token list), plus prune.
"""
import hashlib
import json
import os
import struct

import numpy as np
import pytest

import oracle as O
from zerollm_b200 import ggml, gguf, synth
from zerollm_b200.prefix_cache import PrefixCache, kernel_flavour, model_fingerprint

PREFIX = [(i * 17 + 5) % 250 for i in range(21)]      # test/prefix-cache.test.js:16


def _model(quant="q4_k_m", seed=5, **kw):
    cfg = synth.tiny(**kw)
    return cfg, synth.make_model(cfg, seed=seed, quant=quant, dist="tame", output_type=ggml.F16)


def _mats(w):
    yield "token_embd.weight", w["tok_embd"]
    if w.get("output") is not None:
        yield "output.weight", w["output"]
    names = dict(gguf._LAYER_NAMES)
    for l, L in enumerate(w["layers"]):
        for k, v in L.items():
            if isinstance(v, dict):
                yield f"blk.{l}.{names[k]}", v


def test_gguf_round_trip(tmp_path):
    cfg, w = _model(qkv_bias=True)
    p = str(tmp_path / "m.gguf")
    gguf.write_gguf(p, cfg, w)
    g = gguf.read_gguf(p)
    assert g.version == 3 and g.alignment == 32 and g.data_start % 32 == 0
    c = gguf.model_config(g)
    for k in ("arch", "n_embd", "n_layer", "n_ff", "n_head", "n_head_kv", "head_dim", "n_rot", "vocab", "rope_type"):
        assert c[k] == cfg[k], k
    assert c["rms_eps"] == cfg["rms_eps"] and c["rope_base"] == cfg["rope_base"]
    assert c["qk_norm"] and c["qkv_bias"] and not c["tied"]
    cfg2, w2 = gguf.load_model(p)
    for name, t in _mats(w):
        info = g.require_tensor(name)
        assert (info.type, info.rows, info.cols) == (t["type"], t["rows"], t["cols"]), name
        assert info.abs_offset % 32 == 0
        assert np.array_equal(g.tensor_data(info), t["data"]), name
    for l in range(cfg["n_layer"]):
        for k in ("attn_norm", "ffn_norm", "q_norm", "k_norm", "bq", "bk", "bv"):
            assert np.array_equal(w2["layers"][l][k], w["layers"][l][k]), (l, k)
    assert np.array_equal(w2["output_norm"], w["output_norm"])


def test_gguf_py_agrees(tmp_path):
    gp = pytest.importorskip("gguf")
    cfg, w = _model()
    p = str(tmp_path / "m.gguf")
    gguf.write_gguf(p, cfg, w)
    r = gp.GGUFReader(p)
    theirs = {t.name: t for t in r.tensors}
    g = gguf.read_gguf(p)
    assert set(theirs) == {t.name for t in g.tensors}
    for t in g.tensors:
        o = theirs[t.name]
        assert int(o.tensor_type) == t.type and [int(d) for d in o.shape] == t.dims, t.name
        assert int(o.data_offset) == t.abs_offset, t.name
        assert np.array_equal(np.asarray(o.data).view(np.uint8).reshape(-1), g.tensor_data(t)), t.name
    assert str(bytes(r.fields["general.architecture"].parts[-1]), "utf-8") == "qwen3"

    # and a file gguf-py writes (a raw Q4_K matrix plus an f32 vector) reads back here
    q = str(tmp_path / "theirs.gguf")
    wr = gp.GGUFWriter(q, "qwen3")
    rng = np.random.default_rng(2)
    m = synth.tensor(ggml.Q4_K, 48, 512, rng, "bench")
    raw = m["data"].reshape(48, ggml.row_bytes(ggml.Q4_K, 512))
    wr.add_tensor("blk.0.attn_q.weight", raw, raw_dtype=gp.GGMLQuantizationType.Q4_K)
    vec = rng.standard_normal(512).astype(np.float32)
    wr.add_tensor("blk.0.attn_norm.weight", vec)
    wr.write_header_to_file()
    wr.write_kv_data_to_file()
    wr.write_tensors_to_file()
    wr.close()
    h = gguf.read_gguf(q)
    t = h.require_tensor("blk.0.attn_q.weight")
    assert (t.type, t.rows, t.cols) == (ggml.Q4_K, 48, 512)
    assert np.array_equal(h.tensor_data(t), m["data"])
    assert np.array_equal(gguf._vector(h, h.require_tensor("blk.0.attn_norm.weight")), vec)
    assert h.get("general.architecture") == "qwen3"


def test_oracle_over_file_weights_is_identical(tmp_path):
    cfg, w = _model(seed=8)
    p = str(tmp_path / "m.gguf")
    gguf.write_gguf(p, cfg, w)
    cfg2, w2 = gguf.load_model(p)
    a = O.OracleModel(cfg, w, ctx=32, kv_f16=True)
    b = O.OracleModel(cfg2, w2, ctx=32, kv_f16=True)
    for t in (3, 17, 42, 5):
        assert np.array_equal(a.forward(t), b.forward(t))


def test_gguf_errors(tmp_path):
    cfg, w = _model()
    p = str(tmp_path / "m.gguf")
    gguf.write_gguf(p, cfg, w)
    good = open(p, "rb").read()
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"GGUX" + good[4:])
    with pytest.raises(ValueError, match="not a GGUF file"):
        gguf.read_gguf(str(bad))
    bad.write_bytes(good[:4] + struct.pack("<I", 4) + good[8:])
    with pytest.raises(ValueError, match="unsupported GGUF version 4"):
        gguf.read_gguf(str(bad))
    bad.write_bytes(good[:-100])
    with pytest.raises(ValueError, match="extends past end of file"):
        gguf.read_gguf(str(bad))
    bad.write_bytes(good[:40])
    with pytest.raises(ValueError, match="unexpected end of file"):
        gguf.read_gguf(str(bad))


# ------------------------------------------------------------------------------ prefix cache
class _KvModel:
    """The model surface PrefixCache drives (pos, cfg, kvGet / kvSet, restorePrefix), over a
    numpy KV store."""

    def __init__(self, cfg, ctx=64, seed=None):
        self.cfg, self.kernels, self.kv = cfg, "cuda", "f16"
        kv_dim = cfg["n_head_kv"] * cfg["head_dim"]
        self.store = np.zeros((cfg["n_layer"], 2, ctx, kv_dim), np.float32)
        self.tokens = []
        if seed is not None:
            self.store[:] = np.random.default_rng(seed).standard_normal(self.store.shape)

    @property
    def pos(self):
        return len(self.tokens)

    def kvGet(self, layer, isV, n):
        return self.store[layer, isV, :n].reshape(-1).copy()

    def kvSet(self, layer, isV, n, data):
        self.store[layer, isV, :n] = np.asarray(data, np.float32).reshape(n, -1)

    def restorePrefix(self, ids):
        self.tokens = list(ids)


def test_prefix_cache_round_trip_and_layout(tmp_path):
    cfg = synth.tiny()
    src = _KvModel(cfg, seed=1)
    src.tokens = PREFIX + [9, 33]
    fp = "m.gguf|123|456|" + kernel_flavour(src)
    assert fp.endswith("cuda/kv-f16")
    cache = PrefixCache(str(tmp_path), fp)
    path = cache.save(src, PREFIX)
    want = hashlib.sha1(fp.encode() + b"\n" + np.asarray(PREFIX, "<i4").tobytes()).hexdigest()
    assert os.path.basename(path) == want + ".kv"
    raw = open(path, "rb").read()
    assert raw[:8] == b"ZLLMKV01"
    hlen = struct.unpack_from("<I", raw, 8)[0]
    h = json.loads(raw[12:12 + hlen])
    kv_dim, n = cfg["n_head_kv"] * cfg["head_dim"], len(PREFIX)
    assert h == {"fingerprint": fp, "nLayer": cfg["n_layer"], "kvDim": kv_dim, "n": n, "tokens": PREFIX}
    body = np.frombuffer(raw[12 + hlen:], "<f4").reshape(cfg["n_layer"], 2, n, kv_dim)
    assert np.array_equal(body, src.store[:, :, :n])           # per layer K then V, f32 LE
    dst = _KvModel(cfg)
    assert cache.load(dst, PREFIX)
    assert dst.pos == n and dst.tokens == PREFIX
    assert np.array_equal(dst.store[:, :, :n], src.store[:, :, :n])
    assert not dst.store[:, :, n:].any()


def test_prefix_cache_refuses_mismatches_and_damage(tmp_path):
    cfg = synth.tiny()
    src = _KvModel(cfg, seed=2)
    src.tokens = list(PREFIX)
    fp = "m.gguf|1|2|cuda/kv-f16"
    cache = PrefixCache(str(tmp_path), fp)
    file = cache.save(src, PREFIX)
    fresh = lambda: _KvModel(cfg)                                    # noqa: E731
    assert cache.load(fresh(), PREFIX)
    assert not cache.load(fresh(), PREFIX[:-1] + [99])               # different tokens -> no file
    assert not PrefixCache(str(tmp_path), fp + "x").load(fresh(), PREFIX)
    used = fresh()
    used.tokens = [1, 2]
    assert not cache.load(used, PREFIX)                              # only into a fresh model
    assert not cache.load(fresh(), [])
    good = open(file, "rb").read()
    hlen = struct.unpack_from("<I", good, 8)[0]
    head = json.loads(good[12:12 + hlen])
    head["tokens"][3] = 249
    nh = json.dumps(head).encode()
    cases = [good[:-7], good + bytes([1, 2, 3]), b"NOTACACH" + good[8:], b"garbage",
             good[:8] + struct.pack("<I", len(nh)) + nh + good[12 + hlen:]]
    for bad in cases:
        open(file, "wb").write(bad)
        m = fresh()
        assert not cache.load(m, PREFIX)
        assert m.pos == 0 and not m.store.any()                      # nothing was written
    other = dict(cfg, n_layer=cfg["n_layer"] + 1)
    open(file, "wb").write(good)
    assert not cache.load(_KvModel(other), PREFIX)                   # a different layer count


def test_prefix_cache_prune_and_fingerprint(tmp_path):
    cfg = synth.tiny()
    src = _KvModel(cfg, seed=3)
    src.tokens = list(range(40))
    cache = PrefixCache(str(tmp_path), "fp")
    for i in range(20):
        p = cache.save(src, list(range(i + 1)))
        os.utime(p, (1000 + i, 1000 + i))
    cache.prune(16)
    left = sorted(os.listdir(tmp_path))
    assert len(left) == 16
    assert os.path.basename(cache.file(list(range(20)))) in left
    assert os.path.basename(cache.file([0])) not in left
    mp = tmp_path / "model.gguf"
    mp.write_bytes(b"x" * 10)
    fp = model_fingerprint(str(mp), "cuda/kv-f16")
    assert fp.startswith("model.gguf|10|") and fp.endswith("|cuda/kv-f16")


def test_gguf_llama_tied_and_missing_keys(tmp_path):
    cfg = synth.tiny(arch="llama", qk_norm=False, tied=True)
    w = synth.make_model(cfg, seed=3, quant="q8_0", dist="tame")
    p = str(tmp_path / "llama.gguf")
    gguf.write_gguf(p, cfg, w)
    c, w2 = gguf.load_model(p)
    assert c["arch"] == "llama" and c["rope_type"] == "norm"       # config.js: llama -> 'norm', others 'neox'
    assert c["tied"] and w2["output"] is None and not c["qk_norm"]
    assert w2["layers"][0]["q_norm"] is None and w2["layers"][0]["wq"]["type"] == ggml.Q8_0
    g = gguf.read_gguf(p)
    del g.metadata["llama.block_count"]
    with pytest.raises(ValueError, match="missing metadata key llama.block_count"):
        gguf.model_config(g)
    g.metadata["general.architecture"] = "mamba"
    with pytest.raises(ValueError, match='architecture "mamba" is not supported'):
        gguf.model_config(g)
