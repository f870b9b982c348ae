"""Tensor-parallel sharding (zerollm_b200.tp), checked on the CPU with the oracle: the column-parallel
shards' outputs concatenate to the full projection, the row-parallel shards' partial sums add up
to it, and every shard is a valid GGUF matrix (cut at whole blocks)."""
import numpy as np
import pytest

import oracle as O
from zerollm_b200 import ggml, synth
from zerollm_b200.tp import ffn_ranges, ranges, shard_cols, shard_model, shard_rows


def test_ranges_cover_evenly():
    for n, size in ((100, 8), (100, 3), (8, 8), (5, 2)):
        rs = ranges(n, size)
        assert rs[0][0] == 0 and rs[-1][1] == n
        assert all(a1 == b0 for (_, a1), (b0, _) in zip(rs, rs[1:]))
        assert max(b - a for a, b in rs) - min(b - a for a, b in rs) <= 1


@pytest.mark.parametrize("size", [2, 4])
def test_shards_reassemble_the_projections(size):
    cfg = synth.tiny(n_embd=256, n_ff=1024, n_head=16, n_head_kv=4, head_dim=64)
    w = synth.make_model(cfg, seed=2, quant="q4_k_q6", dist="tame")
    L = w["layers"][0]
    E, F = cfg["n_embd"], cfg["n_ff"]
    rng = np.random.default_rng(0)
    x = rng.standard_normal(E).astype(np.float32)
    h = rng.standard_normal(F).astype(np.float32)
    full_gate = O.matvec(L["gate"]["type"], L["gate"]["data"], F, E, x)
    full_down = O.matvec(L["down"]["type"], L["down"]["data"], E, F, h)
    fr = ffn_ranges(cfg, w, size)
    assert all(a % 256 == 0 and b % 256 == 0 for a, b in fr)
    parts_gate, parts_down = [], np.zeros(E)
    for r in range(size):
        lc, lw = shard_model(cfg, w, r, size)
        M = lw["layers"][0]
        assert lc["n_head"] == cfg["n_head"] // size and lc["n_ff"] == fr[r][1] - fr[r][0]
        parts_gate.append(O.matvec(M["gate"]["type"], M["gate"]["data"], lc["n_ff"], E, x))
        parts_down += O.matvec(M["down"]["type"], M["down"]["data"], E, lc["n_ff"], h[fr[r][0]:fr[r][1]]).astype(np.float64)
    assert np.array_equal(np.concatenate(parts_gate), full_gate)          # column-parallel: the same rows
    # row-parallel: each shard's blocks are the full row's blocks; only the order of the f64 sum moves
    assert np.abs(parts_down - full_down).max() <= 1e-5 * np.abs(full_down).max()


def test_shard_cuts_whole_blocks():
    rng = np.random.default_rng(1)
    t = synth.tensor(ggml.Q6_K, 8, 1024, rng, "bench")
    s = shard_cols(t, 256, 768)
    assert s["cols"] == 512 and s["data"].size == 8 * ggml.row_bytes(ggml.Q6_K, 512)
    with pytest.raises(ValueError):
        shard_cols(t, 100, 356)
    assert shard_rows(t, 2, 5)["data"].size == 3 * ggml.row_bytes(ggml.Q6_K, 1024)


@pytest.mark.parametrize("size", [2, 4])
def test_output_head_splits_by_vocab_rows(size):
    """The output head goes out by vocab rows, rank r holding [r V / size, (r + 1) V / size): the
    slices' logits, in rank order, are the full head's logits bit for bit."""
    cfg = synth.tiny(n_embd=256, n_ff=1024, n_head=16, n_head_kv=4, head_dim=64, vocab=321)
    w = synth.make_model(cfg, seed=5, quant="q4_k_m", dist="tame", output_type=ggml.F16)
    V, E = cfg["vocab"], cfg["n_embd"]
    x = np.random.default_rng(2).standard_normal(E).astype(np.float32)
    full = O.matvec(w["output"]["type"], w["output"]["data"], V, E, x)
    parts = []
    for r in range(size):
        lc, lw = shard_model(cfg, w, r, size)
        v0, n = lc["vocab_shard"]
        assert (v0, v0 + n) == (r * V // size, (r + 1) * V // size) and lc["vocab"] == V
        parts.append(O.matvec(lw["output"]["type"], lw["output"]["data"], n, E, x))
    assert np.array_equal(np.concatenate(parts), full)
    tied = dict(w, output=None)
    lc, lw = shard_model(cfg, tied, 0, size)
    assert "vocab_shard" not in lc and lw["output"] is None
