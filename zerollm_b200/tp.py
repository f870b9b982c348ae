"""Tensor-parallel sharding of a model's weights over GPUs (one process and one CudaModel per GPU).

The reference runs a model in one process (its worker pool splits KV heads across threads,
src/compute/worker.js:123, :296-337, but every thread holds every weight); BASELINE config 4 shards
a model too large for one GPU the Megatron way:

* q / k / v and gate / up are column-parallel: rank r keeps its query heads
  [r*H/T, (r+1)*H/T), the matching KV heads [r*KV/T, ...) (so grouped-query attention stays local)
  and its range of FFN units;
* attn_output and ffn_down are row-parallel: rank r keeps the matching input columns (cut at whole
  quantization blocks, so every shard is itself a valid GGUF matrix) and produces a partial sum,
  which the ranks add with one NCCL all-reduce after each (zllm_model_set_tp);
* the output head is split by vocab rows (rank r: rows [r*V/T, (r+1)*V/T)); every pass gathers
  the ranks' logits slices, so every rank ends a pass with the same full logits and the same greedy
  token; a head tied to the token embedding stays replicated;
* norms and the token embedding are replicated.
"""
from __future__ import annotations

import numpy as np

from . import ggml


def ranges(n_units: int, size: int) -> list[tuple[int, int]]:
    """An even split of n_units over `size` ranks: [(start, end)] in units."""
    return [(r * n_units // size, (r + 1) * n_units // size) for r in range(size)]


def _block(t: int) -> tuple[int, int]:
    name, bs, ts = ggml.TYPE_INFO[t]
    return bs, ts


def shard_rows(t: dict, r0: int, r1: int) -> dict:
    """Rows [r0, r1) of a raw matrix."""
    rb = ggml.row_bytes(t["type"], t["cols"])
    data = np.asarray(t["data"], np.uint8).reshape(t["rows"], rb)[r0:r1]
    return {"type": t["type"], "rows": r1 - r0, "cols": t["cols"], "data": np.ascontiguousarray(data).reshape(-1)}


def shard_cols(t: dict, c0: int, c1: int) -> dict:
    """Input columns [c0, c1) of every row of a raw matrix; c0 and c1 on quantization-block bounds."""
    bs, ts = _block(t["type"])
    if c0 % bs or c1 % bs:
        raise ValueError(f"column cut {c0}:{c1} is not on a {bs}-value block boundary")
    rb = ggml.row_bytes(t["type"], t["cols"])
    data = np.asarray(t["data"], np.uint8).reshape(t["rows"], rb)[:, c0 // bs * ts:c1 // bs * ts]
    return {"type": t["type"], "rows": t["rows"], "cols": c1 - c0, "data": np.ascontiguousarray(data).reshape(-1)}


def ffn_ranges(cfg: dict, weights: dict, size: int) -> list[tuple[int, int]]:
    """Each rank's FFN units, cut at the ffn_down blocks (256 values for the k-quants)."""
    unit = max(_block(L["down"]["type"])[0] for L in weights["layers"])
    F = cfg["n_ff"]
    if F % unit:
        raise ValueError(f"n_ff {F} is not a whole number of {unit}-value blocks")
    return [(a * unit, b * unit) for a, b in ranges(F // unit, size)]


def shard_model(cfg: dict, weights: dict, rank: int, size: int) -> tuple[dict, dict]:
    """(local config, local weights) of rank `rank` of `size`."""
    H, KV, hd = cfg["n_head"], cfg["n_head_kv"], cfg["head_dim"]
    if H % size or KV % size:
        raise ValueError(f"{H} query / {KV} KV heads do not split over {size} ranks")
    Hl, KVl = H // size, KV // size
    q0, q1 = rank * Hl * hd, (rank + 1) * Hl * hd
    k0, k1 = rank * KVl * hd, (rank + 1) * KVl * hd
    f0, f1 = ffn_ranges(cfg, weights, size)[rank]
    lc = dict(cfg, n_head=Hl, n_head_kv=KVl, n_ff=f1 - f0)
    lw = {k: v for k, v in weights.items() if k != "layers"}
    if weights.get("output") is not None:
        v0, v1 = ranges(weights["output"]["rows"], size)[rank]
        lw["output"] = shard_rows(weights["output"], v0, v1)
        lc["vocab_shard"] = (v0, v1 - v0)
    layers = []
    for L in weights["layers"]:
        M = dict(L)
        M["wq"], M["wk"], M["wv"] = shard_rows(L["wq"], q0, q1), shard_rows(L["wk"], k0, k1), shard_rows(L["wv"], k0, k1)
        M["wo"] = shard_cols(L["wo"], q0, q1)
        M["gate"], M["up"] = shard_rows(L["gate"], f0, f1), shard_rows(L["up"], f0, f1)
        M["down"] = shard_cols(L["down"], f0, f1)
        for b, (a0, a1) in (("bq", (q0, q1)), ("bk", (k0, k1)), ("bv", (k0, k1))):
            if L.get(b) is not None:
                M[b] = np.ascontiguousarray(L[b][a0:a1])
        layers.append(M)
    lw["layers"] = layers
    return lc, lw
