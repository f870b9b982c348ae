#!/usr/bin/env python3
"""Regenerate the golden fixtures in tests/golden/ (run in the build container, not on the GPU box).

1. ``ref_quant_vectors.json`` -- the reference's own golden dequantization vectors
   (zerollm ``test/data/quant-vectors.json``: Q5_0 / Q4_K / Q5_K / Q6_K, 6 rows, random plus
   extreme blocks, produced by gguf-py), copied byte for byte from the reference checkout
   when it is present.  It is test data, not source.
2. ``ggufpy_vectors.npz`` -- fresh vectors minted here with the same independent
   implementation (gguf-py, ``gguf.quants.dequantize``; version recorded in the file) for
   every type on the hot path (Q4_0, Q5_0, Q8_0, Q4_K, Q5_K, Q6_K, F16, BF16), in two
   flavours: raw random bytes with odd / extreme f16 scales (NaN, inf, denormals, 0xFF and
   all-zero blocks), and the benchmark distribution of the k-quant configs (nibbles uniform,
   6-bit scales and mins uniform, d = f16(|N(0,1)| * 0.01); Q6_K sub-block scales uniform in
   [-32, 31]).

Usage:  python tests/golden/make_golden.py [--reference /path/to/zerollm]
"""
import argparse
import os
import shutil

import numpy as np
import gguf
from gguf import GGMLQuantizationType as Q
from gguf import quants

HERE = os.path.dirname(os.path.abspath(__file__))
TYPES = {"Q4_0": Q.Q4_0, "Q5_0": Q.Q5_0, "Q8_0": Q.Q8_0, "Q4_K": Q.Q4_K, "Q5_K": Q.Q5_K,
         "Q6_K": Q.Q6_K, "F16": Q.F16, "BF16": Q.BF16}
ODD_F16 = np.array([0.0, 1.0, -1.0, 0.0123, -0.0456, 2.0 ** -24, -(2.0 ** -24), 2.0 ** -14, 3.5,
                    0.00031, -7.25, 60000.0, np.inf, -np.inf, np.nan], dtype=np.float16)


def f16b(v):
    return np.frombuffer(np.array([v], dtype=np.float16).tobytes(), dtype=np.uint8)


def scale_offsets(name):
    """byte offsets of the f16 scale fields inside one block"""
    return {"Q4_0": [0], "Q5_0": [0], "Q8_0": [0], "Q4_K": [0, 2], "Q5_K": [0, 2], "Q6_K": [208]}.get(name, [])


def raw_blocks(rng, name, n_blocks):
    bs, ts = gguf.GGML_QUANT_SIZES[TYPES[name]]
    raw = rng.integers(0, 256, size=(n_blocks, ts), dtype=np.uint8)
    if name in ("F16", "BF16"):
        return raw
    for b in range(n_blocks):
        for off in scale_offsets(name):
            raw[b, off:off + 2] = f16b(ODD_F16[rng.integers(0, len(ODD_F16))])
    raw[1, :] = 0                         # all-zero block
    raw[2, :] = 0xFF                      # all-ones block (NaN scales)
    if n_blocks > 3:
        raw[3, 2:] = 0xFF                 # extreme quants, finite first scale
        for off in scale_offsets(name):
            raw[3, off:off + 2] = f16b(0.5)
    return raw


def bench_blocks(rng, name, n_blocks):
    """the BASELINE configs' weight distribution"""
    bs, ts = gguf.GGML_QUANT_SIZES[TYPES[name]]
    raw = rng.integers(0, 256, size=(n_blocks, ts), dtype=np.uint8)
    d = lambda: f16b(np.float16(abs(rng.standard_normal()) * 0.01))
    for b in range(n_blocks):
        if name in ("Q4_K", "Q5_K"):
            raw[b, 0:2] = d(); raw[b, 2:4] = d()
        elif name == "Q6_K":
            raw[b, 192:208] = rng.integers(-32, 32, size=16).astype(np.int8).view(np.uint8)
            raw[b, 208:210] = d()
        elif name in ("Q4_0", "Q5_0", "Q8_0"):
            raw[b, 0:2] = d()
        elif name == "F16":
            raw[b] = np.frombuffer((rng.standard_normal(ts // 2) * 0.02).astype(np.float16).tobytes(), np.uint8)
        elif name == "BF16":
            f = (rng.standard_normal(ts // 2) * 0.02).astype(np.float32)
            raw[b] = np.frombuffer((f.view(np.uint32) >> 16).astype(np.uint16).tobytes(), np.uint8)
    return raw


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("ZLLM_REFERENCE"),
                    help="checkout of the reference repository (its test/data/quant-vectors.json is copied)")
    args = ap.parse_args()
    src = os.path.join(args.reference, "test", "data", "quant-vectors.json") if args.reference else ""
    if src and os.path.exists(src):
        shutil.copyfile(src, os.path.join(HERE, "ref_quant_vectors.json"))
        print("copied", src)
    rng = np.random.default_rng(20261201)
    out = {"gguf_version": np.array(getattr(gguf, "__version__", "0.19.0"))}
    for name, qt in TYPES.items():
        bs, ts = gguf.GGML_QUANT_SIZES[qt]
        blocks_per_row = 4 if bs == 256 else (8 if bs == 32 else 256)
        rows = 6
        for flavour, gen in (("raw", raw_blocks), ("bench", bench_blocks)):
            raw = gen(rng, name, rows * blocks_per_row).reshape(rows, blocks_per_row * ts)
            with np.errstate(all="ignore"):
                deq = quants.dequantize(raw, qt).astype(np.float32)
            out[f"{name}.{flavour}.raw"] = raw
            out[f"{name}.{flavour}.expected"] = deq
    np.savez_compressed(os.path.join(HERE, "ggufpy_vectors.npz"), **out)
    print("wrote ggufpy_vectors.npz", len(out), "arrays")


if __name__ == "__main__":
    main()
