"""Seeded synthetic weights and activations in raw GGUF block layout.

Two weight distributions:

* ``"bench"`` -- the benchmark configs' distribution: k-quant nibbles / 6-bit quants uniform,
  Q4_K/Q5_K 6-bit scales and mins uniform in [0, 63], Q6_K int8 sub-block scales uniform in
  [-32, 31], every f16 super-block scale ``d`` (and ``dmin``) = f16(|N(0,1)| * 0.01).
* ``"tame"`` -- the reference's test-model recipe (tools/random-blocks.js:20-37): random raw
  blocks whose f16 scales make dequantized weights small and centred (Q4_K d = 2.5e-4 * U[0.5,1.5),
  dmin = 7.5 d; Q5_K 1.3e-4 / 15.5; Q6_K 2e-5; Q5_0 0.004), so tiny random networks stay
  well conditioned.

All randomness comes from ``numpy.random.default_rng(seed)``; the seed is part of every
benchmark and test configuration.
"""
from __future__ import annotations

import numpy as np

from . import ggml

TAME = {ggml.Q5_0: (0.004, None), ggml.Q4_K: (2.5e-4, 7.5), ggml.Q5_K: (1.3e-4, 15.5), ggml.Q6_K: (2e-5, None),
        ggml.Q8_0: (4e-4, None), ggml.Q4_0: (6e-3, None)}


def f16_bits(v) -> np.ndarray:
    return np.asarray(v, dtype=np.float32).astype(np.float16).view(np.uint16)


def _scale_field(vals) -> np.ndarray:
    """f16 bytes of a vector of scales, shape (n, 2)"""
    return f16_bits(vals).reshape(-1, 1).view(np.uint8).reshape(-1, 2)


def quant_blocks(t: int, rows: int, cols: int, rng: np.random.Generator, dist: str = "bench") -> np.ndarray:
    """rows x row_bytes uint8 array of raw ggml blocks of type ``t``."""
    name, bs, ts = ggml.TYPE_INFO[t]
    rb = ggml.row_bytes(t, cols)
    nblk = rows * (cols // bs)
    raw = rng.integers(0, 256, size=(nblk, ts), dtype=np.uint8)
    if dist == "bench":
        d = np.abs(rng.standard_normal(nblk)) * 0.01
        if t in (ggml.Q4_K, ggml.Q5_K):
            raw[:, 0:2] = _scale_field(d)
            raw[:, 2:4] = _scale_field(np.abs(rng.standard_normal(nblk)) * 0.01)
        elif t == ggml.Q6_K:
            raw[:, 192:208] = rng.integers(-32, 32, size=(nblk, 16)).astype(np.int8).view(np.uint8)
            raw[:, 208:210] = _scale_field(d)
        else:
            raw[:, 0:2] = _scale_field(d)
    elif dist == "tame":
        base, dmin_ratio = TAME[t]
        d = base * (0.5 + rng.random(nblk))
        if t == ggml.Q6_K:
            raw[:, 208:210] = _scale_field(d)
        else:
            raw[:, 0:2] = _scale_field(d)
            if dmin_ratio is not None:
                raw[:, 2:4] = _scale_field(d * dmin_ratio)
    else:
        raise ValueError(dist)
    return raw.reshape(rows, rb)


def float_tensor(t: int, rows: int, cols: int, rng: np.random.Generator, std: float) -> np.ndarray:
    """rows x row_bytes uint8 of an F32 / F16 / BF16 matrix with N(0, std) entries."""
    f = (rng.standard_normal((rows, cols)) * std).astype(np.float32)
    if t == ggml.F32:
        return f.view(np.uint8).reshape(rows, cols * 4)
    if t == ggml.F16:
        return f.astype(np.float16).view(np.uint8).reshape(rows, cols * 2)
    if t == ggml.BF16:
        return (f.view(np.uint32) >> 16).astype(np.uint16).view(np.uint8).reshape(rows, cols * 2)
    raise ValueError(t)


def tensor(t: int, rows: int, cols: int, rng: np.random.Generator, dist: str = "bench", std: float = 0.02) -> dict:
    data = quant_blocks(t, rows, cols, rng, dist) if t in ggml.QUANTIZED else float_tensor(t, rows, cols, rng, std)
    return {"type": t, "rows": rows, "cols": cols, "data": np.ascontiguousarray(data).reshape(-1)}


# ------------------------------------------------------------------------------------- models
def qwen3_config(n_embd, n_layer, n_ff, n_head, n_head_kv, head_dim, vocab, **kw) -> dict:
    c = dict(arch="qwen3", n_embd=n_embd, n_layer=n_layer, n_ff=n_ff, n_head=n_head, n_head_kv=n_head_kv,
             head_dim=head_dim, n_rot=head_dim, vocab=vocab, rms_eps=float(np.float32(1e-6)),
             rope_base=1e6, rope_type="neox", qk_norm=True, qkv_bias=False, tied=False)
    c.update(kw)
    return c


def qwen3_8b() -> dict:
    """Qwen3-8B shapes (config 3)."""
    return qwen3_config(4096, 36, 12288, 32, 8, 128, 151936)


def qwen3_32b() -> dict:
    """Qwen3-32B shapes (config 4)."""
    return qwen3_config(5120, 64, 25600, 64, 8, 128, 151936)


def tiny(**kw) -> dict:
    """A small qwen3-shaped config for oracle-speed parity tests."""
    base = dict(n_embd=256, n_layer=2, n_ff=512, n_head=4, n_head_kv=2, head_dim=64, vocab=320)
    base.update({k: v for k, v in kw.items() if k in base})
    rest = {k: v for k, v in kw.items() if k not in base}
    return qwen3_config(**base, **rest)


def layer_type(name: str, quant: str) -> int:
    """Per-tensor type.  'q4_k_m' follows the Q4_K_M mix of the reference's tiny-model tool
    (tools/make-tiny-gguf.js:70-71): Q6_K for attn_v / ffn_down / output, Q4_K for the rest."""
    if quant == "q4_k_m":
        return ggml.Q6_K if name in ("wv", "down", "output") else ggml.Q4_K
    if quant == "q4_k_q6":
        # the benchmark mix: Q4_K everywhere except ffn_down (Q6_K)
        return ggml.Q6_K if name == "down" else ggml.Q4_K
    return {"q4_k": ggml.Q4_K, "q5_k": ggml.Q5_K, "q6_k": ggml.Q6_K, "q8_0": ggml.Q8_0, "q4_0": ggml.Q4_0,
            "q5_0": ggml.Q5_0, "f16": ggml.F16, "bf16": ggml.BF16, "f32": ggml.F32}[quant]


def make_model(cfg: dict, seed: int = 1, quant: str = "q4_k_m", dist: str = "tame", output_type: int | None = None,
               embd_type: int | None = None, norm_std: float = 0.05, std: float = 0.05) -> dict:
    """Weights of a random-init model of ``cfg`` (raw GGUF bytes per matrix, f32 vectors)."""
    rng = np.random.default_rng(seed)
    E, F, H, KV, hd, V = cfg["n_embd"], cfg["n_ff"], cfg["n_head"], cfg["n_head_kv"], cfg["head_dim"], cfg["vocab"]
    q_dim, kv_dim = H * hd, KV * hd

    def mat(name, rows, cols, t=None):
        t = layer_type(name, quant) if t is None else t
        if cols % ggml.TYPE_INFO[t][1]:
            t = ggml.F32          # rows that are not whole blocks fall back to F32 (make-tiny-gguf.js:69-71)
        return tensor(t, rows, cols, rng, dist, std)

    def vec(n):
        return (1 + rng.standard_normal(n) * norm_std).astype(np.float32)

    w = {"tok_embd": mat("tok_embd", V, E, embd_type), "output_norm": vec(E), "rope_freqs": None}
    w["output"] = None if cfg.get("tied") else mat("output", V, E, output_type)
    layers = []
    for _ in range(cfg["n_layer"]):
        L = {"attn_norm": vec(E), "wq": mat("wq", q_dim, E), "wk": mat("wk", kv_dim, E), "wv": mat("wv", kv_dim, E),
             "wo": mat("wo", E, q_dim), "ffn_norm": vec(E), "gate": mat("gate", F, E), "up": mat("up", F, E),
             "down": mat("down", E, F)}
        if cfg.get("qk_norm"):
            L["q_norm"], L["k_norm"] = vec(hd), vec(hd)
        if cfg.get("qkv_bias"):
            L["bq"] = (rng.standard_normal(q_dim) * 0.02).astype(np.float32)
            L["bk"] = (rng.standard_normal(kv_dim) * 0.02).astype(np.float32)
            L["bv"] = (rng.standard_normal(kv_dim) * 0.02).astype(np.float32)
        layers.append(L)
    w["layers"] = layers
    return w
