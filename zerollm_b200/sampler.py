"""Token sampling with the candidate selection on the device (src/sampling/sampler.js).

``createSampler`` (sampler.js:86-155) applies the repetition / frequency / presence penalties,
keeps the top-k logits (topKSelect, :20-42), takes a softmax with temperature over them, cuts to
min-p then top-p, and draws with a seeded mulberry32 (src/util/rng.js:4-13).  Here the O(vocab)
part -- the penalties and the top-k selection -- runs on the GPU over the logits the last pass left
on the device (``zllm_model_topk``), and only the k (id, value) pairs come back; the softmax, cuts
and draw over those k values run here in doubles in the reference's order, so a seeded sampler
draws the tokens the reference's sampler would (up to the last bit of the host's ``exp``).

Greedy sampling (temperature <= 0) is the k = 1 case: the largest logit after the penalties,
the first on ties.  A top-k of 0 or above 256 (the reference then sorts the whole vocabulary)
is not offered on the device: ``Sampler`` raises for it.
"""
from __future__ import annotations

import ctypes as C
import math
import time
from dataclasses import dataclass

import numpy as np

from .lib import ZllmError

MAX_TOP_K = 256             # kTopkMax of the device selection
MAX_PENALISED = 4096        # kTopkMaxPen


def mulberry32(seed: int):
    """The reference's seeded uniform generator (src/util/rng.js:4-13; mulberry32 by Tommy
    Ettinger), in 32-bit unsigned arithmetic: returns a function giving floats in [0, 1)."""
    M = 0xFFFFFFFF
    state = [seed & M]

    def imul(a, b):
        return (a * b) & M

    def rand() -> float:
        state[0] = (state[0] + 0x6D2B79F5) & M
        t = state[0]
        t = imul(t ^ (t >> 15), t | 1)
        t = (t ^ ((t + imul(t ^ (t >> 7), t | 61)) & M)) & M
        return ((t ^ (t >> 14)) & M) / 4294967296.0

    return rand


@dataclass
class TokenDist:
    """The distribution a draw uses (sampler.js:51-61): ``ids[i]`` with weight ``probs[i] / total``."""
    ids: np.ndarray
    probs: np.ndarray
    total: float
    greedy: bool


class Sampler:
    """``createSampler(o)`` (sampler.js:86-155) with its defaults."""

    def __init__(self, temperature=0.8, top_k=40, top_p=0.95, min_p=0.0, repeat_penalty=1.0, repeat_last_n=64,
                 presence_penalty=0.0, frequency_penalty=0.0, seed=None):
        self.temperature, self.top_k, self.top_p, self.min_p = float(temperature), int(top_k), float(top_p), float(min_p)
        self.repeat_penalty, self.repeat_last_n = float(repeat_penalty), int(repeat_last_n)
        self.presence, self.frequency = float(presence_penalty), float(frequency_penalty)
        if seed is None:
            seed = (int(time.time() * 1000) ^ int(np.random.default_rng().integers(0, 2 ** 32))) & 0xFFFFFFFF
        self.rand = mulberry32(int(seed))
        self.greedy = self.temperature <= 0
        self.uses_history = self.repeat_penalty != 1 or self.presence != 0 or self.frequency != 0

    def penalised(self, history):
        """The distinct tokens of the last ``repeat_last_n`` of ``history`` with their counts, in
        order of first appearance (sampler.js:100-101)."""
        if not self.uses_history or not history:
            return [], []
        counts = {}
        for t in history[max(0, len(history) - self.repeat_last_n):]:
            counts[int(t)] = counts.get(int(t), 0) + 1
        return list(counts), list(counts.values())

    def candidates(self, model, history=(), rows: int = 1, k: int | None = None):
        """The k best (ids, values) of the last pass's first ``rows`` logits rows, after the
        penalties, selected on the device.  ids [rows][k] int32 (-1 past a row's finite values),
        values [rows][k] float32."""
        k = (1 if self.greedy else self.top_k) if k is None else int(k)
        if k <= 0 or k > MAX_TOP_K:
            raise ValueError(f"top-k of {k}: the device selection keeps 1..{MAX_TOP_K} candidates")
        toks, cnts = self.penalised(list(history))
        if len(toks) > MAX_PENALISED:
            raise ValueError(f"{len(toks)} penalised tokens (max {MAX_PENALISED})")
        pt = np.asarray(toks, np.int32)
        pc = np.asarray(cnts, np.int32)
        ids = np.empty((rows, k), np.int32)
        vals = np.empty((rows, k), np.float32)
        model._guard()
        lib = model.lib
        rc = lib.zllm_model_topk(model.h, int(rows), k, pt.ctypes.data_as(C.c_void_p) if pt.size else None,
                                 pc.ctypes.data_as(C.c_void_p) if pc.size else None, int(pt.size), self.repeat_penalty,
                                 self.frequency, self.presence, ids.ctypes.data_as(C.c_void_p),
                                 vals.ctypes.data_as(C.c_void_p))
        if rc:
            raise ZllmError(rc, lib.zllm_last_error(model.context.h).decode())
        return ids, vals

    def from_candidates(self, ids, vals) -> TokenDist:
        """Softmax with temperature, min-p, top-p over candidates sorted by value (sampler.js:116-137)."""
        keep_valid = np.asarray(ids) >= 0
        ids = np.asarray(ids, np.int32)[keep_valid]
        vals = [float(v) for v in np.asarray(vals, np.float32)[keep_valid]]
        if self.greedy:
            return TokenDist(ids[:1].copy(), np.ones(1), 1.0, True)
        n = len(vals)
        mx = vals[0]
        probs = [math.exp((v - mx) / self.temperature) for v in vals]
        s = 0.0
        for p in probs:
            s += p
        probs = [p / s for p in probs]
        keep = n
        if self.min_p > 0:
            thr = self.min_p * probs[0]
            keep = 1
            while keep < n and probs[keep] >= thr:
                keep += 1
        if self.top_p < 1:
            c, i = 0.0, 0
            while i < keep:
                c += probs[i]
                i += 1
                if c >= self.top_p:
                    break
            keep = max(1, i)
        total = 0.0
        for p in probs[:keep]:
            total += p
        return TokenDist(ids[:keep].copy(), np.asarray(probs[:keep], np.float64), total, False)

    def distribution(self, model, history=(), row: int = 0) -> TokenDist:
        """The distribution of logits row ``row`` of the last pass (no random number consumed)."""
        ids, vals = self.candidates(model, history, rows=row + 1)
        return self.from_candidates(ids[row], vals[row])

    def draw(self, d: TokenDist) -> int:
        """One random number -> token (sampler.js:140-147)."""
        if d.greedy:
            return int(d.ids[0])
        r = self.rand() * d.total
        for i in range(len(d.ids)):
            r -= d.probs[i]
            if r <= 0:
                return int(d.ids[i])
        return int(d.ids[-1])

    def sample(self, model, history=(), row: int = 0) -> int:
        return self.draw(self.distribution(model, history, row))
