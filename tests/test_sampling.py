"""Sampling over device-selected candidates (src/sampling/sampler.js), the host half on the CPU.

The candidates come here from the oracle's restatement of the penalties and topKSelect (the GPU
tests check the device selection against the same restatement); these tests pin the host half --
softmax with temperature, min-p, top-p and the seeded draw -- to the behaviours
test/sampler.test.js checks, and the two statements of mulberry32 against each other.
"""
import numpy as np

import oracle as O
from zerollm_b200.sampler import Sampler, mulberry32


def _gauss(rand, n):
    out = []
    for _ in range(n):                                           # src/util/rng.js:16-20
        u = 0.0
        while u == 0.0:
            u = rand()
        out.append(np.sqrt(-2 * np.log(u)) * np.cos(2 * np.pi * rand()))
    return np.asarray(out, np.float32)


def _sample(s: Sampler, logits, history=(), k=None):
    l = O.penalize(logits, history, s.repeat_penalty, s.frequency, s.presence, s.repeat_last_n)
    k = (1 if s.greedy else (s.top_k if 0 < s.top_k < len(l) else len(l))) if k is None else k
    ids, vals = O.topk_select(l, k)
    return s.draw(s.from_candidates(ids, vals))


def test_mulberry32_statements_agree():
    for seed in (0, 1, 5, 0xDEADBEEF, 2 ** 32 - 1):
        a, b = mulberry32(seed), O.mulberry32(seed)
        xs = [a() for _ in range(2000)]
        assert xs == [b() for _ in range(2000)]
        assert all(0 <= x < 1 for x in xs)


def test_topk_select_matches_full_sort():
    rand = mulberry32(3)
    for n, k in ((1000, 40), (50, 50), (10, 10), (5000, 1), (777, 100)):
        l = _gauss(rand, n)
        ids, vals = O.topk_select(l, k)
        want = sorted(range(n), key=lambda i: (-float(l[i]), i))[:k]
        assert list(ids) == want and np.array_equal(vals, l[want])
    l = np.asarray([1, 3, 3, np.nan, 3, -np.inf, 2], np.float32)     # ties by index, NaN left out
    assert list(O.topk_select(l, 7)[0]) == [1, 2, 4, 6, 0, 5]


def test_greedy_and_supports():
    assert _sample(Sampler(temperature=0, seed=1), np.asarray([0.1, 3, 2, -1], np.float32)) == 1
    s = Sampler(temperature=5, top_k=2, top_p=1, seed=1)
    assert {_sample(s, np.asarray([5, 4, 3, 2, 1, 0], np.float32)) for _ in range(500)} == {0, 1}
    s = Sampler(temperature=1, top_k=0, top_p=0.5, seed=2)
    assert {_sample(s, np.asarray([10, 0, 0, 0], np.float32)) for _ in range(100)} == {0}
    s = Sampler(temperature=1, top_k=0, top_p=0.5, seed=2)
    assert {_sample(s, np.zeros(4, np.float32)) for _ in range(300)} == {0, 1}
    s = Sampler(temperature=1, top_k=0, top_p=1, min_p=0.2, seed=4)
    assert {_sample(s, np.asarray([4, 3.9, 0, 0, 0], np.float32)) for _ in range(300)} == {0, 1}


def test_seeded_reproducible_and_empirical():
    rand = mulberry32(1)
    l = _gauss(rand, 200) * np.float32(0.5)
    run = lambda seed: [_sample(s, l) for s in [Sampler(temperature=1, top_k=0, top_p=1, seed=seed)] for _ in range(30)]  # noqa: E731
    assert run(5) == run(5) and run(5) != run(6)
    l = np.asarray([1, 0.5, 0, -0.5], np.float32)
    T = 0.8
    w = np.exp(l.astype(np.float64) / T)
    s = Sampler(temperature=T, top_k=0, top_p=1, seed=11)
    counts = np.bincount([_sample(s, l) for _ in range(40000)], minlength=4)
    assert np.all(np.abs(counts / 40000 - w / w.sum()) < 0.01)


def test_penalties():
    l = np.asarray([2, 1.9, 0, 0], np.float32)
    before = l.copy()
    assert _sample(Sampler(temperature=0, repeat_penalty=1.5), l, [0]) == 1
    assert np.array_equal(l, before)
    assert _sample(Sampler(temperature=0, repeat_penalty=2), np.asarray([-1, -1.5], np.float32), [0]) == 1
    assert _sample(Sampler(temperature=0, presence_penalty=0.5), l, [0, 0, 0]) == 1
    assert _sample(Sampler(temperature=0, frequency_penalty=0.05), l, [0]) == 0
    assert _sample(Sampler(temperature=0, frequency_penalty=0.05), l, [0, 0, 0]) == 1
    assert _sample(Sampler(temperature=0, repeat_penalty=1.5, repeat_last_n=1), l, [0, 2]) == 0
    s = Sampler(repeat_penalty=1.1, repeat_last_n=4)
    assert s.penalised([5, 1, 2, 2, 3, 2]) == ([2, 3], [3, 1])
