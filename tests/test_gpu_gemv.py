"""GPU parity of activation quantization and the decode GEMVs against the CPU oracle.

Contract: every matmul output within max|d| / max|ref| <= 1e-3 of the oracle.  The k-quant
GEMVs compute their block terms in f32 on exact integer dots and are held to a much tighter bar
here (5e-6); the legacy quants Q8_0 / Q4_0 / Q5_0 keep the oracle's double arithmetic (1e-6, and
>= 99% of outputs bit-identical); quantization is bit-exact.
"""
import numpy as np
import pytest

import oracle as O
from zerollm_b200 import ggml, synth
from zerollm_b200.kernels import Act, Context, Weight, matvec, matvec_host

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def ctx():
    c = Context(0)
    yield c
    c.close()


def _rel(got, want):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    return float(np.abs(got - want).max() / max(np.abs(want).max(), 1e-30))


def test_quantize_act_bit_exact(ctx):
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.standard_normal(4096), rng.standard_normal(4096) * 1e-3, rng.standard_normal(4096) * 1e4,
                        np.zeros(64), np.repeat([2.5, -2.5, 0.5, 127.0], 16)]).astype(np.float32)
    x[7] = np.nan
    x[4096 + 100] = np.inf
    a = Act(ctx, x).quant()
    torch.cuda.synchronize()
    q, d, s = O.quantize_act(x)
    assert np.array_equal(a.q.cpu().numpy().ravel(), q)
    assert np.array_equal(a.d.cpu().numpy().ravel().view(np.uint32), d.view(np.uint32))
    assert np.array_equal(a.s.cpu().numpy().ravel(), s)


CASES = [
    (ggml.Q4_K, 4096, 4096), (ggml.Q4_K, 1024, 4096), (ggml.Q4_K, 37, 256), (ggml.Q4_K, 1, 512), (ggml.Q4_K, 12288, 4096),
    (ggml.Q5_K, 300, 1024), (ggml.Q6_K, 4096, 12288), (ggml.Q6_K, 77, 512), (ggml.Q6_K, 5, 25600), (ggml.Q6_K, 129, 768),
    (ggml.Q8_0, 513, 4096), (ggml.Q8_0, 3, 96), (ggml.Q4_0, 129, 1024), (ggml.Q5_0, 200, 2048),
    (ggml.F16, 1000, 4096), (ggml.F16, 3, 8), (ggml.BF16, 64, 1024), (ggml.F32, 33, 256), (ggml.F32, 7, 12),
]


@pytest.mark.parametrize("t,rows,cols", CASES, ids=[f"{ggml.type_name(t)}-{r}x{c}" for t, r, c in CASES])
def test_matvec_matches_oracle(ctx, t, rows, cols):
    rng = np.random.default_rng(rows * 31 + cols + t)
    wt = synth.tensor(t, rows, cols, rng, "bench")
    x = rng.standard_normal(cols).astype(np.float32)
    want = O.matvec(t, wt["data"], rows, cols, x, nthreads=8)
    w = Weight.from_tensor(ctx, wt)
    y = torch.full((1, rows), float("nan"), device="cuda")    # unwritten rows would stay NaN
    got = matvec(w, Act(ctx, x), y=y).cpu().numpy().ravel()
    ctx.sync()                                                # raises on a device-side timeout
    assert np.isfinite(got).all(), np.argwhere(~np.isfinite(got))[:10]
    rel = _rel(got, want)
    assert rel <= 1e-3
    if t in (ggml.Q4_K, ggml.Q5_K, ggml.Q6_K):
        assert rel <= 5e-6, rel
    elif t in ggml.QUANTIZED:
        assert rel <= 1e-6, rel
        assert np.mean(got == want) >= 0.99
    else:
        assert rel <= 1e-5, rel


@pytest.mark.parametrize("name", ["Q4_0", "Q5_0", "Q8_0", "Q4_K", "Q5_K", "Q6_K", "F16", "BF16"])
def test_extreme_blocks_match_oracle(ctx, name):
    """gguf-py's extreme blocks (NaN / inf / denormal scales, 0x00 and 0xFF blocks): same values, NaNs in the same rows."""
    import os
    z = np.load(os.path.join(os.path.dirname(__file__), "golden", "ggufpy_vectors.npz"))
    raw = z[f"{name}.raw.raw"]
    rows, cols = z[f"{name}.raw.expected"].shape
    t = ggml.NAMES[name]
    x = np.random.default_rng(1).standard_normal(cols).astype(np.float32)
    with np.errstate(all="ignore"):
        want = O.matvec(t, raw.reshape(-1), rows, cols, x)
    got = matvec(Weight(ctx, t, rows, cols, raw.reshape(-1)), Act(ctx, x)).cpu().numpy().ravel()
    assert np.array_equal(np.isnan(got), np.isnan(want))
    fin = np.isfinite(want)
    assert np.array_equal(np.isinf(got), np.isinf(want))
    if fin.any():
        assert _rel(got[fin], want[fin]) <= (5e-6 if t in ggml.QUANTIZED else 1e-5)


def test_batched_equals_per_token_and_residual(ctx):
    rng = np.random.default_rng(5)
    wt = synth.tensor(ggml.Q4_K, 768, 2048, rng, "bench")
    w = Weight.from_tensor(ctx, wt)
    X = rng.standard_normal((3, 2048)).astype(np.float32)
    Y = matvec(w, Act(ctx, X)).cpu().numpy()
    for t in range(3):
        y1 = matvec(w, Act(ctx, X[t])).cpu().numpy().ravel()
        assert np.array_equal(Y[t], y1)
    base = torch.as_tensor(rng.standard_normal((3, 768)).astype(np.float32)).cuda()
    out = base.clone()
    matvec(w, Act(ctx, X), y=out, y_add=out)
    want = (base.cpu().numpy() + Y).astype(np.float32)
    assert np.array_equal(out.cpu().numpy(), want)


KQ = [(ggml.Q4_K, 4096, 4096), (ggml.Q5_K, 520, 2048), (ggml.Q6_K, 700, 12288), (ggml.Q6_K, 40, 25600),
      (ggml.Q4_K, 1000, 5120)]


@pytest.mark.parametrize("t,rows,cols", KQ, ids=[f"{ggml.type_name(t)}-{r}x{c}" for t, r, c in KQ])
def test_kquant_batches_bit_identical_to_single_tokens(ctx, t, rows, cols):
    """The tensor-core GEMVs add each token's block terms with one formula in an order fixed by the
    matrix shape: a token's outputs are the same bits alone (block-diagonal MMA) or in a batch
    (token MMA, 8 or 16 tokens per launch, more in launches of 16).  From 64 tokens the tcgen05
    GEMM takes over (within 1e-3, tests/test_gpu_gemm.py)."""
    rng = np.random.default_rng(rows + cols + t)
    wt = synth.tensor(t, rows, cols, rng, "bench")
    w = Weight.from_tensor(ctx, wt)
    X = rng.standard_normal((40, cols)).astype(np.float32)
    X[3] *= 1e-3
    singles = np.stack([matvec(w, Act(ctx, X[i])).cpu().numpy().ravel() for i in range(40)])
    for n in (2, 5, 8, 9, 15, 16, 17, 33, 40):
        Y = matvec(w, Act(ctx, X[:n])).cpu().numpy()
        ctx.sync()
        assert np.array_equal(Y, singles[:n]), (n, np.argwhere(Y != singles[:n])[:5])
    for i in (0, 3, 16, 39):
        want = O.matvec(t, wt["data"], rows, cols, X[i], nthreads=8)
        assert _rel(singles[i], want) <= 5e-6


@pytest.mark.parametrize("t", [ggml.Q4_K, ggml.Q5_K, ggml.Q6_K])
def test_in_kernel_quantization_bit_identical(ctx, t):
    """A one-token k-quant GEMV given the f32 activation quantizes it itself, bit-exactly."""
    rng = np.random.default_rng(t)
    rows, cols = 333, 4096
    wt = synth.tensor(t, rows, cols, rng, "bench")
    w = Weight.from_tensor(ctx, wt)
    x = rng.standard_normal(cols).astype(np.float32)
    x[:64] *= 1e-30
    x[100] = np.nan
    x[300] = np.inf
    x[640:672] = 0
    x[700:732] = np.float32(2.5)
    a = matvec(w, Act(ctx, x)).cpu().numpy()
    b = matvec(w, Act(ctx, x), fused_quant=True).cpu().numpy()
    ctx.sync()
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_host_entry_point_equals_device_path(ctx):
    rng = np.random.default_rng(6)
    for t in (ggml.Q6_K, ggml.F16, ggml.Q4_K):
        wt = synth.tensor(t, 300, 1024, rng, "bench")
        w = Weight.from_tensor(ctx, wt)
        for n in (1, 2):
            X = rng.standard_normal((n, 1024)).astype(np.float32)
            a = matvec_host(w, X)
            b = matvec(w, Act(ctx, X)).cpu().numpy()
            assert np.array_equal(a, b)


def test_host_entry_point_pinned_replay(ctx):
    """zllm_matvec on pinned host buffers: a call repeated with the same buffers is recorded as a CUDA
    graph and replayed.  New inputs every call, a second weight, and a larger call that regrows the
    context's scratch in between: each result equals the device path's bits."""
    import ctypes as C
    from zerollm_b200.lib import check
    rng = np.random.default_rng(21)
    rows, cols = 512, 4096
    w1 = Weight.from_tensor(ctx, synth.tensor(ggml.Q4_K, rows, cols, rng, "bench"))
    w2 = Weight.from_tensor(ctx, synth.tensor(ggml.Q6_K, rows, cols, rng, "bench"))
    big = Weight.from_tensor(ctx, synth.tensor(ggml.Q4_K, 2048, 8192, rng, "bench"))
    xh = torch.empty(cols, dtype=torch.float32).pin_memory()
    yh = torch.empty(rows, dtype=torch.float32).pin_memory()
    P = lambda t: C.c_void_p(t.data_ptr())
    for it in range(9):
        w = w2 if it in (4, 5) else w1
        X = rng.standard_normal(cols).astype(np.float32)
        xh.copy_(torch.from_numpy(X))
        check(ctx.lib.zllm_matvec(ctx.h, w.h, P(xh), 1, P(yh)), ctx.h)
        want = matvec(w, Act(ctx, X), fused_quant=True).cpu().numpy().ravel()
        ctx.sync()
        assert np.array_equal(yh.numpy().view(np.uint32), want.view(np.uint32)), it
        if it == 6:                                             # regrows the scratch slots
            matvec_host(big, rng.standard_normal((3, 8192)).astype(np.float32))


def test_rejects_bad_shapes(ctx):
    from zerollm_b200.lib import ZllmError
    with pytest.raises(ZllmError):
        Weight(ctx, ggml.Q4_K, 4, 100, np.zeros(10, np.uint8))
    with pytest.raises(ZllmError):
        Weight(ctx, 3, 4, 256, np.zeros(4 * 160, np.uint8))       # Q4_1 is not a hot-path type


def test_weight_outlives_context():
    """Handles freed after their context is destroyed release only the handle (no crash, no leak)."""
    c = Context(0)
    wt = synth.tensor(ggml.Q4_K, 64, 256, np.random.default_rng(0), "bench")
    w = Weight.from_tensor(c, wt)
    c.close()
    w.free()
