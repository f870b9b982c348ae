"""The tensor-core GEMM (tcgen05, f32 accumulation in TMEM) behind passes of 64 or more tokens.

* the f16 x f16 core (zllm_gemm_f16) against torch's f32 product of the same f16 operands;
* k-quant weights x quantized activations (zllm_mm with >= 64 tokens) against the oracle's matvec
  per token (ref-kernels.js:196-277) within 1.5e-4 of the largest output (the contract is 1e-3; a
  single f16 product measured 3e-4 to 6e-4).  Q4_K, Q5_K and Q6_K with |scale| <= 64 take the
  exact-A kernel (sub-block scale x quant exact in f16, activation as an f16 hi / lo pair, super-
  block scales applied in f32); Q6_K with larger scales (the quantizer's usual +-128) the hi / lo
  kernel (three MMAs);
* partial row / token tiles, the residual add, block scales far outside f16's range (a per-matrix
  power of two), and a NaN scale, which keeps the exact per-token kernel (same bits as single
  tokens).
"""
import ctypes as C

import numpy as np
import pytest

import oracle as O
from zerollm_b200 import ggml, synth
from zerollm_b200.kernels import Act, Context, Weight, matvec
from zerollm_b200.lib import check

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


@pytest.mark.parametrize("m,n,k", [(256, 128, 512), (100, 200, 1024), (1000, 16, 4096)])
def test_gemm_f16_matches_torch(ctx, m, n, k):
    g = torch.Generator(device="cuda").manual_seed(m + n + k)
    A = torch.randn(m, k, device="cuda", generator=g).half()
    B = torch.randn(n, k, device="cuda", generator=g).half()
    D = torch.full((n, m), float("nan"), device="cuda")
    P = lambda t: C.c_void_p(t.data_ptr())
    check(ctx.lib.zllm_gemm_f16(ctx.h, P(A), P(B), m, n, k, P(D), None), ctx.h)
    ctx.sync()
    want = (B.float() @ A.float().T).cpu().numpy()
    got = D.cpu().numpy()
    assert np.isfinite(got).all()
    assert _rel(got, want) <= 1e-5


CASES = [(ggml.Q4_K, 512, 4096, 64), (ggml.Q4_K, 300, 2048, 130), (ggml.Q5_K, 256, 1024, 72),
         (ggml.Q6_K, 200, 3072, 65), (ggml.Q6_K, 4096, 12288, 64)]


@pytest.mark.parametrize("t,rows,cols,ntok", CASES, ids=[f"{ggml.type_name(t)}-{r}x{c}-t{n}" for t, r, c, n in CASES])
def test_kquant_gemm_matches_oracle(ctx, t, rows, cols, ntok):
    rng = np.random.default_rng(rows + cols + ntok + t)
    wt = synth.tensor(t, rows, cols, rng, "bench")
    w = Weight.from_tensor(ctx, wt)
    X = rng.standard_normal((ntok, cols)).astype(np.float32)
    X[1] *= 1e-3
    X[2] *= 50.0
    y = torch.full((ntok, rows), float("nan"), device="cuda")
    got = matvec(w, Act(ctx, X), y=y).cpu().numpy()
    ctx.sync()
    assert np.isfinite(got).all()
    for i in (0, 1, 2, ntok - 1):
        want = O.matvec(t, wt["data"], rows, cols, X[i], nthreads=8)
        assert _rel(got[i], want) <= 1.5e-4, i
    # every token against the exact per-token path
    single = np.stack([matvec(w, Act(ctx, X[i])).cpu().numpy().ravel() for i in range(ntok)])
    assert max(_rel(got[i], single[i]) for i in range(ntok)) <= 1.5e-4


def test_q6k_full_scale_range(ctx):
    """Q6_K sub-block scales over the quantizer's full int8 range: (q - 32) * scale reaches 4096 and
    is not exact in f16, so these matrices take the hi / lo kernel, within the same bound."""
    rng = np.random.default_rng(11)
    rows, cols, ntok = 256, 2048, 70
    raw = synth.quant_blocks(ggml.Q6_K, rows, cols, rng, "bench").reshape(rows, -1, 210).copy()
    raw[:, :, 192:208] = rng.integers(-128, 128, (rows, cols // 256, 16)).astype(np.int8).view(np.uint8)
    w = Weight(ctx, ggml.Q6_K, rows, cols, raw.reshape(-1))
    X = rng.standard_normal((ntok, cols)).astype(np.float32)
    got = matvec(w, Act(ctx, X)).cpu().numpy()
    assert np.isfinite(got).all()
    for i in (0, ntok - 1):
        assert _rel(got[i], O.matvec(ggml.Q6_K, raw.reshape(-1), rows, cols, X[i])) <= 1.5e-4


def test_gemm_residual(ctx):
    rng = np.random.default_rng(9)
    wt = synth.tensor(ggml.Q4_K, 384, 1024, rng, "bench")
    w = Weight.from_tensor(ctx, wt)
    X = rng.standard_normal((70, 1024)).astype(np.float32)
    Y = matvec(w, Act(ctx, X)).cpu().numpy()
    base = torch.as_tensor(rng.standard_normal((70, 384)).astype(np.float32)).cuda()
    out = base.clone()
    matvec(w, Act(ctx, X), y=out, y_add=out)
    assert np.array_equal(out.cpu().numpy(), (base.cpu().numpy() + Y).astype(np.float32))


@pytest.mark.parametrize("scale", [1e-5, 3e3])
def test_gemm_extreme_scale_ranges(ctx, scale):
    """Block scales far below or above f16's comfortable range: the per-matrix power of two keeps
    the dequantized values inside f16, so the GEMM stays within the contract."""
    rng = np.random.default_rng(4)
    rows, cols, ntok = 200, 1024, 66
    raw = synth.quant_blocks(ggml.Q4_K, rows, cols, rng, "bench").reshape(rows, -1, 144).copy()
    d = (np.abs(rng.standard_normal(raw.shape[:2])) * scale).astype(np.float16)
    raw[:, :, 0:2] = d.view(np.uint8).reshape(rows, -1, 2)
    raw[:, :, 2:4] = (d * np.float16(0.5)).view(np.uint8).reshape(rows, -1, 2)
    w = Weight(ctx, ggml.Q4_K, rows, cols, raw.reshape(-1))
    X = rng.standard_normal((ntok, cols)).astype(np.float32)
    got = matvec(w, Act(ctx, X)).cpu().numpy()
    assert np.isfinite(got).all()
    for i in (0, ntok - 1):
        assert _rel(got[i], O.matvec(ggml.Q4_K, raw.reshape(-1), rows, cols, X[i])) <= 1.5e-4


def test_nan_scale_keeps_exact_path(ctx):
    """A Q4_K matrix with a NaN block scale has no f16 image: its batches take the exact kernel,
    which reproduces single tokens bit for bit (NaN rows included)."""
    rng = np.random.default_rng(3)
    rows, cols = 64, 512
    raw = synth.quant_blocks(ggml.Q4_K, rows, cols, rng, "bench").reshape(rows, -1).copy()
    raw[5, 0:2] = np.frombuffer(np.uint16(0x7e00).tobytes(), np.uint8)     # d of row 5, block 0: NaN
    w = Weight(ctx, ggml.Q4_K, rows, cols, raw.reshape(-1))
    X = rng.standard_normal((65, cols)).astype(np.float32)
    Y = matvec(w, Act(ctx, X)).cpu().numpy()
    assert np.isnan(Y[:, 5]).all()
    for i in (0, 64):
        assert np.array_equal(Y[i], matvec(w, Act(ctx, X[i])).cpu().numpy().ravel(), equal_nan=True)
