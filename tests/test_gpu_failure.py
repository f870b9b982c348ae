"""Failure detection on the GPU without faulting it: a bounded device wait that runs out.

The tensor-parallel all-reduce kernel waits for every peer GPU's slice stamp.  Run against a
phantom peer that never stamps (zllm_peer_wait_selftest), the wait gives up after its 2 s limit,
the kernel finishes and returns, and the host reads the status word: ZLLM_E_TIMEOUT with the
peer bit (0x10), the status cleared, and the context still usable for the next call.  Nothing is
trapped, asserted on the device or read out of bounds.
"""
import time

import numpy as np
import pytest

import oracle as O
from zerollm_b200 import ggml, synth
from zerollm_b200.kernels import Act, Context, Weight, matvec
from zerollm_b200.lib import E_TIMEOUT, OK

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def test_peer_wait_expires_and_context_survives():
    ctx = Context(0)
    t0 = time.time()
    rc = ctx.lib.zllm_peer_wait_selftest(ctx.h)
    dt = time.time() - t0
    assert rc == E_TIMEOUT
    assert 1.5 < dt < 60                                   # the 2 s limit, not a hang
    assert b"0x10" in ctx.lib.zllm_last_error(ctx.h)
    assert ctx.lib.zllm_sync(ctx.h) == OK             # the status word was cleared
    rng = np.random.default_rng(3)
    wt = synth.tensor(ggml.Q4_K, 256, 1024, rng, "bench")
    x = rng.standard_normal(1024).astype(np.float32)
    got = matvec(Weight.from_tensor(ctx, wt), Act(ctx, x)).cpu().numpy().ravel()
    want = O.matvec(ggml.Q4_K, wt["data"], 256, 1024, x)
    assert np.abs(got - want).max() <= 1e-3 * np.abs(want).max()
    ctx.close()
