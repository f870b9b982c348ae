"""Tensor-parallel decode over 2 GPUs (BASELINE config 4 in small): two child processes, one per GPU,
each holding its shard (zerollm_b200.tp.shard_model) and joining one NCCL group.  Both ranks end
every pass with the same logits, bit for bit, and those track the single-GPU model within the
reference's SIMD-vs-JS tolerance (the all-reduce adds the partial sums in another order).  Separate
processes on NVLink-connected GPUs map each other's buffers, so the all-reduce is the library's
one-shot kernel over peer memory, not NCCL's.  Needs
two GPUs; NVLS is off for the children (a rank that dies while bound to an NVLink multicast object
can fault its peers)."""
import multiprocessing as mp
import os
import queue

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

TOKS = [3, 17, 42, 5, 88, 1, 250, 7]
BATCH = [(5 * i + 2) % 320 for i in range(64)]     # 64 tokens: the tensor-core GEMM plus the all-reduce


def _model():
    from zerollm_b200 import ggml, synth
    cfg = synth.tiny(n_embd=256, n_ff=1024, n_head=8, n_head_kv=2, head_dim=64)
    return cfg, synth.make_model(cfg, seed=21, quant="q4_k_q6", dist="tame", output_type=ggml.F16)


def _rank(rank, size, uid_q, out_q):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import torch as T
    from zerollm_b200.kernels import Context
    from zerollm_b200.model import CudaModel, tp_unique_id
    from zerollm_b200.tp import shard_model
    T.cuda.set_device(rank)
    ctx = Context(rank)
    if rank == 0:
        uid = tp_unique_id(ctx)
        for _ in range(size - 1):
            uid_q.put(uid)
    else:
        uid = uid_q.get(timeout=120)
    cfg, w = _model()
    lc, lw = shard_model(cfg, w, rank, size)
    m = CudaModel.create(lc, lw, ctx=96, kv="f16", max_batch=64, device=rank, context=ctx, tp=(rank, size, uid))
    step = [m.forward(t).copy() for t in TOKS]
    last = m.forwardBatch(BATCH, logits="last").copy()
    coll = m.tp_collective()
    m.close()
    ctx.close()
    out_q.put((rank, np.stack(step), last, coll))


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_tp2_matches_single_gpu():
    from zerollm_b200.model import CudaModel
    spawn = mp.get_context("spawn")
    uid_q, out_q = spawn.Queue(), spawn.Queue()
    procs = [spawn.Process(target=_rank, args=(r, 2, uid_q, out_q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(2):
            r, step, last, coll = out_q.get(timeout=300)
            res[r] = (step, last, coll)
    except queue.Empty:
        pass
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert sorted(res) == [0, 1], "a rank did not finish"
    assert res[0][2] == res[1][2] == 2, "expected the one-shot NVLink all-reduce on both ranks"
    assert np.array_equal(res[0][0], res[1][0]) and np.array_equal(res[0][1], res[1][1])
    cfg, w = _model()
    one = CudaModel.create(cfg, w, ctx=96, kv="f16", max_batch=64)
    want = [one.forward(t).copy() for t in TOKS] + [one.forwardBatch(BATCH, logits="last").copy()]
    got = list(res[0][0]) + [res[0][1]]
    for g, ww in zip(got, want):
        top = np.abs(ww).max()
        assert np.abs(g - ww).max() <= 2e-2 * top
    one.close()
