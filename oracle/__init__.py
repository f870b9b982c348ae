"""CPU oracle for the zerollm hot path -- TEST INFRASTRUCTURE ONLY.

A C restatement (``zllm_oracle.c``) of the reference's plain-JS single-thread oracle:
``src/compute/ref-kernels.js`` (activation quantization, matvec per ggml type, rmsnorm,
softmax, RoPE), ``src/compute/quant.js`` (block dequantizers), ``src/util/f16.js``
(f32<->f16), ``src/model/forward.js`` (the f32-KV forward pass) and the f16-KV attention
of ``src/compute/worker.js:296-333``.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg import
this package, as the checker or as the timed CPU baseline.  The product library
(``zerollm_b200``) never imports it.

Parity pins: the dequantizers are checked against the reference's own golden vectors
(``test/data/quant-vectors.json``, produced by gguf-py) and fresh gguf-py vectors; the f16
conversion against the reference's known encodings and numpy's round-to-nearest-even; the
matvec in an exact-float regime against exact rational arithmetic.  The reference's JS
cannot run here (no Node.js in this image), so the oracle is not diffed against the JS
itself.
"""
from .oracle import *  # noqa: F401,F403
