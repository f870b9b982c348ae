"""zerollm-b200: B200 (sm_100a) backend for zerollm's decode/prefill hot path.

The compute lives in ``libzllm_cuda.so`` (C ABI: ``include/zllm.h``); this package holds the
host-side mirror of the reference's kernel and model interfaces (``kernels``, ``model``), the
ctypes binding (``lib``), the build script (``build``) and seeded synthetic weights (``synth``).
"""
__all__ = ["ggml", "lib", "kernels", "synth", "build"]
