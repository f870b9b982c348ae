"""The C-ABI library builds, loads without a GPU and exports exactly what include/zllm.h declares."""
import ctypes as C
import os
import subprocess

import pytest

from zerollm_b200 import build, lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def so():
    path = build.build()
    assert os.path.exists(path)
    return path


def test_exports_every_declared_symbol(so):
    L = C.CDLL(so)
    declared = lib.header_functions()
    assert len(declared) >= 10
    missing = [n for n in declared if not hasattr(L, n)]
    assert not missing, missing
    out = subprocess.run(["nm", "-D", "--defined-only", so], capture_output=True, text=True).stdout
    exported = {l.split()[-1] for l in out.splitlines() if " T " in l and l.split()[-1].startswith("zllm_")}
    assert set(declared) <= exported
    # every declared function has a ctypes signature in the binding, and nothing else is bound
    assert set(lib.SIGNATURES) == set(declared)


def test_loads_and_reports_errors_without_gpu(so):
    L = lib.load()
    assert b"sm_100a" in L.zllm_version()
    # null arguments are rejected before any device work
    assert L.zllm_init(0, None) == lib.E_ARG
    assert L.zllm_sync(None) == lib.E_ARG
    assert L.zllm_last_error(None) == b"no context"
