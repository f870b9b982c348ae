"""The Node-API add-on (zerollm_b200/napi/zllm_napi.c) builds against the declared Node-API
prototypes, exports the entry points Node looks up when it loads a .node file, and leaves undefined
only the napi_* functions (resolved from the node executable at load time), the C library and the
libzllm_cuda.so functions include/zllm.h declares."""
import os
import re
import shutil
import subprocess

import pytest

from zerollm_b200 import build, lib

pytestmark = pytest.mark.skipif(shutil.which("nm") is None, reason="needs binutils nm")


def _syms(path, flag):
    out = subprocess.run(["nm", "-D", flag, path], capture_output=True, text=True, check=True).stdout
    return {line.split()[-1].split("@")[0] for line in out.splitlines() if line.strip()}


def test_addon_builds_and_exports_the_module_entry_points():
    path = build.build_napi()
    assert os.path.exists(path)
    defined = _syms(path, "--defined-only")
    assert {"napi_register_module_v1", "node_api_module_get_api_version_v1"} <= defined


def test_addon_needs_only_napi_libc_and_declared_library_functions():
    path = build.build_napi()
    declared = set(lib.header_functions())
    for s in _syms(path, "--undefined-only"):
        if s.startswith("zllm_"):
            assert s in declared, s
        else:
            assert s.startswith("napi_") or re.match(r"^(_|calloc|free|snprintf|malloc|memset|memcpy)", s), s
