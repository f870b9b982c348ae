"""Build libzllm_cuda.so in-tree with nvcc for sm_100a (B200).

    python -m zerollm_b200.build            # incremental
    python -m zerollm_b200.build --force    # rebuild everything

Objects go to zerollm_b200/_build/, the library to zerollm_b200/libzllm_cuda.so.  The CUDA
runtime is linked statically so the library does not depend on which libcudart another module
(torch) loaded first.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libzllm_cuda.so")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
def _nccl_include() -> list[str]:
    """The NCCL header (declarations only: the library is opened at run time by tp.cu)."""
    cands = []
    try:
        import importlib.util
        spec = importlib.util.find_spec("nvidia")
        for base in (spec.submodule_search_locations or []) if spec else []:
            cands.append(os.path.join(base, "nccl", "include"))
    except Exception:
        pass
    cands += ["/usr/include", "/usr/local/cuda/include"]
    for c in cands:
        if os.path.exists(os.path.join(c, "nccl.h")):
            return [f"-I{c}"]
    raise RuntimeError("nccl.h not found")


NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
              "-Xptxas", "-warn-spills", f"-I{os.path.join(ROOT, 'include')}", f"-I{CSRC}", *_nccl_include()]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def sources() -> list[str]:
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def headers() -> list[str]:
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".h", ".cuh"))]
    return hs + [os.path.join(ROOT, "include", f) for f in os.listdir(os.path.join(ROOT, "include"))]


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(src: str, force: bool, verbose: bool) -> str:
    obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
    if force or _stale(obj, [src] + headers()):
        cmd = [nvcc(), *ARCH, *NVCC_FLAGS, "-c", src, "-o", obj]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode:
            raise RuntimeError(f"nvcc failed on {src}:\n{r.stdout}\n{r.stderr}")
        if r.stderr.strip() and verbose:
            print(r.stderr, file=sys.stderr)
    return obj


def build(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    srcs = sources()
    with cf.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        objs = list(ex.map(lambda s: _compile(s, force, verbose), srcs))
    if force or _stale(LIB, objs):
        tmp = LIB + ".tmp"
        cmd = [nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", tmp, *objs, "-lrt", "-ldl", "-lpthread"]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB)
    return LIB


NAPI_SRC = os.path.join(PKG, "napi", "zllm_napi.c")
NAPI_OUT = os.path.join(PKG, "zllm_napi.node")


def build_napi(verbose: bool = False) -> str:
    """The Node-API add-on (zerollm_b200/napi/zllm_napi.c) over libzllm_cuda.so: a plain shared object
    whose napi_* symbols resolve from the node executable when Node loads it; libzllm_cuda.so is
    found beside it ($ORIGIN)."""
    deps = [NAPI_SRC, os.path.join(PKG, "napi", "napi_decl.h"), os.path.join(ROOT, "include", "zllm.h"), LIB]
    if _stale(NAPI_OUT, deps):
        cc = os.environ.get("CC") or shutil.which("gcc") or "cc"
        cmd = [cc, "-O2", "-std=c11", "-Wall", "-Werror", "-fPIC", "-shared", f"-I{os.path.join(ROOT, 'include')}",
               "-o", NAPI_OUT + ".tmp", NAPI_SRC, f"-L{PKG}", "-lzllm_cuda", "-Wl,-rpath,$ORIGIN"]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode:
            raise RuntimeError(f"N-API add-on build failed:\n{r.stdout}\n{r.stderr}")
        os.replace(NAPI_OUT + ".tmp", NAPI_OUT)
    return NAPI_OUT


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    a = ap.parse_args()
    print(build(a.force, a.verbose))
    print(build_napi(a.verbose))
