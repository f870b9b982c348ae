"""On-disk cache of the KV state of a fixed token prefix, in the reference's ``ZLLMKV01`` format.

File (src/model/prefix-cache.js:1-4, :119-135): the 8 bytes ``ZLLMKV01``, a u32 LE header length,
the header as JSON (``fingerprint``, ``nLayer``, ``kvDim``, ``n``, ``tokens``), then for each
layer K[0..n*kvDim) and V[0..n*kvDim) as f32 LE.  The file name is the SHA-1 of the fingerprint,
a newline and the token ids as int32 LE (prefix-cache.js:39-42), so a hit is always the state a
fresh prefill of the same model with the same kernel flavour would compute.

``load`` checks the magic, header, token ids and exact file size and returns False on any
mismatch or damage, never raising for a bad file (prefix-cache.js:50-96).  Each K or V block is
handed to ``model.kvSet``, which on ``CudaModel`` is one host-to-device copy of the f32 rows and
one kernel that casts them (round to nearest even) into the sequence's f16 (or f32) cache rows --
the file is read straight into the device cache, no f16 staging on the host.  ``save`` writes
through a temporary file and a rename, then keeps the 16 newest files (prefix-cache.js:104-143).
Hybrid (``ZLLMKV02``) files are not produced: the backend holds no recurrent state.
"""
from __future__ import annotations

import hashlib
import json
import os
import struct

import numpy as np

MAGIC = b"ZLLMKV01"
MAX_HEADER = 1 << 26          # prefix-cache.js:59


def kernel_flavour(model) -> str:
    """The flavour that goes into the cache key (prefix-cache.js:26-28): the CUDA backend's
    states are their own flavour, ``cuda/kv-f16`` or ``cuda/kv-f32``."""
    kernels = getattr(model, "kernels", "js")
    if kernels == "wasm":
        raise ValueError("the CUDA backend does not compute WASM-flavoured states")
    return f"{kernels}/kv-{getattr(model, 'kv', None) or 'f32'}"


def model_fingerprint(model_path: str, kernels: str) -> str:
    """Identity of a model file plus the kernel flavour (prefix-cache.js:31-34)."""
    st = os.stat(model_path)
    return f"{os.path.basename(model_path)}|{st.st_size}|{round(st.st_mtime * 1000)}|{kernels}"


def _kv_dim(model) -> int:
    return int(model.cfg["n_head_kv"]) * int(model.cfg["head_dim"])


class PrefixCache:
    def __init__(self, dir: str, fingerprint: str):
        self.dir = dir
        self.fingerprint = fingerprint

    def file(self, ids) -> str:
        h = hashlib.sha1()
        h.update(self.fingerprint.encode())
        h.update(b"\n")
        h.update(np.asarray(ids, "<i4").tobytes())
        return os.path.join(self.dir, h.hexdigest() + ".kv")

    def load(self, model, ids) -> bool:
        """Restore the KV state of exactly ``ids`` into a model holding no positions."""
        try:
            ids = [int(i) for i in ids]
            if model.pos != 0 or not ids or model.cfg.get("hybrid"):
                return False
            path = self.file(ids)
            with open(path, "rb") as f:
                head = f.read(12)
                if len(head) != 12 or head[:8] != MAGIC:
                    return False
                hlen = struct.unpack_from("<I", head, 8)[0]
                if hlen > MAX_HEADER:
                    return False
                hb = f.read(hlen)
                if len(hb) != hlen:
                    return False
                h = json.loads(hb.decode("utf-8"))
                kv_dim, n = _kv_dim(model), len(ids)
                if (h.get("fingerprint") != self.fingerprint or h.get("n") != n
                        or h.get("nLayer") != model.cfg["n_layer"] or h.get("kvDim") != kv_dim):
                    return False
                if list(h.get("tokens", [])) != ids:
                    return False
                nbytes = n * kv_dim * 4
                if os.fstat(f.fileno()).st_size != 12 + hlen + nbytes * 2 * model.cfg["n_layer"]:
                    return False                          # truncated or extended
                for layer in range(model.cfg["n_layer"]):
                    for is_v in (0, 1):
                        raw = f.read(nbytes)
                        if len(raw) != nbytes:
                            return False
                        model.kvSet(layer, is_v, n, np.frombuffer(raw, "<f4"))
            model.restorePrefix(ids)
            return True
        except Exception:
            return False

    def save(self, model, ids) -> str:
        """Write the KV state of the first ``len(ids)`` positions the model holds."""
        ids = [int(i) for i in ids]
        if model.cfg.get("hybrid"):
            raise ValueError("hybrid models are not supported by this backend")
        kv_dim, n = _kv_dim(model), len(ids)
        if model.pos < n:
            raise ValueError("model does not hold the prefix")
        os.makedirs(self.dir, exist_ok=True)
        header = json.dumps({"fingerprint": self.fingerprint, "nLayer": model.cfg["n_layer"], "kvDim": kv_dim,
                             "n": n, "tokens": ids}, separators=(",", ":")).encode()
        target = self.file(ids)
        tmp = f"{target}.{os.getpid()}.tmp"
        with open(tmp, "wb") as f:
            f.write(MAGIC + struct.pack("<I", len(header)) + header)
            for layer in range(model.cfg["n_layer"]):
                for is_v in (0, 1):
                    f.write(np.ascontiguousarray(model.kvGet(layer, is_v, n), "<f4").tobytes())
        os.replace(tmp, target)
        self.prune(16)
        return target

    def prune(self, keep: int = 16):
        """Keep only the ``keep`` most recently written ``.kv`` files (best effort)."""
        try:
            files = [os.path.join(self.dir, f) for f in os.listdir(self.dir) if f.endswith(".kv")]
            files.sort(key=lambda p: os.stat(p).st_mtime, reverse=True)
            for p in files[keep:]:
                os.unlink(p)
        except OSError:
            pass
