"""Builds the C oracle (attention_f64.c) into oracle/_build/ -- TEST INFRASTRUCTURE ONLY.

    python oracle/build_oracle.py

Also exposes ``load_f64()`` returning a callable over numpy arrays.
"""

from __future__ import annotations

import ctypes
import hashlib
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
SRC = HERE / "attention_f64.c"
OUT = HERE / "_build" / "liboracle_f64.so"


FLAGS = ["-O2", "-std=c11", "-shared", "-fPIC"]


def build(force: bool = False) -> Path:
    """gcc build of SRC, redone whenever the source or flags differ from the stamped build."""
    OUT.parent.mkdir(parents=True, exist_ok=True)
    digest = hashlib.sha256(" ".join(FLAGS).encode() + b"\0" + SRC.read_bytes()).hexdigest()
    stamp = OUT.with_name(OUT.name + ".stamp")
    if force or not OUT.exists() or not stamp.exists() or stamp.read_text().strip() != digest:
        tmp = OUT.with_suffix(".so.tmp")
        subprocess.run(["gcc", *FLAGS, "-o", str(tmp), str(SRC), "-lm"], check=True)
        tmp.replace(OUT)
        stamp.write_text(digest + "\n")
    return OUT


def load_f64():
    lib = ctypes.CDLL(str(build()))
    fn = lib.oracle_attention_f64
    fn.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_int64] * 3 + [ctypes.c_int, ctypes.c_double, ctypes.c_void_p]
    fn.restype = ctypes.c_int

    def attention_f64(q, k, v, causal=False, softmax_scale=None):
        q = np.ascontiguousarray(q, dtype=np.float16)
        k = np.ascontiguousarray(k, dtype=np.float16)
        v = np.ascontiguousarray(v, dtype=np.float16)
        n, d = q.shape[-2:]
        heads = int(np.prod(q.shape[:-2])) if q.ndim > 2 else 1
        scale = (1.0 / np.sqrt(d)) if softmax_scale is None else float(softmax_scale)
        out = np.empty(q.shape, dtype=np.float64)
        rc = fn(q.ctypes.data, k.ctypes.data, v.ctypes.data, heads, n, d, 1 if causal else 0, scale, out.ctypes.data)
        if rc != 0:
            raise MemoryError("oracle_attention_f64: allocation failed")
        return out

    return attention_f64


if __name__ == "__main__":
    print(build(force=True))
