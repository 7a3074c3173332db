"""Builds the native C-ABI test driver tests/native/capi_check.c -- TEST INFRASTRUCTURE.

    python tests/native/build_native.py

gcc, C11, linked against the product library libfa_b200.so (through include/fa_b200.h only),
the C oracle oracle/attention_f64.c (the checker) and the static CUDA runtime (for cudaMalloc,
streams and events). Output: tests/native/_build/capi_check (git-ignored), with an rpath to the
library's directory so it runs from any working directory of the same tree. Rebuilt whenever
the sources, the library or the flags change.
"""

from __future__ import annotations

import hashlib
import os
import subprocess
from pathlib import Path

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
SRC = HERE / "capi_check.c"
ORACLE = REPO / "oracle" / "attention_f64.c"
LIB_DIR = REPO / "flash-attention-from-scratch_b200" / "fa"
INCLUDE = REPO / "include"
OUT = HERE / "_build" / "capi_check"


def _cuda_home() -> Path:
    for cand in (os.environ.get("CUDA_HOME"), "/usr/local/cuda"):
        if cand and (Path(cand) / "include" / "cuda_runtime.h").exists():
            return Path(cand)
    raise RuntimeError("CUDA toolkit not found (set CUDA_HOME)")


def build(force: bool = False) -> Path:
    cuda = _cuda_home()
    rpath = os.path.relpath(LIB_DIR, OUT.parent)
    cmd = ["gcc", "-O2", "-std=c11", "-Wall", "-I", str(INCLUDE), "-I", str(cuda / "include"),
           "-o", "{out}", str(SRC), str(ORACLE), "-L", str(LIB_DIR), "-lfa_b200",
           "-L", str(cuda / "lib64"), "-lcudart_static", "-ldl", "-lpthread", "-lrt", "-lm",
           f"-Wl,-rpath,$ORIGIN/{rpath}"]
    h = hashlib.sha256("\0".join(cmd).encode())
    for f in (SRC, ORACLE, INCLUDE / "fa_b200.h", LIB_DIR / "libfa_b200.so"):
        h.update(b"\0" + f.read_bytes())
    digest = h.hexdigest()
    stamp = OUT.with_name(OUT.name + ".stamp")
    if not force and OUT.exists() and stamp.exists() and stamp.read_text().strip() == digest:
        return OUT
    OUT.parent.mkdir(parents=True, exist_ok=True)
    tmp = OUT.with_name(OUT.name + ".tmp")
    subprocess.run([c.replace("{out}", str(tmp)) for c in cmd], check=True)
    os.replace(tmp, OUT)
    stamp.write_text(digest + "\n")
    return OUT


if __name__ == "__main__":
    print(build(force=True))
