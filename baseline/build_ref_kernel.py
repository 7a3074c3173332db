"""Compiles the reference's CUDA kernel, unmodified, for sm_100a (a context line for bench.py).

    python baseline/build_ref_kernel.py [--reference DIR]

Sources are read where they lie in the reference checkout (csrc/kernels/flash_fwd.cu with
csrc/common.cuh and csrc/flash_fwd.h); nothing is copied into this repository. The flags are the
reference's own nvcc flags (setup.py:12-18: -O3 -std=c++20 --use_fast_math -lineinfo
--expt-relaxed-constexpr) with a fixed sm_100a target. Output: baseline/_ref/libfa_ref_kernel.so
(git-ignored; it travels with the tree like the product's own libraries).
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref" / "libfa_ref_kernel.so"
DEFAULT_REFERENCE = Path("/root/reference")


def build(reference: Path = DEFAULT_REFERENCE, quiet: bool = False) -> Path | None:
    kernel = reference / "csrc" / "kernels" / "flash_fwd.cu"
    if not kernel.exists():
        if not quiet:
            print(f"[build_ref_kernel] {kernel} not found; skipped")
        return None
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    OUT.parent.mkdir(parents=True, exist_ok=True)
    deps = [kernel, reference / "csrc" / "common.cuh", reference / "csrc" / "flash_fwd.h",
            HERE / "ref_kernel_shim.cu", Path(__file__)]
    if OUT.exists() and all(d.stat().st_mtime <= OUT.stat().st_mtime for d in deps):
        return OUT
    tmp = OUT.with_suffix(".so.tmp")
    cmd = [nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++20",
           "--use_fast_math", "-lineinfo", "--expt-relaxed-constexpr",
           "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden", "-shared",
           "-I", str(reference / "csrc"), "-o", str(tmp), str(kernel), str(HERE / "ref_kernel_shim.cu")]
    if not quiet:
        print("[build_ref_kernel]", " ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError("nvcc failed building the reference kernel")
    os.replace(tmp, OUT)
    return OUT


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", type=Path, default=DEFAULT_REFERENCE)
    a = ap.parse_args()
    print("built", build(a.reference))


if __name__ == "__main__":
    main()
