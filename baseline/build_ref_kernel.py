"""Compiles the reference's CUDA kernel, unmodified, for sm_100a (a context line for bench.py).

    python baseline/build_ref_kernel.py REFERENCE_DIR      (or FA_REFERENCE_DIR=REFERENCE_DIR)

Sources are read where they lie in the reference checkout (csrc/kernels/flash_fwd.cu with
csrc/common.cuh and csrc/flash_fwd.h); nothing is copied into this repository. The flags are the
reference's own nvcc flags (setup.py:12-18: -O3 -std=c++20 --use_fast_math -lineinfo
--expt-relaxed-constexpr) with a fixed sm_100a target. Output: baseline/_ref/libfa_ref_kernel.so
(git-ignored; it travels with the tree like the product's own libraries).
"""

from __future__ import annotations

import hashlib
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref" / "libfa_ref_kernel.so"


def build(reference: Path | None, quiet: bool = False) -> Path | None:
    """Builds OUT from `reference` (a checkout of the reference); returns None when its kernel
    source is not there."""
    if reference is None:
        return None
    reference = Path(reference)
    kernel = reference / "csrc" / "kernels" / "flash_fwd.cu"
    if not kernel.exists():
        if not quiet:
            print(f"[build_ref_kernel] {kernel} not found; skipped")
        return None
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    OUT.parent.mkdir(parents=True, exist_ok=True)
    deps = [kernel, reference / "csrc" / "common.cuh", reference / "csrc" / "flash_fwd.h",
            HERE / "ref_kernel_shim.cu"]
    flags = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++20",
             "--use_fast_math", "-lineinfo", "--expt-relaxed-constexpr",
             "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden", "-shared"]
    h = hashlib.sha256("\0".join(flags).encode())
    for d in deps:
        h.update(b"\0" + d.read_bytes())
    digest = h.hexdigest()
    stamp = OUT.with_name(OUT.name + ".stamp")
    if OUT.exists() and stamp.exists() and stamp.read_text().strip() == digest:
        return OUT
    tmp = OUT.with_suffix(".so.tmp")
    cmd = [nvcc, *flags, "-I", str(reference / "csrc"), "-o", str(tmp), str(kernel),
           str(HERE / "ref_kernel_shim.cu")]
    if not quiet:
        print("[build_ref_kernel]", " ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError("nvcc failed building the reference kernel")
    os.replace(tmp, OUT)
    stamp.write_text(digest + "\n")
    return OUT


def main() -> None:
    ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("FA_REFERENCE_DIR")
    if ref is None:
        raise SystemExit("usage: python baseline/build_ref_kernel.py REFERENCE_DIR (or set FA_REFERENCE_DIR)")
    print("built", build(Path(ref)))


if __name__ == "__main__":
    main()
