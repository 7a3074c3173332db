"""Builds the sm_100a libraries in-tree with nvcc (no PyTorch extension machinery).

    python flash-attention-from-scratch_b200/build.py [--force] [--verbose-ptxas]

Outputs (next to the Python package, so they travel with the source tree):
  fa/libfa_b200.so       the product: kernel + C ABI (include/fa_b200.h)
  fa/libfa_selftest.so   building-block probes used only by the tests

Replaces the reference's setup.py / CMakeLists.txt build of the kernel (setup.py:12-34):
same -O3 -lineinfo spirit, but a fixed sm_100a target and a plain shared library.
"""

from __future__ import annotations

import argparse
import hashlib
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_ROOT = Path(__file__).resolve().parent
CSRC = PKG_ROOT / "csrc"
OUT_DIR = PKG_ROOT / "fa"
INCLUDE = PKG_ROOT.parent / "include"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "--expt-relaxed-constexpr",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
    "-shared",
]

LIBS = {
    "libfa_b200.so": ["flash_fwd_sm100.cu", "capi.cu", "capi_static.cu"],
    "libfa_selftest.so": ["selftest_sm100.cu"],
}
HEADERS = ["sm100_ptx.cuh", "softmax_common.cuh", "fa_internal.h", "tma_host.h", "capi_internal.h"]


def nvcc_path() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _digest(files: list[Path], cmd: list[str]) -> str:
    """SHA-256 over the compile command and the bytes of every input file."""
    h = hashlib.sha256()
    h.update("\0".join(cmd).encode())
    for f in files:
        h.update(b"\0" + f.name.encode() + b"\0")
        h.update(f.read_bytes())
    return h.hexdigest()


def _stamp(target: Path) -> Path:
    return target.with_name(target.name + ".stamp")


def _up_to_date(target: Path, digest: str) -> bool:
    """True when `target` exists and was built from exactly these inputs (its stamp holds their
    digest); a prebuilt library from other sources is rebuilt whatever its timestamps."""
    stamp = _stamp(target)
    return target.exists() and stamp.exists() and stamp.read_text().strip() == digest


def build(force: bool = False, verbose_ptxas: bool = False, quiet: bool = False) -> list[Path]:
    nvcc = nvcc_path()
    built = []
    deps = [CSRC / h for h in HEADERS] + [INCLUDE / "fa_b200.h"]
    for lib, srcs in LIBS.items():
        target = OUT_DIR / lib
        sources = [CSRC / s for s in srcs]
        flags = [*ARCH_FLAGS, *COMMON_FLAGS]
        digest = _digest(sources + deps, flags + srcs)
        if not force and _up_to_date(target, digest):
            built.append(target)
            continue
        tmp = target.with_suffix(".so.tmp")
        cmd = [nvcc, *flags, "-I", str(CSRC), "-I", str(INCLUDE)]
        if verbose_ptxas:
            cmd += ["-Xptxas", "-v"]
        # Export the C ABI (default visibility) while hiding everything else.
        cmd += ["-o", str(tmp), *map(str, sources)]
        if not quiet:
            print("[build]", " ".join(cmd), flush=True)
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            sys.stderr.write(res.stdout + res.stderr)
            raise RuntimeError(f"nvcc failed building {lib}")
        if verbose_ptxas or not quiet:
            out = (res.stdout + res.stderr).strip()
            if out:
                print(out)
        os.replace(tmp, target)
        _stamp(target).write_text(digest + "\n")
        built.append(target)
    return built


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose-ptxas", action="store_true")
    a = ap.parse_args()
    for p in build(force=a.force, verbose_ptxas=a.verbose_ptxas):
        print("built", p)


if __name__ == "__main__":
    main()
