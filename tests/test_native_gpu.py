"""The C ABI driven from a native C program (tests/native/capi_check.c): no Python or PyTorch
between the caller and libfa_b200.so. The counterpart of the reference's standalone driver
(csrc/dev/main.cu:82-188) and GoogleTest API suite (tests/cpp/test_flash_fwd.cu:64-210)."""

import subprocess
import sys
from pathlib import Path

import pytest

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE / "native"))

from build_native import build  # noqa: E402


def _run(*args, timeout=600):
    exe = build()
    return subprocess.run([str(exe), *map(str, args)], capture_output=True, text=True, timeout=timeout)


def test_native_driver_validates_without_gpu():
    """Built with gcc against include/fa_b200.h; the library rejects bad arguments before any
    CUDA call (reference tests/cpp/test_flash_fwd.cu:64-83)."""
    res = _run("--validate-only")
    assert res.returncode == 0, res.stdout + res.stderr
    assert "validation: ok" in res.stdout


@pytest.mark.gpu
def test_native_driver_cases_match_oracle():
    """Nine shapes x variants x element types (two bf16 cases) through fa_flash_fwd and two e4m3
    cases through fa_flash_fwd_fp8 from C, each against the double-precision oracle, a bitwise
    repeat and the watchdog word."""
    res = _run()
    print(res.stdout)
    assert res.returncode == 0, res.stdout + res.stderr
    assert "all cases passed" in res.stdout


@pytest.mark.gpu
def test_native_driver_timed_case():
    """One case with timed launches (the reference driver's CLI shape: B H N D causal variant iters)."""
    res = _run(1, 4, 2048, 128, 1, 1, 10)
    print(res.stdout)
    assert res.returncode == 0, res.stdout + res.stderr
    assert "TFLOPS" in res.stdout
