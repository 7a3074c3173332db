"""The reference's own CUDA kernel on the same inputs, as an accuracy yardstick.

The reference's kernel (csrc/kernels/flash_fwd.cu of aligoldenhat/flash-attention-from-scratch,
an mma.sync FlashAttention-2 kernel) is compiled unmodified for sm_100a by
baseline/build_ref_kernel.py into baseline/_ref/libfa_ref_kernel.so, a built file that travels
with the tree; the test is skipped where it was not built. On config 4's outlier rows the fp16
rounding floor is ~1.95e-3, so neither kernel meets a literal 2e-3 everywhere: this test pins
that our error is no larger than the reference kernel's for the same variant on the same bits,
against the same fp32 reference.
"""

from __future__ import annotations

import ctypes
from pathlib import Path

import pytest
import torch

import fa
from fa.synthetic import cfg4_cases, make_qkv
from parity import err_stats, fp16_floor, gpu_reference

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda:0")
LIB = Path(__file__).resolve().parent.parent / "baseline" / "_ref" / "libfa_ref_kernel.so"
# Variant numbering of the reference's fa::Variant (csrc/flash_fwd.h:12-15).
REF_VARIANT = {"baseline": 0, "opt": 1}


def _ref_kernel():
    if not LIB.exists():
        pytest.skip("baseline/_ref/libfa_ref_kernel.so not built (needs the reference sources)")
    lib = ctypes.CDLL(str(LIB))
    lib.fa_ref_kernel_fwd.restype = ctypes.c_int
    lib.fa_ref_kernel_fwd.argtypes = [ctypes.c_void_p] * 4 + [ctypes.c_int] * 4 + [
        ctypes.c_float, ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_char_p, ctypes.c_int]
    return lib


def _run_ref(lib, q, k, v, causal, variant):
    b, h, n, d = q.shape
    o = torch.empty_like(q)
    err = ctypes.create_string_buffer(256)
    rc = lib.fa_ref_kernel_fwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), b, h, n, d,
                               d ** -0.5, int(causal), REF_VARIANT[variant],
                               ctypes.c_void_p(torch.cuda.current_stream().cuda_stream), err, 256)
    assert rc == 0, err.value.decode()
    torch.cuda.synchronize()
    return o


@pytest.mark.parametrize("case", cfg4_cases(), ids=lambda c: f"N{c['n']}_d{c['d']}_{'causal' if c['causal'] else 'full'}")
def test_cfg4_error_not_above_reference_kernel(case):
    lib = _ref_kernel()
    q, k, v = make_qkv(case["b"], case["h"], case["n"], case["d"], case["seed"], scale=case["scale"], outliers=True)
    qd, kd, vd = q.to(DEV), k.to(DEV), v.to(DEV)
    ref = gpu_reference(qd, kd, vd, case["causal"])
    floor = fp16_floor(ref)
    ours_mx, ours_mean = err_stats(fa.forward_variant(qd, kd, vd, causal=case["causal"], variant="opt"), ref)
    refk_mx, refk_mean = err_stats(_run_ref(lib, qd, kd, vd, case["causal"], "opt"), ref)
    label = f"N{case['n']} d{case['d']} causal={case['causal']}: ours {ours_mx:.3e}/{ours_mean:.2e}, " \
            f"reference kernel {refk_mx:.3e}/{refk_mean:.2e}, fp16 floor {floor:.3e}"
    assert ours_mx <= refk_mx, label
    assert ours_mean <= refk_mean, label
