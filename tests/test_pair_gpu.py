"""The experimental CTA-pair kernel (fa_flash_fwd_pair: two CTAs on two SMs share each
tcgen05.mma, cta_group::2) against the fp32 torch reference and against the default kernel."""

import ctypes

import pytest
import torch

import fa
from fa import _C
from fa.synthetic import make_qkv
from parity import check_tolerance, err_stats, gpu_reference

pytestmark = pytest.mark.gpu

_C.lib.fa_flash_fwd_pair.argtypes = [ctypes.POINTER(_C.FaFwdParams), ctypes.c_void_p]
_C.lib.fa_flash_fwd_pair.restype = ctypes.c_int


def _pair_forward(q, k, v, causal, variant="opt"):
    o = torch.empty_like(q)
    params = _C.make_params(q, k, v, o, causal, q.shape[3] ** -0.5, _C.parse_variant(variant))
    rc = _C.lib.fa_flash_fwd_pair(ctypes.byref(params), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    if rc != _C.FA_OK:
        _C._raise(rc)
    return o


@pytest.mark.parametrize("n", [1, 17, 129, 256, 300, 1000, 4097])
@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("variant", ["baseline", "opt"])
def test_pair_kernel_matches_reference(n, causal, variant):
    q, k, v = (t.cuda() for t in make_qkv(2, 3, n, 128, seed=50 + n))
    out = _pair_forward(q, k, v, causal, variant)
    check_tolerance(out, gpu_reference(q, k, v, causal), variant, f"pair n={n} causal={causal}")
    mx, _ = err_stats(out, fa.forward_splitkv(q, k, v, causal=causal, num_splits=1, variant=variant))
    assert mx <= 2e-3
    assert _C.device_status(0, clear=True) == 0


def test_pair_kernel_rejects_other_shapes():
    q, k, v = (t.cuda() for t in make_qkv(1, 1, 64, 64, seed=1))
    with pytest.raises(ValueError, match="head_dim 128"):
        _pair_forward(q, k, v, False)
