"""Split-KV (fa.forward_splitkv, fa_flash_fwd_splitkv): each row block's key range cut into
num_splits ranges whose partial results are merged by a second kernel. Checked against the fp32
torch reference with the north_star tolerances, against the unsplit kernel, for determinism, and
on ranges that hold no keys for some row blocks (causal, more splits than key tiles)."""

import pytest
import torch

import fa
from fa import _C
from fa.synthetic import make_qkv
from parity import check_tolerance, err_stats, gpu_reference

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda:0")


def _dev(b, h, n, d, seed, scale=1.0):
    return [t.to(DEV) for t in make_qkv(b, h, n, d, seed, scale=scale)]


@pytest.mark.parametrize("n", [300, 1000, 2048, 4097])
@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("splits", [2, 3, 7])
def test_splitkv_matches_reference(n, d, causal, splits):
    q, k, v = _dev(1, 3, n, d, seed=11)
    out = fa.forward_splitkv(q, k, v, causal=causal, num_splits=splits)
    ref = gpu_reference(q, k, v, causal)
    check_tolerance(out, ref, "opt", f"n={n} d={d} causal={causal} splits={splits}")
    # against the unsplit kernel: same algorithm, merged in another order
    base = fa.forward_splitkv(q, k, v, causal=causal, num_splits=1)
    mx, _ = err_stats(out, base)
    assert mx <= 2e-3


@pytest.mark.parametrize("variant", ["baseline", "opt", "fp16acc"])
@pytest.mark.parametrize("d", [64, 128])
def test_splitkv_variants(variant, d):
    q, k, v = _dev(2, 2, 1500, d, seed=12)
    out = _C.forward_splitkv(q, k, v, True, None, variant, 4)
    ref = gpu_reference(q, k, v, True)
    check_tolerance(out, ref, variant, f"{variant} d={d}")


def test_splitkv_more_splits_than_tiles():
    # N = 300 has 3 key tiles: ranges 3..15 are empty for every row block.
    q, k, v = _dev(1, 2, 300, 128, seed=13)
    for causal in (False, True):
        out = fa.forward_splitkv(q, k, v, causal=causal, num_splits=16)
        check_tolerance(out, gpu_reference(q, k, v, causal), "opt", f"causal={causal}")


def test_splitkv_deterministic_and_scale():
    q, k, v = _dev(1, 2, 3000, 64, seed=14)
    a = fa.forward_splitkv(q, k, v, causal=True, softmax_scale=0.05, num_splits=5)
    b = fa.forward_splitkv(q, k, v, causal=True, softmax_scale=0.05, num_splits=5)
    assert torch.equal(a, b)
    # custom scale: scaling q by s/(1/sqrt(d)) under the default scale is the same problem
    ref = gpu_reference((q.float() * (0.05 * 8.0)).half(), k, v, True)
    check_tolerance(a, ref, "opt", "scale 0.05")


def test_forward_chooses_splits_for_few_heads():
    q, k, v = _dev(1, 1, 8192, 128, seed=15)
    params = _C.make_params(q, k, v, torch.empty_like(q), False, 128 ** -0.5, 1)
    splits = _C.choose_splits(params, q.device)
    assert splits > 1  # 32 row blocks on 148 SMs
    out = fa.forward(q, k, v)
    assert torch.equal(out, fa.forward_splitkv(q, k, v, num_splits=splits))
    check_tolerance(out, gpu_reference(q, k, v, False), "opt", "auto split")
    assert _C.device_status(0, clear=True) == 0
