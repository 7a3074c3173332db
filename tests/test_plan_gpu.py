"""The library's runtime schedule on the GPU (fa.forward -> fa_flash_fwd_auto): the tail split
of a non-causal grid's partial last wave and the balanced causal head groups, each against the
fp32 reference of every head and against the unsplit kernel."""

import pytest
import torch

import fa
from fa import _C
from fa.synthetic import make_qkv
from parity import check_tolerance, gpu_reference

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def _plan(q, causal, variant):
    return _C.plan_params(_C.make_params(q, q, q, q, causal, 1.0, _C.parse_variant(variant)), 0)


@pytest.mark.parametrize("variant", ["baseline", "opt", "fp16acc"])
@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("n", [4096, 4000])
def test_tail_split_matches_reference(n, d, variant):
    # B1 H10: ceil(n / rows_per_item) * 10 row blocks; 148 SMs leave a partial last wave that the
    # planner cuts into key ranges (the ragged N = 4000 puts a short block in the tail).
    q, k, v = (t.to(DEV) for t in make_qkv(1, 10, n, d, seed=31))
    pl = _plan(q, False, variant)
    if _C._sm_count(DEV) == 148:
        assert pl["tail_blocks"] > 0, pl
    out = fa.forward_variant(q, k, v, causal=False, variant=variant)
    ref = gpu_reference(q, k, v, False)
    check_tolerance(out, ref, variant, f"tail split {pl['tail_blocks']}x{pl['tail_splits']} n={n} d={d}")
    unsplit = fa.forward_splitkv(q, k, v, causal=False, num_splits=1, variant=variant)
    bound = 1e-2 if variant == "fp16acc" else 2e-3
    assert (out.float() - unsplit.float()).abs().max().item() <= bound
    # deterministic
    assert torch.equal(out, fa.forward_variant(q, k, v, causal=False, variant=variant))


def test_tail_split_cfg3_shard_of_eight_heads():
    """A GPU's shard of config 3 at 8 GPUs (8 heads of N = 16384, non-causal)."""
    q, k, v = (t.to(DEV) for t in make_qkv(1, 8, 16384, 128, seed=3, scale=0.5))
    pl = _plan(q, False, "opt")
    out = fa.forward(q, k, v)
    ref = gpu_reference(q, k, v, False)
    check_tolerance(out, ref, "opt", f"cfg3nc shard tail {pl['tail_blocks']}x{pl['tail_splits']}")
    assert fa._C.device_status(0, clear=True) == 0


@pytest.mark.parametrize("heads", [5, 8, 13])
def test_causal_head_groups_cover_every_block(heads):
    # N = 8192 d128: 4 MiB of K and V per head; 13 heads = 52 MiB (one group) and the
    # multi-group case below both have to cover every (head, row block) exactly once.
    q, k, v = (t.to(DEV) for t in make_qkv(1, heads, 8192, 128, seed=32))
    out = fa.forward(q, k, v, causal=True)
    check_tolerance(out, gpu_reference(q, k, v, True), "opt", f"causal heads={heads}")


def test_causal_balanced_groups_many_heads():
    # 50 heads of N = 8192 d128: 200 MiB of K and V -> 4 groups of 13, 13, 12 and 12 heads.
    q, k, v = (t.to(DEV) for t in make_qkv(1, 50, 8192, 128, seed=33))
    pl = _plan(q, True, "opt")
    assert pl["head_groups"] == 4
    out = fa.forward(q, k, v, causal=True)
    check_tolerance(out, gpu_reference(q, k, v, True), "opt", "causal 50 heads, 4 groups")
