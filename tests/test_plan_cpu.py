"""The runtime schedule (fa_plan, include/fa_b200.h) on the host, no GPU: which grid, key
splits, tail split and head groups the library picks for the BASELINE shapes and the shards
of config 3. The reference fixes its schedule in a compile-time tile table
(csrc/kernels/flash_fwd.cu:596-617)."""

import pytest

from fa import _C


def plan(b, h, n, d, causal, variant="opt", sms=148):
    p = _C.FaFwdParams()
    p.q = p.k = p.v = p.o = 0x10000
    p.batch, p.heads, p.seqlen, p.head_dim = b, h, n, d
    p.softmax_scale, p.causal, p.variant = 0.1, int(causal), _C.VARIANTS[variant]
    return _C.plan_params(p, sms)


@pytest.mark.parametrize("heads", [64, 32, 16, 8])
def test_cfg3_shards_causal_single_sweep_when_kv_fits_l2(heads):
    pl = plan(1, heads, 16384, 128, True)
    assert pl["rows_per_item"] == 256 and pl["persistent"] == 0 and pl["num_splits"] == 1
    assert pl["tail_blocks"] == 0 and pl["workspace_bytes"] == 0
    assert pl["items"] == pl["ctas"] == heads * 64
    # K and V of a head: 4 N d bytes = 8 MiB; one group up to 96 MiB, else 64 MiB groups
    assert pl["head_groups"] == (1 if heads * 8 <= 96 else -(-heads * 8 // 64))


def test_cfg3_noncausal_eight_heads_splits_the_partial_last_wave():
    # 8 heads x 64 row blocks = 512 items = 3 waves of 148 + 68: the 68 tail blocks run as
    # two half-key-range items each (136 <= 148), so the last wave takes half an item.
    pl = plan(1, 8, 16384, 128, False)
    assert (pl["tail_blocks"], pl["tail_splits"]) == (68, 2)
    assert pl["items"] == 512 - 68 + 136
    assert pl["workspace_bytes"] == 68 * 2 * 256 * (128 + 2) * 4


@pytest.mark.parametrize("heads", [64, 32, 16])
def test_cfg3_noncausal_many_waves_no_tail_split(heads):
    assert plan(1, heads, 16384, 128, False)["tail_blocks"] == 0


def test_few_row_blocks_split_kv():
    pl = plan(1, 1, 16384, 128, False)
    assert pl["num_splits"] == 2 and pl["tail_blocks"] == 0
    assert plan(1, 1, 16384, 128, False, sms=256)["num_splits"] == 4


def test_short_rows_persistent_grid():
    pl = plan(16, 16, 1000, 128, True)
    assert pl["persistent"] == 1 and pl["ctas"] == 148 and pl["items"] == 4 * 256
    assert plan(16, 16, 3000, 128, True)["persistent"] == 0


def test_fp16acc_d128_one_query_tile_per_item():
    assert plan(1, 4, 4096, 128, False, "fp16acc")["rows_per_item"] == 128
    assert plan(1, 4, 4096, 64, False, "fp16acc")["rows_per_item"] == 256


@pytest.mark.parametrize("n", [3000, 4096, 8192])
def test_noncausal_rows_up_to_8192_persistent_grid(n):
    # equal-cost items: the static assignment of a persistent grid stays balanced
    pl = plan(16, 16, n, 128, False)
    assert pl["persistent"] == 1 and pl["ctas"] == 148
    assert plan(16, 16, n, 128, True)["persistent"] == (1 if n <= 2048 else 0)
    assert plan(16, 16, 8193, 128, False)["persistent"] == 0


def test_tail_split_needs_eight_key_tiles_per_piece():
    # N = 1024: 8 key tiles, a piece of half would hold 4: no tail split
    assert plan(1, 80, 1024, 128, False)["tail_blocks"] == 0
    # B1 H10 N4096: 160 row blocks = 1 wave + 12: the 12 run as 4 key ranges of 8 tiles
    pl = plan(1, 10, 4096, 128, False)
    assert (pl["tail_blocks"], pl["tail_splits"]) == (12, 4)


def test_plan_validates_like_the_forward():
    p = _C.FaFwdParams()
    p.q = p.k = p.v = p.o = 0x10000
    p.batch, p.heads, p.seqlen, p.head_dim = 1, 1, 128, 96
    with pytest.raises(ValueError, match="head_dim"):
        _C.plan_params(p, 148)
