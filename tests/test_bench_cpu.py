"""bench.py's host logic without a GPU: the reference arm runs the reference's CPU path
without importing the product package, on the same workload and `config` as the repo's arm."""

import json
import subprocess
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(REPO))

import bench  # noqa: E402
from fa.shard import plan_shards  # noqa: E402


@pytest.mark.parametrize("total,world", [(64, 1), (64, 2), (64, 8), (10, 4), (3, 8)])
def test_bench_shards_match_plan_shards(total, world):
    assert bench.shard_ranges(total, world) == [(s.start, s.stop) for s in plan_shards(total, world)]


def test_config_identical_across_arms_and_sizes():
    c = bench.workload("cfg3")
    assert bench.config_dict(c, 8) == bench.config_dict(bench.workload("cfg3"), 8)
    assert bench.config_dict(c, 8)["heads_per_gpu"] == [8] * 8
    assert bench.flops_of(c) == 4.0 * 64 * 16384 * 16384 * 128 / 2


def test_reference_arm_loads_no_product_library():
    """One small step of --impl reference in a fresh interpreter: the product package `fa` is
    never imported and libfa_b200.so is never mapped; the line carries the repo arm's config."""
    code = (
        "import sys, json\n"
        "sys.argv = ['bench.py', '--impl', 'reference', '--steps', '1', '--warmup', '0',"
        " '--workload', 'shape:1:2:256:64:1']\n"
        "import bench\n"
        "bench.main()\n"
        "maps = open('/proc/self/maps').read()\n"
        "assert 'fa' not in sys.modules, 'fa imported'\n"
        "assert 'libfa_b200' not in maps, 'product library mapped'\n"
    )
    res = subprocess.run([sys.executable, "-c", code], cwd=REPO, capture_output=True, text=True, timeout=300)
    assert res.returncode == 0, res.stdout + res.stderr
    line = json.loads(res.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference"
    c = bench.workload("shape:1:2:256:64:1")
    assert line["config"] == bench.config_dict(c, 1)
    assert line["cpu_baseline"]["kind"] in ("reference", "port")
    if (REPO / "oracle" / "_ref" / "attention_reference.pt").exists():
        assert line["cpu_baseline"]["kind"] == "reference"
    assert line["e2e"]["h2d_bytes_per_step"] == 0


def test_compiled_reference_matches_oracle():
    """The TorchScript build of the reference's attention_reference (oracle/_ref/) against the
    numpy restatement, when it has been built here."""
    ref = bench._compiled_reference()
    if ref is None:
        pytest.skip("oracle/_ref/attention_reference.pt not built (no reference checkout)")
    import numpy as np
    import torch

    from oracle import attention as oracle

    q, k, v = bench.synthetic().make_head_qkv(range(2), 77, 64, 9)
    for causal in (False, True):
        got = ref(q, k, v, causal).numpy()
        want = oracle.attention(q.numpy(), k.numpy(), v.numpy(), causal=causal)
        np.testing.assert_allclose(got, want, atol=2e-6, rtol=0)
