"""The CPU oracle pinned against the reference's own outputs (tests/golden/, produced by the
reference's fa/reference.py::attention_reference), plus its known-answer properties. CPU only."""

import json
import math

import numpy as np
import pytest
import torch

from fa.synthetic import make_qkv
from oracle import attention as oracle
from oracle.build_oracle import load_f64

CASES = json.loads((__import__("pathlib").Path(__file__).parent / "golden" / "cases.json").read_text())["cases"]


def _load(golden_dir, name):
    z = np.load(golden_dir / f"{name}.npz")
    return {k: z[k] for k in z.files}


@pytest.mark.parametrize("case", CASES, ids=[c["name"] for c in CASES])
def test_oracle_matches_reference_golden(golden_dir, case):
    g = _load(golden_dir, case["name"])
    out = oracle.attention(g["q"], g["k"], g["v"], causal=case["causal"])
    np.testing.assert_allclose(out, g["out"], atol=2e-6, rtol=2e-5)


def test_oracle_matches_reference_golden_cfg0_causal(golden_dir):
    g = _load(golden_dir, "cfg0")
    out = oracle.attention(g["q"], g["k"], g["v"], causal=True)
    np.testing.assert_allclose(out, g["out_causal"], atol=2e-6, rtol=2e-5)


@pytest.mark.parametrize("case", CASES, ids=[c["name"] for c in CASES])
def test_f64_oracle_matches_reference_golden(golden_dir, case):
    g = _load(golden_dir, case["name"])
    f64 = load_f64()
    out = f64(g["q"], g["k"], g["v"], causal=case["causal"])
    # fp32 (reference) vs double: the differences are the reference's own fp32 rounding, largest
    # where the logits are large (outlier channels: |score| in the tens).
    np.testing.assert_allclose(out, g["out"], atol=3e-5, rtol=1e-4)


@pytest.mark.parametrize("case", CASES, ids=[c["name"] for c in CASES])
def test_synthetic_inputs_reproduce_golden_inputs(golden_dir, case):
    """The seeded generator reproduces the stored inputs bit for bit, so GPU tests and the bench
    can regenerate inputs of any size from (shape, seed) alone."""
    g = _load(golden_dir, case["name"])
    q, k, v = make_qkv(case["b"], case["h"], case["n"], case["d"], case["seed"], scale=case["scale"], outliers=case["outliers"])
    for name, t in (("q", q), ("k", k), ("v", v)):
        assert np.array_equal(t.numpy().view(np.uint16), g[name].view(np.uint16)), name


def test_cfg0_golden_statistics_pinned(golden_dir):
    """cfg0 statistics recorded when the reference oracle was first run (seed 0)."""
    g = _load(golden_dir, "cfg0")
    assert float(g["q"].astype(np.float64).sum()) == pytest.approx(-523.3561, abs=1e-3)
    assert float(g["k"].astype(np.float64).sum()) == pytest.approx(-365.6528, abs=1e-3)
    assert float(g["v"].astype(np.float64).sum()) == pytest.approx(-394.9726, abs=1e-3)
    out = g["out"].astype(np.float64)
    assert out.sum() == pytest.approx(-363.6109, abs=1e-3)
    assert np.abs(out).mean() == pytest.approx(0.059422, abs=1e-6)
    assert np.abs(out).max() == pytest.approx(0.433530, abs=1e-6)
    oc = g["out_causal"].astype(np.float64)
    assert oc.sum() == pytest.approx(-377.9130, abs=1e-3)
    assert np.abs(oc).mean() == pytest.approx(0.106946, abs=1e-6)
    assert np.abs(oc).max() == pytest.approx(3.066406, abs=1e-5)
    np.testing.assert_array_equal(oc[0, :, 0, :], g["v"][0, :, 0, :].astype(np.float32))


def test_oracle_uniform_scores_is_mean_of_v():
    _, k, v = make_qkv(1, 2, 300, 64, seed=6)
    q = torch.zeros_like(k)
    out = oracle.attention(q.numpy(), k.numpy(), v.numpy())
    np.testing.assert_allclose(out, np.broadcast_to(v.float().numpy().mean(axis=2, keepdims=True), out.shape), atol=1e-6)


def test_oracle_causal_first_row_is_v0():
    q, k, v = make_qkv(1, 1, 130, 64, seed=4)
    out = oracle.attention(q.numpy(), k.numpy(), v.numpy(), causal=True)
    np.testing.assert_array_equal(out[0, 0, 0], v[0, 0, 0].float().numpy())


def test_oracle_custom_scale_identity():
    """ref(q, scale) == ref(q * scale * sqrt(d)) (tests/test_flash_fwd.py:97-103 of the reference)."""
    q, k, v = make_qkv(1, 2, 200, 128, seed=3)
    a = oracle.attention(q.numpy(), k.numpy(), v.numpy(), softmax_scale=0.3)
    b = oracle.attention(q.float().numpy() * 0.3 * math.sqrt(128), k.numpy(), v.numpy())
    np.testing.assert_allclose(a, b, atol=1e-5, rtol=1e-5)


def test_oracle_chunked_threaded_equals_single_chunk():
    q, k, v = make_qkv(2, 3, 160, 64, seed=9)
    a = oracle.attention(q.numpy(), k.numpy(), v.numpy(), causal=True)
    b = oracle.attention(q.numpy(), k.numpy(), v.numpy(), causal=True, threads=4, max_chunk_bytes=160 * 160 * 4)
    np.testing.assert_array_equal(a, b)


def test_oracle_sampled_heads():
    q, k, v = make_qkv(2, 3, 64, 64, seed=9)
    full = oracle.attention(q.numpy(), k.numpy(), v.numpy()).reshape(6, 64, 64)
    part = oracle.attention_sampled_heads(q.numpy(), k.numpy(), v.numpy(), [5, 0, 3])
    np.testing.assert_array_equal(part, full[[5, 0, 3]])


def test_planted_mistake_is_caught(golden_dir):
    """A deliberately wrong oracle (mask on the diagonal too) must fail the golden check: the
    golden comparison has teeth."""
    g = _load(golden_dir, "n130_d64_causal")
    q32, k32, v32 = (g[x].astype(np.float32) for x in ("q", "k", "v"))
    s = q32 @ np.swapaxes(k32, -1, -2) / np.float32(8.0)
    s[..., np.triu(np.ones((130, 130), dtype=bool), k=0)] = -np.inf  # wrong: k=0 masks the diagonal
    s[..., 0, 0] = 0.0  # keep row 0 finite
    s -= s.max(-1, keepdims=True)
    p = np.exp(s)
    p /= p.sum(-1, keepdims=True)
    wrong = p @ v32
    assert not np.allclose(wrong, g["out"], atol=1e-3)
