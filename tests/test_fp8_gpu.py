"""fp8 (e4m3) inputs through fa.forward_fp8 / fa_flash_fwd_fp8 (an extension: the reference lists
fp8 attention as not done, docs/fa3_fa4_techniques.md:22,132-138).

Inputs are seeded fp32 draws quantised per tensor (fa.quantize_fp8: x8 = x / s in e4m3,
s = max|x| / 448). Two references (tests/parity.py):
  * the kernel's algorithm emulated in fp32 torch (128-key tiles, the variant's lazy running
    max, P * 2^(8 - threshold) rounded to e4m3, sums of the rounded P): max-abs <= 2e-2 and
    mean-abs <= 2e-4 (a p within ~1e-4 of an e4m3 rounding midpoint may round the other way in
    the kernel, whose fp32 sums run in another order; the emulation computes the kernel's
    polynomial 2^x on the same columns; the rows a flip moves most are causal rows with few
    keys);
  * exact fp32 attention of the dequantized inputs: relative RMS error <= 5e-2, mean-abs <= 1e-2
    (P's e4m3 rounding costs up to 2^-4 relative per element; measured: 1.5-2.6% RMS, mean-abs
    <= 4.1e-3)."""

import math

import pytest
import torch

import fa
from fa.synthetic import CONFIGS, make_qkv
from parity import err_stats, fp8_emulated_reference, fp8_exact_reference

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda:0")
MAX_ABS_EMUL = 2e-2
MEAN_ABS_EMUL = 2e-4
REL_RMS_EXACT = 5e-2
MEAN_ABS_EXACT = 1e-2


def _inputs(b, h, n, seed=0, scale=1.0, outliers=False):
    q, k, v = (t.to(DEV) for t in make_qkv(b, h, n, 128, seed, scale=scale, outliers=outliers, dtype=torch.float32))
    return fa.quantize_fp8(q), fa.quantize_fp8(k), fa.quantize_fp8(v)


def _check(o, q8, k8, v8, qs, ks, vs, causal, variant, label, max_emul=MAX_ABS_EMUL, mean_emul=MEAN_ABS_EMUL):
    assert o.dtype == torch.float16 and torch.isfinite(o).all(), label
    em = fp8_emulated_reference(q8, k8, v8, qs, ks, vs, causal, variant)
    mx, mean = err_stats(o, em)
    assert mx <= max_emul and mean <= mean_emul, f"{label} vs emulation: max {mx:.3e} mean {mean:.3e}"
    ex = fp8_exact_reference(q8, k8, v8, qs, ks, vs, causal)
    _, mean_x = err_stats(o, ex)
    rms = float(((o.float() - ex) ** 2).mean().sqrt() / (ex**2).mean().sqrt().clamp_min(1e-30))
    assert rms <= REL_RMS_EXACT and mean_x <= MEAN_ABS_EXACT, f"{label} vs exact: rel rms {rms:.3e} mean {mean_x:.3e}"


@pytest.mark.parametrize("n", [1, 17, 65, 257, 1000, 2048, 3000])
@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("variant", ["baseline", "opt"])
def test_fp8_matches_references(n, causal, variant):
    (q8, qs), (k8, ks), (v8, vs) = _inputs(2, 3, n, seed=n)
    o = fa.forward_fp8(q8, k8, v8, qs, ks, vs, causal=causal, variant=variant)
    _check(o, q8, k8, v8, qs, ks, vs, causal, variant, f"fp8 n={n} causal={causal} {variant}")


def test_fp8_uniform_scores_give_mean_of_v():
    """q = 0: every score is 0, every p = 2^(8 - threshold) exactly (in e4m3), O = mean(V)."""
    (_, _), (k8, ks), (v8, vs) = _inputs(1, 2, 4096, seed=6)
    q8 = torch.zeros_like(k8)
    o = fa.forward_fp8(q8, k8, v8, 1.0, ks, vs)
    want = (v8.float() * vs).mean(dim=2, keepdim=True).expand_as(o)
    torch.testing.assert_close(o.float(), want, atol=2e-3, rtol=2e-3)


def test_fp8_causal_first_row_is_v0():
    (q8, qs), (k8, ks), (v8, vs) = _inputs(1, 2, 300, seed=8)
    o = fa.forward_fp8(q8, k8, v8, qs, ks, vs, causal=True)
    torch.testing.assert_close(o[:, :, 0].float(), (v8[:, :, 0].float() * vs).half().float(), atol=0, rtol=0)


@pytest.mark.parametrize("causal", [False, True])
def test_fp8_large_logits_and_outliers(causal):
    """Scores in the hundreds (values x4) and the outlier channel (x8 on q, k channel 0): the
    lazy rule must rescale, and P stays within e4m3's range. With |scores| ~ 100 in log2 units,
    differences between the tensor cores' and torch's fp32 sums of the 128 e4m3 products move
    many p across e4m3 rounding boundaries, so the emulation is matched loosely here (measured
    on B200: max-abs 4.3e-3, mean-abs 5.6e-4) and the exact reference carries the check."""
    (q8, qs), (k8, ks), (v8, vs) = _inputs(1, 2, 1024, seed=2, scale=4.0, outliers=True)
    o = fa.forward_fp8(q8, k8, v8, qs, ks, vs, causal=causal)
    _check(o, q8, k8, v8, qs, ks, vs, causal, "opt", f"fp8 large logits causal={causal}", max_emul=5e-2,
           mean_emul=2e-3)


def test_fp8_short_rows_persistent_grid():
    """B16 H16 N1000 causal: the persistent grid (one CTA per SM walks the work items)."""
    (q8, qs), (k8, ks), (v8, vs) = _inputs(16, 16, 1000, seed=4)
    o = fa.forward_fp8(q8, k8, v8, qs, ks, vs, causal=True)
    _check(o, q8, k8, v8, qs, ks, vs, True, "opt", "fp8 B16 H16 N1000 causal")


@pytest.mark.parametrize("causal", [True, False])
def test_fp8_cfg3_sampled_heads(causal):
    """Config 3's shape (B2 H32 N16384, values x0.5): the full launch, two heads checked."""
    c = CONFIGS["cfg3"]
    (q8, qs), (k8, ks), (v8, vs) = _inputs(c["b"], c["h"], c["n"], seed=c["seed"], scale=c["scale"])
    o = fa.forward_fp8(q8, k8, v8, qs, ks, vs, causal=causal)
    for b, h in [(0, 5), (1, 30)]:
        sl = (slice(b, b + 1), slice(h, h + 1))
        _check(o[sl], q8[sl], k8[sl], v8[sl], qs, ks, vs, causal, "opt", f"fp8 cfg3 head ({b},{h})")


def test_fp8_deterministic():
    (q8, qs), (k8, ks), (v8, vs) = _inputs(2, 4, 3000, seed=10)
    a = fa.forward_fp8(q8, k8, v8, qs, ks, vs, causal=True)
    b = fa.forward_fp8(q8, k8, v8, qs, ks, vs, causal=True)
    assert torch.equal(a, b)


def test_fp8_rejections():
    (q8, qs), (k8, ks), (v8, vs) = _inputs(1, 1, 64, seed=1)
    with pytest.raises(RuntimeError, match="float8_e4m3fn"):
        fa.forward_fp8(q8.half(), k8, v8, qs, ks, vs)
    with pytest.raises(RuntimeError, match="float16"):
        fa.forward(q8, k8, v8)
    with pytest.raises(ValueError, match="descales must be positive"):
        fa.forward_fp8(q8, k8, v8, -1.0, ks, vs)
    with pytest.raises(ValueError, match="head_dim 128"):
        q64 = q8[..., :64].contiguous()
        fa.forward_fp8(q64, q64, q64, 1.0, 1.0, 1.0)
    with pytest.raises(ValueError, match="baseline or opt"):
        fa.forward_fp8(q8, k8, v8, qs, ks, vs, variant="fp16acc")
