"""The parity helpers themselves (no GPU): the literal-bound report of tests/parity.py."""

import warnings

import torch

from parity import LITERAL_MISSES, MAX_ABS_FP32, LiteralBoundMiss, check_tolerance


def test_literal_bound_miss_is_reported():
    # One exact value just below the midpoint between two fp16 neighbours in [4, 8) (spacing
    # 3.9e-3): rounding it to fp16 already costs ~1.95e-3; the rest of the tile is exact.
    ref = torch.zeros(16, 64, dtype=torch.float32)
    ref[3, 5] = 4.0 + 0.00195
    out = ref.half().float()
    out[3, 5] -= 1.0e-4  # away from the exact value: within floor + slack, above 2e-3
    before = len(LITERAL_MISSES)
    with warnings.catch_warnings(record=True) as rec:
        warnings.simplefilter("always")
        mx, _ = check_tolerance(out, ref, "opt", "planted case")
    assert mx > MAX_ABS_FP32
    assert any(issubclass(w.category, LiteralBoundMiss) and "planted case" in str(w.message) for w in rec)
    assert len(LITERAL_MISSES) == before + 1


def test_literal_bound_met_reports_nothing():
    ref = torch.linspace(-1, 1, 64).reshape(8, 8)
    out = ref.half().float()
    with warnings.catch_warnings(record=True) as rec:
        warnings.simplefilter("always")
        check_tolerance(out, ref, "opt", "clean case")
    assert not any(issubclass(w.category, LiteralBoundMiss) for w in rec)


def test_fp8_emulation_tracks_exact_attention():
    """The fp8 emulated reference (tests/parity.py) against exact attention of the same e4m3
    values: differences are P's e4m3 rounding only (relative RMS a few percent), and with every
    p exactly representable (q = 0: all p = 2^(8 - threshold)) it is exact up to fp32."""
    import torch

    import fa
    from fa.reference import attention_reference
    from parity import fp8_emulated_reference

    g = torch.Generator().manual_seed(3)
    q, k, v = (torch.randn(1, 2, 300, 128, generator=g) for _ in range(3))
    (q8, qs), (k8, ks), (v8, vs) = fa.quantize_fp8(q), fa.quantize_fp8(k), fa.quantize_fp8(v)
    for causal in (False, True):
        for variant in ("opt", "baseline"):
            em = fp8_emulated_reference(q8, k8, v8, qs, ks, vs, causal, variant)
            ex = attention_reference(q8.float() * qs, k8.float() * ks, v8.float() * vs, causal)
            rms = float(((em - ex) ** 2).mean().sqrt() / (ex**2).mean().sqrt())
            assert rms < 5e-2, (causal, variant, rms)
    zq = torch.zeros_like(q8)
    em = fp8_emulated_reference(zq, k8, v8, 1.0, ks, vs, False)
    ex = (v8.float() * vs).mean(dim=2, keepdim=True).expand_as(em)
    assert float((em - ex).abs().max()) < 1e-5
