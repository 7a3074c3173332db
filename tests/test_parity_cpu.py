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
