"""Fits the polynomial used by the kernel's software 2^x (fa_sm100::exp2_poly).

    python flash-attention-from-scratch_b200/csrc/fit_exp2_poly.py [degree]

The kernel computes 2^x = 2^j * 2^f with j = round(x) (the 1.5 * 2^23 rounding trick) and
f = x - j in [-1/2, 1/2], so only 2^f on [-1/2, 1/2] is approximated. The constant term is
pinned to 1 (2^0 == 1 exactly), p(f) = 1 + c1 f + ... + cn f^n.

Method: Lawson's algorithm (iteratively reweighted least squares converging to the minimax
solution) for the RELATIVE error p(f) / 2^f - 1 on Chebyshev-distributed points. Prints the
float32 coefficients and the max relative error of float32 Horner evaluation on a dense grid.
"""

from __future__ import annotations

import sys

import numpy as np


def lawson_relative(deg: int, points: int = 4000, iters: int = 400) -> np.ndarray:
    x = 0.5 * np.cos(np.pi * (np.arange(points) + 0.5) / points)
    basis = np.stack([x ** (j + 1) for j in range(deg)], axis=1) / (2.0 ** x)[:, None]
    target = (2.0 ** x - 1.0) / 2.0 ** x
    w = np.full(points, 1.0 / points)
    coef = None
    for _ in range(iters):
        sw = np.sqrt(w)
        coef, *_ = np.linalg.lstsq(basis * sw[:, None], target * sw, rcond=None)
        err = np.abs(basis @ coef - target)
        w = w * err
        w /= w.sum()
    return np.concatenate([[1.0], coef])


def horner_f32(c32: np.ndarray, f: np.ndarray) -> np.ndarray:
    p = np.full_like(f, c32[-1])
    for c in c32[-2::-1]:
        p = (p * f + c).astype(np.float32)
    return p


def main() -> None:
    deg = int(sys.argv[1]) if len(sys.argv) > 1 else 4
    c = lawson_relative(deg)
    c32 = c.astype(np.float32)
    f = np.linspace(-0.5, 0.5, 2_000_001, dtype=np.float32)
    rel = np.abs(horner_f32(c32, f).astype(np.float64) / np.exp2(f.astype(np.float64)) - 1.0)
    print(f"degree {deg}: max relative error (float32 Horner) {rel.max():.3e}")
    for i, v in enumerate(c32):
        print(f"  c{i} = {float(v)!r}f  ({v.view(np.uint32):#010x})")


if __name__ == "__main__":
    main()
