"""Seeded synthetic inputs for the benchmark configurations and the tests.

One CPU generator ``torch.Generator().manual_seed(seed)``; q, then k, then v drawn as fp32
``torch.randn``; multiplied by ``scale``; optionally an outlier channel block of q and k
multiplied by ``outlier_factor``; then rounded to fp16. Drawing on the CPU makes the bits
identical on every machine and lets the CPU oracle see exactly what the GPU sees.

Outliers ("1% outlier channel scaled x8" of the ragged sweep): channels
[0, max(1, round(0.01 * d))) of q and k, i.e. channel 0 for d = 64 and d = 128.
"""

from __future__ import annotations

import torch


def outlier_channels(d: int) -> int:
    return max(1, round(0.01 * d))


def make_qkv(
    b: int,
    h: int,
    n: int,
    d: int,
    seed: int,
    scale: float = 1.0,
    outliers: bool = False,
    outlier_factor: float = 8.0,
    dtype: torch.dtype = torch.float16,
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """CPU q, k, v of shape [b, h, n, d], rounded to `dtype` (fp16, or bf16 for the bfloat16
    path) from the same fp32 draws."""
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(b, h, n, d, generator=g) * scale
    k = torch.randn(b, h, n, d, generator=g) * scale
    v = torch.randn(b, h, n, d, generator=g) * scale
    if outliers:
        c = outlier_channels(d)
        q[..., :c] *= outlier_factor
        k[..., :c] *= outlier_factor
    return q.to(dtype), k.to(dtype), v.to(dtype)


def make_head_qkv(
    heads: range,
    n: int,
    d: int,
    seed: int,
    scale: float = 1.0,
    outliers: bool = False,
    outlier_factor: float = 8.0,
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """CPU fp16 q, k, v of shape [1, len(heads), n, d]: head h of a workload drawn from its own
    generator seeded with seed * 65536 + h (q, then k, then v), with the same value scale and
    outliers as make_qkv. A shard of a workload's heads is generated without drawing the other
    heads, and a head's values do not depend on how the heads are sharded."""
    out = [torch.empty(1, len(heads), n, d, dtype=torch.float16) for _ in range(3)]
    for i, h in enumerate(heads):
        g = torch.Generator().manual_seed(seed * 65536 + h)
        for t in out:
            x = torch.randn(n, d, generator=g) * scale
            if outliers and t is not out[2]:
                x[:, : outlier_channels(d)] *= outlier_factor
            t[0, i] = x.half()
    return out[0], out[1], out[2]


# BASELINE.json configs (shapes, seeds, value scales). cfg0 is the CPU anchor.
CONFIGS = {
    "cfg0": dict(b=1, h=4, n=512, d=64, causal=False, seed=0, scale=1.0),
    "cfg1": dict(b=4, h=16, n=4096, d=128, causal=True, seed=1, scale=1.0),
    "cfg2": dict(b=8, h=32, n=8192, d=64, causal=False, seed=2, scale=1.0),
    "cfg3": dict(b=2, h=32, n=16384, d=128, causal=True, seed=3, scale=0.5),
    "cfg3nc": dict(b=2, h=32, n=16384, d=128, causal=False, seed=3, scale=0.5),
}


def cfg4_cases() -> list[dict]:
    """Ragged sweep: B16 H16, N in {1000, 3000, 8191, 12345} x d x causal, seed 4, outliers."""
    out = []
    for n in (1000, 3000, 8191, 12345):
        for d in (64, 128):
            for causal in (False, True):
                out.append(dict(b=16, h=16, n=n, d=d, causal=causal, seed=4, scale=1.0, outliers=True))
    return out


def attention_flops(b: int, h: int, n: int, d: int, causal: bool) -> float:
    """The reference's count (bench/benchmark.py:142): 4 B H N^2 d, halved for causal."""
    return 4.0 * b * h * n * n * d / (2.0 if causal else 1.0)
