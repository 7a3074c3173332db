"""Plain PyTorch attention in fp32, part of the public API as in the reference
(fa/reference.py:8-30), used to check large problems on the GPU itself.

These are ordinary torch ops (they run on whatever device the inputs are on); they are not
used by ``fa.forward``.
"""

import math

import torch


def attention_reference(
    q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool = False
) -> torch.Tensor:
    """Exact attention in float32: softmax(q k^T / sqrt(d)) v, causal mask above the diagonal."""
    qf, kf, vf = q.float(), k.float(), v.float()
    d = q.shape[-1]
    logits = torch.matmul(qf, kf.transpose(-1, -2)).mul_(1.0 / math.sqrt(d))
    if causal:
        n = q.shape[-2]
        above = torch.triu(torch.ones(n, n, dtype=torch.bool, device=q.device), diagonal=1)
        logits = logits.masked_fill(above, float("-inf"))
    return torch.matmul(torch.softmax(logits, dim=-1), vf)


def attention_naive_fp16(
    q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool = False
) -> torch.Tensor:
    """The same computation left in fp16 with the full N x N matrix materialised."""
    d = q.shape[-1]
    logits = torch.matmul(q, k.transpose(-1, -2)) * (1.0 / math.sqrt(d))
    if causal:
        n = q.shape[-2]
        above = torch.triu(torch.ones(n, n, dtype=torch.bool, device=q.device), diagonal=1)
        logits = logits.masked_fill(above, float("-inf"))
    return torch.matmul(torch.softmax(logits, dim=-1), v)
