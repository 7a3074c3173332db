"""Attention on host-resident tensors with the transfers overlapped with the kernels.

``forward_host`` takes q, k, v in (pinned) CPU memory and returns O in CPU memory. The heads are
cut into chunks; each chunk's host-to-device copy runs on one stream, its kernel on the device's
current stream and its device-to-host copy on a third, so the copies of one chunk overlap the
kernel of another (and PCIe carries both directions at once). Not in the reference, whose API
takes device tensors only (fa/__init__.py:14-28); the kernels are the same fa.forward kernels.
"""

from __future__ import annotations

import torch

from fa import _C

_STREAMS: dict[int, tuple[torch.cuda.Stream, torch.cuda.Stream]] = {}


def _side_streams(device: torch.device) -> tuple[torch.cuda.Stream, torch.cuda.Stream]:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    if idx not in _STREAMS:
        _STREAMS[idx] = (torch.cuda.Stream(idx), torch.cuda.Stream(idx))
    return _STREAMS[idx]


def _check_host(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> None:
    for t in (q, k, v):
        if t.is_cuda:
            raise RuntimeError("forward_host: q, k, v must be CPU tensors (use fa.forward for CUDA tensors)")
        if t.dtype not in (torch.float16, torch.bfloat16):
            raise RuntimeError("q, k, v must be float16 (or bfloat16)")
        if t.dtype != q.dtype:
            raise RuntimeError("q, k, v must have the same dtype")
        if not t.is_contiguous():
            raise RuntimeError("q, k, v must be contiguous")
        if t.dim() != 4:
            raise RuntimeError("q, k, v must have shape [B, H, N, D]")
    if q.shape != k.shape or q.shape != v.shape:
        raise RuntimeError("q, k, v must have the same shape")


def forward_host(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    causal: bool = False,
    softmax_scale: float | None = None,
    fp16_accum: bool = False,
    *,
    variant: str | None = None,
    out: torch.Tensor | None = None,
    device: torch.device | None = None,
    chunks: int | None = None,
) -> torch.Tensor:
    """O = softmax(Q K^T * scale) V for CPU q, k, v [B, H, N, D] fp16 (pin them for overlap).

    Returns O in CPU memory (``out`` if given, else a new pinned tensor). The work is queued
    behind the device's current stream, and the current stream waits for all of it: synchronize
    that stream (or the device) before reading O. ``chunks`` (default min(B*H, 8)) contiguous
    head ranges are pipelined; ``variant`` overrides fp16_accum ('baseline', 'opt', 'fp16acc')."""
    _check_host(q, k, v)
    if out is not None and (out.shape != q.shape or out.dtype != q.dtype or out.is_cuda or not out.is_contiguous()):
        raise RuntimeError("forward_host: out must be a contiguous CPU tensor like q")
    variant = variant or ("fp16acc" if fp16_accum else "opt")
    _C.parse_variant(variant)
    b, h, n, d = (int(x) for x in q.shape)
    heads = b * h
    if heads == 0 or n == 0:
        return out if out is not None else torch.empty_like(q)
    dev = device if device is not None else torch.device("cuda", torch.cuda.current_device())
    if out is None:
        out = torch.empty(q.shape, dtype=q.dtype, pin_memory=True)
    nchunks = max(1, min(heads, chunks if chunks is not None else 8))
    bounds = [(heads * i) // nchunks for i in range(nchunks + 1)]
    qv, kv, vv, ov = (t.view(heads, 1, n, d) for t in (q, k, v, out))
    cur = torch.cuda.current_stream(dev)
    s_in, s_out = _side_streams(dev)
    s_in.wait_stream(cur)
    s_out.wait_stream(cur)
    for i in range(nchunks):
        h0, h1 = bounds[i], bounds[i + 1]
        if h0 == h1:
            continue
        with torch.cuda.stream(s_in):
            qd = qv[h0:h1].to(dev, non_blocking=True)
            kd = kv[h0:h1].to(dev, non_blocking=True)
            vd = vv[h0:h1].to(dev, non_blocking=True)
        cur.wait_stream(s_in)
        for t in (qd, kd, vd):
            t.record_stream(cur)
        with torch.cuda.stream(cur):
            od = _C.forward(qd, kd, vd, causal, softmax_scale, variant)
        s_out.wait_stream(cur)
        with torch.cuda.stream(s_out):
            ov[h0:h1].copy_(od, non_blocking=True)
        od.record_stream(s_out)
    cur.wait_stream(s_out)
    return out
