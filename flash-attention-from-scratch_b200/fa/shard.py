"""Multi-GPU head sharding for the forward pass (no collective).

Every (b, h) head is a complete attention problem (the reference's grid.y = B*H,
csrc/kernels/flash_fwd.cu:571-572), so a multi-GPU run splits the flattened B*H heads into
contiguous, balanced ranges, one per GPU. A contiguous range of heads is a contiguous slice of
a [B*H, N, d] tensor, so shards need no repacking; each shard runs as a (1, heads_i, N, d)
problem on its own GPU, outputs stay on their owner, and gathering them to one device is done
only for verification.

Two launch styles share ``plan_shards``:
  * one process driving several GPUs: ``forward_sharded`` (one C-ABI call,
    fa_flash_fwd_sharded, enqueues every shard on its device's current stream);
  * one process per GPU (torchrun): each rank takes ``plan_shards(...)[rank]``.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class Shard:
    """Heads [start, stop) of the flattened B*H head list."""

    rank: int
    start: int
    stop: int

    @property
    def heads(self) -> int:
        return self.stop - self.start


def plan_shards(total_heads: int, world: int) -> list[Shard]:
    """Balanced contiguous split: the first total_heads % world shards get one extra head."""
    if total_heads < 0 or world <= 0:
        raise ValueError("plan_shards: total_heads must be >= 0 and world > 0")
    base, extra = divmod(total_heads, world)
    out, start = [], 0
    for r in range(world):
        n = base + (1 if r < extra else 0)
        out.append(Shard(r, start, start + n))
        start += n
    return out


def split_heads(x: torch.Tensor, shards: list[Shard], devices: list[torch.device]) -> list[torch.Tensor]:
    """[B, H, N, d] -> per-shard (1, heads_i, N, d) tensors placed on their devices."""
    b, h, n, d = x.shape
    flat = x.reshape(1, b * h, n, d)
    return [flat[:, s.start : s.stop].to(dev, non_blocking=False).contiguous() for s, dev in zip(shards, devices)]


def gather_heads(parts: list[torch.Tensor], shape: torch.Size, device: torch.device) -> torch.Tensor:
    """Inverse of split_heads, on one device (verification only)."""
    return torch.cat([p.to(device) for p in parts], dim=1).reshape(shape)


def forward_sharded(
    q_parts: list[torch.Tensor],
    k_parts: list[torch.Tensor],
    v_parts: list[torch.Tensor],
    causal: bool = False,
    softmax_scale: float | None = None,
    variant: str = "opt",
) -> list[torch.Tensor]:
    """Runs every shard on its own GPU with one launcher call; returns the per-shard outputs.

    Each q_parts[i], k_parts[i], v_parts[i] is a [b_i, h_i, N, d] fp16 CUDA tensor on one device
    (see split_heads). The call is asynchronous on each device's current stream. Shards run
    unsplit (one range of keys per row block, as fa.forward_splitkv(..., num_splits=1)): a
    shard is a slice of a workload large enough to be spread over GPUs.
    """
    from fa import _C  # local: keeps plan_shards importable for host-only tests

    if not (len(q_parts) == len(k_parts) == len(v_parts)):
        raise RuntimeError("forward_sharded: q, k, v shard lists differ in length")
    vid = _C.parse_variant(variant)
    outs, params, devs, streams = [], [], [], []
    for q, k, v in zip(q_parts, k_parts, v_parts):
        _C.check_inputs(q, k, v)
        with torch.cuda.device(q.device):
            o = torch.empty_like(q)
        outs.append(o)
        if q.shape[2] == 0 or q.numel() == 0:
            continue
        scale = softmax_scale if softmax_scale is not None else q.shape[3] ** -0.5
        params.append(_C.make_params(q, k, v, o, causal, scale, vid))
        devs.append(q.device.index)
        streams.append(torch.cuda.current_stream(q.device).cuda_stream)
    if params:
        n = len(params)
        arr = (_C.FaFwdParams * n)(*params)
        dev_arr = (ctypes.c_int32 * n)(*devs)
        st_arr = (ctypes.c_void_p * n)(*streams)
        rc = _C.lib.fa_flash_fwd_sharded(arr, dev_arr, st_arr, n)
        if rc != _C.FA_OK:
            _C._raise(rc)
    return outs
