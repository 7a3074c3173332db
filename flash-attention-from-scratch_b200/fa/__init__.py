"""FlashAttention-2 forward for NVIDIA B200 (sm_100a), written from scratch.

    import fa
    o = fa.forward(q, k, v, causal=False)      # q, k, v: [B, H, N, D] fp16 CUDA, D in {64, 128}
    o = fa.forward(q, k, v, fp16_accum=True)   # P.V accumulated in fp16 per key tile
    o = fa.forward(qb, kb, vb)                  # bfloat16 q, k, v (an extension): O in bf16

Same public surface as the reference package (fa/__init__.py:14-38): ``forward``,
``forward_variant`` and ``attention_reference``; plus ``forward_splitkv``, ``forward_host`` (CPU
tensors in and out, transfers overlapped with the kernels) and the multi-GPU ``forward_sharded`` /
``plan_shards``. The kernel is tcgen05 / TMEM / TMA code for sm_100a in
libfa_b200.so; there is no CPU or fallback path.
"""

import torch

from fa import _C
from fa.host import forward_host
from fa.reference import attention_reference
from fa.shard import forward_sharded, plan_shards


def forward(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    causal: bool = False,
    softmax_scale: float | None = None,
    fp16_accum: bool = False,
) -> torch.Tensor:
    """O = softmax(Q K^T * scale) V.

    fp16_accum: accumulate P @ V in fp16 within each 128-key tile (folded into fp32 between
    tiles), the reference's "fp16acc" build. On B200 it runs no faster than fp32 accumulation;
    it exists for API and numerical parity. float16 inputs only.

    q, k, v may also be bfloat16 (all three; not in the reference): the same kernel with bf16
    operands and fp32 accumulation, O returned in bf16.
    """
    variant = "fp16acc" if fp16_accum else "opt"
    return _C.forward(q, k, v, causal, softmax_scale, variant)


def forward_variant(
    q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool = False, variant: str = "opt"
) -> torch.Tensor:
    """Run a specific kernel build: 'baseline', 'opt' or 'fp16acc' (benchmarks, tests)."""
    return _C.forward(q, k, v, causal, None, variant)


def forward_splitkv(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    causal: bool = False,
    softmax_scale: float | None = None,
    num_splits: int | None = None,
    variant: str = "opt",
) -> torch.Tensor:
    """forward() with each row block's key range cut into ``num_splits`` ranges that run as
    separate CTAs and are merged by a second kernel (not in the reference; it lists split-KV
    as not done). None picks the count the library would use inside forward(): 1 unless the
    row blocks leave SMs idle (few heads x long N)."""
    return _C.forward_splitkv(q, k, v, causal, softmax_scale, variant, num_splits)


__all__ = ["forward", "forward_variant", "forward_splitkv", "forward_host", "attention_reference",
           "forward_sharded", "plan_shards"]
