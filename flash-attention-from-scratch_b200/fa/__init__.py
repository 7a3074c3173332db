"""FlashAttention-2 forward for NVIDIA B200 (sm_100a), written from scratch.

    import fa
    o = fa.forward(q, k, v, causal=False)      # q, k, v: [B, H, N, D] fp16 CUDA, D in {64, 128}
    o = fa.forward(q, k, v, fp16_accum=True)   # P.V accumulated in fp16 per key tile
    o = fa.forward(qb, kb, vb)                  # bfloat16 q, k, v (an extension): O in bf16
    o = fa.forward_fp8(q8, k8, v8, qs, ks, vs)  # e4m3 q, k, v with descales (an extension): fp16 O

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


def quantize_fp8(x: torch.Tensor) -> tuple[torch.Tensor, float]:
    """Per-tensor e4m3 quantisation for forward_fp8: (x / s rounded to float8_e4m3fn, s) with
    s = max|x| / 448 (e4m3's largest finite value), so that x ~ x8 * s."""
    amax = float(x.detach().abs().max()) if x.numel() > 0 else 0.0
    s = amax / 448.0 if amax > 0.0 else 1.0
    return (x.float() / s).to(torch.float8_e4m3fn), s


def forward_fp8(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    q_descale: float,
    k_descale: float,
    v_descale: float,
    causal: bool = False,
    softmax_scale: float | None = None,
    variant: str = "opt",
) -> torch.Tensor:
    """fp8 forward (not in the reference, which lists fp8 as not done): q, k, v are
    float8_e4m3fn [B, H, N, 128] holding x / descale (see quantize_fp8); returns the float16
    O = softmax(scale (q q_descale)(k k_descale)^T) (v v_descale). Scores and accumulators are
    fp32; P enters the P.V MMA as e4m3 (scaled into e4m3's range), so the result carries fp8
    rounding, unlike forward(). variant 'opt' (lazy threshold 2^4 here) or 'baseline'."""
    return _C.forward_fp8(q, k, v, q_descale, k_descale, v_descale, causal, softmax_scale, variant)


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


__all__ = ["forward", "forward_variant", "forward_splitkv", "forward_fp8", "quantize_fp8", "forward_host",
           "attention_reference", "forward_sharded", "plan_shards"]
