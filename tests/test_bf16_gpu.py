"""bfloat16 inputs (an extension: the reference takes float16 only, csrc/bindings.cpp:34, and
lists bf16 among the formats it has not built, docs/fa3_fa4_techniques.md:22,90).

The kernel is the float16 one with bfloat16 operands: Q, K, V and P are bf16 in the MMAs, the
scores, softmax statistics and O accumulate in fp32, O is rounded to bf16. The checks mirror
the float16 suite: the reference's shapes against the CPU oracle (the bf16 values widened to
fp32 exactly), the known answers, every schedule (one CTA per item, persistent grid, split-KV
and tail split), the full-size configurations against the fp32 torch reference on the GPU, and
bitwise determinism. Tolerance: the float16 bounds times 8, the ratio of the formats' unit
roundoffs (tests/parity.py)."""

import numpy as np
import pytest
import torch

import fa
from fa import _C
from fa.synthetic import CONFIGS, make_qkv
from oracle import attention as oracle
from parity import REF_ATOL, check_tolerance_bf16, gpu_reference

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda:0")
BF = torch.bfloat16


def _qkv(b, h, n, d, seed=0, scale=1.0, outliers=False):
    q, k, v = make_qkv(b, h, n, d, seed, scale=scale, outliers=outliers, dtype=BF)
    return q, k, v, q.to(DEV), k.to(DEV), v.to(DEV)


def _oracle(q, k, v, causal=False):
    f = lambda t: t.float().numpy()  # bf16 -> fp32 is exact
    return torch.from_numpy(oracle.attention(f(q), f(k), f(v), causal=causal, threads=oracle.default_threads()))


@pytest.mark.parametrize("n", [1, 17, 65, 128, 257, 1000, 2048])
@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("variant", ["baseline", "opt"])
def test_bf16_matches_oracle(n, d, causal, variant):
    q, k, v, qd, kd, vd = _qkv(2, 3, n, d)
    out = fa.forward_variant(qd, kd, vd, causal=causal, variant=variant)
    assert out.dtype == BF and out.shape == qd.shape
    ref = _oracle(q, k, v, causal=causal)
    check_tolerance_bf16(out.cpu(), ref, f"bf16 n={n} d={d} causal={causal} {variant}")


def test_bf16_matches_fp16_kernel_on_fp16_exact_inputs():
    """Inputs representable in both formats (bf16 values, those below fp16's smallest normal
    2^-14 set to 0, so that fp16's 11 significant bits hold each exactly): the two kernels see
    the same numbers and differ only by P's and O's rounding."""
    _, _, _, qd, kd, vd = _qkv(2, 4, 777, 128, seed=3)
    qd, kd, vd = (torch.where(t.abs() < 2.0**-14, torch.zeros_like(t), t) for t in (qd, kd, vd))
    for t in (qd, kd, vd):
        assert torch.equal(t.half().bfloat16(), t)
    ob = fa.forward(qd, kd, vd, causal=True).float()
    oh = fa.forward(qd.half(), kd.half(), vd.half(), causal=True).float()
    check_tolerance_bf16(ob.cpu(), oh.cpu(), "bf16 vs fp16 kernel")


@pytest.mark.parametrize("causal", [False, True])
def test_bf16_large_logits_are_stable(causal):
    q, k, v, qd, kd, vd = _qkv(1, 2, 512, 64, seed=2, scale=4.0)
    out = fa.forward(qd, kd, vd, causal=causal)
    assert torch.isfinite(out.float()).all()
    ref = _oracle(q, k, v, causal=causal)
    torch.testing.assert_close(out.float().cpu(), ref, atol=8 * REF_ATOL, rtol=8 * REF_ATOL)


@pytest.mark.parametrize("d", [64, 128])
def test_bf16_uniform_scores(d):
    """q = 0: every p = 1 and O = mean(V)."""
    _, k, v, _, kd, vd = _qkv(1, 2, 4096, d, seed=6)
    qd = torch.zeros_like(kd)
    out = fa.forward(qd, kd, vd)
    want = v.float().mean(dim=2, keepdim=True).expand_as(out)
    check_tolerance_bf16(out.float().cpu(), want, "bf16 q=0")


def test_bf16_causal_first_row_is_v0():
    _, _, v, qd, kd, vd = _qkv(1, 2, 300, 128, seed=8)
    out = fa.forward(qd, kd, vd, causal=True)
    torch.testing.assert_close(out[:, :, 0].float().cpu(), v[:, :, 0].float(), atol=0, rtol=0)


def test_bf16_huge_values_keep_range():
    """bf16's point: values far outside fp16's range (|V| ~ 1e6, |q k| scaled to stay finite)."""
    q, k, v, qd, kd, vd = _qkv(1, 2, 1000, 64, seed=9)
    v = (v.float() * 1e6).to(BF)
    out = fa.forward(qd, kd, v.to(DEV), causal=True)
    assert torch.isfinite(out.float()).all()
    ref = _oracle(q, k, v, causal=True)
    err = (out.float().cpu() - ref).abs().max() / ref.abs().max()
    assert err <= 8e-3, float(err)


def test_bf16_rejects_fp16acc_and_mixed_dtypes():
    _, _, _, qd, kd, vd = _qkv(1, 1, 64, 64)
    with pytest.raises(ValueError, match="fp16acc variant needs float16"):
        fa.forward(qd, kd, vd, fp16_accum=True)
    with pytest.raises(RuntimeError, match="same dtype"):
        fa.forward(qd, kd.half(), vd)


def test_bf16_deterministic():
    _, _, _, qd, kd, vd = _qkv(2, 4, 3000, 128, seed=10)
    a = fa.forward(qd, kd, vd, causal=True)
    b = fa.forward(qd, kd, vd, causal=True)
    assert torch.equal(a, b)


@pytest.mark.parametrize("splits", [2, 5])
@pytest.mark.parametrize("d", [64, 128])
def test_bf16_splitkv_combine(splits, d):
    """The split-KV partials are fp32; the combine kernel rounds the merged O to bf16."""
    q, k, v, qd, kd, vd = _qkv(1, 2, 4096, d, seed=11)
    out = fa.forward_splitkv(qd, kd, vd, causal=True, num_splits=splits)
    assert out.dtype == BF
    ref = _oracle(q, k, v, causal=True)
    check_tolerance_bf16(out.cpu(), ref, f"bf16 split {splits} d={d}")
    one = fa.forward_splitkv(qd, kd, vd, causal=True, num_splits=1)
    check_tolerance_bf16(out.float().cpu(), one.float().cpu(), "bf16 split vs one range")


def test_bf16_tail_split_schedule():
    """B1 H20 N8192 d128 non-causal: 640 row blocks on 148 SMs leave a partial last wave, which
    the library's schedule cuts into key ranges merged by the combine kernel."""
    _, _, _, qd, kd, vd = _qkv(1, 20, 8192, 128, seed=12)
    plan = _C.plan_params(_C.make_params(qd, kd, vd, qd, False, 1.0, 1), 148)
    assert plan["tail_blocks"] > 0 and plan["tail_splits"] > 1, plan
    out = fa.forward(qd, kd, vd)
    ref = gpu_reference(qd, kd, vd, False)
    check_tolerance_bf16(out.float(), ref, f"bf16 tail split plan {plan}")


@pytest.mark.parametrize("name", ["cfg1", "cfg2"])
def test_bf16_config_full_size(name):
    """Configs 1 and 2 with bf16 inputs, every head against the fp32 torch reference."""
    c = CONFIGS[name]
    _, _, _, qd, kd, vd = _qkv(c["b"], c["h"], c["n"], c["d"], seed=c["seed"], scale=c["scale"])
    out = fa.forward(qd, kd, vd, causal=c["causal"])
    ref = gpu_reference(qd, kd, vd, c["causal"])
    check_tolerance_bf16(out.float(), ref, f"bf16 {name}")
    del ref


@pytest.mark.parametrize("causal", [True, False])
def test_bf16_cfg3_sampled_heads(causal):
    """Config 3's shape (B2 H32 N16384 d128, values x0.5) with bf16 inputs: the full launch, four
    heads checked against the fp32 torch reference."""
    c = CONFIGS["cfg3"]
    _, _, _, qd, kd, vd = _qkv(c["b"], c["h"], c["n"], c["d"], seed=c["seed"], scale=c["scale"])
    out = fa.forward(qd, kd, vd, causal=causal)
    for b, h in [(0, 0), (0, 31), (1, 7), (1, 30)]:
        sl = (slice(b, b + 1), slice(h, h + 1))
        ref = gpu_reference(qd[sl], kd[sl], vd[sl], causal)
        check_tolerance_bf16(out[sl].float(), ref, f"bf16 cfg3 head ({b},{h}) causal={causal}")


def test_bf16_forward_host_matches_device_call():
    """Host buffers in and out (fa.forward_host). In one chunk it runs the device call's
    schedule and gives its bits; pipelined over head chunks, each chunk's few heads get their own
    schedule (split-KV ranges for few row blocks), so the sums run in another order and the
    result is checked against the oracle instead."""
    q, k, v, qd, kd, vd = _qkv(2, 5, 1000, 128, seed=13)
    want = fa.forward(qd, kd, vd, causal=True).cpu()
    qp, kp, vp = q.pin_memory(), k.pin_memory(), v.pin_memory()
    one = fa.forward_host(qp, kp, vp, causal=True, chunks=1)
    chunked = fa.forward_host(qp, kp, vp, causal=True)
    torch.cuda.synchronize()
    assert one.dtype == BF and torch.equal(one, want)
    check_tolerance_bf16(chunked.float(), _oracle(q, k, v, causal=True), "bf16 forward_host chunked")
