"""Host-side behaviour of the Python API that needs no GPU: the public surface of the reference
package, the first validation step, the synthetic inputs and the FLOP count."""

import pytest
import torch

import fa
from fa.synthetic import CONFIGS, attention_flops, cfg4_cases, make_qkv, outlier_channels


def test_public_surface_matches_reference():
    for name in ("forward", "forward_variant", "attention_reference"):
        assert callable(getattr(fa, name))
    import inspect

    sig = inspect.signature(fa.forward)
    assert list(sig.parameters) == ["q", "k", "v", "causal", "softmax_scale", "fp16_accum"]
    assert sig.parameters["causal"].default is False
    assert sig.parameters["softmax_scale"].default is None
    assert sig.parameters["fp16_accum"].default is False
    sig = inspect.signature(fa.forward_variant)
    assert list(sig.parameters) == ["q", "k", "v", "causal", "variant"]
    assert sig.parameters["variant"].default == "opt"
    sig = inspect.signature(fa._C.forward)
    assert list(sig.parameters) == ["q", "k", "v", "causal", "softmax_scale", "variant"]


def test_cpu_tensors_rejected():
    q = torch.zeros(1, 1, 64, 64, dtype=torch.float16)
    with pytest.raises(RuntimeError, match="CUDA"):
        fa.forward(q, q, q)


def test_attention_reference_runs_on_cpu():
    q, k, v = make_qkv(1, 2, 33, 64, seed=1)
    out = fa.attention_reference(q, k, v, causal=True)
    assert out.dtype == torch.float32 and out.shape == q.shape
    torch.testing.assert_close(out[0, :, 0], v[0, :, 0].float())


def test_outlier_channel_rule():
    assert outlier_channels(64) == 1 and outlier_channels(128) == 1
    q0, k0, v0 = make_qkv(1, 1, 8, 64, seed=4)
    q1, k1, v1 = make_qkv(1, 1, 8, 64, seed=4, outliers=True)
    torch.testing.assert_close(q1[..., 0].float(), (q0[..., 0].float() * 8).half().float(), atol=0, rtol=0)
    assert torch.equal(q1[..., 1:], q0[..., 1:]) and torch.equal(v1, v0)


def test_flops_formula():
    assert attention_flops(4, 16, 4096, 128, True) == 4 * 4 * 16 * 4096 * 4096 * 128 / 2
    assert attention_flops(1, 1, 10, 64, False) == 4 * 100 * 64


def test_config_table():
    assert CONFIGS["cfg1"] == dict(b=4, h=16, n=4096, d=128, causal=True, seed=1, scale=1.0)
    assert len(cfg4_cases()) == 16 and all(c["b"] * c["h"] == 256 for c in cfg4_cases())


def test_forward_host_validates_before_touching_a_gpu():
    import fa

    q = torch.zeros(1, 1, 8, 64, dtype=torch.float16)
    with pytest.raises(RuntimeError, match="float16"):
        fa.forward_host(q.float(), q, q)
    with pytest.raises(RuntimeError, match="same shape"):
        fa.forward_host(q, q[:, :, :4].contiguous(), q)
    with pytest.raises(RuntimeError, match="out must be"):
        fa.forward_host(q, q, q, out=torch.zeros(1, 1, 8, 32, dtype=torch.float16))


def test_forward_host_empty_sequence_needs_no_gpu():
    import fa

    q = torch.zeros(2, 3, 0, 64, dtype=torch.float16)
    out = fa.forward_host(q, q, q)
    assert out.shape == q.shape


def test_bf16_inputs_validate_before_touching_a_gpu():
    import fa

    q = torch.zeros(1, 1, 8, 64, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="same dtype"):
        fa.forward_host(q, q.half(), q)
    out = fa.forward_host(torch.zeros(2, 3, 0, 64, dtype=torch.bfloat16), torch.zeros(2, 3, 0, 64, dtype=torch.bfloat16),
                          torch.zeros(2, 3, 0, 64, dtype=torch.bfloat16))
    assert out.dtype == torch.bfloat16 and out.shape == (2, 3, 0, 64)


def test_make_qkv_bf16_rounds_the_same_draws():
    from fa.synthetic import make_qkv

    qh, kh, vh = make_qkv(1, 2, 16, 64, seed=3)
    qb, kb, vb = make_qkv(1, 2, 16, 64, seed=3, dtype=torch.bfloat16)
    assert qb.dtype == torch.bfloat16
    # both are roundings of the same fp32 values: within bf16's half ulp of the fp16 values
    assert float((qb.float() - qh.float()).abs().max()) <= 2.0**-8 * float(qh.float().abs().max())
