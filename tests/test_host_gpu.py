"""fa.forward_host: CPU q, k, v in, CPU O out, copies overlapped with the kernels over head
chunks. Checked against fa.forward on the same data (bit-equal for one chunk) and the fp32
reference."""

import pytest
import torch

import fa
from fa.synthetic import make_qkv
from parity import check_tolerance, gpu_reference

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("chunks", [1, 3, 8])
@pytest.mark.parametrize("causal", [False, True])
def test_forward_host_matches_device_forward(chunks, causal):
    q, k, v = make_qkv(2, 5, 1000, 128, seed=61)
    qh, kh, vh = q.pin_memory(), k.pin_memory(), v.pin_memory()
    out = fa.forward_host(qh, kh, vh, causal=causal, chunks=chunks)
    torch.cuda.synchronize()
    dev = [t.cuda() for t in (q, k, v)]
    if chunks == 1:
        assert torch.equal(out, fa.forward(*dev, causal=causal).cpu())
    check_tolerance(out, gpu_reference(*dev, causal).cpu(), "opt", f"chunks={chunks}")


def test_forward_host_fp16acc_and_out():
    q, k, v = make_qkv(1, 4, 700, 64, seed=62)
    out = torch.empty_like(q).pin_memory()
    res = fa.forward_host(q.pin_memory(), k.pin_memory(), v.pin_memory(), fp16_accum=True, out=out, chunks=2)
    torch.cuda.synchronize()
    assert res.data_ptr() == out.data_ptr()
    check_tolerance(out, gpu_reference(q.cuda(), k.cuda(), v.cuda(), False).cpu(), "fp16acc", "fp16acc host")
