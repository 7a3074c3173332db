"""Short rows (N <= 2048) run on a persistent grid: one CTA per SM walks several work items, with
every barrier phase carried from one item to the next (Q buffer reuse, S / P / P.V counts, the
K/V ring). These shapes give each CTA three to four items, for every variant, head dim and
mask, including a ragged N whose last row block has a single query tile; each result is
checked against the fp32 torch reference of every head, and repeated launches must agree
bit for bit."""

import pytest
import torch

import fa
from fa.synthetic import make_qkv

from parity import check_tolerance, gpu_reference

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("variant", ["baseline", "opt", "fp16acc"])
@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("n", [1024, 1900])
def test_persistent_items_match_reference(variant, d, causal, n):
    b, h = 8, 16  # 4 (N = 1024) or 8 (N = 1900) row blocks x 128 heads: 512-1024 items
    q, k, v = make_qkv(b, h, n, d, seed=31 + d + n, scale=1.0)
    q, k, v = q.cuda(), k.cuda(), v.cuda()
    out = fa.forward_variant(q, k, v, causal=causal, variant=variant)
    ref = gpu_reference(q, k, v, causal)
    check_tolerance(out, ref, variant, label=f"{variant} d{d} causal={causal} N{n}")
    again = fa.forward_variant(q, k, v, causal=causal, variant=variant)
    assert torch.equal(out, again)
