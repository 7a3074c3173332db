"""Building-block probe of the sm_100a data path (libfa_selftest.so): TMA 3-D loads into
128-byte-swizzled smem, K-major / MN-major UMMA descriptors, tcgen05.mma SS and TS, the fp16
accumulator cell layout in TMEM, tcgen05.ld/st and the swizzled TMA store. Small-integer inputs
make every expected value exact, so the comparisons are exact (as in the reference's
tests/cpp/test_ptx.cu exact-equality layout tests)."""

import ctypes
from pathlib import Path

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

LIB = Path(__file__).resolve().parent.parent / "flash-attention-from-scratch_b200" / "fa" / "libfa_selftest.so"


def _lib():
    lib = ctypes.CDLL(str(LIB))
    lib.fa_selftest_umma.argtypes = [ctypes.c_void_p] * 9 + [ctypes.c_int]
    lib.fa_selftest_umma.restype = ctypes.c_int
    lib.fa_selftest_error.restype = ctypes.c_char_p
    return lib


@pytest.mark.parametrize("d", [64, 128])
def test_umma_probe_exact(d):
    g = torch.Generator().manual_seed(100 + d)
    q = torch.randint(-2, 3, (128, d), generator=g).half()
    k = torch.randint(-2, 3, (128, d), generator=g).half()
    v = torch.randint(-2, 3, (128, d), generator=g).half()
    p = (torch.randint(0, 3, (128, 128), generator=g).float() * 0.5).half()
    dev = torch.device("cuda:0")
    qd, kd, vd, pd = (t.to(dev).contiguous() for t in (q, k, v, p))
    s_out = torch.full((128, 128), float("nan"), device=dev)
    o_out = torch.full((128, d), float("nan"), device=dev)
    o16 = torch.zeros((128, d), dtype=torch.int32, device=dev)
    o_half = torch.zeros((128, d), dtype=torch.float16, device=dev)
    flags = torch.zeros(2, dtype=torch.int32, device=dev)
    lib = _lib()
    rc = lib.fa_selftest_umma(
        qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), pd.data_ptr(), s_out.data_ptr(), o_out.data_ptr(),
        o16.data_ptr(), o_half.data_ptr(), flags.data_ptr(), d,
    )
    assert rc == 0, lib.fa_selftest_error().decode()
    assert flags.tolist() == [1, 1]
    s_ref = q.float() @ k.float().T
    o_ref = p.float() @ v.float()
    s_got = s_out.cpu()
    o_got = o_out.cpu()
    # Diagnose before asserting: which operand layout is off.
    assert torch.equal(s_got, s_ref), f"S = Q K^T mismatch: max err {(s_got - s_ref).abs().max()}"
    assert torch.equal(o_got, o_ref), f"O = P V (fp32 acc) mismatch: max err {(o_got - o_ref).abs().max()}"
    cells = o16.cpu().numpy().view(np.uint32)
    lo = (cells & 0xFFFF).astype(np.uint16).view(np.float16).astype(np.float32)
    hi = (cells >> 16).astype(np.uint16).view(np.float16).astype(np.float32)
    lo_ok = np.array_equal(lo, o_ref.numpy())
    hi_ok = np.array_equal(hi, o_ref.numpy())
    assert lo_ok, f"fp16 accumulator not in the low half of each TMEM cell (high half matches: {hi_ok})"
    assert torch.equal(o_half.cpu().float(), o_ref), "TMA store of the swizzled fp16 tile mismatch"


def test_exp2_implementations_error_bounds():
    """The kernel's software 2^x (exp2_poly2, degree-4 minimax polynomial) and the SFU
    ex2.approx, against exp2 in double, over the range the softmax uses ([-126, 8] plus the
    masked -inf). Bound for the polynomial: 2.9e-6 fitted + float32 rounding; both far below the
    fp16 rounding (4.9e-4) applied to P afterwards."""
    lib = ctypes.CDLL(str(LIB))
    lib.fa_selftest_exp2.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_int]
    lib.fa_selftest_error.restype = ctypes.c_char_p
    x = torch.cat([torch.linspace(-126.0, 8.0, 1 << 20), torch.tensor([0.0, 1.0, -1.0, 8.0, -0.5, 0.5, float("-inf"), -200.0])])
    x = x[: (x.numel() // 2) * 2].float()
    xd = x.cuda()
    poly = torch.empty_like(xd)
    sfu = torch.empty_like(xd)
    assert lib.fa_selftest_exp2(xd.data_ptr(), poly.data_ptr(), sfu.data_ptr(), xd.numel()) == 0, lib.fa_selftest_error()
    exact = torch.exp2(x.double())
    fin = x >= -126.0
    rel_poly = ((poly.cpu().double() - exact) / exact)[fin].abs().max().item()
    big = x > -100.0  # ex2.approx.ftz flushes results below 2^-126
    rel_sfu = ((sfu.cpu().double() - exact) / exact)[big].abs().max().item()
    assert rel_poly < 4e-6, rel_poly
    assert rel_sfu < 4e-6, rel_sfu
    # exact powers of two and the masked entries
    p = poly.cpu()
    assert p[x == 0.0].eq(1.0).all() and p[x == 1.0].eq(2.0).all() and p[x == -1.0].eq(0.5).all()
    assert (p[~fin] < 1e-37).all() and (p[~fin] >= 0).all()
    assert (p[~fin].half() == 0).all()


def test_exp2_degree3_error_bound():
    """The degree-3 software 2^x (exp2_poly2_deg3, used for 1 of 8 pairs at d = 128): max
    relative error 1.0e-4 fitted (float32 Horner adds a little), below the 2.4e-4 worst relative
    rounding of the fp16 value it feeds; exact at powers of two; 0 for masked scores."""
    lib = ctypes.CDLL(str(LIB))
    lib.fa_selftest_exp2_deg3.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int]
    lib.fa_selftest_error.restype = ctypes.c_char_p
    x = torch.cat([torch.linspace(-126.0, 8.0, 1 << 20), torch.tensor([0.0, 1.0, -1.0, 8.0, float("-inf"), -200.0])]).float()
    xd = x.cuda()
    poly = torch.empty_like(xd)
    assert lib.fa_selftest_exp2_deg3(xd.data_ptr(), poly.data_ptr(), xd.numel()) == 0, lib.fa_selftest_error()
    exact = torch.exp2(x.double())
    fin = x >= -126.0
    rel = ((poly.cpu().double() - exact) / exact)[fin].abs().max().item()
    assert rel < 1.2e-4, rel
    p = poly.cpu()
    assert p[x == 0.0].eq(1.0).all() and p[x == 1.0].eq(2.0).all() and p[x == -1.0].eq(0.5).all()
    assert (p[~fin].half() == 0).all() and (p[~fin] >= 0).all()


def test_bounded_wait_times_out_without_fault():
    """Failure detection on the GPU without a fault: the kernels' bounded mbarrier wait, on a
    barrier nothing arrives on, gives up after its time limit (1 s), records its code in the
    status word and returns; the CUDA context stays usable afterwards."""
    import time

    lib = ctypes.CDLL(str(LIB))
    lib.fa_selftest_watchdog.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
    lib.fa_selftest_error.restype = ctypes.c_char_p
    flags = torch.zeros(2, dtype=torch.int32, device="cuda")
    code = ctypes.c_uint32(0)
    t0 = time.time()
    rc = lib.fa_selftest_watchdog(flags.data_ptr(), ctypes.byref(code))
    elapsed = time.time() - t0
    assert rc == 0, lib.fa_selftest_error()
    assert flags.tolist() == [1, 1]
    assert code.value == 1 << 2  # kStatusTimeoutSoftmax
    assert 0.9 < elapsed < 30.0
    # the context is still healthy: run the real kernel
    import fa
    from fa.synthetic import make_qkv

    q, k, v = (t.cuda() for t in make_qkv(1, 1, 64, 64, seed=1))
    assert torch.isfinite(fa.forward(q, k, v)).all()
    assert fa._C.device_status(0, clear=True) == 0
