"""fa_flash_fwd_splitkv_static: split-KV with the partials in the library's fixed 32 MiB device
scratch instead of a caller workspace (allocates nothing). Named to be collected last, after the
rest of the suite has used the device; it also passes on its own."""

import ctypes

import pytest
import torch

import fa
from fa import _C
from fa.synthetic import make_qkv

_C.lib.fa_flash_fwd_splitkv_static.argtypes = [ctypes.POINTER(_C.FaFwdParams), ctypes.c_int32, ctypes.c_void_p]
_C.lib.fa_flash_fwd_splitkv_static.restype = ctypes.c_int

SCRATCH_BYTES = 32 << 20


def test_static_scratch_rejects_oversize_problem():
    # 128 heads x 16384 rows x 2 splits x (128 + 2) x 4 B = 2.2 GB of partials > 32 MiB;
    # the size check precedes any CUDA call (the pointers are never dereferenced).
    p = _C.FaFwdParams()
    p.q, p.k, p.v, p.o = 0x10000, 0x20000, 0x30000, 0x40000
    p.batch, p.heads, p.seqlen, p.head_dim = 8, 16, 16384, 128
    p.softmax_scale, p.causal, p.variant = 128 ** -0.5, 0, 1
    rc = _C.lib.fa_flash_fwd_splitkv_static(ctypes.byref(p), 2, None)
    assert rc == _C.FA_ERR_INVALID_ARGUMENT
    msg = _C.lib.fa_last_error().decode()
    assert "static scratch holds 33554432" in msg and "2181038080" in msg


@pytest.mark.gpu
def test_static_scratch_matches_workspace_entry_two_calls_in_a_row():
    dev = torch.device("cuda:0")
    splits = 4
    cases = [(make_qkv(1, 1, 8192, 128, seed=41), False), (make_qkv(1, 1, 8192, 128, seed=42), True)]
    stream = torch.cuda.current_stream(dev)
    outs, inputs = [], []
    for (q, k, v), causal in cases:
        qd, kd, vd = q.to(dev), k.to(dev), v.to(dev)
        o = torch.empty_like(qd)
        params = _C.make_params(qd, kd, vd, o, causal, 128 ** -0.5, 1)
        nbytes = ctypes.c_uint64(0)
        assert _C.lib.fa_splitkv_workspace_size(ctypes.byref(params), splits, ctypes.byref(nbytes)) == _C.FA_OK
        assert 0 < nbytes.value <= SCRATCH_BYTES
        # two calls in a row on one stream, no synchronisation in between
        rc = _C.lib.fa_flash_fwd_splitkv_static(ctypes.byref(params), splits, ctypes.c_void_p(stream.cuda_stream))
        assert rc == _C.FA_OK, _C.lib.fa_last_error().decode()
        outs.append(o)
        inputs.append((qd, kd, vd, causal))
    # the existing entry point (caller workspace) on the same inputs and split count
    refs = [fa.forward_splitkv(qd, kd, vd, causal=causal, num_splits=splits) for qd, kd, vd, causal in inputs]
    torch.cuda.synchronize(dev)
    for o, r in zip(outs, refs):
        assert torch.equal(o, r)
