"""The C ABI (include/fa_b200.h) without a GPU: the library loads, exports every declared entry
point, its struct layout matches what a C compiler makes of the header, and argument validation
mirrors the reference's fa::flash_fwd (csrc/kernels/flash_fwd.cu:625-651) -- all of which runs
before any CUDA call."""

import ctypes
import re
import subprocess
from pathlib import Path

import pytest
import torch

from fa import _C

REPO = Path(__file__).resolve().parent.parent
HEADER = REPO / "include" / "fa_b200.h"


def _declared_functions():
    text = HEADER.read_text()
    return re.findall(r"FA_API\s+[\w\s\*]+?\b(fa_\w+)\s*\(", text)


def test_header_declares_entry_points():
    names = _declared_functions()
    assert set(names) >= {"fa_flash_fwd", "fa_flash_fwd_sharded", "fa_last_error", "fa_device_status", "fa_kernel_info",
                          "fa_splitkv_workspace_size", "fa_splitkv_choose", "fa_flash_fwd_splitkv"}


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(str(_C._LIB_PATH))
    for name in _declared_functions():
        assert hasattr(lib, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", str(_C._LIB_PATH)], capture_output=True, text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    assert set(_declared_functions()) <= exported


def test_params_struct_layout_matches_c_header(tmp_path):
    src = tmp_path / "layout.c"
    src.write_text(
        '#include <stdio.h>\n#include <stddef.h>\n#include "fa_b200.h"\n'
        "int main(void){printf(\"%zu %zu %zu %zu %zu %zu %zu %zu %zu %d %d\\n\", sizeof(FaFwdParams),"
        " offsetof(FaFwdParams,o), offsetof(FaFwdParams,batch), offsetof(FaFwdParams,seqlen),"
        " offsetof(FaFwdParams,head_dim), offsetof(FaFwdParams,softmax_scale),"
        " offsetof(FaFwdParams,causal), offsetof(FaFwdParams,variant), offsetof(FaFwdParams,dtype),"
        " FA_DTYPE_FLOAT16, FA_DTYPE_BFLOAT16); return 0;}\n"
    )
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-std=c99", "-I", str(REPO / "include"), "-o", str(exe), str(src)], check=True)
    got = [int(x) for x in subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split()]
    P = _C.FaFwdParams
    want = [ctypes.sizeof(P), P.o.offset, P.batch.offset, P.seqlen.offset, P.head_dim.offset,
            P.softmax_scale.offset, P.causal.offset, P.variant.offset, P.dtype.offset,
            _C.DTYPES[torch.float16], _C.DTYPES[torch.bfloat16]]
    assert got == want


def _params(**kw):
    p = _C.FaFwdParams()
    p.q, p.k, p.v, p.o = 0x10000, 0x20000, 0x30000, 0x40000  # never dereferenced: validation fails first
    p.batch, p.heads, p.seqlen, p.head_dim = 1, 1, 64, 64
    p.softmax_scale, p.causal, p.variant = 0.125, 0, 1
    for k, v in kw.items():
        setattr(p, k, v)
    return p


@pytest.mark.parametrize(
    "kw, msg",
    [
        (dict(head_dim=32), "head_dim must be 64 or 128, got 32"),
        (dict(seqlen=0), "must be positive"),
        (dict(batch=0), "must be positive"),
        (dict(batch=300, heads=300), "65535"),
        (dict(q=0x10002), "16-byte aligned"),
        (dict(variant=7), "unknown variant"),
        (dict(dtype=3), "dtype must be FA_DTYPE_FLOAT16, FA_DTYPE_BFLOAT16 or FA_DTYPE_FLOAT8_E4M3"),
        (dict(dtype=2), "float8 inputs need head_dim 128"),
        (dict(dtype=2, head_dim=128), "float8 inputs go through fa_flash_fwd_fp8"),
        (dict(dtype=1, variant=2), "fp16acc variant needs float16 inputs"),
    ],
)
def test_validation_rejects(kw, msg):
    rc = _C.lib.fa_flash_fwd(ctypes.byref(_params(**kw)), None)
    assert rc == _C.FA_ERR_INVALID_ARGUMENT
    assert msg in _C.lib.fa_last_error().decode()


def test_validation_maps_to_value_error():
    with pytest.raises(ValueError, match="head_dim"):
        _C._raise(_C.lib.fa_flash_fwd(ctypes.byref(_params(head_dim=96)), None))


def test_sharded_rejects_bad_list():
    rc = _C.lib.fa_flash_fwd_sharded(None, None, None, 3)
    assert rc == _C.FA_ERR_INVALID_ARGUMENT


@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("variant", ["baseline", "opt", "fp16acc"])
def test_kernel_info(d, variant):
    smem, threads = _C.kernel_info(d, variant)
    assert 114 * 1024 < smem <= 227 * 1024  # one CTA per SM, within the opt-in limit
    assert threads in (256, 384)  # whole warpgroups: softmax WG(s) + producer/MMA WG


def test_parse_variant_message():
    with pytest.raises(RuntimeError, match="variant must be 'opt', 'fp16acc' or 'baseline', got 'x'"):
        _C.parse_variant("x")


def test_splitkv_workspace_size_formula():
    p = _params(batch=2, heads=3, seqlen=1000, head_dim=128)
    out = ctypes.c_uint64(0)
    assert _C.lib.fa_splitkv_workspace_size(ctypes.byref(p), 4, ctypes.byref(out)) == _C.FA_OK
    rows = 1024  # ceil(1000 / 256) * 256
    assert out.value == 4 * 6 * rows * (128 + 2) * 4
    assert _C.lib.fa_splitkv_workspace_size(ctypes.byref(p), 1, ctypes.byref(out)) == _C.FA_OK
    assert out.value == 0


@pytest.mark.parametrize(
    "b,h,n,d,variant,sms,want",
    [
        (4, 16, 4096, 128, 1, 148, 1),   # 1024 row blocks: no split
        (1, 1, 16384, 128, 1, 148, 2),   # 64 row blocks
        (1, 1, 4096, 128, 1, 148, 9),    # 16 row blocks, 32 key tiles
        (1, 1, 1000, 64, 1, 148, 4),     # 4 row blocks, 8 key tiles: at least 2 tiles a range
        (1, 1, 65536, 128, 1, 148, 1),   # 256 row blocks
        (1, 1, 4096, 128, 2, 148, 4),    # fp16acc d=128: 128-row blocks (32), 32 key tiles
        (1, 1, 100000, 64, 1, 4, 1),
    ],
)
def test_splitkv_choose(b, h, n, d, variant, sms, want):
    p = _params(batch=b, heads=h, seqlen=n, head_dim=d, variant=variant)
    out = ctypes.c_int32(0)
    assert _C.lib.fa_splitkv_choose(ctypes.byref(p), sms, ctypes.byref(out)) == _C.FA_OK
    assert out.value == want


@pytest.mark.parametrize(
    "splits, ws, nbytes, msg",
    [
        (0, 0x50000, 1 << 30, "num_splits must be in 1 .. 64"),
        (65, 0x50000, 1 << 30, "num_splits must be in 1 .. 64"),
        (2, 0, 1 << 30, "workspace"),
        (2, 0x50000, 16, "workspace"),
        (2, 0x50008, 1 << 30, "16-byte aligned"),
    ],
)
def test_splitkv_validation(splits, ws, nbytes, msg):
    p = _params(seqlen=4096)
    rc = _C.lib.fa_flash_fwd_splitkv(ctypes.byref(p), splits, ctypes.c_void_p(ws), nbytes, None)
    assert rc == _C.FA_ERR_INVALID_ARGUMENT
    assert msg in _C.lib.fa_last_error().decode()


def test_fp8_entry_validates_before_any_cuda_call():
    p = _params(dtype=2, head_dim=128, batch=2, heads=3, seqlen=1000)
    out = ctypes.c_uint64(0)
    assert _C.lib.fa_fp8_workspace_size(ctypes.byref(p), ctypes.byref(out)) == _C.FA_OK
    assert out.value == 2 * 3 * 128 * 1008  # seqlen rounded up to 16
    ws, n = 0x50000, out.value
    call = lambda prm, qd, kd, vd, w, nb: _C.lib.fa_flash_fwd_fp8(ctypes.byref(prm), qd, kd, vd, w, nb, None)
    assert call(p, 0.0, 1.0, 1.0, ws, n) == _C.FA_ERR_INVALID_ARGUMENT
    assert "descales must be positive" in _C.lib.fa_last_error().decode()
    assert call(p, 1.0, float("inf"), 1.0, ws, n) == _C.FA_ERR_INVALID_ARGUMENT
    assert call(p, 1.0, 1.0, 1.0, ws, n - 1) == _C.FA_ERR_INVALID_ARGUMENT
    assert "workspace must be 16-byte aligned" in _C.lib.fa_last_error().decode()
    assert call(p, 1.0, 1.0, 1.0, ws + 8, n) == _C.FA_ERR_INVALID_ARGUMENT
    assert call(_params(head_dim=128), 1.0, 1.0, 1.0, ws, n) == _C.FA_ERR_INVALID_ARGUMENT
    assert "must be FA_DTYPE_FLOAT8_E4M3" in _C.lib.fa_last_error().decode()
