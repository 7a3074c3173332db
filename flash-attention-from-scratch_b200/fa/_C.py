"""Python binding of libfa_b200.so (the C ABI in include/fa_b200.h), via ctypes.

Mirrors the reference's Torch binding ``_C.forward`` (csrc/bindings.cpp:28-73, fa/_C.pyi:4-11):
same signature, same checks in the same order, same messages, same exception types
(TORCH_CHECK -> RuntimeError; the kernel's std::invalid_argument -> ValueError). The output is
allocated with ``torch.empty_like(q)`` and the kernel is enqueued on the current CUDA stream of
q's device; the call does not synchronise.

There is no fallback: if the shared library is missing or fails to load, importing this module
raises ImportError.
"""

from __future__ import annotations

import ctypes
import math
import os
from pathlib import Path

import torch

_LIB_NAME = "libfa_b200.so"
_LIB_PATH = Path(os.environ.get("FA_B200_LIB", Path(__file__).resolve().parent / _LIB_NAME))

FA_OK = 0
FA_ERR_INVALID_ARGUMENT = 1
FA_ERR_CUDA = 2
FA_ERR_DEVICE_TIMEOUT = 3

VARIANTS = {"baseline": 0, "opt": 1, "fp16acc": 2}

# FaFwdParams.dtype (FA_DTYPE_*): the element type of q, k, v and O. bfloat16 is an extension
# of the reference, which takes float16 only (csrc/bindings.cpp:34).
DTYPES = {torch.float16: 0, torch.bfloat16: 1}
FA_DTYPE_FLOAT8_E4M3 = 2


class FaFwdParams(ctypes.Structure):
    """ctypes image of ``FaFwdParams`` (include/fa_b200.h)."""

    _fields_ = [
        ("q", ctypes.c_void_p),
        ("k", ctypes.c_void_p),
        ("v", ctypes.c_void_p),
        ("o", ctypes.c_void_p),
        ("batch", ctypes.c_int32),
        ("heads", ctypes.c_int32),
        ("seqlen", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("softmax_scale", ctypes.c_float),
        ("causal", ctypes.c_uint8),
        ("variant", ctypes.c_uint8),
        ("dtype", ctypes.c_uint8),
        ("reserved", ctypes.c_uint8),
    ]


class FaPlan(ctypes.Structure):
    """ctypes image of ``FaPlan`` (include/fa_b200.h): the schedule fa_flash_fwd_auto runs."""

    _fields_ = [
        ("rows_per_item", ctypes.c_int32),
        ("persistent", ctypes.c_int32),
        ("num_splits", ctypes.c_int32),
        ("tail_blocks", ctypes.c_int32),
        ("tail_splits", ctypes.c_int32),
        ("head_groups", ctypes.c_int32),
        ("items", ctypes.c_int32),
        ("ctas", ctypes.c_int32),
        ("workspace_bytes", ctypes.c_uint64),
    ]


def _load() -> ctypes.CDLL:
    if not _LIB_PATH.exists():
        raise ImportError(
            f"{_LIB_PATH} not found: build it with "
            "`python flash-attention-from-scratch_b200/build.py` (nvcc, sm_100a)"
        )
    lib = ctypes.CDLL(str(_LIB_PATH))
    lib.fa_flash_fwd.argtypes = [ctypes.POINTER(FaFwdParams), ctypes.c_void_p]
    lib.fa_flash_fwd.restype = ctypes.c_int
    lib.fa_flash_fwd_sharded.argtypes = [
        ctypes.POINTER(FaFwdParams),
        ctypes.POINTER(ctypes.c_int32),
        ctypes.POINTER(ctypes.c_void_p),
        ctypes.c_int32,
    ]
    lib.fa_flash_fwd_sharded.restype = ctypes.c_int
    lib.fa_last_error.argtypes = []
    lib.fa_last_error.restype = ctypes.c_char_p
    lib.fa_device_status.argtypes = [ctypes.c_int32, ctypes.c_int32, ctypes.POINTER(ctypes.c_uint32)]
    lib.fa_device_status.restype = ctypes.c_int
    lib.fa_kernel_info.argtypes = [
        ctypes.c_int32,
        ctypes.c_int32,
        ctypes.POINTER(ctypes.c_int32),
        ctypes.POINTER(ctypes.c_int32),
    ]
    lib.fa_kernel_info.restype = ctypes.c_int
    lib.fa_splitkv_workspace_size.argtypes = [
        ctypes.POINTER(FaFwdParams), ctypes.c_int32, ctypes.POINTER(ctypes.c_uint64)]
    lib.fa_splitkv_workspace_size.restype = ctypes.c_int
    lib.fa_splitkv_choose.argtypes = [
        ctypes.POINTER(FaFwdParams), ctypes.c_int32, ctypes.POINTER(ctypes.c_int32)]
    lib.fa_splitkv_choose.restype = ctypes.c_int
    lib.fa_flash_fwd_splitkv.argtypes = [
        ctypes.POINTER(FaFwdParams), ctypes.c_int32, ctypes.c_void_p, ctypes.c_uint64, ctypes.c_void_p]
    lib.fa_flash_fwd_splitkv.restype = ctypes.c_int
    lib.fa_plan.argtypes = [ctypes.POINTER(FaFwdParams), ctypes.c_int32, ctypes.POINTER(FaPlan)]
    lib.fa_plan.restype = ctypes.c_int
    lib.fa_flash_fwd_auto.argtypes = [ctypes.POINTER(FaFwdParams), ctypes.c_void_p, ctypes.c_uint64, ctypes.c_void_p]
    lib.fa_flash_fwd_auto.restype = ctypes.c_int
    lib.fa_fp8_workspace_size.argtypes = [ctypes.POINTER(FaFwdParams), ctypes.POINTER(ctypes.c_uint64)]
    lib.fa_fp8_workspace_size.restype = ctypes.c_int
    lib.fa_flash_fwd_fp8.argtypes = [ctypes.POINTER(FaFwdParams), ctypes.c_float, ctypes.c_float, ctypes.c_float,
                                     ctypes.c_void_p, ctypes.c_uint64, ctypes.c_void_p]
    lib.fa_flash_fwd_fp8.restype = ctypes.c_int
    return lib


lib = _load()


def _raise(rc: int) -> None:
    msg = lib.fa_last_error().decode()
    if rc == FA_ERR_INVALID_ARGUMENT:
        raise ValueError(msg)
    raise RuntimeError(msg or f"flash_fwd failed with code {rc}")


def parse_variant(name: str) -> int:
    """Reference: parse_variant, csrc/bindings.cpp:15-26."""
    if name in VARIANTS:
        return VARIANTS[name]
    raise RuntimeError(f"variant must be 'opt', 'fp16acc' or 'baseline', got '{name}'")


def check_inputs(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> None:
    """The TORCH_CHECKs of csrc/bindings.cpp:31-40, in the same order and wording; the dtype
    check also admits bfloat16 (all three tensors the same type), which the reference lacks."""
    for t in (q, k, v):
        if not t.is_cuda:
            raise RuntimeError("q, k, v must be CUDA tensors")
        if t.dtype not in DTYPES:
            raise RuntimeError("q, k, v must be float16 (or bfloat16)")
        if t.dtype != q.dtype:
            raise RuntimeError("q, k, v must have the same dtype")
        if not t.is_contiguous():
            raise RuntimeError("q, k, v must be contiguous")
        if t.dim() != 4:
            raise RuntimeError("q, k, v must have shape [B, H, N, D]")
    if q.shape != k.shape or q.shape != v.shape:
        raise RuntimeError("q, k, v must have the same shape")
    if q.device != k.device or q.device != v.device:
        raise RuntimeError("q, k, v must be on the same device")


def make_params(q, k, v, o, causal: bool, softmax_scale: float, variant: int) -> FaFwdParams:
    p = FaFwdParams()
    p.q, p.k, p.v, p.o = q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr()
    p.batch, p.heads, p.seqlen, p.head_dim = (int(x) for x in q.shape)
    p.softmax_scale = float(softmax_scale)
    p.causal = 1 if causal else 0
    p.variant = variant
    p.dtype = DTYPES[q.dtype]
    return p


_SM_COUNT: dict[int, int] = {}


def _sm_count(device: torch.device) -> int:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    if idx not in _SM_COUNT:
        _SM_COUNT[idx] = torch.cuda.get_device_properties(idx).multi_processor_count
    return _SM_COUNT[idx]


def choose_splits(params: FaFwdParams, device: torch.device) -> int:
    """Split count the library picks for `params` on `device` (1 = no split)."""
    out = ctypes.c_int32(1)
    rc = lib.fa_splitkv_choose(ctypes.byref(params), _sm_count(device), ctypes.byref(out))
    if rc != FA_OK:
        _raise(rc)
    return int(out.value)


def plan_params(params: FaFwdParams, num_sms: int = 0) -> dict:
    """The schedule the library runs for `params` (fa_plan); num_sms <= 0: the current device."""
    out = FaPlan()
    rc = lib.fa_plan(ctypes.byref(params), int(num_sms), ctypes.byref(out))
    if rc != FA_OK:
        _raise(rc)
    return {name: int(getattr(out, name)) for name, _ in FaPlan._fields_}


_WORKSPACE: dict[tuple, int] = {}


def _auto_workspace_bytes(params: FaFwdParams, device: torch.device) -> int:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    key = (idx, params.batch, params.heads, params.seqlen, params.head_dim, params.causal, params.variant)
    if key not in _WORKSPACE:
        _WORKSPACE[key] = plan_params(params, _sm_count(device))["workspace_bytes"]
    return _WORKSPACE[key]


def forward(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    causal: bool = False,
    softmax_scale: float | None = None,
    variant: str = "opt",
) -> torch.Tensor:
    """O = softmax(Q K^T * scale) V (reference csrc/bindings.cpp:28-64), on the library's
    schedule (fa_flash_fwd_auto: split-KV for few row blocks, a tail split of a partial last
    wave); the split partials' workspace is a torch allocation on the current stream, like O."""
    return forward_splitkv(q, k, v, causal, softmax_scale, variant, None)


def forward_splitkv(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    causal: bool = False,
    softmax_scale: float | None = None,
    variant: str = "opt",
    num_splits: int | None = None,
) -> torch.Tensor:
    """forward() with an explicit split-KV count (not in the reference): each row block's key
    range is cut into ``num_splits`` ranges (None = the library's schedule, fa_flash_fwd_auto).
    The workspace is a torch allocation on the current stream, like O itself."""
    check_inputs(q, k, v)
    with torch.cuda.device(q.device):
        o = torch.empty_like(q)
        head_dim = q.shape[3]
        scale = softmax_scale if softmax_scale is not None else 1.0 / math.sqrt(head_dim)
        vid = parse_variant(variant)
        if q.shape[2] > 0:
            params = make_params(q, k, v, o, causal, scale, vid)
            stream = torch.cuda.current_stream(q.device).cuda_stream
            splits = None if num_splits is None else int(num_splits)
            if splits is None:
                nbytes = _auto_workspace_bytes(params, q.device)
                ws = torch.empty(nbytes, dtype=torch.uint8, device=q.device) if nbytes > 0 else None
                rc = lib.fa_flash_fwd_auto(ctypes.byref(params), ctypes.c_void_p(ws.data_ptr() if ws is not None else 0),
                                           nbytes, ctypes.c_void_p(stream))
            elif splits == 1:
                rc = lib.fa_flash_fwd(ctypes.byref(params), ctypes.c_void_p(stream))
            else:
                nbytes = ctypes.c_uint64(0)
                rc = lib.fa_splitkv_workspace_size(ctypes.byref(params), splits, ctypes.byref(nbytes))
                if rc == FA_OK:
                    ws = torch.empty(int(nbytes.value), dtype=torch.uint8, device=q.device)
                    rc = lib.fa_flash_fwd_splitkv(ctypes.byref(params), splits, ctypes.c_void_p(ws.data_ptr()),
                                                  nbytes.value, ctypes.c_void_p(stream))
            if rc != FA_OK:
                _raise(rc)
    return o


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
    """fp8 forward (not in the reference): q, k, v float8_e4m3fn [B, H, N, 128] CUDA tensors
    holding x / descale per tensor; O = softmax(scale * (q q_descale)(k k_descale)^T)
    (v v_descale) as float16. fa_flash_fwd_fp8 on the current stream; its transposed-V workspace
    is a torch allocation, like O."""
    for t in (q, k, v):
        if not t.is_cuda:
            raise RuntimeError("q, k, v must be CUDA tensors")
        if t.dtype != torch.float8_e4m3fn:
            raise RuntimeError("q, k, v must be float8_e4m3fn")
        if not t.is_contiguous():
            raise RuntimeError("q, k, v must be contiguous")
        if t.dim() != 4:
            raise RuntimeError("q, k, v must have shape [B, H, N, D]")
    if q.shape != k.shape or q.shape != v.shape:
        raise RuntimeError("q, k, v must have the same shape")
    if q.device != k.device or q.device != v.device:
        raise RuntimeError("q, k, v must be on the same device")
    with torch.cuda.device(q.device):
        o = torch.empty(q.shape, dtype=torch.float16, device=q.device)
        head_dim = q.shape[3]
        scale = softmax_scale if softmax_scale is not None else 1.0 / math.sqrt(head_dim)
        if q.shape[2] > 0:
            p = FaFwdParams()
            p.q, p.k, p.v, p.o = q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr()
            p.batch, p.heads, p.seqlen, p.head_dim = (int(x) for x in q.shape)
            p.softmax_scale = float(scale)
            p.causal = 1 if causal else 0
            p.variant = parse_variant(variant)
            p.dtype = FA_DTYPE_FLOAT8_E4M3
            nbytes = ctypes.c_uint64(0)
            rc = lib.fa_fp8_workspace_size(ctypes.byref(p), ctypes.byref(nbytes))
            if rc == FA_OK:
                ws = torch.empty(max(16, int(nbytes.value)), dtype=torch.uint8, device=q.device)
                stream = torch.cuda.current_stream(q.device).cuda_stream
                rc = lib.fa_flash_fwd_fp8(ctypes.byref(p), float(q_descale), float(k_descale), float(v_descale),
                                          ctypes.c_void_p(ws.data_ptr()), ws.numel(), ctypes.c_void_p(stream))
            if rc != FA_OK:
                _raise(rc)
    return o


def device_status(device: int, clear: bool = True) -> int:
    """Sticky watchdog bits of `device` (0 = no kernel gave up a wait). Synchronises."""
    out = ctypes.c_uint32(0)
    rc = lib.fa_device_status(int(device), 1 if clear else 0, ctypes.byref(out))
    if rc != FA_OK:
        _raise(rc)
    return int(out.value)


def kernel_info(head_dim: int, variant: str = "opt") -> tuple[int, int]:
    """(shared-memory bytes, threads) per CTA of the kernel for (head_dim, variant)."""
    smem, thr = ctypes.c_int32(0), ctypes.c_int32(0)
    rc = lib.fa_kernel_info(int(head_dim), parse_variant(variant), ctypes.byref(smem), ctypes.byref(thr))
    if rc != FA_OK:
        _raise(rc)
    return int(smem.value), int(thr.value)
