"""ctypes binding of ``libfd_b200.so`` (the C ABI declared in include/fd_b200.h).

The library is loaded lazily on first use.  There is no fallback: if the
shared object is missing or CUDA is unavailable, every operator raises
``RuntimeError``.  Each call passes raw device pointers and the current torch
CUDA stream, so kernels order correctly with surrounding torch work.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "libfd_b200.so"

FD_OK = 0
FD_ERR_ARG = 1
FD_ERR_CUDA = 2
FD_ERR_TIMEOUT = 3
FD_ERR_UNSUPPORTED = 4

FD_STATUS_TIMEOUT = 1
FD_STATUS_BOUNDS = 2

DT_BF16, DT_F16, DT_F32, DT_E4M3, DT_I8 = 0, 1, 2, 3, 4
GEMM_STORE_BF16 = -1


class GemmProblem(ctypes.Structure):
    """fd_gemm_problem (include/fd_b200.h)."""
    _fields_ = [("a", ctypes.c_void_p), ("a_s", ctypes.c_void_p), ("b", ctypes.c_void_p), ("b_s", ctypes.c_void_p),
                ("bias", ctypes.c_void_p), ("c", ctypes.c_void_p), ("c_s", ctypes.c_void_p),
                ("M", ctypes.c_int64), ("N", ctypes.c_int64), ("K", ctypes.c_int64)]


class QkvStream(ctypes.Structure):
    """fd_qkv_stream (include/fd_b200.h)."""
    _fields_ = [("q_norm", ctypes.c_void_p), ("k_norm", ctypes.c_void_p), ("freqs", ctypes.c_void_p),
                ("S", ctypes.c_int64), ("s_off", ctypes.c_int64), ("eps", ctypes.c_float)]


QK_INT8, QK_FP8 = 0, 1
GRAN_TOKEN, GRAN_BLOCK = 0, 1
PV_BF16, PV_FP8, PV_FP8_TILE = 0, 1, 2
ACT_NONE, ACT_GELU_TANH, ACT_SILU_GATE = 0, 1, 2

_DT_CODE = {
    torch.bfloat16: DT_BF16,
    torch.float16: DT_F16,
    torch.float32: DT_F32,
    torch.float8_e4m3fn: DT_E4M3,
    torch.int8: DT_I8,
}

_P = ctypes.c_void_p
_I = ctypes.c_int
_L = ctypes.c_int64
_F = ctypes.c_float

# name -> argtypes (every function returns int unless listed in _RESTYPES)
_SIGS: dict[str, list] = {
    "fd_version": [],
    "fd_last_error": [],
    "fd_get_status": [ctypes.POINTER(ctypes.c_uint), _I],
    "fd_div_full_f32": [_P, _P, _P, _L, _P],
    "fd_probe_tmem_ld": [_I, _I, _I, _I, _I, _P, _P, _P],
    "fd_attn_quant_v_tile": [_P, _L, _L, _P, _P, _P],
    "fd_fp8_act_quant": [_P, _I, _P, _P, _L, _L, _I, _P],
    "fd_fp8_weight_quant": [_P, _I, _P, _P, _L, _L, _I, _P],
    "fd_fp8_dequant_blockwise": [_P, _P, _P, _I, _L, _L, _I, _P],
    "fd_fp8_gemm_blockwise": [_P, _P, _P, _P, _P, _I, _P, _I, _L, _L, _L, _I, _P],
    "fd_fp8_gemm_quant": [_P, _P, _P, _P, _P, _I, _P, _P, _L, _L, _L, _I, _P],
    "fd_fp8_gemm_quant_ld": [_P, _P, _P, _P, _P, _I, _P, _P, _L, _L, _L, _I, _L, _L, _P],
    "fd_fp8_gemm_grouped2": [_P, _P, _I, _I, _P],
    "fd_fp8_gemm_qkv_quant": [_P, _P, _P, _P, _I, _L, _L, _L, _I, _I, _I, _F, _P, _P, _P, _P, _P, _P],
    "fd_fp8_gemm_blockwise_lora": [_P, _P, _P, _P, _P, _I, _P, _I, _L, _L, _L, _P, _P, _L, _P],
    "fd_fp8_silu_gate_quant": [_P, _P, _P, _L, _L, _I, _P],
    "fd_fp8_gelu_tanh_quant": [_P, _P, _P, _L, _L, _I, _P],
    "fd_fp8_gelu_requant": [_P, _P, _P, _P, _L, _L, _I, _P],
    "fd_rms_norm_modulate": [_P, _P, _I, _P, _I, _P, _L, _L, _L, _F, _P],
    "fd_rms_norm_modulate_quant": [_P, _P, _I, _P, _I, _P, _P, _L, _L, _L, _F, _P],
    "fd_rms_norm_gate_residual": [_P, _P, _I, _P, _I, _P, _P, _L, _L, _L, _F, _P],
    "fd_rms_norm_modulate_ranges": [_P, _P, _I, _P, _I, _P, _L, _L, _F, _P, _P, _L, _L, _P],
    "fd_rms_norm_modulate_quant_ranges": [_P, _P, _I, _P, _I, _P, _P, _L, _L, _F, _P, _P, _L, _L, _P],
    "fd_rms_norm_gate_residual_ranges": [_P, _P, _I, _P, _I, _P, _P, _L, _L, _F, _P, _P, _L, _L, _P],
    "fd_qkv_postprocess": [_P, _P, _P, _P, _P, _P, _P, _L, _L, _L, _L, _F, _P],
    "fd_qkv_postprocess_into": [_P, _P, _P, _P, _P, _P, _P, _L, _L, _L, _L, _F, _L, _L, _P],
    "fd_attn_quant_workspace_floats": [_L, _L],
    "fd_qkv_quant_workspace_floats": [_L, _L],
    "fd_qkv_postprocess_quant": [_P, _P, _P, _P, _L, _L, _L, _F, _L, _L, _I, _I, _I, _F, _P, _P, _P, _P, _P, _P],
    "fd_attn_quant_kv": [_P, _P, _L, _L, _I, _I, _I, _I, _P, _P, _P, _P, _P, _P, _P],
    "fd_attn_quant": [_P, _P, _P, _L, _L, _I, _I, _I, _I, _I, _F, _P, _P, _P, _P, _P, _P, _P, _P, _P],
    "fd_attn_quant_noalloc_max_floats": [],
    "fd_attn_quant_noalloc": [_P, _P, _P, _L, _L, _I, _I, _I, _I, _I, _F, _P, _P, _P, _P, _P, _P, _P, _P],
    "fd_sage_attn_fwd": [_P, _P, _P, _P, _P, _P, _P, _L, _P, _P, _L, _L, _I, _I, _I, _I, _P],
    "fd_sage_attn_fwd_bnhd": [_P, _P, _P, _P, _P, _P, _P, _L, _P, _P, _L, _L, _L, _I, _I, _I, _I, _P],
    "fd_sage_attn_fwd_quant_out": [_P, _P, _P, _P, _P, _P, _P, _L, _P, _L, _L, _L, _I, _I, _I, _I,
                                   _P, _P, _L, _L, _P, _P, _L, _L, _L, _P],
    "fd_sage_attn_bwd_prepass": [_P, _P, _P, _L, _L, _P],
    "fd_sage_attn_bwd": [_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _L, _P, _P, _P, _L, _L, _I, _F, _P],
}
_RESTYPES = {
    "fd_version": ctypes.c_char_p,
    "fd_last_error": ctypes.c_char_p,
    "fd_attn_quant_workspace_floats": ctypes.c_int64,
    "fd_qkv_quant_workspace_floats": ctypes.c_int64,
    "fd_attn_quant_noalloc_max_floats": ctypes.c_int64,
}

_lib = None
_lock = threading.Lock()


class FDError(RuntimeError):
    """Raised when a futudiffu_b200 C-ABI call returns a non-zero status."""


def exported_symbols() -> list[str]:
    """Every C-ABI entry point this binding expects the library to export."""
    return list(_SIGS)


def load(path: str | os.PathLike | None = None):
    """Load and bind the shared library (idempotent); raises if it is missing."""
    global _lib
    with _lock:
        if _lib is not None and path is None:
            return _lib
        p = Path(path) if path is not None else LIB_PATH
        if not p.exists():
            raise RuntimeError(
                f"futudiffu_b200 native library not found at {p}; "
                "build it with `python -m futudiffu_b200.build` (no CPU fallback exists)"
            )
        lib = ctypes.CDLL(str(p))
        for name, args in _SIGS.items():
            fn = getattr(lib, name)
            fn.argtypes = args
            fn.restype = _RESTYPES.get(name, ctypes.c_int)
        if path is None:
            _lib = lib
        return lib


def lib():
    return _lib if _lib is not None else load()


def require_cuda(*tensors: torch.Tensor) -> None:
    if not torch.cuda.is_available():
        raise RuntimeError("futudiffu_b200 requires a CUDA device (sm_100a); no CPU fallback exists")
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise RuntimeError("futudiffu_b200 operators take CUDA tensors only")


def stream_ptr(device: torch.device | None = None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def dtype_code(dt: torch.dtype) -> int:
    try:
        return _DT_CODE[dt]
    except KeyError:
        raise ValueError(f"unsupported dtype {dt}") from None


def call(name: str, *args) -> None:
    """Invoke a C-ABI function and raise FDError on a non-zero status."""
    fn = getattr(lib(), name)
    rc = fn(*args)
    if rc != FD_OK:
        msg = lib().fd_last_error().decode(errors="replace")
        if rc == FD_ERR_ARG:
            raise ValueError(f"{name}: {msg}")
        raise FDError(f"{name} failed with status {rc}: {msg}")


def get_status(clear: bool = True) -> int:
    """Synchronise the device and return (optionally clearing) the status word."""
    out = ctypes.c_uint(0)
    call("fd_get_status", ctypes.byref(out), 1 if clear else 0)
    return int(out.value)


def device_divide(a, b) -> torch.Tensor:
    """a / b on the device with the quantisers' f32 divide (Triton's `/`, div.full.f32).

    a, b: tensors or numbers (broadcast together); returns a CPU float32 tensor.
    """
    require_cuda()
    at = torch.as_tensor(a, dtype=torch.float32)
    bt = torch.as_tensor(b, dtype=torch.float32)
    shape = torch.broadcast_shapes(at.shape, bt.shape)
    ad = torch.broadcast_to(at.to("cuda"), shape).contiguous()
    bd = torch.broadcast_to(bt.to("cuda"), shape).contiguous()
    out = torch.empty_like(ad)
    call("fd_div_full_f32", ptr(ad), ptr(bd), ptr(out), ad.numel(), stream_ptr(ad.device))
    return out.cpu()


def check_status() -> None:
    """Raise FDError if any kernel recorded a timeout or bounds fault."""
    st = get_status(clear=True)
    if st & FD_STATUS_TIMEOUT:
        raise FDError("a futudiffu_b200 kernel hit its bounded-wait timeout")
    if st & FD_STATUS_BOUNDS:
        raise FDError("a futudiffu_b200 kernel recorded an out-of-bounds access")
