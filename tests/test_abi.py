"""C ABI: the library loads, exports every entry point the header declares, and
rejects bad arguments on the host before touching a GPU (CPU only)."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "fd_b200.h"


def header_functions() -> list[str]:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(fd_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    from futudiffu_b200 import _lib

    return _lib.load()


def test_header_declares_functions():
    names = header_functions()
    assert "fd_fp8_gemm_blockwise" in names and "fd_sage_attn_fwd" in names and "fd_attn_quant" in names


def test_library_exports_every_header_symbol(lib):
    for name in header_functions():
        assert hasattr(lib, name), name


def test_binding_covers_header():
    from futudiffu_b200 import _lib

    assert sorted(_lib.exported_symbols()) == header_functions()


def test_version(lib):
    assert b"sm_100a" in lib.fd_version()


def _rc(lib, name, *args):
    return getattr(lib, name)(*args)


def test_bad_arguments_rejected_without_gpu(lib):
    from futudiffu_b200 import _lib as L

    # K not a multiple of 128
    assert _rc(lib, "fd_fp8_act_quant", None, 0, None, None, 4, 100, 128, None) == L.FD_ERR_ARG
    assert b"multiple of 128" in lib.fd_last_error()
    # block size other than 128
    assert _rc(lib, "fd_fp8_act_quant", None, 0, None, None, 4, 256, 64, None) == L.FD_ERR_ARG
    # GEMM: N not a multiple of 16, bad layout, null pointers
    assert _rc(lib, "fd_fp8_gemm_blockwise", None, None, None, None, None, 0, None, 0, 8, 100, 128, 0, None) == L.FD_ERR_ARG
    assert _rc(lib, "fd_fp8_gemm_blockwise", None, None, None, None, None, 0, None, 0, 8, 128, 128, 3, None) == L.FD_ERR_ARG
    assert _rc(lib, "fd_fp8_gemm_blockwise", None, None, None, None, None, 0, None, 0, 8, 128, 128, 0, None) == L.FD_ERR_ARG
    # weight quant needs both dims % 128
    assert _rc(lib, "fd_fp8_weight_quant", None, 0, None, None, 100, 128, 128, None) == L.FD_ERR_ARG
    # attention: bad kinds / shapes
    assert _rc(lib, "fd_sage_attn_fwd", None, None, None, None, None, None, None, 0, None, None, 1, 128, 7, 0, 0, 0, None) == L.FD_ERR_ARG
    assert _rc(lib, "fd_sage_attn_fwd", None, None, None, None, None, None, None, 0, None, None, 0, 128, 0, 0, 0, 0, None) == L.FD_ERR_ARG
    assert _rc(lib, "fd_attn_quant", None, None, None, 1, 128, 1, 0, 0, 0, 0, ctypes.c_float(1.0), None, None,
               None, None, None, None, None, None, None) == L.FD_ERR_ARG
    # qkv postprocess only for head_dim 128
    assert _rc(lib, "fd_qkv_postprocess", None, None, None, None, None, None, None, 1, 4, 2, 64, ctypes.c_float(1e-5), None) == L.FD_ERR_ARG
    # norms: dim must be a multiple of 8
    assert _rc(lib, "fd_rms_norm_modulate", None, None, 0, None, 0, None, 1, 4, 100, ctypes.c_float(1e-5), None) == L.FD_ERR_ARG


def test_empty_inputs_are_noops(lib):
    from futudiffu_b200 import _lib as L

    assert _rc(lib, "fd_fp8_act_quant", None, 0, None, None, 0, 256, 128, None) == L.FD_OK
    assert _rc(lib, "fd_fp8_silu_gate_quant", None, None, None, 0, 256, 128, None) == L.FD_OK
    assert _rc(lib, "fd_fp8_gemm_blockwise", None, None, None, None, None, 0, None, 0, 0, 128, 128, 0, None) == L.FD_OK


def test_workspace_size(lib):
    assert lib.fd_attn_quant_workspace_floats(48, 4096) == 2 * 48 * 16 * 128
    assert lib.fd_attn_quant_workspace_floats(1, 1) == 2 * 128
