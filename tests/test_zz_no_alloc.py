"""fd_attn_quant_noalloc: the attention quantisation prologue for callers that
cannot allocate device memory (a serving host that plans every device buffer
up front and hands this library only inputs and outputs, or a foreign runtime
calling the C ABI without an allocator).  Its scratch is a fixed device array
inside the library.  Checked through the C ABI against fd_attn_quant (which
takes a caller-allocated workspace), on two calls in a row with different
inputs, so stale scratch from the first call cannot hide a bug in the second.

This file is named to be collected last.
"""

from __future__ import annotations

import ctypes
import math

import pytest
import torch

pytestmark = pytest.mark.gpu

SL2E = (1.0 / math.sqrt(128)) * math.log2(math.e)


def _inputs(BH, N, seed):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(BH, N, 128, generator=g).to(torch.bfloat16).cuda()
    k = (torch.randn(BH, N, 128, generator=g) + 2 * torch.randn(128, generator=g)).to(torch.bfloat16).cuda()
    v = torch.randn(BH, N, 128, generator=g).to(torch.bfloat16).cuda()
    return q, k, v


def _outputs(BH, N, gran, qk=0, pv=1):
    from futudiffu_b200.sage_attention import _desc_stride

    dev = "cuda"
    code_dt = torch.int8 if qk == 0 else torch.float8_e4m3fn
    return {
        "q_codes": torch.empty(BH, N, 128, dtype=code_dt, device=dev),
        "k_codes": torch.empty(BH, N, 128, dtype=code_dt, device=dev),
        "q_desc": torch.empty(BH, _desc_stride(N, gran, 128), device=dev),
        "k_desc": torch.empty(BH, _desc_stride(N, gran, 64), device=dev),
        "v_codes": torch.empty(BH, N, 128, dtype=torch.float8_e4m3fn, device=dev),
        "v_desc": torch.empty(BH, 128, device=dev),
        "k_mean": torch.empty(BH, 128, device=dev),
    }


def _run(lib, name, q, k, v, BH, N, gran, out, ws=None, smooth=1, qk=0, pv=1):
    from futudiffu_b200 import _lib as L

    fp8v = pv == L.PV_FP8
    args = [L.ptr(q), L.ptr(k), L.ptr(v), BH, N, smooth, qk, gran, gran, pv, ctypes.c_float(SL2E),
            L.ptr(out["q_codes"]), L.ptr(out["q_desc"]), L.ptr(out["k_codes"]), L.ptr(out["k_desc"]),
            L.ptr(out["v_codes"]) if fp8v else None, L.ptr(out["v_desc"]) if fp8v else None, L.ptr(out["k_mean"])]
    if ws is not None:
        args.append(L.ptr(ws))
    args.append(L.stream_ptr())
    rc = getattr(lib, name)(*args)
    assert rc == L.FD_OK, lib.fd_last_error()


def _same(a, b, keys):
    for key in keys:
        x, y = a[key], b[key]
        if x.dtype == torch.float8_e4m3fn:
            x, y = x.view(torch.uint8), y.view(torch.uint8)
        assert torch.equal(x, y), key


# (granularity, smooth_k, qk kind, pv kind, N): both granularities with INT8 / FP8
# Q/K codes and e4m3 or bf16 V, smoothing on and off, and a ragged N below one
# 256-row scratch chunk
CASES = [(0, 1, 0, 1, 1500), (1, 1, 0, 1, 1500), (0, 1, 1, 1, 1500), (1, 0, 0, 0, 1500), (0, 0, 1, 0, 1500),
         (1, 1, 1, 0, 100), (0, 1, 0, 1, 100)]


@pytest.mark.parametrize("gran,smooth,qk,pv,N", CASES)
def test_noalloc_matches_allocating_entry_point(gran, smooth, qk, pv, N):
    """Two calls in a row with different inputs: the second call's results cannot
    come from scratch that the first call left behind."""
    from futudiffu_b200 import _lib as L

    lib = L.load()
    BH = 6
    keys = ["q_codes", "q_desc", "k_codes", "k_desc"] + (["v_codes", "v_desc"] if pv == L.PV_FP8 else [])
    keys += ["k_mean"] if smooth else []
    for seed in (1, 2):
        q, k, v = _inputs(BH, N, seed + 10 * N)
        ref = _outputs(BH, N, gran, qk, pv)
        ws = torch.empty(int(lib.fd_attn_quant_workspace_floats(BH, N)), device="cuda")
        _run(lib, "fd_attn_quant", q, k, v, BH, N, gran, ref, ws, smooth, qk, pv)
        got = _outputs(BH, N, gran, qk, pv)
        _run(lib, "fd_attn_quant_noalloc", q, k, v, BH, N, gran, got, None, smooth, qk, pv)
        torch.cuda.synchronize()
        _same(got, ref, keys)
    L.check_status()


def test_noalloc_rejects_oversized_scratch():
    from futudiffu_b200 import _lib as L

    lib = L.load()
    cap = lib.fd_attn_quant_noalloc_max_floats()
    assert cap == 1048576
    BH, N = 64, 256 * 70  # 2 * 64 * 70 * 128 floats > cap
    assert lib.fd_attn_quant_workspace_floats(BH, N) > cap
    rc = lib.fd_attn_quant_noalloc(None, None, None, BH, N, 1, 0, 0, 0, 1, ctypes.c_float(1.0),
                                   None, None, None, None, None, None, None, None)
    assert rc == L.FD_ERR_ARG
    assert b"maximum" in lib.fd_last_error()
    # an N so large that the scratch size would wrap is rejected before it is computed
    rc = lib.fd_attn_quant_noalloc(None, None, None, 1, 1 << 62, 1, 0, 0, 0, 1, ctypes.c_float(1.0),
                                   None, None, None, None, None, None, None, None)
    assert rc == L.FD_ERR_ARG
    assert b"too large" in lib.fd_last_error()
