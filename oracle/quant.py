"""FP8 / INT8 quantisers (oracle; test infrastructure only).

Rounding rules of the reference:
  * fp32 -> e4m3: round-to-nearest-even after an explicit clamp to +-448
    (torch ``Tensor.to(torch.float8_e4m3fn)`` is RNE).
  * fp32 -> int8: truncation toward zero (Triton ``.to(tl.int8)``,
    src/futudiffu/sage_kernels.py:580-588).
  * every divide is an IEEE fp32 divide.
"""

from __future__ import annotations

import contextlib

import torch

FP8_MAX = 448.0
E4M3 = torch.float8_e4m3fn


def _f32(x):
    return x.detach().to("cpu", torch.float32)


def div_ieee(a, b) -> torch.Tensor:
    """Correctly rounded fp32 quotient (the quotient is formed in float64 and
    rounded once; for division double rounding through 53 bits is exact)."""
    a64 = torch.as_tensor(a, dtype=torch.float64)
    b64 = torch.as_tensor(b, dtype=torch.float64)
    return (a64 / b64).to(torch.float32)


# The reference computes its quantisation scales in Triton, whose f32 `/`
# compiles to a GPU divide instruction that is within 2 ulp of the correctly
# rounded quotient (its exact results are a property of the hardware).  On the
# CPU the oracle uses the correctly rounded quotient; parity tests on the GPU
# evaluate the quotients with a Triton kernel (``division(tests.helpers.
# triton_divide)``), i.e. the reference's own compiler path, so the scale
# arithmetic is reproduced bit for bit without using the library under test.
_TRITON_DIV = div_ieee


def triton_div(a, b) -> torch.Tensor:
    return _TRITON_DIV(torch.as_tensor(a, dtype=torch.float32), torch.as_tensor(b, dtype=torch.float32))


@contextlib.contextmanager
def division(fn):
    """Temporarily evaluate Triton-kernel quotients with ``fn(a, b)``."""
    global _TRITON_DIV
    old = _TRITON_DIV
    _TRITON_DIV = fn
    try:
        yield
    finally:
        _TRITON_DIV = old


def quant_e4m3_groups(xf: torch.Tensor):
    """xf (..., G, 128) fp32 -> (codes e4m3, dequant scale (..., G)).

    fp8_act_quant_kernel, src/futudiffu/fp8_kernels.py:65-76:
      scale = max(amax / 448, 1e-12); y = clamp(x * (448 / max(amax, 1e-12)), +-448)
    """
    amax = xf.abs().amax(dim=-1)
    scale = torch.clamp(triton_div(amax, FP8_MAX), min=1e-12)
    qs = triton_div(FP8_MAX, torch.clamp(amax, min=1e-12))
    y = (xf * qs.unsqueeze(-1)).clamp(-FP8_MAX, FP8_MAX).to(E4M3)
    return y, scale


def act_quant(x: torch.Tensor, block: int = 128):
    """G1 fp8_act_quant (src/futudiffu/fp8_kernels.py:54-90): (..., K) -> codes, (..., K/128)."""
    xf = _f32(x)
    K = xf.shape[-1]
    g = xf.reshape(*xf.shape[:-1], K // block, block)
    y, s = quant_e4m3_groups(g)
    return y.reshape(xf.shape), s


def weight_quant(w: torch.Tensor, block: int = 128):
    """G6 quantize_fp8_blockwise (src/futudiffu/fp8.py:352-369): 128 x 128 tiles.

    Returns codes (N, K) e4m3 and the stored scale 1 / (448 / max(amax, 1e-12)).
    Both quotients follow torch's ``scalar / tensor``, which evaluates
    ``tensor.reciprocal() * scalar`` (two roundings), exactly as the reference.
    """
    t = _f32(w)
    N, K = t.shape
    blocked = t.reshape(N // block, block, K // block, block).permute(0, 2, 1, 3)
    block_max = blocked.abs().amax(dim=(2, 3))
    qs = FP8_MAX / block_max.clamp_min(1e-12)
    q = (blocked * qs[..., None, None]).clamp(-FP8_MAX, FP8_MAX).to(E4M3)
    return q.permute(0, 2, 1, 3).reshape(N, K), (1.0 / qs).float()


def dequant_blockwise(w8: torch.Tensor, s: torch.Tensor, block: int = 128, out_dtype=torch.bfloat16):
    """G6 dequantize_fp8_blockwise (src/futudiffu/fp8.py:469-480)."""
    wf = w8.detach().cpu().to(torch.float32)
    N, K = wf.shape
    out = wf.reshape(N // block, block, K // block, block) * s.cpu().reshape(N // block, 1, K // block, 1)
    return out.reshape(N, K).to(out_dtype)


def silu_gate_quant(x: torch.Tensor, block: int = 128):
    """G4 fp8_silu_gate_quant (src/futudiffu/fp8_kernels.py:877-905): silu(w1) * w3 then G1."""
    xf = _f32(x)
    N = xf.shape[-1] // 2
    w1, w3 = xf[..., :N], xf[..., N:]
    gated = (w1 * triton_div(1.0, 1.0 + torch.exp(-w1))) * w3
    return act_quant(gated, block)


def gelu_tanh_quant(x: torch.Tensor, block: int = 128):
    """F.gelu(approximate='tanh') in fp32, then the G1 quantiser (MMDiT MLP activation)."""
    xf = _f32(x)
    return act_quant(torch.nn.functional.gelu(xf, approximate="tanh"), block)


def gelu_requant(x8: torch.Tensor, sx: torch.Tensor, block: int = 128):
    """fp8_gelu (src/futudiffu/fp8_kernels.py:740-786): dequant -> erf GELU -> requant."""
    xf = x8.cpu().to(torch.float32)
    K = xf.shape[-1]
    g = xf.reshape(*xf.shape[:-1], K // block, block) * sx.cpu().unsqueeze(-1)
    sqrt_2 = torch.tensor(1.41421356237, dtype=torch.float32)
    ge = g * 0.5 * (1.0 + torch.erf(triton_div(g, sqrt_2)))
    y, s = quant_e4m3_groups(ge)
    return y.reshape(xf.shape), s


def int8_trunc(x: torch.Tensor) -> torch.Tensor:
    """fp32 -> int8 with truncation toward zero (Triton .to(tl.int8))."""
    return x.to(torch.int8)
