"""FP8 blockwise GEMM (oracle; test infrastructure only).

fp8_gemm_blockwise_kernel, src/futudiffu/fp8_kernels.py:169-188: for each
128-wide K slice the fp8 dot product is formed in fp32 and promoted as
``acc += dot * a_s[m, kb] * b_s[n/128, kb]``; the bias (fp8_addmm, :290-292)
is added in fp32 before the cast.  Each slice dot product is formed here in
float64 and rounded once (the products of two e4m3 values are exact in fp32).
"""

from __future__ import annotations

import contextlib

import torch

# Timing mode of the CPU baseline (bench.py only): the reference's torch-eager
# "dequantize and compute" formulation, in which each operand is dequantised
# (dequantize_fp8_blockwise, src/futudiffu/fp8.py:452-480; activations by their
# 1 x 128 scales) and multiplied in one fp32 matmul.  Parity tests use the
# per-slice promotion form below (the reference kernel's order of operations).
_DEQUANT_COMPUTE = False


@contextlib.contextmanager
def dequant_compute():
    """Evaluate gemm_blockwise in the dequantize-then-fp32-matmul form."""
    global _DEQUANT_COMPUTE
    old = _DEQUANT_COMPUTE
    _DEQUANT_COMPUTE = True
    try:
        yield
    finally:
        _DEQUANT_COMPUTE = old


def gemm_dequant(a8, a_s, b8, b_s, bias=None, out_dtype=torch.bfloat16):
    """Y = dequant(A) dequant(B)^T in fp32 (+ bias), B (N, K) with (N/128, K/128) scales."""
    a = a8.cpu().to(torch.float32)
    a = a.reshape(-1, a.shape[-1])
    M, K = a.shape
    a = (a.reshape(M, K // 128, 128) * a_s.cpu().reshape(M, K // 128, 1).float()).reshape(M, K)
    b = b8.cpu().to(torch.float32)
    N = b.shape[0]
    bs = b_s.cpu().float()
    b = (b.reshape(N // 128, 128, K // 128, 128) * bs.reshape(N // 128, 1, K // 128, 1)).reshape(N, K)
    acc = a @ b.t()
    if bias is not None:
        acc = acc + bias.cpu().to(torch.float32)[None, :]
    return acc.to(out_dtype)


def gemm_blockwise(a8, a_s, b8, b_s, bias=None, out_dtype=torch.bfloat16, b_layout: int = 0):
    """b_layout 0: b (N, K), b_s (N/128, K/128); 1: b (K, N), b_s (K/128, N/128);
    2: b (N, K), b_s (N,) applied after the K loop (fp8_gemm_rowwise, :386-408)."""
    if _DEQUANT_COMPUTE and b_layout == 0 and b8.shape[0] % 128 == 0:
        return gemm_dequant(a8, a_s, b8, b_s, bias, out_dtype)
    a = a8.cpu().to(torch.float64)
    a = a.reshape(-1, a.shape[-1])
    b = b8.cpu().to(torch.float64)
    if b_layout == 1:
        b = b.t()
    M, K = a.shape
    N = b.shape[0]
    a_s = a_s.cpu().reshape(M, K // 128).to(torch.float32)
    b_s = b_s.cpu().to(torch.float32)
    acc = torch.zeros(M, N, dtype=torch.float32)
    for kb in range(K // 128):
        dot = (a[:, kb * 128:(kb + 1) * 128] @ b[:, kb * 128:(kb + 1) * 128].T).to(torch.float32)
        if b_layout == 2:
            acc += dot * a_s[:, kb:kb + 1]
        else:
            bs = b_s[:, kb] if b_layout == 0 else b_s[kb, :]
            bs = bs.repeat_interleave(128)[:N]
            acc += (dot * a_s[:, kb:kb + 1]) * bs[None, :]
    if b_layout == 2:
        acc = acc * b_s[None, :N]
    if bias is not None:
        acc = acc + bias.cpu().to(torch.float32)[None, :]
    return acc.to(out_dtype)
