"""FP8 blockwise GEMM (oracle; test infrastructure only).

fp8_gemm_blockwise_kernel, src/futudiffu/fp8_kernels.py:169-188: for each
128-wide K slice the fp8 dot product is formed in fp32 and promoted as
``acc += dot * a_s[m, kb] * b_s[n/128, kb]``; the bias (fp8_addmm, :290-292)
is added in fp32 before the cast.  Each slice dot product is formed here in
float64 and rounded once (the products of two e4m3 values are exact in fp32).
"""

from __future__ import annotations

import torch


def gemm_blockwise(a8, a_s, b8, b_s, bias=None, out_dtype=torch.bfloat16, b_layout: int = 0):
    """b_layout 0: b (N, K), b_s (N/128, K/128); 1: b (K, N), b_s (K/128, N/128);
    2: b (N, K), b_s (N,) applied after the K loop (fp8_gemm_rowwise, :386-408)."""
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
