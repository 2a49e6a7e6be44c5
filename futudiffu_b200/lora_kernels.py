"""Multi-LoRA delta on the sm_100a GEMM (drop-in for futudiffu.lora_kernels).

    out[b, s, d] = sum_i (scale[b, i] * (x[b, s, :] @ A[i].T) @ B[i].T)[d]

Reference: `_multi_lora_kernel` / `multi_lora_forward`,
src/futudiffu/lora_kernels.py:55-278.  Here the mid projection h = x A^T of all
adapters runs as one bf16 GEMM (cuBLAS, a plain library GEMM), the per-sample
scales are applied to h, and the up-projection sum_i h_i B_i^T runs as the bf16
LoRA slices of the tcgen05 GEMM kernel (``fd_fp8_gemm_blockwise_lora`` with no FP8
slices), accumulating every adapter in fp32 before one bf16 rounding.  Zero
scales cost no branch: their h columns are zero.
"""

from __future__ import annotations

import torch
from torch import Tensor

from . import _lib as L

LORA_K_ALIGN = 64


def lora_operands(h: Tensor, B_cat: Tensor) -> tuple[Tensor, Tensor, int]:
    """Pad the scaled mid activations (M, K) and the side-by-side B (N, K) to a
    multiple of 64 columns (the kernel's bf16 slice width)."""
    K = h.shape[1]
    Kp = (K + LORA_K_ALIGN - 1) // LORA_K_ALIGN * LORA_K_ALIGN
    if Kp != K:
        h = torch.nn.functional.pad(h, (0, Kp - K))
        B_cat = torch.nn.functional.pad(B_cat, (0, Kp - K))
    return h.contiguous(), B_cat.contiguous(), Kp


def lora_delta_gemm(h: Tensor, B_cat: Tensor, out_dtype: torch.dtype = torch.bfloat16) -> Tensor:
    """h (M, K) bf16 @ B_cat (N, K)^T -> (M, N) on the tcgen05 kernel (fp32 accumulate)."""
    L.require_cuda(h, B_cat)
    hp, bp, Kp = lora_operands(h, B_cat)
    M, N = h.shape[0], B_cat.shape[0]
    out = torch.empty(M, N, dtype=out_dtype, device=h.device)
    if M == 0:
        return out
    L.call("fd_fp8_gemm_blockwise_lora", None, None, None, None, None, 0, L.ptr(out), L.dtype_code(out_dtype),
           M, N, 0, L.ptr(hp), L.ptr(bp), Kp, L.stream_ptr(h.device))
    return out


def multi_lora_forward(
    x: Tensor,
    A_all: Tensor,
    B_all: Tensor,
    scale_all: Tensor,
    *,
    BLOCK_M: int = 64,
    BLOCK_N: int = 64,
    BLOCK_K: int = 64,
    num_warps: int = 4,
    num_stages: int = 1,
) -> Tensor:
    """Sparse multi-LoRA delta (reference :162-278).  The tile keyword arguments of
    the reference are accepted and ignored (the sm_100a kernel has fixed tiles).

    x (B, S, IN) bf16, A_all (N, R, IN) bf16, B_all (N, OUT, R) bf16, scale_all (B, N)
    fp32 (alpha / rank folded in) -> (B, S, OUT) bf16.
    """
    del BLOCK_M, BLOCK_N, BLOCK_K, num_warps, num_stages
    assert x.ndim == 3, f"x must be 3D (B, S, IN), got {x.ndim}D"
    assert A_all.ndim == 3, f"A_all must be 3D (N, R, IN), got {A_all.ndim}D"
    assert B_all.ndim == 3, f"B_all must be 3D (N, OUT, R), got {B_all.ndim}D"
    assert scale_all.ndim == 2, f"scale_all must be 2D (B, N), got {scale_all.ndim}D"
    B, seq_len, in_features = x.shape
    n_ad, rank, in_features_A = A_all.shape
    n_ad_b, out_features, rank_b = B_all.shape
    assert in_features == in_features_A, (
        f"in_features mismatch: x has {in_features}, A has {in_features_A}")
    assert n_ad == n_ad_b, f"N_ADAPTERS mismatch: A has {n_ad}, B has {n_ad_b}"
    assert rank == rank_b, f"rank mismatch: A has {rank}, B has {rank_b}"
    assert scale_all.shape == (B, n_ad), (
        f"scale_all shape mismatch: expected ({B}, {n_ad}), got {scale_all.shape}")
    assert x.dtype == torch.bfloat16, f"x must be BF16, got {x.dtype}"
    assert A_all.dtype == torch.bfloat16, f"A_all must be BF16, got {A_all.dtype}"
    assert B_all.dtype == torch.bfloat16, f"B_all must be BF16, got {B_all.dtype}"
    assert scale_all.dtype == torch.float32, f"scale_all must be float32, got {scale_all.dtype}"
    assert x.is_contiguous(), "x must be contiguous"
    assert A_all.is_contiguous(), "A_all must be contiguous"
    assert B_all.is_contiguous(), "B_all must be contiguous"
    assert scale_all.is_contiguous(), "scale_all must be contiguous"
    L.require_cuda(x, A_all, B_all, scale_all)
    x2 = x.reshape(B * seq_len, in_features)
    h = x2 @ A_all.reshape(n_ad * rank, in_features).t()                      # (M, N R) bf16
    tok_scale = scale_all.repeat_interleave(seq_len, dim=0)                    # (M, N)
    hs = (h.float() * tok_scale.repeat_interleave(rank, dim=1)).to(torch.bfloat16)
    B_cat = B_all.permute(1, 0, 2).reshape(out_features, n_ad * rank)
    return lora_delta_gemm(hs, B_cat).reshape(B, seq_len, out_features)
