"""Attention dispatch and RoPE / RMSNorm helpers: drop-in for ``futudiffu.attention``.

``set_attention_backend`` / ``sdpa_attention`` keep the reference dispatch
rules (src/futudiffu/attention.py:19-119): with backend "sage" or "auto", a
uint8 block mask routes to the masked SageAttention kernel and mask=None
routes to ``sage_attn_op``; the "sdpa" backend and FlexAttention BlockMasks
stay on PyTorch's own kernels, as in the reference.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F
from torch import Tensor

_ATTENTION_BACKEND = "sdpa"


def set_attention_backend(backend: str) -> None:
    global _ATTENTION_BACKEND
    if backend not in ("sdpa", "sage", "auto"):
        raise ValueError(f"Unknown attention backend: {backend!r}")
    _ATTENTION_BACKEND = backend


def get_attention_backend() -> str:
    return _ATTENTION_BACKEND


def sdpa_attention(
    q: Tensor,
    k: Tensor,
    v: Tensor,
    heads: int,
    mask: Tensor | None = None,
    skip_reshape: bool = False,
    block_mask=None,
) -> Tensor:
    """Scaled dot-product attention with the reference's backend dispatch; returns (B, seq, heads*dim)."""
    if skip_reshape:
        b, _, _, dim_head = q.shape
    else:
        b, _, dim_head = q.shape
        dim_head //= heads
        q, k, v = (t.view(b, -1, heads, dim_head).transpose(1, 2) for t in (q, k, v))

    if block_mask is not None and isinstance(block_mask, Tensor):
        if block_mask.dtype == torch.uint8 and _ATTENTION_BACKEND in ("sage", "auto"):
            try:
                from .sage_attention import sage_attn_forward_masked

                out = sage_attn_forward_masked(q, k, v, block_mask, 1.0 / (dim_head ** 0.5))
                return out.transpose(1, 2).reshape(b, -1, heads * dim_head)
            except Exception:
                if _ATTENTION_BACKEND == "sage":
                    raise

    if block_mask is not None:
        from torch.nn.attention.flex_attention import flex_attention

        out = flex_attention(q, k, v, block_mask=block_mask)
        return out.transpose(1, 2).reshape(b, -1, heads * dim_head)

    if mask is None and _ATTENTION_BACKEND in ("sage", "auto"):
        try:
            from .sage_attention import sage_attn_op

            out, _lse = sage_attn_op(q, k, v, 1.0 / (dim_head ** 0.5))
            return out.transpose(1, 2).reshape(b, -1, heads * dim_head)
        except Exception:
            if _ATTENTION_BACKEND == "sage":
                raise

    if mask is not None:
        if mask.ndim == 2:
            mask = mask.unsqueeze(0)
        if mask.ndim == 3:
            mask = mask.unsqueeze(1)
    out = F.scaled_dot_product_attention(q, k, v, attn_mask=mask, dropout_p=0.0, is_causal=False)
    return out.transpose(1, 2).reshape(b, -1, heads * dim_head)


def rope_embed(pos: Tensor, dim: int, theta: float) -> Tensor:
    """Flux/Lumina RoPE rotation matrices (..., n, dim/2, 2, 2) float32 (reference :124-136)."""
    assert dim % 2 == 0
    device = pos.device
    scale = torch.linspace(0, (dim - 2) / dim, steps=dim // 2, dtype=torch.float64, device=device)
    omega = 1.0 / (theta ** scale)
    out = torch.einsum("...n,d->...nd", pos.to(dtype=torch.float32, device=device), omega)
    out = torch.stack([torch.cos(out), -torch.sin(out), torch.sin(out), torch.cos(out)], dim=-1)
    out = out.reshape(*out.shape[:-1], 2, 2)
    return out.to(dtype=torch.float32, device=device)


def apply_rope_flux(xq: Tensor, xk: Tensor, freqs_cis: Tensor) -> tuple[Tensor, Tensor]:
    return _apply_rope1_flux(xq, freqs_cis), _apply_rope1_flux(xk, freqs_cis)


def _apply_rope1_flux(x: Tensor, freqs_cis: Tensor) -> Tensor:
    x_ = x.to(dtype=freqs_cis.dtype).reshape(*x.shape[:-1], -1, 1, 2)
    x_out = freqs_cis[..., 0] * x_[..., 0]
    x_out.addcmul_(freqs_cis[..., 1], x_[..., 1])
    return x_out.reshape(*x.shape).type_as(x)


def rms_norm(x: Tensor, weight: Tensor | None = None, eps: float = 1e-6) -> Tensor:
    if weight is None:
        return torch.nn.functional.rms_norm(x, (x.shape[-1],), eps=eps)
    return torch.nn.functional.rms_norm(x, weight.shape, weight=weight.to(dtype=x.dtype, device=x.device), eps=eps)
