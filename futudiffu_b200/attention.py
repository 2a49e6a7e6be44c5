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
    """RoPE rotations (Flux / Lumina form) for positions ``pos`` (..., n).

    Channel pair i < dim / 2 turns by the angle a = pos * theta^(-2 i / dim); the
    result holds the 2 x 2 rotation [[cos a, -sin a], [sin a, cos a]] per pair,
    shape (..., n, dim / 2, 2, 2), float32.  The frequencies and angles are
    evaluated in float64 and rounded once (reference src/futudiffu/attention.py:124-136;
    the fused QKV post-process consumes this layout)."""
    assert dim % 2 == 0
    half = dim // 2
    # exponents 2 i / dim, i = 0 .. half - 1, as evenly spaced float64 values
    expo = torch.linspace(0.0, (dim - 2) / dim, steps=half, dtype=torch.float64, device=pos.device)
    inv_freq = 1.0 / (theta ** expo)
    ang = pos.to(torch.float32).to(torch.float64).unsqueeze(-1) * inv_freq
    cos, sin = torch.cos(ang), torch.sin(ang)
    rot = torch.stack((torch.stack((cos, -sin), dim=-1), torch.stack((sin, cos), dim=-1)), dim=-2)
    return rot.to(torch.float32)


def apply_rope_flux(xq: Tensor, xk: Tensor, freqs_cis: Tensor) -> tuple[Tensor, Tensor]:
    """Rotate the channel pairs of Q and K by ``freqs_cis`` (rope_embed's layout)."""
    return _apply_rope1_flux(xq, freqs_cis), _apply_rope1_flux(xk, freqs_cis)


def _apply_rope1_flux(x: Tensor, freqs_cis: Tensor) -> Tensor:
    """(x_2i, x_2i+1) -> R_i (x_2i, x_2i+1) in freqs_cis' dtype, returned in x's dtype:
    out = R[:, 0] x_2i + R[:, 1] x_2i+1 (each output channel a row of R)."""
    pairs = x.to(freqs_cis.dtype).unflatten(-1, (-1, 1, 2))
    out = torch.addcmul(freqs_cis[..., 0] * pairs[..., 0], freqs_cis[..., 1], pairs[..., 1])
    return out.reshape(x.shape).type_as(x)


def rms_norm(x: Tensor, weight: Tensor | None = None, eps: float = 1e-6) -> Tensor:
    """x / sqrt(mean(x^2) + eps) over the last dimension, times ``weight`` (cast to
    x's dtype) when given: torch's fused RMSNorm."""
    shape = (x.shape[-1],) if weight is None else tuple(weight.shape)
    w = None if weight is None else weight.to(dtype=x.dtype, device=x.device)
    return F.rms_norm(x, shape, weight=w, eps=eps)
