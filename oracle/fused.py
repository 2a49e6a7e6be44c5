"""Fused RMSNorm prologues (oracle; test infrastructure only).

Restates the Triton kernels (fp32 throughout, one rounding at the store):
  P1 fused_rms_norm_modulate_kernel     src/futudiffu/fused_kernels.py:66-86
  P2 fused_rms_norm_gate_residual_kernel src/futudiffu/fused_kernels.py:123-148
  P3 fused_qkv_postprocess_kernel        src/futudiffu/fused_kernels.py:304-385
"""

from __future__ import annotations

import torch


def _rrms(x: torch.Tensor, eps: float) -> torch.Tensor:
    mean_sq = (x * x).sum(dim=-1, keepdim=True) / x.shape[-1]
    return 1.0 / torch.sqrt(mean_sq + eps)


def rms_norm_modulate(x, w, scale, eps=1e-5):
    xf = x.cpu().float()
    normed = (xf * _rrms(xf, eps)) * w.cpu().float()
    return (normed * (1.0 + scale.cpu().float().unsqueeze(1))).to(x.dtype)


def rms_norm_gate_residual(x, w, gate, residual, eps=1e-5):
    xf = x.cpu().float()
    normed = (xf * _rrms(xf, eps)) * w.cpu().float()
    return (residual.cpu().float() + torch.tanh(gate.cpu().float()).unsqueeze(1) * normed).to(x.dtype)


def qkv_postprocess(qkv, q_w, k_w, freqs, n_heads, head_dim, eps=1e-5):
    """qkv (B, S, 3*H*hd) -> Q, K, V (B, H, S, hd); freqs (B, S, [1,] hd/2, 2, 2)."""
    B, S, _ = qkv.shape
    dim = n_heads * head_dim
    x = qkv.cpu().float().reshape(B, S, 3, n_heads, head_dim)
    q, k, v = x[:, :, 0], x[:, :, 1], x[:, :, 2]
    f = freqs.cpu().float()
    if f.ndim == 6:
        f = f.squeeze(2)
    f = f.reshape(B, S, 1, head_dim // 2, 2, 2)
    cos, nsin, sin = f[..., 0, 0], f[..., 0, 1], f[..., 1, 0]

    def norm_rope(t, w):
        n = (t * _rrms(t, eps)) * w.cpu().float()
        e, o = n[..., 0::2], n[..., 1::2]
        re = cos * e + nsin * o
        ro = sin * e + cos * o
        return torch.stack([re, ro], dim=-1).reshape(t.shape)

    qo = norm_rope(q, q_w).permute(0, 2, 1, 3)
    ko = norm_rope(k, k_w).permute(0, 2, 1, 3)
    vo = v.permute(0, 2, 1, 3)
    dt = qkv.dtype
    return qo.to(dt), ko.to(dt), vo.to(dt)
