"""Quantized attention (oracle; test infrastructure only).

Restates, on the CPU, the arithmetic of the reference SageAttention path:
  A1 _smooth_k                      src/futudiffu/sage_attention.py:63-71
  A2 INT8 per-token Q/K quant       src/futudiffu/sage_kernels.py:1416-1422, :1443-1449
  A3 FP8 per-token Q/K quant        src/futudiffu/sage_kernels.py:151-155, :176-179
  A4 FP8 P/V quant (per 64-key tile) src/futudiffu/sage_kernels.py:1135-1154
  A5 online softmax over 64-key tiles, LSE = m + log2 l
                                    src/futudiffu/sage_kernels.py:1424-1477
  A6 block-mask tile skipping       src/futudiffu/sage_kernels.py:1428-1438
  A7 backward (P recompute from LSE) src/futudiffu/sage_kernels.py:322-349, :805-1015
Per-block granularity (Q per 128 rows, K per 64 rows) and the per-channel V /
static-P fp8 PV variant apply the same formulas at the stated granularity.
"""

from __future__ import annotations

import contextlib
import math

import torch

from .quant import triton_div

LOG2E = math.log2(math.e)
E4M3 = torch.float8_e4m3fn
# Matmul type of the restatement: float64 (exact INT8 dot products, one rounding
# of each fp8 / bf16 dot product) for parity; bench.py's CPU-baseline timing
# evaluates the same formulas in fp32 (matmul_dtype(torch.float32)), as a torch
# eager CPU implementation would.
_MM = torch.float64


@contextlib.contextmanager
def matmul_dtype(dt):
    global _MM
    old = _MM
    _MM = dt
    try:
        yield
    finally:
        _MM = old


def smooth_k(k: torch.Tensor) -> torch.Tensor:
    """k - k.mean(dim=-2, keepdim=True) in bf16 (torch semantics), k (..., N, D) bf16."""
    k = k.cpu()
    return k - k.mean(dim=-2, keepdim=True)


def smooth_k_with_mean(k: torch.Tensor, mean_bf16: torch.Tensor) -> torch.Tensor:
    """bf16(k - mean) for a given bf16-valued mean (..., D)."""
    return (k.cpu().float() - mean_bf16.cpu().float().unsqueeze(-2)).to(torch.bfloat16)


def quant_rows(x: torch.Tensor, kind: str, rows_per_scale: int = 1, extra_scale: float = 1.0):
    """Quantise (BH, N, D) rows to int8 (trunc) / e4m3 with one scale per
    ``rows_per_scale`` rows (1 = per token).

    Returns codes (BH, N, D) and descales (BH, ceil(N / rows_per_scale)) with
    descale = (amax / qmax) * extra_scale.
    """
    xf = x.cpu().float()
    BH, N, D = xf.shape
    qmax = 127.0 if kind == "int8" else 448.0
    R = rows_per_scale
    nb = (N + R - 1) // R
    pad = nb * R - N
    xp = torch.nn.functional.pad(xf, (0, 0, 0, pad)) if pad else xf
    amax = xp.reshape(BH, nb, R * D).abs().amax(dim=-1)
    inv = triton_div(qmax, torch.clamp(amax, min=1e-12))
    inv_rows = inv.repeat_interleave(R, dim=1)[:, :N]
    y = xf * inv_rows.unsqueeze(-1)
    codes = y.to(torch.int8) if kind == "int8" else y.to(E4M3)
    desc = triton_div(amax, qmax) * torch.tensor(extra_scale, dtype=torch.float32)
    return codes, desc


def quant_v_per_channel(v: torch.Tensor):
    """V (BH, N, D) -> e4m3 codes with one scale per (bh, d) over the sequence."""
    vf = v.cpu().float()
    amax = vf.abs().amax(dim=1)  # (BH, D)
    inv = triton_div(448.0, torch.clamp(amax, min=1e-12))
    codes = (vf * inv.unsqueeze(1)).clamp(-448.0, 448.0).to(E4M3)
    return codes, triton_div(amax, 448.0)


def _mask_rows(block_mask, BH: int, N: int, tile: int):
    """Per-row boolean 'this 64-key tile is computed' (BH, N) for KV tile index ``tile``."""
    if block_mask is None:
        return None
    bm = block_mask.cpu().to(torch.bool)
    if bm.ndim == 2:
        bm = bm.unsqueeze(0).expand(BH, -1, -1)
    col = bm[:, :, tile]  # (BH, nq)
    return col.repeat_interleave(128, dim=1)[:, :N]


def attention_forward(
    q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, sm_scale: float | None = None,
    qk_quant: str = "int8", granularity: str = "per_token", pv_quant: str = "bf16",
    smooth: bool = True, block_mask=None, k_mean: torch.Tensor | None = None,
):
    """Reference online-softmax attention over 64-key tiles.

    q, k, v: (BH, N, 128) bf16.  pv_quant:
      "bf16"        P.to(bf16) @ V (production, :1466-1468)
      "fp8_tile"    reference A4: P per row per tile, V per column per tile
      "fp8_channel" e4m3 P = e4m3(448 p) (p <= 1 after max subtraction),
                    V per channel over the whole sequence
    Returns out (BH, N, 128) bf16 and lse (BH, N) fp32 (log2 domain).
    """
    BH, N, D = q.shape
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(D)
    sl2e = sm_scale * LOG2E
    ks = k.cpu()
    if smooth:
        ks = smooth_k(ks) if k_mean is None else smooth_k_with_mean(ks, k_mean)
    rq, rk = (1, 1) if granularity == "per_token" else (128, 64)
    qc, qd = quant_rows(q, qk_quant, rq, sl2e)
    kc, kd = quant_rows(ks, qk_quant, rk)
    qd_rows = qd.repeat_interleave(rq, dim=1)[:, :N]
    kd_rows = kd.repeat_interleave(rk, dim=1)[:, :N]
    qf = qc.to(_MM)
    kf = kc.to(_MM)
    vb = v.cpu()
    if pv_quant == "fp8_channel":
        vc, vdesc = quant_v_per_channel(vb)
    m = torch.full((BH, N), -math.inf)
    l = torch.zeros(BH, N)
    o = torch.zeros(BH, N, D)
    for t in range((N + 63) // 64):
        n0, n1 = t * 64, min(N, t * 64 + 64)
        active = _mask_rows(block_mask, BH, N, t)
        s = (qf @ kf[:, n0:n1].transpose(1, 2)).to(torch.float32)
        s = (s * qd_rows.unsqueeze(-1)) * kd_rows[:, None, n0:n1]
        m_new = torch.maximum(m, s.amax(dim=-1))
        alpha = torch.exp2(m - m_new)
        alpha = torch.where(torch.isnan(alpha), torch.zeros_like(alpha), alpha)
        p = torch.exp2(s - m_new.unsqueeze(-1))
        l_new = alpha * l + p.sum(dim=-1)
        if pv_quant == "bf16":
            pv = (p.to(torch.bfloat16).to(_MM) @ vb[:, n0:n1].to(_MM)).to(torch.float32)
        elif pv_quant == "fp8_tile":
            pam = p.abs().amax(dim=-1)
            p8 = (p * triton_div(448.0, torch.clamp(pam, min=1e-12)).unsqueeze(-1)).to(E4M3)
            vt = vb[:, n0:n1].float()
            vam = vt.abs().amax(dim=1)
            v8 = (vt * triton_div(448.0, torch.clamp(vam, min=1e-12)).unsqueeze(1)).to(E4M3)
            pv = (p8.to(_MM) @ v8.to(_MM)).to(torch.float32)
            pv = (pv * triton_div(pam, 448.0).unsqueeze(-1)) * triton_div(vam, 448.0).unsqueeze(1)
        elif pv_quant == "fp8_channel":
            p8 = (p * 448.0).clamp(max=448.0).to(E4M3)
            pv = (p8.to(_MM) @ vc[:, n0:n1].to(_MM)).to(torch.float32)
            pv = pv * (vdesc.unsqueeze(1) / 448.0)
        else:
            raise ValueError(pv_quant)
        o_new = o * alpha.unsqueeze(-1) + pv
        if active is None:
            m, l, o = m_new, l_new, o_new
        else:
            m = torch.where(active, m_new, m)
            l = torch.where(active, l_new, l)
            o = torch.where(active.unsqueeze(-1), o_new, o)
    lse = m + torch.log2(l)
    out = (o / l.unsqueeze(-1)).to(torch.bfloat16)
    return out, lse


def attention_exact(q, k, v, sm_scale: float | None = None):
    """Unquantised fp32 softmax attention (the reference's own SDPA fallback semantics)."""
    qf, kf, vf = q.cpu().float(), k.cpu().float(), v.cpu().float()
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(q.shape[-1])
    s = (qf @ kf.transpose(-1, -2)) * sm_scale
    return (torch.softmax(s, dim=-1) @ vf).to(torch.bfloat16)


def attention_backward(q, k, v, out, lse, dout, *, sm_scale: float, qk_quant: str = "int8",
                       smooth: bool = True, block_mask=None, k_mean=None, granularity: str = "per_token"):
    """dQ, dK, dV with the forward's quantised P (reference :322-349, :805-1015).

    P is recomputed from the saved LSE with the forward's Q/K quantisation: per
    token (the reference) or per block (128 Q rows, 64 K rows).  Block-masked
    pairs (128-row Q block x 64-key tile) contribute nothing (:1491-1722).
    """
    BH, N, D = q.shape
    sl2e = sm_scale * LOG2E
    ks = k.cpu()
    if smooth:
        ks = smooth_k(ks) if k_mean is None else smooth_k_with_mean(ks, k_mean)
    rq, rk = (1, 1) if granularity == "per_token" else (128, 64)
    qc, qd = quant_rows(q, qk_quant, rq, sl2e)
    kc, kd = quant_rows(ks, qk_quant, rk)
    qd = qd.repeat_interleave(rq, dim=1)[:, :N]
    kd = kd.repeat_interleave(rk, dim=1)[:, :N]
    s = (qc.to(torch.float64) @ kc.to(torch.float64).transpose(1, 2)).to(torch.float32)
    s = (s * qd.unsqueeze(-1)) * kd.unsqueeze(1)
    p = torch.exp2(s - lse.cpu().unsqueeze(-1))
    if block_mask is not None:
        bm = block_mask.cpu().to(torch.bool)
        if bm.ndim == 2:
            bm = bm.unsqueeze(0).expand(BH, -1, -1)
        full = bm.repeat_interleave(128, dim=1)[:, :N].repeat_interleave(64, dim=2)[:, :, :N]
        p = torch.where(full, p, torch.zeros_like(p))
    dof = dout.cpu().to(torch.float64)
    delta = (dout.cpu().float() * out.cpu().float()).sum(-1)
    dp = (dof @ v.cpu().to(torch.float64).transpose(1, 2)).to(torch.float32)
    ds = p * (dp - delta.unsqueeze(-1))
    dv = (p.to(torch.bfloat16).to(torch.float64).transpose(1, 2) @ dof).to(torch.float32)
    dk = ((ds * sm_scale).to(torch.bfloat16).to(torch.float64).transpose(1, 2)
          @ q.cpu().to(torch.float64)).to(torch.float32)
    dq = (ds.to(torch.bfloat16).to(torch.float64) @ ks.to(torch.float64)).to(torch.float32) * sm_scale
    return dq.to(torch.bfloat16), dk.to(torch.bfloat16), dv.to(torch.bfloat16), delta
