"""Fused RMSNorm / adaLN / RoPE prologues, B200 edition: drop-in for
``futudiffu.fused_kernels``.

Same ``futudiffu::`` custom ops, signatures, fakes and analytic autograd as
src/futudiffu/fused_kernels.py:561-790, backed by the sm_100a kernels in
``csrc/norm.cu``:

* ``fused_rms_norm_modulate``      rmsnorm(x) * w * (1 + scale[b])      (P1, :43-86)
* ``fused_rms_norm_gate_residual`` residual + tanh(gate[b]) * rmsnorm(x) * w (P2, :99-148)
* ``fused_qkv_postprocess``        split QKV, per-head RMSNorm Q/K, Flux RoPE,
  transpose to (B, H, S, hd)                                          (P3, :270-471)
"""

from __future__ import annotations

import torch

from . import _lib as L

_USE_FUSED_CUSTOM_OP = True


def _fused_rms_norm_modulate_cuda(x, weight, scale, eps=1e-5):
    assert x.ndim == 3, f"Expected x to be 3D (B, seq, dim), got {x.ndim}D"
    assert x.is_contiguous(), "Input x must be contiguous"
    assert weight.is_contiguous(), "Weight must be contiguous"
    assert scale.is_contiguous(), "Scale must be contiguous"
    B, seq_len, dim = x.shape
    assert weight.shape == (dim,), f"Weight shape mismatch: {weight.shape} vs ({dim},)"
    assert scale.shape == (B, dim), f"Scale shape mismatch: {scale.shape} vs ({B}, {dim})"
    assert x.dtype == torch.bfloat16, "x must be bf16"
    L.require_cuda(x, weight, scale)
    out = torch.empty_like(x)
    L.call("fd_rms_norm_modulate", L.ptr(x), L.ptr(weight), L.dtype_code(weight.dtype), L.ptr(scale),
           L.dtype_code(scale.dtype), L.ptr(out), B, seq_len, dim, float(eps), L.stream_ptr(x.device))
    return out


def fused_rms_norm_modulate_quant(x, weight, scale, eps=1e-5):
    """``fp8_act_quant(fused_rms_norm_modulate(x, weight, scale, eps))`` in one pass.

    Returns e4m3 codes (B, seq, dim) and fp32 dequant scales (B, seq, dim / 128),
    code for code equal to the two-kernel path, without the bf16 intermediate.
    (No single reference op: the reference runs the norm and the quantiser
    separately, fused_kernels.py:43-86 and fp8_kernels.py:54-90.)
    """
    assert x.ndim == 3, f"Expected x to be 3D (B, seq, dim), got {x.ndim}D"
    assert x.is_contiguous() and weight.is_contiguous() and scale.is_contiguous()
    B, seq_len, dim = x.shape
    assert weight.shape == (dim,) and scale.shape == (B, dim)
    assert x.dtype == torch.bfloat16, "x must be bf16"
    assert dim % 128 == 0, "dim must be a multiple of 128"
    L.require_cuda(x, weight, scale)
    y = torch.empty(B, seq_len, dim, dtype=torch.float8_e4m3fn, device=x.device)
    y_s = torch.empty(B, seq_len, dim // 128, dtype=torch.float32, device=x.device)
    L.call("fd_rms_norm_modulate_quant", L.ptr(x), L.ptr(weight), L.dtype_code(weight.dtype), L.ptr(scale),
           L.dtype_code(scale.dtype), L.ptr(y), L.ptr(y_s), B, seq_len, dim, float(eps), L.stream_ptr(x.device))
    return y, y_s


def qkv_postprocess_into(qkv, q_norm_weight, k_norm_weight, freqs_cis, q_out, k_out, v_out, seq_offset,
                         norm_eps=1e-5):
    """``fused_qkv_postprocess`` writing rows [seq_offset, seq_offset + S) of
    preallocated (B, H, S_total, 128) outputs (the streams of a joint attention
    share one buffer).  ``freqs_cis`` is (B, S, 64, 2, 2) fp32 contiguous."""
    B, S, three_dim = qkv.shape
    _, H, S_total, hd = q_out.shape
    assert hd == 128 and three_dim == 3 * H * hd
    assert qkv.is_contiguous() and q_out.is_contiguous() and k_out.is_contiguous() and v_out.is_contiguous()
    assert freqs_cis.dtype == torch.float32 and freqs_cis.is_contiguous()
    L.require_cuda(qkv, q_out)
    # the fp32 copies must stay referenced until the launch: a temporary freed
    # inside the argument list could hand its block to the next one
    qw = q_norm_weight.float().contiguous()
    kw = k_norm_weight.float().contiguous()
    L.call("fd_qkv_postprocess_into", L.ptr(qkv), L.ptr(qw),
           L.ptr(kw), L.ptr(freqs_cis), L.ptr(q_out), L.ptr(k_out), L.ptr(v_out),
           B, S, H, hd, float(norm_eps), S_total, seq_offset, L.stream_ptr(qkv.device))


def _range_args(x, params, range_rows, range_param):
    dim = x.shape[-1]
    assert x.is_contiguous() and x.dtype == torch.bfloat16, "x must be contiguous bf16"
    assert params.ndim == 2 and params.shape[1] == dim and params.is_contiguous(), "params must be (n, dim)"
    assert range_rows.dtype == torch.int32 and range_param.dtype == torch.int32
    assert range_rows.numel() == range_param.numel() + 1, "range_rows needs one more entry than range_param"
    L.require_cuda(x, params, range_rows, range_param)
    return x.numel() // dim, dim, range_param.numel(), params.shape[0]


def rms_norm_modulate_ranges(x, weight, scale, range_rows, range_param, eps=1e-5):
    """P1 over a packed sequence: rows [range_rows[i], range_rows[i + 1]) of x
    (..., dim) are modulated by (1 + scale[range_param[i]]), scale (n_images, dim).

    The per-token path of the reference block (src_ii/transformer.py:656-677)
    with the per-image rows it scatters by document_id
    (src_ii/zimage_model.py:496-512) left unscattered.  Rows in no range are
    not written."""
    rows, dim, n, n_params = _range_args(x, scale, range_rows, range_param)
    out = torch.empty_like(x)
    L.call("fd_rms_norm_modulate_ranges", L.ptr(x), L.ptr(weight), L.dtype_code(weight.dtype), L.ptr(scale),
           L.dtype_code(scale.dtype), L.ptr(out), rows, dim, float(eps), L.ptr(range_rows), L.ptr(range_param),
           n, n_params, L.stream_ptr(x.device))
    return out


def rms_norm_modulate_quant_ranges(x, weight, scale, range_rows, range_param, eps=1e-5):
    """``rms_norm_modulate_ranges`` quantised 1 x 128 to e4m3 in the same pass:
    codes (..., dim) and fp32 dequant scales (..., dim / 128)."""
    rows, dim, n, n_params = _range_args(x, scale, range_rows, range_param)
    assert dim % 128 == 0, "dim must be a multiple of 128"
    y = torch.empty(x.shape, dtype=torch.float8_e4m3fn, device=x.device)
    y_s = torch.empty(*x.shape[:-1], dim // 128, dtype=torch.float32, device=x.device)
    L.call("fd_rms_norm_modulate_quant_ranges", L.ptr(x), L.ptr(weight), L.dtype_code(weight.dtype),
           L.ptr(scale), L.dtype_code(scale.dtype), L.ptr(y), L.ptr(y_s), rows, dim, float(eps),
           L.ptr(range_rows), L.ptr(range_param), n, n_params, L.stream_ptr(x.device))
    return y, y_s


def rms_norm_gate_residual_ranges(x, weight, gate, residual, range_rows, range_param, eps=1e-5):
    """P2 over a packed sequence: residual + tanh(gate[range_param[i]]) *
    rmsnorm(x) * w on the rows of range i."""
    rows, dim, n, n_params = _range_args(x, gate, range_rows, range_param)
    assert residual.shape == x.shape and residual.is_contiguous() and residual.dtype == torch.bfloat16
    out = torch.empty_like(x)
    L.call("fd_rms_norm_gate_residual_ranges", L.ptr(x), L.ptr(weight), L.dtype_code(weight.dtype), L.ptr(gate),
           L.dtype_code(gate.dtype), L.ptr(residual), L.ptr(out), rows, dim, float(eps), L.ptr(range_rows),
           L.ptr(range_param), n, n_params, L.stream_ptr(x.device))
    return out


def _fused_rms_norm_gate_residual_cuda(x, weight, gate, residual, eps=1e-5):
    assert x.ndim == 3, f"Expected x to be 3D (B, seq, dim), got {x.ndim}D"
    assert x.is_contiguous(), "Input x must be contiguous"
    assert weight.is_contiguous(), "Weight must be contiguous"
    assert gate.is_contiguous(), "Gate must be contiguous"
    assert residual.is_contiguous(), "Residual must be contiguous"
    B, seq_len, dim = x.shape
    assert weight.shape == (dim,), f"Weight shape mismatch: {weight.shape} vs ({dim},)"
    assert gate.shape == (B, dim), f"Gate shape mismatch: {gate.shape} vs ({B}, {dim})"
    assert residual.shape == x.shape, f"Residual shape mismatch: {residual.shape} vs {x.shape}"
    assert x.dtype == torch.bfloat16 and residual.dtype == torch.bfloat16, "x and residual must be bf16"
    L.require_cuda(x, weight, gate, residual)
    out = torch.empty_like(x)
    L.call("fd_rms_norm_gate_residual", L.ptr(x), L.ptr(weight), L.dtype_code(weight.dtype),
           L.ptr(gate), L.dtype_code(gate.dtype), L.ptr(residual), L.ptr(out), B, seq_len, dim,
           float(eps), L.stream_ptr(x.device))
    return out


def _fused_qkv_postprocess_cuda(qkv, q_norm_weight, k_norm_weight, freqs_cis, n_heads, head_dim,
                                norm_eps=1e-5):
    assert qkv.ndim == 3, f"Expected qkv to be 3D (B, seq, 3*dim), got {qkv.ndim}D"
    assert qkv.is_contiguous(), "QKV must be contiguous"
    B, seq_len, total_dim = qkv.shape
    dim = n_heads * head_dim
    assert total_dim == 3 * dim, f"QKV last dim {total_dim} != 3 * {dim}"
    n_pairs = head_dim // 2
    assert head_dim % 2 == 0, f"head_dim must be even, got {head_dim}"
    assert head_dim == 128, "head_dim must be 128"
    assert q_norm_weight.shape == (head_dim,), f"q_norm shape {q_norm_weight.shape} != ({head_dim},)"
    assert k_norm_weight.shape == (head_dim,), f"k_norm shape {k_norm_weight.shape} != ({head_dim},)"
    assert qkv.dtype == torch.bfloat16, "qkv must be bf16"
    if freqs_cis.ndim == 6:
        assert freqs_cis.shape[2] == 1, f"Expected freqs_cis dim 2 to be 1, got {freqs_cis.shape[2]}"
        freqs_flat = freqs_cis.squeeze(2).reshape(B * seq_len, n_pairs, 2, 2)
    elif freqs_cis.ndim == 5:
        freqs_flat = freqs_cis.reshape(B * seq_len, n_pairs, 2, 2)
    else:
        raise ValueError(f"Unexpected freqs_cis ndim: {freqs_cis.ndim}, shape: {freqs_cis.shape}")
    freqs_flat = freqs_flat.to(torch.float32).contiguous()
    L.require_cuda(qkv, q_norm_weight, k_norm_weight, freqs_flat)
    out_q = torch.empty(B, n_heads, seq_len, head_dim, dtype=qkv.dtype, device=qkv.device)
    out_k = torch.empty_like(out_q)
    out_v = torch.empty_like(out_q)
    qw = q_norm_weight.to(dtype=torch.float32).contiguous()
    kw = k_norm_weight.to(dtype=torch.float32).contiguous()
    L.call("fd_qkv_postprocess", L.ptr(qkv), L.ptr(qw), L.ptr(kw), L.ptr(freqs_flat), L.ptr(out_q),
           L.ptr(out_k), L.ptr(out_v), B, seq_len, n_heads, head_dim, float(norm_eps),
           L.stream_ptr(qkv.device))
    return out_q, out_k, out_v


@torch.library.custom_op("futudiffu::fused_rms_norm_modulate", mutates_args=())
def fused_rms_norm_modulate(
    x: torch.Tensor,
    weight: torch.Tensor,
    scale: torch.Tensor,
    eps: float = 1e-5,
) -> torch.Tensor:
    return _fused_rms_norm_modulate_cuda(x, weight, scale, eps)


@fused_rms_norm_modulate.register_fake
def _fused_rms_norm_modulate_fake(x, weight, scale, eps=1e-5):
    return x.new_empty(*x.shape)


@torch.library.custom_op("futudiffu::fused_rms_norm_gate_residual", mutates_args=())
def fused_rms_norm_gate_residual(
    x: torch.Tensor,
    weight: torch.Tensor,
    gate: torch.Tensor,
    residual: torch.Tensor,
    eps: float = 1e-5,
) -> torch.Tensor:
    return _fused_rms_norm_gate_residual_cuda(x, weight, gate, residual, eps)


@fused_rms_norm_gate_residual.register_fake
def _fused_rms_norm_gate_residual_fake(x, weight, gate, residual, eps=1e-5):
    return x.new_empty(*x.shape)


@torch.library.custom_op("futudiffu::fused_qkv_postprocess", mutates_args=())
def fused_qkv_postprocess(
    qkv: torch.Tensor,
    q_norm_weight: torch.Tensor,
    k_norm_weight: torch.Tensor,
    freqs_cis: torch.Tensor,
    n_heads: int,
    head_dim: int,
    norm_eps: float = 1e-5,
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    return _fused_qkv_postprocess_cuda(qkv, q_norm_weight, k_norm_weight, freqs_cis, n_heads,
                                       head_dim, norm_eps)


@fused_qkv_postprocess.register_fake
def _fused_qkv_postprocess_fake(qkv, q_norm_weight, k_norm_weight, freqs_cis, n_heads, head_dim,
                                norm_eps=1e-5):
    B, seq_len = qkv.shape[0], qkv.shape[1]
    return (qkv.new_empty(B, n_heads, seq_len, head_dim), qkv.new_empty(B, n_heads, seq_len, head_dim),
            qkv.new_empty(B, n_heads, seq_len, head_dim))


# ---------------------------------------------------------------------------
# Analytic backward (frozen norm weights / adaLN / RoPE), reference :658-790
# ---------------------------------------------------------------------------

def _rms_norm_modulate_setup(ctx, inputs, output):
    x, weight, scale, eps = inputs
    ctx.save_for_backward(x, weight, scale)
    ctx.eps = eps


def _rms_norm_modulate_backward(ctx, grad_output):
    x, weight, scale = ctx.saved_tensors
    D = x.shape[-1]
    m = 1 + scale.unsqueeze(1)
    g = (grad_output * m * weight).float()
    x_f32 = x.float()
    rrms = torch.rsqrt((x_f32 * x_f32).mean(dim=-1, keepdim=True) + ctx.eps)
    c = (g * x_f32).sum(dim=-1, keepdim=True) / D
    dx = (rrms * (g - x_f32 * rrms * rrms * c)).to(x.dtype)
    return dx, None, None, None


fused_rms_norm_modulate.register_autograd(_rms_norm_modulate_backward,
                                          setup_context=_rms_norm_modulate_setup)


def _rms_norm_gate_residual_setup(ctx, inputs, output):
    x, weight, gate, residual, eps = inputs
    ctx.save_for_backward(x, weight, gate)
    ctx.eps = eps


def _rms_norm_gate_residual_backward(ctx, grad_output):
    x, weight, gate = ctx.saved_tensors
    D = x.shape[-1]
    gate_tanh = gate.unsqueeze(1).tanh()
    g = (grad_output * gate_tanh * weight).float()
    x_f32 = x.float()
    rrms = torch.rsqrt((x_f32 * x_f32).mean(dim=-1, keepdim=True) + ctx.eps)
    c = (g * x_f32).sum(dim=-1, keepdim=True) / D
    dx = (rrms * (g - x_f32 * rrms * rrms * c)).to(x.dtype)
    return dx, None, None, grad_output, None


fused_rms_norm_gate_residual.register_autograd(_rms_norm_gate_residual_backward,
                                               setup_context=_rms_norm_gate_residual_setup)


def _qkv_postprocess_setup(ctx, inputs, output):
    qkv, q_norm_w, k_norm_w, freqs_cis, n_heads, head_dim, norm_eps = inputs
    ctx.save_for_backward(qkv, q_norm_w, k_norm_w, freqs_cis)
    ctx.n_heads = n_heads
    ctx.head_dim = head_dim
    ctx.norm_eps = norm_eps


def _qkv_postprocess_backward(ctx, grad_q, grad_k, grad_v):
    qkv, q_norm_w, k_norm_w, freqs_cis = ctx.saved_tensors
    n_heads, head_dim, norm_eps = ctx.n_heads, ctx.head_dim, ctx.norm_eps
    B, seq_len, _ = qkv.shape
    dim = n_heads * head_dim
    n_pairs = head_dim // 2
    dq = grad_q.movedim(1, 2).contiguous()
    dk = grad_k.movedim(1, 2).contiguous()
    dv = grad_v.movedim(1, 2).contiguous()
    freqs = freqs_cis.squeeze(2) if freqs_cis.ndim == 6 else freqs_cis
    cos_val = freqs[:, :, :, 0, 0].unsqueeze(2)
    sin_val = freqs[:, :, :, 1, 0].unsqueeze(2)

    def inv_rope(d):
        pr = d.reshape(B, seq_len, n_heads, n_pairs, 2)
        e, o = pr[..., 0], pr[..., 1]
        return torch.stack([cos_val * e + sin_val * o, -sin_val * e + cos_val * o],
                           dim=-1).reshape(B, seq_len, n_heads, head_dim)

    def norm_bwd(d_pre, raw, w):
        r32 = raw.float()
        rrms = torch.rsqrt((r32 * r32).mean(dim=-1, keepdim=True) + norm_eps)
        g = (d_pre * w).float()
        c = (g * r32).sum(dim=-1, keepdim=True) / head_dim
        return (rrms * (g - r32 * rrms * rrms * c)).to(qkv.dtype)

    dq_raw = norm_bwd(inv_rope(dq), qkv[:, :, :dim].reshape(B, seq_len, n_heads, head_dim), q_norm_w)
    dk_raw = norm_bwd(inv_rope(dk), qkv[:, :, dim:2 * dim].reshape(B, seq_len, n_heads, head_dim), k_norm_w)
    dqkv = torch.cat([dq_raw.reshape(B, seq_len, dim), dk_raw.reshape(B, seq_len, dim),
                      dv.reshape(B, seq_len, dim)], dim=-1)
    return dqkv, None, None, None, None, None, None


fused_qkv_postprocess.register_autograd(_qkv_postprocess_backward, setup_context=_qkv_postprocess_setup)
