"""CPU restatement of the reference's DiT block (oracle; test infrastructure only).

JointTransformerBlock.forward, src_ii/transformer.py:630-701, composed from the
oracle's restatements of the ops it calls:
  per-batch adaLN (scale / gate (B, dim)): the fused path (:679-699) --
    P1 fused_rms_norm_modulate, FP8Linear (G1 act quant + G2 GEMM) for qkv,
    P3 fused_qkv_postprocess, the masked INT8-QK / bf16-PV attention
    (sage_attn_masked_op -> sage_attention.py:461-531), output linear,
    P2 gate + residual, the FFN chain (w1w3 GEMM -> bf16 -> fp8_silu_gate_quant
    -> w2 GEMM, :551-571), P2;
  per-token adaLN (scale / gate (B, L, dim)): the unfused torch path
    (:656-677): F.rms_norm in bf16, `* (1 + scale)` and `* gate.tanh() + x` as
    bf16 tensor ops, then the same linears and attention.
Weights are read from the B200 module (FP8 codes and scales, norm weights).
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from oracle import attention as OA
from oracle import fused as OF
from oracle import gemm as OG
from oracle import quant as OQ


def _cpu(t):
    return t.detach().cpu()


def _linear(x, lin):
    """FP8Linear.forward: G1 on x (..., K), G2 with the block weights (+ bias)."""
    a8, a_s = OQ.act_quant(x)
    bias = None if lin.bias is None else _cpu(lin.bias)
    out = OG.gemm_blockwise(a8, a_s, _cpu(lin.weight), _cpu(lin.weight_scale), bias=bias, out_dtype=torch.bfloat16)
    return out.reshape(*x.shape[:-1], out.shape[-1])


def attention(att, x, freqs, block_mask):
    """JointAttention.forward (:447-471) on bf16 x (B, L, dim)."""
    B, Lq, dim = x.shape
    H = att.n_local_heads
    qkv = _linear(x, att.qkv)
    q, k, v = OF.qkv_postprocess(qkv, att.q_norm.weight, att.k_norm.weight, freqs, H, 128, att.q_norm.eps)
    o, _ = OA.attention_forward(q.reshape(B * H, Lq, 128), k.reshape(B * H, Lq, 128), v.reshape(B * H, Lq, 128),
                                qk_quant="int8", granularity="per_token", pv_quant="bf16",
                                block_mask=_cpu(block_mask))
    o = o.reshape(B, H, Lq, 128).transpose(1, 2).reshape(B, Lq, dim)
    return _linear(o, att.out)


def feed_forward(ffn, x):
    """The fused FP8 chain (:551-571)."""
    h = _linear(x, ffn.w1w3)                      # bf16 (.., 2 hidden)
    g8, g_s = OQ.silu_gate_quant(h)
    w2 = ffn.w2
    out = OG.gemm_blockwise(g8.reshape(-1, g8.shape[-1]), g_s.reshape(-1, g_s.shape[-1]), _cpu(w2.weight),
                            _cpu(w2.weight_scale), out_dtype=torch.bfloat16)
    return out.reshape(*x.shape[:-1], out.shape[-1])


def _rms_norm_bf16(x, w, eps):
    return F.rms_norm(x, (x.shape[-1],), weight=w.to(x.dtype), eps=eps)


def block_forward(blk, x, freqs, scales, block_mask):
    """scales = (scale_msa, gate_msa, scale_mlp, gate_mlp), each (B, dim) or (B, L, dim)."""
    x = _cpu(x)
    scale_msa, gate_msa, scale_mlp, gate_mlp = (_cpu(s) for s in scales)
    n1, n2 = blk.attention_norm1, blk.attention_norm2
    f1, f2 = blk.ffn_norm1, blk.ffn_norm2
    if scale_msa.dim() == 3:
        attn_in = _rms_norm_bf16(x, _cpu(n1.weight), n1.eps) * (1 + scale_msa)
        attn_out = attention(blk.attention, attn_in, freqs, block_mask)
        x = _rms_norm_bf16(attn_out, _cpu(n2.weight), n2.eps) * gate_msa.tanh() + x
        ffn_in = _rms_norm_bf16(x, _cpu(f1.weight), f1.eps) * (1 + scale_mlp)
        ffn_out = feed_forward(blk.feed_forward, ffn_in)
        return _rms_norm_bf16(ffn_out, _cpu(f2.weight), f2.eps) * gate_mlp.tanh() + x
    attn_in = OF.rms_norm_modulate(x, _cpu(n1.weight), scale_msa, n1.eps)
    attn_out = attention(blk.attention, attn_in, freqs, block_mask)
    x = OF.rms_norm_gate_residual(attn_out, _cpu(n2.weight), gate_msa, x, n2.eps)
    ffn_in = OF.rms_norm_modulate(x, _cpu(f1.weight), scale_mlp, f1.eps)
    ffn_out = feed_forward(blk.feed_forward, ffn_in)
    return OF.rms_norm_gate_residual(ffn_out, _cpu(f2.weight), gate_mlp, x, f2.eps)


def random_joint_block(dim: int, heads: int, hidden: int, seed: int = 0):
    """Weights of one JointTransformerBlock built on the CPU alone (oracle weight
    quantiser), with the attribute layout ``block_forward`` reads."""
    from types import SimpleNamespace

    from oracle import quant as OQ

    g = torch.Generator().manual_seed(seed)

    def norm(n):
        return SimpleNamespace(weight=(1 + 0.05 * torch.randn(n, generator=g)).to(torch.bfloat16), eps=1e-5)

    def fp8_linear(n, k):
        w8, ws = OQ.weight_quant(torch.randn(n, k, generator=g) * (k ** -0.5))
        return SimpleNamespace(weight=w8, weight_scale=ws, bias=None)

    att = SimpleNamespace(n_local_heads=heads, qkv=fp8_linear(3 * dim, dim), out=fp8_linear(dim, dim),
                          q_norm=norm(128), k_norm=norm(128))
    ffn = SimpleNamespace(w1w3=fp8_linear(2 * hidden, dim), w2=fp8_linear(dim, hidden))
    return SimpleNamespace(attention=att, feed_forward=ffn, attention_norm1=norm(dim), attention_norm2=norm(dim),
                           ffn_norm1=norm(dim), ffn_norm2=norm(dim))
