"""CPU restatement of the DiT blocks (oracle; test infrastructure only).

Composes the oracle's restatements of the hot-path ops exactly as
futudiffu_b200.dit composes the kernels: G1 activation quant + G2 blockwise
GEMM for every linear (the GELU-tanh MLP through the bf16 GEMM output and the
G1 quantiser, as the fused epilogue defines it), P1/P2 norms, P3 QKV
post-processing and the A1-A5 quantized attention (per-block INT8 QK, e4m3 P
and V).  The torch bf16 glue (adaLN, timestep MLP, patch projections) runs in
fp32 on the CPU from the same weights.  Each step is a reference-path
computation: act quant fp8_kernels.py:54-90, GEMM :125-343, norms
fused_kernels.py:43-247, QKV :270-471, attention sage_kernels.py:1379-1477.
"""

from __future__ import annotations

import contextlib

import torch

from oracle import attention as OA
from oracle import fused as OF
from oracle import gemm as OG
from oracle import quant as OQ


def _cpu(t):
    return t.detach().cpu()


def _gemm(a8, a_s, w8, ws, bias=None):
    """G2 on (..., K) codes -> (..., N) bf16."""
    out = OG.gemm_blockwise(a8, a_s, _cpu(w8), _cpu(ws), bias=bias, out_dtype=torch.bfloat16)
    return out.reshape(*a8.shape[:-1], out.shape[-1])


def linear(x, lin):
    a8, a_s = OQ.act_quant(x)
    bias = None if lin.bias is None else _cpu(lin.bias)
    return _gemm(a8, a_s, lin.weight, lin.weight_scale, bias)


def mlp(x, w_in, w_out):
    h = linear(x, w_in)                         # bf16 GEMM output
    g8, g_s = OQ.gelu_tanh_quant(h)             # GELU(tanh) + G1
    return _gemm(g8, g_s, w_out.weight, w_out.weight_scale)


def _torch_linear(x, lin):
    return (x.float() @ _cpu(lin.weight).float().t() + _cpu(lin.bias).float()).to(torch.bfloat16)


def attention(q, k, v, cfg):
    B, H, N, D = q.shape
    pv = "fp8_channel" if cfg.pv_quant == "fp8" else "bf16"
    o, _ = OA.attention_forward(q.reshape(B * H, N, D), k.reshape(B * H, N, D), v.reshape(B * H, N, D),
                                qk_quant=cfg.qk_quant, granularity=cfg.granularity, pv_quant=pv)
    return o.reshape(B, H, N, D).transpose(1, 2).reshape(B, N, H * D)


def double_block(blk, x_txt, x_img, vec, freqs_txt, freqs_img):
    cfg = blk.cfg
    x_txt, x_img, vec = _cpu(x_txt), _cpu(x_img), _cpu(vec)
    B = x_txt.shape[0]
    mods, qs, ks, vs = [], [], [], []
    for st, x, fr in ((blk.txt, x_txt, freqs_txt), (blk.img, x_img, freqs_img)):
        m = _torch_linear(torch.nn.functional.silu(vec.float()).to(torch.bfloat16), st.adaln).chunk(4, dim=-1)
        mods.append(m)
        h = OF.rms_norm_modulate(x, _cpu(st.norm_w[0]), m[0], cfg.eps)
        qkv = linear(h, st.qkv)
        q, k, v = OF.qkv_postprocess(qkv, _cpu(st.q_norm), _cpu(st.k_norm), _cpu(fr), cfg.heads, 128, cfg.eps)
        qs.append(q.to(torch.bfloat16))
        ks.append(k.to(torch.bfloat16))
        vs.append(v.to(torch.bfloat16))
    o = attention(torch.cat(qs, 2), torch.cat(ks, 2), torch.cat(vs, 2), cfg)
    o_txt, o_img = o.split([x_txt.shape[1], x_img.shape[1]], dim=1)
    outs = []
    for st, x, o_s, m in ((blk.txt, x_txt, o_txt, mods[0]), (blk.img, x_img, o_img, mods[1])):
        a = linear(o_s.contiguous(), st.proj)
        x = OF.rms_norm_gate_residual(a, _cpu(st.norm_w[1]), m[1], x, cfg.eps)
        h = OF.rms_norm_modulate(x, _cpu(st.norm_w[2]), m[2], cfg.eps)
        f = mlp(h, st.mlp_in, st.mlp_out)
        x = OF.rms_norm_gate_residual(f, _cpu(st.norm_w[3]), m[3], x, cfg.eps)
        outs.append(x)
    return outs[0], outs[1]


def single_block(blk, x, vec, freqs):
    cfg = blk.cfg
    x, vec = _cpu(x), _cpu(vec)
    B, N, D = x.shape
    scale, gate = _torch_linear(torch.nn.functional.silu(vec.float()).to(torch.bfloat16), blk.adaln).chunk(2, dim=-1)
    h = OF.rms_norm_modulate(x, _cpu(blk.norm_w[0]), scale, cfg.eps)
    a8, a_s = OQ.act_quant(h)
    w, ws = _cpu(blk.linear1.weight), _cpu(blk.linear1.weight_scale)
    n_qkv = 3 * D
    qkv = _gemm(a8, a_s, w[:n_qkv], ws[: n_qkv // 128])
    hm = _gemm(a8, a_s, w[n_qkv:], ws[n_qkv // 128:])
    m8, m_s = OQ.gelu_tanh_quant(hm)
    q, k, v = OF.qkv_postprocess(qkv, _cpu(blk.q_norm), _cpu(blk.k_norm), _cpu(freqs), cfg.heads, 128, cfg.eps)
    o = attention(q.to(torch.bfloat16), k.to(torch.bfloat16), v.to(torch.bfloat16), cfg)
    o8, o_s = OQ.act_quant(o)
    cat8 = torch.cat([o8.view(torch.uint8), m8.view(torch.uint8)], -1).view(torch.float8_e4m3fn)
    y = _gemm(cat8, torch.cat([o_s, m_s], -1), blk.linear2.weight, blk.linear2.weight_scale)
    return OF.rms_norm_gate_residual(y, _cpu(blk.norm_w[1]), gate, x, cfg.eps)


def dit_forward(model, img, txt, t):
    """The DiT forward on the CPU: timestep MLP, blocks, final modulated projection."""
    import math

    cfg = model.cfg
    img, txt, t = _cpu(img), _cpu(txt), _cpu(t)
    half = cfg.time_dim // 2
    freqs = torch.exp(-math.log(10000.0) * torch.arange(half, dtype=torch.float32) / half)
    args = (t.float() * 1000.0)[:, None] * freqs[None]
    temb = torch.cat([torch.cos(args), torch.sin(args)], -1).to(torch.bfloat16)
    vec = _torch_linear(torch.nn.functional.silu(_torch_linear(temb, model.time_in1).float()).to(torch.bfloat16),
                        model.time_in2)
    x_img = _torch_linear(img, model.img_in)
    x_txt = txt
    B = img.shape[0]
    f_txt, f_img, f_all = (_cpu(f).unsqueeze(0).expand(B, *f.shape).contiguous()
                           for f in (model.freqs_txt, model.freqs_img, model.freqs_all))
    for blk in model.double_blocks:
        x_txt, x_img = double_block(blk, x_txt, x_img, vec, f_txt, f_img)
    x = torch.cat([x_txt, x_img], 1)
    for blk in model.single_blocks:
        x = single_block(blk, x, vec, f_all)
    x_img = x[:, cfg.txt_tokens:].contiguous()
    scale = _torch_linear(torch.nn.functional.silu(vec.float()).to(torch.bfloat16), model.final_adaln)
    h = OF.rms_norm_modulate(x_img, _cpu(model.final_norm), scale, cfg.eps)
    return _torch_linear(h, model.final_out)


def random_double_block(cfg, seed: int = 0):
    """Weights of one double-stream block built on the CPU alone (oracle weight
    quantiser), with the attribute layout of futudiffu_b200.dit.DoubleStreamBlock."""
    from types import SimpleNamespace

    g = torch.Generator().manual_seed(seed)
    D, R = cfg.hidden, cfg.mlp_ratio

    def rand(shape, std, mean=0.0):
        return (torch.randn(shape, generator=g) * std + mean).to(torch.bfloat16)

    def fp8_linear(n, k):
        w8, ws = OQ.weight_quant(torch.randn(n, k, generator=g) * 0.02)
        return SimpleNamespace(weight=w8, weight_scale=ws, bias=None)

    def stream():
        return SimpleNamespace(
            adaln=SimpleNamespace(weight=rand((4 * D, D), 0.02), bias=rand((4 * D,), 0.02)),
            norm_w=[rand((D,), 0.05, 1.0) for _ in range(4)],
            q_norm=rand((128,), 0.05, 1.0), k_norm=rand((128,), 0.05, 1.0),
            qkv=fp8_linear(3 * D, D), proj=fp8_linear(D, D),
            mlp_in=fp8_linear(R * D, D), mlp_out=fp8_linear(D, R * D))

    return SimpleNamespace(cfg=cfg, txt=stream(), img=stream())


def random_single_block(cfg, seed: int = 0):
    """Weights of one single-stream block built on the CPU alone, with the
    attribute layout of futudiffu_b200.dit.SingleStreamBlock."""
    from types import SimpleNamespace

    g = torch.Generator().manual_seed(seed)
    D, R = cfg.hidden, cfg.mlp_ratio

    def rand(shape, std, mean=0.0):
        return (torch.randn(shape, generator=g) * std + mean).to(torch.bfloat16)

    def fp8_linear(n, k):
        w8, ws = OQ.weight_quant(torch.randn(n, k, generator=g) * 0.02)
        return SimpleNamespace(weight=w8, weight_scale=ws, bias=None)

    return SimpleNamespace(
        cfg=cfg, adaln=SimpleNamespace(weight=rand((2 * D, D), 0.02), bias=rand((2 * D,), 0.02)),
        norm_w=[rand((D,), 0.05, 1.0) for _ in range(2)],
        q_norm=rand((128,), 0.05, 1.0), k_norm=rand((128,), 0.05, 1.0),
        linear1=fp8_linear(3 * D + R * D, D), linear2=fp8_linear(D, D + R * D))


@contextlib.contextmanager
def eager_cpu_timing():
    """The reference's torch-eager dequantize-and-compute CPU formulation, used
    only to time the CPU baseline: linears as dequantised operands in one fp32
    matmul (oracle.gemm.dequant_compute), attention matmuls in fp32.  Quantisers,
    norms and the online softmax are the same restatements as in parity mode."""
    with OG.dequant_compute(), OA.matmul_dtype(torch.float32):
        yield


def random_video_block(cfg, seed: int = 0):
    """Weights of one video block built on the CPU alone, with the attribute layout
    of futudiffu_b200.dit.VideoBlock."""
    from types import SimpleNamespace

    g = torch.Generator().manual_seed(seed)
    D = cfg.hidden

    def rand(shape, std, mean=0.0):
        return (torch.randn(shape, generator=g) * std + mean).to(torch.bfloat16)

    def fp8_linear(n, k):
        w8, ws = OQ.weight_quant(torch.randn(n, k, generator=g) * 0.02)
        return SimpleNamespace(weight=w8, weight_scale=ws, bias=None)

    return SimpleNamespace(
        cfg=cfg, adaln=SimpleNamespace(weight=rand((4 * D, D), 0.02), bias=rand((4 * D,), 0.02)),
        norm_w=[rand((D,), 0.05, 1.0) for _ in range(6)], cross_gate=rand((1, D), 0.5),
        q_norm=rand((128,), 0.05, 1.0), k_norm=rand((128,), 0.05, 1.0),
        qkv=fp8_linear(3 * D, D), proj=fp8_linear(D, D), cq=fp8_linear(D, D), ckv=fp8_linear(2 * D, D),
        co=fp8_linear(D, D), ffn_in=fp8_linear(cfg.ffn, D), ffn_out=fp8_linear(D, cfg.ffn))


def video_block(blk, x, vec, txt, freqs):
    """futudiffu_b200.dit.VideoBlock on the CPU, single rank (the whole sequence)."""
    cfg = blk.cfg
    x, vec, txt = _cpu(x), _cpu(vec), _cpu(txt)
    _, L, D = x.shape
    H = cfg.heads
    m = _torch_linear(torch.nn.functional.silu(vec.float()).to(torch.bfloat16), blk.adaln).chunk(4, dim=-1)
    h = OF.rms_norm_modulate(x, _cpu(blk.norm_w[0]), m[0], cfg.eps)
    qkv = linear(h, blk.qkv)
    q, k, v = OF.qkv_postprocess(qkv, _cpu(blk.q_norm), _cpu(blk.k_norm), _cpu(freqs), H, 128, cfg.eps)
    o = attention(q.to(torch.bfloat16), k.to(torch.bfloat16), v.to(torch.bfloat16), cfg)
    x = OF.rms_norm_gate_residual(linear(o, blk.proj), _cpu(blk.norm_w[1]), m[1], x, cfg.eps)
    hc = OF.rms_norm_modulate(x, _cpu(blk.norm_w[2]), torch.zeros_like(m[0]), cfg.eps)
    qc = linear(hc, blk.cq).view(1, L, H, 128).transpose(1, 2).float()
    kv = linear(txt, blk.ckv).view(1, -1, 2, H, 128).float()
    kc, vc = kv[:, :, 0].transpose(1, 2), kv[:, :, 1].transpose(1, 2)
    oc = torch.nn.functional.scaled_dot_product_attention(qc, kc, vc).to(torch.bfloat16)
    ac = linear(oc.transpose(1, 2).reshape(1, L, D), blk.co)
    x = OF.rms_norm_gate_residual(ac, _cpu(blk.norm_w[3]), _cpu(blk.cross_gate), x, cfg.eps)
    hf = OF.rms_norm_modulate(x, _cpu(blk.norm_w[4]), m[2], cfg.eps)
    f = mlp(hf, blk.ffn_in, blk.ffn_out)
    return OF.rms_norm_gate_residual(f, _cpu(blk.norm_w[5]), m[3], x, cfg.eps)
