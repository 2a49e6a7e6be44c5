"""GPU parity: fused RMSNorm / adaLN / RoPE prologues vs the CPU oracle."""

from __future__ import annotations

import pytest
import torch

from oracle import fused as OF
from tests.conftest import gen
from tests.helpers import bf16_ulp_diff, cosine

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _triton_division():
    """Evaluate the oracle's Triton-kernel quotients with Triton's own fp32 divide on the GPU."""
    from oracle import quant as _OQ
    from tests.helpers import triton_divide

    with _OQ.division(triton_divide):
        yield


def _close(a, b):
    # one rounding to bf16 in both; rsqrt/sum order may move the last bit
    assert torch.allclose(a.float().cpu(), b.float(), rtol=2**-7, atol=2**-7)
    assert cosine(a, b) > 0.99999


@pytest.mark.parametrize("B,S,dim", [(1, 1, 128), (2, 40, 512), (1, 4608, 3072), (2, 4288, 3840), (3, 7, 8192)])
@pytest.mark.parametrize("wdt", [torch.bfloat16, torch.float32])
def test_rms_norm_modulate(cuda_device, B, S, dim, wdt):
    from futudiffu_b200.fused_kernels import fused_rms_norm_modulate

    g = gen(B * S + dim)
    x = torch.randn(B, S, dim, generator=g).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(dim, generator=g)).to(wdt)
    sc = (0.5 * torch.randn(B, dim, generator=g)).to(torch.bfloat16)
    out = fused_rms_norm_modulate(x.to(cuda_device), w.to(cuda_device), sc.to(cuda_device), 1e-5)
    _close(out, OF.rms_norm_modulate(x, w, sc))


@pytest.mark.parametrize("B,S,dim", [(2, 40, 512), (1, 4608, 3072)])
def test_rms_norm_gate_residual(cuda_device, B, S, dim):
    from futudiffu_b200.fused_kernels import fused_rms_norm_gate_residual

    g = gen(S)
    x = torch.randn(B, S, dim, generator=g).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(dim, generator=g)).to(torch.bfloat16)
    gt = torch.randn(B, dim, generator=g).to(torch.bfloat16)
    r = torch.randn(B, S, dim, generator=g).to(torch.bfloat16)
    d = lambda t: t.to(cuda_device)  # noqa: E731
    out = fused_rms_norm_gate_residual(d(x), d(w), d(gt), d(r), 1e-5)
    _close(out, OF.rms_norm_gate_residual(x, w, gt, r))


def test_fused_golden(cuda_device, golden_dir):
    from futudiffu_b200.fused_kernels import (
        fused_qkv_postprocess,
        fused_rms_norm_gate_residual,
        fused_rms_norm_modulate,
    )

    d = torch.load(golden_dir / "fused_norms.pt")
    c = lambda t: t.to(cuda_device)  # noqa: E731
    mod = fused_rms_norm_modulate(c(d["x"]), c(d["w"]), c(d["scale"]), 1e-5)
    assert bf16_ulp_diff(mod, d["modulate"]).max().item() <= 2
    gr = fused_rms_norm_gate_residual(c(d["x"]), c(d["w"]), c(d["gate"]), c(d["res"]), 1e-5)
    assert torch.allclose(gr.float().cpu(), d["gate_residual"].float(), rtol=2**-7, atol=2**-6)
    q, k, v = fused_qkv_postprocess(c(d["qkv"]), c(d["qw"]), c(d["kw"]), c(d["freqs"]), d["H"], d["hd"], 1e-5)
    assert torch.equal(v.cpu(), d["v"])
    for a, b in ((q, d["q"]), (k, d["k"])):
        for h in range(d["H"]):
            assert cosine(a[:, h], b[:, h]) > 0.999


@pytest.mark.parametrize("B,S,H", [(1, 3, 1), (2, 40, 4), (1, 4608, 24)])
def test_qkv_postprocess(cuda_device, B, S, H):
    from futudiffu_b200.attention import rope_embed
    from futudiffu_b200.fused_kernels import fused_qkv_postprocess

    hd = 128
    g = gen(S * H)
    qkv = torch.randn(B, S, 3 * H * hd, generator=g).to(torch.bfloat16)
    qw = 1 + 0.1 * torch.randn(hd, generator=g)
    kw = 1 + 0.1 * torch.randn(hd, generator=g)
    pos = torch.stack([torch.zeros(S), (torch.arange(S) % 64).float(), (torch.arange(S) // 64).float()], -1)
    freqs = torch.cat([rope_embed(pos[None, :, i], dd, 256.0) for i, dd in enumerate((32, 48, 48))], dim=-3)
    freqs = freqs.expand(B, S, hd // 2, 2, 2).unsqueeze(2).contiguous()
    c = lambda t: t.to(cuda_device)  # noqa: E731
    q, k, v = fused_qkv_postprocess(c(qkv), c(qw), c(kw), c(freqs), H, hd, 1e-5)
    rq, rk, rv = OF.qkv_postprocess(qkv, qw, kw, freqs, H, hd)
    assert torch.equal(v.cpu(), rv)
    _close(q, rq)
    _close(k, rk)


def test_fused_backward_runs(cuda_device):
    from futudiffu_b200.fused_kernels import fused_rms_norm_modulate

    x = torch.randn(1, 8, 256, device=cuda_device, dtype=torch.bfloat16, requires_grad=True)
    w = torch.ones(256, device=cuda_device, dtype=torch.bfloat16)
    s = torch.zeros(1, 256, device=cuda_device, dtype=torch.bfloat16)
    fused_rms_norm_modulate(x, w, s).float().sum().backward()
    ref_x = x.detach().float().requires_grad_(True)
    (ref_x * torch.rsqrt((ref_x * ref_x).mean(-1, keepdim=True) + 1e-5)).sum().backward()
    assert torch.allclose(x.grad.float(), ref_x.grad, rtol=2e-2, atol=2e-2)


@pytest.mark.parametrize("B,S,dim,wdt", [(1, 1, 128, torch.bfloat16), (2, 37, 384, torch.float32),
                                         (1, 4608, 3072, torch.bfloat16), (3, 5, 5120, torch.bfloat16)])
def test_rms_norm_modulate_quant(cuda_device, B, S, dim, wdt):
    """Norm + 1 x 128 quant in one pass equals the norm followed by the quantiser, code for code."""
    from futudiffu_b200.fp8_kernels import fp8_act_quant
    from futudiffu_b200.fused_kernels import fused_rms_norm_modulate, fused_rms_norm_modulate_quant

    g = gen(B * S + dim)
    x = (torch.randn(B, S, dim, generator=g) * 3).to(torch.bfloat16).to(cuda_device)
    w = (1 + 0.1 * torch.randn(dim, generator=g)).to(wdt).to(cuda_device)
    sc = (0.2 * torch.randn(B, dim, generator=g)).to(torch.bfloat16).to(cuda_device)
    y8, ys = fused_rms_norm_modulate_quant(x, w, sc)
    r8, rs = fp8_act_quant(fused_rms_norm_modulate(x, w, sc))
    assert y8.shape == (B, S, dim) and ys.shape == (B, S, dim // 128)
    assert torch.equal(y8.view(torch.uint8).cpu(), r8.view(torch.uint8).cpu())
    assert torch.equal(ys.cpu(), rs.reshape(B, S, dim // 128).cpu())


@pytest.mark.parametrize("wdt", [torch.float32, torch.bfloat16])
def test_qkv_postprocess_into_joint_buffer(cuda_device, wdt):
    """Writing two streams into one joint buffer equals concatenating their outputs
    (bf16 norm weights: the wrapper's fp32 copies of Q's and K's weights must stay
    distinct until the launch)."""
    from futudiffu_b200.fused_kernels import fused_qkv_postprocess, qkv_postprocess_into

    B, H = 2, 3
    g = gen(77)
    parts = []
    for S in (5, 131):
        qkv = torch.randn(B, S, 3 * H * 128, generator=g).to(torch.bfloat16).to(cuda_device)
        fr = torch.randn(B, S, 64, 2, 2, generator=g).to(cuda_device)
        parts.append((qkv, fr))
    qw = (1 + 0.1 * torch.randn(128, generator=g)).to(wdt).to(cuda_device)
    kw = (1 + 0.1 * torch.randn(128, generator=g)).to(wdt).to(cuda_device)
    N = 5 + 131
    q, k, v = (torch.empty(B, H, N, 128, dtype=torch.bfloat16, device=cuda_device) for _ in range(3))
    off = 0
    refs = []
    for qkv, fr in parts:
        qkv_postprocess_into(qkv, qw, kw, fr, q, k, v, off)
        refs.append(fused_qkv_postprocess(qkv, qw, kw, fr, H, 128))
        off += qkv.shape[1]
    for i, t in enumerate((q, k, v)):
        assert torch.equal(t.cpu(), torch.cat([r[i] for r in refs], dim=2).cpu())


@pytest.mark.parametrize("qk,gran,pv", [("int8", "per_block", "fp8"), ("int8", "per_token", "bf16"),
                                        ("fp8", "per_token", "fp8"), ("fp8", "per_block", "bf16")])
def test_fused_qkv_prologue_matches_unfused(cuda_device, qk, gran, pv):
    """P3 fused with the quantisation prologue (two streams of a joint attention)
    gives the Q codes and scales, the bf16 K / V and the V codes of P3 followed by
    the separate prologue; the K mean (summed in another order) within one bf16
    rounding, the K codes wherever the means agree."""
    import math

    from futudiffu_b200.attention import rope_embed
    from futudiffu_b200.fused_kernels import fused_qkv_postprocess
    from futudiffu_b200.sage_attention import quantize_qkv, quantize_qkv_streams

    g = gen(71)
    B, H, S1, S2 = 2, 3, 256, 300
    N = S1 + S2
    d = lambda t: t.to(cuda_device)  # noqa: E731
    qkvs = [d(torch.randn(B, S, 3 * H * 128, generator=g).to(torch.bfloat16)) for S in (S1, S2)]
    qkvs[0][..., H * 128:2 * H * 128] += 2.0  # a K offset for the smoothing to remove
    frs = []
    for S in (S1, S2):
        pos = torch.arange(S).float()
        f = torch.cat([rope_embed(pos, 64, 256.0), rope_embed(pos * 0.5, 64, 256.0)], dim=-3)
        frs.append(d(f.unsqueeze(0).expand(B, S, 64, 2, 2).contiguous()))
    # bf16 norm weights as the models hold them; the reference P3 is the fused op
    qw = d((1 + 0.1 * torch.randn(128, generator=g)).to(torch.bfloat16))
    kw = d((1 + 0.1 * torch.randn(128, generator=g)).to(torch.bfloat16))
    parts = [fused_qkv_postprocess(qkvs[i], qw, kw, frs[i], H, 128) for i in range(2)]
    q, k, v = (torch.cat([parts[0][j], parts[1][j]], dim=2) for j in range(3))
    sm = 1 / math.sqrt(128)
    BH = B * H
    ref = quantize_qkv(q.reshape(BH, N, 128), k.reshape(BH, N, 128), v.reshape(BH, N, 128), sm, smooth_k=True,
                       qk_quant=qk, granularity=gran, pv_quant=pv)
    got = quantize_qkv_streams([(qkvs[0], qw, kw, frs[0], 0, 1e-5), (qkvs[1], qw, kw, frs[1], S1, 1e-5)], H, N, sm,
                               smooth_k=True, qk_quant=qk, granularity=gran, pv_quant=pv)
    assert torch.equal(got["k"], k.reshape(BH, N, 128)) and torch.equal(got["v"], v.reshape(BH, N, 128))
    assert torch.equal(got["q_codes"].view(torch.uint8), ref["q_codes"].view(torch.uint8))
    assert torch.equal(got["q_desc"], ref["q_desc"])
    if pv == "fp8":
        assert torch.equal(got["v_codes"].view(torch.uint8), ref["v_codes"].view(torch.uint8))
        assert torch.equal(got["v_desc"], ref["v_desc"])
    dm = (got["k_mean"] - ref["k_mean"]).abs()
    assert (dm <= ref["k_mean"].abs() * 2 ** -7 + 1e-30).all()
    same = (dm == 0).all(dim=1)  # heads whose means agree exactly
    assert same.float().mean() >= 0.5
    kc_g, kc_r = got["k_codes"].view(torch.uint8)[same], ref["k_codes"].view(torch.uint8)[same]
    assert torch.equal(kc_g, kc_r)
    assert torch.equal(got["k_desc"][same], ref["k_desc"][same])


@pytest.mark.parametrize("qk,gran,pv,two,bias", [("int8", "per_block", "bf16", True, False),
                                                 ("int8", "per_token", "fp8", True, True),
                                                 ("fp8", "per_block", "fp8", False, False),
                                                 ("fp8", "per_token", "bf16", False, True),
                                                 ("int8", "per_block", "fp8", False, True)])
def test_qkv_linear_fused_prologue_matches_unfused(cuda_device, qk, gran, pv, two, bias):
    """The QKV linear with P3 and the prologue's first pass in its epilogue
    (fd_fp8_gemm_qkv_quant, one or two streams in one launch) equals the bf16 GEMM
    followed by the fused P3 + prologue, code for code: Q codes and descales, bf16
    K / V, the K mean, K / V codes and descales."""
    import math

    from futudiffu_b200 import fp8_kernels as FK
    from futudiffu_b200.attention import rope_embed
    from futudiffu_b200.sage_attention import quantize_qkv_linear_streams, quantize_qkv_streams
    from oracle import quant as OQ

    g = gen(73)
    B, H, K = 2, 4, 256
    lens = (256, 384) if two else (512,)
    N = sum(lens)
    d = lambda t: t.to(cuda_device)  # noqa: E731
    streams_lin, streams_bf16 = [], []
    off = 0
    for S in lens:
        x = torch.randn(B, S, K, generator=g)
        w = torch.randn(3 * H * 128, K, generator=g) * 0.05
        w[H * 128:2 * H * 128] += 0.02  # a K offset for the smoothing to remove
        a8, a_s = (d(t) for t in OQ.act_quant(x.to(torch.bfloat16)))
        w8, ws = (d(t) for t in OQ.weight_quant(w))
        bv = d((torch.randn(3 * H * 128, generator=g) * 0.1).to(torch.bfloat16)) if bias else None
        pos = torch.arange(S).float()
        f = torch.cat([rope_embed(pos, 64, 256.0), rope_embed(pos * 0.5, 64, 256.0)], dim=-3)
        fr = d(f.unsqueeze(0).expand(B, S, 64, 2, 2).contiguous())
        qw = d((1 + 0.1 * torch.randn(128, generator=g)).to(torch.bfloat16))
        kw = d((1 + 0.1 * torch.randn(128, generator=g)).to(torch.bfloat16))
        qkv = (FK.fp8_addmm_blockwise(a8, a_s, w8, ws, bias=bv, output_dtype=torch.bfloat16) if bias
               else FK.fp8_gemm_blockwise(a8, a_s, w8, ws, output_dtype=torch.bfloat16))
        streams_lin.append((a8, a_s, w8, ws, bv, qw, kw, fr, off, 1e-5))
        streams_bf16.append((qkv, qw, kw, fr, off, 1e-5))
        off += S
    sm = 1 / math.sqrt(128)
    kw_ = dict(smooth_k=True, qk_quant=qk, granularity=gran, pv_quant=pv)
    got = quantize_qkv_linear_streams(streams_lin, H, N, sm, **kw_)
    ref = quantize_qkv_streams(streams_bf16, H, N, sm, **kw_)
    for key in ("k", "v", "q_codes", "q_desc", "k_mean", "k_codes", "k_desc", "v_codes", "v_desc"):
        a, b = got[key], ref[key]
        if a is None:
            assert b is None
            continue
        if a.dtype in (torch.int8, torch.float8_e4m3fn):
            a, b = a.view(torch.uint8), b.view(torch.uint8)
        assert torch.equal(a, b), key
