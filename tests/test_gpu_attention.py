"""GPU parity: attention quantisation prologue (bit-exact) and tcgen05 attention vs the oracle."""

from __future__ import annotations

import math

import pytest
import torch

from oracle import attention as OA
from oracle import block_mask as OB
from tests.conftest import gen
from tests.helpers import cosine, e4m3_bits

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _triton_division():
    """Evaluate the oracle's Triton-kernel quotients with Triton's own fp32 divide on the GPU."""
    from oracle import quant as _OQ
    from tests.helpers import triton_divide

    with _OQ.division(triton_divide):
        yield

SM = 1.0 / math.sqrt(128)


def qkv(BH, N, seed, koff=2.0):
    g = gen(seed)
    q = torch.randn(BH, N, 128, generator=g).to(torch.bfloat16)
    k = (torch.randn(BH, N, 128, generator=g) + koff * torch.randn(128, generator=g)).to(torch.bfloat16)
    v = torch.randn(BH, N, 128, generator=g).to(torch.bfloat16)
    return q, k, v


@pytest.fixture(autouse=True)
def _reset_sage():
    from futudiffu_b200 import sage_attention as SA

    yield
    SA.configure_sage()


@pytest.mark.parametrize("qk", ["int8", "fp8"])
@pytest.mark.parametrize("gran", ["per_token", "per_block"])
@pytest.mark.parametrize("N", [64, 200, 1024, 4288])
def test_prologue_codes_bit_exact(cuda_device, qk, gran, N):
    from futudiffu_b200.sage_attention import quantize_qkv

    q, k, v = qkv(3, N, N)
    qz = quantize_qkv(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device), SM, smooth_k=True,
                      qk_quant=qk, granularity=gran, pv_quant="fp8")
    # smoothing mean: bf16-rounded, within one bf16 ulp of torch's
    km_ref = k.float().mean(dim=1).to(torch.bfloat16).float()
    km = qz["k_mean"].cpu()
    assert ((km - km_ref).abs() <= km_ref.abs() * 2**-7 + 1e-30).all()
    # codes and scales bit-exact given the kernel's mean
    ks = OA.smooth_k_with_mean(k, km.to(torch.bfloat16))
    rq, rk = (1, 1) if gran == "per_token" else (128, 64)
    qc, qd = OA.quant_rows(q, qk, rq, SM * OA.LOG2E)
    kc, kd = OA.quant_rows(ks, qk, rk)
    bits = (lambda t: t.cpu().view(torch.uint8)) if qk == "fp8" else (lambda t: t.cpu())
    assert torch.equal(bits(qz["q_codes"]), bits(qc))
    assert torch.equal(bits(qz["k_codes"]), bits(kc))
    assert torch.equal(qz["q_desc"].cpu()[:, :qd.shape[1]], qd)
    assert torch.equal(qz["k_desc"].cpu()[:, :kd.shape[1]], kd)
    vc, vd = OA.quant_v_per_channel(v)
    assert torch.equal(e4m3_bits(qz["v_codes"]), e4m3_bits(vc))
    assert torch.equal(qz["v_desc"].cpu(), vd)


def test_prologue_deterministic(cuda_device):
    from futudiffu_b200.sage_attention import quantize_qkv

    q, k, v = (t.to(cuda_device) for t in qkv(4, 3000, 1))
    a = quantize_qkv(q, k, v, SM, smooth_k=True, qk_quant="int8", granularity="per_token", pv_quant="fp8")
    b = quantize_qkv(q, k, v, SM, smooth_k=True, qk_quant="int8", granularity="per_token", pv_quant="fp8")
    for key in ("q_codes", "k_codes", "q_desc", "k_desc", "v_desc", "k_mean"):
        assert torch.equal(a[key], b[key]), key


# (qk_quant, granularity, pv_quant for the API, oracle pv mode, min cosine vs oracle)
MODES = [
    ("int8", "per_token", "bf16", "bf16", 0.9995),
    ("fp8", "per_token", "bf16", "bf16", 0.9995),
    ("int8", "per_block", "bf16", "bf16", 0.9995),
    ("int8", "per_block", "fp8", "fp8_channel", 0.9995),
    ("fp8", "per_block", "fp8", "fp8_channel", 0.9995),
    # the reference's FP8-PV kernel: P per row and V per column, per 64-key tile
    ("fp8", "per_token", "fp8_tile", "fp8_tile", 0.9995),
    ("int8", "per_token", "fp8_tile", "fp8_tile", 0.9995),
]


def _run(q, k, v, dev, qk, gran, pv, mask=None, lse=True):
    from futudiffu_b200 import sage_attention as SA

    SA.configure_sage(smooth_k=True, qk_quant=qk, pv_quant="fp8" if pv == "fp8_tile" else pv, qk_granularity=gran)
    d = lambda t: t.to(dev)  # noqa: E731
    B = 1
    q4, k4, v4 = (d(t).unsqueeze(0) for t in (q, k, v))
    if mask is not None:
        out, l = SA._attn_forward(q4, k4, v4, SM, block_mask=d(mask), qk_quant=qk, pv_quant=pv,
                                  granularity=gran, want_lse=True)
    else:
        out, l = SA._attn_forward(q4, k4, v4, SM, block_mask=None, qk_quant=qk, pv_quant=pv,
                                  granularity=gran, want_lse=True)
    return out[0].cpu(), l.cpu()


def check_fp8p_accuracy(out, ref, q, k, v, margin=2e-4):
    """e4m3-P results carry ~3% element noise that differs between two valid
    roundings (this kernel rescales against a running max that may trail the
    true max by up to 2 log2 units, the reference formulation against the true
    max).  Gate: at least as close to exact attention as the reference
    formulation, and close to it."""
    exact = OA.attention_exact(q, k, v, SM)
    c_ours, c_ref = cosine(out, exact), cosine(ref, exact)
    assert c_ours >= c_ref - margin, (c_ours, c_ref)
    assert cosine(out, ref) >= 0.998


@pytest.mark.parametrize("mode", MODES, ids=lambda m: "-".join(m[:3]))
@pytest.mark.parametrize("BH,N", [(2, 128), (3, 200), (2, 1024), (1, 4288)])
def test_attention_vs_oracle(cuda_device, mode, BH, N):
    qk, gran, pv, opv, tol = mode
    q, k, v = qkv(BH, N, BH * N)
    out, lse = _run(q, k, v, cuda_device, qk, gran, pv)
    ref, rlse = OA.attention_forward(q, k, v, sm_scale=SM, qk_quant=qk, granularity=gran, pv_quant=opv)
    assert torch.isfinite(out.float()).all()
    if opv in ("bf16", "fp8_tile"):
        # bf16 P, or e4m3 P rounded exactly as the oracle (the reference's per-tile scales)
        c = cosine(out, ref)
        assert c >= tol, c
    else:
        check_fp8p_accuracy(out, ref, q, k, v)
    err = (out.float() - ref.float()).abs().max().item()
    assert err <= 0.05 * ref.float().abs().max().item() + 0.02, err
    assert torch.allclose(lse, rlse, rtol=0, atol=2e-3 * max(1.0, rlse.abs().max().item()))


def test_attention_fp8_pv_reference_tile_mode(cuda_device):
    # reference A4 (per-64-key-tile P/V scales) vs this build's per-channel V: tolerance gate
    q, k, v = qkv(2, 1024, 7)
    out, _ = _run(q, k, v, cuda_device, "fp8", "per_token", "fp8")
    ref, _ = OA.attention_forward(q, k, v, sm_scale=SM, qk_quant="fp8", pv_quant="fp8_tile")
    check_fp8p_accuracy(out, ref, q, k, v, margin=5e-4)


def test_attention_close_to_exact(cuda_device):
    q, k, v = qkv(2, 2048, 3)
    exact = OA.attention_exact(q, k, v, SM)
    out, _ = _run(q, k, v, cuda_device, "int8", "per_block", "fp8")
    assert cosine(out, exact) >= 0.998
    out, _ = _run(q, k, v, cuda_device, "int8", "per_token", "bf16")
    assert cosine(out, exact) >= 0.9995


@pytest.mark.parametrize("segs,total", [([128, 256, 64], None), ([100, 160, 40], None), ([1000, 2000], 3100),
                                        ([2144, 2144], 4288)])
def test_attention_block_mask(cuda_device, segs, total):
    N = total or sum(segs)
    mask = torch.from_numpy(OB.build_block_mask(segs, total))
    q, k, v = qkv(2, N, N)
    for qk, gran, pv, opv, _ in (MODES[0], MODES[3]):
        out, lse = _run(q, k, v, cuda_device, qk, gran, pv, mask=mask)
        ref, rlse = OA.attention_forward(q, k, v, sm_scale=SM, qk_quant=qk, granularity=gran,
                                         pv_quant=opv, block_mask=mask)
        assert cosine(out, ref) >= (0.9995 if opv == "bf16" else 0.998)
        assert torch.allclose(lse, rlse, atol=5e-3)


def test_attention_mask_3d_and_fully_masked_rows(cuda_device):
    N = 256
    q, k, v = qkv(2, N, 11)
    mask = torch.ones(2, 2, 4, dtype=torch.uint8)
    mask[1, 1, :] = 0  # head 1, q block 1 sees nothing -> NaN output, -inf lse
    mask[0, 0, 2:] = 0
    out, lse = _run(q, k, v, cuda_device, "int8", "per_token", "bf16", mask=mask)
    ref, rlse = OA.attention_forward(q, k, v, sm_scale=SM, qk_quant="int8", block_mask=mask)
    assert torch.isnan(out[1, 128:].float()).all()
    assert torch.isneginf(lse[1, 128:]).all()
    good = torch.ones(2, N, dtype=torch.bool)
    good[1, 128:] = False
    assert cosine(out[good], ref[good]) >= 0.9995


def test_attention_public_api(cuda_device):
    from futudiffu_b200 import sage_attention as SA
    from futudiffu_b200.attention import sdpa_attention, set_attention_backend

    B, H, N = 2, 3, 256
    g = gen(2)
    q = torch.randn(B, H, N, 128, generator=g).to(torch.bfloat16).to(cuda_device)
    k = torch.randn(B, H, N, 128, generator=g).to(torch.bfloat16).to(cuda_device)
    v = torch.randn(B, H, N, 128, generator=g).to(torch.bfloat16).to(cuda_device)
    SA.configure_sage(qk_quant="int8")
    o1 = SA.sage_attn_forward(q, k, v)
    o2, lse = SA.sage_attn_forward_with_lse(q, k, v)
    o3, lse3 = SA.sage_attn_op(q, k, v, SM)
    assert o1.shape == (B, H, N, 128) and lse.shape == (B * H, N)
    assert torch.equal(o1, o2) and torch.equal(o2, o3) and torch.equal(lse, lse3)
    set_attention_backend("sage")
    try:
        flat = sdpa_attention(q.transpose(1, 2).reshape(B, N, H * 128), k.transpose(1, 2).reshape(B, N, H * 128),
                              v.transpose(1, 2).reshape(B, N, H * 128), heads=H)
    finally:
        set_attention_backend("sdpa")
    assert torch.equal(flat, o3.transpose(1, 2).reshape(B, N, H * 128))


def test_attention_deterministic(cuda_device):
    q, k, v = qkv(4, 2048, 5)
    a, la = _run(q, k, v, cuda_device, "int8", "per_block", "fp8")
    b, lb = _run(q, k, v, cuda_device, "int8", "per_block", "fp8")
    assert torch.equal(a, b) and torch.equal(la, lb)


def test_attention_config2_full_size(cuda_device):
    # benchmark config 2: B2 H24 S4096, K offset ~N(0, 4); all heads vs GPU fp32 softmax,
    # two heads vs the CPU oracle
    from futudiffu_b200 import sage_attention as SA

    B, H, N = 2, 24, 4096
    g = gen(2024)
    q = torch.randn(B, H, N, 128, generator=g).to(torch.bfloat16)
    k = (torch.randn(B, H, N, 128, generator=g) + 2.0 * torch.randn(128, generator=g)).to(torch.bfloat16)
    v = torch.randn(B, H, N, 128, generator=g).to(torch.bfloat16)
    SA.configure_sage(smooth_k=True, qk_quant="int8", pv_quant="fp8", qk_granularity="per_block")
    out = SA.sage_attn_forward(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device))
    qd, kd, vd = (t.to(cuda_device).float() for t in (q, k, v))
    exact = torch.nn.functional.scaled_dot_product_attention(qd, kd, vd)
    assert cosine(out, exact) >= 0.998
    q2, k2, v2 = (t[0, :2].contiguous() for t in (q, k, v))
    ref, _ = OA.attention_forward(q2, k2, v2, sm_scale=SM, qk_quant="int8", granularity="per_block",
                                  pv_quant="fp8_channel")
    check_fp8p_accuracy(out[0, :2].cpu(), ref, q2, k2, v2)


def test_attention_status_clean(cuda_device):
    from futudiffu_b200 import check_status

    check_status()


@pytest.mark.parametrize("gran", ["per_token", "per_block"])
@pytest.mark.parametrize("qk", ["int8", "fp8"])
@pytest.mark.parametrize("N,docs", [(256, None), (200, None), (201, None), (65, None), (384, [128, 256]),
                                    (448, [200, 248])])
def test_attention_backward_vs_oracle(cuda_device, qk, N, docs, gran):
    """The tcgen05 backward (dK/dV and dQ kernels) at aligned, ragged and masked
    sizes (documents of 200 + 248 tokens leave half-masked 128-key tiles and
    skipped steps).  Both granularities: the backward recomputes P with the
    forward's Q/K scales (bf16 PV, so the forward is the oracle's)."""
    from futudiffu_b200 import sage_attention as SA

    BH = 2
    q, k, v = qkv(BH, N, 31 + N)
    g = gen(77)
    dout = torch.randn(BH, N, 128, generator=g).to(torch.bfloat16)
    mask = None
    masked = docs is not None
    if masked:
        mask = torch.from_numpy(OB.build_block_mask(docs))
    SA.configure_sage(smooth_k=True, qk_quant=qk, pv_quant="bf16", qk_granularity=gran)
    d = lambda t: t.to(cuda_device).unsqueeze(0)  # noqa: E731
    if masked:
        out, lse = SA.sage_attn_forward_masked_with_lse(d(q), d(k), d(v), mask.to(cuda_device), SM)
        dq, dk, dv = SA.sage_attn_backward_masked(d(q), d(k), d(v), out, lse, d(dout), mask.to(cuda_device), SM)
        qkr = "int8"
    else:
        out, lse = SA.sage_attn_forward_with_lse(d(q), d(k), d(v), SM)
        dq, dk, dv = SA.sage_attn_backward(d(q), d(k), d(v), out, lse, d(dout), SM)
        qkr = qk
    # the forward's LSE normalises the oracle's P at the same granularity: rows sum to 1
    ks = OA.smooth_k(k)
    rq, rk = (1, 1) if gran == "per_token" else (128, 64)
    qc, qd = OA.quant_rows(q, qkr, rq, SM * OA.LOG2E)
    kc, kd = OA.quant_rows(ks, qkr, rk)
    s = (qc.double() @ kc.double().transpose(1, 2)).float()
    s = (s * qd.repeat_interleave(rq, 1)[:, :N, None]) * kd.repeat_interleave(rk, 1)[:, None, :N]
    p = torch.exp2(s - lse.cpu().unsqueeze(-1))
    if masked:
        full = mask.bool().repeat_interleave(128, 0)[:N].repeat_interleave(64, 1)[:, :N]
        p = p * full
    assert torch.allclose(p.sum(-1), torch.ones(BH, N), atol=5e-3), p.sum(-1)
    rdq, rdk, rdv, _ = OA.attention_backward(q, k, v, out[0].cpu(), lse.cpu(), dout, sm_scale=SM, qk_quant=qkr,
                                             block_mask=mask, granularity=gran)
    for a, b in ((dq, rdq), (dk, rdk), (dv, rdv)):
        assert torch.isfinite(a.float()).all()
        assert cosine(a[0].cpu(), b) >= 0.999


@pytest.mark.parametrize("pv", ["bf16", "fp8"])
def test_sage_op_autograd_per_block(cuda_device, pv):
    """configure_sage(qk_granularity="per_block") through the autograd op: the
    gradients equal the oracle's backward at per-block granularity."""
    from futudiffu_b200 import sage_attention as SA

    BH, N = 2, 384
    q, k, v = qkv(BH, N, 55)
    w = torch.linspace(-1, 1, 128)
    SA.configure_sage(smooth_k=True, qk_quant="int8", pv_quant=pv, qk_granularity="per_block")
    qg, kg, vg = (t.to(cuda_device).unsqueeze(0).requires_grad_(True) for t in (q, k, v))
    out, lse = SA.sage_attn_op(qg, kg, vg, SM)
    (out.float() * w.to(cuda_device)).sum().backward()
    dout = (torch.ones(BH, N, 128) * w).to(torch.bfloat16)
    rdq, rdk, rdv, _ = OA.attention_backward(q, k, v, out[0].detach().cpu(), lse.detach().cpu(), dout,
                                             sm_scale=SM, qk_quant="int8", granularity="per_block")
    for a, b in ((qg.grad, rdq), (kg.grad, rdk), (vg.grad, rdv)):
        assert cosine(a[0].cpu(), b) >= 0.999


def test_sage_op_autograd(cuda_device):
    from futudiffu_b200 import sage_attention as SA

    SA.configure_sage(smooth_k=True, qk_quant="int8")
    q, k, v = (t.to(cuda_device).unsqueeze(0).requires_grad_(True) for t in qkv(2, 256, 3))
    out, _ = SA.sage_attn_op(q, k, v, SM)
    (out.float() * torch.linspace(-1, 1, 128, device=cuda_device)).sum().backward()
    qr, kr, vr = (t.detach().float().requires_grad_(True) for t in (q, k, v))
    ref = torch.nn.functional.scaled_dot_product_attention(qr, kr, vr)
    (ref * torch.linspace(-1, 1, 128, device=cuda_device)).sum().backward()
    # reference test threshold: backward vs SDPA cosine > 0.95 (test_sage_backward.py:91-93)
    for a, b in ((q.grad, qr.grad), (k.grad, kr.grad), (v.grad, vr.grad)):
        assert cosine(a, b) > 0.95


def test_attention_bnhd_output_layout(cuda_device):
    """The (B, N, H*128) output layout holds exactly the transposed (B, H, N, 128) result."""
    from futudiffu_b200.sage_attention import _attn_forward

    g = gen(91)
    B, H, N = 2, 3, 300
    q, k, v = (torch.randn(B, H, N, 128, generator=g).to(torch.bfloat16).to(cuda_device) for _ in range(3))
    for qk, pv, gran in (("int8", "fp8", "per_block"), ("int8", "bf16", "per_token"), ("fp8", "bf16", "per_token")):
        a, _ = _attn_forward(q, k, v, None, block_mask=None, qk_quant=qk, pv_quant=pv, granularity=gran,
                             want_lse=False)
        b, _ = _attn_forward(q, k, v, None, block_mask=None, qk_quant=qk, pv_quant=pv, granularity=gran,
                             want_lse=False, out_bnhd=True)
        assert b.shape == (B, N, H * 128)
        assert torch.equal(b.cpu(), a.transpose(1, 2).reshape(B, N, H * 128).cpu())


@pytest.mark.parametrize("masked", [False, True])
def test_attention_quantised_output(cuda_device, masked):
    """The quantised-output epilogue writes exactly fp8_act_quant of the bf16
    (B, N, H*128) output, split into two row regions or into a column window of
    wider rows."""
    from futudiffu_b200.block_mask import build_block_mask
    from futudiffu_b200.fp8_kernels import fp8_act_quant
    from futudiffu_b200.sage_attention import _attn_forward, attn_forward_quant_out

    g = gen(93)
    B, H, N = 2, 3, 300
    D = H * 128
    q, k, v = (torch.randn(B, H, N, 128, generator=g).to(torch.bfloat16).to(cuda_device) for _ in range(3))
    mask = build_block_mask([100, 200], device=cuda_device) if masked else None
    split = 77
    modes = [("int8", "fp8", "per_block"), ("int8", "bf16", "per_token"), ("fp8", "bf16", "per_token")]
    for qk, pv, gran in modes:
        o, _ = _attn_forward(q, k, v, None, block_mask=mask, qk_quant=qk, pv_quant=pv, granularity=gran,
                             want_lse=False, out_bnhd=True)
        r8, rs = fp8_act_quant(o)
        r8 = r8.view(torch.uint8)
        # two regions: rows n < split and n >= split of every sample
        regions = [(torch.empty(B, n, D, dtype=torch.float8_e4m3fn, device=cuda_device),
                    torch.empty(B, n, D // 128, dtype=torch.float32, device=cuda_device)) for n in (split, N - split)]
        attn_forward_quant_out(q, k, v, None, block_mask=mask, qk_quant=qk, pv_quant=pv, granularity=gran,
                               regions=regions, split=split)
        assert torch.equal(regions[0][0].view(torch.uint8), r8[:, :split])
        assert torch.equal(regions[1][0].view(torch.uint8), r8[:, split:])
        assert torch.equal(regions[0][1], rs[:, :split]) and torch.equal(regions[1][1], rs[:, split:])
        # one region: a column window of wider rows (the [attention | MLP] input of a fused linear)
        W = D + 256
        buf = torch.zeros(B, N, W, dtype=torch.uint8, device=cuda_device)
        sbuf = torch.zeros(B, N, W // 128, dtype=torch.float32, device=cuda_device)
        attn_forward_quant_out(q, k, v, None, block_mask=mask, qk_quant=qk, pv_quant=pv, granularity=gran,
                               regions=[(buf[..., :D], sbuf[..., :D // 128])])
        assert torch.equal(buf[..., :D], r8) and not buf[..., D:].any()
        assert torch.equal(sbuf[..., :D // 128], rs) and not sbuf[..., D // 128:].any()



def _torch_backward_fp32(qf, kf, vf, dof, lse, delta, qz, ks, sm, mask=None):
    """fp32 torch restatement on the GPU of the backward arithmetic, head by head:
    S from the quantised codes, p = exp2((S q_desc) k_desc - lse) (0 on masked
    128 x 64 tiles), dS = p (dO V^T - Delta), dV = bf16(p)^T dO, dK = bf16(dS sm)^T Q,
    dQ = sm bf16(dS) Ks, each gradient rounded to bf16 once."""
    BH, N, _ = qf.shape
    f32, bf16 = torch.float32, torch.bfloat16
    qd, kd = qz["q_desc"][:, :N], qz["k_desc"][:, :N]
    dq, dk, dv = (torch.empty_like(qf) for _ in range(3))
    for h in range(BH):
        s = qz["q_codes"][h].to(f32) @ qz["k_codes"][h].to(f32).t()
        p = torch.exp2((s * qd[h, :, None]) * kd[h, None, :] - lse[h, :, None])
        if mask is not None:
            m = mask[h if mask.shape[0] > 1 else 0].bool()
            p = torch.where(m.repeat_interleave(128, 0)[:N].repeat_interleave(64, 1)[:, :N], p, 0.0)
        dp = dof[h].float() @ vf[h].float().t()
        ds = p * (dp - delta[h, :, None])
        dv[h] = (p.to(bf16).float().t() @ dof[h].float()).to(bf16)
        dk[h] = ((ds * sm).to(bf16).float().t() @ qf[h].float()).to(bf16)
        dq[h] = ((ds.to(bf16).float() @ ks[h].float()) * sm).to(bf16)
    return dq, dk, dv


def _bwd_inputs(BH, N, seed, qk="int8", gran="per_token"):
    from futudiffu_b200 import _lib as L
    from futudiffu_b200 import sage_attention as SA

    dev = torch.device("cuda")
    q, k, v = (t.to(dev) for t in qkv(BH, N, seed))
    dof = torch.randn(BH, N, 128, generator=gen(seed + 1)).to(torch.bfloat16).to(dev)
    SA.configure_sage(smooth_k=True, qk_quant=qk, pv_quant="bf16", qk_granularity=gran)
    out, lse = SA.sage_attn_forward_with_lse(q.unsqueeze(0), k.unsqueeze(0), v.unsqueeze(0), SM)
    qz = SA.quantize_qkv(q, k, v, SM, smooth_k=True, qk_quant=qk, granularity=gran, pv_quant="bf16")
    qz["q_desc"], qz["k_desc"] = SA._per_token_descales(qz, N)
    delta = (dof.float() * out[0].float()).sum(-1)
    ks = (k - qz["k_mean"].to(torch.bfloat16).unsqueeze(1)).contiguous()
    return q, k, v, out, lse, dof, qz, delta, ks


@pytest.mark.parametrize("qk", ["int8", "fp8"])
def test_backward_config2_vs_torch_fp32(cuda_device, qk):
    """Benchmark config 2's shape (B 2, H 24, N 4096) against the fp32 torch
    restatement of the same quantised arithmetic on the GPU."""
    from futudiffu_b200 import sage_attention as SA

    BH, N = 48, 4096
    q, k, v, out, lse, dof, qz, delta, ks = _bwd_inputs(BH, N, 91, qk)
    dq, dk, dv = SA.sage_attn_backward(q.unsqueeze(0), k.unsqueeze(0), v.unsqueeze(0), out, lse,
                                       dof.unsqueeze(0), SM)
    rq, rk, rv = _torch_backward_fp32(q, k, v, dof, lse, delta, qz, ks, SM)
    for a, b in ((dq[0], rq), (dk[0], rk), (dv[0], rv)):
        assert torch.isfinite(a.float()).all()
        assert cosine(a.float().cpu(), b.float().cpu()) >= 0.9999
    from futudiffu_b200 import check_status

    check_status()


@pytest.mark.parametrize("masked", [False, True])
def test_backward_deterministic(cuda_device, masked):
    """No atomics in the backward: two runs give the same bits, and a 3-D (per
    head) mask with skipped steps matches the fp32 torch restatement."""
    from futudiffu_b200 import sage_attention as SA

    BH, N = 3, 704
    q, k, v, out, lse, dof, qz, delta, ks = _bwd_inputs(BH, N, 41)
    mask = None
    if masked:
        mask = torch.stack([torch.from_numpy(OB.build_block_mask(d)) for d in ([200, 504], [704], [64, 320, 320])])
        mask = mask.to(cuda_device)
        out, lse = SA.sage_attn_forward_masked_with_lse(q.unsqueeze(0), k.unsqueeze(0), v.unsqueeze(0), mask, SM)
        delta = (dof.float() * out[0].float()).sum(-1)
        run = lambda: SA.sage_attn_backward_masked(q.unsqueeze(0), k.unsqueeze(0), v.unsqueeze(0), out, lse,  # noqa: E731
                                                   dof.unsqueeze(0), mask, SM)
    else:
        run = lambda: SA.sage_attn_backward(q.unsqueeze(0), k.unsqueeze(0), v.unsqueeze(0), out, lse,  # noqa: E731
                                            dof.unsqueeze(0), SM)
    a, b = run(), run()
    for x, y in zip(a, b):
        assert torch.equal(x, y)
    ref = _torch_backward_fp32(q, k, v, dof, lse, delta, qz, ks, SM, mask)
    for x, r in zip(a, ref):
        assert torch.isfinite(x.float()).all()
        assert cosine(x[0].float().cpu(), r.float().cpu()) >= 0.9999
    from futudiffu_b200 import check_status

    check_status()
