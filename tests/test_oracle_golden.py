"""The CPU oracle checked against fixtures produced by the reference itself (CPU only)."""

from __future__ import annotations

import numpy as np
import torch

from oracle import attention as OA
from oracle import block_mask as OB
from oracle import fused as OF
from oracle import quant as OQ
from tests.helpers import bf16_ulp_diff, cosine, e4m3_bits, e4m3_step_diff


def test_smooth_k_matches_reference(golden_dir):
    d = torch.load(golden_dir / "smooth_k.pt")
    ks = OA.smooth_k(d["k"])
    assert torch.equal(ks.view(torch.int16), d["ks"].view(torch.int16))


def test_block_mask_matches_reference(golden_dir):
    d = torch.load(golden_dir / "block_mask.pt")
    for (seg, tl), ref in zip(d["cases"], d["masks"]):
        assert np.array_equal(OB.build_block_mask(seg, tl), ref.numpy())


def test_block_mask_module_matches_reference(golden_dir):
    from futudiffu_b200.block_mask import build_block_mask

    d = torch.load(golden_dir / "block_mask.pt")
    for (seg, tl), ref in zip(d["cases"], d["masks"]):
        assert torch.equal(build_block_mask(seg, tl, device="cpu"), ref)


def test_padding_tail_attends_image_zero(golden_dir):
    # reference quirk: tokens past the segments keep document id 0
    d = torch.load(golden_dir / "block_mask.pt")
    (seg, tl), ref = d["cases"][3], d["masks"][3]
    assert tl > sum(seg)
    tail_kv = (sum(seg) + 63) // 64
    assert ref[0, tail_kv:].all()


def test_dequant_matches_reference(golden_dir):
    d = torch.load(golden_dir / "dequant.pt")
    out = OQ.dequant_blockwise(d["codes"], d["scales"])
    assert torch.equal(out.view(torch.int16), d["out"].view(torch.int16))


def test_weight_quant_matches_reference(golden_dir):
    d = torch.load(golden_dir / "weight_quant.pt")
    q, s = OQ.weight_quant(d["w"])
    assert torch.equal(e4m3_bits(q), e4m3_bits(d["codes"]))
    assert torch.equal(s, d["scales"])
    assert (e4m3_bits(q)[0:128, 128:256] == 0).all()


def test_act_quant_scales_match_reference_kernel(golden_dir):
    d = torch.load(golden_dir / "act_quant_scales.pt")
    _, s = OQ.act_quant(d["x"])
    assert torch.equal(s, d["scales"])
    assert s[3, 1].item() == torch.tensor(1e-12, dtype=torch.float32).item()


def test_act_quant_codes_follow_weight_quant_formula(golden_dir):
    # The per-element formula of the 1x128 activation quantiser is the same as
    # the reference weight quantiser's; a 1x128 group equals a 128x128 tile
    # whose rows are copies of that group.
    d = torch.load(golden_dir / "weight_quant.pt")
    w = d["w"][:1, :128].float().expand(128, 128).contiguous()
    qw, _ = OQ.weight_quant(w)
    qa, _ = OQ.act_quant(d["w"][:1, :128])
    assert torch.equal(e4m3_bits(qa), e4m3_bits(qw)[:1])


def test_silu_gate_matches_reference_fallback(golden_dir):
    d = torch.load(golden_dir / "silu_gate.pt")
    q, s = OQ.silu_gate_quant(d["x"])
    assert torch.allclose(s, d["scales"], rtol=1e-6, atol=0)
    diff = e4m3_step_diff(q, d["codes"])
    assert diff.max().item() <= 1
    assert (diff == 0).float().mean().item() >= 0.999


def test_fused_norms_match_reference_fallback(golden_dir):
    d = torch.load(golden_dir / "fused_norms.pt")
    mod = OF.rms_norm_modulate(d["x"], d["w"], d["scale"])
    gr = OF.rms_norm_gate_residual(d["x"], d["w"], d["gate"], d["res"])
    # the fallback rounds the normalised value to bf16 before modulating; the
    # kernel formula rounds once at the end: at most a couple of bf16 ulps apart
    assert bf16_ulp_diff(mod, d["modulate"]).max().item() <= 2
    # the residual add cancels near zero: compare with an absolute floor there
    assert torch.allclose(gr.float(), d["gate_residual"].float(), rtol=2**-7, atol=2**-6)
    assert cosine(mod, d["modulate"]) > 0.99999
    assert cosine(gr, d["gate_residual"]) > 0.99999


def test_qkv_postprocess_matches_reference(golden_dir):
    d = torch.load(golden_dir / "fused_norms.pt")
    q, k, v = OF.qkv_postprocess(d["qkv"], d["qw"], d["kw"], d["freqs"], d["H"], d["hd"])
    assert torch.equal(v.view(torch.int16), d["v"].view(torch.int16))
    for a, b in ((q, d["q"]), (k, d["k"])):
        # reference test threshold: per-head min cosine > 0.999 (fused_kernels.py:954)
        for h in range(d["H"]):
            assert cosine(a[:, h], b[:, h]) > 0.999
        # the reference rounds to bf16 after the norm and again after RoPE
        assert torch.allclose(a.float(), b.float(), rtol=2**-6, atol=2**-6)


def test_int8_quant_truncates_toward_zero():
    x = torch.tensor([[[1.0, -1.0, 0.5, -0.5] + [0.0] * 124]]).to(torch.bfloat16)
    x[0, 0, 4] = 127.9 / 127.0  # near the top of the range
    codes, desc = OA.quant_rows(x, "int8")
    amax = x.float().abs().max()
    inv = 127.0 / amax
    expect = (x.float() * inv).to(torch.int8)
    assert torch.equal(codes, expect)
    assert codes[0, 0, 2].item() == int((0.5 * inv).item())  # truncation, not rounding


def test_oracle_attention_close_to_exact():
    g = torch.Generator().manual_seed(0)
    BH, N = 2, 256
    q = torch.randn(BH, N, 128, generator=g).to(torch.bfloat16)
    k = (torch.randn(BH, N, 128, generator=g) + 2 * torch.randn(128, generator=g)).to(torch.bfloat16)
    v = torch.randn(BH, N, 128, generator=g).to(torch.bfloat16)
    exact = OA.attention_exact(q, k, v)
    for qk in ("int8", "fp8"):
        for gran in ("per_token", "per_block"):
            out, lse = OA.attention_forward(q, k, v, qk_quant=qk, granularity=gran)
            assert cosine(out, exact) > (0.999 if qk == "int8" else 0.99)
            assert torch.isfinite(lse).all()
    out, _ = OA.attention_forward(q, k, v, qk_quant="int8", granularity="per_block", pv_quant="fp8_channel")
    assert cosine(out, exact) > 0.995


# ---------------------------------------------------------------- the reference's own Triton kernels
# tests/golden/ref_kernels.pt holds the reference's kernels run in the Triton CPU
# interpreter (round-to-nearest-even casts, exact f32 dot; make_golden.py).  The
# interpreter evaluates divides, exp2 and sqrt correctly rounded, the oracle's CPU
# default, so quantised codes and scales must agree bit for bit; fp32 sums may
# differ in order (the interpreter's matmul vs the oracle's float64 tile sums), so
# GEMM accumulators agree to 2 fp32 ulp and attention outputs in all but a few
# elements, each within a few bf16 ulp.

import pytest  # noqa: E402

from oracle import gemm as OG  # noqa: E402


@pytest.fixture(scope="module")
def ref_kernels(golden_dir):
    return torch.load(golden_dir / "ref_kernels.pt", weights_only=False)


def test_act_quant_matches_reference_kernel(ref_kernels):
    d = ref_kernels["act"]
    y, s = OQ.act_quant(d["x"])
    assert torch.equal(e4m3_bits(y), e4m3_bits(d["codes"]))
    assert torch.equal(s, d["scales"])


def test_gemm_matches_reference_kernel(ref_kernels):
    g = ref_kernels["gemm"]
    args = (g["a8"], g["a_s"], g["b8"], g["b_s"])
    for bias, key in ((None, "c"), (g["bias"], "c_bias")):
        acc = OG.gemm_blockwise(*args, bias=bias, out_dtype=torch.float32)
        want = g[f"{key}_f32"]
        tol = 2 * torch.finfo(torch.float32).eps * want.abs().amax()
        assert (acc - want).abs().max() <= tol
        out = OG.gemm_blockwise(*args, bias=bias, out_dtype=torch.bfloat16)
        assert torch.equal(out.view(torch.int16), g[f"{key}_bf16"].view(torch.int16))
    # rowwise, v1t (B as (K, N)) and v2 (bf16 A quantised per K slice in the kernel)
    bt, bst = g["b8"].t().contiguous(), g["b_s"].t().contiguous()
    a8, a_s = OQ.act_quant(g["xa"])
    for got, want in (
            (OG.gemm_blockwise(g["a8"], g["a_s"], g["b8"], g["b_row"], out_dtype=torch.float32, b_layout=2),
             g["c_rowwise_f32"]),
            (OG.gemm_blockwise(g["a8"], g["a_s"], bt, bst, out_dtype=torch.float32, b_layout=1), g["c_v1t_f32"]),
            (OG.gemm_blockwise(a8, a_s, bt, bst, out_dtype=torch.float32, b_layout=1), g["c_v2_f32"])):
        assert (got - want).abs().max() <= 2 * torch.finfo(torch.float32).eps * want.abs().amax()


def test_gemm_requant_epilogues_match_reference_kernels(ref_kernels):
    g = ref_kernels["gemm"]
    acc = OG.gemm_blockwise(g["a8"], g["a_s"], g["b8"], g["b_s"], out_dtype=torch.float32)
    y, s = OQ.act_quant(acc)
    c, cs = g["quant"]
    assert torch.equal(e4m3_bits(y), e4m3_bits(c))
    torch.testing.assert_close(s, cs, rtol=4e-7, atol=0)  # amax of an accumulator: one fp32 ulp
    y, s = OQ.gelu_requant(g["a8"], g["a_s"])
    c, cs = g["gelu"]
    assert torch.equal(e4m3_bits(y), e4m3_bits(c))
    torch.testing.assert_close(s, cs, rtol=4e-7, atol=0)
    d = ref_kernels["silu_gate"]
    y, s = OQ.silu_gate_quant(d["x"])
    assert torch.equal(e4m3_bits(y), e4m3_bits(d["out"][0]))
    assert torch.equal(s, d["out"][1])


def test_fused_prologues_match_reference_kernels(golden_dir, ref_kernels):
    fz = torch.load(golden_dir / "fused_norms.pt", weights_only=False)
    n = ref_kernels["norms"]
    y = OF.rms_norm_modulate(fz["x"], fz["w"], fz["scale"], 1e-5)
    assert torch.equal(y.view(torch.int16), n["modulate"].view(torch.int16))
    got = OF.qkv_postprocess(fz["qkv"], fz["qw"], fz["kw"], fz["freqs"], fz["H"], fz["hd"])
    for a, b in zip(got, n["qkv"]):
        assert torch.equal(a.view(torch.int16), b.view(torch.int16))


_ATTN_MODES = {  # fixture key -> (qk_quant, pv_quant, masked)
    "int8_bf16": ("int8", "bf16", False),
    "int8_bf16_masked": ("int8", "bf16", True),
    "int8_bf16_masked_lse": ("int8", "bf16", True),
    "fp8_bf16": ("fp8", "bf16", False),
    "fp8_bf16_masked": ("fp8", "bf16", True),
    "fp8_fp8tile": ("fp8", "fp8_tile", False),
}


def _close_bf16(got, want, max_frac=2e-3, max_abs=4e-3):
    differ = got.view(torch.int16) != want.view(torch.int16)
    assert differ.float().mean().item() <= max_frac
    assert (got.float() - want.float()).abs().max().item() <= max_abs


@pytest.mark.parametrize("mode", sorted(_ATTN_MODES))
def test_attention_forward_matches_reference_kernels(ref_kernels, mode):
    a = ref_kernels["attention"]
    qk, pv, masked = _ATTN_MODES[mode]
    f = lambda t: t.reshape(-1, t.shape[-2], 128)  # noqa: E731
    out, lse = OA.attention_forward(f(a["q"]), f(a["k"]), f(a["v"]), qk_quant=qk, granularity="per_token",
                                    pv_quant=pv, block_mask=a["mask"] if masked else None)
    ref_out, ref_lse = a["fwd"][mode]
    _close_bf16(out, f(ref_out))
    if ref_lse is not None:
        assert (lse - ref_lse).abs().max().item() <= 4e-6


@pytest.mark.parametrize("mode", ["int8", "fp8", "int8_masked"])
def test_attention_backward_matches_reference_kernels(ref_kernels, mode):
    a = ref_kernels["attention"]
    f = lambda t: t.reshape(-1, t.shape[-2], 128)  # noqa: E731
    qk = mode.split("_")[0]
    masked = mode.endswith("masked")
    o, lse = a["fwd"]["int8_bf16_masked_lse" if masked else f"{qk}_bf16"]
    got = OA.attention_backward(f(a["q"]), f(a["k"]), f(a["v"]), f(o), lse, f(a["dout"]), sm_scale=a["sm_scale"],
                                qk_quant=qk, block_mask=a["mask"] if masked else None)
    for g, w in zip(got[:3], a["bwd"][mode]):
        _close_bf16(g, f(w))


def test_multi_lora_delta_matches_reference(ref_kernels):
    """src_ii MultiLoRALinear.adapter_delta (per-image scales, token routing with
    padding sentinels, an empty slot) equals the oracle bit for bit."""
    from oracle import lora as OL

    lo = ref_kernels["lora"]
    x2 = lo["x"].reshape(-1, lo["x"].shape[-1])
    eff = OL.effective_scales(x2.shape[0], lo["scales"], lo["token_to_image"], lo["scalings"], lo["active"])
    d = OL.adapter_delta(x2, lo["A"], lo["B"], eff)
    assert torch.equal(d.view(torch.int16), lo["delta"].reshape(d.shape).view(torch.int16))


def test_multi_lora_kernel_restated(ref_kernels):
    """_multi_lora_kernel (lora_kernels.py:100-157): mid rounded to bf16 per adapter,
    s * (mid @ B^T) summed in fp32 over adapters, one bf16 rounding."""
    k = ref_kernels["lora"]["kernel"]
    x = ref_kernels["lora"]["x"]
    acc = torch.zeros(*x.shape[:-1], k["B_all"].shape[1])
    for i in range(k["A_all"].shape[0]):
        mid = (x.float() @ k["A_all"][i].float().t()).to(torch.bfloat16).float()
        acc += k["scale_all"][:, i].view(-1, 1, 1) * (mid @ k["B_all"][i].float().t())
    assert torch.equal(acc.to(torch.bfloat16).view(torch.int16), k["out"].view(torch.int16))
