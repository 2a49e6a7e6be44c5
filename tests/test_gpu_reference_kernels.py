"""The CUDA path, called through the reference-named API, against the outputs of
the reference's own Triton kernels (tests/golden/ref_kernels.pt, made by
tests/golden/make_golden.py in the Triton CPU interpreter with round-to-nearest-
even casts and an exact f32 dot).

The interpreter divides, takes exp2 and square roots correctly rounded; the GPU
kernels here reproduce the compiled reference (div.full.f32, ex2.approx,
sqrt.approx), so a scale may move by up to 2 fp32 ulp and a code by one e4m3
step where it sits on a rounding edge.  Float results carry the tolerances
written beside each check.
"""

from __future__ import annotations

import pytest
import torch

from tests.helpers import bf16_ulp_diff, cosine, e4m3_step_diff

pytestmark = pytest.mark.gpu

SCALE_RTOL = 2.5e-7  # two fp32 ulp: div.full.f32 vs the correctly rounded quotient


@pytest.fixture(scope="module")
def R(golden_dir):
    return torch.load(golden_dir / "ref_kernels.pt", weights_only=False)


def _lse_close(got, want):
    # LSE in log2 units; FP8 Q/K codes move where a scale differs by an ulp
    # (div.full vs IEEE) or the bf16 smoothing mean by one ulp: 2e-3 relative
    assert (got.cpu() - want).abs().max().item() <= 2e-3 * max(1.0, want.abs().max().item())


def _codes_close(got, want, max_frac=0.01):
    d = e4m3_step_diff(got.cpu(), want)
    assert d.max().item() <= 1
    assert (d > 0).float().mean().item() <= max_frac


def test_fp8_act_quant(cuda_device, R):
    from futudiffu_b200.fp8_kernels import fp8_act_quant

    d = R["act"]
    y, s = fp8_act_quant(d["x"].to(cuda_device))
    torch.testing.assert_close(s.cpu(), d["scales"], rtol=SCALE_RTOL, atol=0)
    _codes_close(y, d["codes"])


def test_fp8_gemm_and_addmm(cuda_device, R):
    from futudiffu_b200.fp8_kernels import fp8_addmm_blockwise, fp8_gemm_blockwise

    g = R["gemm"]
    a8, a_s, b8, b_s, bias = (g[k].to(cuda_device) for k in ("a8", "a_s", "b8", "b_s", "bias"))
    for out_dtype, key in ((torch.bfloat16, "bf16"), (torch.float32, "f32")):
        c = fp8_gemm_blockwise(a8, a_s, b8, b_s, output_dtype=out_dtype).cpu()
        cb = fp8_addmm_blockwise(a8, a_s, b8, b_s, bias=bias, output_dtype=out_dtype).cpu()
        for got, want in ((c, g[f"c_{key}"]), (cb, g[f"c_bias_{key}"])):
            if key == "bf16":
                # tensor-core sums in another order: at most one bf16 ulp, rarely
                d = bf16_ulp_diff(got, want)
                assert d.max().item() <= 1 and (d > 0).float().mean().item() <= 0.01
            else:
                tol = 8 * torch.finfo(torch.float32).eps * want.abs().amax()
                assert (got - want).abs().max() <= tol


def test_fp8_gemm_rowwise_v1t_v2(cuda_device, R):
    from futudiffu_b200.fp8_kernels import fp8_gemm_rowwise, fp8_gemm_v1t, fp8_gemm_v2

    g = R["gemm"]
    a8, a_s, b8, b_s, b_row, xa = (g[k].to(cuda_device) for k in ("a8", "a_s", "b8", "b_s", "b_row", "xa"))
    bt, bst = b8.t().contiguous(), b_s.t().contiguous()
    f32 = torch.float32
    for got, want in ((fp8_gemm_rowwise(a8, a_s, b8, b_row, output_dtype=f32), g["c_rowwise_f32"]),
                      (fp8_gemm_v1t(a8, a_s, bt, bst, output_dtype=f32), g["c_v1t_f32"])):
        assert (got.cpu() - want).abs().max() <= 8 * torch.finfo(f32).eps * want.abs().amax()
    # v2 = the act quantiser (div.full scales, as the compiled reference) + the v1t
    # GEMM; the fixture quantised with correctly rounded divides, so rows where a
    # code sits on a rounding edge differ by one e4m3 step.  Rows whose codes equal
    # the correctly rounded quantiser's (scales within 2 ulp) agree to 16 fp32 eps.
    from futudiffu_b200.fp8_kernels import fp8_act_quant
    from oracle import quant as OQ

    got = fp8_gemm_v2(xa, bt, bst, output_dtype=f32)
    a8g, asg = fp8_act_quant(xa)
    assert torch.equal(got, fp8_gemm_v1t(a8g, asg, bt, bst, output_dtype=f32))
    a8r, asr = OQ.act_quant(g["xa"])
    torch.testing.assert_close(asg.cpu(), asr, rtol=SCALE_RTOL, atol=0)
    same = (a8g.cpu().view(torch.uint8) == a8r.view(torch.uint8)).all(1)
    assert same.float().mean().item() >= 0.5
    got, want = got.cpu(), g["c_v2_f32"]
    assert (got[same] - want[same]).abs().max() <= 16 * torch.finfo(f32).eps * want.abs().amax()
    assert cosine(got, want) >= 0.99999


def test_fp8_gemm_quant_gelu_and_silu_gate(cuda_device, R):
    from futudiffu_b200.fp8_kernels import fp8_gelu, fp8_gemm_quant, fp8_silu_gate_quant

    g = R["gemm"]
    a8, a_s, b8, b_s = (g[k].to(cuda_device) for k in ("a8", "a_s", "b8", "b_s"))
    for (y, s), (wy, ws) in ((fp8_gemm_quant(a8, a_s, b8, b_s), g["quant"]), (fp8_gelu(a8, a_s), g["gelu"])):
        torch.testing.assert_close(s.cpu(), ws, rtol=1e-6, atol=0)
        _codes_close(y, wy)
    d = R["silu_gate"]
    y, s = fp8_silu_gate_quant(d["x"].to(cuda_device))
    torch.testing.assert_close(s.cpu(), d["out"][1], rtol=1e-6, atol=0)
    _codes_close(y, d["out"][0])


def test_fused_norm_and_qkv_postprocess(cuda_device, golden_dir, R):
    from futudiffu_b200.fused_kernels import fused_qkv_postprocess, fused_rms_norm_modulate

    fz = torch.load(golden_dir / "fused_norms.pt", weights_only=False)
    n = R["norms"]
    y = fused_rms_norm_modulate(*(fz[k].to(cuda_device) for k in ("x", "w", "scale")))
    d = bf16_ulp_diff(y.cpu(), n["modulate"])  # rsqrt.approx vs a correctly rounded 1/sqrt
    assert d.max().item() <= 1 and (d > 0).float().mean().item() <= 0.01
    got = fused_qkv_postprocess(*(fz[k].to(cuda_device) for k in ("qkv", "qw", "kw", "freqs")), fz["H"], fz["hd"])
    for a, b in zip(got, n["qkv"]):
        d = bf16_ulp_diff(a.cpu(), b)
        assert d.max().item() <= 2 and (d > 0).float().mean().item() <= 0.01


@pytest.mark.parametrize("qk", ["int8", "fp8"])
def test_sage_forward_and_backward(cuda_device, R, qk):
    from futudiffu_b200 import sage_attention as SA

    a = R["attention"]
    q, k, v, do, mask = (a[x].to(cuda_device) for x in ("q", "k", "v", "dout", "mask"))
    SA.configure_sage(smooth_k=True, qk_quant=qk, pv_quant="bf16")
    try:
        o, lse = SA.sage_attn_forward_with_lse(q, k, v)
        ro, rlse = a["fwd"][f"{qk}_bf16"]
        # P rounded to bf16 from ex2.approx: reference tolerance of the INT8 / FP8 modes
        assert cosine(o.cpu(), ro) >= (0.9999 if qk == "int8" else 0.9995)
        _lse_close(lse, rlse)
        om = SA.sage_attn_forward_masked(q, k, v, mask)
        assert cosine(om.cpu(), a["fwd"][f"{qk}_bf16_masked"][0]) >= (0.9999 if qk == "int8" else 0.9995)
        dq, dk, dv = SA.sage_attn_backward(q, k, v, o, lse, do, a["sm_scale"])
        for x, w in zip((dq, dk, dv), a["bwd"][qk]):
            assert cosine(x.cpu(), w) >= 0.999
        if qk == "int8":
            o2, l2 = SA.sage_attn_forward_masked_with_lse(q, k, v, mask)
            ro2, rl2 = a["fwd"]["int8_bf16_masked_lse"]
            assert cosine(o2.cpu(), ro2) >= 0.9999
            _lse_close(l2, rl2)
            grads = SA.sage_attn_backward_masked(q, k, v, o2, l2, do, mask, a["sm_scale"])
            for x, w in zip(grads, a["bwd"]["int8_masked"]):
                assert cosine(x.cpu(), w) >= 0.999
    finally:
        SA.configure_sage()


def test_sage_forward_fp8_pv(cuda_device, R):
    """FP8 PV: the reference scales P per row and V per column over each 64-key
    tile; this build uses per-channel V and a static P scale (two valid
    roundings of ~3 % element noise), so the gate is a cosine."""
    from futudiffu_b200 import sage_attention as SA

    a = R["attention"]
    q, k, v = (a[x].to(cuda_device) for x in ("q", "k", "v"))
    SA.configure_sage(smooth_k=True, qk_quant="fp8", pv_quant="fp8")
    try:
        o, lse = SA.sage_attn_forward_with_lse(q, k, v)
    finally:
        SA.configure_sage()
    ro, rlse = a["fwd"]["fp8_fp8tile"]
    assert cosine(o.cpu(), ro) >= 0.998
    _lse_close(lse, rlse)


def _lora_close(got, want):
    # this build folds the per-token scale into the bf16 mid activations and sums
    # all adapters in one fp32 accumulator; the reference rounds per adapter
    assert cosine(got.cpu(), want) >= 0.9999
    assert (got.cpu().float() - want.float()).abs().max().item() <= 0.02 * want.float().abs().max().item()


def test_multi_lora(cuda_device, R):
    from futudiffu_b200.lora_kernels import multi_lora_forward
    from futudiffu_b200.multi_lora import MultiLoRALinear

    lo = R["lora"]
    OUT, IN = lo["base_w"].shape
    base = torch.nn.Linear(IN, OUT, bias=True, device=cuda_device, dtype=torch.bfloat16)
    with torch.no_grad():
        base.weight.copy_(lo["base_w"])
        base.bias.copy_(lo["base_b"])
    m = MultiLoRALinear(base, max_adapters=len(lo["A"]), max_rank=lo["A"][0].shape[0])
    for j in range(len(lo["A"])):
        if lo["active"][j] > 0:
            m.assign_adapter(j, f"s{j}", rank=lo["A"][0].shape[0], alpha=1.0, init_a="zeros")
            with torch.no_grad():
                m.lora_A[j].copy_(lo["A"][j])
                m.lora_B[j].copy_(lo["B"][j])
    m._lora_scalings.copy_(lo["scalings"])
    x, sc, t2i = lo["x"].to(cuda_device), lo["scales"].to(cuda_device), lo["token_to_image"].to(cuda_device)
    _lora_close(m.adapter_delta(x, sc, t2i), lo["delta"])
    _lora_close(m(x, sc, t2i), lo["out"])
    k = lo["kernel"]
    got = multi_lora_forward(x, k["A_all"].to(cuda_device), k["B_all"].to(cuda_device), k["scale_all"].to(cuda_device))
    _lora_close(got, k["out"])
