"""Host-side API behaviour that needs no GPU: config validation, error types,
no-CPU-fallback guarantee, fake-tensor shapes of the custom ops (CPU only)."""

from __future__ import annotations

from pathlib import Path

import pytest
import torch


def test_configure_sage_validation():
    from futudiffu_b200 import sage_attention as SA

    with pytest.raises(ValueError):
        SA.configure_sage(qk_quant="int4")
    with pytest.raises(ValueError):
        SA.configure_sage(pv_quant="fp16")
    with pytest.raises(ValueError):
        SA.configure_sage(qk_granularity="per_head")
    SA.configure_sage(smooth_k=False, qk_quant="int8", pv_quant="fp8", qk_granularity="per_block")
    assert SA.get_sage_config() == {"smooth_k": False, "qk_quant": "int8", "pv_quant": "fp8",
                                    "qk_granularity": "per_block"}
    SA.configure_sage()
    assert SA.get_sage_config()["qk_quant"] == "fp8"


def test_set_attention_backend_validation():
    from futudiffu_b200 import attention as A

    with pytest.raises(ValueError):
        A.set_attention_backend("flash")
    A.set_attention_backend("auto")
    assert A.get_attention_backend() == "auto"
    A.set_attention_backend("sdpa")


def test_no_cpu_fallback():
    from futudiffu_b200.fp8_kernels import fp8_act_quant, fp8_gemm_blockwise
    from futudiffu_b200.fused_kernels import fused_rms_norm_modulate
    from futudiffu_b200.sage_attention import sage_attn_forward

    x = torch.zeros(4, 256, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError):
        fp8_act_quant(x)
    a8 = torch.zeros(4, 256, dtype=torch.float8_e4m3fn)
    with pytest.raises(RuntimeError):
        fp8_gemm_blockwise(a8, torch.ones(4, 2), torch.zeros(128, 256, dtype=torch.float8_e4m3fn), torch.ones(1, 2))
    with pytest.raises(RuntimeError):
        fused_rms_norm_modulate(torch.zeros(1, 2, 128, dtype=torch.bfloat16), torch.ones(128), torch.zeros(1, 128))
    q = torch.zeros(1, 1, 128, 128, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError):
        sage_attn_forward(q, q, q)


def test_sage_asserts_match_reference():
    from futudiffu_b200.sage_attention import sage_attn_forward

    with pytest.raises(AssertionError):
        sage_attn_forward(*(torch.zeros(1, 1, 16, 64, dtype=torch.bfloat16),) * 3)
    with pytest.raises(AssertionError):
        sage_attn_forward(*(torch.zeros(1, 1, 16, 128, dtype=torch.float16),) * 3)


def test_fake_tensor_shapes():
    from torch._subclasses.fake_tensor import FakeTensorMode

    import futudiffu_b200.fp8  # noqa: F401  (registers futudiffu::fp8_linear*)
    import futudiffu_b200.fused_kernels  # noqa: F401
    import futudiffu_b200.sage_attention  # noqa: F401

    with FakeTensorMode():
        q = torch.empty(2, 3, 256, 128, dtype=torch.bfloat16)
        out, lse = torch.ops.futudiffu.sage_attn(q, q, q, 0.1)
        assert out.shape == (2, 3, 256, 128) and lse.shape == (6, 256) and out.is_contiguous()
        m = torch.empty(2, 4, dtype=torch.uint8)
        out, lse = torch.ops.futudiffu.sage_attn_masked(q, q, q, m, 0.1)
        assert out.shape == (2, 3, 256, 128)
        x = torch.empty(2, 7, 512, dtype=torch.bfloat16)
        w = torch.empty(1024, 512, dtype=torch.float8_e4m3fn)
        ws = torch.empty(8, 4)
        y = torch.ops.futudiffu.fp8_linear(x, w, ws, 128, 0)
        assert y.shape == (2, 7, 1024) and y.dtype == torch.bfloat16
        y = torch.ops.futudiffu.fp8_linear_bias(x, w, ws, torch.empty(1024), 128, 2)
        assert y.dtype == torch.float32
        g, s = torch.ops.futudiffu.fp8_silu_gate_quant(torch.empty(5, 512, dtype=torch.bfloat16), 128, 3)
        assert g.shape == (5, 256) and s.shape == (5, 2)
        qkv = torch.empty(2, 9, 3 * 4 * 128, dtype=torch.bfloat16)
        oq, ok, ov = torch.ops.futudiffu.fused_qkv_postprocess(qkv, torch.empty(128), torch.empty(128),
                                                              torch.empty(2, 9, 1, 64, 2, 2), 4, 128, 1e-5)
        assert oq.shape == (2, 4, 9, 128)


def test_block_mask_on_cpu_device():
    from futudiffu_b200.block_mask import build_block_mask

    m = build_block_mask([128, 128], device="cpu")
    assert m.shape == (2, 4) and m.dtype == torch.uint8
    assert m.tolist() == [[1, 1, 0, 0], [0, 0, 1, 1]]


def test_fp8_linear_replacement_logic():
    import torch.nn as nn

    from futudiffu_b200.fp8 import FP8Linear, replace_linear_with_fp8

    model = nn.Sequential(nn.Linear(256, 128), nn.Sequential(nn.Linear(128, 256)))
    sd = {"0.weight": torch.zeros(128, 256, dtype=torch.float8_e4m3fn), "0.weight_scale": torch.ones(1, 2),
          "1.0.weight": torch.zeros(256, 128)}
    replace_linear_with_fp8(model, sd)
    assert isinstance(model[0], FP8Linear) and isinstance(model[1][0], nn.Linear)
    assert model[0].in_features == 256 and model[0].out_features == 128


def test_dit_config_arithmetic():
    """Config-4 shapes and FLOP accounting (no GPU needed)."""
    from futudiffu_b200.dit import DiTConfig, batch_freqs, flops_per_sample_step, image_freqs, sigmas, text_freqs

    cfg = DiTConfig()
    assert cfg.tokens == 4608 and cfg.img_tokens == 4096 and cfg.hidden == 24 * 128
    assert abs(flops_per_sample_step(cfg) / 1e12 - 74.36) < 0.05
    s = sigmas(28)
    assert len(s) == 29 and s[0] == 1.0 and s[-1] == 0.0
    small = DiTConfig(hidden=256, heads=2, txt_tokens=4, img_grid=(2, 3))
    fi = image_freqs(small, "cpu")
    assert fi.shape == (6, 64, 2, 2)
    assert torch.allclose(fi[0], torch.eye(2).expand(64, 2, 2))  # position (0, 0): identity
    ft = text_freqs(small, "cpu")
    assert torch.equal(ft, torch.eye(2).expand(4, 64, 2, 2))
    assert batch_freqs(fi, 3).shape == (3, 6, 64, 2, 2)


def test_multi_lora_slot_api():
    """Slot bookkeeping of MultiLoRALinear (no GPU work)."""
    from futudiffu_b200.multi_lora import MultiLoRALinear

    base = torch.nn.Linear(256, 128, bias=False)
    lin = MultiLoRALinear(base, max_adapters=2, max_rank=8, device="cpu")
    lin.assign_adapter(0, "a", rank=4, alpha=8.0)
    assert float(lin._lora_scalings[0]) == 2.0 and float(lin._slot_active[0]) == 1.0
    assert torch.count_nonzero(lin.lora_A[0][4:]) == 0 and torch.count_nonzero(lin.lora_A[0][:4]) > 0
    with pytest.raises(ValueError):
        lin.assign_adapter(1, "a", rank=4, alpha=1.0)
    with pytest.raises(ValueError):
        lin.assign_adapter(1, "b", rank=16, alpha=1.0)
    with pytest.raises(IndexError):
        lin.assign_adapter(2, "b", rank=4, alpha=1.0)
    lin.release_adapter(0)
    assert lin._slot_names == [None, None] and float(lin._lora_scalings[0]) == 0.0
    assert lin.in_features == 256 and lin.out_features_val == 128
    eff = lin._effective_scales(5, torch.tensor([[1.0, 2.0], [3.0, 4.0]]), torch.tensor([0, 1, -1, 1, 0]))
    assert eff.shape == (5, 2)


def test_lora_operand_padding():
    from futudiffu_b200.lora_kernels import lora_operands

    h, b, kp = lora_operands(torch.ones(3, 40), torch.ones(5, 40))
    assert kp == 64 and h.shape == (3, 64) and b.shape == (5, 64)
    assert h[:, 40:].abs().sum() == 0


def test_rope_embed_equals_reference_fixture():
    """rope_embed reproduces the reference's own rotations bit for bit
    (tests/golden/fused_norms.pt: reference attention.rope_embed on Z-Image axes)."""
    from futudiffu_b200.attention import rope_embed

    d = torch.load(Path(__file__).parent / "golden" / "fused_norms.pt", weights_only=False)
    B, S, hd = d["x"].shape[0], d["x"].shape[1], d["hd"]
    pos = torch.zeros(S, 3)
    pos[:, 0] = 1.0
    pos[:, 1] = (torch.arange(S) % 7).float()
    pos[:, 2] = (torch.arange(S) // 7).float()
    freqs = torch.cat([rope_embed(pos[None, :, i], dd, 256.0) for i, dd in enumerate((32, 48, 48))], dim=-3)
    freqs = freqs.expand(B, S, hd // 2, 2, 2).unsqueeze(2).contiguous()
    assert torch.equal(freqs, d["freqs"])
