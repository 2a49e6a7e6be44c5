"""FP8 checkpoint format (reference fp8.py:374-449, :564-599) against the
reference's own quantize_model output (tests/golden/checkpoint.pt)."""

from __future__ import annotations

import json
from pathlib import Path

import pytest
import torch
from torch import nn

G = torch.load(Path(__file__).parent / "golden" / "checkpoint.pt", weights_only=False)


def test_reference_checkpoint_layout():
    """What replace_linear_with_fp8 and FP8Linear read: e4m3 (N, K) weight,
    f32 (N/128, K/128) weight_scale, comfy_quant JSON bytes; the rest kept."""
    out = G["output"]
    for key, w in G["input"].items():
        q = out[key]
        if key.endswith(".weight") and w.dim() == 2 and w.shape[0] % 128 == 0 and w.shape[1] % 128 == 0 \
                and w.numel() >= 4096:
            assert q.dtype == torch.float8_e4m3fn and q.shape == w.shape
            s = out[key.replace(".weight", ".weight_scale")]
            assert s.dtype == torch.float32 and s.shape == (w.shape[0] // 128, w.shape[1] // 128)
            meta = json.loads(bytes(out[key.replace(".weight", ".comfy_quant")].tolist()))
            assert meta == {"format": "float8_e4m3fn_blockwise", "group_size": 128, "orig_dtype": str(w.dtype),
                            "orig_shape": list(w.shape)}
        else:
            assert torch.equal(q, w)


@pytest.mark.gpu
def test_quantize_model_matches_reference(cuda_device, tmp_path):
    from safetensors.torch import load_file, save_file

    from futudiffu_b200.fp8 import quantize_model

    src, dst = tmp_path / "in.safetensors", tmp_path / "out.safetensors"
    save_file(G["input"], str(src))
    stats = quantize_model(str(src), str(dst))
    assert stats == G["stats"]
    out = load_file(str(dst))
    assert set(out) == set(G["output"])
    for k, v in G["output"].items():
        mine = out[k]
        assert mine.dtype == v.dtype and mine.shape == v.shape, k
        if v.dtype == torch.float8_e4m3fn:
            assert torch.equal(mine.view(torch.uint8), v.view(torch.uint8)), k
        else:
            assert torch.equal(mine, v), k


@pytest.mark.gpu
def test_replace_linear_loads_reference_checkpoint(cuda_device):
    """The reference checkpoint loads into FP8Linear layers whose forward equals
    the bf16 product with the dequantised weight to FP8 accuracy."""
    from futudiffu_b200.fp8 import FP8Linear, dequantize_fp8_blockwise, replace_linear_with_fp8

    class Attn(nn.Module):
        def __init__(self):
            super().__init__()
            self.qkv = nn.Linear(128, 384, bias=False)
            self.out = nn.Linear(128, 128, bias=True)

    class Block(nn.Module):
        def __init__(self):
            super().__init__()
            self.attn = Attn()

    root = nn.Module()
    root.blocks = nn.ModuleList([Block()])
    sd = {k: v.to(cuda_device) for k, v in G["output"].items()}
    replace_linear_with_fp8(root, sd)
    qkv, out = root.blocks[0].attn.qkv, root.blocks[0].attn.out
    assert isinstance(qkv, FP8Linear) and isinstance(out, FP8Linear) and out.bias is not None
    x = torch.randn(40, 128, device=cuda_device).to(torch.bfloat16)
    y = qkv(x)
    w = dequantize_fp8_blockwise(sd["blocks.0.attn.qkv.weight"], sd["blocks.0.attn.qkv.weight_scale"])
    ref = x.float() @ w.float().t()
    cos = torch.nn.functional.cosine_similarity(y.float().flatten(), ref.flatten(), dim=0)
    assert cos > 0.999
