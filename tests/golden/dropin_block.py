"""The drop-in check on the reference's own model code: src_ii.transformer's
JointTransformerBlock (src_ii/transformer.py:588-717), unmodified, run once on
the reference's kernels and once with this library's modules installed under
the reference's module names (the sys.modules swap of INTEGRATION.md).

Both runs use the same seeded Z-Image-class layer (dim 3840, 30 heads, FFN
10240, FP8 block-quantised linears loaded through the reference's
replace_linear_with_fp8 and fused by its fuse_w1w3 / enable_fused_chain, Q/K
RMSNorm, per-sample adaLN), the same packed input of two documents with the
uint8 block mask, and INT8 QK + bf16 PV attention (configure_sage, the
reference's production setting).  Each run is a fresh interpreter, so the two
module sets never mix.

Usage (on a GPU machine):
  python tests/golden/dropin_block.py --reference <reference path> [--record out.json]
"""

from __future__ import annotations

import argparse
import json
import math
import os
import subprocess
import sys
import tempfile
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent

DIM, HEADS, FFN_MULT, N = 3840, 30, 8.0 / 3.0, 1536
SWAP = {
    "futudiffu.sage_attention": "futudiffu_b200.sage_attention",
    "futudiffu.fp8_kernels": "futudiffu_b200.fp8_kernels",
    "futudiffu.fp8": "futudiffu_b200.fp8",
    "futudiffu.fused_kernels": "futudiffu_b200.fused_kernels",
    "futudiffu.attention": "futudiffu_b200.attention",
    "src_ii.attention_srcii": "futudiffu_b200.attention_srcii",
    "src_ii.block_mask": "futudiffu_b200.block_mask",
    "futudiffu.lora_kernels": "futudiffu_b200.lora_kernels",
    "src_ii.multi_lora": "futudiffu_b200.multi_lora",
}


def make_inputs(path: Path) -> None:
    """Seeded layer weights (FP8 linears quantised 128 x 128 as the reference's
    checkpoints are), the packed input, RoPE rotations, mask and adaLN input."""
    sys.path.insert(0, str(ROOT))
    from oracle.quant import weight_quant
    from futudiffu_b200.block_mask import build_block_mask

    g = torch.Generator().manual_seed(2024)
    hidden = 256 * ((int(FFN_MULT * DIM) + 255) // 256)
    sd = {}
    for name, (n, k) in {"attention.qkv": (3 * DIM, DIM), "attention.out": (DIM, DIM),
                         "feed_forward.w1": (hidden, DIM), "feed_forward.w2": (DIM, hidden),
                         "feed_forward.w3": (hidden, DIM)}.items():
        w8, ws = weight_quant(torch.randn(n, k, generator=g) * 0.02)
        sd[f"{name}.weight"], sd[f"{name}.weight_scale"] = w8, ws
    for name in ("attention_norm1", "ffn_norm1", "attention_norm2", "ffn_norm2"):
        sd[f"{name}.weight"] = (1 + 0.05 * torch.randn(DIM, generator=g)).to(torch.bfloat16)
    for name in ("attention.q_norm", "attention.k_norm"):
        sd[f"{name}.weight"] = (1 + 0.05 * torch.randn(DIM // HEADS, generator=g)).to(torch.bfloat16)
    sd["adaLN_modulation.0.weight"] = (torch.randn(4 * DIM, 256, generator=g) * 0.02).to(torch.bfloat16)
    sd["adaLN_modulation.0.bias"] = (torch.randn(4 * DIM, generator=g) * 0.02).to(torch.bfloat16)
    ang = torch.rand(1, N, 64, generator=g) * 6.283185307179586
    c, s = torch.cos(ang), torch.sin(ang)
    freqs = torch.stack([torch.stack([c, -s], -1), torch.stack([s, c], -1)], -2).unsqueeze(2).contiguous()
    torch.save({"sd": sd, "x": torch.randn(1, N, DIM, generator=g).to(torch.bfloat16), "freqs": freqs,
                "mask": build_block_mask([896, 576], total_len=N, device="cpu"),
                "adaln": torch.randn(1, 256, generator=g).to(torch.bfloat16)}, path)


def run_block(ref: Path, inputs: Path, out: Path, swapped: bool) -> None:
    """One forward of the reference's JointTransformerBlock (in a fresh interpreter)."""
    sys.path.insert(0, str(ROOT))
    for p in (ref / "src", ref):
        if p.exists():
            sys.path.insert(0, str(p))
    if swapped:
        import importlib

        for ref_name, mod in SWAP.items():
            sys.modules[ref_name] = importlib.import_module(mod)
    from futudiffu.fp8 import replace_linear_with_fp8
    from futudiffu.sage_attention import configure_sage
    from src_ii.transformer import JointTransformerBlock

    d = torch.load(inputs, weights_only=False)
    dev = torch.device("cuda:0")
    torch.manual_seed(0)
    blk = JointTransformerBlock(0, DIM, HEADS, HEADS, 256, FFN_MULT, 1e-5, True, modulation=True,
                                z_image_modulation=True, use_sage=True, device=dev, dtype=torch.bfloat16)
    sd = {k: v.to(dev) for k, v in d["sd"].items()}
    replace_linear_with_fp8(blk, sd)
    blk.load_state_dict({k: v for k, v in sd.items() if not k.endswith("weight_scale")
                         and not k.startswith(("attention.qkv", "attention.out", "feed_forward"))}, strict=False)
    blk.feed_forward.fuse_w1w3()
    blk.feed_forward.enable_fused_chain()
    configure_sage(smooth_k=True, qk_quant="int8", pv_quant="bf16")
    with torch.no_grad():
        y = blk(d["x"].to(dev), None, d["freqs"].to(dev), adaln_input=d["adaln"].to(dev),
                block_mask=d["mask"].to(dev))
    torch.cuda.synchronize()
    kern = sys.modules["futudiffu.fp8_kernels"].__name__
    torch.save({"y": y.cpu(), "kernels_module": kern}, out)


def compare(ref: Path) -> dict:
    with tempfile.TemporaryDirectory() as td:
        inputs = Path(td) / "in.pt"
        make_inputs(inputs)
        outs = {}
        for mode in ("reference", "swapped"):
            o = Path(td) / f"{mode}.pt"
            subprocess.run([sys.executable, __file__, "--reference", str(ref), "--child", mode, "--inputs",
                            str(inputs), "--out", str(o)], check=True)
            outs[mode] = torch.load(o, weights_only=False)
    a, b = outs["reference"]["y"].float(), outs["swapped"]["y"].float()
    cos = float((a.flatten().double() @ b.flatten().double()) / (a.norm() * b.norm()).double())
    err = (a - b).abs().max().item()
    return {"block": "src_ii.transformer.JointTransformerBlock (unmodified reference code)",
            "shape": {"dim": DIM, "heads": HEADS, "ffn": 256 * ((int(FFN_MULT * DIM) + 255) // 256), "tokens": N,
                      "documents": [896, 576]},
            "attention": "configure_sage(smooth_k=True, qk_quant='int8', pv_quant='bf16')",
            "kernels": {m: outs[m]["kernels_module"] for m in outs},
            "finite": bool(torch.isfinite(b).all()), "cosine": cos, "max_abs_err": err,
            "max_abs_ref": a.abs().max().item(), "device": torch.cuda.get_device_name(0)}


if __name__ == "__main__":
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--reference", required=True, type=Path)
    ap.add_argument("--record", type=Path, default=None)
    ap.add_argument("--child", choices=["reference", "swapped"], default=None)
    ap.add_argument("--inputs", type=Path, default=None)
    ap.add_argument("--out", type=Path, default=None)
    a = ap.parse_args()
    if a.child:
        run_block(a.reference, a.inputs, a.out, a.child == "swapped")
    else:
        rec = compare(a.reference)
        print(json.dumps(rec, indent=1))
        if a.record:
            a.record.write_text(json.dumps(rec, indent=1) + "\n")
