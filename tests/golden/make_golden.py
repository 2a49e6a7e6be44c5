"""Generate the golden fixtures in this directory from the reference itself.

Runs the reference project's (sqcu/futudiffu) own CPU-runnable code on seeded
inputs and stores inputs and outputs as ``.pt`` files:

  smooth_k.pt          futudiffu.sage_attention._smooth_k           (sage_attention.py:63-71)
  block_mask.pt        src_ii.block_mask.build_block_mask            (block_mask.py:35-99)
  dequant.pt           futudiffu.fp8.dequantize_fp8_blockwise        (fp8.py:452-480)
  weight_quant.pt      futudiffu.fp8.quantize_fp8_blockwise          (fp8.py:337-371),
                       its CUDA transfer replaced by an identity so it runs on the CPU
  act_quant_scales.pt  futudiffu.fp8_kernels.fp8_act_quant (Triton kernel under the
                       Triton CPU interpreter; only the scales are kept -- the
                       interpreter's fp8 cast is not round-to-nearest-even)
  ref_kernels.pt       the reference's Triton kernels (act quant, blockwise GEMM / addmm,
                       rowwise / v1t / v2 GEMMs, GEMM + requant, GELU requant, SiLU-gate
                       quant, RMSNorm+modulate, QKV postprocess, attention forward and
                       backward in every QK / PV mode, masked and not, multi-LoRA) in
                       the Triton CPU interpreter, with its float downcasts made
                       round-to-nearest-even and its dot made an exact f32 dot (see
                       _install_interpreter_fixes); and src_ii.multi_lora
                       MultiLoRALinear (torch) on an nn.Linear base
  silu_gate.pt         fp8_silu_gate_quant torch fallback            (fp8_kernels.py:1725-1747)
  fused_norms.pt       fused_kernels torch fallbacks + _qkv_postprocess_reference
                       (fused_kernels.py:479-541, :802-842) and attention.rope_embed
  checkpoint.pt        futudiffu.fp8.quantize_model on a small safetensors state dict
                       (device transfer made an identity): every output tensor
  packing.pt           src_ii.bin_packer (BinPackScheduler on seeded item lists and
                       plans, estimate_efficiency, the length constants),
                       src_ii.transformer.build_packed_sequence / build_packed_rope
                       / EmbedND, src_ii.forward_packed._pad_plan_to_fixed_len and
                       the Euler update of src_ii.triumphant_future_reduction_ops

Usage:  python tests/golden/make_golden.py --reference <path to the reference checkout>

The reference is needed only to regenerate; tests read the stored files.
Sections that need Triton blocked run in a child process of this script.
"""

from __future__ import annotations

import argparse
import importlib.abc
import os
import subprocess
import sys
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent


class _BlockTriton(importlib.abc.MetaPathFinder):
    def find_spec(self, name, path, target=None):
        if name == "triton" or name.startswith("triton."):
            raise ImportError("triton blocked for fallback capture")
        return None


def _gen(seed: int) -> torch.Generator:
    return torch.Generator().manual_seed(seed)


def main_triton(ref: Path) -> None:
    sys.path.insert(0, str(ref / "src"))
    sys.path.insert(0, str(ref))
    from futudiffu.sage_attention import _smooth_k
    from futudiffu import fp8 as rfp8
    from src_ii.block_mask import build_block_mask

    # ---- smooth_k: bf16 K with a per-channel offset (std 2) over (B, H, N, D)
    g = _gen(0)
    k = torch.randn(2, 3, 200, 128, generator=g, dtype=torch.float32)
    k = (k + 2.0 * torch.randn(128, generator=g)).to(torch.bfloat16)
    torch.save({"k": k, "ks": _smooth_k(k)}, HERE / "smooth_k.pt")

    # ---- block masks, including a padding tail that keeps document id 0
    cases = [([128, 256, 64], None), ([100, 160, 40], None), ([4288], None), ([1000, 2000], 3100),
             ([2144, 2144], 4288), ([96, 32, 200, 72], None)]
    masks = [build_block_mask(seg, total_len=tl, device="cpu") for seg, tl in cases]
    torch.save({"cases": cases, "masks": masks}, HERE / "block_mask.pt")

    # ---- dequantize_fp8_blockwise on random codes / scales
    g = _gen(1)
    codes = (torch.randn(256, 384, generator=g) * 100).clamp(-448, 448).to(torch.float8_e4m3fn)
    scales = torch.rand(2, 3, generator=g) * 0.01 + 1e-4
    torch.save({"codes": codes, "scales": scales,
                "out": rfp8.dequantize_fp8_blockwise(codes, scales)}, HERE / "dequant.pt")

    # ---- quantize_fp8_blockwise with the device transfer made an identity
    g = _gen(2)
    w = (torch.randn(256, 384, generator=g) * 0.02).to(torch.bfloat16)
    w[0:128, 128:256] = 0.0  # an all-zero tile exercises the 1e-12 clamp
    saved = torch.Tensor.cuda
    torch.Tensor.cuda = lambda self, *a, **kw: self  # type: ignore[assignment]
    try:
        q, s = rfp8.quantize_fp8_blockwise(w)
    finally:
        torch.Tensor.cuda = saved  # type: ignore[assignment]
    torch.save({"w": w, "codes": q, "scales": s}, HERE / "weight_quant.pt")

    main_packing(ref)
    main_checkpoint(ref)

    # ---- fp8_act_quant Triton kernel in the CPU interpreter: scales only
    env = dict(os.environ, TRITON_INTERPRET="1")
    subprocess.run([sys.executable, __file__, "--reference", str(ref), "--section", "interp"],
                   check=True, env=env)
    # ---- the reference's kernels in the interpreter with RNE casts and an exact dot
    subprocess.run([sys.executable, __file__, "--reference", str(ref), "--section", "kernels"],
                   check=True, env=env)
    # ---- torch fallbacks (Triton blocked)
    subprocess.run([sys.executable, __file__, "--reference", str(ref), "--section", "fallback"],
                   check=True)


def main_checkpoint(ref: Path) -> None:
    import tempfile

    from safetensors.torch import load_file, save_file

    from futudiffu import fp8 as rfp8

    g = _gen(8)
    sd = {
        "blocks.0.attn.qkv.weight": (torch.randn(384, 128, generator=g) * 0.02).to(torch.bfloat16),
        "blocks.0.attn.out.weight": (torch.randn(128, 128, generator=g) * 0.02).to(torch.float16),
        "blocks.0.attn.out.bias": torch.randn(128, generator=g).to(torch.bfloat16),
        "blocks.0.mlp.w2.weight": torch.randn(128, 256, generator=g) * 0.05,
        "blocks.0.odd.weight": (torch.randn(200, 128, generator=g) * 0.02).to(torch.bfloat16),
        "blocks.0.small.weight": (torch.randn(16, 128, generator=g)).to(torch.bfloat16),
        "blocks.0.steps": torch.arange(7, dtype=torch.int64),
    }
    saved = torch.Tensor.cuda
    torch.Tensor.cuda = lambda self, *a, **kw: self  # type: ignore[assignment]
    try:
        with tempfile.TemporaryDirectory() as d:
            src, dst = f"{d}/in.safetensors", f"{d}/out.safetensors"
            save_file(sd, src)
            stats = rfp8.quantize_model(src, dst)
            out = load_file(dst)
    finally:
        torch.Tensor.cuda = saved  # type: ignore[assignment]
    torch.save({"input": sd, "output": dict(out), "stats": stats}, HERE / "checkpoint.pt")


def main_packing(ref: Path) -> None:
    import random

    from src_ii import bin_packer as rbp
    from src_ii import forward_packed as rfp
    from src_ii import transformer as rt
    from src_ii import triumphant_future_reduction_ops as rops

    rng = random.Random(7)
    item_lists = []
    for n in (1, 5, 17, 40):
        item_lists.append([{"id": i, "seq_len": rng.choice([96, 640, 1088, 2144, 4288, 5000, rng.randint(32, 4288)])}
                           for i in range(n)])
    sched = rbp.BinPackScheduler()
    packs = [[[it["id"] for it in b] for b in sched.pack(items)] for items in item_lists]
    effs = [sched.estimate_efficiency(sched.pack(items)) for items in item_lists]
    sizes = [(1280, 832), (832, 1280), (1024, 1024), (512, 512), (640, 384), (256, 256), (320, 192), (448, 576)]
    plan = [{"id": i, "width": w, "height": h, **({"cap_tokens": rng.randint(20, 200)} if i % 3 else {})}
            for i, (w, h) in enumerate(rng.choice(sizes) for _ in range(23))]
    plan_bins = [[(it["id"], it["seq_len"], it["img_seq_len"], it["cap_tokens"]) for it in b]
                 for b in rbp.BinPackScheduler(max_seq_len=6000).pack_generation_plan(plan)]
    training_items = [(i, f"s{i}", w, h) for i, (w, h) in enumerate(rng.choice(sizes) for _ in range(11))]
    training = rbp.BinPackScheduler().pack_for_training(training_items)

    g = _gen(6)
    caps = [torch.randn(1, n, 16, generator=g) for n in (40, 113, 7)]
    grids = [(12, 16), (8, 8), (4, 6)]
    imgs = [torch.randn(1, h * w, 16, generator=g) for h, w in grids]
    cap_pad, x_pad = torch.randn(16, generator=g), torch.randn(16, generator=g)
    packed, info = rt.build_packed_sequence(caps, imgs, grids, [40, 113, 7], 32, cap_pad, x_pad)
    rope = rt.build_packed_rope(info, rt.EmbedND(128, 256.0, [32, 48, 48]), 32, torch.device("cpu"))
    seg_doc = info.document_id.clone()
    info_p, rope_p = rfp._pad_plan_to_fixed_len(info, rope, 768)

    x = torch.randn(2, 16, 8, 8, generator=g)
    guided = torch.randn(2, 16, 8, 8, generator=g)
    euler = rops.euler_step(x, guided, torch.tensor(0.7), torch.tensor(0.55))
    denoised = rops.denoise_all([x, guided], [guided, x], [torch.tensor(0.3), torch.tensor(0.9)])

    torch.save({
        "constants": (rbp.REFERENCE_SEQ_LEN, rbp.DEFAULT_CAP_TOKENS, rbp.REFERENCE_TOTAL_LEN),
        "item_lists": item_lists, "packs": packs, "effs": effs,
        "plan": plan, "plan_bins": plan_bins, "training_items": training_items, "training": training,
        "caps": caps, "imgs": imgs, "grids": grids, "cap_pad": cap_pad, "x_pad": x_pad,
        "packed": packed, "segments": info.segments, "document_id": seg_doc, "rope": rope,
        "doc_padded": info_p.document_id, "rope_padded_shape": tuple(rope_p.shape),
        "x": x, "guided": guided, "euler": euler, "denoised": denoised,
    }, HERE / "packing.pt")


def main_interp(ref: Path) -> None:
    sys.path.insert(0, str(ref / "src"))
    from futudiffu.fp8_kernels import fp8_act_quant

    g = _gen(3)
    x = (torch.randn(16, 512, generator=g) * torch.rand(16, 1, generator=g) * 10).to(torch.bfloat16)
    x[3, 128:256] = 0.0
    _, s = fp8_act_quant(x)
    torch.save({"x": x, "scales": s}, HERE / "act_quant_scales.pt")


def _install_interpreter_fixes() -> None:
    """Make the Triton CPU interpreter compute what the compiled kernels compute.

    Two defects of the interpreter (triton/runtime/interpreter.py) would
    otherwise make the reference's kernels disagree with their own GPU builds:
      * float downcasts (f32 -> bf16 in ``cast_impl``, f32 -> e4m3 / bf16 / f16
        in ``create_fp_to_fp``) go through ``_convert_float``, which truncates the
        significand (or rounds ties away from zero) instead of rounding to nearest
        even as the GPU's ``cvt.rn`` does;
      * ``create_dot`` multiplies bf16 operands as their raw uint16 bit patterns.
    The replacement downcast rounds to nearest even through torch's own
    conversions; the replacement dot widens float operands exactly to f32 and
    accumulates in f32 (integer operands keep the int32 matmul).  Divides,
    exp2 / log2 and sqrt stay numpy's correctly rounded versions, so the fixtures
    pin the reference's formulas with IEEE arithmetic (the oracle's CPU default).
    """
    import numpy as np
    import triton.language as tl
    from triton.runtime import interpreter as TI

    orig = TI._convert_float
    narrow = {tl.bfloat16: (torch.bfloat16, torch.int16, np.uint16), tl.float16: (torch.float16, torch.int16, np.uint16),
              tl.float8e4nv: (torch.float8_e4m3fn, torch.uint8, np.uint8),
              tl.float8e5: (torch.float8_e5m2, torch.uint8, np.uint8)}

    def widen(data, dtype):
        if dtype == tl.float32:
            return data.astype(np.float32, copy=False)
        return orig(data, dtype, tl.float32, None).view(np.float32)  # exact: upcasts only shift bits

    def convert(data, src, dst, rounding_mode):
        if src.primitive_bitwidth > dst.primitive_bitwidth and dst in narrow:
            td, view, nd = narrow[dst]
            f = torch.from_numpy(np.ascontiguousarray(widen(data, src)))
            return f.to(td).view(view).numpy().view(nd)
        return orig(data, src, dst, rounding_mode)

    def dot(self, a, b, d, input_precision, max_num_imprecise_acc):
        ad = widen(a.data, a.dtype) if a.dtype.is_floating() else a.data
        bd = widen(b.data, b.dtype) if b.dtype.is_floating() else b.data
        return TI.TensorHandle(np.matmul(ad, bd, dtype=d.data.dtype) + d.data, d.dtype.scalar)

    TI._convert_float = convert
    TI.InterpreterBuilder.create_dot = dot


def main_kernels(ref: Path) -> None:
    """ref_kernels.pt: the reference's own Triton kernels run in the CPU
    interpreter (TRITON_INTERPRET=1, set by the parent) with the fixes above.

    act quant (fp8_kernels.py:54-90), blockwise GEMM / addmm kernels (:125-343,
    launched with one of their autotune configs, BLOCK_SIZE_M 64, as the
    autotuner cannot time on the CPU), fp8_gemm_quant (:573-709), fp8_gelu
    (:716-833), fp8_silu_gate_quant (:842-978), the fused RMSNorm+modulate and
    QKV-postprocess kernels (fused_kernels.py:43-86, :270-471; the gate+residual
    kernel calls libdevice tanh, which the interpreter lacks), and the attention
    forward / backward entry points of sage_attention.py (:121-341, :344-458,
    :461-648) in their INT8 / FP8 QK and bf16 / FP8 PV modes, masked and not.
    """
    _install_interpreter_fixes()
    sys.path.insert(0, str(ref / "src"))
    sys.path.insert(0, str(ref))
    from futudiffu import fp8_kernels as rk
    from futudiffu import fused_kernels as rf
    from futudiffu import sage_attention as rsa

    out = {}
    # ---- G1 act quant: codes and scales
    g = _gen(3)
    x = (torch.randn(16, 512, generator=g) * torch.rand(16, 1, generator=g) * 10).to(torch.bfloat16)
    x[3, 128:256] = 0.0
    y, s = rk.fp8_act_quant(x)
    out["act"] = {"x": x, "codes": y, "scales": s}

    # ---- G2 GEMM / addmm (bf16 and f32 outputs), G2+requant, GELU requant
    g = _gen(6)
    M, N, K = 72, 256, 384
    xa = torch.randn(M, K, generator=g).to(torch.bfloat16)
    w = (torch.randn(N, K, generator=g) * 0.02).to(torch.bfloat16)
    a8, a_s = rk.fp8_act_quant(xa)
    saved = torch.Tensor.cuda
    torch.Tensor.cuda = lambda self, *a, **kw: self  # type: ignore[assignment]
    try:
        from futudiffu.fp8 import quantize_fp8_blockwise

        b8, b_s = quantize_fp8_blockwise(w)
    finally:
        torch.Tensor.cuda = saved  # type: ignore[assignment]
    bias = torch.randn(N, generator=g).to(torch.bfloat16)
    grid = ((M + 63) // 64, N // 128)
    gemm = {"a8": a8, "a_s": a_s, "b8": b8, "b_s": b_s, "bias": bias}
    for name, dt in (("bf16", torch.bfloat16), ("f32", torch.float32)):
        c = torch.empty(M, N, dtype=dt)
        rk.fp8_gemm_blockwise_kernel.fn[grid](a8, b8, c, a_s, b_s, M, N, K, 128,
                                              BLOCK_SIZE_M=64, BLOCK_SIZE_N=128, BLOCK_SIZE_K=128)
        cb = torch.empty(M, N, dtype=dt)
        rk.fp8_addmm_blockwise_kernel.fn[grid](a8, b8, cb, bias, a_s, b_s, M, N, K, 128, BLOCK_SIZE_M=64,
                                               BLOCK_SIZE_N=128, BLOCK_SIZE_K=128, HAS_BIAS=True)
        gemm[f"c_{name}"], gemm[f"c_bias_{name}"] = c, cb
    # rowwise (per-output-row weight scale), v1t (B pre-transposed to (K, N)),
    # v2 (bf16 A quantised per 128-K slice inside the kernel), each with one of
    # its autotune configs
    b_row = (torch.rand(N, generator=g) * 1e-3 + 1e-4).float()
    c = torch.empty(M, N, dtype=torch.float32)
    rk.fp8_gemm_rowwise_kernel.fn[grid](a8, b8, c, a_s, b_row, M, N, K, 128,
                                        BLOCK_SIZE_M=64, BLOCK_SIZE_N=128, BLOCK_SIZE_K=128)
    gemm["b_row"], gemm["c_rowwise_f32"] = b_row, c
    bt, bst = b8.t().contiguous(), b_s.t().contiguous()
    c = torch.empty(M, N, dtype=torch.float32)
    rk.fp8_gemm_v1t_kernel.fn[(grid[0], N // 128)](a8, bt, c, a_s, bst, M, N, K, 128,
                                                   BLOCK_SIZE_M=64, BLOCK_SIZE_N=128, BLOCK_SIZE_K=128)
    gemm["c_v1t_f32"] = c
    c = torch.empty(M, N, dtype=torch.float32)
    rk.fp8_gemm_v2_kernel.fn[(grid[0], N // 128)](xa, bt, c, bst, M, N, K, 128,
                                                  BLOCK_SIZE_M=64, BLOCK_SIZE_N=128, FP8_MAX=448.0)
    gemm["xa"], gemm["c_v2_f32"] = xa, c
    gemm["quant"] = rk.fp8_gemm_quant(a8, a_s, b8, b_s)
    gemm["gelu"] = rk.fp8_gelu(a8, a_s)
    out["gemm"] = gemm
    g = _gen(7)
    xs = (torch.randn(40, 2 * 256, generator=g) * 2).to(torch.bfloat16)
    out["silu_gate"] = {"x": xs, "out": rk.fp8_silu_gate_quant(xs)}

    # ---- P1 / P3 Triton kernels on the inputs stored in fused_norms.pt
    fz = torch.load(HERE / "fused_norms.pt", weights_only=False)
    out["norms"] = {
        "modulate": rf._fused_rms_norm_modulate_triton(fz["x"], fz["w"], fz["scale"], 1e-5),
        "qkv": rf._fused_qkv_postprocess_triton(fz["qkv"], fz["qw"], fz["kw"], fz["freqs"], fz["H"], fz["hd"], 1e-5),
    }

    # ---- attention: ragged N (two Q blocks, three 64-key tiles), a mask with skipped tiles
    g = _gen(8)
    B, H, Na = 1, 2, 136
    q = torch.randn(B, H, Na, 128, generator=g).to(torch.bfloat16)
    k = (torch.randn(B, H, Na, 128, generator=g) + 2.0 * torch.randn(128, generator=g)).to(torch.bfloat16)
    v = torch.randn(B, H, Na, 128, generator=g).to(torch.bfloat16)
    do = torch.randn(B, H, Na, 128, generator=g).to(torch.bfloat16)
    mask = torch.tensor([[1, 0, 1], [1, 1, 0]], dtype=torch.uint8)
    sm = 1.0 / 128 ** 0.5
    att = {"q": q, "k": k, "v": v, "dout": do, "mask": mask, "sm_scale": sm, "fwd": {}, "bwd": {}}
    for qk in ("int8", "fp8"):
        rsa.configure_sage(smooth_k=True, qk_quant=qk, pv_quant="bf16")
        o, lse = rsa.sage_attn_forward_with_lse(q, k, v)
        att["fwd"][f"{qk}_bf16"] = (o, lse)
        att["fwd"][f"{qk}_bf16_masked"] = (rsa.sage_attn_forward_masked(q, k, v, mask), None)
        att["bwd"][qk] = rsa.sage_attn_backward(q, k, v, o, lse, do, sm)
    rsa.configure_sage(smooth_k=True, qk_quant="fp8", pv_quant="fp8")
    att["fwd"]["fp8_fp8tile"] = rsa.sage_attn_forward_with_lse(q, k, v)
    rsa.configure_sage(smooth_k=True, qk_quant="int8", pv_quant="bf16")
    o, lse = rsa.sage_attn_forward_masked_with_lse(q, k, v, mask)
    att["fwd"]["int8_bf16_masked_lse"] = (o, lse)
    att["bwd"]["int8_masked"] = rsa.sage_attn_backward_masked(q, k, v, o, lse, do, mask, sm)
    out["attention"] = att

    # ---- multi-LoRA: src_ii MultiLoRALinear (torch, the production path) on an
    # nn.Linear base, and the Triton _multi_lora_kernel (lora_kernels.py:55-157)
    from futudiffu.lora_kernels import multi_lora_forward
    from src_ii.multi_lora import MultiLoRALinear

    g = _gen(9)
    IN, OUT, S = 256, 384, 40
    base = torch.nn.Linear(IN, OUT, bias=True).to(torch.bfloat16)
    with torch.no_grad():
        base.weight.copy_(torch.randn(OUT, IN, generator=g) * 0.05)
        base.bias.copy_(torch.randn(OUT, generator=g) * 0.1)
    m = MultiLoRALinear(base, max_adapters=3, max_rank=16)
    m.assign_adapter(0, "a", rank=8, alpha=16.0, init_a="zeros")
    m.assign_adapter(2, "c", rank=16, alpha=8.0, init_a="zeros")
    with torch.no_grad():
        for j, r in ((0, 8), (2, 16)):
            m.lora_A[j][:r].copy_(torch.randn(r, IN, generator=g) * 0.05)
            m.lora_B[j][:, :r].copy_(torch.randn(OUT, r, generator=g) * 0.05)
    xl = torch.randn(2, S, IN, generator=g).to(torch.bfloat16)
    scales = torch.rand(2, 3, generator=g) * 2.0
    t2i = torch.tensor([0] * 16 + [1] * 20 + [-1] * 4)  # per position, repeated per sample
    with torch.no_grad():
        lora = {"base_w": base.weight.detach().clone(), "base_b": base.bias.detach().clone(),
                "A": [p.detach().clone() for p in m.lora_A], "B": [p.detach().clone() for p in m.lora_B],
                "scalings": m._lora_scalings.clone(), "active": m._slot_active.clone(),
                "x": xl, "scales": scales, "token_to_image": t2i,
                "delta": m.adapter_delta(xl, scales, t2i), "out": m(xl, scales, t2i)}
        A_all = torch.stack(lora["A"])
        B_all = torch.stack(lora["B"])
        scale_all = scales * (m._lora_scalings * m._slot_active)[None, :]
        lora["kernel"] = {"A_all": A_all, "B_all": B_all, "scale_all": scale_all,
                          "out": multi_lora_forward(xl, A_all, B_all, scale_all)}
    out["lora"] = lora
    torch.save(out, HERE / "ref_kernels.pt")


def main_fallback(ref: Path) -> None:
    sys.meta_path.insert(0, _BlockTriton())
    sys.path.insert(0, str(ref / "src"))
    from futudiffu import fp8_kernels as rk
    from futudiffu import fused_kernels as rf
    from futudiffu.attention import rope_embed

    assert not rk._HAS_TRITON and not rf._HAS_TRITON
    g = _gen(4)
    x = (torch.randn(8, 2 * 256, generator=g) * 2).to(torch.bfloat16)
    y, s = rk.fp8_silu_gate_quant(x)
    torch.save({"x": x, "codes": y, "scales": s}, HERE / "silu_gate.pt")

    g = _gen(5)
    B, S, H, hd = 2, 40, 4, 128
    dim = H * hd
    xn = torch.randn(B, S, dim, generator=g).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(dim, generator=g)).to(torch.bfloat16)
    scale = (0.5 * torch.randn(B, dim, generator=g)).to(torch.bfloat16)
    gate = torch.randn(B, dim, generator=g).to(torch.bfloat16)
    res = torch.randn(B, S, dim, generator=g).to(torch.bfloat16)
    mod = rf._fused_rms_norm_modulate_fallback(xn, w, scale, 1e-5)
    gr = rf._fused_rms_norm_gate_residual_fallback(xn, w, gate, res, 1e-5)
    qkv = torch.randn(B, S, 3 * dim, generator=g).to(torch.bfloat16)
    qw = 1 + 0.1 * torch.randn(hd, generator=g)
    kw = 1 + 0.1 * torch.randn(hd, generator=g)
    pos = torch.zeros(S, 3)
    pos[:, 0] = 1.0
    pos[:, 1] = (torch.arange(S) % 7).float()
    pos[:, 2] = (torch.arange(S) // 7).float()
    freqs = torch.cat([rope_embed(pos[None, :, i], d, 256.0) for i, d in enumerate((32, 48, 48))], dim=-3)
    freqs = freqs.expand(B, S, hd // 2, 2, 2).unsqueeze(2).contiguous()
    q_ref, k_ref, v_ref = rf._qkv_postprocess_reference(qkv, qw, kw, freqs, H, hd, 1e-5)
    torch.save({"x": xn, "w": w, "scale": scale, "gate": gate, "res": res, "modulate": mod,
                "gate_residual": gr, "qkv": qkv, "qw": qw, "kw": kw, "freqs": freqs,
                "q": q_ref, "k": k_ref, "v": v_ref, "H": H, "hd": hd}, HERE / "fused_norms.pt")


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, type=Path)
    ap.add_argument("--section", default="main", choices=["main", "interp", "kernels", "fallback"])
    a = ap.parse_args()
    {"main": main_triton, "interp": main_interp, "kernels": main_kernels,
     "fallback": main_fallback}[a.section](a.reference)
