"""Run the reference's own Triton kernels on a B200: golden outputs and timings.

The reference (sqcu/futudiffu) implements this path as Triton kernels that need
a GPU.  This script imports the reference from ``--reference`` (a checkout, or
the package directory laid out as an install: ``futudiffu/`` and ``src_ii/``),
runs its kernels on the seeded inputs of ``gpu_cases.py`` and stores

  * the outputs (``--out``, a .pt file): SHA-256 digests of full outputs for the
    bit-exact gates (quantised codes and scales), full small outputs, and fixed
    row samples of large floating-point outputs for the tolerance gates;
  * the timings (``--timing``, JSON): every reference kernel timed as the
    reference's own benchmarks time it (bench/bench_attention.py:33-53,
    bench/bench_fp8_gemm.py:38-49: CUDA events, 5 warm-up calls, median of 20),
    next to this build's kernel behind the same API at the same shapes.

Usage (on a GPU machine):
  python tests/golden/make_gpu_golden.py --reference <reference path> \\
      --out tests/golden/ref_gpu.pt --timing <timings.json>

Reference entry points used: futudiffu.fp8_kernels.fp8_act_quant (:54-90),
fp8_gemm_blockwise (:125-227), fp8_gemm_quant (:573-709), fp8_gelu (:716-833),
fp8_silu_gate_quant (:842-978); futudiffu.fp8.quantize_fp8_blockwise (:337-371);
futudiffu.fused_kernels._fused_rms_norm_modulate_triton /
_fused_rms_norm_gate_residual_triton / _fused_qkv_postprocess_triton (:155-247,
:388-471); futudiffu.sage_attention.configure_sage, sage_attn_forward_with_lse,
sage_attn_forward_masked_with_lse, sage_attn_backward (:37-60, :271-458, :461-531).
"""

from __future__ import annotations

import argparse
import json
import statistics
import sys
import time
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
for p in (str(ROOT), str(HERE)):
    if p not in sys.path:
        sys.path.insert(0, p)

import gpu_cases as C  # noqa: E402

DEV = torch.device("cuda:0")


def _import_reference(ref: Path):
    for p in (ref / "src", ref):
        if p.exists():
            sys.path.insert(0, str(p))
    from futudiffu import fp8 as rfp8
    from futudiffu import fp8_kernels as rk
    from futudiffu import fused_kernels as rf
    from futudiffu import sage_attention as rsa

    assert rk._HAS_TRITON and rf._HAS_TRITON, "the reference's Triton kernels are not available"
    return rk, rfp8, rf, rsa


def bench(fn, warmup: int = 5, iters: int = 20) -> float:
    """Median CUDA-event time (ms) of fn(), as the reference's benchmarks measure."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    ts = []
    for _ in range(iters):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        fn()
        e1.record()
        torch.cuda.synchronize()
        ts.append(e0.elapsed_time(e1))
    return statistics.median(ts)


def _rows(t: torch.Tensor, rows: torch.Tensor) -> torch.Tensor:
    return t[rows.to(t.device)].cpu().clone()


def run(ref: Path, out_path: Path, timing_path: Path | None, skip_timing: bool) -> None:
    rk, rfp8, rf, rsa = _import_reference(ref)
    import futudiffu_b200.fp8_kernels as ok
    import futudiffu_b200.fused_kernels as of
    from futudiffu_b200 import sage_attention as osa
    from futudiffu_b200.fp8 import quantize_fp8_blockwise_cuda

    out: dict = {"act": {}, "silu": {}, "gemm": {}, "norm": {}, "attn": {}, "attn_bwd": {}}
    timing: list[dict] = []

    def record(name, work, unit, ref_fn, ours_fn, **extra):
        if skip_timing:
            return
        r = bench(ref_fn)
        o = bench(ours_fn)
        timing.append({"name": name, "ref_ms": r, "ours_ms": o, "work": work, "unit": unit,
                       "ref_rate": work / (r * 1e-3) / 1e12, "ours_rate": work / (o * 1e-3) / 1e12,
                       "speedup": r / o, **extra})
        print(f"{name:44s} ref {r:8.3f} ms  ours {o:8.3f} ms  x{r / o:5.2f}", flush=True)

    # ------------------------------------------------------------ G1 activation quantiser
    for name in C.ACT_SHAPES:
        x = C.act_input(name).to(DEV)
        y, s = rk.fp8_act_quant(x)
        d = {"codes": C.digest(y), "scales": C.digest(s), "head_codes": y[:4].cpu(), "head_scales": s[:4].cpu()}
        if name in ("small", "ragged"):
            d["codes_full"], d["scales_full"] = y.cpu(), s.cpu()
        out["act"][name] = d
        if name in ("config1", "ref"):
            M, K = C.ACT_SHAPES[name]
            record(f"act_quant {M}x{K}", 3.0 * M * K + 4.0 * M * K / 128, "TB/s",
                   lambda: rk.fp8_act_quant(x), lambda: ok.fp8_act_quant(x))

    # ------------------------------------------------------------ G4 SiLU gate + quant
    for name in C.SILU_SHAPES:
        x = C.silu_input(name).to(DEV)
        y, s = rk.fp8_silu_gate_quant(x)
        d = {"codes": C.digest(y), "scales": C.digest(s), "head_codes": y[:4].cpu(), "head_scales": s[:4].cpu()}
        if name == "small":
            d["codes_full"], d["scales_full"] = y.cpu(), s.cpu()
        out["silu"][name] = d
        if name == "zimage":
            M, N2 = C.SILU_SHAPES[name]
            record(f"silu_gate_quant {M}x{N2}", 2.0 * M * N2 + M * N2 / 2 * (1 + 4 / 128), "TB/s",
                   lambda: rk.fp8_silu_gate_quant(x), lambda: ok.fp8_silu_gate_quant(x))

    # ------------------------------------------------------------ G6 + G2 GEMM, requant, GELU
    for name, (M, N, K) in C.GEMM_SHAPES.items():
        x, w = C.gemm_inputs(name)
        x, w = x.to(DEV), w.to(DEV)
        a8, a_s = rk.fp8_act_quant(x)
        b8, b_s = (t.to(DEV) for t in rfp8.quantize_fp8_blockwise(w))  # returned on the CPU (fp8.py:371)
        c = rk.fp8_gemm_blockwise(a8, a_s, b8, b_s, output_dtype=torch.bfloat16)
        rows = C.row_sample(M, C.GEMM_SAMPLE_ROWS[name])
        d = {"a_codes": C.digest(a8), "a_scales": C.digest(a_s), "b_codes": C.digest(b8), "b_scales": C.digest(b_s),
             "c": C.digest(c), "rows": rows, "c_rows": _rows(c, rows)}
        gq, gs = rk.fp8_gemm_quant(a8, a_s, b8, b_s)
        d.update(quant_codes=C.digest(gq), quant_scales=C.digest(gs), quant_rows_codes=_rows(gq, rows),
                 quant_rows_scales=_rows(gs, rows))
        ge, ges = rk.fp8_gelu(a8, a_s)
        d.update(gelu_codes=C.digest(ge), gelu_scales=C.digest(ges), gelu_head_codes=ge[:4].cpu(),
                 gelu_head_scales=ges[:4].cpu())
        if name == "small":
            d.update(c_full=c.cpu(), b8_full=b8.cpu(), b_s_full=b_s.cpu())
        out["gemm"][name] = d
        if name != "small":
            ob8, ob_s = quantize_fp8_blockwise_cuda(w)
            record(f"fp8_gemm_blockwise {M}x{N}x{K}", 2.0 * M * N * K, "TFLOP/s",
                   lambda: rk.fp8_gemm_blockwise(a8, a_s, b8, b_s, output_dtype=torch.bfloat16),
                   lambda: ok.fp8_gemm_blockwise(a8, a_s, ob8, ob_s, output_dtype=torch.bfloat16))
        del x, w, a8, a_s, b8, b_s, c
    # the remaining Z-Image shapes of the reference's GEMM benchmark (bench_fp8_gemm.py:24-30)
    if not skip_timing:
        g = C.gen(399)
        for (M, K, N) in ((8576, 3840, 3840), (8576, 3840, 20480), (8576, 10240, 3840)):
            x = torch.randn(M, K, generator=g).to(torch.bfloat16).to(DEV)
            w = (torch.randn(N, K, generator=g) * 0.02).to(torch.bfloat16).to(DEV)
            a8, a_s = rk.fp8_act_quant(x)
            b8, b_s = (t.to(DEV) for t in rfp8.quantize_fp8_blockwise(w))
            record(f"fp8_gemm_blockwise {M}x{N}x{K}", 2.0 * M * N * K, "TFLOP/s",
                   lambda: rk.fp8_gemm_blockwise(a8, a_s, b8, b_s, output_dtype=torch.bfloat16),
                   lambda: ok.fp8_gemm_blockwise(a8, a_s, b8, b_s, output_dtype=torch.bfloat16))
            del x, w, a8, a_s, b8, b_s

    # ------------------------------------------------------------ P1 / P2 / P3
    ni = {k: v.to(DEV) for k, v in C.norm_inputs().items()}
    rows = C.row_sample(C.NORM_SHAPE[1], C.NORM_SAMPLE_ROWS)
    mod = rf._fused_rms_norm_modulate_triton(ni["x"], ni["w"], ni["scale"], 1e-5)
    gr = rf._fused_rms_norm_gate_residual_triton(ni["x"], ni["w"], ni["gate"], ni["res"], 1e-5)
    qi = C.qkv_inputs()
    qkv, qw, kw, fr = (qi[k].to(DEV) for k in ("qkv", "qw", "kw", "freqs"))
    q, k, v = rf._fused_qkv_postprocess_triton(qkv, qw, kw, fr, qi["H"], 128, 1e-5)
    out["norm"] = {"rows": rows, "modulate": C.digest(mod), "modulate_rows": mod[0, rows.to(DEV)].cpu(),
                   "gate_residual": C.digest(gr), "gate_residual_rows": gr[0, rows.to(DEV)].cpu(),
                   "q": C.digest(q), "k": C.digest(k), "v": C.digest(v),
                   "qkv_heads": torch.arange(0, qi["H"], 6),
                   **{f"{n}_rows": t[0, ::6][:, rows.to(DEV)].cpu() for n, t in (("q", q), ("k", k), ("v", v))}}
    B, S, Dm = C.NORM_SHAPE
    record(f"fused_rms_norm_modulate {B}x{S}x{Dm}", 4.0 * B * S * Dm, "TB/s",
           lambda: rf._fused_rms_norm_modulate_triton(ni["x"], ni["w"], ni["scale"], 1e-5),
           lambda: of.fused_rms_norm_modulate(ni["x"], ni["w"], ni["scale"], 1e-5))
    record(f"fused_rms_norm_gate_residual {B}x{S}x{Dm}", 6.0 * B * S * Dm, "TB/s",
           lambda: rf._fused_rms_norm_gate_residual_triton(ni["x"], ni["w"], ni["gate"], ni["res"], 1e-5),
           lambda: of.fused_rms_norm_gate_residual(ni["x"], ni["w"], ni["gate"], ni["res"], 1e-5))
    record(f"fused_qkv_postprocess {B}x{S}x{qi['H']}x128", 12.0 * B * S * qi["H"] * 128, "TB/s",
           lambda: rf._fused_qkv_postprocess_triton(qkv, qw, kw, fr, qi["H"], 128, 1e-5),
           lambda: of.fused_qkv_postprocess(qkv, qw, kw, fr, qi["H"], 128, 1e-5))
    del ni, mod, gr, qkv, q, k, v

    # ------------------------------------------------------------ A1-A7 attention
    for name, modes in C.ATTN_MODES.items():
        q, k, v, do = (t.to(DEV) for t in C.attn_inputs(name))
        Bb, Hh, N = C.ATTN_SHAPES[name]
        heads, rows = C.attn_sample(name)
        mask = C.attn_mask(name).to(DEV)
        ops = 4.0 * Bb * Hh * N * N * 128
        for qk, pv, masked in modes:
            key = f"{qk}_{pv}" + ("_masked" if masked else "")
            rsa.configure_sage(smooth_k=True, qk_quant=qk, pv_quant=pv)
            osa.configure_sage(smooth_k=True, qk_quant=qk, pv_quant=pv)
            if masked:
                o, lse = rsa.sage_attn_forward_masked_with_lse(q, k, v, mask)
                rfn = lambda: rsa.sage_attn_forward_masked_with_lse(q, k, v, mask)  # noqa: E731
                ofn = lambda: osa.sage_attn_forward_masked_with_lse(q, k, v, mask)  # noqa: E731
            else:
                o, lse = rsa.sage_attn_forward_with_lse(q, k, v)
                rfn = lambda: rsa.sage_attn_forward_with_lse(q, k, v)  # noqa: E731
                ofn = lambda: osa.sage_attn_forward_with_lse(q, k, v)  # noqa: E731
            of_ = o.reshape(Bb * Hh, N, 128)
            out["attn"][f"{name}/{key}"] = {
                "heads": heads, "rows": rows, "out": of_[heads.to(DEV)][:, rows.to(DEV)].cpu(),
                "lse": lse[heads.to(DEV)][:, rows.to(DEV)].cpu(), "out_digest": C.digest(o),
                "finite_rows": torch.isfinite(of_.float()).all(-1).sum().item()}
            if name != "ragged":
                dens = float(mask.float().mean()) if masked else 1.0
                record(f"attention {name} {key} B{Bb} H{Hh} N{N}", ops * dens, "TOP/s", rfn, ofn,
                       mask_density=dens)
        for qk in C.ATTN_BWD.get(name, []):
            rsa.configure_sage(smooth_k=True, qk_quant=qk, pv_quant="bf16")
            o, lse = rsa.sage_attn_forward_with_lse(q, k, v)
            dq, dk, dv = rsa.sage_attn_backward(q, k, v, o, lse, do, C.SM)
            out["attn_bwd"][f"{name}/{qk}"] = {
                "heads": heads, "rows": rows,
                **{n: t.reshape(Bb * Hh, N, 128)[heads.to(DEV)][:, rows.to(DEV)].cpu()
                   for n, t in (("dq", dq), ("dk", dk), ("dv", dv))}}
        rsa.configure_sage()
        osa.configure_sage()
        del q, k, v, do

    out["meta"] = {"device": torch.cuda.get_device_name(0), "torch": torch.__version__,
                   "triton": __import__("triton").__version__,
                   "when": time.strftime("%Y-%m-%dT%H:%M:%SZ", time.gmtime())}
    out_path.parent.mkdir(parents=True, exist_ok=True)
    torch.save(out, out_path)
    print(f"wrote {out_path} ({out_path.stat().st_size / 1e6:.2f} MB)")
    if timing_path is not None and not skip_timing:
        timing_path.parent.mkdir(parents=True, exist_ok=True)
        timing_path.write_text(json.dumps({"meta": out["meta"], "method": "CUDA events, 5 warm-up calls, median of "
                                           "20 (the reference's bench_attention.py / bench_fp8_gemm.py); no L2 "
                                           "flush", "rows": timing}, indent=1))


if __name__ == "__main__":
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--reference", required=True, type=Path)
    ap.add_argument("--out", required=True, type=Path)
    ap.add_argument("--timing", type=Path, default=None)
    ap.add_argument("--skip-timing", action="store_true")
    a = ap.parse_args()
    run(a.reference, a.out, a.timing, a.skip_timing)
