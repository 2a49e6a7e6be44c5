"""Benchmarks of the quantized DiT hot path on B200.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                  [--workload dit|video|attention|gemm|packed|block]

Workloads (one "step" each):
  dit (default, benchmark config 4, the headline metric "DiT denoise steps/s"):
      one rectified-flow Euler step of the 12B-class DiT (19 double + 38
      single blocks, hidden 3072, 4096 image + 512 text tokens) over the whole
      batch of 8, random-init FP8 weights.  The batch is sharded by sample:
      8/N samples per rank, no collective on the data path (strong scaling);
      value = batch-8 steps per second = 1 / max-over-ranks step time.
  attention (benchmark config 2): quantisation prologue + tcgen05 attention on
      B=2, H=24, S=4096, D=128 (int8 per-block QK, e4m3 P/V); replicas per rank.
  gemm (benchmark config 1, or the reference's Z-Image shapes): one FP8 block GEMM.
  block (benchmark config 3): one MMDiT double-stream block forward at batch 1
      (512 text + 4096 image tokens), replayed as a CUDA graph; replicas per rank.
  video (benchmark config 5): one denoise step of the 14B-class video DiT with
      Ulysses sequence parallelism (NCCL all-to-all around the attention).
  packed (the reference's production shape): a bin of the bin packer (two
      images + captions in 4288 tokens) through 30 Z-Image-class
      JointTransformerBlocks with per-image adaLN and the block mask.

``--impl reference`` times the CPU restatement of the reference algorithm (the
oracle) on a bounded sample on rank 0; the other ranks exit without work.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

import torch  # noqa: E402

B, H, S, D = 2, 24, 4096, 128
OPS_PER_STEP = 4 * B * H * S * S * D  # 412.3 G ops (2 for QK^T + 2 for PV per MAC pair)
METRIC = "SageAttn TOPS (B2 H24 S4096 D128, INT8 QK + FP8 PV)"
UNIT = "TOPS"
# Measured DRAM traffic of one attention launch at this workload (ncu
# dram__bytes_read.sum + dram__bytes_write.sum of attn_fwd_kernel): 75.6 + 16.1 MB.
ATTN_TRAFFIC_BYTES = 91.7e6
# Same for one GEMM launch at the reference QKV shape (M 8576, N 11520, K 3840).
GEMM_TRAFFIC_BYTES = {"ref_qkv": 352.5e6}


def peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"bf16_tflops": d["bf16_tflops"], "hbm_gbs": d["hbm_gbs"], "source": "measured",
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"])}
    return {"bf16_tflops": 1590.0, "hbm_gbs": 6650.0, "source": "fallback", "bf16_tflops_sustained": 1400.0}


class ClockSampler:
    """nvidia-smi clock / throttle samples while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[str] = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
        except (OSError, FileNotFoundError):
            self.proc = None
        time.sleep(0.3)
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for nm, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(nm)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"]}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def make_inputs(seed: int, device=None):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, H, S, D, generator=g, dtype=torch.float32).to(torch.bfloat16)
    k = (torch.randn(B, H, S, D, generator=g) + 2.0 * torch.randn(D, generator=g)).to(torch.bfloat16)
    v = torch.randn(B, H, S, D, generator=g, dtype=torch.float32).to(torch.bfloat16)
    if device is not None:
        q, k, v = q.to(device), k.to(device), v.to(device)
    return q, k, v


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        backend = "nccl" if torch.cuda.is_available() else "gloo"
        opts = None
        if torch.cuda.is_available():
            torch.cuda.set_device(local)
            # NCCL kernels on a high-priority stream: the pipelined Ulysses exchange
            # gets SMs as soon as attention CTAs retire
            opts = dist.ProcessGroupNCCL.Options()
            opts.is_high_priority_stream = True
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=120), pg_options=opts)
    return world, rank, local


def max_over_ranks(x: float, world: int, device) -> float:
    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world: int):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def cpu_baseline_sample(seconds_budget: float = 20.0) -> dict:
    """Time the CPU restatement of the reference algorithm on a bounded sample."""
    from oracle import attention as OA

    threads = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(0)
    heads, done_ops, t_total = 0, 0, 0.0
    while t_total < seconds_budget and heads < B * H:
        q = torch.randn(1, S, D, generator=g).to(torch.bfloat16)
        k = (torch.randn(1, S, D, generator=g) + 2.0 * torch.randn(D, generator=g)).to(torch.bfloat16)
        v = torch.randn(1, S, D, generator=g).to(torch.bfloat16)
        t0 = time.perf_counter()
        OA.attention_forward(q, k, v, sm_scale=1 / math.sqrt(D), qk_quant="int8", granularity="per_block",
                             pv_quant="fp8_channel")
        t_total += time.perf_counter() - t0
        heads += 1
        done_ops += 4 * S * S * D
    return {"value": done_ops / t_total / 1e12, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"{heads} of {B * H} (b,h) heads at S={S}, oracle.attention.attention_forward "
                      f"(torch CPU, {threads} threads), {t_total:.1f} s"}


def run_reference(args, world, rank):
    if rank != 0:
        return 0
    per_step = []
    cb = None
    for i in range(args.warmup + args.steps):
        r = cpu_baseline_sample(seconds_budget=max(2.0, 60.0 / max(1, args.warmup + args.steps)))
        if i >= args.warmup:
            per_step.append(r["value"])
        cb = r
    val = statistics.mean(per_step) if per_step else cb["value"]
    line = {
        "impl": "reference", "metric": METRIC, "value": val, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": OPS_PER_STEP / (val * 1e12) * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8/fp8",
        "data": "synthetic",
        "config": {"workload": "config2_quantized_attention", "B": B, "H": H, "S": S, "D": D,
                   "qk": "int8 per-block", "pv": "fp8 per-channel V, static P"},
        "cpu_baseline": {**cb, "value": val},
        "e2e": {"value": val, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def run_ours(args, world, rank, local):
    from futudiffu_b200 import _lib as L
    from futudiffu_b200 import check_status
    from futudiffu_b200 import sage_attention as SA

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    SA.configure_sage(smooth_k=True, qk_quant="int8", pv_quant="fp8", qk_granularity="per_block")
    q, k, v = make_inputs(1234 + rank, dev)
    BH = B * H
    qf, kf, vf = (t.reshape(BH, S, D) for t in (q, k, v))
    stream = torch.cuda.current_stream(dev)
    sm = 1.0 / math.sqrt(D)

    def step(ev_pair=None):
        qz = SA.quantize_qkv(qf, kf, vf, sm, smooth_k=True, qk_quant="int8", granularity="per_block",
                             pv_quant="fp8")
        out = torch.empty_like(qf)
        if ev_pair is not None:
            ev_pair[0].record(stream)
        L.call("fd_sage_attn_fwd", L.ptr(qz["q_codes"]), L.ptr(qz["q_desc"]), L.ptr(qz["k_codes"]),
               L.ptr(qz["k_desc"]), L.ptr(qz["v_codes"]), L.ptr(qz["v_desc"]), None, 0, L.ptr(out), None,
               BH, S, L.QK_INT8, L.GRAN_BLOCK, L.GRAN_BLOCK, L.PV_FP8, L.stream_ptr(dev))
        if ev_pair is not None:
            ev_pair[1].record(stream)
        return out

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    check_status()

    kev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize()
    with ClockSampler(dev.index if "CUDA_VISIBLE_DEVICES" not in os.environ else local) as clocks:
        start.record(stream)
        for i in range(args.steps):
            step(kev[i])
        end.record(stream)
        torch.cuda.synchronize()
    barrier(world)
    ms_local = start.elapsed_time(end) / args.steps
    kernel_ms = statistics.mean(a.elapsed_time(b) for a, b in kev)
    ms = max_over_ranks(ms_local, world, dev)
    kernel_ms = max_over_ranks(kernel_ms, world, dev)
    value = world * OPS_PER_STEP / (ms * 1e-3) / 1e12
    check_status()

    # ---------------- end to end: pinned host inputs -> device -> public API -> host output
    hq, hk, hv = (t.cpu().pin_memory() for t in (q, k, v))
    hout = torch.empty(B, H, S, D, dtype=torch.bfloat16).pin_memory()
    h2d = 3 * q.numel() * q.element_size()
    d2h = hout.numel() * hout.element_size()
    e2e_steps = max(3, min(args.steps, 20))

    def e2e_step():
        dq, dk, dv = (t.to(dev, non_blocking=True) for t in (hq, hk, hv))
        o = SA.sage_attn_forward(dq, dk, dv)
        hout.copy_(o, non_blocking=True)

    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize()
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / e2e_steps, world, dev)
    e2e_val = world * OPS_PER_STEP / (e2e_ms * 1e-3) / 1e12
    check_status()

    if rank == 0:
        pk = peaks()
        peak_tops = 2.0 * pk["bf16_tflops"]
        achieved = OPS_PER_STEP / (kernel_ms * 1e-3) / 1e12
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8/fp8", "data": "synthetic",
            "config": {"workload": "config2_quantized_attention", "B": B, "H": H, "S": S, "D": D,
                       "qk": "int8 per-block (Q 128 rows, K 64 rows), K mean-smoothed",
                       "pv": "fp8 e4m3 P (static scale), fp8 e4m3 V (per-channel)",
                       "step": "quantisation prologue + tcgen05 attention",
                       "l2": "inputs 151 MB bf16 > 126 MB L2; no explicit flush",
                       "parallelism": f"replicas x{world}"},
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak_tops, "unit": "TOP/s",
                         "frac": achieved / peak_tops, "traffic": ATTN_TRAFFIC_BYTES,
                         "kernel": "attn_fwd_kernel<int8, block, fp8>",
                         "kernel_ms": kernel_ms,
                         "peak_source": f"2 x {pk['source']} bf16 dense ({pk['bf16_tflops']} TF/s): "
                                        "int8/fp8 dense rate is twice bf16"},
            "cpu_baseline": cpu_baseline_sample(15.0) if world == 1 else None,
            "e2e": {"value": e2e_val, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "ms_per_step": e2e_ms, "api": "futudiffu_b200.sage_attention.sage_attn_forward"},
            "gpu_launches": 3 * args.steps,
            "clocks": clocks.summary(),
        }
        print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------------ config 4: DiT denoise
DIT_BATCH = 8
DIT_METRIC = "DiT denoise steps/s (12B-class, 19 double + 38 single blocks, 4096+512 tokens, batch 8)"
KERNELS_PER_CALL = {"fd_attn_quant": 3, "fd_attn_quant_noalloc": 3, "fd_attn_quant_kv": 2, "fd_sage_attn_bwd": 2}


class LaunchRecorder:
    """Counts this library's kernel launches and times every GEMM / attention
    launch with CUDA events on the launching stream while ``active``."""

    GEMMS = ("fd_fp8_gemm_blockwise", "fd_fp8_gemm_quant", "fd_fp8_gemm_quant_ld")

    def __init__(self):
        from futudiffu_b200 import _lib as L

        self.L = L
        self.orig = L.call
        self.active = False
        self.launches = 0
        self.pending = []  # (kind, work, e0, e1)
        L.call = self._call

    def _call(self, name, *args):
        if not self.active:
            return self.orig(name, *args)
        self.launches += KERNELS_PER_CALL.get(name, 1)
        kind = work = None
        if name in self.GEMMS:
            M, N, K = args[8], args[9], args[10]
            mult = 2 if (name == "fd_fp8_gemm_quant" and args[11] == self.L.ACT_SILU_GATE) else 1
            kind, work = "gemm", 2.0 * M * N * K * mult
        elif name == "fd_fp8_gemm_grouped2":
            probs = [self.L.GemmProblem.from_address(a) for a in args[:2]]
            mult = 2 if args[3] == self.L.ACT_SILU_GATE else 1
            kind, work = "gemm", sum(2.0 * q.M * q.N * q.K * mult for q in probs)
        elif name == "fd_fp8_gemm_qkv_quant":
            # the QKV linear(s) with the fused P3 + Q quantisation epilogue: GEMM work
            # plus the prologue's first pass, kept apart from the plain GEMM rate
            probs = [self.L.GemmProblem.from_address(a) for a in (args[0], args[2]) if a]
            kind, work = "gemm_qkv", sum(2.0 * q.M * q.N * q.K for q in probs)
        elif name in ("fd_sage_attn_fwd", "fd_sage_attn_fwd_bnhd"):
            BH, N = args[10], args[11]
            kind, work = "attn", 4.0 * BH * N * N * 128
        elif name == "fd_sage_attn_fwd_quant_out":
            BH, N = args[9], args[10]
            kind, work = "attn", 4.0 * BH * N * N * 128
        if kind is None:
            return self.orig(name, *args)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        r = self.orig(name, *args)
        e1.record()
        self.pending.append((kind, work, e0, e1))
        return r

    def summary(self, kind):
        ms = sum(a.elapsed_time(b) for k, _, a, b in self.pending if k == kind)
        work = sum(w for k, w, _, _ in self.pending if k == kind)
        n = sum(1 for k, *_ in self.pending if k == kind)
        return work, ms, n

    def close(self):
        self.L.call = self.orig


_DIT_CPU_BLOCKS: dict = {}


def _cpu_threads() -> int:
    threads = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()
    torch.set_num_threads(threads)
    return threads


def dit_cpu_block_seconds(kind: str, img_tokens: int = 4096) -> float:
    """Seconds for one config-4 block ("double" or "single") of one sample at 512
    text + ``img_tokens`` image tokens through the oracle on the host cores, in the
    reference's torch-eager dequantize-and-compute formulation (CPU-built weights)."""
    from futudiffu_b200.dit import DiTConfig, image_freqs, text_freqs
    from oracle import dit as OD

    cfg = DiTConfig(img_grid=(img_tokens // 64, 64))
    key = (kind, img_tokens)
    if key not in _DIT_CPU_BLOCKS:
        blk = OD.random_double_block(cfg, seed=0) if kind == "double" else OD.random_single_block(cfg, seed=1)
        cg = torch.Generator().manual_seed(1)
        x_txt = torch.randn(1, cfg.txt_tokens, cfg.hidden, generator=cg).to(torch.bfloat16)
        x_img = torch.randn(1, cfg.img_tokens, cfg.hidden, generator=cg).to(torch.bfloat16)
        vec = torch.randn(1, cfg.hidden, generator=cg).to(torch.bfloat16)
        ft = text_freqs(cfg, "cpu").unsqueeze(0)
        fi = image_freqs(cfg, "cpu").unsqueeze(0)
        _DIT_CPU_BLOCKS[key] = (blk, x_txt, x_img, vec, ft, fi)
    blk, x_txt, x_img, vec, ft, fi = _DIT_CPU_BLOCKS[key]
    with OD.eager_cpu_timing():
        t0 = time.perf_counter()
        if kind == "double":
            OD.double_block(blk, x_txt, x_img, vec, ft, fi)
        else:
            OD.single_block(blk, torch.cat([x_txt, x_img], 1), vec, torch.cat([ft, fi], 1))
        return time.perf_counter() - t0


def dit_cpu_step_seconds(t_double: float, t_single: float) -> float:
    """A batch-8 Euler step of config 4 from per-block times: linear in the block
    counts and the batch (every block of every sample does the same work)."""
    from futudiffu_b200.dit import DiTConfig

    cfg = DiTConfig()
    return DIT_BATCH * (cfg.n_double * t_double + cfg.n_single * t_single)


def dit_cpu_sample() -> dict:
    """cpu_baseline of the config-4 line: one full-size double-stream and one
    single-stream block (512 text + 4096 image tokens) on the host cores,
    extrapolated over block count x batch."""
    threads = _cpu_threads()
    td = dit_cpu_block_seconds("double")
    ts = dit_cpu_block_seconds("single")
    step_s = dit_cpu_step_seconds(td, ts)
    return {"value": 1.0 / step_s, "unit": "steps/s", "cores": threads, "kind": "port",
            "extrapolated": True,
            "sample": f"one double-stream ({td:.2f} s) and one single-stream ({ts:.2f} s) block at 512 text + "
                      f"4096 image tokens through oracle.dit (torch-eager dequantize-and-compute: fp32 matmuls "
                      f"of dequantised fp8 operands, restated int8/fp8 attention; {threads} threads), times "
                      f"batch 8 x (19 double + 38 single) blocks ({step_s:.0f} s/step)"}


def dit_config(cfg, gpus: int) -> dict:
    """The config-4 workload description, identical in both arms."""
    return {"workload": "config4_dit_denoise", "batch": DIT_BATCH, "per_gpu_batch": DIT_BATCH // gpus,
            "blocks": f"{cfg.n_double} double + {cfg.n_single} single", "hidden": cfg.hidden, "heads": cfg.heads,
            "tokens": f"{cfg.img_tokens} image + {cfg.txt_tokens} text", "euler_steps": 28,
            "linears": "fp8 e4m3, 1x128 activation / 128x128 weight fp32 scales",
            "attention": f"{cfg.qk_quant} {cfg.granularity.replace('_', '-')} QK (K mean-smoothed), "
                         f"{cfg.pv_quant} P and V",
            "l2": "weights 11 GB and activations >> 126 MB L2; no explicit flush",
            "parallelism": f"batch sharded by sample x{gpus}, no collective"}


def run_dit_reference(args, world, rank):
    """The reference arm: the oracle's CPU formulation on rank 0.  Each warm-up step
    is a small block (512 + 256 tokens); each timed step is one full-size block,
    double and single alternating (a pair when one step is asked for); the value
    is extrapolated over block count x batch from the mean block times."""
    if rank != 0:
        return 0
    from futudiffu_b200.dit import DiTConfig

    threads = _cpu_threads()
    for i in range(args.warmup):
        dit_cpu_block_seconds("double" if i % 2 == 0 else "single", img_tokens=256)
    times = {"double": [], "single": []}
    for i in range(args.steps):
        kinds = ("double", "single") if args.steps == 1 else (("double",) if i % 2 == 0 else ("single",))
        for kind in kinds:
            times[kind].append(dit_cpu_block_seconds(kind))
    td, ts = statistics.mean(times["double"]), statistics.mean(times["single"])
    step_s = dit_cpu_step_seconds(td, ts)
    val = 1.0 / step_s
    timed_s = sum(times["double"]) + sum(times["single"])
    cb = {"value": val, "unit": "steps/s", "cores": threads, "kind": "port", "extrapolated": True,
          "sample": f"{len(times['double'])} double-stream and {len(times['single'])} single-stream blocks at "
                    f"512 text + 4096 image tokens through oracle.dit (torch-eager dequantize-and-compute; "
                    f"{threads} threads; mean {td:.2f} s / {ts:.2f} s per block), times batch 8 x "
                    f"(19 double + 38 single) blocks ({step_s:.0f} s/step)"}
    print(json.dumps({
        "impl": "reference", "metric": DIT_METRIC, "value": val, "unit": "steps/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": timed_s / args.steps * 1e3,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "fp8/int8",
        "data": "synthetic (random-init weights, N(0,1) activations)",
        "config": dit_config(DiTConfig(), args.gpus),
        "extrapolated": True,
        "extrapolation": "each timed step is one full-size block (ms_per_step is its CPU time); value = 1 / "
                         "(8 samples x (19 x mean double-block s + 38 x mean single-block s))",
        "cpu_baseline": cb,
        "e2e": {"value": val, "unit": "steps/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)
    return 0


def time_gemm(dev, shape: str, steps: int, warmup: int, epilogue: str = "bf16") -> list[float]:
    """CUDA-event durations (ms) of ``steps`` FP8 block-GEMM launches at one of
    GEMM_SHAPES, with a 256 MiB write between launches so that every launch reads
    its operands from HBM (the operands of the smaller shapes fit in L2).
    ``epilogue``: "bf16" output, "gelu" (GELU(tanh) + 1 x 128 e4m3 requant, the
    MMDiT MLP-in epilogue) or "qkv" (the config-4 single-stream QKV linear, rows =
    samples x 4608 tokens, N = 3 x 24 heads x 128, with P3 and the Q quantisation in
    its epilogue: fd_fp8_gemm_qkv_quant, INT8 per-block Q, one launch)."""
    from futudiffu_b200 import _lib as L
    from futudiffu_b200.fp8 import quantize_fp8_blockwise_cuda
    from futudiffu_b200.fp8_kernels import fp8_act_quant

    M, N, K = GEMM_SHAPES[shape]
    g = torch.Generator().manual_seed(0)
    x = torch.randn(M, K, generator=g).to(torch.bfloat16).to(dev)
    w = (torch.randn(N, K, generator=g) * 0.02).to(dev)
    w8, ws = quantize_fp8_blockwise_cuda(w)
    a8, a_s = fp8_act_quant(x)
    stream = torch.cuda.current_stream(dev)
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)
    if epilogue == "qkv":
        H, S = N // 384, 4608
        assert N == 3 * H * 128 and M % S == 0
        Bq = M // S
        qn = torch.ones(128, dtype=torch.float32, device=dev)
        fr = torch.zeros(M, 64, 2, 2, dtype=torch.float32, device=dev)
        fr[:, :, 0, 0] = fr[:, :, 1, 1] = 1.0
        q_codes = torch.empty(Bq * H, S, 128, dtype=torch.int8, device=dev)
        q_desc = torch.empty(Bq * H, S // 128, dtype=torch.float32, device=dev)
        k_out = torch.empty(Bq * H, S, 128, dtype=torch.bfloat16, device=dev)
        v_out = torch.empty_like(k_out)
        wsp = torch.empty(int(L.lib().fd_qkv_quant_workspace_floats(Bq * H, S)), dtype=torch.float32, device=dev)
        prob = L.GemmProblem(L.ptr(a8), L.ptr(a_s), L.ptr(w8), L.ptr(ws), None, None, None, M, N, K)
        desc = L.QkvStream(L.ptr(qn), L.ptr(qn), L.ptr(fr), S, 0, 1e-6)
        import ctypes

        def gemm():
            L.call("fd_fp8_gemm_qkv_quant", ctypes.addressof(prob), ctypes.addressof(desc), None, None, L.DT_BF16,
                   Bq, H, S, L.QK_INT8, L.GRAN_BLOCK, L.PV_BF16, 0.1275, L.ptr(q_codes), L.ptr(q_desc),
                   L.ptr(k_out), L.ptr(v_out), L.ptr(wsp), L.stream_ptr(dev))
    elif epilogue == "gelu":
        c = torch.empty(M, N, dtype=torch.uint8, device=dev)
        c_s = torch.empty(M, N // 128, dtype=torch.float32, device=dev)

        def gemm():
            L.call("fd_fp8_gemm_quant", L.ptr(a8), L.ptr(a_s), L.ptr(w8), L.ptr(ws), None, 0, L.ptr(c), L.ptr(c_s),
                   M, N, K, L.ACT_GELU_TANH, L.stream_ptr(dev))
    else:
        c = torch.empty(M, N, dtype=torch.bfloat16, device=dev)

        def gemm():
            L.call("fd_fp8_gemm_blockwise", L.ptr(a8), L.ptr(a_s), L.ptr(w8), L.ptr(ws), None, 0, L.ptr(c),
                   L.DT_BF16, M, N, K, 0, L.stream_ptr(dev))

    for _ in range(warmup):
        gemm()
    torch.cuda.synchronize()
    ev = []
    for _ in range(steps):
        flush.zero_()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        gemm()
        e1.record(stream)
        ev.append((e0, e1))
    torch.cuda.synchronize()
    return [a.elapsed_time(b) for a, b in ev]


def time_attention(dev, pv: str, steps: int, warmup: int, seed: int = 1234) -> tuple[list[float], list[float]]:
    """Config 2 (B2 H24 S4096 D128, INT8 per-block Q/K, ``pv`` P and V): CUDA-event
    durations (ms) of the attention kernel alone and of the whole public call
    (``sage_attn_forward``: quantisation prologue + attention kernel)."""
    from futudiffu_b200 import _lib as L
    from futudiffu_b200 import sage_attention as SA

    q, k, v = make_inputs(seed, dev)
    BH = B * H
    qf, kf, vf = (t.reshape(BH, S, D) for t in (q, k, v))
    stream = torch.cuda.current_stream(dev)
    pvk = L.PV_FP8 if pv == "fp8" else L.PV_BF16
    qz = SA.quantize_qkv(qf, kf, vf, 1.0 / math.sqrt(D), smooth_k=True, qk_quant="int8", granularity="per_block",
                         pv_quant=pv)
    vsrc = qz["v_codes"] if pv == "fp8" else vf
    out = torch.empty_like(qf)

    def kernel():
        L.call("fd_sage_attn_fwd", L.ptr(qz["q_codes"]), L.ptr(qz["q_desc"]), L.ptr(qz["k_codes"]),
               L.ptr(qz["k_desc"]), L.ptr(vsrc), L.ptr(qz["v_desc"]), None, 0, L.ptr(out), None,
               BH, S, L.QK_INT8, L.GRAN_BLOCK, L.GRAN_BLOCK, pvk, L.stream_ptr(dev))

    SA.configure_sage(smooth_k=True, qk_quant="int8", pv_quant=pv, qk_granularity="per_block")
    try:
        res = []
        for fn in (kernel, lambda: SA.sage_attn_forward(q, k, v)):
            for _ in range(warmup):
                fn()
            torch.cuda.synchronize()
            ev = []
            for _ in range(steps):
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                fn()
                e1.record(stream)
                ev.append((e0, e1))
            torch.cuda.synchronize()
            res.append([a.elapsed_time(b) for a, b in ev])
    finally:
        SA.configure_sage()
    return res[0], res[1]


def sub_entries(dev, world: int, local: int) -> dict:
    """BASELINE.json's other two metrics, measured in the same process on every
    rank (replicas; max over ranks): FP8 block-GEMM TFLOPS at config 1 and at the
    reference's QKV shape, SageAttn TOPS at config 2."""
    pk = peaks()
    out = {}
    with ClockSampler(dev.index if "CUDA_VISIBLE_DEVICES" not in os.environ else local) as clocks:
        for shape in ("config1", "ref_qkv"):
            M, N, K = GEMM_SHAPES[shape]
            ms = max_over_ranks(statistics.mean(time_gemm(dev, shape, 30, 5)), world, dev)
            tf = 2.0 * M * N * K / (ms * 1e-3) / 1e12
            out[f"gemm_{shape}"] = {
                "metric": "FP8 block-GEMM TFLOPS", "value": tf * world, "unit": "TFLOPS", "per_gpu": tf,
                "ms": ms, "shape": {"M": M, "N": N, "K": K}, "l2": "flushed between launches",
                "frac_of_2x_burst_bf16": tf / (2.0 * pk["bf16_tflops"])}
        for pv in ("fp8", "bf16"):
            kms, sms = time_attention(dev, pv, 20, 5)
            kms = max_over_ranks(statistics.mean(kms), world, dev)
            sms = max_over_ranks(statistics.mean(sms), world, dev)
            kt, st = OPS_PER_STEP / (kms * 1e-3) / 1e12, OPS_PER_STEP / (sms * 1e-3) / 1e12
            out[f"attention_config2_{pv}_pv"] = {
                "metric": "SageAttn TOPS", "value": st * world, "unit": "TOPS", "per_gpu": st,
                "ms": sms, "kernel_ms": kms, "kernel_tops": kt,
                "mode": f"int8 per-block QK (K mean-smoothed), {'e4m3 P and per-channel V' if pv == 'fp8' else 'bf16 P and V'}",
                "timed": "sage_attn_forward (quantisation prologue + attention kernel); kernel_* the attention "
                         "kernel alone",
                "frac_of_2x_burst_bf16": kt / (2.0 * pk["bf16_tflops"])}
    for v in out.values():
        v["clocks"] = clocks.summary()
    return out


def run_dit(args, world, rank, local):
    from futudiffu_b200 import check_status
    from futudiffu_b200.dit import DiT, DiTConfig, EulerStepGraph, euler_step, flops_per_sample_step, sigmas

    if DIT_BATCH % world:
        raise SystemExit(f"batch {DIT_BATCH} does not shard over {world} GPUs")
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    cfg = DiTConfig()
    model = DiT(cfg, seed=0, device=dev)  # identical weights on every rank
    bl = DIT_BATCH // world
    g = torch.Generator().manual_seed(100 + rank)  # this rank's samples
    img = torch.randn(bl, cfg.img_tokens, cfg.patch_dim, generator=g).to(torch.bfloat16)
    txt = torch.randn(bl, cfg.txt_tokens, cfg.hidden, generator=g).to(torch.bfloat16)
    d_img, d_txt = img.to(dev), txt.to(dev)
    sig = sigmas(28)
    stream = torch.cuda.current_stream(dev)

    def step(i, x):
        return euler_step(model, x, d_txt, sig[i % 28], sig[i % 28 + 1])

    x = d_img
    for i in range(args.warmup):
        x = step(i, x)
    torch.cuda.synchronize()
    check_status()
    # Kernel accounting (not timed as the result): two eager steps with CUDA events
    # around every GEMM / attention launch and the launch count of one step.
    rec = LaunchRecorder()
    rec.active = True
    n_rec = 2
    for i in range(n_rec):
        x = step(i, x)
    rec.active = False
    torch.cuda.synchronize()
    gemm_work, gemm_ms, n_gemm = rec.summary("gemm")
    qkv_work, qkv_ms, n_qkv = rec.summary("gemm_qkv")
    attn_work, attn_ms, n_attn = rec.summary("attn")
    launches_per_step = rec.launches // n_rec
    rec.close()
    # The timed steps replay the step captured as one CUDA graph (EulerStepGraph).
    graph = EulerStepGraph(model, x, d_txt)
    for i in range(2):
        x = graph(x, d_txt, sig[i % 28], sig[i % 28 + 1])
    torch.cuda.synchronize()
    # settle: untimed replays for 3 s, so that the timed steps run at the clock the
    # GPU holds under this load (power-capped) whatever the per-GPU batch
    t_settle = time.perf_counter()
    n_settle = 0
    while time.perf_counter() - t_settle < 3.0:
        x = graph(x, d_txt, sig[n_settle % 28], sig[n_settle % 28 + 1])
        n_settle += 1
        if n_settle % 4 == 0:
            torch.cuda.synchronize()
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev.index if "CUDA_VISIBLE_DEVICES" not in os.environ else local) as clocks:
        if args.profile:
            torch.cuda.cudart().cudaProfilerStart()
        start.record(stream)
        for i in range(args.steps):
            x = graph(x, d_txt, sig[i % 28], sig[i % 28 + 1])
            if args.profile and i == 0:
                torch.cuda.synchronize()
                torch.cuda.cudart().cudaProfilerStop()
        end.record(stream)
        torch.cuda.synchronize()
    barrier(world)
    ms_local = start.elapsed_time(end) / args.steps
    ms = max_over_ranks(ms_local, world, dev)
    launches = launches_per_step * args.steps
    check_status()
    value = 1e3 / ms

    # ---------------- end to end: pinned host latents + text -> device -> Euler step -> host
    h_img, h_txt = img.pin_memory(), txt.pin_memory()
    h_out = torch.empty_like(img).pin_memory()
    h2d = (img.numel() + txt.numel()) * 2
    d2h = img.numel() * 2

    def e2e_step(i):
        y = graph(h_img.to(dev, non_blocking=True), h_txt.to(dev, non_blocking=True), sig[i], sig[i + 1])
        h_out.copy_(y, non_blocking=True)

    e2e_step(0)
    torch.cuda.synchronize()
    barrier(world)
    e2e_n = 3
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(e2e_n):
        e2e_step(i)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / e2e_n, world, dev)
    check_status()

    subs = sub_entries(dev, world, local) if not args.no_sub else {}
    if world >= 2 and not args.no_sub:
        del graph
        torch.cuda.empty_cache()
        subs["video_config5"] = video_sub_entry(dev, world, rank, local)
    check_status()

    if rank == 0:
        pk = peaks()
        peak = 2.0 * pk["bf16_tflops_sustained"]
        gemm_tf = gemm_work / (gemm_ms * 1e-3) / 1e12
        step_flops = flops_per_sample_step(cfg) * DIT_BATCH
        clk = clocks.summary()
        line = {
            "metric": DIT_METRIC, "value": value, "unit": "steps/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "fp8/int8", "data": "synthetic (random-init weights, N(0,1) latents/text)",
            "config": dit_config(cfg, world),
            "detail": {"model_tflop_per_step": step_flops / 1e12,
                       "model_tflops": step_flops / (ms * 1e-3) / 1e12,
                       "attention_kernel_tops": attn_work / (attn_ms * 1e-3) / 1e12 if attn_ms else None,
                       "time_share": {"gemm": (gemm_ms + qkv_ms) / n_rec / ms_local,
                                      "attention": attn_ms / n_rec / ms_local},
                       "qkv_linear_fused_prologue": {
                           "launches_per_step": n_qkv // n_rec,
                           "share": qkv_ms / n_rec / ms_local,
                           "gemm_tflops": qkv_work / (qkv_ms * 1e-3) / 1e12 if qkv_ms else None,
                           "note": "the QKV linears with P3 + Q quantisation in the GEMM epilogue "
                                   "(fd_fp8_gemm_qkv_quant); their time includes the prologue's first pass"},
                       "launch": f"each timed step replays the step's {launches_per_step} kernels as one "
                                 "captured CUDA graph",
                       "settle": f"{n_settle} untimed replays (3 s) before the timed steps"},
            "clock_normalised": {"sm_mhz_median": clk.get("sm_mhz"),
                                 "ms_x_mhz": ms * clk["sm_mhz"] if clk.get("sm_mhz") else None,
                                 "note": "step time x median SM clock under load; compare across N"},
            "roofline": {"bound": "tensor", "achieved": gemm_tf, "peak": peak, "unit": "TFLOP/s",
                         "frac": gemm_tf / peak, "traffic": None,
                         "kernel": f"gemm_fp8_kernel ({n_gemm // n_rec} GEMM launches of a step: every FP8 "
                                   "linear but the QKV linears with the fused prologue, see "
                                   "detail.qkv_linear_fused_prologue; flop-weighted, CUDA events per launch "
                                   "over two eager steps)",
                         "peak_source": f"2 x {pk['source']} sustained bf16 dense "
                                        f"({pk['bf16_tflops_sustained']} TF/s, kernels inside a long step): "
                                        "fp8 dense rate is twice bf16"},
            "cpu_baseline": dit_cpu_sample() if world == 1 else None,
            "e2e": {"value": 1e3 / e2e_ms, "unit": "steps/s", "h2d_bytes_per_step": h2d * world,
                    "d2h_bytes_per_step": d2h * world, "ms_per_step": e2e_ms,
                    "api": "futudiffu_b200.dit.EulerStepGraph (pinned host inputs copied in, result copied out)"},
            "gpu_launches": launches,
            "clocks": clk,
            "sub": subs,
        }
        print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------------ config 3: one MMDiT double-stream block
BLOCK_METRIC = "MMDiT double-stream block TFLOP/s (hidden 3072, 24 heads, 512 text + 4096 image tokens, batch 1)"


def block_flops(cfg) -> float:
    """Algorithmic FLOPs of one double-stream block forward of one sample."""
    D, R, N = cfg.hidden, cfg.mlp_ratio, cfg.tokens
    return 2 * (3 + 1 + 2 * R) * D * D * N + 4 * N * N * D


def block_cpu_sample() -> dict:
    """The oracle's double-stream block at its full size (512 text + 4096 image
    tokens) on the host cores, in the torch-eager dequantize-and-compute
    formulation, as a FLOP rate."""
    from futudiffu_b200.dit import DiTConfig

    threads = _cpu_threads()
    td = dit_cpu_block_seconds("double")
    return {"value": block_flops(DiTConfig()) / td / 1e12, "unit": "TFLOPS", "cores": threads, "kind": "port",
            "sample": f"one double-stream block at 512 text + 4096 image tokens through oracle.dit.double_block "
                      f"(torch-eager dequantize-and-compute, {threads} threads): {td:.2f} s"}


def run_block_reference(args, world, rank):
    if rank != 0:
        return 0
    from futudiffu_b200.dit import DiTConfig

    threads = _cpu_threads()
    full = block_flops(DiTConfig())
    for _ in range(args.warmup):
        dit_cpu_block_seconds("double", img_tokens=256)
    times = [dit_cpu_block_seconds("double") for _ in range(args.steps)]
    td = statistics.mean(times)
    val = full / td / 1e12
    cb = {"value": val, "unit": "TFLOPS", "cores": threads, "kind": "port",
          "sample": f"{len(times)} double-stream blocks at 512 text + 4096 image tokens through "
                    f"oracle.dit.double_block (torch-eager dequantize-and-compute, {threads} threads), "
                    f"mean {td:.2f} s"}
    print(json.dumps({
        "impl": "reference", "metric": BLOCK_METRIC, "value": val, "unit": "TFLOPS", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": td * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp8/int8",
        "data": "synthetic (random-init weights, N(0,1) activations)", "config": block_config(DiTConfig(), args.gpus),
        "cpu_baseline": cb,
        "e2e": {"value": val, "unit": "TFLOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)
    return 0


def block_config(cfg, gpus: int) -> dict:
    """The config-3 workload description, identical in both arms."""
    return {"workload": "config3_mmdit_block", "batch": 1, "hidden": cfg.hidden, "heads": cfg.heads,
            "tokens": f"{cfg.txt_tokens} text + {cfg.img_tokens} image", "mlp": "ratio 4, GELU-tanh",
            "linears": "fp8 e4m3, 1x128 activation / 128x128 weight fp32 scales",
            "attention": f"{cfg.qk_quant} {cfg.granularity.replace('_', '-')} QK (K mean-smoothed), "
                         f"{cfg.pv_quant} P and V",
            "l2": "block weights 226 MB fp8 > 126 MB L2; no explicit flush",
            "parallelism": f"replica per GPU x{gpus}"}


def run_block(args, world, rank, local):
    """benchmark config 3: one double-stream block forward (B 1, 512 + 4096 tokens),
    replicated per rank.  Each step is the block replayed as a captured CUDA graph."""
    from futudiffu_b200 import check_status
    from futudiffu_b200.dit import DiTConfig, DoubleStreamBlock, batch_freqs, image_freqs, text_freqs

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    cfg = DiTConfig()
    gen = torch.Generator(device=dev).manual_seed(0)
    blk = DoubleStreamBlock(cfg, gen, dev)
    g = torch.Generator().manual_seed(100 + rank)
    h_txt = torch.randn(1, cfg.txt_tokens, cfg.hidden, generator=g).to(torch.bfloat16).pin_memory()
    h_img = torch.randn(1, cfg.img_tokens, cfg.hidden, generator=g).to(torch.bfloat16).pin_memory()
    h_vec = torch.randn(1, cfg.hidden, generator=g).to(torch.bfloat16).pin_memory()
    d_txt, d_img, d_vec = (t.to(dev) for t in (h_txt, h_img, h_vec))
    f_txt, f_img = batch_freqs(text_freqs(cfg, dev), 1), batch_freqs(image_freqs(cfg, dev), 1)
    stream = torch.cuda.current_stream(dev)
    flops = block_flops(cfg)

    with torch.no_grad():
        for _ in range(args.warmup):
            blk(d_txt, d_img, d_vec, f_txt, f_img)
        torch.cuda.synchronize()
        check_status()
        rec = LaunchRecorder()
        rec.active = True
        n_rec = 3
        for _ in range(n_rec):
            blk(d_txt, d_img, d_vec, f_txt, f_img)
        rec.active = False
        torch.cuda.synchronize()
        gemm_work, gemm_ms, n_gemm = rec.summary("gemm")
        qkv_work, qkv_ms, n_qkv = rec.summary("gemm_qkv")
        attn_work, attn_ms, _ = rec.summary("attn")
        launches_per_step = rec.launches // n_rec
        rec.close()
        # capture the block (inputs stay at the static d_* addresses)
        side = torch.cuda.Stream(dev)
        side.wait_stream(stream)
        with torch.cuda.stream(side):
            for _ in range(2):
                blk(d_txt, d_img, d_vec, f_txt, f_img)
        stream.wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            o_txt, o_img = blk(d_txt, d_img, d_vec, f_txt, f_img)
        for _ in range(3):
            graph.replay()
        torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    with ClockSampler(dev.index if "CUDA_VISIBLE_DEVICES" not in os.environ else local) as clocks:
        for n, (e0, e1) in enumerate(ev):
            if args.profile and n == 0:
                torch.cuda.cudart().cudaProfilerStart()
            e0.record(stream)
            graph.replay()
            e1.record(stream)
            if args.profile and n == 0:
                torch.cuda.synchronize()
                torch.cuda.cudart().cudaProfilerStop()
        torch.cuda.synchronize()
    barrier(world)
    ms_local = statistics.mean(a.elapsed_time(b) for a, b in ev)
    ms = max_over_ranks(ms_local, world, dev)
    check_status()
    # end to end: pinned host activations + vec -> device -> block -> both outputs to host
    o_h = [torch.empty_like(o_txt, device="cpu").pin_memory(), torch.empty_like(o_img, device="cpu").pin_memory()]

    def e2e_step():
        d_txt.copy_(h_txt, non_blocking=True)
        d_img.copy_(h_img, non_blocking=True)
        d_vec.copy_(h_vec, non_blocking=True)
        graph.replay()
        o_h[0].copy_(o_txt, non_blocking=True)
        o_h[1].copy_(o_img, non_blocking=True)

    e2e_step()
    torch.cuda.synchronize()
    barrier(world)
    e2e_n = 10
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(e2e_n):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / e2e_n, world, dev)
    check_status()
    h2d = (h_txt.numel() + h_img.numel() + h_vec.numel()) * 2
    d2h = (o_txt.numel() + o_img.numel()) * 2
    if rank == 0:
        pk = peaks()
        peak = 2.0 * pk["bf16_tflops"]
        gemm_tf = gemm_work / (gemm_ms * 1e-3) / 1e12
        tf = flops / (ms * 1e-3) / 1e12
        print(json.dumps({
            "metric": BLOCK_METRIC, "value": tf * world, "unit": "TFLOPS", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "fp8/int8", "data": "synthetic (random-init weights, N(0,1) activations)",
            "config": block_config(cfg, world),
            "detail": {"block_tflop": flops / 1e12,
                       "linears": "the two streams' linears as grouped launches",
                       "attention": "fused RMSNorm/RoPE/quant prologue, then the tcgen05 attention kernel",
                       "time_share": {"gemm": (gemm_ms + qkv_ms) / n_rec / ms_local, "attention": attn_ms / n_rec / ms_local,
                                      "qkv_linear_fused_prologue": qkv_ms / n_rec / ms_local},
                       "attention_kernel_tops": attn_work / (attn_ms * 1e-3) / 1e12 if attn_ms else None,
                       "launch": f"each step replays the block's {launches_per_step} kernels as one CUDA graph"},
            "roofline": {"bound": "tensor", "achieved": gemm_tf, "peak": peak, "unit": "TFLOP/s",
                         "frac": gemm_tf / peak, "traffic": None,
                         "kernel": f"gemm_fp8_kernel (the {n_gemm // n_rec} GEMM launches of a block but the QKV linears with "
                                   "the fused prologue, flop-weighted, "
                                   "CUDA events per launch over three eager forwards)",
                         "peak_source": f"2 x {pk['source']} burst bf16 dense ({pk['bf16_tflops']} TF/s): "
                                        "fp8 dense rate is twice bf16"},
            "cpu_baseline": block_cpu_sample() if world == 1 else None,
            "e2e": {"value": flops / (e2e_ms * 1e-3) / 1e12 * world, "unit": "TFLOPS", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms,
                    "api": "futudiffu_b200.dit.DoubleStreamBlock captured as a CUDA graph (pinned host inputs "
                           "copied in, both stream outputs copied out)"},
            "gpu_launches": launches_per_step * args.steps,
            "clocks": clocks.summary(),
        }), flush=True)
    return 0


# ------------------------------------------------------------------ config 5: video DiT, Ulysses
VIDEO_METRIC = "video DiT denoise steps/s (14B-class, 40 blocks, 32760 video + 512 text tokens, Ulysses)"


_VIDEO_CPU_BLOCKS: dict = {}


def video_cpu_sample(tokens: int = 1024) -> dict:
    """One config-5 video block through the oracle on the host cores (CPU-built
    weights) with ``tokens`` video tokens and the 512 text tokens, extrapolated to
    the 40-block step over 32760 tokens by FLOPs."""
    from futudiffu_b200.dit import VideoDiTConfig, video_flops_per_step, video_freqs
    from oracle import dit as OD

    threads = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()
    torch.set_num_threads(threads)
    cfg = VideoDiTConfig()
    if "blk" not in _VIDEO_CPU_BLOCKS:
        _VIDEO_CPU_BLOCKS["blk"] = OD.random_video_block(cfg, seed=0)
    blk = _VIDEO_CPU_BLOCKS["blk"]
    cg = torch.Generator().manual_seed(3)
    D, F, T = cfg.hidden, cfg.ffn, cfg.txt_tokens
    x = torch.randn(1, tokens, D, generator=cg).to(torch.bfloat16)
    txt = torch.randn(1, T, D, generator=cg).to(torch.bfloat16)
    vec = torch.randn(1, D, generator=cg).to(torch.bfloat16)
    freqs = video_freqs(cfg, "cpu", 0, tokens).unsqueeze(0)
    t0 = time.perf_counter()
    OD.video_block(blk, x, vec, txt, freqs)
    dt = time.perf_counter() - t0
    L = tokens
    blk_flops = 2 * L * (4 * D * D + 2 * D * D + 2 * D * F) + 2 * T * 2 * D * D + 4 * L * L * D + 4 * L * T * D
    step_s = dt * video_flops_per_step(cfg) / blk_flops
    return {"value": 1.0 / step_s, "unit": "steps/s", "cores": threads, "kind": "port",
            "sample": f"one video block at {tokens} video + {T} text tokens through oracle.dit.video_block "
                      f"({dt:.1f} s, {threads} threads), extrapolated to the {cfg.n_blocks}-block step over "
                      f"{cfg.tokens} tokens by FLOP ratio ({step_s:.0f} s/step)"}


def run_video_reference(args, world, rank):
    if rank != 0:
        return 0
    vals, cb = [], None
    for i in range(args.warmup + args.steps):
        cb = video_cpu_sample()
        if i >= args.warmup:
            vals.append(cb["value"])
    val = statistics.mean(vals)
    print(json.dumps({
        "impl": "reference", "metric": VIDEO_METRIC, "value": val, "unit": "steps/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 / val, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "fp8/int8", "data": "synthetic",
        "config": {"workload": "config5_video_dit_ulysses"},
        "cpu_baseline": {**cb, "value": val},
        "e2e": {"value": val, "unit": "steps/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)
    return 0


class ExchangeRecorder:
    """CUDA events around every Ulysses all-to-all (``futudiffu_b200.ulysses``) while
    active: the exchange's share of a video step and the bytes this rank sends."""

    def __init__(self):
        from futudiffu_b200 import ulysses as U

        self.U = U
        self.orig = U.dist.all_to_all_single
        self.active = False
        self.events, self.bytes = [], 0
        U.dist.all_to_all_single = self._a2a

    class _Done:
        def wait(self):
            return True

    def _a2a(self, out, inp, *a, **kw):
        if not self.active:
            return self.orig(out, inp, *a, **kw)
        # run each exchange alone (an asynchronous one synchronously) between two events:
        # its own duration, not the part the pipelined schedule leaves exposed
        pipelined = kw.pop("async_op", False)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        r = self.orig(out, inp, *a, **kw)
        e1.record()
        self.events.append((e0, e1))
        self.bytes += inp.numel() * inp.element_size()
        return self._Done() if pipelined else r

    def summary(self):
        return sum(a.elapsed_time(b) for a, b in self.events), len(self.events), self.bytes

    def close(self):
        self.U.dist.all_to_all_single = self.orig


def video_sub_entry(dev, world: int, rank: int, local: int, steps: int = 3, warmup: int = 2) -> dict:
    """Config 5 inside the default line at N >= 2 GPUs: one denoise step of the
    14B-class video DiT with Ulysses sequence parallelism over all ranks (NCCL
    all-to-all around every self-attention), device-timed, max over ranks."""
    from futudiffu_b200 import check_status
    from futudiffu_b200.dit import VideoDiT, VideoDiTConfig, sigmas, video_flops_per_step

    cfg = VideoDiTConfig()
    model = VideoDiT(cfg, seed=0, device=dev, group=None)
    Ls = model.local_tokens
    g = torch.Generator().manual_seed(200)
    lat = torch.randn(1, cfg.tokens, cfg.patch_dim, generator=g).to(torch.bfloat16)
    txt = torch.randn(1, cfg.txt_tokens, cfg.hidden, generator=g).to(torch.bfloat16).to(dev)
    x = lat[:, rank * Ls:(rank + 1) * Ls].contiguous().to(dev)
    sig = sigmas(28)
    stream = torch.cuda.current_stream(dev)

    def step(i, x):
        t = torch.full((1,), sig[i % 28], device=dev)
        v = model(x, txt, t)
        return (x.float() + (sig[i % 28 + 1] - sig[i % 28]) * v.float()).to(x.dtype)

    for i in range(warmup):
        x = step(i, x)
    torch.cuda.synchronize()
    barrier(world)
    with ClockSampler(dev.index if "CUDA_VISIBLE_DEVICES" not in os.environ else local) as clocks:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for i in range(steps):
            x = step(i, x)
        e1.record(stream)
        torch.cuda.synchronize()
    barrier(world)
    ms_local = e0.elapsed_time(e1) / steps
    ms = max_over_ranks(ms_local, world, dev)
    # one more (untimed) step with CUDA events around every all-to-all
    xr = ExchangeRecorder()
    xr.active = True
    x = step(0, x)
    xr.active = False
    torch.cuda.synchronize()
    a2a_ms, n_a2a, a2a_bytes = xr.summary()
    xr.close()
    a2a_ms = max_over_ranks(a2a_ms, world, dev)
    # the same steps with the exchange pipelined by head groups (the smallest group
    # count > 1 that divides this rank's heads), for comparison with the default
    Hp = cfg.heads // world
    G = next((d for d in range(2, Hp + 1) if Hp % d == 0), None)
    ms_pipe = None
    if G is not None:
        model.head_groups = G
        x = step(0, x)
        torch.cuda.synchronize()
        barrier(world)
        e0.record(stream)
        for i in range(steps):
            x = step(i, x)
        e1.record(stream)
        torch.cuda.synchronize()
        barrier(world)
        ms_pipe = max_over_ranks(e0.elapsed_time(e1) / steps, world, dev)
        model.head_groups = 1
    check_status()
    del model
    torch.cuda.empty_cache()
    fl = video_flops_per_step(cfg)
    return {"metric": VIDEO_METRIC, "value": 1e3 / ms, "unit": "steps/s", "ms": ms, "steps": steps, "warmup": warmup,
            "parallelism": f"Ulysses sequence parallel x{world} (NCCL all_to_all_single around each self-attention)",
            "nccl_ranks": world,
            "all_to_all": {"calls_per_step": n_a2a, "ms_per_step": a2a_ms, "share_of_step": a2a_ms / ms,
                           "bytes_sent_per_rank": a2a_bytes, "gb_s_per_rank": a2a_bytes / (a2a_ms * 1e6) if a2a_ms else None,
                           "timed": "CUDA events around each all_to_all_single of one extra step, each run alone "
                                    "(not overlapped), max over ranks; Q, K, V cross as bf16, the attention output "
                                    "as 1x128 e4m3 codes + scales",
                           "pipelined": {"head_groups": G, "ms_step": ms_pipe,
                                         "note": "the same step with heads in G groups: every group's Q/K/V "
                                                 "exchange queued up front, groups attending alternately on two "
                                                 "streams while NCCL moves the next group's inputs and the last "
                                                 "group's output codes; the default step uses one exchange per "
                                                 "tensor (G = 1)"}},
            "model_tflops": fl / (ms * 1e-3) / 1e12, "tokens": cfg.tokens, "blocks": cfg.n_blocks,
            "clocks": clocks.summary()}


def run_video(args, world, rank, local):
    import torch.distributed as dist

    from futudiffu_b200 import check_status
    from futudiffu_b200.dit import VideoDiT, VideoDiTConfig, sigmas, video_flops_per_step

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    cfg = VideoDiTConfig()
    model = VideoDiT(cfg, seed=0, device=dev, group=None)
    Ls = model.local_tokens
    g = torch.Generator().manual_seed(200)  # the whole sample, sliced per rank
    lat = torch.randn(1, cfg.tokens, cfg.patch_dim, generator=g).to(torch.bfloat16)
    txt = torch.randn(1, cfg.txt_tokens, cfg.hidden, generator=g).to(torch.bfloat16).to(dev)
    x = lat[:, rank * Ls:(rank + 1) * Ls].contiguous().to(dev)
    sig = sigmas(28)
    stream = torch.cuda.current_stream(dev)

    def step(i, x):
        t = torch.full((1,), sig[i % 28], device=dev)
        v = model(x, txt, t)
        return (x.float() + (sig[i % 28 + 1] - sig[i % 28]) * v.float()).to(x.dtype)

    for i in range(args.warmup):
        x = step(i, x)
    torch.cuda.synchronize()
    check_status()
    rec = LaunchRecorder()
    barrier(world)
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev.index if "CUDA_VISIBLE_DEVICES" not in os.environ else local) as clocks:
        rec.active = True
        start.record(stream)
        for i in range(args.steps):
            x = step(i, x)
        end.record(stream)
        rec.active = False
        torch.cuda.synchronize()
    barrier(world)
    ms_local = start.elapsed_time(end) / args.steps
    ms = max_over_ranks(ms_local, world, dev)
    gemm_work, gemm_ms, _ = rec.summary("gemm")
    attn_work, attn_ms, _ = rec.summary("attn")
    launches = rec.launches
    rec.close()
    check_status()
    # ---------------- end to end: host latent shard -> device -> step -> host
    h_x = lat[:, rank * Ls:(rank + 1) * Ls].contiguous().pin_memory()
    h_out = torch.empty_like(h_x).pin_memory()
    step(0, h_x.to(dev, non_blocking=True))
    torch.cuda.synchronize()
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(2):
        h_out.copy_(step(i, h_x.to(dev, non_blocking=True)), non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / 2, world, dev)
    if rank == 0:
        pk = peaks()
        peak = 2.0 * pk["bf16_tflops_sustained"]
        gemm_tf = gemm_work / (gemm_ms * 1e-3) / 1e12
        fl = video_flops_per_step(cfg)
        print(json.dumps({
            "metric": VIDEO_METRIC, "value": 1e3 / ms, "unit": "steps/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "fp8/int8", "data": "synthetic (random-init weights, N(0,1) latents/text)",
            "config": {"workload": "config5_video_dit_ulysses", "tokens": cfg.tokens, "text_tokens": cfg.txt_tokens,
                       "hidden": cfg.hidden, "heads": cfg.heads, "ffn": cfg.ffn, "blocks": cfg.n_blocks,
                       "parallelism": f"Ulysses sequence parallel x{world} (NCCL all_to_all_single)",
                       "model_pflop_per_step": fl / 1e15, "model_tflops": fl / (ms * 1e-3) / 1e12,
                       "attention_kernel_tops_per_gpu": attn_work / (attn_ms * 1e-3) / 1e12 if attn_ms else None,
                       "time_share": {"gemm": gemm_ms / args.steps / ms_local,
                                      "attention": attn_ms / args.steps / ms_local},
                       "cross_attention": "bf16 torch SDPA (512 text keys, <1% of FLOPs)",
                       "l2": "weights 14 GB, activations >> L2"},
            "roofline": {"bound": "tensor", "achieved": gemm_tf, "peak": peak, "unit": "TFLOP/s",
                         "frac": gemm_tf / peak, "traffic": None, "kernel": "gemm_fp8_kernel (flop-weighted, rank 0)",
                         "peak_source": f"2 x {pk['source']} sustained bf16 dense ({pk['bf16_tflops_sustained']} TF/s)"},
            "cpu_baseline": video_cpu_sample() if world == 1 else None,
            "e2e": {"value": 1e3 / e2e_ms, "unit": "steps/s", "h2d_bytes_per_step": h_x.numel() * 2 * world,
                    "d2h_bytes_per_step": h_x.numel() * 2 * world, "ms_per_step": e2e_ms,
                    "api": "futudiffu_b200.dit.VideoDiT"},
            "gpu_launches": launches, "clocks": clocks.summary(),
        }), flush=True)
    return 0


# config 1, the reference benchmark's Z-Image QKV / FFN-out shapes, and the config-4
# MLP-in linear at one sample (4608 tokens) and at the batch of 8
GEMM_SHAPES = {"config1": (2048, 3072, 3072), "ref_qkv": (8576, 11520, 3840), "ref_w2": (8576, 3840, 10240),
               "dit_mlp_in": (4608, 12288, 3072), "dit_mlp_in_b8": (36864, 12288, 3072),
               "dit_qkv": (4608, 9216, 3072), "dit_qkv_b8": (36864, 9216, 3072)}


PACKED_METRIC = "packed multi-image forward tokens/s (Z-Image-class blocks, 3840 hidden, 30 heads, 4288-token bin)"


_PACKED_CPU_BLOCKS: dict = {}


def packed_cpu_sample(tokens: int = 1024, layers: int = 30) -> dict:
    """One Z-Image-class JointTransformerBlock through the oracle on the host cores
    (CPU-built weights) on a one-image sequence of ``tokens`` tokens, extrapolated
    to the packed 30-layer forward of a 4288-token bin by FLOPs."""
    from futudiffu_b200 import transformer as T
    from futudiffu_b200.bin_packer import REFERENCE_TOTAL_LEN
    from futudiffu_b200.block_mask import build_block_mask
    from oracle import transformer as OT

    threads = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()
    torch.set_num_threads(threads)
    dim, heads, hidden = 3840, 30, 10240
    if "blk" not in _PACKED_CPU_BLOCKS:
        _PACKED_CPU_BLOCKS["blk"] = OT.random_joint_block(dim, heads, hidden, seed=0)
    blk = _PACKED_CPU_BLOCKS["blk"]
    cg = torch.Generator().manual_seed(2)
    cap = 64
    grid = (tokens - cap) // 16
    _, info = T.build_packed_sequence([torch.zeros(1, cap, 1)], [torch.zeros(1, grid * 16, 1)], [(grid, 16)],
                                      [cap], 32, torch.zeros(1), torch.zeros(1))
    rope = T.build_packed_rope(info, device="cpu")
    n = info.total_len
    x = torch.randn(1, n, dim, generator=cg).to(torch.bfloat16)
    scales = tuple((0.1 * torch.randn(1, dim, generator=cg)).to(torch.bfloat16) for _ in range(4))
    mask = build_block_mask([n], device="cpu")
    t0 = time.perf_counter()
    OT.block_forward(blk, x, rope, scales, mask)
    dt = time.perf_counter() - t0
    lin = 2 * (3 * dim * dim + dim * dim + 2 * hidden * dim + hidden * dim)
    sample_flops = lin * n + 4 * n * n * dim
    full_flops = layers * (lin * REFERENCE_TOTAL_LEN + 4 * 0.63 * REFERENCE_TOTAL_LEN ** 2 * dim)
    step_s = dt * full_flops / sample_flops
    return {"value": REFERENCE_TOTAL_LEN / step_s, "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"one JointTransformerBlock (3840 hidden, 30 heads, FFN 10240) on {n} tokens through "
                      f"oracle.transformer.block_forward ({dt:.1f} s, {threads} threads), extrapolated to the "
                      f"{layers}-layer forward of a {REFERENCE_TOTAL_LEN}-token bin (mask density 0.63) by FLOP "
                      f"ratio ({step_s:.0f} s/forward)"}


def run_packed_reference(args, world, rank):
    if rank != 0:
        return 0
    vals, cb = [], None
    for i in range(args.warmup + args.steps):
        cb = packed_cpu_sample(layers=args.layers)
        if i >= args.warmup:
            vals.append(cb["value"])
    val = statistics.mean(vals)
    print(json.dumps({
        "impl": "reference", "metric": PACKED_METRIC, "value": val, "unit": "tokens/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 4288 / val * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp8/int8", "data": "synthetic",
        "config": {"workload": "packed_zimage_trunk", "layers": args.layers, "hidden": 3840, "heads": 30},
        "cpu_baseline": {**cb, "value": val},
        "e2e": {"value": val, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)
    return 0


def run_packed(args, world, rank, local):
    """The reference's production shape: one bin of the bin packer (two images of
    different resolution with their captions, padded to REFERENCE_TOTAL_LEN = 4288
    tokens) through ``--layers`` JointTransformerBlocks with per-image adaLN and
    the block-diagonal mask; one step = one forward of the layer stack."""
    from futudiffu_b200 import check_status
    from futudiffu_b200.bin_packer import REFERENCE_TOTAL_LEN, BinPackScheduler
    from futudiffu_b200.block_mask import build_block_mask_from_packing_info
    from futudiffu_b200.forward_packed import _pad_plan_to_fixed_len
    from futudiffu_b200.transformer import PackedTrunk, build_packed_rope, build_packed_sequence, row_ranges

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dim, heads = 3840, 30
    plan = [{"width": 1024, "height": 768, "cap_tokens": 50}, {"width": 512, "height": 512, "cap_tokens": 50}]
    bins = BinPackScheduler().pack_generation_plan(plan)
    assert len(bins) == 1
    g = torch.Generator().manual_seed(7 + rank)
    caps = [torch.randn(1, it["cap_tokens"], dim, generator=g).to(torch.bfloat16) for it in bins[0]]
    grids = [(it["height"] // 16, it["width"] // 16) for it in bins[0]]
    imgs = [torch.randn(1, h * w, dim, generator=g).to(torch.bfloat16) for h, w in grids]
    pad = torch.zeros(dim, dtype=torch.bfloat16)
    packed, info = build_packed_sequence(caps, imgs, grids, [it["cap_tokens"] for it in bins[0]], 32, pad, pad)
    natural = info.total_len
    info, rope = _pad_plan_to_fixed_len(info, build_packed_rope(info, device="cpu"), REFERENCE_TOTAL_LEN)
    host_x = torch.cat([packed, packed.new_zeros(1, REFERENCE_TOTAL_LEN - natural, dim)], 1).contiguous()
    x0 = host_x.to(dev)
    rope = rope.to(dev)
    mask = build_block_mask_from_packing_info(info, device=dev)
    mask_density = float(mask.float().mean())
    ranges = row_ranges(info.document_id, n_params=info.n_images, device=dev)
    adaln = torch.randn(info.n_images, 256, generator=g).to(torch.bfloat16).to(dev)
    trunk = PackedTrunk(args.layers, dim, heads, seed=0, device=dev)
    stream = torch.cuda.current_stream(dev)

    def step():
        return trunk(x0, adaln, ranges, mask, rope)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    check_status()
    rec = LaunchRecorder()
    barrier(world)
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev.index if "CUDA_VISIBLE_DEVICES" not in os.environ else local) as clocks:
        rec.active = True
        start.record(stream)
        for n in range(args.steps):
            if args.profile and n == 0:
                torch.cuda.cudart().cudaProfilerStart()
            step()
            if args.profile and n == 0:
                torch.cuda.synchronize()
                torch.cuda.cudart().cudaProfilerStop()
        end.record(stream)
        rec.active = False
        torch.cuda.synchronize()
    barrier(world)
    ms_local = start.elapsed_time(end) / args.steps
    ms = max_over_ranks(ms_local, world, dev)
    gemm_work, gemm_ms, n_gemm = rec.summary("gemm")
    attn_work, attn_ms, n_attn = rec.summary("attn")
    launches = rec.launches
    rec.close()
    check_status()

    # end to end: the packed bin from pinned host memory, the output back to the host
    h_x = host_x.pin_memory()
    h_out = torch.empty_like(host_x).pin_memory()

    def e2e_step():
        xi = h_x.to(dev, non_blocking=True)
        h_out.copy_(trunk(xi, adaln, ranges, mask, rope), non_blocking=True)

    e2e_step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(3):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / 3, world, dev)
    check_status()
    if rank == 0:
        pk = peaks()
        peak = 2.0 * pk["bf16_tflops_sustained"]
        gemm_tf = gemm_work / (gemm_ms * 1e-3) / 1e12
        toks = REFERENCE_TOTAL_LEN * world
        line = {
            "metric": PACKED_METRIC, "value": toks / (ms * 1e-3), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "fp8/int8",
            "data": "synthetic (random-init weights, N(0,1) captions/patches)",
            "config": {"workload": "packed_zimage_trunk", "layers": args.layers, "hidden": dim, "heads": heads,
                       "ffn_hidden": 10240, "bin": [(it["width"], it["height"], it["cap_tokens"]) for it in bins[0]],
                       "tokens": f"{natural} packed + {REFERENCE_TOTAL_LEN - natural} padding",
                       "adaln": "per image (row ranges)", "attention": "int8 per-token QK, bf16 PV, block mask",
                       "l2": "weights and activations exceed the 126 MB L2; no explicit flush",
                       "parallelism": f"one bin per GPU x{world}, no collective",
                       # the mask skips tiles that mix images: count the computed tiles only
                       "attention_mask_density": mask_density,
                       "attention_kernel_tops": (attn_work * mask_density / (attn_ms * 1e-3) / 1e12
                                                 if attn_ms else None),
                       "time_share": {"gemm": gemm_ms / args.steps / ms_local,
                                      "attention": attn_ms / args.steps / ms_local}},
            "roofline": {"bound": "tensor", "achieved": gemm_tf, "peak": peak, "unit": "TFLOP/s",
                         "frac": gemm_tf / peak, "traffic": None,
                         "kernel": f"gemm_fp8_kernel ({n_gemm // max(1, args.steps)} launches per step, flop-weighted)",
                         "peak_source": f"2 x {pk['source']} sustained bf16 dense ({pk['bf16_tflops_sustained']} TF/s)"},
            "cpu_baseline": packed_cpu_sample(layers=args.layers) if world == 1 else None,
            "e2e": {"value": toks / (e2e_ms * 1e-3), "unit": "tokens/s",
                    "h2d_bytes_per_step": host_x.numel() * 2 * world, "d2h_bytes_per_step": host_x.numel() * 2 * world,
                    "ms_per_step": e2e_ms, "api": "futudiffu_b200.transformer.PackedTrunk"},
            "gpu_launches": launches,
            "clocks": clocks.summary(),
        }
        print(json.dumps(line), flush=True)
    return 0


def run_gemm(args, world, rank, local):
    """FP8 block-GEMM TFLOPS (benchmark config 1, or the reference's Z-Image shapes)."""
    from futudiffu_b200 import check_status

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    M, N, K = GEMM_SHAPES[args.gemm_shape]
    with ClockSampler(local) as clocks:
        times = time_gemm(dev, args.gemm_shape, args.steps, args.warmup, args.gemm_epilogue)
    ms = max_over_ranks(statistics.mean(times), world, dev)
    check_status()
    flops = 2.0 * M * N * K
    pk = peaks()
    peak = 2.0 * pk["bf16_tflops"]
    tf = flops / (ms * 1e-3) / 1e12
    if rank == 0:
        print(json.dumps({
            "metric": "FP8 block-GEMM TFLOPS", "value": tf * world, "unit": "TFLOPS", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "fp8 e4m3 (1x128 / 128x128 f32 scales)",
            "data": "synthetic",
            "config": {"workload": f"gemm_{args.gemm_shape}", "M": M, "N": N, "K": K, "l2": "flushed",
                       "epilogue": {"gelu": "GELU(tanh) + 1x128 e4m3 requant",
                                    "qkv": "P3 + INT8 per-block Q codes, bf16 K / V, K / V column statistics"}.get(
                                        args.gemm_epilogue, "bf16")},
            "roofline": {"bound": "tensor", "achieved": tf, "peak": peak, "unit": "TFLOP/s",
                         "frac": tf / peak, "traffic": GEMM_TRAFFIC_BYTES.get(args.gemm_shape),
                         "peak_source": f"2 x {pk['source']} bf16 dense: fp8 dense rate is twice bf16"},
            "gpu_launches": args.steps, "clocks": clocks.summary(),
        }), flush=True)
    return 0


def run_tmem_probe(args, world, rank, local):
    """TMEM -> register load throughput (fd_probe_tmem_ld): bytes per clock per SM
    for load widths, loads per wait and warp counts, pure loads and with the FP8
    GEMM's promotion arithmetic.  One JSON line with the table (rank 0)."""
    from futudiffu_b200 import _lib as L
    from futudiffu_b200 import check_status

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    nsm = torch.cuda.get_device_properties(dev).multi_processor_count
    cycles = torch.zeros(nsm * 12, dtype=torch.int64, device=dev)
    sink = torch.zeros(1, dtype=torch.float32, device=dev)
    iters = 2048
    rows = []
    cases = [(w, l, n, 0) for (w, l) in ((16, 1), (16, 2), (16, 4), (32, 1), (32, 2), (32, 4), (64, 1), (64, 2))
             for n in (4, 8, 12)]
    cases += [(w, l, n, 1) for (w, l) in ((16, 1), (16, 2), (16, 4), (32, 1), (32, 2), (64, 1)) for n in (4, 8)]
    with ClockSampler(local) as clocks:
        for w, l, n, f in cases:
            for rep in range(2):  # first launch warms up
                cycles.zero_()
                L.call("fd_probe_tmem_ld", w, l, n, f, iters, L.ptr(cycles), L.ptr(sink), L.stream_ptr(dev))
                torch.cuda.synchronize()
            cyc = cycles.view(nsm, 12)[:, :n].double()
            per_sm = cyc.max(dim=1).values  # the slowest warp of each SM
            bytes_sm = n * 32 * 128 * 4 * iters
            rows.append({"width": w, "per_wait": l, "warps": n, "fma": bool(f),
                         "bytes_per_clk_sm": bytes_sm / per_sm.median().item(),
                         "cycles_per_128col_round": per_sm.median().item() / iters})
    check_status()
    if rank == 0:
        best = max(rows, key=lambda r: r["bytes_per_clk_sm"])
        print(json.dumps({"metric": "TMEM load throughput (B/clk/SM)", "value": best["bytes_per_clk_sm"],
                          "unit": "B/clk/SM", "n_gpus": 1, "higher_is_better": True,
                          "config": {"workload": "tmem_probe", "iters": iters,
                                     "need": "FP8 GEMM promotion at the full MMA rate: 256 B/clk/SM"},
                          "rows": rows, "clocks": clocks.summary()}), flush=True)
    return 0


def run_attn_bwd(args, world, rank, local):
    """Attention backward at the config-2 shape (B 2, H 24, N 4096, head dim 128):
    one `sage_attn_backward` call per step (six launches: the forward's Q/K quantisation redone,
    the Delta pre-pass, the tcgen05 dK/dV and dQ kernels), INT8 per-token QK as
    configured by default.  Inputs (q, k, v, dO: 4 x 100 MB) exceed L2.  value =
    TFLOP/s counted over the five products of the reference's formulation
    (S, dP, dV, dK, dQ: 5 x 2 x B x H x N^2 x 128)."""
    from futudiffu_b200 import check_status
    from futudiffu_b200 import sage_attention as SA

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    B, H, N = 2, 24, 4096
    g = torch.Generator(device=dev).manual_seed(1234 + rank)
    q, k, v, do = (torch.randn(B, H, N, 128, device=dev, generator=g).to(torch.bfloat16) for _ in range(4))
    sm = 128 ** -0.5
    SA.configure_sage(smooth_k=True, qk_quant="int8", pv_quant="bf16", qk_granularity="per_token")
    out, lse = SA.sage_attn_forward_with_lse(q, k, v, sm)
    for _ in range(args.warmup):
        SA.sage_attn_backward(q, k, v, out, lse, do, sm)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    torch.cuda.synchronize()
    with ClockSampler(local) as clocks:
        for e0, e1 in ev:
            e0.record()
            SA.sage_attn_backward(q, k, v, out, lse, do, sm)
            e1.record()
        torch.cuda.synchronize()
    ms = max_over_ranks(statistics.mean(a.elapsed_time(b) for a, b in ev), world, dev)
    check_status()
    flops = 5 * 2.0 * B * H * N * N * 128
    tf = flops / (ms * 1e-3) / 1e12
    pk = peaks()
    peak = pk["bf16_tflops"]
    if rank == 0:
        print(json.dumps({
            "metric": "SageAttn backward TFLOPS (5 products)", "value": tf * world, "unit": "TFLOPS",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "int8 QK recompute, bf16 dP / dV / dK / dQ operands, fp32 accumulation", "data": "synthetic",
            "config": {"workload": "attn_bwd_config2", "B": B, "H": H, "N": N, "head_dim": 128,
                       "qk": "int8 per-token", "l2": "inputs larger than L2"},
            "roofline": {"bound": "tensor", "achieved": tf, "peak": peak, "unit": "TFLOP/s", "frac": tf / peak,
                         "traffic": None, "peak_source": f"{pk['source']} bf16 dense (burst)"},
            "gpu_launches": 6 * args.steps, "clocks": clocks.summary(),
        }), flush=True)
    return 0


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None, help="timed steps (default: 10 dit, 50 otherwise)")
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["dit", "video", "attention", "attn_bwd", "gemm", "packed", "block",
                                           "tmem_probe"],
                    default="dit",
                    help="dit = benchmark config 4 (headline); video = config 5 (Ulysses); "
                         "block = config 3 (one double-stream block); "
                         "attention = config 2; gemm = config 1; packed = the reference's packed "
                         "4288-token bin through Z-Image-class JointTransformerBlocks")
    ap.add_argument("--gemm-shape", choices=sorted(GEMM_SHAPES), default="config1")
    ap.add_argument("--gemm-epilogue", choices=["bf16", "gelu", "qkv"], default="bf16",
                    help="gemm: bf16 output, the GELU(tanh) + 1x128 requant epilogue, or the QKV "
                         "linear's fused P3 + Q-quantisation epilogue (--gemm-shape dit_qkv*)")
    ap.add_argument("--layers", type=int, default=30, help="packed: JointTransformerBlocks in the stack")
    ap.add_argument("--no-sub", action="store_true",
                    help="dit: skip the config-1 GEMM / config-2 attention sub-measurements")
    ap.add_argument("--profile", action="store_true",
                    help="dit, block, packed: bracket the first timed step with cudaProfilerStart/Stop "
                         "(for ncu --profile-from-start off); timing of that run is not a result")
    args = ap.parse_args(argv)
    args.warmup = max(3, args.warmup)
    if args.steps is None:
        args.steps = {"dit": 10, "video": 3, "packed": 10}.get(args.workload, 50)
    world, rank, local = dist_setup()
    try:
        if args.workload == "dit":
            if args.impl == "reference":
                return run_dit_reference(args, world, rank)
            return run_dit(args, world, rank, local)
        if args.workload == "video":
            if args.impl == "reference":
                return run_video_reference(args, world, rank)
            return run_video(args, world, rank, local)
        if args.workload == "block":
            if args.impl == "reference":
                return run_block_reference(args, world, rank)
            return run_block(args, world, rank, local)
        if args.workload == "packed":
            if args.impl == "reference":
                return run_packed_reference(args, world, rank)
            return run_packed(args, world, rank, local)
        if args.workload == "tmem_probe":
            return run_tmem_probe(args, world, rank, local)
        if args.workload == "attn_bwd":
            return run_attn_bwd(args, world, rank, local)
        if args.impl == "reference":
            return run_reference(args, world, rank)
        if args.workload == "gemm":
            return run_gemm(args, world, rank, local)
        return run_ours(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    sys.exit(main())
