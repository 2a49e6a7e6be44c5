"""SageAttention API, B200 edition: drop-in for ``futudiffu.sage_attention``.

Public names, signatures, config globals, assertions, output layouts and the
``futudiffu::sage_attn`` / ``futudiffu::sage_attn_masked`` custom ops follow
src/futudiffu/sage_attention.py.  Each call runs two sm_100a kernels:

1. the quantisation prologue (``fd_attn_quant``): K mean-smoothing
   (``_smooth_k``, :63-71), Q/K quantisation to INT8 (truncating) or e4m3 with
   per-token or per-block scales, and optional e4m3 V with per-channel scales;
2. the tcgen05 attention kernel (``fd_sage_attn_fwd``): QK^T on the INT8 or
   FP8 tensor-core path, exp2 online softmax, PV on bf16 or e4m3, LSE.

Dispatch mirrors the reference exactly (which kernel each entry point uses
for each ``configure_sage`` setting) with one addition: ``qk_granularity``.
``"per_token"`` (default) is the reference's quantisation; ``"per_block"``
selects per-128-row Q / per-64-row K scales and honours ``pv_quant`` in every
entry point (the INT8-QK + FP8-PV combination of the B200 headline config).
"""

from __future__ import annotations

import ctypes
import math

import torch
from torch import Tensor

from . import _lib as L

_LOG2E = math.log2(math.e)

_SAGE_SMOOTH_K = True
_SAGE_QK_QUANT = "fp8"
_SAGE_PV_QUANT = "bf16"
_SAGE_QK_GRAN = "per_token"


def configure_sage(
    *,
    smooth_k: bool = True,
    qk_quant: str = "fp8",
    pv_quant: str = "bf16",
    qk_granularity: str = "per_token",
) -> None:
    """Select the SageAttention variant (reference sage_attention.py:37-60).

    qk_granularity: "per_token" (reference) or "per_block" (Q per 128 rows,
    K per 64 rows; also enables fp8 PV together with int8 QK).
    """
    global _SAGE_SMOOTH_K, _SAGE_QK_QUANT, _SAGE_PV_QUANT, _SAGE_QK_GRAN
    if qk_quant not in ("fp8", "int8"):
        raise ValueError(f"Unknown qk_quant: {qk_quant!r}")
    if pv_quant not in ("bf16", "fp8"):
        raise ValueError(f"Unknown pv_quant: {pv_quant!r}")
    if qk_granularity not in ("per_token", "per_block"):
        raise ValueError(f"Unknown qk_granularity: {qk_granularity!r}")
    _SAGE_SMOOTH_K = smooth_k
    _SAGE_QK_QUANT = qk_quant
    _SAGE_PV_QUANT = pv_quant
    _SAGE_QK_GRAN = qk_granularity


def get_sage_config() -> dict:
    return {
        "smooth_k": _SAGE_SMOOTH_K,
        "qk_quant": _SAGE_QK_QUANT,
        "pv_quant": _SAGE_PV_QUANT,
        "qk_granularity": _SAGE_QK_GRAN,
    }


def _smooth_k(k: Tensor) -> Tensor:
    """k - k.mean(dim=2, keepdim=True) in k's dtype (reference :63-71).

    Kept for API parity; the attention entry points fuse this into the
    quantisation prologue kernel instead of calling it.
    """
    return k - k.mean(dim=2, keepdim=True)


def _check_sm_capability() -> tuple[int, int]:
    if not torch.cuda.is_available():
        raise RuntimeError("SageAttention requires CUDA")
    cap = torch.cuda.get_device_capability()
    if cap < (10, 0):
        raise RuntimeError(f"futudiffu_b200 SageAttention requires SM 10.0 (B200), got SM {cap[0]}.{cap[1]}")
    return cap


def _desc_stride(N: int, gran: int, rows: int) -> int:
    return ((N + 127) // 128) * 128 if gran == L.GRAN_TOKEN else (N + rows - 1) // rows


def quantize_qkv(
    q: Tensor, k: Tensor, v: Tensor, sm_scale: float, *, smooth_k: bool, qk_quant: str,
    granularity: str, pv_quant: str,
) -> dict:
    """Run the quantisation prologue on (BH, N, 128) bf16 Q/K/V; returns codes and scales.

    Layouts: codes (BH, N, 128); per-token descales (BH, round_up(N, 128)),
    per-block descales (BH, ceil(N/128)) for Q and (BH, ceil(N/64)) for K;
    v_desc (BH, 128) for pv_quant "fp8" (per channel), (BH, ceil(N/64), 128) for
    "fp8_tile" (the reference's per-64-row-tile V scales); k_mean (BH, 128)
    (bf16-rounded smoothing mean as f32).
    """
    BH, N, D = q.shape
    dev = q.device
    qk = L.QK_INT8 if qk_quant == "int8" else L.QK_FP8
    gran = L.GRAN_TOKEN if granularity == "per_token" else L.GRAN_BLOCK
    pv = {"fp8": L.PV_FP8, "fp8_tile": L.PV_FP8_TILE}.get(pv_quant, L.PV_BF16)
    code_dt = torch.int8 if qk == L.QK_INT8 else torch.float8_e4m3fn
    q_codes = torch.empty(BH, N, D, dtype=code_dt, device=dev)
    k_codes = torch.empty(BH, N, D, dtype=code_dt, device=dev)
    q_desc = torch.empty(BH, _desc_stride(N, gran, 128), dtype=torch.float32, device=dev)
    k_desc = torch.empty(BH, _desc_stride(N, gran, 64), dtype=torch.float32, device=dev)
    k_mean = torch.empty(BH, D, dtype=torch.float32, device=dev)
    v_codes = v_desc = None
    if pv != L.PV_BF16:
        v_codes = torch.empty(BH, N, D, dtype=torch.float8_e4m3fn, device=dev)
        # per-channel: one scale per (bh, d); per tile: one per (bh, 64-row tile, d)
        v_desc = torch.empty(BH, D, dtype=torch.float32, device=dev) if pv == L.PV_FP8 else \
            torch.empty(BH, (N + 63) // 64, D, dtype=torch.float32, device=dev)
    ws = torch.empty(int(L.lib().fd_attn_quant_workspace_floats(BH, N)), dtype=torch.float32, device=dev)
    pv_prologue = L.PV_FP8 if pv == L.PV_FP8 else L.PV_BF16
    L.call(
        "fd_attn_quant", L.ptr(q), L.ptr(k), L.ptr(v), BH, N, int(bool(smooth_k)), qk, gran, gran, pv_prologue,
        float(sm_scale * _LOG2E), L.ptr(q_codes), L.ptr(q_desc), L.ptr(k_codes), L.ptr(k_desc),
        L.ptr(v_codes) if pv == L.PV_FP8 else None, L.ptr(v_desc) if pv == L.PV_FP8 else None,
        L.ptr(k_mean), L.ptr(ws), L.stream_ptr(dev),
    )
    if pv == L.PV_FP8_TILE:
        L.call("fd_attn_quant_v_tile", L.ptr(v), BH, N, L.ptr(v_codes), L.ptr(v_desc), L.stream_ptr(dev))
    return {
        "q_codes": q_codes, "q_desc": q_desc, "k_codes": k_codes, "k_desc": k_desc,
        "v_codes": v_codes, "v_desc": v_desc, "k_mean": k_mean,
        "qk": qk, "gran": gran, "pv": pv,
    }


def _normalize_mask(block_mask: Tensor | None, N: int) -> tuple[Tensor | None, int]:
    if block_mask is None:
        return None, 0
    bm = block_mask.contiguous()
    if bm.dtype != torch.uint8:
        bm = bm.to(torch.uint8)
    nq, nk = (N + 127) // 128, (N + 63) // 64
    if bm.ndim == 2:
        stride = 0
    elif bm.ndim == 3:
        stride = bm.shape[1] * bm.shape[2]
    else:
        raise ValueError(f"block_mask must be 2D or 3D, got {bm.ndim}D")
    if tuple(bm.shape[-2:]) != (nq, nk):
        raise ValueError(f"block_mask must have trailing shape ({nq}, {nk}), got {tuple(bm.shape)}")
    return bm, stride


def _attn_forward(
    q: Tensor, k: Tensor, v: Tensor, sm_scale: float | None, *, block_mask: Tensor | None,
    qk_quant: str, pv_quant: str, granularity: str, want_lse: bool, out_bnhd: bool = False,
) -> tuple[Tensor, Tensor | None]:
    """(B, H, N, 128) bf16 -> out (B, H, N, 128), or (B, N, H * 128) when ``out_bnhd``."""
    B, H, N, D = q.shape
    assert D == 128, f"SageAttention currently requires head_dim=128, got {D}"
    assert q.dtype == torch.bfloat16, f"Expected BF16 input, got {q.dtype}"
    L.require_cuda(q, k, v)
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(D)
    BH = B * H
    qf = q.reshape(BH, N, D).contiguous()
    kf = k.reshape(BH, N, D).contiguous()
    vf = v.reshape(BH, N, D).contiguous()
    bm, bm_stride = _normalize_mask(block_mask, N)
    qz = quantize_qkv(qf, kf, vf, sm_scale, smooth_k=_SAGE_SMOOTH_K, qk_quant=qk_quant,
                      granularity=granularity, pv_quant=pv_quant)
    out = torch.empty(B, N, H * D, dtype=q.dtype, device=q.device) if out_bnhd else torch.empty_like(qf)
    lse = torch.empty(BH, N, dtype=torch.float32, device=q.device) if want_lse else None
    vsrc = qz["v_codes"] if qz["pv"] != L.PV_BF16 else vf
    common = (L.ptr(qz["q_codes"]), L.ptr(qz["q_desc"]), L.ptr(qz["k_codes"]), L.ptr(qz["k_desc"]),
              L.ptr(vsrc), L.ptr(qz["v_desc"]), L.ptr(bm), bm_stride, L.ptr(out), L.ptr(lse), BH, N)
    kinds = (qz["qk"], qz["gran"], qz["gran"], qz["pv"], L.stream_ptr(q.device))
    if out_bnhd:
        L.call("fd_sage_attn_fwd_bnhd", *common, H, *kinds)
        return out, lse
    L.call("fd_sage_attn_fwd", *common, *kinds)
    return out.reshape(B, H, N, D), lse


def _freqs_rows(freqs: Tensor, B: int, S: int) -> Tensor:
    """(B, S, [1,] 64, 2, 2) RoPE rotations as contiguous fp32 rows."""
    if freqs.ndim == 6:
        assert freqs.shape[2] == 1
        freqs = freqs.squeeze(2)
    return freqs.reshape(B * S, 64, 2, 2).to(torch.float32).contiguous()


def fused_prologue_ok(stream_lengths: list[int]) -> bool:
    """Streams laid out back to back qualify for the fused P3 + prologue when every
    stream but the last holds a multiple of 128 rows (blocks never straddle)."""
    return all(n % 128 == 0 for n in stream_lengths[:-1])


def quantize_qkv_streams(
    streams: list[tuple], H: int, N: int, sm_scale: float | None, *, smooth_k: bool, qk_quant: str,
    granularity: str, pv_quant: str,
) -> dict:
    """P3 (per-head Q/K RMSNorm + RoPE) fused with the attention prologue, for
    attention inputs straight from the QKV linear(s).  ``streams``: one
    (qkv (B, S, 3 H 128) bf16, q_norm_w, k_norm_w, freqs (B, S, [1,] 64, 2, 2), s_off,
    eps) per stream of a joint attention, rows [s_off, s_off + S) of the N joint
    rows (see fused_prologue_ok).  Returns quantize_qkv's dict plus the bf16 K and
    V ("k", "v", (B H, N, 128)); codes and scales equal fused_qkv_postprocess /
    qkv_postprocess_into followed by quantize_qkv."""
    qkv0 = streams[0][0]
    B, dev = qkv0.shape[0], qkv0.device
    BH = B * H
    D = 128
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(D)
    qk = L.QK_INT8 if qk_quant == "int8" else L.QK_FP8
    gran = L.GRAN_TOKEN if granularity == "per_token" else L.GRAN_BLOCK
    pv = L.PV_FP8 if pv_quant == "fp8" else L.PV_BF16
    code_dt = torch.int8 if qk == L.QK_INT8 else torch.float8_e4m3fn
    q_codes = torch.empty(BH, N, D, dtype=code_dt, device=dev)
    q_desc = torch.empty(BH, _desc_stride(N, gran, 128), dtype=torch.float32, device=dev)
    k = torch.empty(BH, N, D, dtype=torch.bfloat16, device=dev)
    v = torch.empty(BH, N, D, dtype=torch.bfloat16, device=dev)
    ws = torch.empty(int(L.lib().fd_qkv_quant_workspace_floats(BH, N)), dtype=torch.float32, device=dev)
    stream_ptr = L.stream_ptr(dev)
    for qkv, qw, kw, freqs, s_off, eps in streams:
        Bq, S, C = qkv.shape
        assert Bq == B and C == 3 * H * D and qkv.dtype == torch.bfloat16 and qkv.is_contiguous()
        fr = _freqs_rows(freqs, B, S)
        # keep the fp32 copies referenced until the launch (a temporary freed inside
        # the argument list could hand its memory to the next one)
        qw32, kw32 = qw.float().contiguous(), kw.float().contiguous()
        L.call("fd_qkv_postprocess_quant", L.ptr(qkv), L.ptr(qw32), L.ptr(kw32),
               L.ptr(fr), B, S, H, float(eps), N, s_off, qk, gran, pv, float(sm_scale * _LOG2E), L.ptr(q_codes),
               L.ptr(q_desc), L.ptr(k), L.ptr(v), L.ptr(ws), stream_ptr)
    k_codes = torch.empty(BH, N, D, dtype=code_dt, device=dev)
    k_desc = torch.empty(BH, _desc_stride(N, gran, 64), dtype=torch.float32, device=dev)
    k_mean = torch.empty(BH, D, dtype=torch.float32, device=dev)
    v_codes = torch.empty(BH, N, D, dtype=torch.float8_e4m3fn, device=dev) if pv == L.PV_FP8 else None
    v_desc = torch.empty(BH, D, dtype=torch.float32, device=dev) if pv == L.PV_FP8 else None
    L.call("fd_attn_quant_kv", L.ptr(k), L.ptr(v), BH, N, int(bool(smooth_k)), qk, gran, pv, L.ptr(k_codes),
           L.ptr(k_desc), L.ptr(v_codes), L.ptr(v_desc), L.ptr(k_mean), L.ptr(ws), stream_ptr)
    return {
        "q_codes": q_codes, "q_desc": q_desc, "k_codes": k_codes, "k_desc": k_desc,
        "v_codes": v_codes, "v_desc": v_desc, "k_mean": k_mean, "qk": qk, "gran": gran, "pv": pv,
        "k": k, "v": v, "B": B, "H": H, "N": N,
    }


def linear_prologue_ok(stream_lengths: list[int], H: int) -> bool:
    """Streams qualify for the QKV linear fused with P3 and the prologue's first
    pass (quantize_qkv_linear_streams) when every stream holds a multiple of 128
    rows (a GEMM row tile is one 128-row block of one sample), there are at most
    two, and the heads pair up into the GEMM's 256-column tiles."""
    return len(stream_lengths) <= 2 and H % 2 == 0 and all(n % 128 == 0 for n in stream_lengths)


def quantize_qkv_linear_streams(
    streams: list[tuple], H: int, N: int, sm_scale: float | None, *, smooth_k: bool, qk_quant: str,
    granularity: str, pv_quant: str,
) -> dict:
    """quantize_qkv_streams with the QKV linears in the same launch: the FP8 GEMM's
    epilogue runs P3 and the Q quantisation (``fd_fp8_gemm_qkv_quant``), so the
    bf16 Q/K/V never go to HBM before the prologue reads them.  ``streams``: one or
    two (a8 (B, S, K) e4m3, a_s (B, S, K / 128) f32, w8 (3 H 128, K) e4m3, w_s
    (3 H, K / 128) f32, bias (3 H 128,) bf16 or None, q_norm_w, k_norm_w, freqs
    (B, S, [1,] 64, 2, 2), s_off, eps), rows [s_off, s_off + S) of the N joint rows
    (see linear_prologue_ok).  Returns quantize_qkv_streams' dict, equal to it for
    the bf16 outputs of the same linears."""
    a0 = streams[0][0]
    B, dev = a0.shape[0], a0.device
    BH = B * H
    D = 128
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(D)
    assert len(streams) in (1, 2) and linear_prologue_ok([st[0].shape[1] for st in streams], H)
    qk = L.QK_INT8 if qk_quant == "int8" else L.QK_FP8
    gran = L.GRAN_TOKEN if granularity == "per_token" else L.GRAN_BLOCK
    pv = L.PV_FP8 if pv_quant == "fp8" else L.PV_BF16
    code_dt = torch.int8 if qk == L.QK_INT8 else torch.float8_e4m3fn
    q_codes = torch.empty(BH, N, D, dtype=code_dt, device=dev)
    q_desc = torch.empty(BH, _desc_stride(N, gran, 128), dtype=torch.float32, device=dev)
    k = torch.empty(BH, N, D, dtype=torch.bfloat16, device=dev)
    v = torch.empty(BH, N, D, dtype=torch.bfloat16, device=dev)
    ws = torch.empty(int(L.lib().fd_qkv_quant_workspace_floats(BH, N)), dtype=torch.float32, device=dev)
    probs, descs, keep = [], [], []
    for a8, a_s, w8, w_s, bias, qw, kw, freqs, s_off, eps in streams:
        Ba, S, K = a8.shape
        assert Ba == B and a8.dtype == torch.float8_e4m3fn and a8.is_contiguous() and a_s.is_contiguous()
        assert w8.shape == (3 * H * D, K) and w8.is_contiguous() and w_s.is_contiguous()
        L.require_cuda(a8, a_s, w8, w_s, bias, qw, kw, freqs)
        if bias is not None:
            bias = bias.contiguous()
            assert bias.dtype == torch.bfloat16
        fr = _freqs_rows(freqs, B, S)
        qw32, kw32 = qw.float().contiguous(), kw.float().contiguous()
        keep += [bias, fr, qw32, kw32]
        probs.append(L.GemmProblem(L.ptr(a8), L.ptr(a_s), L.ptr(w8), L.ptr(w_s), L.ptr(bias), None, None,
                                   B * S, 3 * H * D, K))
        descs.append(L.QkvStream(L.ptr(qw32), L.ptr(kw32), L.ptr(fr), S, s_off, float(eps)))
    p1 = ctypes.addressof(probs[1]) if len(probs) == 2 else None
    s1 = ctypes.addressof(descs[1]) if len(descs) == 2 else None
    stream_ptr = L.stream_ptr(dev)
    L.call("fd_fp8_gemm_qkv_quant", ctypes.addressof(probs[0]), ctypes.addressof(descs[0]), p1, s1, L.DT_BF16,
           B, H, N, qk, gran, pv, float(sm_scale * _LOG2E), L.ptr(q_codes), L.ptr(q_desc), L.ptr(k), L.ptr(v),
           L.ptr(ws), stream_ptr)
    k_codes = torch.empty(BH, N, D, dtype=code_dt, device=dev)
    k_desc = torch.empty(BH, _desc_stride(N, gran, 64), dtype=torch.float32, device=dev)
    k_mean = torch.empty(BH, D, dtype=torch.float32, device=dev)
    v_codes = torch.empty(BH, N, D, dtype=torch.float8_e4m3fn, device=dev) if pv == L.PV_FP8 else None
    v_desc = torch.empty(BH, D, dtype=torch.float32, device=dev) if pv == L.PV_FP8 else None
    L.call("fd_attn_quant_kv", L.ptr(k), L.ptr(v), BH, N, int(bool(smooth_k)), qk, gran, pv, L.ptr(k_codes),
           L.ptr(k_desc), L.ptr(v_codes), L.ptr(v_desc), L.ptr(k_mean), L.ptr(ws), stream_ptr)
    return {
        "q_codes": q_codes, "q_desc": q_desc, "k_codes": k_codes, "k_desc": k_desc,
        "v_codes": v_codes, "v_desc": v_desc, "k_mean": k_mean, "qk": qk, "gran": gran, "pv": pv,
        "k": k, "v": v, "B": B, "H": H, "N": N,
    }


def attn_quant_out_from_linear(
    streams: list[tuple], H: int, N: int, sm_scale: float | None, *, block_mask: Tensor | None, qk_quant: str,
    pv_quant: str, granularity: str, regions: list[tuple[Tensor, Tensor]], split: int | None = None,
) -> None:
    """quantize_qkv_linear_streams + the quantised-output attention: from the QKV
    linears' FP8 inputs to the output linears' 1 x 128 e4m3 inputs."""
    qz = quantize_qkv_linear_streams(streams, H, N, sm_scale, smooth_k=_SAGE_SMOOTH_K, qk_quant=qk_quant,
                                     granularity=granularity, pv_quant=pv_quant)
    vsrc = qz["v_codes"] if qz["pv"] == L.PV_FP8 else qz["v"]
    _quant_out_call(qz, vsrc, qz["B"], H, N, block_mask, regions, split, qz["k"].device)


def _quant_out_call(qz: dict, vsrc: Tensor, B: int, H: int, N: int, block_mask: Tensor | None,
                    regions: list[tuple[Tensor, Tensor]], split: int | None, dev) -> None:
    D = 128
    split = N if split is None else split
    assert 1 <= split <= N and len(regions) == (1 if split == N else 2)
    bm, bm_stride = _normalize_mask(block_mask, N)
    reg = []
    for i, (c, sc) in enumerate(regions):
        rows = B * (split if i == 0 else N - split)
        assert c.dtype in (torch.float8_e4m3fn, torch.uint8) and sc.dtype == torch.float32
        assert c.stride(-1) == 1 and sc.stride(-1) == 1
        assert c.numel() // c.shape[-1] >= rows and c.shape[-1] >= H * D and sc.shape[-1] >= H
        reg.append((L.ptr(c), L.ptr(sc), c.stride(-2), sc.stride(-2)))
    if len(reg) == 1:
        reg.append((None, None, 0, 0))
    L.call("fd_sage_attn_fwd_quant_out", L.ptr(qz["q_codes"]), L.ptr(qz["q_desc"]), L.ptr(qz["k_codes"]),
           L.ptr(qz["k_desc"]), L.ptr(vsrc), L.ptr(qz["v_desc"]), L.ptr(bm), bm_stride, None, B * H, N, H,
           qz["qk"], qz["gran"], qz["gran"], qz["pv"], *reg[0], *reg[1], split, L.stream_ptr(dev))


def attn_quant_out_from_streams(
    streams: list[tuple], H: int, N: int, sm_scale: float | None, *, block_mask: Tensor | None, qk_quant: str,
    pv_quant: str, granularity: str, regions: list[tuple[Tensor, Tensor]], split: int | None = None,
) -> None:
    """quantize_qkv_streams + the quantised-output attention (attn_forward_quant_out)
    for attention inputs straight from the QKV linear(s)."""
    qz = quantize_qkv_streams(streams, H, N, sm_scale, smooth_k=_SAGE_SMOOTH_K, qk_quant=qk_quant,
                              granularity=granularity, pv_quant=pv_quant)
    vsrc = qz["v_codes"] if qz["pv"] == L.PV_FP8 else qz["v"]
    _quant_out_call(qz, vsrc, qz["B"], H, N, block_mask, regions, split, qz["k"].device)


def attn_forward_quant_out(
    q: Tensor, k: Tensor, v: Tensor, sm_scale: float | None, *, block_mask: Tensor | None, qk_quant: str,
    pv_quant: str, granularity: str, regions: list[tuple[Tensor, Tensor]], split: int | None = None,
) -> None:
    """(B, H, N, 128) bf16 attention whose output is written as the 1 x 128 e4m3
    codes + fp32 scales of the output linear's input (one group per token row and
    head), code for code equal to ``fp8_act_quant`` of the (B, N, H * 128) bf16
    output.  ``regions``: one or two (codes (rows, >= H * 128), scales (rows, >= H))
    row-major views (row strides may exceed the width, e.g. a column window of a
    wider buffer); rows n < split of every sample go to region 0 (B * split rows),
    the rest to region 1."""
    B, H, N, D = q.shape
    assert D == 128 and q.dtype == torch.bfloat16
    L.require_cuda(q, k, v)
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(D)
    BH = B * H
    qf = q.reshape(BH, N, D).contiguous()
    kf = k.reshape(BH, N, D).contiguous()
    vf = v.reshape(BH, N, D).contiguous()
    qz = quantize_qkv(qf, kf, vf, sm_scale, smooth_k=_SAGE_SMOOTH_K, qk_quant=qk_quant,
                      granularity=granularity, pv_quant=pv_quant)
    vsrc = qz["v_codes"] if qz["pv"] != L.PV_BF16 else vf
    _quant_out_call(qz, vsrc, B, H, N, block_mask, regions, split, q.device)


def _pv_for(default_pv: str) -> str:
    return _SAGE_PV_QUANT if _SAGE_QK_GRAN == "per_block" else default_pv


def sage_attn_forward(q: Tensor, k: Tensor, v: Tensor, sm_scale: float | None = None) -> Tensor:
    """Attention forward without LSE (reference :121-180): qk_quant QK, bf16 PV."""
    out, _ = _attn_forward(q, k, v, sm_scale, block_mask=None, qk_quant=_SAGE_QK_QUANT,
                           pv_quant=_pv_for("bf16"), granularity=_SAGE_QK_GRAN, want_lse=False)
    return out


def sage_attn_forward_masked(
    q: Tensor, k: Tensor, v: Tensor, block_mask: Tensor, sm_scale: float | None = None,
) -> Tensor:
    """Block-masked forward (reference :183-268); mask is (nq, nk64) or (BH, nq, nk64) uint8."""
    out, _ = _attn_forward(q, k, v, sm_scale, block_mask=block_mask, qk_quant=_SAGE_QK_QUANT,
                           pv_quant=_pv_for("bf16"), granularity=_SAGE_QK_GRAN, want_lse=False)
    return out


def sage_attn_forward_with_lse(
    q: Tensor, k: Tensor, v: Tensor, sm_scale: float | None = None
) -> tuple[Tensor, Tensor]:
    """Forward returning (out, lse (BH, N) log2-domain) (reference :271-341).

    Reference dispatch: pv_quant == "fp8" -> FP8 QK + FP8 PV; else qk_quant QK + bf16 PV.
    """
    if _SAGE_QK_GRAN == "per_block":
        qk, pv = _SAGE_QK_QUANT, _SAGE_PV_QUANT
    elif _SAGE_PV_QUANT == "fp8":
        # the reference's FP8-QK / FP8-PV kernel: P and V scaled per 64-key tile
        qk, pv = "fp8", "fp8_tile"
    else:
        qk, pv = _SAGE_QK_QUANT, "bf16"
    return _attn_forward(q, k, v, sm_scale, block_mask=None, qk_quant=qk, pv_quant=pv,
                         granularity=_SAGE_QK_GRAN, want_lse=True)


def sage_attn_forward_masked_with_lse(
    q: Tensor, k: Tensor, v: Tensor, block_mask: Tensor, sm_scale: float | None = None,
) -> tuple[Tensor, Tensor]:
    """Masked forward with LSE; always INT8 QK + bf16 PV like the reference (:461-531)."""
    return _attn_forward(q, k, v, sm_scale, block_mask=block_mask, qk_quant="int8",
                         pv_quant=_pv_for("bf16"), granularity=_SAGE_QK_GRAN, want_lse=True)


def _per_token_descales(qz: dict, N: int) -> tuple[Tensor, Tensor]:
    """Q / K descales in the per-token layout (BH, round_up(N, 128)) that the
    backward kernels index by row.  Per-block scales (one per 128 Q rows, one per
    64 K rows) are repeated over their rows; the padding tail is zero."""
    if qz["gran"] == L.GRAN_TOKEN:
        return qz["q_desc"], qz["k_desc"]
    width = _desc_stride(N, L.GRAN_TOKEN, 1)
    qd = qz["q_desc"].repeat_interleave(128, dim=1)[:, :width]
    kd = qz["k_desc"].repeat_interleave(64, dim=1)[:, :width]
    qt = torch.zeros(qd.shape[0], width, dtype=torch.float32, device=qd.device)
    kt = torch.zeros_like(qt)
    qt[:, :N] = qd[:, :N]
    kt[:, :N] = kd[:, :N]
    return qt, kt


def _attn_backward(q, k, v, out, lse, dout, sm_scale, block_mask, qk_quant, granularity):
    """dQ, dK, dV on the tensor cores (fd_sage_attn_bwd: a dK/dV kernel and a dQ
    kernel, fp32 accumulation in TMEM, masked tiles skipped)."""
    B, H, N, D = q.shape
    BH = B * H
    L.require_cuda(q, k, v, out, lse, dout)
    assert D == 128 and q.dtype == k.dtype == v.dtype == out.dtype == torch.bfloat16, "bf16 (B, H, N, 128) inputs"
    qf = q.reshape(BH, N, D).contiguous()
    kf = k.reshape(BH, N, D).contiguous()
    vf = v.reshape(BH, N, D).contiguous()
    of = out.reshape(BH, N, D).contiguous()
    dof = dout.reshape(BH, N, D).contiguous().to(torch.bfloat16)
    lse = lse.contiguous()
    bm, bm_stride = _normalize_mask(block_mask, N)
    # the forward's codes, scales and smoothed K: P = exp2(S - LSE) is only the
    # forward's P when S is recomputed at the forward's quantisation granularity
    qz = quantize_qkv(qf, kf, vf, sm_scale, smooth_k=_SAGE_SMOOTH_K, qk_quant=qk_quant,
                      granularity=granularity, pv_quant="bf16")
    qz["q_desc"], qz["k_desc"] = _per_token_descales(qz, N)
    delta = torch.empty(BH, N, dtype=torch.float32, device=q.device)
    L.call("fd_sage_attn_bwd_prepass", L.ptr(dof), L.ptr(of), L.ptr(delta), BH, N, L.stream_ptr(q.device))
    if _SAGE_SMOOTH_K:
        ks = (kf - qz["k_mean"].to(torch.bfloat16).unsqueeze(1)).contiguous()
    else:
        ks = kf
    dq = torch.empty_like(qf)
    dk = torch.empty_like(qf)
    dv = torch.empty_like(qf)
    L.call(
        "fd_sage_attn_bwd", L.ptr(qf), L.ptr(ks), L.ptr(vf), L.ptr(dof), L.ptr(lse), L.ptr(delta),
        L.ptr(qz["q_codes"]), L.ptr(qz["q_desc"]), L.ptr(qz["k_codes"]), L.ptr(qz["k_desc"]),
        L.ptr(bm), bm_stride, L.ptr(dq), L.ptr(dk), L.ptr(dv), BH, N, qz["qk"], float(sm_scale),
        L.stream_ptr(q.device),
    )
    return dq.reshape(B, H, N, D), dk.reshape(B, H, N, D), dv.reshape(B, H, N, D)


def sage_attn_backward(
    q: Tensor, k: Tensor, v: Tensor, out: Tensor, lse: Tensor, dout: Tensor, sm_scale: float,
) -> tuple[Tensor, Tensor, Tensor]:
    """dQ, dK, dV with the forward's quantised P recomputation (reference :344-458).

    P is recomputed with the Q/K quantisation that the forward entry points use
    under the current ``configure_sage`` setting (per-token, or per-block when
    ``qk_granularity="per_block"``), so it equals the forward's P."""
    return _attn_backward(q, k, v, out, lse, dout, sm_scale, None, _SAGE_QK_QUANT, _SAGE_QK_GRAN)


def sage_attn_backward_masked(
    q: Tensor, k: Tensor, v: Tensor, out: Tensor, lse: Tensor, dout: Tensor, block_mask: Tensor,
    sm_scale: float,
) -> tuple[Tensor, Tensor, Tensor]:
    """Masked backward, INT8 recompute (reference :534-648), at the forward's
    quantisation granularity."""
    return _attn_backward(q, k, v, out, lse, dout, sm_scale, block_mask, "int8", _SAGE_QK_GRAN)


def smoke_test_fp8_dot(n: int = 128) -> dict:
    """FP8 per-row quantised dot check on this GPU (reference :90-118).

    Quantises two random (n, n) bf16 matrices per row with the G1 quantiser
    (one 128-wide block per row) and multiplies them on the tcgen05 GEMM.
    """
    _check_sm_capability()
    from .fp8_kernels import fp8_act_quant, fp8_gemm_blockwise

    assert n % 128 == 0
    a = torch.randn(n, n, dtype=torch.bfloat16, device="cuda")
    b = torch.randn(n, n, dtype=torch.bfloat16, device="cuda")
    a8, a_s = fp8_act_quant(a)
    b8, b_s_rows = fp8_act_quant(b)
    # per-row B scales act as rowwise weight scales when n == 128
    from .fp8_kernels import fp8_gemm_rowwise

    if n == 128:
        c = fp8_gemm_rowwise(a8, a_s, b8, b_s_rows.reshape(-1).contiguous())
    else:
        c = fp8_gemm_blockwise(a8, a_s, b8, torch.ones(n // 128, n // 128, device="cuda"))
    ref = a.float() @ b.float().T
    c_f32 = c.float()
    cos_sim = torch.nn.functional.cosine_similarity(c_f32.flatten().unsqueeze(0), ref.flatten().unsqueeze(0)).item()
    return {"cosine_similarity": cos_sim, "max_error": (c_f32 - ref).abs().max().item()}


# ---------------------------------------------------------------------------
# custom ops (reference :650-807)
# ---------------------------------------------------------------------------

_USE_CUSTOM_OP = True
_USE_MASKED_CUSTOM_OP = True


@torch.library.custom_op("futudiffu::sage_attn", mutates_args=())
def sage_attn_op(q: Tensor, k: Tensor, v: Tensor, sm_scale: float) -> tuple[Tensor, Tensor]:
    """SageAttention forward: returns (output, lse) for backward."""
    return sage_attn_forward_with_lse(q, k, v, sm_scale)


@sage_attn_op.register_fake
def _sage_attn_op_fake(q, k, v, sm_scale):
    B, H, N, D = q.shape
    return q.new_empty(B, H, N, D), q.new_empty(B * H, N, dtype=torch.float32)


def _setup_context(ctx, inputs, output):
    q, k, v, sm_scale = inputs
    out, lse = output
    ctx.save_for_backward(q, k, v, out, lse)
    ctx.sm_scale = sm_scale


def _backward(ctx, grad_out, grad_lse):
    q, k, v, out, lse = ctx.saved_tensors
    dq, dk, dv = sage_attn_backward(q, k, v, out, lse, grad_out, ctx.sm_scale)
    return dq, dk, dv, None


sage_attn_op.register_autograd(_backward, setup_context=_setup_context)


@torch.library.custom_op("futudiffu::sage_attn_masked", mutates_args=())
def sage_attn_masked_op(
    q: Tensor, k: Tensor, v: Tensor, block_mask: Tensor, sm_scale: float
) -> tuple[Tensor, Tensor]:
    """Masked SageAttention forward: returns (output, lse) for backward."""
    return sage_attn_forward_masked_with_lse(q, k, v, block_mask, sm_scale)


@sage_attn_masked_op.register_fake
def _sage_attn_masked_op_fake(q, k, v, block_mask, sm_scale):
    B, H, N, D = q.shape
    return q.new_empty(B, H, N, D), q.new_empty(B * H, N, dtype=torch.float32)


def _masked_setup_context(ctx, inputs, output):
    q, k, v, block_mask, sm_scale = inputs
    out, lse = output
    ctx.save_for_backward(q, k, v, out, lse, block_mask)
    ctx.sm_scale = sm_scale


def _masked_backward(ctx, grad_out, grad_lse):
    q, k, v, out, lse, block_mask = ctx.saved_tensors
    dq, dk, dv = sage_attn_backward_masked(q, k, v, out, lse, grad_out, block_mask, ctx.sm_scale)
    return dq, dk, dv, None, None


sage_attn_masked_op.register_autograd(_masked_backward, setup_context=_masked_setup_context)
