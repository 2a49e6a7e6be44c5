"""Seeded inputs of the reference-on-B200 fixtures (``ref_gpu.pt``).

``make_gpu_golden.py`` runs the reference's own Triton kernels on a B200 on
these inputs; the ``-m gpu`` tests regenerate the same inputs on the CPU
(``torch.Generator``, so the bits do not depend on the device) and compare this
build's outputs with the stored ones.  Large outputs are stored as a SHA-256
digest of their bytes (bit-exact gates) or as a fixed sample of rows (tolerance
gates); the sampled indices are defined here too.
"""

from __future__ import annotations

import hashlib
import math

import torch

SM = 1.0 / math.sqrt(128)


def gen(seed: int) -> torch.Generator:
    return torch.Generator().manual_seed(seed)


def digest(t: torch.Tensor) -> str:
    """SHA-256 of a tensor's bytes (contiguous, on the CPU)."""
    t = t.detach().contiguous().cpu()
    if t.dtype in (torch.float8_e4m3fn, torch.bfloat16, torch.float16):
        t = t.view(torch.uint8 if t.element_size() == 1 else torch.int16)
    return hashlib.sha256(t.numpy().tobytes()).hexdigest()


# ---------------------------------------------------------------- G1 activation quantiser
# config 1 / config 3 activations, the reference's Z-Image shape, ragged rows
ACT_SHAPES = {"config1": (2048, 3072), "config3": (4608, 3072), "ref": (8576, 3840), "ragged": (333, 1280),
              "small": (16, 512)}


def act_input(name: str) -> torch.Tensor:
    """bf16 rows with per-row scales over four decades, one all-zero 128-group and
    a few large outliers (exercising the 1e-12 clamp and the saturating cast)."""
    M, K = ACT_SHAPES[name]
    g = gen(100 + sum(map(ord, name)))
    row = torch.exp(torch.empty(M, 1).uniform_(-4.0, 4.0, generator=g))
    x = torch.randn(M, K, generator=g) * row
    x[3 % M, :128] = 0.0
    x[min(5, M - 1), 7] = 3.0e4
    return x.to(torch.bfloat16)


# ---------------------------------------------------------------- G4 SiLU gate + quant
SILU_SHAPES = {"zimage": (1024, 2 * 10240), "small": (40, 2 * 256)}


def silu_input(name: str) -> torch.Tensor:
    M, N2 = SILU_SHAPES[name]
    g = gen(200 + sum(map(ord, name)))
    return (torch.randn(M, N2, generator=g) * 2.0).to(torch.bfloat16)


# ---------------------------------------------------------------- G2 block GEMM (+ requant / GELU)
GEMM_SHAPES = {"config1": (2048, 3072, 3072), "ref_qkv": (8576, 11520, 3840), "small": (72, 256, 384)}
GEMM_SAMPLE_ROWS = {"config1": 16, "ref_qkv": 8, "small": 72}


def gemm_inputs(name: str) -> tuple[torch.Tensor, torch.Tensor]:
    """X (M, K) bf16 ~N(0, 1), W (N, K) bf16 ~N(0, 0.02) (BASELINE config 1's distributions)."""
    M, N, K = GEMM_SHAPES[name]
    g = gen(300 + sum(map(ord, name)))
    x = torch.randn(M, K, generator=g).to(torch.bfloat16)
    w = (torch.randn(N, K, generator=g) * 0.02).to(torch.bfloat16)
    return x, w


def row_sample(M: int, n: int) -> torch.Tensor:
    """``n`` rows spread over [0, M), first and last included."""
    if n >= M:
        return torch.arange(M)
    return torch.linspace(0, M - 1, n).round().long()


# ---------------------------------------------------------------- P1 / P2 / P3 fused prologues
NORM_SHAPE = (1, 4608, 3072)  # config 3: 512 text + 4096 image tokens, hidden 3072
QKV_SHAPE = (1, 4608, 24)     # (B, S, heads), head_dim 128
NORM_SAMPLE_ROWS = 24


def norm_inputs() -> dict:
    B, S, Dm = NORM_SHAPE
    g = gen(400)
    return {
        "x": torch.randn(B, S, Dm, generator=g).to(torch.bfloat16),
        "w": (1 + 0.1 * torch.randn(Dm, generator=g)).to(torch.bfloat16),
        "scale": (0.5 * torch.randn(B, Dm, generator=g)).to(torch.bfloat16),
        "gate": torch.randn(B, Dm, generator=g).to(torch.bfloat16),
        "res": torch.randn(B, S, Dm, generator=g).to(torch.bfloat16),
    }


def qkv_inputs() -> dict:
    """QKV linear output (B, S, 3 H 128), Q/K RMSNorm weights and RoPE rotations
    (B, S, 1, 64, 2, 2) fp32 from random angles (cos, -sin; sin, cos)."""
    B, S, H = QKV_SHAPE
    g = gen(401)
    ang = torch.rand(B, S, 64, generator=g) * 6.283185307179586
    c, s = torch.cos(ang), torch.sin(ang)
    freqs = torch.stack([torch.stack([c, -s], -1), torch.stack([s, c], -1)], -2).unsqueeze(2).contiguous()
    return {
        "qkv": torch.randn(B, S, 3 * H * 128, generator=g).to(torch.bfloat16),
        "qw": (1 + 0.1 * torch.randn(128, generator=g)).to(torch.bfloat16),
        "kw": (1 + 0.1 * torch.randn(128, generator=g)).to(torch.bfloat16),
        "freqs": freqs, "H": H,
    }


# ---------------------------------------------------------------- A1-A7 attention
# config 2 (B2 H24 S4096, K offset ~N(0, 4)), the reference's shape (B2 H30 N4288),
# a ragged case that also runs the backward
ATTN_SHAPES = {"config2": (2, 24, 4096), "ref": (2, 30, 4288), "ragged": (1, 3, 1000)}
# (qk_quant, pv_quant, masked) of each stored forward; "fp8/fp8" is the reference's
# per-64-key-tile P / V mode (sage_kernels.py:1135-1154)
ATTN_MODES = {
    "config2": [("int8", "bf16", False), ("fp8", "bf16", False), ("fp8", "fp8", False)],
    "ref": [("int8", "bf16", False), ("int8", "bf16", True)],
    "ragged": [("int8", "bf16", False), ("fp8", "bf16", False), ("fp8", "fp8", False), ("int8", "bf16", True)],
}
ATTN_BWD = {"ragged": ["int8", "fp8"]}


def attn_inputs(name: str) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    """q, k, v, dout (B, H, N, 128) bf16 ~N(0, 1); K plus one per-channel offset
    ~N(0, 4) shared over batch, heads and tokens (exercises the smoothing)."""
    B, H, N = ATTN_SHAPES[name]
    g = gen(500 + sum(map(ord, name)))
    q = torch.randn(B, H, N, 128, generator=g).to(torch.bfloat16)
    k = (torch.randn(B, H, N, 128, generator=g) + 2.0 * torch.randn(128, generator=g)).to(torch.bfloat16)
    v = torch.randn(B, H, N, 128, generator=g).to(torch.bfloat16)
    do = torch.randn(B, H, N, 128, generator=g).to(torch.bfloat16)
    return q, k, v, do


def attn_mask(name: str) -> torch.Tensor:
    """Block mask of a packed sequence: documents of 40 %, 35 % and 25 % of N, the
    padding tail attached to document 0 (build_block_mask's quirk)."""
    from futudiffu_b200.block_mask import build_block_mask

    N = ATTN_SHAPES[name][2]
    a = int(N * 0.4) // 32 * 32
    b = int(N * 0.35) // 32 * 32
    return build_block_mask([a, b, N - a - b - 16], total_len=N, device="cpu")


def attn_sample(name: str) -> tuple[torch.Tensor, torch.Tensor]:
    """Flattened (b h) indices and row indices of the stored output / LSE sample."""
    B, H, N = ATTN_SHAPES[name]
    BH = B * H
    heads = torch.tensor(sorted({0, BH // 2, BH - 1}))
    rows = row_sample(N, min(N, 67))
    return heads, rows
