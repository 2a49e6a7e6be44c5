"""Shared comparison helpers for the parity tests."""

from __future__ import annotations

import torch


def cosine(a: torch.Tensor, b: torch.Tensor) -> float:
    a = a.detach().float().flatten().cpu().double()
    b = b.detach().float().flatten().cpu().double()
    return float((a @ b) / (a.norm() * b.norm()).clamp_min(1e-300))


def e4m3_bits(t: torch.Tensor) -> torch.Tensor:
    return t.detach().cpu().view(torch.uint8)


def e4m3_step_diff(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """|difference| between two e4m3 tensors measured in representable steps (sign-magnitude order)."""
    def ordinal(t):
        u = e4m3_bits(t).to(torch.int32)
        mag = u & 0x7F
        return torch.where((u & 0x80) != 0, -mag, mag)
    return (ordinal(a) - ordinal(b)).abs()


def bf16_ulp_diff(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """|difference| in bf16 units in the last place (sign-magnitude ordinals)."""
    def ordinal(t):
        u = t.detach().cpu().to(torch.bfloat16).view(torch.int16).to(torch.int32)
        mag = u & 0x7FFF
        return torch.where(u < 0, -mag, mag)
    return (ordinal(a) - ordinal(b)).abs()
