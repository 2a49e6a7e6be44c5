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


_DIV_KERNEL = None


def triton_divide(a, b) -> torch.Tensor:
    """a / b in fp32 evaluated by a Triton kernel on the GPU.

    The reference computes every quantisation scale with Triton's fp32 ``/``
    (e.g. src/futudiffu/fp8_kernels.py:65-76, sage_kernels.py:632-663), whose
    result the GPU instruction Triton compiles it to decides.  The parity tests
    evaluate the oracle's quotients through this function, so the quotients come
    from the reference's own compiler path and not from the library under test.
    a, b: tensors or numbers (broadcast together); returns a CPU float32 tensor.
    """
    global _DIV_KERNEL
    import triton
    import triton.language as tl

    if _DIV_KERNEL is None:
        @triton.jit
        def _div(a_ptr, b_ptr, o_ptr, n, BLOCK: tl.constexpr):
            i = tl.program_id(0) * BLOCK + tl.arange(0, BLOCK)
            m = i < n
            x = tl.load(a_ptr + i, mask=m, other=1.0)
            y = tl.load(b_ptr + i, mask=m, other=1.0)
            tl.store(o_ptr + i, x / y, mask=m)

        _DIV_KERNEL = _div
    at = torch.as_tensor(a, dtype=torch.float32)
    bt = torch.as_tensor(b, dtype=torch.float32)
    shape = torch.broadcast_shapes(at.shape, bt.shape)
    ad = torch.broadcast_to(at.to("cuda"), shape).contiguous()
    bd = torch.broadcast_to(bt.to("cuda"), shape).contiguous()
    out = torch.empty_like(ad)
    n = ad.numel()
    if n:
        _DIV_KERNEL[(triton.cdiv(n, 1024),)](ad, bd, out, n, BLOCK=1024)
    return out.cpu()
