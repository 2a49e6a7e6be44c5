"""Ulysses sequence parallelism for the quantized attention.

Each of the P ranks of a process group holds L / P consecutive tokens of the
sequence for every head.  Attention needs every token of a head, so before the
attention the Q/K/V shards are exchanged with one NCCL all-to-all (sequence ->
head sharding: afterwards a rank holds all L tokens of H / P heads), the
attention kernel runs locally on those heads, and a second all-to-all brings
the output back to sequence sharding (head -> sequence).  Everything lands in
this GPU's memory before a kernel reads it: the kernels never touch a peer's
memory, and there is no collective inside a kernel.

Layouts (one sample):
  sequence-sharded activations: (H, L/P, 128), heads contiguous;
  head-sharded attention inputs: (H/P, L, 128).
The exchange is the only cross-GPU step of the video DiT; everything else is
rank-local.
"""

from __future__ import annotations

import torch
import torch.distributed as dist
from torch import Tensor


def _world(group) -> int:
    return dist.get_world_size(group) if dist.is_initialized() else 1


def seq_to_head(x: Tensor, group=None) -> Tensor:
    """(H, L/P, D) on every rank -> (H/P, L, D): rank r receives heads
    [r H/P, (r+1) H/P) of all ranks' tokens, in sequence order."""
    P = _world(group)
    H, Ls, D = x.shape
    if H % P:
        raise ValueError(f"{H} heads do not split over {P} ranks")
    if P == 1:
        return x
    send = x.contiguous()                       # (P, H/P, L/P, D): chunk p goes to rank p
    recv = torch.empty_like(send)               # (P_src, H/P, L/P, D)
    dist.all_to_all_single(recv, send, group=group)
    return recv.view(P, H // P, Ls, D).transpose(0, 1).reshape(H // P, P * Ls, D)


def head_to_seq(o: Tensor, group=None) -> Tensor:
    """(H/P, L, D) -> (L/P, H * D): this rank's token shard of every head, in the
    row layout of the output projection."""
    P = _world(group)
    Hp, L, D = o.shape
    if L % P:
        raise ValueError(f"sequence {L} does not split over {P} ranks")
    if P == 1:
        return o.transpose(0, 1).reshape(L, Hp * D)
    Ls = L // P
    send = o.view(Hp, P, Ls, D).transpose(0, 1).contiguous()  # (P_dst, H/P, L/P, D)
    recv = torch.empty_like(send)                             # (P_src = head group, H/P, L/P, D)
    dist.all_to_all_single(recv, send, group=group)
    return recv.permute(2, 0, 1, 3).reshape(Ls, P * Hp * D)


def head_to_seq_rows(x: Tensor, group=None) -> Tensor:
    """(L, H/P * W) token-major rows of this rank's heads -> (L/P, H * W): this rank's
    token shard with every head, in head_to_seq's column order.  W is any per-head
    width: 128 e4m3 codes of the quantised attention output, or its one scale, so
    the output projection's input crosses NVLink as 1 x 128 codes + scales
    (1 + 4/128 bytes per value instead of 2)."""
    P = _world(group)
    L, C = x.shape
    if P == 1:
        return x
    if L % P:
        raise ValueError(f"sequence {L} does not split over {P} ranks")
    send = x.contiguous()                        # rows [p L/P, (p+1) L/P) go to rank p
    recv = torch.empty_like(send)                # (P_src, L/P, C)
    dist.all_to_all_single(recv, send, group=group)
    return recv.view(P, L // P, C).transpose(0, 1).reshape(L // P, P * C)


def ulysses_attention_codes(q: Tensor, k: Tensor, v: Tensor, attn_codes_fn, group=None) -> tuple[Tensor, Tensor]:
    """Sequence-sharded (H, L/P, D) Q/K/V -> attention -> the output projection's
    quantised input for this rank's tokens: codes (L/P, H * 128) uint8 and scales
    (L/P, H).  ``attn_codes_fn(q, k, v)`` runs on (1, H/P, L, D) and returns codes
    (L, H/P * 128) uint8 and scales (L, H/P) fp32."""
    qh, kh, vh = (seq_to_head(t, group) for t in (q, k, v))
    codes, scales = attn_codes_fn(qh.unsqueeze(0), kh.unsqueeze(0), vh.unsqueeze(0))
    return head_to_seq_rows(codes.view(torch.uint8), group), head_to_seq_rows(scales, group)


def ulysses_attention(q: Tensor, k: Tensor, v: Tensor, attn_fn, group=None) -> Tensor:
    """Sequence-sharded (H, L/P, D) Q/K/V -> attention -> (L/P, H * D).

    ``attn_fn(q, k, v)`` runs on (1, H/P, L, D) tensors and returns the same
    shape (the quantized attention kernel on the GPU; any exact attention in
    the CPU tests)."""
    qh, kh, vh = (seq_to_head(t, group) for t in (q, k, v))
    o = attn_fn(qh.unsqueeze(0), kh.unsqueeze(0), vh.unsqueeze(0))[0]
    return head_to_seq(o, group)
