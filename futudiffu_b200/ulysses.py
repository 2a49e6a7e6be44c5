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

import contextlib

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


def ulysses_attention_codes(q: Tensor, k: Tensor, v: Tensor, attn_codes_fn, group=None,
                            head_groups: int = 1) -> tuple[Tensor, Tensor]:
    """Sequence-sharded (H, L/P, D) Q/K/V -> attention -> the output projection's
    quantised input for this rank's tokens: codes (L/P, H * 128) uint8 and scales
    (L/P, H).  ``attn_codes_fn(q, k, v)`` runs on (1, h, L, D) for the heads this
    rank attends and returns codes (L, h * 128) uint8 and scales (L, h) fp32.

    ``head_groups`` = G > 1 pipelines the exchange with the attention.  Heads are
    cut into G groups of H / G consecutive labels; group g's slice of Q/K/V is one
    contiguous (H / G, L/P, D) block, so its sequence -> head exchange is one
    ``all_to_all_single`` per tensor with no gather copy, and rank p attends the
    group's labels [g H/G + p h, g H/G + (p + 1) h), h = H / (P G).  Every
    exchange is issued asynchronously on the process group's stream: group g + 1's
    Q/K/V cross NVLink while group g attends, and group g's output codes travel
    back while later groups attend; groups attend alternately on two streams so
    that one group's last partial wave overlaps the next group's launch.  The
    output columns land at each head's own label, so the projection sees the same
    input for every G (the assignment of heads to ranks changes, each head's
    attention does not).  On two power-capped B200s (config 5, 40 heads, 32760
    tokens) G = 2 and G = 4 ran no faster than G = 1: an exchange alone hides
    under the attention, but inside the full step the GPU is at its power limit
    and the concurrent NCCL kernels slow the attention by about what they save."""
    P = _world(group)
    G = head_groups
    if P == 1 or G <= 1:
        qh, kh, vh = (seq_to_head(t, group) for t in (q, k, v))
        codes, scales = attn_codes_fn(qh.unsqueeze(0), kh.unsqueeze(0), vh.unsqueeze(0))
        return head_to_seq_rows(codes.view(torch.uint8), group), head_to_seq_rows(scales, group)
    H, Ls, D = q.shape
    if H % (P * G):
        raise ValueError(f"{H} heads do not split into {G} groups over {P} ranks")
    h, W = H // (P * G), H // G

    def post_in(g):
        bufs, works = [], []
        for t in (q, k, v):
            send = t[g * W:(g + 1) * W]             # (P, h, L/P, D): chunk p goes to rank p
            recv = torch.empty_like(send)           # (P_src, h, L/P, D)
            works.append(dist.all_to_all_single(recv, send, group=group, async_op=True))
            bufs.append(recv)
        return bufs, works

    # every group's Q/K/V exchange is queued up front on the process group's stream;
    # groups attend alternately on this stream and a side stream, so the short
    # per-group launches overlap each other's last partial wave as well as NCCL
    ins = [post_in(g) for g in range(G)]
    cur = torch.cuda.current_stream(q.device) if q.is_cuda else None
    side = _side_stream(q.device) if q.is_cuda else None
    if side is not None:
        side.wait_stream(cur)
    back = []
    for g in range(G):
        st = side if (side is not None and g % 2) else cur
        with torch.cuda.stream(st) if st is not None else contextlib.nullcontext():
            bufs, works = ins[g]
            for w in works:
                w.wait()
            qh, kh, vh = (b.view(P, h, Ls, D).transpose(0, 1).reshape(1, h, P * Ls, D) for b in bufs)
            c8, cs = attn_codes_fn(qh, kh, vh)      # (L, h * 128), (L, h): rows [p L/P, ...) go to rank p
            c8 = c8.view(torch.uint8)
            rc, rs = torch.empty_like(c8), torch.empty_like(cs)
            if st is side and side is not None:
                rc.record_stream(cur)
                rs.record_stream(cur)
            back.append((g, rc, rs, dist.all_to_all_single(rc, c8.contiguous(), group=group, async_op=True),
                         dist.all_to_all_single(rs, cs.contiguous(), group=group, async_op=True)))
    if side is not None:
        cur.wait_stream(side)
    cw, sw = back[0][1].shape[1] // h, back[0][2].shape[1] // h   # per-head widths (128 codes, 1 scale)
    codes = torch.empty(Ls, H * cw, dtype=back[0][1].dtype, device=q.device)
    scales = torch.empty(Ls, H * sw, dtype=back[0][2].dtype, device=q.device)
    for g, rc, rs, w1, w2 in back:
        w1.wait()
        w2.wait()
        # source rank p holds labels g W + p h + [0, h): columns [g W + p h, ...) of this token shard
        codes.view(Ls, G, W * cw)[:, g] = rc.view(P, Ls, h * cw).transpose(0, 1).reshape(Ls, W * cw)
        scales.view(Ls, G, W * sw)[:, g] = rs.view(P, Ls, h * sw).transpose(0, 1).reshape(Ls, W * sw)
    return codes, scales


_SIDE: dict[int, "torch.cuda.Stream"] = {}


def _side_stream(device) -> "torch.cuda.Stream":
    """One extra compute stream per device for the pipelined exchange."""
    idx = torch.device(device).index
    if idx not in _SIDE:
        _SIDE[idx] = torch.cuda.Stream(device=device)
    return _SIDE[idx]


def ulysses_attention(q: Tensor, k: Tensor, v: Tensor, attn_fn, group=None) -> Tensor:
    """Sequence-sharded (H, L/P, D) Q/K/V -> attention -> (L/P, H * D).

    ``attn_fn(q, k, v)`` runs on (1, H/P, L, D) tensors and returns the same
    shape (the quantized attention kernel on the GPU; any exact attention in
    the CPU tests)."""
    qh, kh, vh = (seq_to_head(t, group) for t in (q, k, v))
    o = attn_fn(qh.unsqueeze(0), kh.unsqueeze(0), vh.unsqueeze(0))[0]
    return head_to_seq(o, group)
