"""Ulysses sequence parallelism on CPU: world sizes 2 and 4 over gloo, exact
attention as the per-rank kernel; the sharded result must equal full attention.
World size 4 with one head per rank and group is the layout of the 14B-class
video workload at 8 GPUs (40 heads, 5 per rank, 5 head groups)."""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _exact(q, k, v):
    s = torch.einsum("bhqd,bhkd->bhqk", q.float(), k.float()) / q.shape[-1] ** 0.5
    return torch.einsum("bhqk,bhkd->bhqd", s.softmax(-1), v.float())


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, H, L, D, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from futudiffu_b200.ulysses import head_to_seq, head_to_seq_rows, seq_to_head, ulysses_attention

        g = torch.Generator().manual_seed(0)
        q, k, v = (torch.randn(H, L, D, generator=g) for _ in range(3))
        Ls = L // world
        sl = slice(rank * Ls, (rank + 1) * Ls)
        # the exchange itself: sequence -> head -> sequence is the identity
        qh = seq_to_head(q[:, sl].contiguous())
        assert torch.equal(qh, q[rank * H // world:(rank + 1) * H // world])
        back = head_to_seq(qh)
        assert torch.equal(back, q[:, sl].transpose(0, 1).reshape(Ls, H * D))
        # token-major rows of this rank's heads (codes / scales of the quantised output)
        # land in head_to_seq's layout
        rows = qh.transpose(0, 1).reshape(L, (H // world) * D)
        assert torch.equal(head_to_seq_rows(rows), back)
        codes = torch.randint(0, 256, (L, (H // world) * 128), generator=g, dtype=torch.uint8)
        got = head_to_seq_rows(codes)
        want = head_to_seq(codes.view(L, H // world, 128).transpose(0, 1).contiguous())
        assert torch.equal(got, want)
        o = ulysses_attention(q[:, sl].contiguous(), k[:, sl].contiguous(), v[:, sl].contiguous(), _exact)
        ref = _exact(q[None], k[None], v[None])[0][:, sl].transpose(0, 1).reshape(Ls, H * D)
        out[rank] = float((o - ref).abs().max())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,H,L", [(2, 4, 12), (2, 6, 10), (4, 8, 12)])
def test_ulysses_attention_world2(world, H, L):
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    out = mgr.dict()
    mp.start_processes(_worker, args=(world, _free_port(), H, L, 8, out), nprocs=world, join=True,
                       start_method="spawn")
    assert len(out) == world
    assert max(out.values()) < 1e-5


def test_ulysses_single_rank_is_plain_attention():
    from futudiffu_b200.ulysses import ulysses_attention

    g = torch.Generator().manual_seed(1)
    q, k, v = (torch.randn(3, 7, 8, generator=g) for _ in range(3))
    o = ulysses_attention(q, k, v, _exact)
    assert torch.allclose(o, _exact(q[None], k[None], v[None])[0].transpose(0, 1).reshape(7, 24), atol=1e-6)


def _codes_fn(q, k, v):
    """Stand-in for the attention kernel's quantised output: per-(token, head) scale
    and uint8 codes, token-major (L, h * D) / (L, h), from exact attention."""
    o = _exact(q, k, v)[0]                                   # (h, L, D)
    s = o.abs().amax(-1).clamp_min(1e-6)                     # (h, L)
    c = ((o / s[..., None]) * 127 + 128).round().clamp(0, 255).to(torch.uint8)
    return c.transpose(0, 1).reshape(o.shape[1], -1), s.transpose(0, 1).contiguous()


def _worker_groups(rank, world, port, H, L, D, groups, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from futudiffu_b200.ulysses import ulysses_attention_codes

        g = torch.Generator().manual_seed(3)
        q, k, v = (torch.randn(H, L, D, generator=g) for _ in range(3))
        Ls = L // world
        sl = slice(rank * Ls, (rank + 1) * Ls)
        shards = [t[:, sl].contiguous() for t in (q, k, v)]
        ref_c, ref_s = _codes_fn(q[None], k[None], v[None])
        ref_c, ref_s = ref_c[sl], ref_s[sl]
        res = {}
        for G in (1,) + tuple(groups):
            c, s = ulysses_attention_codes(*shards, _codes_fn, head_groups=G)
            res[G] = (torch.equal(c, ref_c), float((s - ref_s).abs().max()))
        out[rank] = res
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,H,L,groups", [(2, 8, 12, (2, 4)), (2, 12, 10, (2, 3, 6)), (4, 20, 12, (5,))])
def test_ulysses_head_group_pipeline_world2(world, H, L, groups):
    """The pipelined exchange (head groups, async all-to-all) returns the same codes
    and scales as the one-shot exchange and as unsharded attention."""
    ctx = mp.get_context("spawn")
    out = ctx.Manager().dict()
    mp.start_processes(_worker_groups, args=(world, _free_port(), H, L, 8, groups, out), nprocs=world, join=True,
                       start_method="spawn")
    assert len(out) == world
    for res in out.values():
        for G, (codes_equal, scale_err) in res.items():
            assert codes_equal, G
            assert scale_err < 1e-6, G

