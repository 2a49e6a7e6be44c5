"""Ulysses sequence parallelism on two GPUs (NCCL): a reduced video DiT whose
tokens are sharded over two ranks, with the NCCL all-to-all around every
self-attention, gives the same output as the same model on one GPU.

Every per-token step (norms, 1 x 128 activation quantisation, FP8 GEMMs) sees
the same rows, and every head's attention sees the same full sequence in the
same order on both layouts, so the two results agree to the last bits; only the
bf16 cross-attention (torch SDPA over 64 text keys) may pick another kernel for
the shorter query count.  Skipped with fewer than two GPUs.
"""

from __future__ import annotations

import datetime
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _cfg():
    from futudiffu_b200.dit import VideoDiTConfig

    return VideoDiTConfig(hidden=1024, heads=8, ffn=2816, n_blocks=2, grid=(2, 16, 32), txt_tokens=64,
                          rope_axes=(44, 42, 42))


def _inputs(cfg):
    g = torch.Generator().manual_seed(5)
    lat = torch.randn(1, cfg.tokens, cfg.patch_dim, generator=g).to(torch.bfloat16)
    txt = torch.randn(1, cfg.txt_tokens, cfg.hidden, generator=g).to(torch.bfloat16)
    return lat, txt


def _worker(rank, world, port, out):
    import torch.distributed as dist

    from futudiffu_b200 import check_status
    from futudiffu_b200.dit import VideoDiT

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    cfg = _cfg()
    lat, txt = _inputs(cfg)
    t = torch.tensor([0.7], device=dev)
    try:
        model = VideoDiT(cfg, seed=0, device=dev)
        assert model.P == world
        Ls = model.local_tokens
        xl = lat[:, rank * Ls:(rank + 1) * Ls].contiguous().to(dev)
        model.head_groups = 1
        y = model(xl, txt.to(dev), t)
        # the pipelined exchange (head groups, async all-to-all) changes which rank
        # attends which head, not any head's result: bit-identical output
        same = []
        for G in (2, 4):
            model.head_groups = G
            same.append(torch.equal(model(xl, txt.to(dev), t), y))
        parts = [torch.empty_like(y) for _ in range(world)]
        dist.all_gather(parts, y)
        torch.cuda.synchronize()
        check_status()
        out[f"groups_equal_{rank}"] = all(same)
        if rank == 0:
            out["sharded"] = torch.cat(parts, 1).cpu()
        del model
    finally:
        dist.destroy_process_group()
    if rank == 0:
        # the same model on one GPU (no process group: P = 1)
        model = VideoDiT(cfg, seed=0, device=dev)
        assert model.P == 1
        out["single"] = model(lat.to(dev), txt.to(dev), t).cpu()
        check_status()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_video_dit_two_ranks_equal_one():
    import torch.multiprocessing as mp

    from tests.helpers import cosine

    ctx = mp.get_context("spawn")
    out = ctx.Manager().dict()
    mp.start_processes(_worker, args=(2, _free_port(), out), nprocs=2, join=True, start_method="spawn")
    assert out["groups_equal_0"] and out["groups_equal_1"]
    a, b = out["sharded"].float(), out["single"].float()
    assert torch.isfinite(a).all()
    assert cosine(a, b) >= 0.99999
    assert (a - b).abs().max().item() <= 0.02 * b.abs().max().item()
