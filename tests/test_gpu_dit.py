"""GPU parity of the DiT workloads (MMDiT double-stream block, single-stream
block, DiT forward + Euler step) against the CPU composition of the oracle ops."""

from __future__ import annotations

import pytest
import torch

from oracle import dit as OD
from tests.conftest import gen
from tests.helpers import cosine

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _triton_division():
    from oracle import quant as _OQ
    from tests.helpers import triton_divide

    with _OQ.division(triton_divide):
        yield


def _small_cfg(**kw):
    from futudiffu_b200.dit import DiTConfig

    base = dict(hidden=256, heads=2, mlp_ratio=4, n_double=1, n_single=1, txt_tokens=64,
                img_grid=(8, 16), patch_dim=64, rope_axes=(64, 64))
    base.update(kw)
    return DiTConfig(**base)


def _close(a, b, cos_min=0.999):
    af, bf = a.float().cpu(), b.float().cpu()
    assert torch.isfinite(af).all()
    c = cosine(af, bf)
    assert c >= cos_min, c
    err = (af - bf).abs().max().item()
    assert err <= 0.05 * bf.abs().max().item() + 1e-2, err


@pytest.mark.parametrize("B", [1, 2])
def test_double_stream_block(cuda_device, B):
    from futudiffu_b200.dit import DoubleStreamBlock, batch_freqs, image_freqs, text_freqs

    cfg = _small_cfg()
    g = torch.Generator(device=cuda_device).manual_seed(3)
    blk = DoubleStreamBlock(cfg, g, cuda_device)
    cg = gen(4)
    x_txt = torch.randn(B, cfg.txt_tokens, cfg.hidden, generator=cg).to(torch.bfloat16)
    x_img = torch.randn(B, cfg.img_tokens, cfg.hidden, generator=cg).to(torch.bfloat16)
    vec = torch.randn(B, cfg.hidden, generator=cg).to(torch.bfloat16)
    f_txt = batch_freqs(text_freqs(cfg, cuda_device), B)
    f_img = batch_freqs(image_freqs(cfg, cuda_device), B)
    with torch.no_grad():
        o_txt, o_img = blk(x_txt.to(cuda_device), x_img.to(cuda_device), vec.to(cuda_device), f_txt, f_img)
        r_txt, r_img = OD.double_block(blk, x_txt, x_img, vec, f_txt, f_img)
    _close(o_txt, r_txt)
    _close(o_img, r_img)


def test_double_stream_block_config3_full_size(cuda_device):
    """Benchmark config 3 at its real shape (hidden 3072, 24 heads, 512 text + 4096
    image tokens, batch 1) against the oracle composition.  The oracle runs its
    linears as dequantised fp32 matmuls and its attention matmuls in fp32: the same
    quantised operands and the same quantisers as the exact form, summed in another
    order, which keeps the CPU side to seconds at this size."""
    from futudiffu_b200.dit import DiTConfig, DoubleStreamBlock, batch_freqs, image_freqs, text_freqs

    cfg = DiTConfig()
    assert (cfg.hidden, cfg.heads, cfg.txt_tokens, cfg.img_tokens) == (3072, 24, 512, 4096)
    g = torch.Generator(device=cuda_device).manual_seed(13)
    blk = DoubleStreamBlock(cfg, g, cuda_device)
    cg = gen(14)
    x_txt = torch.randn(1, cfg.txt_tokens, cfg.hidden, generator=cg).to(torch.bfloat16)
    x_img = torch.randn(1, cfg.img_tokens, cfg.hidden, generator=cg).to(torch.bfloat16)
    vec = torch.randn(1, cfg.hidden, generator=cg).to(torch.bfloat16)
    f_txt = batch_freqs(text_freqs(cfg, cuda_device), 1)
    f_img = batch_freqs(image_freqs(cfg, cuda_device), 1)
    with torch.no_grad():
        o_txt, o_img = blk(x_txt.to(cuda_device), x_img.to(cuda_device), vec.to(cuda_device), f_txt, f_img)
    with OD.eager_cpu_timing():
        r_txt, r_img = OD.double_block(blk, x_txt, x_img, vec, f_txt.cpu(), f_img.cpu())
    _close(o_txt, r_txt)
    _close(o_img, r_img)


def test_single_stream_block(cuda_device):
    from futudiffu_b200.dit import SingleStreamBlock, batch_freqs, image_freqs, text_freqs

    cfg = _small_cfg()
    g = torch.Generator(device=cuda_device).manual_seed(5)
    blk = SingleStreamBlock(cfg, g, cuda_device)
    B = 2
    cg = gen(6)
    x = torch.randn(B, cfg.tokens, cfg.hidden, generator=cg).to(torch.bfloat16)
    vec = torch.randn(B, cfg.hidden, generator=cg).to(torch.bfloat16)
    f = batch_freqs(torch.cat([text_freqs(cfg, cuda_device), image_freqs(cfg, cuda_device)]), B)
    with torch.no_grad():
        o = blk(x.to(cuda_device), vec.to(cuda_device), f)
        r = OD.single_block(blk, x, vec, f)
    _close(o, r)


def test_dit_forward_and_euler(cuda_device):
    from futudiffu_b200.dit import DiT, euler_step

    cfg = _small_cfg(n_double=2, n_single=2, img_grid=(8, 8))
    model = DiT(cfg, seed=7, device=cuda_device)
    B = 2
    cg = gen(8)
    img = torch.randn(B, cfg.img_tokens, cfg.patch_dim, generator=cg).to(torch.bfloat16)
    txt = torch.randn(B, cfg.txt_tokens, cfg.hidden, generator=cg).to(torch.bfloat16)
    t = torch.tensor([0.9, 0.3])
    v = model(img.to(cuda_device), txt.to(cuda_device), t.to(cuda_device))
    assert v.shape == (B, cfg.img_tokens, cfg.patch_dim)
    _close(v, OD.dit_forward(model, img, txt, t), cos_min=0.995)
    x1 = euler_step(model, img.to(cuda_device), txt.to(cuda_device), 1.0, 0.5)
    assert torch.isfinite(x1.float()).all() and x1.shape == img.shape


def test_euler_step_graph_matches_eager(cuda_device):
    """The CUDA-graph replay of an Euler step gives the eager step's output bit for
    bit, step after step (new inputs and sigmas each call)."""
    from futudiffu_b200.dit import DiT, EulerStepGraph, euler_denoise, euler_step, sigmas

    cfg = _small_cfg(n_double=1, n_single=2, img_grid=(8, 8))
    model = DiT(cfg, seed=3, device=cuda_device)
    cg = gen(12)
    img = torch.randn(2, cfg.img_tokens, cfg.patch_dim, generator=cg).to(torch.bfloat16).to(cuda_device)
    txt = torch.randn(2, cfg.txt_tokens, cfg.hidden, generator=cg).to(torch.bfloat16).to(cuda_device)
    g = EulerStepGraph(model, img, txt)
    s = sigmas(4)
    xe, xg = img, img
    for i in range(4):
        xe = euler_step(model, xe, txt, s[i], s[i + 1])
        xg = g(xg, txt, s[i], s[i + 1]).clone()
        assert torch.equal(xe, xg), i
    assert torch.equal(euler_denoise(model, img, txt, steps=4, graph=True), xe)


def test_video_block_single_rank(cuda_device):
    """Video DiT block (Ulysses path at P = 1) against the CPU composition of the oracle ops."""
    from futudiffu_b200.dit import VideoBlock, VideoDiTConfig, video_freqs

    cfg = VideoDiTConfig(hidden=256, heads=2, ffn=512, n_blocks=1, grid=(2, 4, 24), txt_tokens=64,
                         rope_axes=(44, 42, 42))
    g = torch.Generator(device=cuda_device).manual_seed(9)
    blk = VideoBlock(cfg, g, cuda_device)
    cg = gen(10)
    L = cfg.tokens
    x = torch.randn(1, L, cfg.hidden, generator=cg).to(torch.bfloat16)
    vec = torch.randn(1, cfg.hidden, generator=cg).to(torch.bfloat16)
    txt = torch.randn(1, cfg.txt_tokens, cfg.hidden, generator=cg).to(torch.bfloat16)
    fr = video_freqs(cfg, cuda_device).unsqueeze(0).contiguous()
    with torch.no_grad():
        o = blk(x.to(cuda_device), vec.to(cuda_device), txt.to(cuda_device), fr)
        r = OD.video_block(blk, x, vec, txt, fr)
    _close(o, r)


def test_video_dit_forward(cuda_device):
    from futudiffu_b200.dit import VideoDiT, VideoDiTConfig

    cfg = VideoDiTConfig(hidden=256, heads=2, ffn=512, n_blocks=2, grid=(2, 4, 8), txt_tokens=32)
    model = VideoDiT(cfg, seed=3, device=cuda_device)
    cg = gen(11)
    x = torch.randn(1, cfg.tokens, cfg.patch_dim, generator=cg).to(torch.bfloat16).to(cuda_device)
    txt = torch.randn(1, cfg.txt_tokens, cfg.hidden, generator=cg).to(torch.bfloat16).to(cuda_device)
    v1 = model(x, txt, torch.tensor([0.5], device=cuda_device))
    v2 = model(x, txt, torch.tensor([0.5], device=cuda_device))
    assert v1.shape == (1, cfg.tokens, cfg.patch_dim) and torch.isfinite(v1.float()).all()
    assert torch.equal(v1, v2)
