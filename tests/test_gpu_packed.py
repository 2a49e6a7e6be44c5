"""GPU parity of the packed multi-image path: row-range norm kernels, the
reference's JointTransformerBlock (src_ii/transformer.py:588-701) in its
per-batch and per-token adaLN forms, and a packed bin vs its images run alone."""

from __future__ import annotations

import pytest
import torch

from oracle import fused as OF
from oracle import transformer as OT
from tests.conftest import gen
from tests.helpers import cosine

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _triton_division():
    from oracle import quant as _OQ
    from tests.helpers import triton_divide

    with _OQ.division(triton_divide):
        yield


def _ranges(seg_lens, device):
    from futudiffu_b200.transformer import row_ranges

    doc = torch.cat([torch.full((n,), i, dtype=torch.int32) for i, n in enumerate(seg_lens)])
    return doc, row_ranges(doc, device=device)


@pytest.mark.parametrize("dim", [512, 3840])
def test_range_norms_equal_per_segment_kernels(cuda_device, dim):
    """Each row range of the packed kernels gives exactly what the per-sample
    kernel gives for that segment, and matches the oracle."""
    from futudiffu_b200 import fused_kernels as FK

    seg = [300, 45, 1000, 7]
    doc, r = _ranges(seg, cuda_device)
    Lt = sum(seg)
    g = gen(dim)
    x = torch.randn(Lt, dim, generator=g).to(torch.bfloat16).to(cuda_device)
    res = torch.randn(Lt, dim, generator=g).to(torch.bfloat16).to(cuda_device)
    w = (1 + 0.1 * torch.randn(dim, generator=g)).to(torch.bfloat16).to(cuda_device)
    sc = (0.5 * torch.randn(len(seg), dim, generator=g)).to(torch.bfloat16).to(cuda_device)
    gt = torch.randn(len(seg), dim, generator=g).to(torch.bfloat16).to(cuda_device)
    y = FK.rms_norm_modulate_ranges(x, w, sc, r.rows, r.param)
    q8, qs = FK.rms_norm_modulate_quant_ranges(x, w, sc, r.rows, r.param)
    gr = FK.rms_norm_gate_residual_ranges(x, w, gt, res, r.rows, r.param)
    o = 0
    for i, n in enumerate(seg):
        xs = x[o:o + n].unsqueeze(0).contiguous()
        assert torch.equal(y[o:o + n], FK.fused_rms_norm_modulate(xs, w, sc[i:i + 1].contiguous())[0])
        c8, cs = FK.fused_rms_norm_modulate_quant(xs, w, sc[i:i + 1].contiguous())
        assert torch.equal(q8[o:o + n].view(torch.uint8), c8[0].view(torch.uint8))
        assert torch.equal(qs[o:o + n], cs[0])
        ref = FK.fused_rms_norm_gate_residual(xs, w, gt[i:i + 1].contiguous(), res[o:o + n].unsqueeze(0).contiguous())
        assert torch.equal(gr[o:o + n], ref[0])
        o += n
    # the oracle on the gathered per-token rows
    tok = sc[doc.long().to(cuda_device)]
    want = OF.rms_norm_modulate(x.cpu().unsqueeze(1), w.cpu(), tok.cpu())
    assert cosine(y.cpu(), want.squeeze(1)) > 0.99999


def test_ranges_skip_out_of_bounds(cuda_device):
    """A range past the end of x or naming a missing parameter row writes nothing."""
    from futudiffu_b200 import fused_kernels as FK

    dim = 256
    x = torch.randn(64, dim, device=cuda_device).to(torch.bfloat16)
    w = torch.ones(dim, device=cuda_device, dtype=torch.bfloat16)
    sc = torch.zeros(2, dim, device=cuda_device, dtype=torch.bfloat16)
    rows = torch.tensor([0, 32, 200], dtype=torch.int32, device=cuda_device)   # second range too long
    param = torch.tensor([1, 0], dtype=torch.int32, device=cuda_device)
    y = FK.rms_norm_modulate_ranges(x, w, sc, rows, param)
    ok = FK.rms_norm_modulate_ranges(x[:32].contiguous(), w, sc, rows[:2].contiguous(), param[:1].contiguous())
    assert torch.equal(y[:32], ok)
    param_bad = torch.tensor([5, 0], dtype=torch.int32, device=cuda_device)     # missing parameter row
    rows2 = torch.tensor([0, 32, 64], dtype=torch.int32, device=cuda_device)
    y2 = FK.rms_norm_modulate_ranges(x, w, sc, rows2, param_bad)
    assert torch.equal(y2[32:], FK.rms_norm_modulate_ranges(x[32:].contiguous(), w, sc,
                                                            torch.tensor([0, 32], dtype=torch.int32, device=cuda_device),
                                                            torch.tensor([0], dtype=torch.int32, device=cuda_device)))
    from futudiffu_b200 import check_status
    check_status()


def _block(dim=256, heads=2, seed=0, device=None):
    from futudiffu_b200.transformer import JointTransformerBlock

    torch.manual_seed(seed)
    blk = JointTransformerBlock(0, dim, heads, None, 128, 8.0 / 3.0, 1e-5, qk_norm=True, modulation=True,
                                z_image_modulation=True, device=device, dtype=torch.bfloat16)
    with torch.no_grad():
        for n in (blk.attention_norm1, blk.attention_norm2, blk.ffn_norm1, blk.ffn_norm2,
                  blk.attention.q_norm, blk.attention.k_norm):
            n.weight.copy_(1 + 0.1 * torch.randn_like(n.weight.float()).to(n.weight.dtype))
    return blk.to_fp8()


def _packed_inputs(dim, device, caps=(40, 24, 16), grids=((12, 16), (8, 8), (4, 6)), total=None, seed=3):
    from futudiffu_b200 import forward_packed as FP
    from futudiffu_b200 import transformer as T

    g = gen(seed)
    cap_t = [torch.randn(1, n, dim, generator=g).to(torch.bfloat16) for n in caps]
    img_t = [torch.randn(1, h * w, dim, generator=g).to(torch.bfloat16) for h, w in grids]
    pad = torch.zeros(dim, dtype=torch.bfloat16)
    packed, info = T.build_packed_sequence(cap_t, img_t, list(grids), list(caps), 32, pad, pad)
    rope = T.build_packed_rope(info, device="cpu")
    if total is not None:
        info, rope = FP._pad_plan_to_fixed_len(info, rope, total)
        packed = torch.cat([packed, packed.new_zeros(1, total - packed.shape[1], dim)], 1)
    return packed.to(device), info, rope.to(device)


@pytest.mark.parametrize("per_token", [False, True])
def test_joint_block_vs_oracle(cuda_device, per_token):
    from futudiffu_b200.block_mask import build_block_mask_from_packing_info
    from futudiffu_b200.transformer import per_image_adaln, row_ranges

    dim = 256
    blk = _block(dim, device=cuda_device)
    x, info, rope = _packed_inputs(dim, cuda_device, total=640)
    mask = build_block_mask_from_packing_info(info, device=cuda_device)
    g = gen(11)
    if per_token:
        adaln_in = torch.randn(info.n_images, 256, generator=g).to(torch.bfloat16).to(cuda_device)
        r = row_ranges(info.document_id, n_params=info.n_images, device=cuda_device)
        pre = per_image_adaln(blk, adaln_in, r)
        y = blk(x, None, rope, precomputed_adaln=pre, block_mask=mask)
        d = info.document_id.clone().long()
        d[d < 0] = 0
        scales = tuple(p.params[d.to(cuda_device)].unsqueeze(0) for p in pre)   # the reference's scatter
        # the same per-token rows passed as (1, L, dim) tensors: identical kernel arithmetic
        y3 = blk(x, None, rope, precomputed_adaln=scales, block_mask=mask)
        assert torch.equal(y, y3)
        cos_min = 0.999   # the reference's per-token path is unfused bf16 torch (extra roundings)
    else:
        adaln_in = torch.randn(1, 256, generator=g).to(torch.bfloat16).to(cuda_device)
        scales = blk.adaln_params(adaln_in)
        y = blk(x, None, rope, adaln_input=adaln_in, block_mask=mask)
        cos_min = 0.9995
    want = OT.block_forward(blk, x, rope, scales, mask)
    got = y.float().cpu()
    assert torch.isfinite(got).all()
    c = cosine(got, want.float())
    assert c >= cos_min, c


def test_packed_bin_matches_images_alone(cuda_device):
    """Block-aligned segments: each image's rows of the packed forward equal the
    block run on that image alone (the mask skips every cross-image tile), up to
    the K smoothing mean, which the packed attention takes over the whole bin."""
    from futudiffu_b200.block_mask import build_block_mask, build_block_mask_from_packing_info
    from futudiffu_b200.transformer import per_image_adaln, row_ranges

    dim = 256
    blk = _block(dim, seed=4, device=cuda_device)
    # caption 128 + image 256 per image: every segment a multiple of 128 tokens
    x, info, rope = _packed_inputs(dim, cuda_device, caps=(100, 128), grids=((16, 16), (8, 32)), seed=9)
    mask = build_block_mask_from_packing_info(info, device=cuda_device)
    adaln_in = torch.randn(2, 256, generator=gen(5)).to(torch.bfloat16).to(cuda_device)
    r = row_ranges(info.document_id, n_params=2, device=cuda_device)
    y = blk(x, None, rope, precomputed_adaln=per_image_adaln(blk, adaln_in, r), block_mask=mask)
    for i, (ts, tl, is_, il) in enumerate(info.segments):
        n = tl + il
        xi = x[:, ts:ts + n].contiguous()
        yi = blk(xi, None, rope[:, ts:ts + n].contiguous(), adaln_input=adaln_in[i:i + 1],
                 block_mask=build_block_mask([n], device=cuda_device))
        c = cosine(y[:, ts:ts + n].float().cpu(), yi.float().cpu())
        assert c > 0.999, (i, c)
