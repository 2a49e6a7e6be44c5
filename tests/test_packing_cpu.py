"""Packed-forward host logic vs the reference's own outputs (tests/golden/packing.pt,
made by tests/golden/make_golden.py from src_ii.bin_packer, src_ii.transformer,
src_ii.forward_packed and src_ii.triumphant_future_reduction_ops)."""

from __future__ import annotations

from pathlib import Path

import pytest
import torch

from futudiffu_b200 import bin_packer as BP
from futudiffu_b200 import forward_packed as FP
from futudiffu_b200 import transformer as T

G = torch.load(Path(__file__).parent / "golden" / "packing.pt", weights_only=False)


def test_constants():
    assert (BP.REFERENCE_SEQ_LEN, BP.DEFAULT_CAP_TOKENS, BP.REFERENCE_TOTAL_LEN) == G["constants"]


def test_pack_matches_reference():
    sched = BP.BinPackScheduler()
    for items, want, eff in zip(G["item_lists"], G["packs"], G["effs"]):
        bins = sched.pack(items)
        assert [[it["id"] for it in b] for b in bins] == want
        assert sched.estimate_efficiency(bins) == eff


def test_pack_generation_plan_and_training():
    bins = BP.BinPackScheduler(max_seq_len=6000).pack_generation_plan(G["plan"])
    got = [[(it["id"], it["seq_len"], it["img_seq_len"], it["cap_tokens"]) for it in b] for b in bins]
    assert got == G["plan_bins"]
    assert BP.BinPackScheduler().pack_for_training(G["training_items"]) == G["training"]


def test_pack_properties():
    sched = BP.BinPackScheduler(max_seq_len=1000)
    assert sched.pack([]) == []
    items = [{"seq_len": s} for s in (1200, 500, 500, 400, 100, 999)]
    bins = sched.pack(items)
    assert [sum(it["seq_len"] for it in b) for b in bins] == [1200, 999, 1000, 500]
    for b in bins[1:]:
        assert sum(it["seq_len"] for it in b) <= 1000
    with pytest.raises(ValueError):
        BP.BinPackScheduler(max_seq_len=0)


@pytest.mark.parametrize("wh,ok", [((1280, 832), True), ((48, 64), False), ((1280, 840), False), ((0, 64), False)])
def test_validate_resolution(wh, ok):
    if ok:
        BP.validate_resolution(*wh)
    else:
        with pytest.raises(ValueError):
            BP.validate_resolution(*wh)


def test_build_packed_sequence_and_rope():
    packed, info = T.build_packed_sequence(G["caps"], G["imgs"], G["grids"], [40, 113, 7], 32, G["cap_pad"],
                                           G["x_pad"])
    assert torch.equal(packed, G["packed"])
    assert info.segments == G["segments"]
    assert torch.equal(info.document_id, G["document_id"])
    rope = T.build_packed_rope(info, device="cpu")
    assert torch.equal(rope, G["rope"])
    info, rope_p = FP._pad_plan_to_fixed_len(info, rope, 768)
    assert torch.equal(info.document_id, G["doc_padded"]) and tuple(rope_p.shape) == G["rope_padded_shape"]
    assert torch.equal(rope_p[:, :rope.shape[1]], rope) and not rope_p[:, rope.shape[1]:].any()
    with pytest.raises(ValueError):
        FP._pad_plan_to_fixed_len(info, rope_p, 512)


def test_row_ranges_cover_padding_as_image_zero():
    doc = G["doc_padded"]
    r = T.row_ranges(doc, device="cpu")
    rows, param = r.rows.tolist(), r.param.tolist()
    assert rows[0] == 0 and rows[-1] == doc.numel()
    d = doc.clone()
    d[d < 0] = 0
    for i, p in enumerate(param):
        assert (d[rows[i]:rows[i + 1]] == p).all()
    assert r.n_params == int(doc.max()) + 1


def test_euler_ops():
    assert torch.equal(FP.euler_step(G["x"], G["guided"], torch.tensor(0.7), torch.tensor(0.55)), G["euler"])
    got = FP.denoise_all([G["x"], G["guided"]], [G["guided"], G["x"]], [torch.tensor(0.3), torch.tensor(0.9)])
    assert all(torch.equal(a, b) for a, b in zip(got, G["denoised"]))
