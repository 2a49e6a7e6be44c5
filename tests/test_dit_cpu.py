"""Host-side layout of the DiT workload on CPU: the stacked adaLN modulation.

``DiT.modulations`` computes every block's adaLN(SiLU(vec)) with one batched GEMM
over a (C, D, D) weight stack whose chunks the blocks' own adaLN parameters view.
The FP8 linears need the GPU quantiser, so they are stubbed here; the adaLN
linears, the stacking and the chunk order are plain torch.
"""

from __future__ import annotations

import torch
from torch import nn


class _StubLinear(nn.Module):
    def __init__(self, out_f: int, in_f: int):
        super().__init__()
        self.weight = torch.zeros(out_f, in_f)
        self.bias = None


def _tiny_dit(monkeypatch):
    import futudiffu_b200.dit as D

    monkeypatch.setattr(D, "random_fp8_linear", lambda n, k, gen, dev, *a, **kw: _StubLinear(n, k))
    cfg = D.DiTConfig(hidden=256, heads=2, n_double=2, n_single=3, txt_tokens=16, img_grid=(8, 8))
    return D.DiT(cfg, seed=0, device="cpu")


def test_modulations_equal_per_block_linears(monkeypatch):
    m = _tiny_dit(monkeypatch)
    vec = torch.randn(3, 256, generator=torch.Generator().manual_seed(1)).to(torch.bfloat16)
    mods = m.modulations(vec)
    assert mods.shape == (2 * 8 + 3 * 2, 3, 256) and mods.is_contiguous()
    c = 0
    for blk in m.double_blocks:
        for st in (blk.txt, blk.img):          # text stream's four chunks, then the image stream's
            for k, ref in enumerate(st.modulation(vec)):
                assert torch.equal(mods[c + k], ref), (c, k)
            c += 4
    for blk in m.single_blocks:                # (scale, gate)
        for k, ref in enumerate(blk.adaln(torch.nn.functional.silu(vec)).chunk(2, dim=-1)):
            assert torch.equal(mods[c + k], ref), (c, k)
        c += 2
    assert c == m.mod_w.shape[0]


def test_block_adaln_parameters_view_the_stack(monkeypatch):
    m = _tiny_dit(monkeypatch)
    D = 256
    first = m.double_blocks[0].txt.adaln
    last = m.single_blocks[-1].adaln
    assert first.weight.data_ptr() == m.mod_w.data_ptr() and first.weight.shape == (4 * D, D)
    assert last.bias.data_ptr() == m.mod_b[-2].data_ptr() and last.weight.shape == (2 * D, D)
    # a change through the stack is seen by the block, and the reverse
    with torch.no_grad():
        m.mod_w[-1, 0, 0] = 7.0
        assert last.weight[D, 0].item() == 7.0
        first.bias[5] = -3.0
        assert m.mod_b[0, 0, 5].item() == -3.0


def test_modulations_follow_replaced_parameters(monkeypatch):
    """load_state_dict(assign=True) replaces the adaLN parameters, so they stop
    viewing the stack: the next modulations() restacks and uses the new weights."""
    m = _tiny_dit(monkeypatch)
    vec = torch.randn(2, 256, generator=torch.Generator().manual_seed(2)).to(torch.bfloat16)
    sd = {k: v.clone() for k, v in m.state_dict().items()}
    key = "single_blocks.1.adaln.weight"
    sd[key] = torch.randn(sd[key].shape, generator=torch.Generator().manual_seed(3)).to(torch.bfloat16)
    m.load_state_dict(sd, strict=False, assign=True)
    mods = m.modulations(vec)
    blk = m.single_blocks[1]
    assert torch.equal(blk.adaln.weight, sd[key])
    assert blk.adaln.weight.data_ptr() == m.mod_w[16 + 2].data_ptr()   # a view of the new stack
    for k, ref in enumerate(blk.adaln(torch.nn.functional.silu(vec)).chunk(2, dim=-1)):
        assert torch.equal(mods[16 + 2 + k], ref)
    # in place: no restack needed, the views carry the values
    with torch.no_grad():
        m.double_blocks[0].img.adaln.bias.add_(1.0)
    ref = m.double_blocks[0].img.modulation(vec)
    mods = m.modulations(vec)
    assert all(torch.equal(mods[4 + k], ref[k]) for k in range(4))


def test_f32_norm_copies_follow_the_parameters(monkeypatch):
    import futudiffu_b200.dit as D

    m = _tiny_dit(monkeypatch)
    for st in (m.double_blocks[0].txt, m.double_blocks[1].img, m.single_blocks[2]):
        q32, k32 = D.f32_norms(st)
        assert q32.dtype == torch.float32 and torch.equal(q32, st.q_norm.float())
        assert torch.equal(k32, st.k_norm.float())
        assert D.f32_norms(st)[0] is q32                     # cached while unchanged
        with torch.no_grad():
            st.q_norm.mul_(2.0)                              # in place: version counter moves
        assert torch.equal(D.f32_norms(st)[0], st.q_norm.float())
        st.k_norm = torch.nn.Parameter(st.k_norm.detach() + 1, requires_grad=False)   # replaced
        assert torch.equal(D.f32_norms(st)[1], st.k_norm.float())
