"""Multi-LoRA on the tcgen05 GEMM vs the restated reference (MultiLoRALinear,
src_ii/multi_lora.py:231-325; _multi_lora_kernel, lora_kernels.py:55-157)."""

from __future__ import annotations

import pytest
import torch

from oracle import gemm as OG
from oracle import lora as OL
from oracle import quant as OQ
from tests.conftest import gen
from tests.helpers import cosine

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _triton_division():
    from oracle import quant as _OQ
    from tests.helpers import triton_divide

    with _OQ.division(triton_divide):
        yield


def _close(a, b, cos_min=0.9999, rel=0.02):
    af, bf = a.float().cpu(), b.float().cpu()
    assert torch.isfinite(af).all()
    assert cosine(af, bf) >= cos_min
    assert (af - bf).abs().max().item() <= rel * bf.abs().max().item() + 1e-3


@pytest.mark.parametrize("B,S,IN,OUT,N,R", [(2, 33, 256, 384, 3, 16), (1, 300, 512, 256, 4, 8), (3, 7, 128, 128, 1, 64)])
def test_multi_lora_forward(cuda_device, B, S, IN, OUT, N, R):
    from futudiffu_b200.lora_kernels import multi_lora_forward

    g = gen(B * S + N)
    x = torch.randn(B, S, IN, generator=g).to(torch.bfloat16)
    A = (torch.randn(N, R, IN, generator=g) * 0.05).to(torch.bfloat16)
    Bm = (torch.randn(N, OUT, R, generator=g) * 0.05).to(torch.bfloat16)
    sc = torch.rand(B, N, generator=g)
    sc[0, 0] = 0.0  # a skipped (batch, adapter) pair
    d = multi_lora_forward(x.to(cuda_device), A.to(cuda_device), Bm.to(cuda_device), sc.to(cuda_device))
    eff = sc.repeat_interleave(S, dim=0)
    ref = OL.adapter_delta(x.reshape(-1, IN), list(A), list(Bm), eff).reshape(B, S, OUT)
    _close(d, ref)


@pytest.mark.parametrize("bias", [False, True])
def test_multi_lora_linear_fused_fp8(cuda_device, bias):
    """FP8 base GEMM + adapter delta in one kernel, per-image routing with padding tokens."""
    from futudiffu_b200.fp8 import FP8Linear, quantize_fp8_blockwise_cuda
    from futudiffu_b200.multi_lora import MultiLoRALinear

    g = gen(21)
    IN, OUT, T = 512, 768, 200
    w8, ws = quantize_fp8_blockwise_cuda((torch.randn(OUT, IN, generator=g) * 0.02).to(cuda_device))
    bvec = (torch.randn(OUT, generator=g) * 0.1).to(torch.bfloat16).to(cuda_device) if bias else None
    lin = MultiLoRALinear(FP8Linear(w8, ws, bvec), max_adapters=3, max_rank=16)
    torch.manual_seed(0)
    lin.assign_adapter(0, "a", rank=16, alpha=8.0)
    lin.assign_adapter(2, "c", rank=8, alpha=4.0)
    for j in (0, 2):
        lin.lora_B[j].data.copy_((torch.randn(OUT, 16, generator=g) * 0.05).to(torch.bfloat16))
    x = torch.randn(1, T, IN, generator=g).to(torch.bfloat16)
    routing = torch.cat([torch.zeros(90), torch.ones(100), -torch.ones(10)]).long()  # two images + padding
    scales = torch.tensor([[1.0, 0.0, 0.5], [0.25, 1.0, 2.0]])
    y = lin(x.to(cuda_device), scales.to(cuda_device), routing.to(cuda_device))
    # reference: bf16 FP8-linear output + bf16 adapter delta
    a8, a_s = OQ.act_quant(x.reshape(-1, IN))
    base = OG.gemm_blockwise(a8, a_s, w8.cpu(), ws.cpu(), bias=None if bvec is None else bvec.cpu())
    eff = OL.effective_scales(T, scales, routing, lin._lora_scalings.cpu(), lin._slot_active.cpu())
    delta = OL.adapter_delta(x.reshape(-1, IN), [p.data for p in lin.lora_A], [p.data for p in lin.lora_B], eff)
    ref = (base + delta).reshape(1, T, OUT)
    _close(y, ref)
    # adapter_delta alone, and no scales -> base only
    _close(lin.adapter_delta(x.to(cuda_device), scales.to(cuda_device), routing.to(cuda_device)),
           delta.reshape(1, T, OUT), cos_min=0.999, rel=0.03)
    _close(lin(x.to(cuda_device)), base.reshape(1, T, OUT), cos_min=0.99999, rel=0.01)
