"""GPU parity: FP8 quantisers vs the CPU oracle (bit-exact codes and scales)."""

from __future__ import annotations

import pytest
import torch

from oracle import quant as OQ
from tests.conftest import gen
from tests.helpers import e4m3_bits, e4m3_step_diff

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _triton_division():
    """Evaluate the oracle's Triton-kernel quotients with Triton's own fp32 divide on the GPU."""
    from oracle import quant as _OQ
    from tests.helpers import triton_divide

    with _OQ.division(triton_divide):
        yield


def _x(shape, seed, scale=3.0, dtype=torch.bfloat16):
    g = gen(seed)
    row_scale = torch.rand(*shape[:-1], 1, generator=g) * scale + 1e-3
    x = torch.randn(*shape, generator=g) * row_scale
    return x.to(dtype)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("M,K", [(1, 128), (7, 384), (256, 3072), (2048, 3072), (333, 1280)])
def test_act_quant_bit_exact(cuda_device, dtype, M, K):
    from futudiffu_b200.fp8_kernels import fp8_act_quant

    x = _x((M, K), M * 7 + K, dtype=dtype)
    if M > 3:
        x[3, :128] = 0  # all-zero group -> scale 1e-12, codes 0
    y, s = fp8_act_quant(x.to(cuda_device))
    yr, sr = OQ.act_quant(x)
    assert torch.equal(e4m3_bits(y), e4m3_bits(yr))
    assert torch.equal(s.cpu(), sr)


def test_act_quant_batched_shape(cuda_device):
    from futudiffu_b200.fp8_kernels import fp8_act_quant

    x = _x((6, 5, 256), 11).to(cuda_device)
    y, s = fp8_act_quant(x)
    assert y.shape == (6, 5, 256) and s.shape == (6, 5, 2)
    yr, sr = OQ.act_quant(x.cpu())
    assert torch.equal(e4m3_bits(y), e4m3_bits(yr)) and torch.equal(s.cpu(), sr)


def test_act_quant_rejects_bad_k(cuda_device):
    from futudiffu_b200.fp8_kernels import fp8_act_quant

    with pytest.raises(AssertionError):
        fp8_act_quant(torch.zeros(4, 100, device=cuda_device, dtype=torch.bfloat16))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("N,K", [(128, 128), (256, 384), (3072, 3072)])
def test_weight_quant_bit_exact(cuda_device, dtype, N, K):
    from futudiffu_b200.fp8 import quantize_fp8_blockwise_cuda

    w = (torch.randn(N, K, generator=gen(N + K)) * 0.02).to(dtype)
    w[:128, :128] = 0
    q, s = quantize_fp8_blockwise_cuda(w.to(cuda_device))
    qr, sr = OQ.weight_quant(w)
    assert torch.equal(e4m3_bits(q), e4m3_bits(qr))
    assert torch.equal(s.cpu(), sr)


def test_weight_quant_golden(cuda_device, golden_dir):
    from futudiffu_b200.fp8 import quantize_fp8_blockwise

    d = torch.load(golden_dir / "weight_quant.pt")
    q, s = quantize_fp8_blockwise(d["w"])  # CPU in, CUDA compute, CPU out (reference contract)
    assert q.device.type == "cpu"
    assert torch.equal(e4m3_bits(q), e4m3_bits(d["codes"]))
    assert torch.equal(s, d["scales"])


@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_dequant_golden(cuda_device, golden_dir, out_dtype):
    from futudiffu_b200.fp8 import dequantize_fp8_blockwise

    d = torch.load(golden_dir / "dequant.pt")
    out = dequantize_fp8_blockwise(d["codes"].to(cuda_device), d["scales"].to(cuda_device), output_dtype=out_dtype)
    ref = OQ.dequant_blockwise(d["codes"], d["scales"], out_dtype=out_dtype)
    assert torch.equal(out.cpu(), ref)
    if out_dtype == torch.bfloat16:
        assert torch.equal(out.cpu().view(torch.int16), d["out"].view(torch.int16))


@pytest.mark.parametrize("M,N", [(1, 128), (4, 256), (300, 10240), (2048, 1280)])
def test_silu_gate_quant(cuda_device, M, N):
    from futudiffu_b200.fp8_kernels import fp8_silu_gate_quant

    x = (torch.randn(M, 2 * N, generator=gen(M + N)) * 2).to(torch.bfloat16)
    y, s = fp8_silu_gate_quant(x.to(cuda_device))
    yr, sr = OQ.silu_gate_quant(x)
    # exp differs from the CPU's by an ulp at most: scales to 1e-6, codes within one step
    assert torch.allclose(s.cpu(), sr, rtol=2e-6, atol=0)
    diff = e4m3_step_diff(y, yr)
    assert diff.max().item() <= 1
    assert (diff == 0).float().mean().item() >= 0.999


def test_silu_gate_golden(cuda_device, golden_dir):
    from futudiffu_b200.fp8_kernels import fp8_silu_gate_quant

    d = torch.load(golden_dir / "silu_gate.pt")
    y, s = fp8_silu_gate_quant(d["x"].to(cuda_device))
    assert torch.allclose(s.cpu(), d["scales"], rtol=2e-6, atol=0)
    assert e4m3_step_diff(y, d["codes"]).max().item() <= 1


def test_silu_gate_batched(cuda_device):
    from futudiffu_b200.fp8_kernels import fp8_silu_gate_quant

    x = torch.randn(2, 3, 512, generator=gen(5)).to(torch.bfloat16).to(cuda_device)
    y, s = fp8_silu_gate_quant(x)
    assert y.shape == (2, 3, 256) and s.shape == (2, 3, 2)


@pytest.mark.parametrize("M,N", [(3, 128), (4608, 12288)])
def test_gelu_tanh_quant(cuda_device, M, N):
    from futudiffu_b200.fp8_kernels import fp8_gelu_tanh_quant

    x = (torch.randn(M, N, generator=gen(M)) * 2).to(torch.bfloat16)
    y, s = fp8_gelu_tanh_quant(x.to(cuda_device))
    yr, sr = OQ.gelu_tanh_quant(x)
    assert torch.allclose(s.cpu(), sr, rtol=1e-5, atol=0)
    diff = e4m3_step_diff(y, yr)
    assert diff.max().item() <= 1 and (diff == 0).float().mean().item() >= 0.999


def test_gelu_requant(cuda_device):
    from futudiffu_b200.fp8_kernels import fp8_act_quant, fp8_gelu

    x = (torch.randn(64, 512, generator=gen(9)) * 3).to(torch.bfloat16).to(cuda_device)
    x8, sx = fp8_act_quant(x)
    y, sy = fp8_gelu(x8, sx)
    yr, syr = OQ.gelu_requant(x8.cpu(), sx.cpu())
    assert torch.allclose(sy.cpu(), syr, rtol=1e-5, atol=0)
    diff = e4m3_step_diff(y, yr)
    assert diff.max().item() <= 1 and (diff == 0).float().mean().item() >= 0.999


def test_quant_no_device_fault_status(cuda_device):
    from futudiffu_b200 import check_status

    check_status()


def test_device_divide_within_two_ulp_of_ieee(cuda_device):
    from futudiffu_b200._lib import device_divide

    g = gen(123)
    a = torch.rand(1 << 20, generator=g) * 500
    b = torch.rand(1 << 20, generator=g) * 20 + 1e-6
    got = device_divide(a, b)
    ref = OQ.div_ieee(a, b)
    ulp = (got.view(torch.int32) - ref.view(torch.int32)).abs()
    assert ulp.max().item() <= 2
    assert (device_divide(torch.tensor([448.0]), torch.tensor([448.0])) == 1.0).all()


def test_device_divide_equals_triton_divide(cuda_device):
    """The library's f32 divide gives Triton's quotient bit for bit (the quantisers
    use it for every scale; the reference's kernels use Triton's `/`)."""
    from futudiffu_b200._lib import device_divide
    from tests.helpers import triton_divide

    g = gen(124)
    a = torch.cat([torch.rand(1 << 20, generator=g) * 500, torch.full((4,), 448.0), torch.full((4,), 127.0)])
    b = torch.cat([torch.rand(1 << 20, generator=g) * 20 + 1e-6, torch.tensor([448.0, 3.0, 1e-12, 7.0]),
                   torch.tensor([127.0, 3.0, 1e-12, 0.1])])
    assert torch.equal(device_divide(a, b).view(torch.int32), triton_divide(a, b).view(torch.int32))
