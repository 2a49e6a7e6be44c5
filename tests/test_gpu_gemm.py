"""GPU parity: tcgen05 FP8 blockwise GEMM vs the CPU oracle (per-128-K promotion)."""

from __future__ import annotations

import pytest
import torch

from oracle import gemm as OG
from oracle import quant as OQ
from tests.conftest import gen
from tests.helpers import cosine

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _triton_division():
    """Evaluate the oracle's Triton-kernel quotients with Triton's own fp32 divide on the GPU."""
    from oracle import quant as _OQ
    from tests.helpers import triton_divide

    with _OQ.division(triton_divide):
        yield


def _operands(M, N, K, seed, b_layout=0):
    g = gen(seed)
    x = torch.randn(M, K, generator=g).to(torch.bfloat16)
    w = (torch.randn(N, K, generator=g) * 0.02).to(torch.bfloat16)
    a8, a_s = OQ.act_quant(x)
    if b_layout == 2:
        b8, bs = OQ.act_quant(w.reshape(-1, 128))  # per-row scale requires one group per row
        b8 = b8.reshape(N, K)
        bs = torch.rand(N, generator=g) * 1e-3 + 1e-4
    else:
        Np = (N + 127) // 128 * 128
        wp = torch.nn.functional.pad(w.float(), (0, 0, 0, Np - N))
        b8, bs = OQ.weight_quant(wp)
        b8 = b8[:N].contiguous()
        if b_layout == 1:
            b8 = b8.t().contiguous()
            bs = bs.t().contiguous()
    return a8, a_s, b8, bs


def _check(c, ref, tight=True):
    cf, rf = c.float().cpu(), ref.float()
    assert torch.isfinite(cf).all()
    assert cosine(cf, rf) >= 0.99999
    err = (cf - rf).abs().max().item()
    bound = 2 ** -7 * rf.abs().max().item() + 1e-3
    assert err <= bound, (err, bound)


@pytest.mark.parametrize(
    "M,N,K",
    [(1, 128, 128), (128, 128, 128), (129, 256, 256), (100, 144, 384), (256, 3072, 3072),
     (2048, 3072, 3072), (777, 1280, 1024), (4608, 512, 640)],
)
def test_gemm_blockwise(cuda_device, M, N, K):
    from futudiffu_b200.fp8_kernels import fp8_gemm_blockwise

    a8, a_s, b8, bs = _operands(M, N, K, M + N + K)
    c = fp8_gemm_blockwise(a8.to(cuda_device), a_s.to(cuda_device), b8.to(cuda_device), bs.to(cuda_device))
    assert c.dtype == torch.bfloat16 and c.shape == (M, N)
    _check(c, OG.gemm_blockwise(a8, a_s, b8, bs))


@pytest.mark.parametrize("out_dtype", [torch.float32, torch.float16])
@pytest.mark.parametrize("bias_dtype", [None, torch.bfloat16, torch.float32])
def test_addmm_dtypes(cuda_device, out_dtype, bias_dtype):
    from futudiffu_b200.fp8_kernels import fp8_addmm_blockwise

    M, N, K = 200, 384, 512
    a8, a_s, b8, bs = _operands(M, N, K, 3)
    bias = None if bias_dtype is None else torch.randn(N, generator=gen(4)).to(bias_dtype)
    d = lambda t: None if t is None else t.to(cuda_device)  # noqa: E731
    c = fp8_addmm_blockwise(d(a8), d(a_s), d(b8), d(bs), bias=d(bias), output_dtype=out_dtype)
    assert c.dtype == out_dtype
    _check(c, OG.gemm_blockwise(a8, a_s, b8, bs, bias=bias, out_dtype=torch.float32))


def test_gemm_v1t_and_rowwise(cuda_device):
    from futudiffu_b200.fp8_kernels import fp8_addmm_v1t, fp8_gemm_rowwise, fp8_gemm_v1t

    M, N, K = 300, 512, 768
    a8, a_s, b8, bs = _operands(M, N, K, 8, b_layout=1)
    d = lambda t: t.to(cuda_device)  # noqa: E731
    _check(fp8_gemm_v1t(d(a8), d(a_s), d(b8), d(bs)), OG.gemm_blockwise(a8, a_s, b8, bs, b_layout=1))
    bias = torch.randn(N, generator=gen(2)).to(torch.bfloat16)
    _check(fp8_addmm_v1t(d(a8), d(a_s), d(b8), d(bs), bias=d(bias)),
           OG.gemm_blockwise(a8, a_s, b8, bs, bias=bias, b_layout=1))
    a8, a_s, b8, bs = _operands(M, N, K, 9, b_layout=2)
    _check(fp8_gemm_rowwise(d(a8), d(a_s), d(b8), d(bs)), OG.gemm_blockwise(a8, a_s, b8, bs, b_layout=2))


def test_gemm_batched_input_and_quant(cuda_device):
    from futudiffu_b200.fp8_kernels import fp8_act_quant, fp8_gemm_blockwise, fp8_gemm_quant

    x = torch.randn(2, 65, 256, generator=gen(1)).to(torch.bfloat16).to(cuda_device)
    w = (torch.randn(384, 256, generator=gen(2)) * 0.02)
    b8, bs = OQ.weight_quant(w)
    a8, a_s = fp8_act_quant(x)
    c = fp8_gemm_blockwise(a8, a_s, b8.to(cuda_device), bs.to(cuda_device))
    assert c.shape == (2, 65, 384)
    ref = OG.gemm_blockwise(a8.cpu(), a_s.cpu(), b8, bs).reshape(2, 65, 384)
    _check(c, ref)
    q, qs = fp8_gemm_quant(a8, a_s, b8.to(cuda_device), bs.to(cuda_device))
    assert q.shape == (2, 65, 384) and qs.shape == (2, 65, 3)
    rq, rs = OQ.act_quant(OG.gemm_blockwise(a8.cpu(), a_s.cpu(), b8, bs, out_dtype=torch.float32))
    assert cosine(q.float().cpu() * qs.cpu().repeat_interleave(128, -1), rq.float().reshape(2, 65, 384)
                  * rs.reshape(2, 65, 3).repeat_interleave(128, -1)) > 0.999


def test_fp8_linear_module(cuda_device):
    from futudiffu_b200.fp8 import FP8Linear, quantize_fp8_blockwise_cuda

    K, N = 512, 1024
    w = (torch.randn(N, K, generator=gen(3)) * 0.02).to(cuda_device)
    w8, ws = quantize_fp8_blockwise_cuda(w)
    bias = torch.randn(N, generator=gen(4)).to(torch.bfloat16).to(cuda_device)
    lin = FP8Linear(w8, ws, bias=bias)
    x = torch.randn(2, 100, K, generator=gen(5)).to(torch.bfloat16).to(cuda_device)
    out_op = lin(x)
    out_eager = lin._forward_eager(x)
    assert cosine(out_op, out_eager) > 0.9999  # reference test threshold (fp8.py:656)
    assert torch.equal(out_op, out_eager)
    ref = x.float() @ (w8.float() * ws.repeat_interleave(128, 0).repeat_interleave(128, 1)).T + bias.float()
    assert cosine(out_op, ref) > 0.999
    lin.transpose_weight()
    assert cosine(lin(x), out_op) > 0.99999


def test_fp8_linear_backward(cuda_device):
    from futudiffu_b200.fp8 import FP8Linear, dequantize_fp8_blockwise, quantize_fp8_blockwise_cuda

    w = (torch.randn(256, 384, generator=gen(6)) * 0.02).to(cuda_device)
    w8, ws = quantize_fp8_blockwise_cuda(w)
    lin = FP8Linear(w8, ws)
    x = torch.randn(4, 384, generator=gen(7)).to(torch.bfloat16).to(cuda_device).requires_grad_(True)
    lin(x).float().sum().backward()
    expect = torch.ones(4, 256, device=cuda_device, dtype=torch.bfloat16) @ dequantize_fp8_blockwise(w8, ws)
    assert torch.allclose(x.grad.float(), expect.float(), rtol=1e-2, atol=1e-2)


def test_gemm_zero_rows(cuda_device):
    from futudiffu_b200.fp8_kernels import fp8_gemm_blockwise

    a8 = torch.zeros(0, 256, dtype=torch.float8_e4m3fn, device=cuda_device)
    a_s = torch.zeros(0, 2, device=cuda_device)
    b8 = torch.zeros(128, 256, dtype=torch.float8_e4m3fn, device=cuda_device)
    bs = torch.ones(1, 2, device=cuda_device)
    assert fp8_gemm_blockwise(a8, a_s, b8, bs).shape == (0, 128)


def test_gemm_status_clean(cuda_device):
    from futudiffu_b200 import check_status

    check_status()


# ------------------------------------------------------------------ fused quantising epilogues
def _e4m3(t):
    return t.view(torch.uint8).cpu()


@pytest.mark.parametrize("M,N,K", [(1, 128, 128), (129, 256, 384), (777, 1280, 1024), (2048, 3072, 3072)])
def test_gemm_quant_epilogue(cuda_device, M, N, K):
    """fp8_gemm_quant: the fp32 accumulator requantised in the epilogue equals the
    f32 GEMM followed by the 1 x 128 quantiser, code for code."""
    from futudiffu_b200 import fp8_kernels as FK

    a8, a_s, b8, bs = (t.to(cuda_device) for t in _operands(M, N, K, seed=11))
    c, c_s = FK.fp8_gemm_quant(a8, a_s, b8, bs)
    acc = FK.fp8_gemm_blockwise(a8, a_s, b8, bs, output_dtype=torch.float32)
    y, s = FK.fp8_act_quant(acc)
    assert c_s.shape == (M, N // 128)
    assert torch.equal(_e4m3(c), _e4m3(y))
    assert torch.equal(c_s.cpu(), s.reshape(M, N // 128).cpu())
    # and against the oracle: the oracle's fp32 accumulation order differs, so
    # codes may move by one e4m3 step where the product sits on a rounding edge
    ref_acc = OG.gemm_blockwise(a8.cpu(), a_s.cpu(), b8.cpu(), bs.cpu(), out_dtype=torch.float32)
    ry, rs = OQ.act_quant(ref_acc)
    from tests.helpers import e4m3_step_diff

    assert e4m3_step_diff(c.cpu(), ry).max() <= 1
    torch.testing.assert_close(c_s.cpu(), rs.reshape(M, N // 128), rtol=1e-5, atol=0)


@pytest.mark.parametrize("bias", [False, True])
@pytest.mark.parametrize("M,N,K", [(1, 128, 128), (300, 512, 384), (4608, 1024, 768)])
def test_gemm_gelu_tanh_quant_epilogue(cuda_device, M, N, K, bias):
    """GEMM -> bf16 -> GELU(tanh) -> 1 x 128 e4m3 fused equals fp8_addmm + fp8_gelu_tanh_quant."""
    from futudiffu_b200 import fp8_kernels as FK

    a8, a_s, b8, bs = (t.to(cuda_device) for t in _operands(M, N, K, seed=12))
    bvec = (torch.randn(N, generator=gen(5)) * 0.1).to(torch.bfloat16).to(cuda_device) if bias else None
    c, c_s = FK.fp8_gemm_gelu_tanh_quant(a8, a_s, b8, bs, bias=bvec)
    h = FK.fp8_addmm_blockwise(a8, a_s, b8, bs, bias=bvec, output_dtype=torch.bfloat16)
    y, s = FK.fp8_gelu_tanh_quant(h)
    assert torch.equal(_e4m3(c), _e4m3(y))
    assert torch.equal(c_s.cpu(), s.reshape(M, N // 128).cpu())


@pytest.mark.parametrize("bias", [False, True])
@pytest.mark.parametrize("M,H,K", [(1, 128, 128), (257, 384, 256), (2048, 1280, 1024), (4608, 1024, 3072)])
def test_gemm_silu_gate_quant_epilogue(cuda_device, M, H, K, bias):
    """FFN chain head fused: equals fp8_addmm (M, 2H) bf16 -> fp8_silu_gate_quant, code for code."""
    from futudiffu_b200 import fp8_kernels as FK

    a8, a_s, b8, bs = (t.to(cuda_device) for t in _operands(M, 2 * H, K, seed=13))
    bvec = (torch.randn(2 * H, generator=gen(6)) * 0.1).to(torch.bfloat16).to(cuda_device) if bias else None
    c, c_s = FK.fp8_gemm_silu_gate_quant(a8, a_s, b8, bs, bias=bvec)
    w13 = FK.fp8_addmm_blockwise(a8, a_s, b8, bs, bias=bvec, output_dtype=torch.bfloat16)
    y, s = FK.fp8_silu_gate_quant(w13)
    assert c.shape == (M, H) and c_s.shape == (M, H // 128)
    assert torch.equal(_e4m3(c), _e4m3(y))
    assert torch.equal(c_s.cpu(), s.reshape(M, H // 128).cpu())
    # the oracle's SiLU gate of the same bf16 intermediate (CPU exp: within one step)
    from tests.helpers import e4m3_step_diff

    ry, rs = OQ.silu_gate_quant(w13.cpu())
    assert e4m3_step_diff(c.cpu(), ry).max().item() <= 1
    torch.testing.assert_close(c_s.cpu(), rs.reshape(M, H // 128), rtol=2e-6, atol=0)


@pytest.mark.parametrize("M,N,K", [(300, 512, 384), (4608, 1024, 768)])
def test_gemm_quant_into_column_window(cuda_device, M, N, K):
    """The quantising epilogue writes into a column window of wider code / scale
    rows exactly what it writes into a buffer of its own, and nothing outside it."""
    from futudiffu_b200 import fp8_kernels as FK

    a8, a_s, b8, bs = (t.to(cuda_device) for t in _operands(M, N, K, seed=14))
    c, c_s = FK.fp8_gemm_gelu_tanh_quant(a8, a_s, b8, bs)
    off, W = 384, N + 640
    buf = torch.zeros(M, W, dtype=torch.uint8, device=cuda_device)
    sbuf = torch.zeros(M, W // 128, dtype=torch.float32, device=cuda_device)
    FK.fp8_gemm_gelu_tanh_quant(a8, a_s, b8, bs, out=(buf[:, off:off + N], sbuf[:, off // 128:off // 128 + N // 128]))
    assert torch.equal(buf[:, off:off + N], c.view(torch.uint8))
    assert torch.equal(sbuf[:, off // 128:off // 128 + N // 128], c_s)
    assert not buf[:, :off].any() and not buf[:, off + N:].any()


@pytest.mark.parametrize("act", [None, "quant", "gelu", "silu"])
def test_gemm_grouped2_equals_separate_launches(cuda_device, act):
    """Two problems in one grouped launch give exactly what two separate launches give."""
    from futudiffu_b200 import _lib as L
    from futudiffu_b200 import fp8_kernels as FK

    probs = []
    for (M, N, K), seed in (((512, 384, 256), 31), ((1300, 256, 384), 32)):
        Nb = 2 * N if act == "silu" else N
        a8, a_s, b8, bs = (t.to(cuda_device) for t in _operands(M, Nb, K, seed=seed))
        probs.append((a8, a_s, b8, bs, None))
    code = {None: None, "quant": L.ACT_NONE, "gelu": L.ACT_GELU_TANH, "silu": L.ACT_SILU_GATE}[act]
    got = FK.fp8_gemm_grouped2(probs, act=code)
    for (a8, a_s, b8, bs, _), g in zip(probs, got):
        if act is None:
            assert torch.equal(g, FK.fp8_gemm_blockwise(a8, a_s, b8, bs, output_dtype=torch.bfloat16))
            continue
        if act == "quant":
            ref = FK.fp8_gemm_quant(a8, a_s, b8, bs)
        elif act == "gelu":
            ref = FK.fp8_gemm_gelu_tanh_quant(a8, a_s, b8, bs)
        else:
            ref = FK.fp8_gemm_silu_gate_quant(a8, a_s, b8, bs)
        assert torch.equal(g[0].view(torch.uint8), ref[0].view(torch.uint8))
        assert torch.equal(g[1].reshape(ref[1].shape), ref[1])


@pytest.mark.parametrize("grouped", [False, True])
def test_gemm_gelu_absmax_shortcut_and_fallback(cuda_device, grouped):
    """The GELU-tanh epilogue takes a group's absmax from GELU(max x) when that
    exceeds 0.171 and evaluates every value otherwise.  Column groups are pushed
    through a bias into every regime (all strongly negative, around the GELU
    minimum at -0.75, tiny, mixed, large) and rows are scaled down to tiny
    magnitudes, so both paths run; codes and scales equal the unfused pair."""
    from futudiffu_b200 import _lib as L
    from futudiffu_b200 import fp8_kernels as FK

    M, N, K = 300, 1280, 256
    g = gen(21)
    x = torch.randn(M, K, generator=g)
    x = x * torch.tensor([1e-4, 1e-2, 0.3, 1.0, 3.0]).repeat(M // 5 + 1)[:M, None]
    w = torch.randn(N, K, generator=g) * 0.02
    a8, a_s = (t.to(cuda_device) for t in OQ.act_quant(x.to(torch.bfloat16)))
    b8, bs = (t.to(cuda_device) for t in OQ.weight_quant(w))
    offsets = torch.tensor([-6.0, -0.75, 0.0, 0.02, -0.3, 0.25, 0.5, 4.0, -2.0, 1.0])
    bias = offsets.repeat_interleave(128).to(torch.bfloat16).to(cuda_device)
    if grouped:
        out = FK.fp8_gemm_grouped2([(a8, a_s, b8, bs, bias), (a8[:129].contiguous(), a_s[:129].contiguous(), b8, bs, bias)],
                                   act=L.ACT_GELU_TANH)
        pairs = [(out[0], a8, a_s), (out[1], a8[:129].contiguous(), a_s[:129].contiguous())]
    else:
        pairs = [(FK.fp8_gemm_gelu_tanh_quant(a8, a_s, b8, bs, bias=bias), a8, a_s)]
    for (c, c_s), aa, ss in pairs:
        h = FK.fp8_addmm_blockwise(aa, ss, b8, bs, bias=bias, output_dtype=torch.bfloat16)
        y, s = FK.fp8_gelu_tanh_quant(h)
        assert torch.equal(_e4m3(c), _e4m3(y))
        assert torch.equal(c_s.reshape(s.shape).cpu(), s.cpu())
        # the regimes were reached: groups whose largest input stays below 0.25
        hm = h.float().view(h.shape[0], -1, 128).amax(-1)
        assert (hm < 0.25).any() and (hm > 0.25).any()
