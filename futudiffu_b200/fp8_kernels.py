"""FP8 blockwise kernels, B200 edition: drop-in for ``futudiffu.fp8_kernels``.

Same public functions, argument meanings, assertions, output layouts and
``futudiffu::`` custom ops as the reference module
(src/futudiffu/fp8_kernels.py), backed by the sm_100a kernels of
``libfd_b200.so``:

* ``fp8_act_quant``                 1 x 128 activation quantiser (G1, :54-90)
* ``fp8_gemm_blockwise`` / ``fp8_addmm_blockwise``  tcgen05 GEMM with per-128-K
  promotion of fp32 scales (G2, :125-343)
* ``fp8_gemm_v1t`` / ``fp8_addmm_v1t``  weight stored (K, N) (:1417-1699)
* ``fp8_gemm_v2`` / ``fp8_addmm_v2``    bf16 activations, weight (K, N) (:1061-1369)
* ``fp8_gemm_rowwise`` / ``fp8_addmm_rowwise``  per-row weight scales (:349-560)
* ``fp8_gemm_quant``                GEMM + 1 x 128 requantisation (:573-709)
* ``fp8_gelu``                      dequant -> erf GELU -> requant (:716-833)
* ``fp8_silu_gate_quant``           SiLU gate + requant (G4, :842-978)

There is no Triton and no CPU fallback: every function requires CUDA tensors.
"""

from __future__ import annotations

import ctypes
from typing import Optional, Tuple

import torch

from . import _lib as L


def _check_triton_available() -> bool:
    """Kept for API parity; the B200 build needs no Triton."""
    return False


def _get_sm_major() -> int:
    if not torch.cuda.is_available():
        return 0
    return torch.cuda.get_device_capability()[0]


_SM_MAJOR = _get_sm_major()


def fp8_act_quant(
    x: torch.Tensor, block_size: int = 128, dtype: torch.dtype = torch.float8_e4m3fn
) -> Tuple[torch.Tensor, torch.Tensor]:
    """1 x block_size absmax quantisation to e4m3 (reference fp8_kernels.py:78-90)."""
    assert x.is_contiguous(), "Input must be contiguous"
    assert x.size(-1) % block_size == 0
    if dtype != torch.float8_e4m3fn:
        raise ValueError("only float8_e4m3fn is supported")
    L.require_cuda(x)
    y = torch.empty_like(x, dtype=dtype)
    s = x.new_empty(*x.size()[:-1], x.size(-1) // block_size, dtype=torch.float32)
    K = x.size(-1)
    M = x.numel() // K if K else 0
    L.call("fd_fp8_act_quant", L.ptr(x), L.dtype_code(x.dtype), L.ptr(y), L.ptr(s), M, K,
           block_size, L.stream_ptr(x.device))
    return y, s


def _gemm(a, a_s, b, b_s, bias, output_dtype, b_layout: int, N: int) -> torch.Tensor:
    L.require_cuda(a, a_s, b, b_s, bias)
    if a.dtype != torch.float8_e4m3fn or b.dtype != torch.float8_e4m3fn:
        raise ValueError("fp8 GEMM operands must be float8_e4m3fn")
    K = a.size(-1)
    M = a.numel() // K
    if output_dtype is None:
        output_dtype = torch.bfloat16
    c = a.new_empty(*a.shape[:-1], N, dtype=output_dtype)
    if bias is not None:
        bias = bias.contiguous()
    L.call(
        "fd_fp8_gemm_blockwise",
        L.ptr(a), L.ptr(a_s), L.ptr(b), L.ptr(b_s),
        L.ptr(bias), L.dtype_code(bias.dtype) if bias is not None else 0,
        L.ptr(c), L.dtype_code(output_dtype), M, N, K, b_layout,
        L.stream_ptr(a.device),
    )
    return c


def fp8_gemm_blockwise(
    a: torch.Tensor,
    a_s: torch.Tensor,
    b: torch.Tensor,
    b_s: torch.Tensor,
    input_block_size: int = 128,
    output_dtype: torch.dtype = None,
) -> torch.Tensor:
    """C = A @ B.T with 1 x 128 (A) and 128 x 128 (B) fp32 scales (reference :195-227)."""
    assert a.is_contiguous() and b.is_contiguous()
    assert a_s.is_contiguous() and b_s.is_contiguous()
    assert b.dim() == 2
    assert input_block_size == 128, "input_block_size must be 128"
    return _gemm(a, a_s, b, b_s, None, output_dtype, 0, b.shape[0])


def fp8_addmm_blockwise(
    a: torch.Tensor,
    a_s: torch.Tensor,
    b: torch.Tensor,
    b_s: torch.Tensor,
    bias: torch.Tensor = None,
    input_block_size: int = 128,
    output_dtype: torch.dtype = None,
) -> torch.Tensor:
    """fp8_gemm_blockwise + fp32 bias epilogue (reference :301-343)."""
    assert a.is_contiguous() and b.is_contiguous()
    assert a_s.is_contiguous() and b_s.is_contiguous()
    assert input_block_size == 128, "input_block_size must be 128"
    N = b.shape[0]
    if bias is not None:
        assert bias.is_contiguous() and bias.dim() == 1 and bias.size(0) == N
    return _gemm(a, a_s, b, b_s, bias, output_dtype, 0, N)


def fp8_gemm_rowwise(
    a: torch.Tensor,
    a_s: torch.Tensor,
    b: torch.Tensor,
    b_s: torch.Tensor,
    input_block_size: int = 128,
    output_dtype: torch.dtype = None,
) -> torch.Tensor:
    """GEMM with per-row weight scales b_s (N,), applied after the K loop (reference :416-454)."""
    assert a.is_contiguous() and b.is_contiguous()
    assert a_s.is_contiguous() and b_s.is_contiguous()
    assert input_block_size == 128, "input_block_size must be 128"
    return _gemm(a, a_s, b, b_s, None, output_dtype, 2, b.shape[0])


def fp8_addmm_rowwise(
    a: torch.Tensor,
    a_s: torch.Tensor,
    b: torch.Tensor,
    b_s: torch.Tensor,
    bias: torch.Tensor = None,
    input_block_size: int = 128,
    output_dtype: torch.dtype = None,
) -> torch.Tensor:
    """Rowwise GEMM + bias (reference :524-567)."""
    assert a.is_contiguous() and b.is_contiguous()
    assert a_s.is_contiguous() and b_s.is_contiguous()
    assert input_block_size == 128, "input_block_size must be 128"
    N = b.shape[0]
    if bias is not None:
        assert bias.is_contiguous() and bias.dim() == 1 and bias.size(0) == N
    return _gemm(a, a_s, b, b_s, bias, output_dtype, 2, N)


def fp8_gemm_v1t(
    a: torch.Tensor,
    a_s: torch.Tensor,
    b: torch.Tensor,
    b_s: torch.Tensor,
    input_block_size: int = 128,
    output_dtype: torch.dtype = torch.bfloat16,
) -> torch.Tensor:
    """GEMM with the weight pre-transposed to (K, N), scales (K/128, N/128) (reference :1527-1575)."""
    assert a.is_contiguous() and b.is_contiguous()
    assert a_s.is_contiguous() and b_s.is_contiguous()
    assert b.dim() == 2
    K = a.size(-1)
    assert b.shape[0] == K, f"B shape {b.shape} incompatible with K={K}"
    assert input_block_size == 128, "input_block_size must be 128"
    return _gemm(a, a_s, b, b_s, None, output_dtype, 1, b.shape[1])


def fp8_addmm_v1t(
    a: torch.Tensor,
    a_s: torch.Tensor,
    b: torch.Tensor,
    b_s: torch.Tensor,
    bias: torch.Tensor = None,
    input_block_size: int = 128,
    output_dtype: torch.dtype = torch.bfloat16,
) -> torch.Tensor:
    """v1t GEMM + bias (reference :1658-1699)."""
    assert a.is_contiguous() and b.is_contiguous()
    assert a_s.is_contiguous() and b_s.is_contiguous()
    K = a.size(-1)
    assert b.shape[0] == K, f"B shape {b.shape} incompatible with K={K}"
    assert input_block_size == 128, "input_block_size must be 128"
    N = b.shape[1]
    if bias is not None:
        assert bias.is_contiguous() and bias.dim() == 1 and bias.size(0) == N
    return _gemm(a, a_s, b, b_s, bias, output_dtype, 1, N)


def fp8_gemm_v2(
    a: torch.Tensor,
    b: torch.Tensor,
    b_s: torch.Tensor,
    input_block_size: int = 128,
    output_dtype: torch.dtype = torch.bfloat16,
) -> torch.Tensor:
    """bf16 activations (quantised with the G1 formula), weight (K, N) (reference :1167-1212)."""
    assert a.is_contiguous() and b.is_contiguous()
    assert b_s.is_contiguous()
    assert b.dim() == 2
    K = a.size(-1)
    assert b.shape[0] == K, f"B shape {b.shape} incompatible with K={K}"
    a8, a_s = fp8_act_quant(a, input_block_size)
    return _gemm(a8, a_s, b, b_s, None, output_dtype, 1, b.shape[1])


def fp8_addmm_v2(
    a: torch.Tensor,
    b: torch.Tensor,
    b_s: torch.Tensor,
    bias: torch.Tensor = None,
    input_block_size: int = 128,
    output_dtype: torch.dtype = torch.bfloat16,
) -> torch.Tensor:
    """fp8_gemm_v2 + bias (reference :1314-1369)."""
    assert a.is_contiguous() and b.is_contiguous()
    assert b_s.is_contiguous()
    K = a.size(-1)
    assert b.shape[0] == K, f"B shape {b.shape} incompatible with K={K}"
    N = b.shape[1]
    if bias is not None:
        assert bias.is_contiguous() and bias.dim() == 1 and bias.size(0) == N
    a8, a_s = fp8_act_quant(a, input_block_size)
    return _gemm(a8, a_s, b, b_s, bias, output_dtype, 1, N)


def fp8_gemm_quant(
    a: torch.Tensor,
    a_s: torch.Tensor,
    b: torch.Tensor,
    b_s: torch.Tensor,
    input_block_size: int = 128,
    out_block_size: int = 128,
    out_dtype: torch.dtype = torch.float8_e4m3fn,
) -> Tuple[torch.Tensor, torch.Tensor]:
    """GEMM whose fp32 accumulator is requantised 1 x 128 in the epilogue (reference :666-709).

    Returns the e4m3 output (batch shape of ``a``, N) and its dequant scales
    (batch shape of ``a``, N / out_block_size), the layout of the reference.
    """
    assert a.is_contiguous() and b.is_contiguous()
    assert a_s.is_contiguous() and b_s.is_contiguous()
    assert b.dim() == 2
    K = a.size(-1)
    M = a.numel() // K
    N = b.shape[0]
    batch_shape = a.shape[:-1]
    assert N % out_block_size == 0
    assert input_block_size == 128 and out_block_size == 128, "block sizes must be 128"
    return _gemm_quant(a, a_s, b, b_s, None, L.ACT_NONE, M, N, K, batch_shape, out_dtype)


def _gemm_quant(a, a_s, b, b_s, bias, act, M, N, K, batch_shape, out_dtype, out=None):
    L.require_cuda(a, a_s, b, b_s, bias)
    if out_dtype != torch.float8_e4m3fn:
        raise ValueError("quantising GEMM epilogues produce float8_e4m3fn only")
    if bias is not None:
        bias = bias.contiguous()
    bias_args = (L.ptr(bias), L.dtype_code(bias.dtype) if bias is not None else 0)
    if out is not None:
        # a column window of wider row-major code / scale buffers (views)
        c, c_s = out
        assert c.stride(-1) == 1 and c_s.stride(-1) == 1 and c.shape[-1] == N and c_s.shape[-1] == N // 128
        assert c.numel() // N == M and c_s.numel() // (N // 128) == M
        if M:
            L.call("fd_fp8_gemm_quant_ld", L.ptr(a), L.ptr(a_s), L.ptr(b), L.ptr(b_s), *bias_args, L.ptr(c),
                   L.ptr(c_s), M, N, K, act, c.stride(-2), c_s.stride(-2), L.stream_ptr(a.device))
        return c, c_s
    c = a.new_empty(*batch_shape, N, dtype=out_dtype)
    c_s = a.new_empty(M, N // 128, dtype=torch.float32)
    if M == 0:
        return c, c_s
    L.call("fd_fp8_gemm_quant", L.ptr(a), L.ptr(a_s), L.ptr(b), L.ptr(b_s), *bias_args, L.ptr(c), L.ptr(c_s),
           M, N, K, act, L.stream_ptr(a.device))
    if len(batch_shape) > 0:
        c_s = c_s.reshape(*batch_shape, N // 128)
    return c, c_s


def fp8_gemm_grouped2(problems, act: Optional[int] = None):
    """Two FP8 block GEMMs with the same epilogue in one launch (``fd_fp8_gemm_grouped2``).

    ``problems``: two (a8 (..., K) e4m3, a_s (..., K / 128), b8 (N, K), b_s, bias or
    None) tuples.  ``act`` None -> bf16 outputs (..., N); else an ``L.ACT_*``
    quantising epilogue -> (codes, scales) per problem, as fp8_gemm_quant /
    fp8_gemm_gelu_tanh_quant / fp8_gemm_silu_gate_quant produce them.
    """
    assert len(problems) == 2
    structs, outs, keep = [], [], []
    for a, a_s, b, b_s, bias in problems:
        assert a.is_contiguous() and a_s.is_contiguous() and b.is_contiguous() and b_s.is_contiguous()
        L.require_cuda(a, a_s, b, b_s, bias)
        K = a.shape[-1]
        M = a.numel() // K
        N = b.shape[0] // (2 if act == L.ACT_SILU_GATE else 1)
        if bias is not None:
            bias = bias.contiguous()
            assert bias.dtype == torch.bfloat16
        if act is None:
            c, c_s = a.new_empty(*a.shape[:-1], N, dtype=torch.bfloat16), None
            outs.append(c)
        else:
            c = a.new_empty(*a.shape[:-1], N, dtype=torch.float8_e4m3fn)
            c_s = a.new_empty(*a.shape[:-1], N // 128, dtype=torch.float32)
            outs.append((c, c_s))
        keep += [bias, c, c_s]
        structs.append(L.GemmProblem(L.ptr(a), L.ptr(a_s), L.ptr(b), L.ptr(b_s), L.ptr(bias), L.ptr(c), L.ptr(c_s),
                                     M, N, K))
    has_bias = problems[0][4] is not None
    L.call("fd_fp8_gemm_grouped2", ctypes.addressof(structs[0]), ctypes.addressof(structs[1]),
           L.DT_BF16 if has_bias else 0, L.GEMM_STORE_BF16 if act is None else act, L.stream_ptr(problems[0][0].device))
    return outs


def fp8_gemm_gelu_tanh_quant(
    a: torch.Tensor,
    a_s: torch.Tensor,
    b: torch.Tensor,
    b_s: torch.Tensor,
    bias: Optional[torch.Tensor] = None,
    block_size: int = 128,
    out: Optional[Tuple[torch.Tensor, torch.Tensor]] = None,
) -> Tuple[torch.Tensor, torch.Tensor]:
    """``fp8_gelu_tanh_quant(fp8_addmm_blockwise(a, a_s, b, b_s, bias))`` in one kernel.

    The GEMM output is rounded to bf16 (as the unfused pair stores it), passed
    through GELU (tanh approximation) and quantised 1 x 128; codes and scales are
    identical to the two-kernel path.  Scales have shape (batch shape, N / 128).
    ``out``: optional (codes, scales) views with N and N / 128 columns whose rows
    may be wider (a column window of a larger buffer); written in place.
    """
    assert a.is_contiguous() and b.is_contiguous()
    assert a_s.is_contiguous() and b_s.is_contiguous()
    assert b.dim() == 2 and block_size == 128
    K = a.size(-1)
    M = a.numel() // K
    N = b.shape[0]
    assert N % block_size == 0
    return _gemm_quant(a, a_s, b, b_s, bias, L.ACT_GELU_TANH, M, N, K, a.shape[:-1], torch.float8_e4m3fn, out)


def fp8_gemm_silu_gate_quant(
    a: torch.Tensor,
    a_s: torch.Tensor,
    b13: torch.Tensor,
    b13_s: torch.Tensor,
    bias: Optional[torch.Tensor] = None,
    block_size: int = 128,
) -> Tuple[torch.Tensor, torch.Tensor]:
    """The FFN chain head in one kernel (reference src_ii/transformer.py:536-545).

    ``b13`` is the fused w1w3 weight (2 H, K) with scales (2 H / 128, K / 128):
    rows [0, H) are w1, rows [H, 2 H) are w3, the layout of the reference's
    ``w1w3`` FP8Linear.  Equals ``fp8_silu_gate_quant(fp8_addmm_blockwise(a, a_s,
    b13, b13_s, bias))`` code for code without materialising the bf16 (M, 2 H)
    intermediate.  Returns (codes (..., H) e4m3, scales (..., H / 128)).
    """
    assert a.is_contiguous() and b13.is_contiguous()
    assert a_s.is_contiguous() and b13_s.is_contiguous()
    assert b13.dim() == 2 and b13.shape[0] % 2 == 0 and block_size == 128
    K = a.size(-1)
    M = a.numel() // K
    H = b13.shape[0] // 2
    assert H % block_size == 0
    return _gemm_quant(a, a_s, b13, b13_s, bias, L.ACT_SILU_GATE, M, H, K, a.shape[:-1], torch.float8_e4m3fn)


def fp8_gelu(
    x: torch.Tensor,
    s_x: torch.Tensor,
    block_size: int = 128,
    dtype: torch.dtype = torch.float8_e4m3fn,
) -> Tuple[torch.Tensor, torch.Tensor]:
    """Dequant -> erf GELU -> requant, fp8 in and out (reference :788-833)."""
    assert x.is_contiguous() and s_x.is_contiguous()
    assert x.size(-1) % block_size == 0
    assert block_size == 128, "block_size must be 128"
    L.require_cuda(x, s_x)
    N = x.shape[-1]
    M = x.numel() // N
    y = torch.empty_like(x, dtype=dtype)
    s_y = torch.empty_like(s_x, dtype=torch.float32)
    L.call("fd_fp8_gelu_requant", L.ptr(x), L.ptr(s_x), L.ptr(y), L.ptr(s_y), M, N, block_size,
           L.stream_ptr(x.device))
    return y, s_y


def fp8_gelu_tanh_quant(
    x: torch.Tensor, block_size: int = 128, dtype: torch.dtype = torch.float8_e4m3fn
) -> Tuple[torch.Tensor, torch.Tensor]:
    """GELU (tanh approximation) of a bf16 tensor, quantised 1 x 128 to e4m3.

    The MMDiT MLP activation (no counterpart kernel in the reference; its
    arithmetic is F.gelu(approximate="tanh") followed by the G1 quantiser).
    """
    assert x.is_contiguous(), "Input must be contiguous"
    assert x.dtype == torch.bfloat16
    assert x.size(-1) % block_size == 0
    L.require_cuda(x)
    N = x.shape[-1]
    M = x.numel() // N
    y = torch.empty_like(x, dtype=dtype)
    s = x.new_empty(*x.shape[:-1], N // block_size, dtype=torch.float32)
    L.call("fd_fp8_gelu_tanh_quant", L.ptr(x), L.ptr(y), L.ptr(s), M, N, block_size,
           L.stream_ptr(x.device))
    return y, s


def fp8_silu_gate_quant(
    x: torch.Tensor,
    block_size: int = 128,
    dtype: torch.dtype = torch.float8_e4m3fn,
) -> Tuple[torch.Tensor, torch.Tensor]:
    """silu(x[..., :N]) * x[..., N:] quantised 1 x block_size (reference :918-978)."""
    assert x.is_contiguous(), "Input must be contiguous"
    total_cols = x.size(-1)
    assert total_cols % 2 == 0, f"Last dim must be even (got {total_cols})"
    N = total_cols // 2
    assert N % block_size == 0, f"N={N} must be divisible by block_size={block_size}"
    assert x.dtype == torch.bfloat16, "input must be bf16"
    L.require_cuda(x)
    batch_shape = x.shape[:-1]
    M = x.numel() // total_cols
    SN = N // block_size
    y = torch.empty(M, N, dtype=dtype, device=x.device)
    s_y = torch.empty(M, SN, dtype=torch.float32, device=x.device)
    L.call("fd_fp8_silu_gate_quant", L.ptr(x), L.ptr(y), L.ptr(s_y), M, N, block_size,
           L.stream_ptr(x.device))
    if len(batch_shape) > 1:
        y = y.reshape(*batch_shape, N)
        s_y = s_y.reshape(*batch_shape, SN)
    return y, s_y


# ---------------------------------------------------------------------------
# torch.library custom ops (names, fakes and autograd as reference :1761-1953)
# ---------------------------------------------------------------------------

_DTYPE_TO_CODE_K = {
    torch.bfloat16: 0, torch.float16: 1, torch.float32: 2,
    torch.float8_e4m3fn: 3,
}
_CODE_TO_DTYPE_K = {v: k for k, v in _DTYPE_TO_CODE_K.items()}

_USE_FP8_KERNEL_CUSTOM_OP = True


@torch.library.custom_op("futudiffu::fp8_silu_gate_quant", mutates_args=())
def fp8_silu_gate_quant_op(
    x: torch.Tensor,
    block_size: int,
    dtype_code: int = 3,
) -> tuple[torch.Tensor, torch.Tensor]:
    return fp8_silu_gate_quant(x, block_size=block_size, dtype=_CODE_TO_DTYPE_K[dtype_code])


@fp8_silu_gate_quant_op.register_fake
def _fp8_silu_gate_quant_fake(x, block_size, dtype_code=3):
    dtype = _CODE_TO_DTYPE_K[dtype_code]
    N = x.shape[-1] // 2
    SN = N // block_size
    return x.new_empty(*x.shape[:-1], N, dtype=dtype), x.new_empty(*x.shape[:-1], SN, dtype=torch.float32)


@torch.library.custom_op("futudiffu::fp8_gemm_blockwise", mutates_args=())
def fp8_gemm_blockwise_op(
    a: torch.Tensor,
    a_s: torch.Tensor,
    b: torch.Tensor,
    b_s: torch.Tensor,
    input_block_size: int,
    output_dtype_code: int,
) -> torch.Tensor:
    return fp8_gemm_blockwise(a, a_s, b, b_s, input_block_size=input_block_size,
                              output_dtype=_CODE_TO_DTYPE_K[output_dtype_code])


@fp8_gemm_blockwise_op.register_fake
def _fp8_gemm_blockwise_fake(a, a_s, b, b_s, input_block_size, output_dtype_code):
    return a.new_empty(*a.shape[:-1], b.shape[0], dtype=_CODE_TO_DTYPE_K[output_dtype_code])


@torch.library.custom_op("futudiffu::fp8_gemm_v1t", mutates_args=())
def fp8_gemm_v1t_op(
    a: torch.Tensor,
    a_s: torch.Tensor,
    b: torch.Tensor,
    b_s: torch.Tensor,
    input_block_size: int,
    output_dtype_code: int,
) -> torch.Tensor:
    return fp8_gemm_v1t(a, a_s, b, b_s, input_block_size=input_block_size,
                        output_dtype=_CODE_TO_DTYPE_K[output_dtype_code])


@fp8_gemm_v1t_op.register_fake
def _fp8_gemm_v1t_fake(a, a_s, b, b_s, input_block_size, output_dtype_code):
    return a.new_empty(*a.shape[:-1], b.shape[1], dtype=_CODE_TO_DTYPE_K[output_dtype_code])


def _fp8_silu_gate_quant_setup(ctx, inputs, output):
    x, block_size, dtype_code = inputs
    ctx.save_for_backward(x)


def _fp8_silu_gate_quant_backward(ctx, d_gate_fp8, d_gate_scale):
    # Straight-through estimator (reference :1888-1909).
    (x,) = ctx.saved_tensors
    d_gate = d_gate_fp8.to(x.dtype)
    N = x.shape[-1] // 2
    w1_out = x[..., :N]
    w3_out = x[..., N:]
    sig = torch.sigmoid(w1_out)
    d_w3 = d_gate * (w1_out * sig)
    d_w1 = d_gate * w3_out * sig * (1 + w1_out * (1 - sig))
    return torch.cat([d_w1, d_w3], dim=-1), None, None


fp8_silu_gate_quant_op.register_autograd(_fp8_silu_gate_quant_backward,
                                         setup_context=_fp8_silu_gate_quant_setup)


def _fp8_gemm_bw_setup(ctx, inputs, output):
    a, a_s, b, b_s, input_block_size, output_dtype_code = inputs
    ctx.save_for_backward(b, b_s)
    ctx.block_size = b.shape[0] // b_s.shape[0]


def _fp8_gemm_bw_backward(ctx, d_output):
    from .fp8 import dequantize_fp8_blockwise

    b, b_s = ctx.saved_tensors
    w = dequantize_fp8_blockwise(b, b_s, ctx.block_size)
    return d_output @ w, None, None, None, None, None


fp8_gemm_blockwise_op.register_autograd(_fp8_gemm_bw_backward, setup_context=_fp8_gemm_bw_setup)


def _fp8_gemm_v1t_setup(ctx, inputs, output):
    a, a_s, b, b_s, input_block_size, output_dtype_code = inputs
    ctx.save_for_backward(b, b_s)
    ctx.block_size = b.shape[0] // b_s.shape[0]


def _fp8_gemm_v1t_backward(ctx, d_output):
    from .fp8 import dequantize_fp8_blockwise

    b, b_s = ctx.saved_tensors
    w = dequantize_fp8_blockwise(b, b_s, ctx.block_size)
    return d_output @ w.t(), None, None, None, None, None


fp8_gemm_v1t_op.register_autograd(_fp8_gemm_v1t_backward, setup_context=_fp8_gemm_v1t_setup)
