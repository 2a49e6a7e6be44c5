"""FP8 blockwise linear layers, B200 edition: drop-in for ``futudiffu.fp8``.

Mirrors src/futudiffu/fp8.py: the ``futudiffu::fp8_linear*`` custom ops
(:51-202) with their fakes and straight-through autograd (:493-561),
``FP8Linear`` (:210-334), ``quantize_fp8_blockwise`` (:337-371),
``quantize_model`` (:374-449), ``dequantize_fp8_blockwise`` (:452-480) and
``replace_linear_with_fp8`` (:564-599).  Checkpoint format is unchanged:
``weight`` e4m3 (N, K), ``weight_scale`` f32 (N/128, K/128) and a
``comfy_quant`` JSON byte tensor.
"""

from __future__ import annotations

import logging
from typing import Optional

import torch
import torch.nn as nn

from . import _lib as L
from .fp8_kernels import (
    fp8_act_quant,
    fp8_addmm_blockwise,
    fp8_addmm_v1t,
    fp8_gemm_blockwise,
    fp8_gemm_v1t,
)

BLOCK_SIZE = 128

_DTYPE_TO_CODE = {torch.bfloat16: 0, torch.float16: 1, torch.float32: 2}
_CODE_TO_DTYPE = {0: torch.bfloat16, 1: torch.float16, 2: torch.float32}

_USE_FP8_CUSTOM_OP = True

log = logging.getLogger(__name__)


def _quant_act(x: torch.Tensor, block_size: int):
    original_shape = x.shape
    x_flat = x.reshape(-1, x.shape[-1]).contiguous()
    x_fp8, x_scale = fp8_act_quant(x_flat, block_size=block_size)
    x_fp8 = x_fp8.reshape(original_shape[:-1] + (x_fp8.shape[-1],))
    x_scale = x_scale.reshape(original_shape[:-1] + (x_scale.shape[-1],))
    return x_fp8, x_scale


@torch.library.custom_op("futudiffu::fp8_linear", mutates_args=())
def fp8_linear_op(
    x: torch.Tensor,
    weight: torch.Tensor,
    weight_scale: torch.Tensor,
    block_size: int,
    output_dtype_code: int,
) -> torch.Tensor:
    """FP8 linear without bias: G1 activation quant + tcgen05 block GEMM."""
    x_fp8, x_scale = _quant_act(x, block_size)
    return fp8_gemm_blockwise(x_fp8, x_scale, weight, weight_scale, input_block_size=block_size,
                              output_dtype=_CODE_TO_DTYPE[output_dtype_code])


@fp8_linear_op.register_fake
def _fp8_linear_fake(x, weight, weight_scale, block_size, output_dtype_code):
    return x.new_empty(*x.shape[:-1], weight.shape[0], dtype=_CODE_TO_DTYPE[output_dtype_code])


@torch.library.custom_op("futudiffu::fp8_linear_bias", mutates_args=())
def fp8_linear_bias_op(
    x: torch.Tensor,
    weight: torch.Tensor,
    weight_scale: torch.Tensor,
    bias: torch.Tensor,
    block_size: int,
    output_dtype_code: int,
) -> torch.Tensor:
    """FP8 linear with bias."""
    x_fp8, x_scale = _quant_act(x, block_size)
    return fp8_addmm_blockwise(x_fp8, x_scale, weight, weight_scale, bias=bias,
                               input_block_size=block_size,
                               output_dtype=_CODE_TO_DTYPE[output_dtype_code])


@fp8_linear_bias_op.register_fake
def _fp8_linear_bias_fake(x, weight, weight_scale, bias, block_size, output_dtype_code):
    return x.new_empty(*x.shape[:-1], weight.shape[0], dtype=_CODE_TO_DTYPE[output_dtype_code])


@torch.library.custom_op("futudiffu::fp8_linear_v1t", mutates_args=())
def fp8_linear_v1t_op(
    x: torch.Tensor,
    weight: torch.Tensor,
    weight_scale: torch.Tensor,
    block_size: int,
    output_dtype_code: int,
) -> torch.Tensor:
    """FP8 linear with the weight pre-transposed to (K, N)."""
    x_fp8, x_scale = _quant_act(x, block_size)
    return fp8_gemm_v1t(x_fp8, x_scale, weight, weight_scale, input_block_size=block_size,
                        output_dtype=_CODE_TO_DTYPE[output_dtype_code])


@fp8_linear_v1t_op.register_fake
def _fp8_linear_v1t_fake(x, weight, weight_scale, block_size, output_dtype_code):
    return x.new_empty(*x.shape[:-1], weight.shape[1], dtype=_CODE_TO_DTYPE[output_dtype_code])


@torch.library.custom_op("futudiffu::fp8_linear_bias_v1t", mutates_args=())
def fp8_linear_bias_v1t_op(
    x: torch.Tensor,
    weight: torch.Tensor,
    weight_scale: torch.Tensor,
    bias: torch.Tensor,
    block_size: int,
    output_dtype_code: int,
) -> torch.Tensor:
    """FP8 linear with (K, N) weight and bias."""
    x_fp8, x_scale = _quant_act(x, block_size)
    return fp8_addmm_v1t(x_fp8, x_scale, weight, weight_scale, bias=bias,
                         input_block_size=block_size,
                         output_dtype=_CODE_TO_DTYPE[output_dtype_code])


@fp8_linear_bias_v1t_op.register_fake
def _fp8_linear_bias_v1t_fake(x, weight, weight_scale, bias, block_size, output_dtype_code):
    return x.new_empty(*x.shape[:-1], weight.shape[1], dtype=_CODE_TO_DTYPE[output_dtype_code])


class FP8Linear(nn.Module):
    """Linear layer with FP8 blockwise quantized weights (reference fp8.py:210-334).

    ``weight`` (N, K) float8_e4m3fn, ``weight_scale`` (N/bs, K/bs) float32.
    """

    def __init__(
        self,
        weight: torch.Tensor,
        weight_scale: torch.Tensor,
        bias: Optional[torch.Tensor] = None,
        block_size: int = BLOCK_SIZE,
        output_dtype: torch.dtype = torch.bfloat16,
    ):
        super().__init__()
        self.register_buffer("weight", weight)
        self.register_buffer("weight_scale", weight_scale)
        if bias is not None:
            self.register_buffer("bias", bias)
        else:
            self.bias = None
        self.block_size = block_size
        self.output_dtype = output_dtype
        self.in_features = weight.shape[1]
        self.out_features = weight.shape[0]
        self._transposed = False

    def transpose_weight(self) -> None:
        """Store the weight as (K, N) and its scales as (K/bs, N/bs) (v1t path)."""
        if self._transposed:
            return
        self.weight = nn.Parameter(self.weight.data.t().contiguous(), requires_grad=False)
        self.weight_scale = nn.Parameter(self.weight_scale.data.t().contiguous(), requires_grad=False)
        self._transposed = True

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        dtype_code = _DTYPE_TO_CODE[self.output_dtype]
        if self._transposed:
            return self._forward_v1t(x, dtype_code)
        return self._forward_custom_op(x, dtype_code)

    def _forward_custom_op(self, x: torch.Tensor, dtype_code: int) -> torch.Tensor:
        if self.bias is not None:
            return fp8_linear_bias_op(x, self.weight, self.weight_scale, self.bias,
                                      self.block_size, dtype_code)
        return fp8_linear_op(x, self.weight, self.weight_scale, self.block_size, dtype_code)

    def _forward_v1t(self, x: torch.Tensor, dtype_code: int) -> torch.Tensor:
        if self.bias is not None:
            return fp8_linear_bias_v1t_op(x, self.weight, self.weight_scale, self.bias,
                                          self.block_size, dtype_code)
        return fp8_linear_v1t_op(x, self.weight, self.weight_scale, self.block_size, dtype_code)

    def _forward_eager(self, x: torch.Tensor) -> torch.Tensor:
        """Direct (non custom-op) call of the same kernels (reference :310-334)."""
        x_fp8, x_scale = _quant_act(x, self.block_size)
        if self.bias is not None:
            return fp8_addmm_blockwise(x_fp8, x_scale, self.weight, self.weight_scale, bias=self.bias,
                                       input_block_size=self.block_size, output_dtype=self.output_dtype)
        return fp8_gemm_blockwise(x_fp8, x_scale, self.weight, self.weight_scale,
                                  input_block_size=self.block_size, output_dtype=self.output_dtype)


def quantize_fp8_blockwise_cuda(
    tensor: torch.Tensor,
    block_size: int = BLOCK_SIZE,
    dtype: torch.dtype = torch.float8_e4m3fn,
) -> tuple[torch.Tensor, torch.Tensor]:
    """128 x 128 weight quantisation on the device; outputs stay on the device."""
    assert tensor.dim() == 2
    assert block_size == 128, "block_size must be 128"
    assert dtype == torch.float8_e4m3fn
    L.require_cuda(tensor)
    N, K = tensor.shape
    assert N % block_size == 0 and K % block_size == 0
    src = tensor.contiguous()
    if src.dtype not in (torch.bfloat16, torch.float16, torch.float32):
        src = src.float()
    y = torch.empty(N, K, dtype=dtype, device=src.device)
    s = torch.empty(N // block_size, K // block_size, dtype=torch.float32, device=src.device)
    L.call("fd_fp8_weight_quant", L.ptr(src), L.dtype_code(src.dtype), L.ptr(y), L.ptr(s), N, K,
           block_size, L.stream_ptr(src.device))
    return y, s


def quantize_fp8_blockwise(
    tensor: torch.Tensor,
    block_size: int = BLOCK_SIZE,
    dtype: torch.dtype = torch.float8_e4m3fn,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Quantize a 2D tensor to FP8 with 128 x 128 block scales (reference fp8.py:337-371).

    Like the reference, the work runs on CUDA and both outputs are returned on CPU.
    """
    y, s = quantize_fp8_blockwise_cuda(tensor.cuda(), block_size, dtype)
    return y.cpu(), s.cpu()


def quantize_model(
    input_path: str,
    output_path: str,
    block_size: int = BLOCK_SIZE,
    min_elements: int = 4096,
) -> dict:
    """Quantize a safetensors checkpoint to FP8 blockwise + comfy_quant metadata (reference :374-449)."""
    import json
    import os
    from collections import OrderedDict

    from safetensors.torch import load_file, save_file

    state_dict = load_file(input_path)
    output_dict = OrderedDict()
    stats = {"quantized": 0, "kept": 0, "total_params": 0, "quantized_params": 0}
    for key, tensor in state_dict.items():
        stats["total_params"] += tensor.numel()
        is_weight = tensor.dim() == 2 and tensor.numel() >= min_elements
        is_float = tensor.dtype in (torch.float32, torch.float16, torch.bfloat16)
        can_block = is_weight and tensor.shape[0] % block_size == 0 and tensor.shape[1] % block_size == 0
        if is_weight and is_float and can_block:
            qdata, scale = quantize_fp8_blockwise(tensor, block_size)
            output_dict[key] = qdata
            output_dict[key.replace(".weight", ".weight_scale")] = scale
            meta = {
                "format": "float8_e4m3fn_blockwise",
                "group_size": block_size,
                "orig_dtype": str(tensor.dtype),
                "orig_shape": list(tensor.shape),
            }
            output_dict[key.replace(".weight", ".comfy_quant")] = torch.tensor(
                list(json.dumps(meta).encode("utf-8")), dtype=torch.uint8
            )
            stats["quantized"] += 1
            stats["quantized_params"] += tensor.numel()
        else:
            output_dict[key] = tensor
            stats["kept"] += 1
    os.makedirs(os.path.dirname(output_path) or ".", exist_ok=True)
    save_file(output_dict, output_path)
    return stats


def dequantize_fp8_blockwise(
    weight: torch.Tensor,
    scale: torch.Tensor,
    block_size: int = BLOCK_SIZE,
    output_dtype: torch.dtype = torch.bfloat16,
) -> torch.Tensor:
    """Dequantize an FP8 blockwise weight (reference fp8.py:452-480).

    Runs on the device; a CPU input is moved to CUDA and the result moved back,
    so callers see the reference's device-agnostic behaviour without a CPU
    compute path.
    """
    assert block_size == 128, "block_size must be 128"
    on_cpu = not weight.is_cuda
    w = weight.cuda() if on_cpu else weight
    s = scale.to(device=w.device, dtype=torch.float32).contiguous()
    w = w.contiguous()
    N, K = w.shape
    out = torch.empty(N, K, dtype=output_dtype, device=w.device)
    L.call("fd_fp8_dequant_blockwise", L.ptr(w), L.ptr(s), L.ptr(out), L.dtype_code(output_dtype),
           N, K, block_size, L.stream_ptr(w.device))
    return out.cpu() if on_cpu else out


def _fp8_linear_setup(ctx, inputs, output):
    x, weight, weight_scale, block_size, output_dtype_code = inputs
    ctx.save_for_backward(weight, weight_scale)
    ctx.block_size = block_size


def _fp8_linear_backward(ctx, grad_output):
    weight, weight_scale = ctx.saved_tensors
    w = dequantize_fp8_blockwise(weight, weight_scale, ctx.block_size)
    return grad_output @ w, None, None, None, None


fp8_linear_op.register_autograd(_fp8_linear_backward, setup_context=_fp8_linear_setup)


def _fp8_linear_bias_setup(ctx, inputs, output):
    x, weight, weight_scale, bias, block_size, output_dtype_code = inputs
    ctx.save_for_backward(weight, weight_scale)
    ctx.block_size = block_size


def _fp8_linear_bias_backward(ctx, grad_output):
    weight, weight_scale = ctx.saved_tensors
    w = dequantize_fp8_blockwise(weight, weight_scale, ctx.block_size)
    return grad_output @ w, None, None, None, None, None


fp8_linear_bias_op.register_autograd(_fp8_linear_bias_backward, setup_context=_fp8_linear_bias_setup)


def _fp8_linear_v1t_backward(ctx, grad_output):
    weight, weight_scale = ctx.saved_tensors
    w = dequantize_fp8_blockwise(weight, weight_scale, ctx.block_size)
    return grad_output @ w.t(), None, None, None, None


fp8_linear_v1t_op.register_autograd(_fp8_linear_v1t_backward, setup_context=_fp8_linear_setup)


def _fp8_linear_bias_v1t_backward(ctx, grad_output):
    weight, weight_scale = ctx.saved_tensors
    w = dequantize_fp8_blockwise(weight, weight_scale, ctx.block_size)
    return grad_output @ w.t(), None, None, None, None, None


fp8_linear_bias_v1t_op.register_autograd(_fp8_linear_bias_v1t_backward,
                                         setup_context=_fp8_linear_bias_setup)


def replace_linear_with_fp8(
    module: nn.Module,
    state_dict: dict[str, torch.Tensor],
    prefix: str = "",
    block_size: int = BLOCK_SIZE,
    output_dtype: torch.dtype = torch.bfloat16,
) -> None:
    """Swap nn.Linear children for FP8Linear where the state dict holds e4m3 weights + scales
    (reference fp8.py:564-599)."""
    for name, child in list(module.named_children()):
        full_name = f"{prefix}{name}" if prefix else name
        weight_key = f"{full_name}.weight"
        scale_key = f"{full_name}.weight_scale"
        if isinstance(child, nn.Linear) and weight_key in state_dict:
            weight = state_dict[weight_key]
            if weight.dtype == torch.float8_e4m3fn and scale_key in state_dict:
                fp8_linear = FP8Linear(
                    weight=weight,
                    weight_scale=state_dict[scale_key],
                    bias=state_dict.get(f"{full_name}.bias", None),
                    block_size=block_size,
                    output_dtype=output_dtype,
                )
                setattr(module, name, fp8_linear)
                continue
        replace_linear_with_fp8(child, state_dict, f"{full_name}.", block_size, output_dtype)
