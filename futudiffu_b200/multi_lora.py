"""Multi-adapter LoRA linear whose forward is one tcgen05 kernel.

Drop-in for src_ii/multi_lora.py ``MultiLoRALinear`` (:35-357): the same slots,
parameters (``lora_A[j]`` (max_rank, in), ``lora_B[j]`` (out, max_rank)),
scalings (alpha / rank), per-image scales with ``token_to_image`` routing
(padding tokens routed to -1 contribute nothing) and attribute proxy to the base
linear.  When the base is an (untransposed) FP8Linear the base GEMM and the
adapter delta run as one GEMM (``fd_fp8_gemm_blockwise_lora``): the FP8 slices
and the bf16 LoRA slices accumulate into one fp32 tile that is rounded once.
"""

from __future__ import annotations

import math

import torch
from torch import Tensor, nn

from . import _lib as L
from .fp8 import FP8Linear
from .fp8_kernels import fp8_act_quant
from .lora_kernels import lora_delta_gemm, lora_operands


class MultiLoRALinear(nn.Module):
    def __init__(self, base_linear: nn.Module, max_adapters: int, max_rank: int,
                 adapter_dtype: torch.dtype = torch.bfloat16, device: torch.device | None = None):
        super().__init__()
        self.base = base_linear
        if hasattr(base_linear, "in_features"):
            self.in_features = base_linear.in_features
            self.out_features = base_linear.out_features
        elif hasattr(base_linear, "weight"):
            self.out_features, self.in_features = base_linear.weight.shape
        else:
            raise ValueError(f"Cannot infer dimensions from {type(base_linear)}")
        if device is None and hasattr(base_linear, "weight") and base_linear.weight is not None:
            device = base_linear.weight.device
        self.max_adapters = max_adapters
        self.max_rank = max_rank
        self.lora_A = nn.ParameterList([
            nn.Parameter(torch.zeros(max_rank, self.in_features, dtype=adapter_dtype, device=device),
                         requires_grad=False) for _ in range(max_adapters)])
        self.lora_B = nn.ParameterList([
            nn.Parameter(torch.zeros(self.out_features, max_rank, dtype=adapter_dtype, device=device),
                         requires_grad=False) for _ in range(max_adapters)])
        self._slot_names: list[str | None] = [None] * max_adapters
        self._slot_ranks: list[int] = [0] * max_adapters
        self._slot_alphas: list[float] = [0.0] * max_adapters
        self.register_buffer("_lora_scalings", torch.zeros(max_adapters, dtype=torch.float32, device=device))
        self.register_buffer("_slot_active", torch.zeros(max_adapters, dtype=torch.float32, device=device))

    # ---------------------------------------------------------------- slots (reference :125-230)
    def assign_adapter(self, slot_index: int, name: str, rank: int, alpha: float, init_a: str = "kaiming") -> None:
        if slot_index < 0 or slot_index >= self.max_adapters:
            raise IndexError(f"slot_index {slot_index} out of range [0, {self.max_adapters})")
        if rank > self.max_rank:
            raise ValueError(f"rank {rank} exceeds max_rank {self.max_rank}")
        if self._slot_names[slot_index] is not None:
            raise ValueError(f"Slot {slot_index} already occupied by {self._slot_names[slot_index]!r}")
        if name in self._slot_names:
            raise ValueError(f"Adapter {name!r} already assigned to slot {self._slot_names.index(name)}")
        self._slot_names[slot_index] = name
        self._slot_ranks[slot_index] = rank
        self._slot_alphas[slot_index] = alpha
        self.lora_A[slot_index].data.zero_()
        if init_a == "kaiming" and rank > 0:
            nn.init.kaiming_uniform_(self.lora_A[slot_index].data[:rank, :], a=math.sqrt(5))
        self.lora_B[slot_index].data.zero_()
        self._lora_scalings[slot_index] = alpha / rank if rank > 0 else 0.0
        self._slot_active[slot_index] = 1.0

    def release_adapter(self, slot_index: int) -> None:
        if slot_index < 0 or slot_index >= self.max_adapters:
            raise IndexError(f"slot_index {slot_index} out of range [0, {self.max_adapters})")
        self._slot_names[slot_index] = None
        self._slot_ranks[slot_index] = 0
        self._slot_alphas[slot_index] = 0.0
        self.lora_A[slot_index].data.zero_()
        self.lora_B[slot_index].data.zero_()
        self.lora_A[slot_index].requires_grad = False
        self.lora_B[slot_index].requires_grad = False
        self._lora_scalings[slot_index] = 0.0
        self._slot_active[slot_index] = 0.0

    def __getattr__(self, name: str):
        try:
            return super().__getattr__(name)
        except AttributeError:
            return getattr(self.base, name)

    @property
    def out_features_val(self) -> int:
        return self.out_features

    def init_adapter_b(self, slot_index: int, std: float = 0.01) -> None:
        if slot_index < 0 or slot_index >= self.max_adapters:
            raise IndexError(f"slot_index {slot_index} out of range [0, {self.max_adapters})")
        nn.init.normal_(self.lora_B[slot_index], std=std)

    # ---------------------------------------------------------------- compute
    def _effective_scales(self, n_tokens: int, adapter_scales: Tensor, token_to_image: Tensor | None) -> Tensor:
        """(n_tokens, max_adapters) per-token scale x alpha / rank x slot-active
        (reference _compute_adapter_delta :262-283)."""
        scales = adapter_scales.unsqueeze(0) if adapter_scales.dim() == 1 else adapter_scales
        if token_to_image is not None:
            routing = token_to_image
            if n_tokens > routing.shape[0]:
                routing = routing.repeat(n_tokens // routing.shape[0])
        else:
            routing = torch.zeros(n_tokens, dtype=torch.long, device=scales.device)
        valid = routing >= 0
        tok = scales[routing.clamp(min=0).long()].float() * valid.unsqueeze(1).float()
        return tok * (self._lora_scalings * self._slot_active).unsqueeze(0)

    def _lora_operands(self, x_2d: Tensor, adapter_scales: Tensor, token_to_image: Tensor | None):
        eff = self._effective_scales(x_2d.shape[0], adapter_scales, token_to_image)
        A_cat = torch.stack(list(self.lora_A)).reshape(self.max_adapters * self.max_rank, self.in_features)
        B_cat = torch.stack(list(self.lora_B)).permute(1, 0, 2).reshape(self.out_features, -1)
        h = x_2d.to(A_cat.dtype) @ A_cat.t()
        hs = (h.float() * eff.repeat_interleave(self.max_rank, dim=1)).to(torch.bfloat16)
        return hs, B_cat.to(torch.bfloat16)

    def forward(self, x: Tensor, adapter_scales: Tensor | None = None, token_to_image: Tensor | None = None) -> Tensor:
        if adapter_scales is None:
            return self.base(x)
        orig_shape = x.shape
        x_2d = x.reshape(-1, self.in_features)
        hs, B_cat = self._lora_operands(x_2d, adapter_scales, token_to_image)
        base = self.base
        if isinstance(base, FP8Linear) and not getattr(base, "_transposed", False) and x.dtype == torch.bfloat16:
            # one kernel: FP8 base GEMM + bf16 LoRA slices in one accumulator
            a8, a_s = fp8_act_quant(x_2d.contiguous())
            hp, bp, Kp = lora_operands(hs, B_cat)
            M = x_2d.shape[0]
            out = torch.empty(M, self.out_features, dtype=base.output_dtype, device=x.device)
            bias = base.bias.contiguous() if base.bias is not None else None
            if M:
                L.call("fd_fp8_gemm_blockwise_lora", L.ptr(a8), L.ptr(a_s), L.ptr(base.weight),
                       L.ptr(base.weight_scale), L.ptr(bias), L.dtype_code(bias.dtype) if bias is not None else 0,
                       L.ptr(out), L.dtype_code(base.output_dtype), M, self.out_features, self.in_features,
                       L.ptr(hp), L.ptr(bp), Kp, L.stream_ptr(x.device))
            return out.reshape(orig_shape[:-1] + (self.out_features,))
        out = self.base(x).reshape(-1, self.out_features)
        delta = lora_delta_gemm(hs, B_cat, out_dtype=out.dtype)
        return (out + delta).reshape(orig_shape[:-1] + (self.out_features,))

    def adapter_delta(self, x: Tensor, adapter_scales: Tensor | None = None,
                      token_to_image: Tensor | None = None) -> Tensor:
        """Adapter contribution only (reference :327-357)."""
        if adapter_scales is None:
            return x.new_zeros(*x.shape[:-1], self.out_features)
        orig_shape = x.shape
        x_2d = x.reshape(-1, self.in_features)
        hs, B_cat = self._lora_operands(x_2d, adapter_scales, token_to_image)
        return lora_delta_gemm(hs, B_cat).reshape(orig_shape[:-1] + (self.out_features,))
