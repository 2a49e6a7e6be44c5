"""Packed multi-image forward helpers: drop-in for ``src_ii.forward_packed``.

Every packed plan is padded to one fixed length (``REFERENCE_TOTAL_LEN`` by
default) so that all bins run the same shapes; the padding tail carries document
id -1 and zero RoPE rows, and the uint8 block mask (128 x 64 tiles) keeps the
attention kernel off tiles that mix documents (reference forward_packed.py:25-72).
Also the Euler update of the sampler (src_ii/triumphant_future_reduction_ops.py:56-62,
the per-image ``denoise_all`` of src_ii/batch_executor.py).
"""

from __future__ import annotations

from typing import Any

import torch
from torch import Tensor

from .bin_packer import REFERENCE_TOTAL_LEN
from .block_mask import build_block_mask, build_block_mask_from_packing_info


def _pad_plan_to_fixed_len(packing_info, packed_rope: Tensor, target_len: int = REFERENCE_TOTAL_LEN):
    """Extend document_id with -1 and packed_rope (B, L, ...) with zero rows up to
    ``target_len`` (reference :25-72).  Raises ValueError if the plan is longer."""
    n = packing_info.total_len
    if n > target_len:
        raise ValueError(f"Packed sequence length {n} exceeds REFERENCE_TOTAL_LEN {target_len}. Content doesn't fit.")
    if n == target_len:
        return packing_info, packed_rope
    extra = target_len - n
    doc = packing_info.document_id
    packing_info.document_id = torch.cat([doc, torch.full((extra,), -1, dtype=doc.dtype, device=doc.device)])
    packing_info.total_len = target_len
    tail = packed_rope.new_zeros(packed_rope.shape[0], extra, *packed_rope.shape[2:])
    return packing_info, torch.cat([packed_rope, tail], dim=1)


def prepare_packed_forward(model, context_list: list[Tensor], img_sizes: list[tuple[int, int]],
                           cap_lens: list[int], device, target_len: int = REFERENCE_TOTAL_LEN) -> dict[str, Any]:
    """model.prepare_packed_state, padded to ``target_len``, plus its block mask (:75-101)."""
    refined_caps, packing_info, packed_rope = model.prepare_packed_state(context_list, img_sizes, cap_lens, device)
    packing_info, packed_rope = _pad_plan_to_fixed_len(packing_info, packed_rope, target_len)
    return {
        "refined_caps": refined_caps,
        "packing_info": packing_info,
        "packed_rope": packed_rope,
        "block_mask": build_block_mask_from_packing_info(packing_info, device=device),
    }


def packed_forward(model, x_list: list[Tensor], timesteps, refined_caps: list[Tensor], packing_info,
                   block_mask: Tensor, packed_rope: Tensor, adapter_scales: Tensor | None = None):
    """One packed forward with one timestep per image (:104-125)."""
    ts = timesteps if isinstance(timesteps, list) else [timesteps] * len(x_list)
    return model(x_list, ts, refined_caps, packing_info, block_mask, packed_rope, adapter_scales=adapter_scales)


def make_packed_model_fn(model, refined_caps, packing_info, block_mask, packed_rope, cfg: float,
                         multiplier: float, adapter_scales: Tensor | None = None):
    """Sampler callable fn(x_list, t, caps, info, mask, rope) (:128-147)."""
    def fn(x_cfg_list, t_batch, caps, info, mask, rope):
        return model(x_cfg_list, [t_batch] * len(x_cfg_list), caps, info, mask, rope,
                     adapter_scales=adapter_scales)
    return fn


def prepare_and_build_mask(segment_lengths: list[int], total_len: int | None = None,
                           device: torch.device | str = "cuda") -> Tensor:
    """Block mask from raw segment lengths, padded to ``REFERENCE_TOTAL_LEN`` (:150-158)."""
    return build_block_mask(segment_lengths, total_len=REFERENCE_TOTAL_LEN if total_len is None else total_len,
                            device=device)


def denoise_all(x_list: list[Tensor], fields: list[Tensor], sigmas: list[Tensor]) -> list[Tensor]:
    """x - field * sigma per image (reference triumphant_future_reduction_ops.py:52-53)."""
    return [x - f * s for x, f, s in zip(x_list, fields, sigmas)]


def euler_step(x_base: Tensor, guided: Tensor, sigma, sigma_next) -> Tensor:
    """x + (x - guided) / sigma * (sigma_next - sigma) (reference :56-58)."""
    d = (x_base - guided) / sigma
    return x_base + d * (sigma_next - sigma)
