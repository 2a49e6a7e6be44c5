"""uint8 block-diagonal attention masks for packed sequences: drop-in for
``src_ii.block_mask``.

Tile granularity is the attention kernel's mask granularity: 128 query rows by
64 keys (reference src_ii/block_mask.py:28-29).  Semantics follow
``build_block_mask`` (:35-99) exactly, including that each block takes the
document id of its first token and that tokens beyond the listed segments keep
document id 0 (so a padding tail is attended by image 0, reference quirk).
"""

from __future__ import annotations

import torch

BLOCK_M: int = 128
BLOCK_N: int = 64


def _ceildiv(a: int, b: int) -> int:
    return (a + b - 1) // b


def build_block_mask(
    segment_lengths: list[int],
    total_len: int | None = None,
    device: torch.device | str = "cuda",
) -> torch.Tensor:
    """(ceil(T/128), ceil(T/64)) uint8 mask: 1 where the Q and KV blocks share a document."""
    if total_len is None:
        total_len = sum(segment_lengths)
    n_q_blocks = _ceildiv(total_len, BLOCK_M)
    n_kv_blocks = _ceildiv(total_len, BLOCK_N)
    doc_ids = torch.zeros(total_len, dtype=torch.int32, device=device)
    offset = 0
    for img_idx, seg_len in enumerate(segment_lengths):
        doc_ids[offset:offset + seg_len] = img_idx
        offset += seg_len
    q_starts = (torch.arange(n_q_blocks, device=device) * BLOCK_M).clamp(max=total_len - 1)
    kv_starts = (torch.arange(n_kv_blocks, device=device) * BLOCK_N).clamp(max=total_len - 1)
    q_doc = doc_ids[q_starts]
    kv_doc = doc_ids[kv_starts]
    return (q_doc.unsqueeze(1) == kv_doc.unsqueeze(0)).to(torch.uint8)


def build_block_mask_from_packing_info(packing_info, device: torch.device | str = "cuda") -> torch.Tensor:
    """Mask from a PackingInfo (segments of (text_start, text_len, img_start, img_len))."""
    segment_lengths = [text_len + img_len for (_ts, text_len, _is, img_len) in packing_info.segments]
    return build_block_mask(segment_lengths, total_len=packing_info.total_len, device=device)
