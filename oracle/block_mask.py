"""Packed-sequence block mask (oracle; test infrastructure only).

build_block_mask, src_ii/block_mask.py:66-99: document id of each token
(tokens past the listed segments keep id 0), each 128-row Q block and 64-key
KV block takes the id of its first token, mask = equality.
"""

from __future__ import annotations

import numpy as np


def build_block_mask(segment_lengths, total_len=None) -> np.ndarray:
    if total_len is None:
        total_len = int(sum(segment_lengths))
    doc = np.zeros(total_len, dtype=np.int32)
    off = 0
    for i, n in enumerate(segment_lengths):
        doc[off:off + n] = i
        off += n
    nq = (total_len + 127) // 128
    nk = (total_len + 63) // 64
    qd = doc[np.minimum(np.arange(nq) * 128, total_len - 1)]
    kd = doc[np.minimum(np.arange(nk) * 64, total_len - 1)]
    return (qd[:, None] == kd[None, :]).astype(np.uint8)
