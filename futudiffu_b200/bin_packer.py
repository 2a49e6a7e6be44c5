"""Bin scheduling of packed multi-image forwards: drop-in for ``src_ii.bin_packer``.

A bin is one packed sequence of at most ``max_seq_len`` tokens (one forward
pass of the block-masked DiT).  Each item costs its caption tokens plus its
image patch tokens, each padded to a multiple of 32 (the packed layout of
``transformer.build_packed_sequence``).  Items are placed first-fit in order of
decreasing cost, ties broken by input position (reference bin_packer.py:380-497),
so the schedule is deterministic.

Pure Python, like the reference: the schedule is host work done once per
generation plan, and its output feeds the device-side packing (row ranges and
block masks) of each bin.  The reference's deprecated fixed resolution tiers are
not carried over.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Any

_REF_W, _REF_H = 1280, 832
_MAX_SHIFT = 8.0


def _resolution_shift(width: int, height: int) -> float:
    """sqrt(reference pixels / pixels), at most 8 (reference :52-63)."""
    if width * height <= 0:
        raise ValueError(f"Invalid resolution: {width}x{height}")
    return min(math.sqrt(_REF_W * _REF_H / (width * height)), _MAX_SHIFT)


def compute_seq_len(width: int, height: int, vae_scale: int = 8, patch_size: int = 2) -> int:
    """Image patch tokens: (H / vae / patch) * (W / vae / patch), floor at each step (:70-93)."""
    return ((height // vae_scale) // patch_size) * ((width // vae_scale) // patch_size)


def _pad_to_multiple(n: int, multiple: int) -> int:
    return -(-n // multiple) * multiple


def compute_effective_seq_len(width: int, height: int, cap_tokens: int, pad_multiple: int = 32,
                              vae_scale: int = 8, patch_size: int = 2) -> int:
    """Tokens one item occupies in a packed sequence: padded caption + padded image (:101-126)."""
    return (_pad_to_multiple(cap_tokens, pad_multiple)
            + _pad_to_multiple(compute_seq_len(width, height, vae_scale, patch_size), pad_multiple))


def validate_resolution(width: int, height: int, step: int = 32, vae_scale: int = 8, patch_size: int = 2) -> None:
    """Raise ValueError unless both sides are >= 64 and multiples of ``step`` and of
    vae_scale * patch_size (:129-177)."""
    if width <= 0 or height <= 0:
        raise ValueError(f"Resolution must be positive: {width}x{height}")
    if width < 64 or height < 64:
        raise ValueError(f"Resolution {width}x{height} has dimension < 64. Both width and height must be >= 64.")
    if width % step or height % step:
        raise ValueError(f"Resolution {width}x{height} not aligned to {step}. "
                         f"Both width and height must be divisible by {step}.")
    align = vae_scale * patch_size
    if width % align or height % align:
        raise ValueError(f"Resolution {width}x{height} not aligned to {align}. Width and height must be "
                         f"divisible by {align} (vae_scale={vae_scale} * patch_size={patch_size}).")


REFERENCE_SEQ_LEN = compute_seq_len(_REF_W, _REF_H)          # 4160 image tokens
DEFAULT_CAP_TOKENS = 113                                      # p99 caption length of the reference's data
REFERENCE_TOTAL_LEN = compute_effective_seq_len(_REF_W, _REF_H, DEFAULT_CAP_TOKENS)  # 4288


def estimate_sparse_compute_ratio(utilization: float) -> float:
    """Block-diagonal attention cost of a bin relative to a dense one, for a single
    image filling ``utilization`` of it: utilization**2, clamped to [0, 1] (:300-339)."""
    if utilization <= 0.0:
        return 0.0
    if utilization >= 1.0:
        return 1.0
    return utilization * utilization


def estimate_sparse_compute_ratio_detailed(effective_seq_lens: list[int], capacity: int) -> float:
    """sum(s_i**2) / capacity**2 (:342-362)."""
    if capacity <= 0:
        return 0.0
    return sum(s * s for s in effective_seq_lens) / (capacity * capacity)


@dataclass
class Bin:
    """One packed forward pass (reference :369-383)."""
    items: list[dict] = field(default_factory=list)
    used_seq_len: int = 0
    capacity: int = 0

    def remaining(self) -> int:
        return self.capacity - self.used_seq_len

    def can_fit(self, seq_len: int) -> bool:
        return self.used_seq_len + seq_len <= self.capacity

    def add(self, item: dict) -> None:
        self.items.append(item)
        self.used_seq_len += item["seq_len"]


class BinPackScheduler:
    """First-fit-decreasing packing of items with a ``seq_len`` into bins of
    ``max_seq_len`` tokens (reference :386-681)."""

    def __init__(self, max_seq_len: int = REFERENCE_TOTAL_LEN, default_cap_tokens: int = DEFAULT_CAP_TOKENS):
        if max_seq_len <= 0:
            raise ValueError(f"max_seq_len must be positive, got {max_seq_len}")
        self.max_seq_len = max_seq_len
        self.default_cap_tokens = default_cap_tokens

    def pack(self, items: list[dict]) -> list[list[dict]]:
        """Bins in creation order, each listing its items largest first.  An item
        larger than a bin gets a bin of its own."""
        order = sorted(range(len(items)), key=lambda i: (-items[i]["seq_len"], i))
        bins: list[Bin] = []
        # first fit; `free` mirrors each bin's remaining room for a quick scan
        free: list[int] = []
        for i in order:
            item = items[i]
            need = item["seq_len"]
            for j, room in enumerate(free):
                if need <= room:
                    bins[j].add(item)
                    free[j] = room - need
                    break
            else:
                b = Bin(capacity=self.max_seq_len)
                b.add(item)
                bins.append(b)
                free.append(self.max_seq_len - need)
        return [b.items for b in bins]

    def pack_generation_plan(self, plan: list[dict]) -> list[list[dict]]:
        """Pack plan items ('width', 'height', optional 'cap_tokens'); each item is
        copied and given 'img_seq_len', 'cap_tokens' and 'seq_len'."""
        items = []
        for it in plan:
            cap = it.get("cap_tokens", self.default_cap_tokens)
            d = dict(it)
            d["img_seq_len"] = compute_seq_len(it["width"], it["height"])
            d["cap_tokens"] = cap
            d["seq_len"] = compute_effective_seq_len(it["width"], it["height"], cap)
            items.append(d)
        return self.pack(items)

    def pack_for_training(self, items: list[tuple[int, str, int, int]]) -> list[list[tuple[int, str, int, int]]]:
        """Pack (traj_id, step_key, width, height) tuples with the default caption length."""
        dicts = [{"traj_id": t, "step_key": k, "width": w, "height": h,
                  "seq_len": compute_effective_seq_len(w, h, self.default_cap_tokens)} for t, k, w, h in items]
        return [[(d["traj_id"], d["step_key"], d["width"], d["height"]) for d in b] for b in self.pack(dicts)]

    def estimate_efficiency(self, bins: list[list[dict]]) -> dict[str, Any]:
        """Utilisation and block-diagonal attention cost of a schedule (:580-681)."""
        cap = self.max_seq_len
        if not bins:
            return {"n_bins": 0, "n_items": 0, "total_capacity": 0, "total_used": 0, "total_wasted": 0,
                    "utilization": 0.0, "sparse_compute_ratio": 0.0, "per_bin": []}
        per_bin = []
        for b in bins:
            lens = [it["seq_len"] for it in b]
            used = sum(lens)
            per_bin.append({
                "n_items": len(b), "used": used, "capacity": cap,
                "utilization": used / cap if cap > 0 else 0.0, "wasted": cap - used,
                "sparse_compute_ratio": round(estimate_sparse_compute_ratio_detailed(lens, cap), 4),
            })
        total_used = sum(p["used"] for p in per_bin)
        total_cap = cap * len(bins)
        sq = sum(it["seq_len"] ** 2 for b in bins for it in b)
        return {
            "n_bins": len(bins), "n_items": sum(p["n_items"] for p in per_bin),
            "total_capacity": total_cap, "total_used": total_used, "total_wasted": total_cap - total_used,
            "utilization": total_used / total_cap if total_cap > 0 else 0.0,
            "sparse_compute_ratio": round(sq / (cap * cap * len(bins)) if cap > 0 else 0.0, 4),
            "per_bin": per_bin,
        }
