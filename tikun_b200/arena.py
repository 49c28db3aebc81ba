"""Arena-resident leaf storage: the reference's LayoutPlan / MemoryArena
(crates/tikun-core/src/arena.rs:34-103) as one flat device allocation per state
array (p, g, m, v) with every leaf a view at its 64-byte-aligned offset.

One allocation per array means the leaf table never changes between steps, a
ZeRO-1 shard is a contiguous range of the flat buffer, and an all-gather of the
updated parameters is one collective over one buffer.
"""
from __future__ import annotations

from typing import Sequence

import torch

from . import _native


class LayoutPlan:
    """Offsets from tk_layout_from_shapes (64-byte aligned, f32 elements).

    ``slots`` holds (element offset, element count) per leaf; ``total`` is the
    element count of the arena, rounded up to ``pad_to`` elements so that equal
    per-rank shards tile it exactly."""

    def __init__(self, shapes: Sequence[int], pad_to: int = 16):
        offs, total_bytes = _native.layout_from_shapes([int(s) for s in shapes])
        self.sizes = [int(s) for s in shapes]
        self.slots = [(o // 4, n) for o, n in zip(offs, self.sizes)]
        n = (total_bytes + 3) // 4
        self.total = (n + pad_to - 1) // pad_to * pad_to

    def __len__(self):
        return len(self.sizes)


class Arena:
    """Flat zero-filled storage for one layout; ``leaf(i)`` is a view."""

    def __init__(self, plan: LayoutPlan, dtype=torch.float32, device="cuda"):
        self.plan = plan
        self.flat = torch.zeros(plan.total, dtype=dtype, device=device)

    def leaf(self, i: int) -> torch.Tensor:
        off, n = self.plan.slots[i]
        return self.flat[off:off + n]

    def leaves(self) -> list[torch.Tensor]:
        return [self.leaf(i) for i in range(len(self.plan))]

    def ptrs(self) -> list[int]:
        base = self.flat.data_ptr()
        es = self.flat.element_size()
        return [base + off * es for off, _ in self.plan.slots]


def shard_bounds(total: int, world: int, rank: int, align: int = 16) -> tuple[int, int]:
    """ZeRO-1 ownership: rank r owns elements [lo, hi) of the flat space; equal
    aligned shards (``total`` must be a multiple of world * align)."""
    if total % (world * align) != 0:
        raise ValueError(f"arena of {total} elements does not split into {world} shards of "
                         f"{align}-element granules")
    per = total // world
    return rank * per, (rank + 1) * per


def shard_segments(plan: LayoutPlan, lo: int, hi: int) -> list[tuple[int, int, int]]:
    """The pieces of the leaves inside flat range [lo, hi): (leaf, start, count).

    The update is pointwise, so a shard may cut a leaf anywhere; padding
    between leaves belongs to no leaf and is skipped."""
    out = []
    for i, (off, n) in enumerate(plan.slots):
        a, b = max(off, lo), min(off + n, hi)
        if a < b:
            out.append((i, a - off, b - a))
    return out
