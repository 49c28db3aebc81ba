"""Work division across ranks (one process per GPU).

* AdamW: ZeRO-1 over the flat parameter arena (``arena.shard_bounds``,
  ``arena.shard_segments``): contiguous equal slices, leaf boundaries ignored
  because the update is pointwise.
* Muon: whole matrices are owned by one rank each, assigned by
  longest-processing-time bin-packing on their Newton-Schulz FLOPs, so every
  rank's tensor-core work is about equal.  Each rank steps the matrices it
  owns; the updated parameters are then gathered.  ``owner_major_layout`` lays
  the matrices out rank by rank with equal padded per-rank extents so that one
  all-gather of the whole parameter buffer reassembles them.
"""
from __future__ import annotations

from typing import Sequence


def ns_dense_flops(rows: int, cols: int, steps: int = 5) -> int:
    """Dense-equivalent FLOPs of Newton-Schulz on a rows x cols matrix:
    steps * (4 m^2 n + 2 m^3) with m = min, n = max (X X^T, A A, B X)."""
    m, n = min(rows, cols), max(rows, cols)
    return steps * (4 * m * m * n + 2 * m ** 3)


def _sym_tiles(tm: int, tn: int) -> int:
    return sum(tn - (i >> 1) for i in range(tm))


def ns_issued_flops(rows: int, cols: int, steps: int = 5, bm: int = 128, bn: int = 256,
                    bk: int = 64) -> int:
    """FLOPs the tensor cores actually execute for the engine's tiling: 128x256
    tiles, symmetric GEMMs (X X^T, A A) only on and above the diagonal, every
    dimension rounded up to whole tiles."""
    m, n = min(rows, cols), max(rows, cols)
    tm, tn = -(-m // bm), -(-m // bn)
    kx, km = -(-n // bk) * bk, -(-m // bk) * bk
    sym = _sym_tiles(tm, tn) * 2 * bm * bn
    g1 = sym * kx
    g2 = sym * km
    g3 = (-(-n // bm)) * tn * 2 * bm * bn * km
    return steps * (g1 + g2 + g3)


def lpt_assign(costs: Sequence[float], world: int) -> list[int]:
    """Owner rank of each item: items in decreasing cost go to the rank with the
    least load so far (ties: lowest rank; equal costs keep their order)."""
    order = sorted(range(len(costs)), key=lambda i: (-costs[i], i))
    load = [0.0] * world
    owner = [0] * len(costs)
    for i in order:
        r = min(range(world), key=lambda k: (load[k], k))
        owner[i] = r
        load[r] += costs[i]
    return owner


def owner_major_layout(sizes: Sequence[int], owner: Sequence[int], world: int,
                       align: int = 64) -> tuple[list[int], int]:
    """Element offset of each matrix in a buffer laid out rank by rank, and the
    per-rank extent (equal for every rank, a multiple of ``align``).  Rank r's
    matrices live in [r * extent, (r + 1) * extent)."""
    cursor = [0] * world
    offs = [0] * len(sizes)
    for i, n in enumerate(sizes):
        r = owner[i]
        offs[i] = cursor[r]
        cursor[r] += -(-n // align) * align
    extent = max(cursor) if cursor else 0
    extent = -(-max(extent, align) // align) * align
    return [offs[i] + owner[i] * extent for i in range(len(sizes))], extent
