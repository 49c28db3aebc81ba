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


def _sym_tiles(tm: int, tn: int, bm: int, bn: int) -> int:
    """Tiles on or above the diagonal: row block i starts at the column block
    holding row i * bm."""
    return sum(tn - (i * bm) // bn for i in range(tm))


# the engine's tiling rules (tikun_b200/csrc/tk_ns.cu): symmetric products
# computed on every tile up to these K, and the CTA-pair kernel's 256 x 256
# tiles from this many rows on
NS_FULL_K1, NS_FULL_K2, NS_PAIR_MIN_M = 1024, 512, 1024


def ns_issued_flops(rows: int, cols: int, steps: int = 5, bk: int = 64) -> int:
    """FLOPs the tensor cores actually execute for the engine's tiling: 128 x 256
    tiles below NS_PAIR_MIN_M rows and 256 x 256 tiles (CTA pairs) from there
    on; X X^T (K = n) and A A' (K = m) on the tiles on and above the diagonal,
    or on every tile when K is at most NS_FULL_K1 / NS_FULL_K2; every
    dimension rounded up to whole tiles."""
    m, n = min(rows, cols), max(rows, cols)
    bm, bn = (256, 256) if m >= NS_PAIR_MIN_M else (128, 256)
    tm, tn = -(-m // bm), -(-m // bn)
    kx, km = -(-n // bk) * bk, -(-m // bk) * bk
    full = tm * tn * 2 * bm * bn
    sym = _sym_tiles(tm, tn, bm, bn) * 2 * bm * bn
    g1 = (full if n <= NS_FULL_K1 else sym) * kx
    g2 = (full if m <= NS_FULL_K2 else sym) * km
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
