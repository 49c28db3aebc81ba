"""Property tests (random inputs) for the host-side partitioning that every path
depends on: the LayoutPlan offsets (crates/tikun-core/src/arena.rs:34-57), the
ZeRO-1 and chunk-major ownership of the flat arena, and the LPT assignment and
owner-major layout of Muon matrices, in Python and through the C ABI."""
import ctypes

import numpy as np
from hypothesis import example, given, settings
from hypothesis import strategies as st

import oracle
from tikun_b200 import _native
from tikun_b200.arena import LayoutPlan, shard_bounds, shard_segments
from tikun_b200.distributed import chunk_major_pieces, pieces_to_segments
from tikun_b200.sharding import lpt_assign, ns_dense_flops, owner_major_layout

leaf_sizes = st.lists(st.integers(min_value=1, max_value=70_000), min_size=1, max_size=40)
worlds = st.integers(min_value=1, max_value=8)
shapes = st.lists(st.tuples(st.integers(1, 600), st.integers(1, 600)), min_size=1, max_size=60)


@settings(max_examples=150, deadline=None)
@given(leaf_sizes)
def test_native_layout_equals_the_oracle_and_is_aligned(sizes):
    offs, total = _native.layout_from_shapes(sizes)
    assert (offs, total) == oracle.layout_from_shapes(sizes)
    assert all(o % 64 == 0 for o in offs)
    ends = [o + 4 * n for o, n in zip(offs, sizes)]
    assert all(e <= o for e, o in zip(ends, offs[1:])) and total == ends[-1]


@settings(max_examples=150, deadline=None)
@given(leaf_sizes, worlds)
def test_zero1_shards_cover_every_element_once(sizes, world):
    plan = LayoutPlan(sizes, pad_to=16 * world)
    seen = [np.zeros(n, np.int8) for n in sizes]
    for r in range(world):
        lo, hi = shard_bounds(plan.total, world, r)
        assert lo % 16 == 0 and hi % 16 == 0 and hi - lo == plan.total // world
        for i, a, c in shard_segments(plan, lo, hi):
            seen[i][a:a + c] += 1
    assert all((s == 1).all() for s in seen)


@settings(max_examples=100, deadline=None)
@given(leaf_sizes, worlds, st.integers(min_value=1, max_value=6))
def test_chunk_major_pieces_cover_every_element_once(sizes, world, chunks):
    plan = LayoutPlan(sizes, pad_to=16 * world * chunks)
    seen = [np.zeros(n, np.int8) for n in sizes]
    for r in range(world):
        for lo, hi in chunk_major_pieces(plan.total, world, r, chunks):
            assert lo % 16 == 0
            for i, a, c in pieces_to_segments(plan, lo, hi):
                seen[i][a:a + c] += 1
    assert all((s == 1).all() for s in seen)


@settings(max_examples=150, deadline=None)
@given(shapes, worlds)
def test_lpt_and_owner_major_layout_native_equals_python(mats, world):
    costs = [ns_dense_flops(r, c) for r, c in mats]
    owner = lpt_assign(costs, world)
    load = [0] * world
    for i, w in enumerate(owner):
        load[w] += costs[i]
    # greedy onto the least-loaded rank keeps the spread within one matrix
    assert max(load) - min(load) <= max(costs)
    sizes = [r * c for r, c in mats]
    offs, extent = owner_major_layout(sizes, owner, world)
    assert extent % 64 == 0
    for i, (o, n) in enumerate(zip(offs, sizes)):
        assert o % 64 == 0 and owner[i] * extent <= o and o + n <= (owner[i] + 1) * extent
    spans = sorted(zip(offs, sizes))
    assert all(a + n <= b for (a, n), (b, _) in zip(spans, spans[1:]))

    n = len(mats)
    rows = (ctypes.c_int64 * n)(*[r for r, _ in mats])
    cols = (ctypes.c_int64 * n)(*[c for _, c in mats])
    own = (ctypes.c_int32 * n)()
    off = (ctypes.c_uint64 * n)()
    ext = ctypes.c_uint64()
    _native.check(_native.lib().tk_muon_layout(n, rows, cols, world, own, off, ctypes.byref(ext)))
    assert list(own) == owner and list(off) == offs and ext.value == extent


# -- verifier text: crates/tikun-core/src/verifier.rs:14-45 with Rust's {:?} --
def _rust_debug(s):
    out = '"'
    for ch in s:
        code = ord(ch)
        if ch in "\t\r\n\\\"":
            out += {"\t": "\\t", "\r": "\\r", "\n": "\\n", "\\": "\\\\", '"': '\\"'}[ch]
        elif code < 0x20 or code == 0x7f:
            out += "\\u{%x}" % code
        else:
            out += ch
    return out + '"'


def _expected(nodes):
    if not nodes:
        return "Static verification failed: [EmptyPipeline]"
    errs = []
    for name, _, tile, _, width, _ in nodes:
        if tile % 64 != 0:
            errs.append(f"MisalignedCacheLine {{ node_name: {_rust_debug(name)}, tile_size: {tile} }}")
        if width < 4 or width & (width - 1):
            errs.append(f"InvalidVectorWidth {{ node_name: {_rust_debug(name)}, width: {width} }}")
    return "Static verification failed: [" + ", ".join(errs) + "]" if errs else None


ascii_names = st.text(alphabet=st.characters(min_codepoint=1, max_codepoint=127), max_size=10)
nodes = st.lists(st.tuples(ascii_names, st.integers(0, 2), st.integers(0, 1 << 20),
                           st.integers(0, 8),
                           st.one_of(st.sampled_from([0, 1, 2, 3, 4, 6, 8, 16, 64, 1 << 40]),
                                     st.integers(0, 1 << 16)),
                           st.integers(0, 256)), max_size=6)


@settings(max_examples=300, deadline=None)
@given(nodes)
def test_verifier_text_matches_rust_debug_formatting(nodes):
    want = _expected(nodes)
    try:
        _native.verify(nodes)
        got = None
    except _native.TikunError as e:
        got = str(e)
    assert got == want


# -- the Muon exchange's copy kernel (peer_copy_kernel in tikun_b200/csrc/tk_ns.cu) --
def _peer_copy_units(entry_bytes, grid, threads=512, unroll=4):
    """The kernel's work split restated: 16-byte units numbered across the
    entries (unit0 prefix sums), an equal contiguous range per CTA, each thread
    walking its units in order with a cursor over the entries.  Returns
    per-entry byte coverage counts."""
    unit0 = [0]
    for b in entry_bytes:
        unit0.append(unit0[-1] + (b + 15) // 16)
    total, n = unit0[-1], len(entry_bytes)
    cover = [np.zeros(b, np.int32) for b in entry_bytes]
    per = (total + grid - 1) // grid
    for blk in range(grid):
        u0, u1 = blk * per, min(blk * per + per, total)
        for t in range(threads):
            e = 0
            base = u0
            while base < u1:
                for k in range(unroll):
                    u = base + k * threads + t
                    if u >= u1:
                        continue
                    while e + 1 < n and unit0[e + 1] <= u:
                        e += 1
                    off = (u - unit0[e]) * 16
                    rem = entry_bytes[e] - off
                    ln = 16 if rem >= 16 else rem
                    assert 0 < ln <= 16 and off + ln <= entry_bytes[e]
                    cover[e][off:off + ln] += 1
                base += threads * unroll
    return cover


@settings(max_examples=40, deadline=None)
@given(st.lists(st.integers(min_value=0, max_value=40_000), min_size=1, max_size=6),
       st.integers(min_value=1, max_value=12))
def test_peer_copy_split_copies_every_byte_once(entry_bytes, grid):
    cover = _peer_copy_units(entry_bytes, grid, threads=64, unroll=4)
    assert all((c == 1).all() for c in cover)


# -- the pointwise update's and the Tier-1 norm's work split
# (pointwise_kernel and sumsq_partials_kernel in tk_pointwise.cu) --
def _pointwise_cover(sizes, vec_ok, grid, threads=256, unroll=4):
    """The kernels' split restated: the leaves' 4-element groups ("quads") in
    one index space, an equal contiguous quad range per CTA, the leaf found by
    binary search on q_begin, whole quads of aligned leaves through the
    unrolled vector loop (trips of `unroll` quads `threads` apart; the
    pipelined update loop visits the same trips, loading one ahead) and the
    rest element by element.  Returns per-leaf element coverage, and whether
    any vector access ran past a leaf's end."""
    q_begin, total = [], 0
    for n in sizes:
        q_begin.append(total)
        total += (n + 3) // 4
    cover = [np.zeros(n, np.int32) for n in sizes]
    past_end = False
    for blk in range(grid):
        q0, q1 = total * blk // grid, total * (blk + 1) // grid
        if q0 >= q1:
            continue
        lo, hi = 0, len(sizes) - 1  # last leaf with q_begin <= q0
        while lo < hi:
            mid = (lo + hi + 1) >> 1
            lo, hi = (mid, hi) if q_begin[mid] <= q0 else (lo, mid - 1)
        li, q = lo, q0
        while q < q1:
            n = sizes[li]
            seg_end = min(q1, q_begin[li] + (n + 3) // 4)
            a, b = q - q_begin[li], seg_end - q_begin[li]
            full_end = min(b, n >> 2) if vec_ok[li] else a
            for t in range(threads):
                lq = np.arange(a + t, full_end, threads * unroll)
                qq = (lq[:, None] + np.arange(unroll)[None, :] * threads).ravel()
                qq = qq[qq < full_end]
                past_end |= bool((qq * 4 + 4 > n).any())
                for j in range(4):
                    np.add.at(cover[li], qq * 4 + j, 1)
                for tq in range(max(a, full_end) + t, b, threads):
                    cover[li][tq * 4:min(tq * 4 + 4, n)] += 1
            q = seg_end
            li += 1
    return cover, past_end


@settings(max_examples=60, deadline=None)
@given(st.lists(st.tuples(st.integers(min_value=1, max_value=6000), st.booleans()),
                min_size=1, max_size=6),
       st.integers(min_value=1, max_value=9),
       st.sampled_from([(32, 4), (64, 2), (16, 1), (256, 5), (256, 4), (256, 1)]))
def test_pointwise_split_updates_every_element_once(leaves, grid, shape):
    # (256, 5): the pipelined f32 update; (256, 1): bf16 leaves; (256, 4): the
    # Tier-1 norm's four accumulators
    sizes = [n for n, _ in leaves]
    vec_ok = [v for _, v in leaves]
    cover, past_end = _pointwise_cover(sizes, vec_ok, grid, threads=shape[0], unroll=shape[1])
    assert not past_end
    assert all((c == 1).all() for c in cover)


# -- symmetric GEMM tiles (decode_tile / sym_store in tikun_b200/csrc/tk_ns.cu) --
def _sym_writes(m, bm=128, bn=256):
    """The symmetric products' tile plan restated: row block i computes the
    128 x 256 column blocks floor(i/2) .. tiles_n-1, and the epilogue writes
    each entry (r, c) with c >= r of its tile plus the mirror (c, r) for
    c > r.  Returns how often each entry of the m x m output is written."""
    tiles_m, tiles_n = -(-m // bm), -(-m // bn)
    n_tiles = sum(tiles_n - (i >> 1) for i in range(tiles_m))
    writes = np.zeros((m, m), np.int32)
    for t in range(n_tiles):
        r = t
        for i in range(tiles_m):
            cnt = tiles_n - (i >> 1)
            assert cnt >= 1
            if r < cnt:
                tm, tn = i, (i >> 1) + r
                break
            r -= cnt
        rows = np.arange(tm * bm, min(tm * bm + bm, m))
        cols = np.arange(tn * bn, min(tn * bn + bn, m))
        R, C = np.meshgrid(rows, cols, indexing="ij")
        up = C >= R
        np.add.at(writes, (R[up], C[up]), 1)
        lo = C > R
        np.add.at(writes, (C[lo], R[lo]), 1)
    return writes


@settings(max_examples=40, deadline=None)
@given(st.integers(min_value=1, max_value=1100))
@example(1)
@example(127)
@example(128)
@example(129)
@example(255)
@example(256)
@example(257)
@example(383)
@example(384)
@example(385)
@example(768)
@example(1024)
def test_symmetric_tiles_write_every_entry_once(m):
    assert (_sym_writes(m) == 1).all()
