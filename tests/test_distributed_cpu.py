"""Host-side logic of the multi-GPU step, on CPU.

* ZeRO-1 slices of the flat arena cover every leaf element exactly once.
* LPT bin-packing of Muon matrices by Newton-Schulz FLOPs is deterministic
  and balanced; the owner-major layout gives disjoint, aligned, per-rank ranges.
* A 2-rank gloo run of the step's choreography: each rank transforms only the
  elements it owns (a stand-in for the device update, done on CPU tensors), the
  f64 partial sums are all-reduced, and one all-gather per buffer reassembles
  identical full buffers on every rank.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from tikun_b200.arena import LayoutPlan, shard_bounds, shard_segments
from tikun_b200.sharding import (lpt_assign, ns_dense_flops, ns_issued_flops,
                                 owner_major_layout)


def llama8b_mats():
    d, kv, ffn = 4096, 1024, 14336
    return [(d, d), (d, kv), (d, kv), (d, d), (d, ffn), (d, ffn), (ffn, d)] * 32


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_zero1_slices_cover_each_element_once(world):
    sizes = [50257 * 64, 17, 768, 1, 4097, 3 * 64 * 64]
    plan = LayoutPlan(sizes, pad_to=16 * world)
    seen = [np.zeros(n, np.int32) for n in sizes]
    for r in range(world):
        lo, hi = shard_bounds(plan.total, world, r)
        assert lo % 16 == 0 and hi % 16 == 0
        for i, a, c in shard_segments(plan, lo, hi):
            seen[i][a:a + c] += 1
    assert all((s == 1).all() for s in seen)


def test_shard_bounds_rejects_unaligned_arena():
    with pytest.raises(ValueError):
        shard_bounds(100, 3, 0)


@pytest.mark.parametrize("world", [2, 4, 8])
def test_lpt_balances_llama8b_newton_schulz(world):
    mats = llama8b_mats()
    costs = [ns_dense_flops(r, c) for r, c in mats]
    owner = lpt_assign(costs, world)
    assert owner == lpt_assign(costs, world)  # deterministic
    load = [0] * world
    for i, r in enumerate(owner):
        load[r] += costs[i]
    # the 4096x14336 matrices (5.5 TFLOP each) dominate; LPT keeps every rank
    # within one such matrix of the mean
    assert max(load) - min(load) <= max(costs)
    assert max(load) / (sum(load) / world) < 1.05


def test_ns_flop_accounting():
    assert ns_dense_flops(768, 768) == 5 * (4 * 768 ** 3 + 2 * 768 ** 3)
    assert ns_dense_flops(3072, 768) == ns_dense_flops(768, 3072)
    total = sum(ns_dense_flops(r, c) for r, c in llama8b_mats())
    assert abs(total / 1e12 - 665.9) < 0.05
    # symmetric tiles save work: issued < dense-equivalent for square matrices
    assert ns_issued_flops(4096, 4096) < ns_dense_flops(4096, 4096)
    # at short K every tile is computed: 512^2 issues the dense FLOPs; 768^2
    # computes X X^T in full (K = 768 <= 1024) and 12 of A A''s 18 tiles
    assert ns_issued_flops(512, 512) == ns_dense_flops(512, 512)
    assert ns_issued_flops(768, 768) * 18 == ns_dense_flops(768, 768) * 16
    # the CTA-pair tiling (256 x 256 from 1024 rows on) covers the same upper
    # tiles as the 128 x 256 one when m is a multiple of 256
    m, n = 4096, 14336
    upper = 16 * 17 // 2 * 256 * 256
    assert ns_issued_flops(m, n) == 5 * (2 * upper * n + 2 * upper * m + 2 * n * m * m)


def test_owner_major_layout_is_disjoint_and_aligned():
    mats = llama8b_mats()[:14]
    sizes = [r * c for r, c in mats]
    owner = lpt_assign([ns_dense_flops(r, c) for r, c in mats], 4)
    offs, extent = owner_major_layout(sizes, owner, 4)
    spans = sorted((offs[i], offs[i] + sizes[i], owner[i]) for i in range(len(sizes)))
    for (a0, a1, ra), (b0, b1, rb) in zip(spans, spans[1:]):
        assert a1 <= b0
    for i, o in enumerate(offs):
        assert o % 64 == 0
        assert owner[i] * extent <= o and o + sizes[i] <= (owner[i] + 1) * extent


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, result_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        # ZeRO-1 pointwise part
        sizes = [1000, 17, 4097, 64]
        plan = LayoutPlan(sizes, pad_to=16 * world)
        g = torch.Generator().manual_seed(0)
        p = torch.randn(plan.total, generator=g, dtype=torch.float64)
        grad = torch.randn(plan.total, generator=g, dtype=torch.float64)
        lo, hi = shard_bounds(plan.total, world, rank)
        local = torch.zeros(1, dtype=torch.float64)
        for i, a, c in shard_segments(plan, lo, hi):
            off = plan.slots[i][0] + a
            local += (grad[off:off + c] ** 2).sum()
        dist.all_reduce(local)  # f64 sum of squares over ranks
        mask = torch.zeros(plan.total, dtype=torch.bool)
        for i, a, c in shard_segments(plan, lo, hi):
            off = plan.slots[i][0] + a
            mask[off:off + c] = True
        new_p = p.clone()
        new_p[mask] = p[mask] - 0.1 * grad[mask]
        parts = [torch.empty(hi - lo, dtype=torch.float64) for _ in range(world)]
        dist.all_gather(parts, new_p[lo:hi].contiguous())
        gathered = torch.cat(parts)
        # Muon part: owner-major buffer, one gather of equal extents
        mats = [(64, 96), (96, 64), (32, 32), (128, 64), (16, 48)]
        msz = [r * c for r, c in mats]
        owner = lpt_assign([ns_dense_flops(r, c) for r, c in mats], world)
        offs, extent = owner_major_layout(msz, owner, world)
        buf = torch.zeros(extent * world, dtype=torch.float64)
        for i in range(len(mats)):
            if owner[i] == rank:
                buf[offs[i]:offs[i] + msz[i]] = float(i + 1)
        mparts = [torch.empty(extent, dtype=torch.float64) for _ in range(world)]
        dist.all_gather(mparts, buf[rank * extent:(rank + 1) * extent].contiguous())
        mfull = torch.cat(mparts)
        result_q.put((rank, local.item(), gathered.numpy(), mfull.numpy(), offs, msz))
    finally:
        dist.destroy_process_group()


def test_two_rank_gloo_choreography():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    res.sort(key=lambda x: x[0])
    sizes = [1000, 17, 4097, 64]
    plan = LayoutPlan(sizes, pad_to=16 * world)
    g = torch.Generator().manual_seed(0)
    p = torch.randn(plan.total, generator=g, dtype=torch.float64)
    grad = torch.randn(plan.total, generator=g, dtype=torch.float64)
    want_ss = sum(float((grad[o:o + n] ** 2).sum()) for o, n in plan.slots)
    want = p.clone()
    for o, n in plan.slots:
        want[o:o + n] = p[o:o + n] - 0.1 * grad[o:o + n]
    for rank, ss, gathered, mfull, offs, msz in res:
        assert abs(ss - want_ss) <= 1e-12 * want_ss
        for o, n in plan.slots:
            np.testing.assert_array_equal(gathered[o:o + n], want[o:o + n].numpy())
        for i, (o, n) in enumerate(zip(offs, msz)):
            assert (mfull[o:o + n] == i + 1).all()
    np.testing.assert_array_equal(res[0][2], res[1][2])


@pytest.mark.parametrize("world,chunks", [(1, 1), (2, 4), (4, 4), (8, 3)])
def test_chunk_major_pieces_cover_the_arena(world, chunks):
    from tikun_b200.distributed import chunk_major_pieces, pieces_to_segments

    sizes = [50257 * 8, 17, 768, 1, 4097, 3 * 64 * 64]
    plan = LayoutPlan(sizes, pad_to=16 * world * chunks)
    seen = [np.zeros(n, np.int32) for n in sizes]
    cover = np.zeros(plan.total, np.int32)
    for r in range(world):
        pieces = chunk_major_pieces(plan.total, world, r, chunks)
        assert len(pieces) == chunks
        for c, (lo, hi) in enumerate(pieces):
            sup = plan.total // chunks
            assert c * sup <= lo < hi <= (c + 1) * sup and lo % 16 == 0
            cover[lo:hi] += 1
            for i, a, n in pieces_to_segments(plan, lo, hi):
                seen[i][a:a + n] += 1
    assert (cover == 1).all()
    assert all((s == 1).all() for s in seen)


def test_chunk_major_rejects_unaligned_arena():
    from tikun_b200.distributed import chunk_major_pieces

    with pytest.raises(ValueError):
        chunk_major_pieces(1000, 2, 0, 4)


@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_native_muon_layout_matches_python(world):
    """tk_muon_layout (the C ABI's LPT + owner-major layout) assigns and
    places every matrix exactly as tikun_b200.sharding does."""
    import ctypes

    from tikun_b200 import _native

    mats = llama8b_mats()[:21] + [(768, 3072), (3072, 768), (96, 40), (17, 45), (768, 768)] * 3
    n = len(mats)
    rows = (ctypes.c_int64 * n)(*[r for r, _ in mats])
    cols = (ctypes.c_int64 * n)(*[c for _, c in mats])
    owner = (ctypes.c_int32 * n)()
    offs = (ctypes.c_uint64 * n)()
    extent = ctypes.c_uint64()
    _native.check(_native.lib().tk_muon_layout(n, rows, cols, world, owner, offs,
                                               ctypes.byref(extent)))
    want_owner = lpt_assign([ns_dense_flops(r, c) for r, c in mats], world)
    want_offs, want_extent = owner_major_layout([r * c for r, c in mats], want_owner, world)
    assert list(owner) == want_owner
    assert list(offs) == want_offs
    assert extent.value == want_extent


def _dying_worker(rank, world, port, result_q):
    """Rank 1 leaves before the step's first collective; rank 0 runs the step's
    choreography (f64 norm all-reduce, then the parameter all-gather) and must
    get an error from its process group's timeout instead of hanging."""
    import time
    from datetime import timedelta

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=3))
    if rank == 1:
        result_q.put((rank, "left"))
        result_q.close()
        result_q.join_thread()  # the message is out before the process goes
        os._exit(0)  # no collective, no destroy: the rank is simply gone
    t0 = time.monotonic()
    try:
        sumsq = torch.ones(1, dtype=torch.float64)
        dist.all_reduce(sumsq)
        parts = [torch.empty(4) for _ in range(world)]
        dist.all_gather(parts, torch.ones(4))
        result_q.put((rank, "completed"))
    except Exception as e:  # the gloo backend raises on timeout or a lost peer
        result_q.put((rank, f"error after {time.monotonic() - t0:.1f}s: {type(e).__name__}"))


def test_rank_leaving_before_the_exchange_errors_instead_of_hanging():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dying_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert res[1] == "left"
    assert res[0].startswith("error after"), res[0]
    assert float(res[0].split()[2].rstrip("s:")) < 60


def _heartbeat_worker(rank, world, port, result_q):
    """Three host-side steps with a Liveness check before each; rank 1 leaves
    after step 1 (between steps, nothing in flight)."""
    from datetime import timedelta

    from tikun_b200.distributed import Liveness, RankLost

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=30))
    live = Liveness(timeout=2.0)
    out = []
    try:
        for k in (1, 2, 3):
            live.step(k)
            out.append(k)
            if rank == 1 and k == 1:
                result_q.put((rank, out))
                result_q.close()
                result_q.join_thread()
                os._exit(0)
        result_q.put((rank, out))
    except RankLost as e:
        result_q.put((rank, out + [str(e)]))


def test_liveness_reports_a_rank_that_left_between_steps():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_heartbeat_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert res[1] == [1]
    assert res[0][:1] == [1] and "rank(s) [1] did not reach step 2" in res[0][1], res[0]


def test_muon_shard_checks_gradients_before_announcing_the_step():
    # world 1 without a process group: the shard's host side runs on the CPU
    # and every check fires before the (CUDA) step would be enqueued
    from tikun_b200.distributed import MuonShard

    class Beats:
        def __init__(self):
            self.steps = []

        def step(self, k):
            self.steps.append(k)

    sh = MuonShard([(8, 16), (16, 8)], torch.float32, "cpu", lr=0.02)
    sh.liveness = Beats()
    good = [torch.zeros(8, 16), torch.zeros(16, 8)]
    bad_dtype = [torch.zeros(8, 16, dtype=torch.float16), good[1]]
    bad_shape = [torch.zeros(8, 15), good[1]]
    strided = [torch.zeros(16, 8).t(), good[1]]
    for grads, text in ((bad_dtype, "float32 or bfloat16"), (bad_shape, "contiguous 8x16"),
                        (strided, "contiguous 8x16")):
        with pytest.raises(ValueError, match=text):
            sh.step(grads)
        with pytest.raises(ValueError, match=text):
            sh.step_part([0, 1], grads)
    assert sh.step_count == 0 and sh.liveness.steps == []
    assert sh._leaves(sh.mine, good)[0].rows == 8
