"""Multi-GPU ZeRO-1 step against the single-GPU step (needs 2 GPUs; skipped
otherwise).  Two NCCL ranks run 3 optimizer steps on the scaled-down GPT-2
leaf table through

* ZeroPointwise (torch.distributed; chunk-major ownership, f64 norm
  all-reduce, then either overlapped all-gathers or the fused update that
  stores into the peer's arena over NVLink), and
* ShardedStep (the C ABI's tk_shard_*, on PyTorch's communicator or on one
  made by tk_nccl_comm_init), with each exchange (peer stores, copy-engine
  copies, all-gather), for AdamW, Lion and SGD,
* tk_step_buffers_sharded with whole leaves dealt round-robin to the ranks,
  from pinned host buffers, and with every leaf on rank 0 (rank 1 only joins
  the norm all-reduce),

clipped and unclipped; rank 0 runs the same steps through tk_step_buffers on
one GPU.  Parameters must agree within the pointwise bar (1e-6 relative; the
f64 sum order of the norm differs between the two) on both ranks, and the
returned clip scale likewise."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank(rank, world, port, q, cfg):
    import sys
    from datetime import timedelta

    repo = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, repo)
    sys.path.insert(0, os.path.join(repo, "tests"))
    import torch.distributed as dist

    from helpers import gpt2_small_sizes
    from tikun_b200 import _native
    from tikun_b200.arena import Arena, LayoutPlan

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=timedelta(seconds=60))
    try:
        kind, max_norm = cfg["kind"], cfg["max_norm"]
        sizes = gpt2_small_sizes(d=128, vocab=1000, ctx=256)
        plan = LayoutPlan(sizes, pad_to=16 * world * 4)
        gen = torch.Generator(device="cpu").manual_seed(5)
        p0 = torch.randn(plan.total, generator=gen) * 0.02
        grads = [torch.randn(plan.total, generator=gen) * 1e-2 for _ in range(3)]
        P, G = Arena(plan, device=dev), Arena(plan, device=dev)
        P.flat.copy_(p0)
        if cfg["api"].startswith("sharded"):
            out = _run_sharded(cfg, rank, world, dev, plan, sizes, grads, P, G)
        else:
            out = _run_zero(cfg, rank, world, plan, grads, P, G)
        if rank == 0:
            # single-GPU reference through the C ABI
            P1, G1, M1, V1 = (Arena(plan, device=dev) for _ in range(4))
            P1.flat.copy_(p0)
            ref_scales = []
            for s in range(3):
                G1.flat.copy_(grads[s])
                ref_scales.append(_native.step_fast_buffers(
                    P1.ptrs(), G1.ptrs(), M1.ptrs(), V1.ptrs() if kind == "adamw" else [],
                    sizes, max_norm, kind, s + 1, 1e-3, 0.9, 0.999, 1e-8, 0.01))
            out["single"] = P1.flat.cpu().numpy()
            out["ref_scales"] = ref_scales
            out["slots"] = plan.slots
        q.put((rank, out))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def _run_zero(cfg, rank, world, plan, grads, P, G):
    """ZeroPointwise or ShardedStep over replicated arenas."""
    import ctypes

    import torch.distributed as dist

    from tikun_b200 import _native
    from tikun_b200.distributed import ShardedStep, ZeroHParams, ZeroPointwise

    hp = ZeroHParams(max_norm=cfg["max_norm"], kind=cfg["kind"])
    own_comm = None
    if cfg["api"] == "zero":
        zp = ZeroPointwise(plan, P.flat, G.flat, hp, chunks=4, fused=cfg["exchange"] == "peers")
    else:
        if cfg["api"] == "shard-own-comm":
            # a communicator made through the C ABI, not PyTorch's
            idb = ctypes.create_string_buffer(128)
            if rank == 0:
                _native.check(_native.lib().tk_nccl_unique_id(idb))
            obj = [bytes(idb.raw)]
            dist.broadcast_object_list(obj, src=0)
            c = ctypes.c_void_p()
            _native.check(_native.lib().tk_nccl_comm_init(obj[0], world, rank, ctypes.byref(c)))
            own_comm = c.value
        zp = ShardedStep(plan, P.flat, G.flat, hp, exchange=cfg["exchange"], comm=own_comm)
    scales = []
    for s in range(3):
        G.flat.copy_(grads[s])
        if cfg["api"] == "zero":
            zp.step()
        else:
            scales.append(zp.step(return_scale=True))
    torch.cuda.synchronize()
    out = {"zero": P.flat.cpu().numpy(), "scales": scales}
    zp.close()
    if own_comm:
        _native.check(_native.lib().tk_nccl_comm_destroy(ctypes.c_void_p(own_comm)))
    return out


def _run_sharded(cfg, rank, world, dev, plan, sizes, grads, P, G):
    """tk_step_buffers_sharded: each rank steps its own leaves (pinned host
    buffers dealt round-robin, or every leaf on rank 0 in device memory); the
    results are summed across ranks (each element is non-zero on one rank)."""
    import ctypes

    import torch.distributed as dist

    from tikun_b200 import _native
    from tikun_b200.arena import Arena
    from tikun_b200.distributed import nccl_comm_ptr

    comm = nccl_comm_ptr(None, dev)
    host = cfg["api"] == "sharded-host"
    if host:
        mine = [i for i in range(len(sizes)) if i % world == rank]
        hp_ = [P.leaf(i).cpu().pin_memory() for i in mine]
        hg_ = [[grads[k][o:o + n].clone().pin_memory() for k in range(3)]
               for o, n in (plan.slots[i] for i in mine)]
        hm_ = [torch.zeros(sizes[i]).pin_memory() for i in mine]
        hv_ = [torch.zeros(sizes[i]).pin_memory() for i in mine]
    else:
        mine = list(range(len(sizes))) if rank == 0 else []
        M, V = Arena(plan, device=dev), Arena(plan, device=dev)
    hpar = _native.TkHParams(1e-3, 0.9, 0.999, 1e-8, 0.01)
    kind = _native.opt_kind(cfg["kind"])
    scales = []
    for s in range(3):
        if host:
            leaves, nl = _native.make_leaves(
                [t.data_ptr() for t in hp_], [g[s].data_ptr() for g in hg_],
                [t.data_ptr() for t in hm_],
                [t.data_ptr() for t in hv_] if cfg["kind"] == "adamw" else [],
                [sizes[i] for i in mine])
        else:
            G.flat.copy_(grads[s])
            leaves, nl = _native.make_leaves(
                [P.ptrs()[i] for i in mine], [G.ptrs()[i] for i in mine],
                [M.ptrs()[i] for i in mine],
                [V.ptrs()[i] for i in mine] if cfg["kind"] == "adamw" else [],
                [sizes[i] for i in mine])
        sc = ctypes.c_float()
        _native.check(_native.lib().tk_step_buffers_sharded(
            leaves, nl, kind, ctypes.byref(hpar), s + 1, cfg["max_norm"], ctypes.byref(sc),
            comm, torch.cuda.current_stream().cuda_stream))
        scales.append(sc.value)
    if host:
        for j, i in enumerate(mine):
            P.leaf(i).copy_(hp_[j])
    mask = torch.zeros(plan.total, dtype=torch.float32, device=dev)
    for i in mine:
        o, n = plan.slots[i]
        mask[o:o + n] = 1
    full = P.flat * mask
    dist.all_reduce(full)
    torch.cuda.synchronize()
    return {"zero": full.cpu().numpy(), "scales": scales}


CASES = [
    dict(api="zero", exchange="allgather", kind="adamw", max_norm=1.0),
    dict(api="zero", exchange="peers", kind="adamw", max_norm=1.0),
    dict(api="zero", exchange="peers", kind="adamw", max_norm=0.0),
    dict(api="shard", exchange="peers", kind="adamw", max_norm=1.0),
    dict(api="shard", exchange="allgather", kind="adamw", max_norm=1.0),
    dict(api="shard", exchange="copy", kind="adamw", max_norm=1.0),
    dict(api="shard", exchange="copy", kind="sgd", max_norm=0.0),
    dict(api="shard", exchange="peers", kind="lion", max_norm=0.0),
    dict(api="shard", exchange="allgather", kind="sgd", max_norm=1.0),
    dict(api="shard-own-comm", exchange="peers", kind="adamw", max_norm=1.0),
    dict(api="sharded-host", exchange="none", kind="adamw", max_norm=1.0),
    dict(api="sharded-host", exchange="none", kind="lion", max_norm=0.0),
    dict(api="sharded-device", exchange="none", kind="adamw", max_norm=1.0),
]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("cfg", CASES, ids=lambda c: "-".join(str(v) for v in c.values()))
def test_zero1_two_gpus_matches_single_gpu(cfg):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q, cfg)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in range(2))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    single = res[0]["single"]
    for r in (0, 1):
        z = res[r]["zero"]
        for off, n in res[0]["slots"]:
            a, b = z[off:off + n].astype(np.float64), single[off:off + n].astype(np.float64)
            rel = np.abs(a - b) / np.maximum(np.abs(b), 1e-30)
            assert rel.max() <= 1e-6, (r, off, rel.max())
        for got, want in zip(res[r]["scales"], res[0]["ref_scales"]):
            assert abs(got - want) <= 1e-6 * abs(want), (got, want)
    if cfg["max_norm"] > 0:
        assert res[0]["ref_scales"][0] < 1.0  # the clip engaged


# the last two have 1024 and more rows after the transpose of a tall matrix,
# so they run on the CTA-pair GEMM kernel
MUON_SHAPES = [(256, 512), (512, 256), (384, 384), (128, 1024), (640, 320), (256, 512),
               (96, 200), (1024, 256), (1024, 1536), (2048, 1024)]


def _muon_rank(rank, world, port, q, exchange, dtype_name):
    import sys
    from datetime import timedelta

    repo = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, repo)
    import torch.distributed as dist

    from tikun_b200 import _native
    from tikun_b200.distributed import MuonShard

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    if exchange == "copy-engine":
        os.environ["TIKUN_MUON_COPY_ENGINE"] = "1"
        exchange = "copy"
    parts = exchange.endswith("-parts")
    exchange = exchange.replace("-parts", "")
    native = exchange.startswith("native-")
    exchange = exchange.replace("native-", "")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=timedelta(seconds=60))
    try:
        dtype = getattr(torch, dtype_name)
        gen = torch.Generator(device="cpu").manual_seed(11)
        p0 = [torch.randn(r, c, generator=gen) * 0.02 for r, c in MUON_SHAPES]
        grads = [[(torch.randn(r, c, generator=gen) * 1e-3) for r, c in MUON_SHAPES]
                 for _ in range(3)]
        if native:
            from tikun_b200.distributed import NativeMuonShard

            ms = NativeMuonShard(MUON_SHAPES, dtype, dev, lr=0.02, exchange=exchange)
        else:
            ms = MuonShard(MUON_SHAPES, dtype, dev, lr=0.02, exchange=exchange)
        for i in range(len(MUON_SHAPES)):
            ms.param(i).copy_(p0[i])
        for s in range(3):
            gs = {i: grads[s][i].to(dev, dtype).contiguous() for i in ms.mine}
            if parts:  # in two calls, second half first (as backward would)
                half = len(MUON_SHAPES) // 2
                ms.step_begin()
                ms.step_part(range(half, len(MUON_SHAPES)), gs)
                ms.step_part(range(half), gs)
                ms.step_end()
            else:
                ms.step(gs)
        torch.cuda.synchronize()
        out = {"shard": [ms.param(i).float().cpu().numpy() for i in range(len(MUON_SHAPES))],
               "mine": ms.mine}
        ms.close()
        if rank == 0:
            # every matrix on this GPU through tk_muon_step
            ps = [p0[i].to(dev, dtype).contiguous() for i in range(len(MUON_SHAPES))]
            moms = [torch.zeros(r * c, device=dev) for r, c in MUON_SHAPES]
            dt = _native.TK_F32 if dtype == torch.float32 else _native.TK_BF16
            for s in range(3):
                gs = [grads[s][i].to(dev, dtype).contiguous() for i in range(len(MUON_SHAPES))]
                _native.muon_step([(ps[i].data_ptr(), gs[i].data_ptr(), moms[i].data_ptr(), 1,
                                    r, c, dt, dt) for i, (r, c) in enumerate(MUON_SHAPES)],
                                  lr=0.02, momentum=0.95)
            torch.cuda.synchronize()
            out["single"] = [p.float().cpu().numpy() for p in ps]
        q.put((rank, out))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("exchange,dtype_name", [("peers", "bfloat16"), ("peers", "float32"),
                                                 ("copy", "bfloat16"), ("copy", "float32"),
                                                 ("copy-engine", "bfloat16"),
                                                 ("allgather", "bfloat16"),
                                                 ("copy-parts", "bfloat16"),
                                                 ("peers-parts", "float32"),
                                                 ("allgather-parts", "bfloat16"),
                                                 ("native-copy", "bfloat16"),
                                                 ("native-peers", "float32"),
                                                 ("native-allgather", "bfloat16")])
def test_muon_shard_two_gpus_matches_single_gpu(exchange, dtype_name):
    """MuonShard (LPT-assigned matrices; peer stores from the final
    Newton-Schulz epilogue, a copy kernel or the copy engines beside the next
    batch, or an all-gather; in one call or in parts as in backward; through
    the Python class or the C ABI's tk_muon_shard_*) equals tk_muon_step of every
    matrix on one GPU bit for bit, on both ranks: each matrix's arithmetic is
    independent of which batch or GPU it runs in."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_muon_rank, args=(r, 2, port, q, exchange, dtype_name))
             for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in range(2))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert res[0]["mine"] and res[1]["mine"]  # both ranks own matrices
    for r in (0, 1):
        for i, (a, b) in enumerate(zip(res[r]["shard"], res[0]["single"])):
            np.testing.assert_array_equal(a, b, err_msg=f"rank {r} matrix {i}")
