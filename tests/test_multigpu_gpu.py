"""Multi-GPU ZeRO-1 step against the single-GPU step (needs 2 GPUs; skipped
otherwise).  Two NCCL ranks run ZeroPointwise (chunk-major ownership, f64
norm all-reduce, then either overlapped all-gathers or the fused update that
stores into the peer's arena over NVLink) for 3 AdamW steps on the
scaled-down GPT-2 leaf table, clipped and unclipped; rank 0 runs the same
steps through tk_step_buffers on one GPU.  Parameters must agree within the
pointwise bar (1e-6 relative; the f64 sum order of the norm differs between
the two) on both ranks."""
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


def _rank(rank, world, port, q, fused, max_norm):
    import sys
    from datetime import timedelta

    repo = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, repo)
    sys.path.insert(0, os.path.join(repo, "tests"))
    import torch.distributed as dist

    from helpers import gpt2_small_sizes
    from tikun_b200 import _native
    from tikun_b200.arena import Arena, LayoutPlan
    from tikun_b200.distributed import ZeroHParams, ZeroPointwise

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=timedelta(seconds=60))
    try:
        sizes = gpt2_small_sizes(d=128, vocab=1000, ctx=256)
        plan = LayoutPlan(sizes, pad_to=16 * world * 4)
        gen = torch.Generator(device="cpu").manual_seed(5)
        p0 = torch.randn(plan.total, generator=gen) * 0.02
        grads = [torch.randn(plan.total, generator=gen) * 1e-2 for _ in range(3)]
        P, G = Arena(plan, device=dev), Arena(plan, device=dev)
        P.flat.copy_(p0)
        zp = ZeroPointwise(plan, P.flat, G.flat, ZeroHParams(max_norm=max_norm), chunks=4,
                           fused=fused)
        for s in range(3):
            G.flat.copy_(grads[s])
            zp.step()
        torch.cuda.synchronize()
        out = {"zero": P.flat.cpu().numpy()}
        zp.close()
        if rank == 0:
            # single-GPU reference through the C ABI
            P1, G1, M1, V1 = (Arena(plan, device=dev) for _ in range(4))
            P1.flat.copy_(p0)
            for s in range(3):
                G1.flat.copy_(grads[s])
                _native.step_fast_buffers(P1.ptrs(), G1.ptrs(), M1.ptrs(), V1.ptrs(), sizes, max_norm,
                                          "adamw", s + 1, 1e-3, 0.9, 0.999, 1e-8, 0.01)
            out["single"] = P1.flat.cpu().numpy()
            out["slots"] = plan.slots
        q.put((rank, out))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("fused,max_norm", [(False, 1.0), (True, 1.0), (True, 0.0)])
def test_zero1_two_gpus_matches_single_gpu(fused, max_norm):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q, fused, max_norm)) for r in range(2)]
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
