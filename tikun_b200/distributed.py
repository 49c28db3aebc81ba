"""ZeRO-1 pointwise optimizer step across ranks (one process per GPU).

Ownership is chunk-major: the flat parameter arena is cut into ``chunks``
super-chunks and every super-chunk is split evenly across the ranks, so rank r
owns one contiguous piece of each.  A step is

1. Tier 1 on the rank's pieces (f64 partial sum of g^2), one all-reduce of that
   double, the clip scale (crates/tikun-cpu/src/lib.rs:79-125);
2. per super-chunk: Tier 2 on the rank's piece, then an in-place all-gather of
   that super-chunk, issued right away so it overlaps the next piece's update.

With ``fused=True`` there is no all-gather: every rank maps the other ranks'
parameter arenas into its address space (CUDA IPC) and the update kernel
stores each new parameter into the local arena and into every peer's copy
over NVLink as it produces it (tk_apply_pointwise_peers), so the exchange
overlaps the arithmetic.  One 8-byte all-reduce on the same stream after the
update is the end-of-step barrier: no rank reads its arena before every peer
has finished writing into it.

Optimizer state (m, v) exists only for the rank's pieces.  Results are
identical to the single-GPU step: the update is element-wise and the clip
scale comes from the same global sum (up to f64 summation order).
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch
import torch.distributed as dist

from . import _native
from .arena import LayoutPlan


def chunk_major_pieces(total: int, world: int, rank: int, chunks: int,
                       align: int = 16) -> list[tuple[int, int]]:
    """[lo, hi) ranges of the flat arena owned by ``rank``: one per
    super-chunk.  ``total`` must be a multiple of chunks * world * align."""
    if total % (chunks * world * align) != 0:
        raise ValueError(f"arena of {total} elements does not split into {chunks} chunks x "
                         f"{world} ranks x {align}-element granules")
    sup = total // chunks
    per = sup // world
    return [(c * sup + rank * per, c * sup + (rank + 1) * per) for c in range(chunks)]


def pieces_to_segments(plan: LayoutPlan, lo: int, hi: int) -> list[tuple[int, int, int]]:
    """(leaf, start within leaf, count) of the leaf elements inside [lo, hi)."""
    out = []
    for i, (off, n) in enumerate(plan.slots):
        a, b = max(off, lo), min(off + n, hi)
        if a < b:
            out.append((i, a - off, b - a))
    return out


def _close_mappings(ptrs: list[int]) -> None:
    """Unmaps what a failed set-up had already mapped (best effort: the
    set-up's own error is the one raised)."""
    L = _native.lib()
    for p in ptrs:
        L.tk_ipc_close(ctypes.c_void_p(p))
    ptrs.clear()


@dataclass
class ZeroHParams:
    lr: float = 1e-3
    beta1: float = 0.9
    beta2: float = 0.999
    eps: float = 1e-8
    weight_decay: float = 0.01
    max_norm: float = 0.0
    kind: str = "adamw"


class ZeroPointwise:
    """ZeRO-1 AdamW/Lion/SGD over f32 parameter and gradient arenas (flat
    tensors laid out by ``plan``, replicated on every rank)."""

    def __init__(self, plan: LayoutPlan, p_flat: torch.Tensor, g_flat: torch.Tensor,
                 hp: ZeroHParams, group=None, chunks: int = 4, fused: bool = False):
        self.plan, self.p, self.g, self.hp, self.group = plan, p_flat, g_flat, hp, group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.chunks = chunks
        self.pieces = chunk_major_pieces(plan.total, self.world, self.rank, chunks)
        self.kind = _native.opt_kind(hp.kind)
        owned = sum(hi - lo for lo, hi in self.pieces)
        dev = p_flat.device
        self.m = torch.zeros(owned, dtype=torch.float32, device=dev)
        self.v = torch.zeros(owned, dtype=torch.float32, device=dev)
        self.sumsq = torch.zeros(1, dtype=torch.float64, device=dev)
        self.scale = torch.ones(1, dtype=torch.float32, device=dev)
        self.step_count = 0
        # one leaf table per piece (C ABI leaves), plus one over all pieces for Tier 1
        self.tables = []
        base_p, base_g = p_flat.data_ptr(), g_flat.data_ptr()
        base_m, base_v = self.m.data_ptr(), self.v.data_ptr()
        state_off = 0
        all_segs = []
        for lo, hi in self.pieces:
            segs = pieces_to_segments(plan, lo, hi)
            flat = [plan.slots[i][0] + a for i, a, c in segs]
            local = [state_off + (f - lo) for f in flat]
            leaves = _native.make_leaves([base_p + 4 * f for f in flat], [base_g + 4 * f for f in flat],
                                         [base_m + 4 * x for x in local], [base_v + 4 * x for x in local],
                                         [c for _, _, c in segs])
            self.tables.append(leaves)
            all_segs.extend(zip(flat, local, [c for _, _, c in segs]))
            state_off += hi - lo
        self.all_leaves = _native.make_leaves([base_p + 4 * f for f, _, _ in all_segs],
                                              [base_g + 4 * f for f, _, _ in all_segs],
                                              [base_m + 4 * x for _, x, _ in all_segs],
                                              [base_v + 4 * x for _, x, _ in all_segs],
                                              [c for _, _, c in all_segs])
        self.launches_per_step = 0
        self.fused = fused and self.world > 1
        self.peer_ptrs: list[int] = []
        if self.fused:
            self._map_peers()

    def _map_peers(self) -> None:
        """Exchange IPC handles of every rank's parameter arena and map the
        peers' arenas; peer_deltas[i] = peer address - local address."""
        if self.p.dtype != torch.float32 or not self.p.is_contiguous():
            raise ValueError("fused ZeRO-1 needs a contiguous f32 parameter arena")
        L = _native.lib()
        handle = ctypes.create_string_buffer(64)
        off = ctypes.c_uint64(0)
        _native.check(L.tk_ipc_export(self.p.data_ptr(), handle, ctypes.byref(off)))
        mine = (bytes(handle.raw), int(off.value), self.plan.total)
        everyone = [None] * self.world
        dist.all_gather_object(everyone, mine, group=self.group)
        deltas = []
        try:
            for r, (h, o, total) in enumerate(everyone):
                if total != self.plan.total:
                    raise ValueError(f"rank {r} has an arena of {total} elements, "
                                     f"this rank {self.plan.total}")
                if r == self.rank:
                    continue
                ptr = ctypes.c_void_p()
                _native.check(L.tk_ipc_import(h, o, ctypes.byref(ptr)))
                self.peer_ptrs.append(ptr.value)
                deltas.append(ptr.value - self.p.data_ptr())
        except Exception:
            _close_mappings(self.peer_ptrs)
            raise
        self.peer_deltas = (ctypes.c_int64 * max(len(deltas), 1))(*deltas)
        self.barrier_buf = torch.zeros(1, dtype=torch.float64, device=self.p.device)

    def close(self) -> None:
        """Unmaps the peers' arenas (fused mode); call on every rank, before
        the process group is destroyed."""
        if self.peer_ptrs:
            torch.cuda.synchronize(self.p.device)
            if dist.is_initialized():
                dist.barrier(group=self.group)
            L = _native.lib()
            for p in self.peer_ptrs:
                _native.check(L.tk_ipc_close(ctypes.c_void_p(p)))
            self.peer_ptrs = []

    def step(self, update_events=None) -> None:
        """One optimizer step on the current stream; returns once everything
        (the all-gathers included) is enqueued on it."""
        self.step_count += 1
        L = _native.lib()
        s = torch.cuda.current_stream(self.p.device).cuda_stream
        hp = _native.TkHParams(self.hp.lr, self.hp.beta1, self.hp.beta2, self.hp.eps,
                               self.hp.weight_decay)
        launches = 0
        clip = self.hp.max_norm > 0
        if clip:
            _native.check(L.tk_grad_sumsq(self.all_leaves[0], self.all_leaves[1],
                                          self.sumsq.data_ptr(), s))
            if self.world > 1:
                dist.all_reduce(self.sumsq, group=self.group)
            _native.check(L.tk_clip_scale(self.sumsq.data_ptr(), self.hp.max_norm,
                                          self.scale.data_ptr(), s))
            launches += 3
        if self.fused:
            if not clip:
                # the norm all-reduce is not there to order this update after
                # every peer's reads of its arena from the previous step
                dist.all_reduce(self.barrier_buf, group=self.group)
            if update_events is not None:
                update_events[0].record()
            leaves, n = self.all_leaves
            _native.check(L.tk_apply_pointwise_peers(leaves, n, self.kind, ctypes.byref(hp),
                                                     self.step_count,
                                                     self.scale.data_ptr() if clip else None,
                                                     self.peer_deltas, len(self.peer_ptrs), s))
            if update_events is not None:
                update_events[1].record()
            # every peer has written into this arena once this completes
            dist.all_reduce(self.barrier_buf, group=self.group)
            self.launches_per_step = launches + 1
            return
        works = []
        sup = self.plan.total // self.chunks
        for c, (leaves, n) in enumerate(self.tables):
            if update_events is not None and c == 0:
                update_events[0].record()
            _native.check(L.tk_apply_pointwise(leaves, n, self.kind, ctypes.byref(hp),
                                               self.step_count,
                                               self.scale.data_ptr() if clip else None, s))
            launches += 1
            if update_events is not None and c == len(self.tables) - 1:
                update_events[1].record()
            if self.world > 1:
                lo, hi = self.pieces[c]
                works.append(dist.all_gather_into_tensor(self.p[c * sup:(c + 1) * sup],
                                                         self.p[lo:hi], group=self.group,
                                                         async_op=True))
        for w in works:
            w.wait()
        self.launches_per_step = launches


class RankLost(RuntimeError):
    """A rank stopped announcing steps: raised on the host before the next
    launch, so no collective is left waiting for it on the GPU."""


class Liveness:
    """Host-side heartbeat over the process group's key-value store.  Every
    rank announces step k (``beat``) and, before launching step k's kernels and
    collectives, waits at most ``timeout`` seconds for every other rank's
    announcement (``check``); a rank that left between steps is reported as
    RankLost instead of a hang inside a collective."""

    def __init__(self, store=None, rank: int | None = None, world: int | None = None,
                 timeout: float = 10.0, prefix: str = "tikun/alive"):
        from datetime import timedelta

        self.store = store or dist.distributed_c10d._get_default_store()
        self.rank = dist.get_rank() if rank is None else rank
        self.world = dist.get_world_size() if world is None else world
        self.timeout = timedelta(seconds=timeout)
        self.prefix = prefix

    def _key(self, rank: int, step: int) -> str:
        return f"{self.prefix}/{step}/{rank}"

    def beat(self, step: int) -> None:
        self.store.set(self._key(self.rank, step), "1")

    def check(self, step: int) -> None:
        keys = [self._key(r, step) for r in range(self.world)]
        try:
            self.store.wait(keys, self.timeout)
        except Exception as e:  # the store raises on timeout
            missing = [r for r in range(self.world) if not self.store.check([self._key(r, step)])]
            raise RankLost(f"rank(s) {missing} did not reach step {step} within "
                           f"{self.timeout.total_seconds():.0f} s") from e

    def step(self, step: int) -> None:
        """beat + check."""
        self.beat(step)
        self.check(step)


def nccl_comm_ptr(group=None, device=None) -> int:
    """The ncclComm_t behind a PyTorch NCCL process group (created by a tiny
    all-reduce if the group was initialised lazily)."""
    group = group or dist.distributed_c10d._get_default_group()
    device = device or torch.device("cuda", torch.cuda.current_device())
    backend = group._get_backend(device)
    try:
        ptr = backend._comm_ptr()
    except RuntimeError:
        ptr = 0
    if not ptr:
        dist.all_reduce(torch.zeros(1, device=device), group=group)
        torch.cuda.synchronize(device)
        ptr = backend._comm_ptr()
    return int(ptr)


def wait_step(stream, deadline_s: float, own_comm: int | None = None) -> None:
    """Waits on the host for the work enqueued on ``stream`` at most
    ``deadline_s`` seconds (tk_stream_wait_deadline).  On a communicator error
    or at the deadline it raises TikunError; with ``own_comm`` (a communicator
    from tk_nccl_comm_init, never PyTorch's, which PyTorch's watchdog aborts)
    that communicator is aborted first, which ends collectives waiting for a
    rank that is gone.  Results of that step are not valid."""
    _native.check(_native.lib().tk_stream_wait_deadline(
        ctypes.c_void_p(stream.cuda_stream), int(deadline_s * 1000),
        ctypes.c_void_p(own_comm) if own_comm else None))


class ShardedStep:
    """ZeRO-1 clipped AdamW/Lion/SGD through the C ABI (tk_shard_*): the
    native multi-GPU step over a flat f32 parameter/gradient arena laid out by
    ``plan`` and replicated on every rank.  ``exchange`` is "peers" (the
    update kernel stores into every rank's arena over NVLink), "copy" (the
    copy engines copy each updated chunk into every rank's arena) or
    "allgather" (an in-place ncclAllGather after the update).  ``comm`` is an ncclComm_t
    to use instead of the process group's (e.g. from tk_nccl_comm_init).  With
    ``deadline_s`` set, every step waits for its work at most that long
    (``wait_step``), aborting ``comm`` when one was given."""

    def __init__(self, plan: LayoutPlan, p_flat: torch.Tensor, g_flat: torch.Tensor,
                 hp: ZeroHParams, group=None, exchange: str = "peers", comm: int | None = None):
        for t in (p_flat, g_flat):
            if t.dtype != torch.float32 or not t.is_contiguous() or t.numel() != plan.total:
                raise ValueError("ShardedStep needs contiguous f32 arenas of plan.total elements")
        self.plan, self.p, self.g, self.hp = plan, p_flat, g_flat, hp
        self.step_count = 0
        self.kind = _native.opt_kind(hp.kind)
        mode = {"allgather": 0, "peers": 1, "copy": 2}[exchange]
        L = _native.lib()
        offs = (ctypes.c_uint64 * len(plan))(*[o for o, _ in plan.slots])
        lens = (ctypes.c_uint64 * len(plan))(*[n for _, n in plan.slots])
        self.own_comm = comm
        self.deadline_s: float | None = None
        comm = comm or nccl_comm_ptr(group, p_flat.device)
        handle = ctypes.c_void_p()
        s = torch.cuda.current_stream(p_flat.device).cuda_stream
        _native.check(L.tk_shard_init(comm, p_flat.data_ptr(), g_flat.data_ptr(), plan.total,
                                      offs, lens, len(plan), self.kind, mode, s,
                                      ctypes.byref(handle)))
        self.handle = handle
        lo, hi = ctypes.c_uint64(), ctypes.c_uint64()
        _native.check(L.tk_shard_info(handle, ctypes.byref(lo), ctypes.byref(hi), None, None))
        self.lo, self.hi = lo.value, hi.value
        self.hparams = _native.TkHParams(hp.lr, hp.beta1, hp.beta2, hp.eps, hp.weight_decay)
        self.liveness: Liveness | None = None

    def step(self, return_scale: bool = False) -> float | None:
        """One step on the current stream; with ``return_scale`` waits for it
        and returns the clip scale (step_fast_buffers' return value).  With a
        Liveness (``self.liveness``), a rank that left is reported before any
        launch."""
        self.step_count += 1
        if self.liveness is not None:
            self.liveness.step(self.step_count)
        L = _native.lib()
        st = torch.cuda.current_stream(self.p.device)
        out = ctypes.c_float(1.0)
        _native.check(L.tk_shard_step(self.handle, ctypes.byref(self.hparams), self.step_count,
                                      self.hp.max_norm, ctypes.byref(out) if return_scale else None,
                                      st.cuda_stream))
        if self.deadline_s is not None:
            wait_step(st, self.deadline_s, self.own_comm)
        return out.value if return_scale else None

    def close(self) -> None:
        """Collective: every rank calls it before the process group goes."""
        if self.handle:
            s = torch.cuda.current_stream(self.p.device).cuda_stream
            _native.check(_native.lib().tk_shard_destroy(self.handle, s))
            self.handle = None


class PeerArena:
    """Every rank's copy of one device tensor (same size and dtype on every
    rank) mapped into this process with CUDA IPC.  ``deltas[i]`` is the byte
    offset from an address in the local tensor to the same element in the
    i-th other rank's copy (the form the peer-store kernels take)."""

    def __init__(self, t: torch.Tensor, group=None):
        self.group = group
        self.ptrs: list[int] = []
        world = dist.get_world_size(group)
        rank = dist.get_rank(group)
        L = _native.lib()
        handle = ctypes.create_string_buffer(64)
        off = ctypes.c_uint64(0)
        _native.check(L.tk_ipc_export(t.data_ptr(), handle, ctypes.byref(off)))
        mine = (bytes(handle.raw), int(off.value), t.numel() * t.element_size())
        everyone = [None] * world
        dist.all_gather_object(everyone, mine, group=group)
        deltas = []
        try:
            for r, (h, o, nbytes) in enumerate(everyone):
                if nbytes != mine[2]:
                    raise ValueError(f"rank {r} shares {nbytes} bytes, this rank {mine[2]}")
                if r == rank:
                    continue
                ptr = ctypes.c_void_p()
                _native.check(L.tk_ipc_import(h, o, ctypes.byref(ptr)))
                self.ptrs.append(ptr.value)
                deltas.append(ptr.value - t.data_ptr())
        except Exception:
            _close_mappings(self.ptrs)
            raise
        self.n = len(deltas)
        self.deltas = (ctypes.c_int64 * max(self.n, 1))(*deltas)

    def close(self) -> None:
        """Collective: waits for this device and every rank, then unmaps."""
        if self.ptrs:
            torch.cuda.synchronize()
            dist.barrier(group=self.group)
            L = _native.lib()
            for p in self.ptrs:
                _native.check(L.tk_ipc_close(ctypes.c_void_p(p)))
            self.ptrs = []


_MUON_DTYPES = {torch.float32: _native.TK_F32, torch.bfloat16: _native.TK_BF16}


def _check_grad(grads, i: int, r: int, c: int) -> torch.Tensor:
    g = grads[i]
    if g.numel() != r * c or not g.is_contiguous():
        raise ValueError(f"gradient {i} must be a contiguous {r}x{c} tensor")
    if g.dtype not in _MUON_DTYPES:
        raise ValueError(f"gradient {i} is {g.dtype}; Muon gradients are float32 or bfloat16")
    return g


class MuonShard:
    """Muon over matrices split across ranks (one process per GPU).

    Whole matrices are owned by one rank each, assigned by LPT bin-packing on
    their Newton-Schulz FLOPs (``sharding.lpt_assign``); the parameters live
    in an owner-major arena replicated on every rank
    (``sharding.owner_major_layout``); momentum exists on the owner only.
    ``step(grads)`` runs momentum, Nesterov, Newton-Schulz and the update for
    the rank's matrices (tk_muon_step, python/tikun/muon_nd.py:94-160 per
    matrix) and exchanges them: with ``exchange="peers"`` the final GEMM's
    epilogue stores each updated matrix into every rank's arena over NVLink
    (tk_muon_step_peers) and one 8-byte all-reduce closes the step; with
    ``"copy"`` the copy engines copy each finished batch of matrices into every
    rank's arena while the next batch computes (tk_muon_step_copy); with
    ``"allgather"`` an all-gather of the owner-major arena follows."""

    def __init__(self, shapes, dtype: torch.dtype, device, lr: float, momentum: float = 0.95,
                 nesterov: bool = True, ns_steps: int = 5, precision: int | None = None,
                 group=None, exchange: str = "peers"):
        from .sharding import lpt_assign, ns_dense_flops, owner_major_layout

        if dtype not in (torch.float32, torch.bfloat16):
            raise ValueError("Muon parameters are f32 or bf16")
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.shapes = [tuple(s) for s in shapes]
        sizes = [r * c for r, c in self.shapes]
        self.owner = lpt_assign([ns_dense_flops(r, c) for r, c in self.shapes], self.world)
        self.offs, self.extent = owner_major_layout(sizes, self.owner, self.world)
        self.dtype, self.device = dtype, torch.device(device)
        self.params = torch.zeros(self.extent * self.world, dtype=dtype, device=self.device)
        self.mine = [i for i in range(len(sizes)) if self.owner[i] == self.rank]
        self.momentum = {i: torch.zeros(sizes[i], dtype=torch.float32, device=self.device)
                         for i in self.mine}
        self.hp = _native.TkMuonHParams(lr, momentum, 1 if nesterov else 0, ns_steps,
                                        _native.DEFAULT_NS_PRECISION if precision is None
                                        else precision)
        self.exchange = exchange if self.world > 1 else "none"
        if self.exchange not in ("peers", "copy", "allgather", "none"):
            raise ValueError(f"unknown exchange {exchange!r}")
        self.peers = (PeerArena(self.params, group) if self.exchange in ("peers", "copy")
                      else None)
        self.barrier_buf = torch.zeros(1, dtype=torch.float64, device=self.device)
        self.liveness: Liveness | None = None  # optional host heartbeat before each step
        self.step_count = 0

    def param(self, i: int) -> torch.Tensor:
        r, c = self.shapes[i]
        return self.params[self.offs[i]:self.offs[i] + r * c].view(r, c)

    def step(self, grads, events=None) -> None:
        """``grads[i]`` (device tensors, any of f32/bf16, contiguous) for the
        rank's own matrices ``self.mine``; others are not read.  Enqueued on
        the current stream.  ``events`` (two CUDA events) are recorded just
        around the Newton-Schulz launches.  The gradients are checked before
        the step is announced, so a bad argument surfaces on the other ranks as
        a missing heartbeat, not as a collective left waiting."""
        arr = self._leaves(self.mine, grads)
        self.step_count += 1
        if self.liveness is not None:
            self.liveness.step(self.step_count)
        L = _native.lib()
        s = torch.cuda.current_stream(self.device).cuda_stream
        if self.exchange in ("peers", "copy"):
            # the peers are done reading this step's destination ranges
            dist.all_reduce(self.barrier_buf, group=self.group)
            if events:
                events[0].record()
            fn = L.tk_muon_step_peers if self.exchange == "peers" else L.tk_muon_step_copy
            _native.check(fn(arr, len(self.mine), ctypes.byref(self.hp), self.peers.deltas,
                             self.peers.n, s))
            if events:
                events[1].record()
            dist.all_reduce(self.barrier_buf, group=self.group)
        else:
            if events:
                events[0].record()
            _native.check(L.tk_muon_step(arr, len(self.mine), ctypes.byref(self.hp), s))
            if events:
                events[1].record()
            if self.exchange == "allgather":
                lo = self.rank * self.extent
                dist.all_gather_into_tensor(self.params, self.params[lo:lo + self.extent],
                                            group=self.group)

    # -- a step issued in parts (e.g. a layer at a time during backward) --
    def _leaves(self, idx, grads):
        pdt = _MUON_DTYPES[self.dtype]
        arr = (_native.TkMuonLeaf * max(len(idx), 1))()
        for k, i in enumerate(idx):
            r, c = self.shapes[i]
            g = _check_grad(grads, i, r, c)
            arr[k] = _native.TkMuonLeaf(self.param(i).data_ptr(), g.data_ptr(),
                                        self.momentum[i].data_ptr(), 1, r, c, pdt,
                                        _MUON_DTYPES[g.dtype])
        return arr

    def step_begin(self, stream=None) -> None:
        """Collective: opens a step issued in parts (step_part)."""
        self.step_count += 1
        if self.liveness is not None:
            self.liveness.step(self.step_count)
        with torch.cuda.stream(stream or torch.cuda.current_stream(self.device)):
            if self.exchange in ("peers", "copy"):
                dist.all_reduce(self.barrier_buf, group=self.group)

    def step_part(self, idx, grads, stream=None) -> None:
        """Steps the rank's own matrices among ``idx`` on ``stream``; with the
        copy exchange their copies into the peers may still run afterwards."""
        mine = [i for i in idx if self.owner[i] == self.rank]
        if not mine:
            return
        arr = self._leaves(mine, grads)
        L = _native.lib()
        s = (stream or torch.cuda.current_stream(self.device)).cuda_stream
        if self.exchange == "peers":
            _native.check(L.tk_muon_step_peers(arr, len(mine), ctypes.byref(self.hp),
                                               self.peers.deltas, self.peers.n, s))
        elif self.exchange == "copy":
            _native.check(L.tk_muon_step_copy_deferred(arr, len(mine), ctypes.byref(self.hp),
                                                       self.peers.deltas, self.peers.n, s))
        else:
            _native.check(L.tk_muon_step(arr, len(mine), ctypes.byref(self.hp), s))

    def step_end(self, stream=None) -> None:
        """Collective: completes the exchange of a step issued in parts."""
        st = stream or torch.cuda.current_stream(self.device)
        with torch.cuda.stream(st):
            if self.exchange == "copy":
                _native.check(_native.lib().tk_muon_copy_join(st.cuda_stream))
            if self.exchange in ("peers", "copy"):
                dist.all_reduce(self.barrier_buf, group=self.group)
            elif self.exchange == "allgather":
                lo = self.rank * self.extent
                dist.all_gather_into_tensor(self.params, self.params[lo:lo + self.extent],
                                            group=self.group)

    def close(self) -> None:
        if self.peers is not None:
            self.peers.close()
            self.peers = None


class NativeMuonShard:
    """MuonShard through the C ABI (tk_muon_shard_*): the LPT assignment, the
    owner-major layout, the momentum, the exchange and its collectives run in
    the library over the process group's NCCL communicator (or ``comm``).
    ``deadline_s`` works as in ShardedStep."""

    def __init__(self, shapes, dtype: torch.dtype, device, lr: float, momentum: float = 0.95,
                 nesterov: bool = True, ns_steps: int = 5, precision: int | None = None,
                 group=None, exchange: str = "copy", comm: int | None = None):
        if dtype not in (torch.float32, torch.bfloat16):
            raise ValueError("Muon parameters are f32 or bf16")
        L = _native.lib()
        self.shapes = [tuple(s) for s in shapes]
        self.device = torch.device(device)
        self.dtype = dtype
        n = len(self.shapes)
        world = dist.get_world_size(group)
        rows = (ctypes.c_int64 * max(n, 1))(*[r for r, _ in self.shapes])
        cols = (ctypes.c_int64 * max(n, 1))(*[c for _, c in self.shapes])
        owner = (ctypes.c_int32 * max(n, 1))()
        offs = (ctypes.c_uint64 * max(n, 1))()
        extent = ctypes.c_uint64()
        _native.check(L.tk_muon_layout(n, rows, cols, world, owner, offs, ctypes.byref(extent)))
        self.owner, self.offs, self.extent = list(owner)[:n], list(offs)[:n], extent.value
        self.rank = dist.get_rank(group)
        self.mine = [i for i in range(n) if self.owner[i] == self.rank]
        self.params = torch.zeros(self.extent * world, dtype=dtype, device=self.device)
        hp = _native.TkMuonHParams(lr, momentum, 1 if nesterov else 0, ns_steps,
                                   _native.DEFAULT_NS_PRECISION if precision is None
                                   else precision)
        mode = {"allgather": 0, "peers": 1, "copy": 2}[exchange]
        self.own_comm = comm
        self.deadline_s: float | None = None
        comm = comm or nccl_comm_ptr(group, self.device)
        handle = ctypes.c_void_p()
        s = torch.cuda.current_stream(self.device).cuda_stream
        pdt = _native.TK_F32 if dtype == torch.float32 else _native.TK_BF16
        _native.check(L.tk_muon_shard_init(comm, n, rows, cols, self.params.data_ptr(), pdt,
                                           ctypes.byref(hp), mode, s, ctypes.byref(handle)))
        self.handle = handle
        self._n = n
        self.liveness: Liveness | None = None  # optional host heartbeat before each step
        self.step_count = 0

    def param(self, i: int) -> torch.Tensor:
        r, c = self.shapes[i]
        return self.params[self.offs[i]:self.offs[i] + r * c].view(r, c)

    def step(self, grads) -> None:
        """``grads[i]``: contiguous device tensors of one dtype (f32 or bf16)
        for the rank's own matrices; enqueued on the current stream.  Checked
        before the step is announced (see MuonShard.step)."""
        ptrs = (ctypes.c_void_p * max(self._n, 1))()
        gdt = None
        for i in self.mine:
            r, c = self.shapes[i]
            g = _check_grad(grads, i, r, c)
            d = _MUON_DTYPES[g.dtype]
            if gdt is not None and d != gdt:
                raise ValueError("all gradients of a step share one dtype")
            gdt = d
            ptrs[i] = g.data_ptr()
        self.step_count += 1
        if self.liveness is not None:
            self.liveness.step(self.step_count)
        st = torch.cuda.current_stream(self.device)
        _native.check(_native.lib().tk_muon_shard_step(
            self.handle, ptrs, _native.TK_F32 if gdt is None else gdt, st.cuda_stream))
        if self.deadline_s is not None:
            wait_step(st, self.deadline_s, self.own_comm)

    def close(self) -> None:
        """Collective: every rank calls it before the process group goes."""
        if self.handle:
            s = torch.cuda.current_stream(self.device).cuda_stream
            _native.check(_native.lib().tk_muon_shard_destroy(self.handle, s))
            self.handle = None
