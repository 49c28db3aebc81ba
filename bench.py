"""Benchmark of the tikun optimizer step on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl tikun|reference]
                    [--workload gpt2-small-clip|flat-100m|muon-gpt2-d768|
                                muon-1.3b-inbackward|muon-llama3-8b]
                    [--zero auto|fused|copy|allgather]

Default workload (the one the headline metric is quoted on at one GPU):
clipped AdamW (global-norm clip 1.0) over the GPT-2-small PyTree, 148 fp32
leaves, 124,439,808 parameters, lr 1e-3, betas (0.9, 0.999), eps 1e-8,
decay 0.01; params N(0, 0.02) with biases 0 and LayerNorm weights 1, grads
N(0, 1e-2) (seeded synthetic data).

One step = one full optimizer step over every leaf.  ``value`` is parameters
updated per second with all buffers resident in HBM (p, g, m, v: 1.99 GB, well
above the 126 MB L2, so no flush is needed between steps), timed with CUDA
events on the launching stream.  At N GPUs the step is ZeRO-1 through the C
ABI (tk_shard_step): each rank updates its 1/N of the flat parameter space
after an f64 norm all-reduce, and the updated fp32 parameters reach the other
ranks by peer stores from the update kernel itself (``--zero fused``, the
default), copies of finished chunks, or an NCCL all-gather; the time is the
max over ranks.  ``e2e`` is the same step through the C ABI with the leaves
in pinned host memory (the reference engine's calling convention), copies
included: tk_step_buffers at one GPU, tk_step_buffers_sharded over each
rank's slice at N.

The Muon workloads (bf16 parameters and gradients, f32 momentum and AdamW
moments; Muon with momentum 0.95, Nesterov, 5 Newton-Schulz steps, lr 0.02 on
every hidden matrix; AdamW as above on embeddings and norms) report params/s
and the Newton-Schulz tensor throughput (dense-equivalent FLOPs
5(4m^2n + 2m^3) per matrix) against the measured bf16 peak.  At N GPUs the
matrices are spread by FLOP-balanced bin-packing (MuonShard) and the AdamW
leaves by ZeRO-1; finished matrices reach the other ranks through a copy
kernel beside the next batch's tensor-core work (``--zero copy``, the default
for Muon), the last GEMM's epilogue (``fused``) or all-gathers.

``--impl reference`` times the reference's CPU algorithm (the oracle's
restatement of tikun-cpu; the Rust engine cannot be built here) on this host's
cores on the same workload: the requested --steps after --warmup, cut only
where they would run past two minutes each; for the Muon workloads one matrix
per shape group is timed and scaled by the group's count.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import sys
import threading
import time

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

METRIC = "optimizer step ms & params/s (AdamW HBM GB/s, Muon NS TFLOP/s) at 1/2/4/8 B200"


def gpt2_small_sizes(d=768, vocab=50257, ctx=1024, layers=12):
    sizes = [vocab * d, ctx * d]
    for _ in range(layers):
        sizes += [d, d, d * 3 * d, 3 * d, d * d, d, d, d, d * 4 * d, 4 * d, 4 * d * d, d]
    return sizes + [d, d]


def gpt2_kinds(layers=12):
    return ["w", "w"] + ["ln", "b", "w", "b", "w", "b", "ln", "b", "w", "b", "w", "b"] * layers + ["ln", "b"]


WORKLOADS = {
    "gpt2-small-clip": dict(sizes=gpt2_small_sizes(), kinds=gpt2_kinds(), max_norm=1.0,
                            g_std=1e-2,
                            desc="clipped AdamW (max_norm 1.0), GPT-2-small PyTree, 148 fp32 "
                                 "leaves, 124,439,808 params"),
    "flat-100m": dict(sizes=[100_000_000], kinds=["w"], max_norm=0.0, g_std=1e-3,
                      desc="AdamW, one flat fp32 buffer of 100,000,000 params, no clip"),
}
HP = dict(lr=1e-3, b1=0.9, b2=0.999, eps=1e-8, decay=0.01)


def load_peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """Polls the GPU's SM clock and clock-event (throttle) reasons through NVML
    every 2 ms while the timed region runs (nvidia-smi's 200 ms loop is too
    coarse for a region of a few milliseconds)."""

    REASONS = (("hw_slowdown", "nvmlClocksEventReasonHwSlowdown"),
               ("hw_thermal_slowdown", "nvmlClocksEventReasonHwThermalSlowdown"),
               ("sw_thermal_slowdown", "nvmlClocksEventReasonSwThermalSlowdown"),
               ("sw_power_cap", "nvmlClocksEventReasonSwPowerCap"))

    def __init__(self, uuid: str, period_s: float = 0.002):
        self.uuid = uuid
        self.period = period_s
        self.samples = []
        self.error = None
        self._stop = threading.Event()
        self._thread = None

    def __enter__(self):
        try:
            import pynvml

            pynvml.nvmlInit()
            u = self.uuid if self.uuid.startswith("GPU-") else "GPU-" + self.uuid
            self._h = pynvml.nvmlDeviceGetHandleByUUID(u)
            self._nv = pynvml
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        except Exception as e:  # no NVML: report unsampled
            self.error = f"{type(e).__name__}: {e}"
        return self

    def _run(self):
        nv = self._nv
        while not self._stop.is_set():
            try:
                sm = nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM)
                reasons = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                self.samples.append((sm, reasons))
            except Exception as e:
                self.error = f"{type(e).__name__}: {e}"
                return
            time.sleep(self.period)

    def __exit__(self, *a):
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=5)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0,
                    "error": self.error}
        nv = self._nv
        reasons = sorted({name for _, r in self.samples for name, attr in self.REASONS
                          if r & getattr(nv, attr)})
        return {"sm_mhz": statistics.median(s for s, _ in self.samples),
                "sm_max_mhz": self.max_mhz, "reasons": reasons, "samples": len(self.samples),
                "source": "nvml"}


# ------------------------------------------------------------------ workload
def cpu_model() -> str:
    """The host CPU's model name (recorded beside every CPU baseline)."""
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    import platform

    return platform.processor() or platform.machine()


def make_host_state(wl, seed=1234):
    """Seeded synthetic leaves: params N(0, 0.02) (biases 0, LayerNorm weights 1),
    grads N(0, g_std)."""
    rng = np.random.default_rng(seed)
    p, g = [], []
    for n, k in zip(wl["sizes"], wl["kinds"]):
        if k == "w":
            p.append((rng.standard_normal(n, dtype=np.float32) * np.float32(0.02)))
        elif k == "ln":
            p.append(np.ones(n, np.float32))
        else:
            p.append(np.zeros(n, np.float32))
        g.append(rng.standard_normal(n, dtype=np.float32) * np.float32(wl["g_std"]))
    return p, g


def pointwise_config(workload, wl):
    """The workload as both arms report it (``config``)."""
    return {"workload": workload, "desc": wl["desc"], "params": sum(wl["sizes"]),
            "leaves": len(wl["sizes"]), "l2": "inputs (p,g,m,v) larger than L2; no flush"}


def muon_config(workload, wl):
    """The Muon workload as both arms report it (``config``)."""
    return {"workload": workload, "desc": wl["desc"],
            "params": sum(r * c for r, c in wl["mats"]) + sum(wl["adamw"]),
            "muon_matrices": len(wl["mats"]), "adamw_leaves": len(wl["adamw"]),
            "l2": "inputs larger than L2; no flush"}


def cpu_reference_run(wl, steps, warmup, nthreads, budget_s=None, chunk=None):
    """The oracle (tikun-cpu's algorithm, restated) on host cores, threads over
    leaves as tikun-cpu's rayon par_iter over leaves.

    Returns (params/s, ms/step, warm-up steps run, steps timed).  With
    ``budget_s`` the warm-up stops and the timed steps are cut once the
    measured step time says they would run past that many seconds each.
    With ``chunk`` every leaf is cut into contiguous pieces of at most that
    many elements, so that all threads share the large leaves: a faster CPU
    schedule than tikun-cpu's, reported beside it and labelled as such."""
    import oracle

    p, g = make_host_state(wl)
    m = [np.zeros_like(x) for x in p]
    v = [np.zeros_like(x) for x in p]
    if chunk:
        def pieces(arrs):
            return [a[i:i + chunk] for a in arrs for i in range(0, a.size, chunk)]
        p, g, m, v = pieces(p), pieces(g), pieces(m), pieces(v)

    def one(s):
        oracle.step_two_tier(p, g, m, v, oracle.ADAMW, HP["lr"], HP["b1"], HP["b2"], HP["eps"],
                             HP["decay"], s, wl["max_norm"], nthreads)

    warm, t_step = 0, 0.0
    for s in range(max(1, warmup)):
        t0 = time.perf_counter()
        one(s + 1)
        t_step = time.perf_counter() - t0
        warm += 1
        if budget_s is not None and t_step * (s + 2) > budget_s:
            break
    if budget_s is not None:
        steps = max(1, min(steps, int(budget_s / max(t_step, 1e-9))))
    t0 = time.perf_counter()
    for s in range(steps):
        one(warm + s + 1)
    dt = time.perf_counter() - t0
    return sum(wl["sizes"]) * steps / dt, dt / steps * 1e3, warm, steps


def run_reference_muon(args, wl, rank):
    """The reference arm for a Muon workload: --warmup untimed and --steps
    timed bounded samples of the step (cpu_muon_sample) on host cores."""
    if rank != 0:
        return
    nthreads = os.cpu_count() or 1
    value, ms, sample = cpu_muon_run(wl, nthreads, args.steps, args.warmup)
    sample = f"{args.steps} timed samples after {args.warmup} warm-up; each: {sample}"
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": value, "unit": "params/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "f32 Newton-Schulz, bf16 params", "data": "synthetic",
        "config": muon_config(args.workload, wl),
        "parallelism": "host cores (the oracle's restatement of tikun-cpu)",
        "cpu_baseline": {"value": value, "unit": "params/s", "cores": nthreads,
                         "cpu_model": cpu_model(), "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "params/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0}}), flush=True)


def run_reference(args, wl, rank):
    if rank != 0:
        return
    nthreads = os.cpu_count() or 1
    # the requested --steps K after --warmup W; bounded so that each phase
    # stays within two minutes on a slow host (the step is about 0.15 s on a
    # B200 box's host cores)
    value, ms, warm, steps = cpu_reference_run(wl, args.steps, args.warmup, nthreads,
                                               budget_s=120.0)
    sample = (f"full workload ({sum(wl['sizes']):,} params), {steps} timed steps after {warm} "
              f"warm-up, {nthreads} threads over leaves")
    if (steps, warm) != (args.steps, args.warmup):
        sample += f" (cut from {args.steps} / {args.warmup} to stay within the time bound)"
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": value, "unit": "params/s",
        "n_gpus": args.gpus, "steps": steps, "warmup": warm, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": pointwise_config(args.workload, wl),
        "parallelism": "host cores (the oracle's restatement of tikun-cpu)",
        "cpu_baseline": {"value": value, "unit": "params/s", "cores": nthreads, "cpu_model": cpu_model(), "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": "params/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }), flush=True)


def cpu_muon_sample(wl, nthreads, budget_flops=4e10, aw_cap=1 << 22, seed=7):
    """One bounded sample of a Muon workload's step on host cores through the
    oracle, extrapolated to the whole step.

    * Per shape group, the momentum/Nesterov update and the f32 Newton-Schulz
      (tensor_engine.rs:12-77, GEMM rows over ``nthreads`` as rayon does) of
      one matrix, timed at a scaled-down size of the same aspect ratio when its
      Newton-Schulz exceeds ``budget_flops``, times the FLOP ratio and the
      group's count.
    * The AdamW leaves (bf16 p and g, f32 m and v) through the oracle's
      two-tier step, threads over leaves as tikun-cpu's rayon: each leaf cut to
      its first ``aw_cap`` elements, times the element ratio.

    Returns (extrapolated seconds per full step, sample description)."""
    import oracle

    from tikun_b200.sharding import ns_dense_flops

    rng = np.random.default_rng(seed)
    groups = {}
    for rc in wl["mats"]:
        groups[rc] = groups.get(rc, 0) + 1
    total_s, notes = 0.0, []
    for (r, c), cnt in groups.items():
        f = 1
        while ns_dense_flops(r // f, c // f) > budget_flops and min(r, c) // f >= 64:
            f *= 2
        rr, cc = r // f, c // f
        g = (rng.standard_normal((rr, cc)) * 1e-3).astype(np.float32)
        buf = np.zeros_like(g)
        t0 = time.perf_counter()
        u = oracle.muon_momentum(buf, g, MUON_HP["momentum"], True)
        x = np.ascontiguousarray(u, dtype=np.float32)
        oracle.polar_step(x, 5, nthreads)
        dt = time.perf_counter() - t0
        total_s += dt * (ns_dense_flops(r, c) / ns_dense_flops(rr, cc)) * cnt
        notes.append(f"{cnt}x{r}x{c}" + (f" timed at {rr}x{cc}" if f > 1 else ""))
    sizes = wl["adamw"]
    cut = [min(n, aw_cap) for n in sizes]
    p = [oracle.f32_to_bf16((rng.standard_normal(n) * 0.02).astype(np.float32)) for n in cut]
    gr = [oracle.f32_to_bf16((rng.standard_normal(n) * 1e-3).astype(np.float32)) for n in cut]
    m = [np.zeros(n, np.float32) for n in cut]
    v = [np.zeros(n, np.float32) for n in cut]
    t0 = time.perf_counter()
    oracle.step_two_tier(p, gr, m, v, oracle.ADAMW, HP["lr"], HP["b1"], HP["b2"], HP["eps"],
                         HP["decay"], 1, 0.0, min(nthreads, len(cut)))
    # threads over leaves: the step takes as long as its largest leaf
    total_s += (time.perf_counter() - t0) * max(sizes) / max(cut)
    desc = ("Newton-Schulz of one matrix per shape group (" + ", ".join(notes) +
            "), times the FLOP ratio and the group's count; AdamW leaves cut to their first "
            f"{aw_cap:,} elements, times the element ratio; {nthreads} threads; extrapolated")
    return total_s, desc


def cpu_muon_run(wl, nthreads, steps, warmup):
    """``warmup`` untimed and ``steps`` timed bounded samples (cpu_muon_sample)
    of a Muon workload on host cores; returns (params/s, ms per full step
    extrapolated, sample description)."""
    for k in range(warmup):
        cpu_muon_sample(wl, nthreads, seed=100 + k)
    per = []
    desc = ""
    for k in range(steps):
        t, desc = cpu_muon_sample(wl, nthreads, seed=k)
        per.append(t)
    step_s = sum(per) / len(per)
    n_params = sum(r * c for r, c in wl["mats"]) + sum(wl["adamw"])
    return n_params / step_s, step_s * 1e3, desc


def muon_workloads():
    """Muon configurations: (rows, cols) of the hidden matrices and AdamW leaf sizes."""
    def gpt2(d=768, layers=12, vocab=50257):
        mats = [(d, d)] * 4 + [(d, 4 * d), (4 * d, d)]
        return mats * layers, [vocab * d] + [d] * (2 * (2 * layers + 1))

    def gpt13(d=2048, layers=24, ffn=8192, vocab=50304):
        mats = [(d, d)] * 4 + [(d, ffn), (ffn, d)]
        return mats * layers, [vocab * d] + [d] * (2 * layers + 1), layers

    def llama8b(d=4096, layers=32, kv=1024, ffn=14336, vocab=128256):
        mats = [(d, d), (d, kv), (d, kv), (d, d), (d, ffn), (d, ffn), (ffn, d)]
        return mats * layers, [vocab * d, vocab * d] + [d] * (2 * layers + 1)

    m2, a2 = gpt2()
    m3, a3, l3 = gpt13()
    m4, a4 = llama8b()
    return {
        "muon-gpt2-d768": dict(mats=m2, adamw=a2, layers=12, inbackward=False,
                               desc="Muon on 12 x {4 x 768^2, 768x3072, 3072x768} bf16 + AdamW "
                                    "on wte 50257x768 and 25 LayerNorms"),
        "muon-1.3b-inbackward": dict(mats=m3, adamw=a3, layers=l3, inbackward=True,
                                     desc="Muon+AdamW, d=2048, 24 layers, ffn 8192, vocab 50304, "
                                          "bf16; in-backward: per-layer steps fire in reverse "
                                          "layer order on a side stream as each layer's "
                                          "synthetic grads are produced"),
        "muon-llama3-8b": dict(mats=m4, adamw=a4, layers=32, inbackward=False,
                               desc="Muon+AdamW on Llama-3-8B shapes (d 4096, 32 layers, "
                                    "GQA 4096x1024, ffn 14336, vocab 128256), bf16 params, "
                                    "f32 momentum and moments"),
    }


MUON = muon_workloads()
MUON_HP = dict(lr=0.02, momentum=0.95)


def timed_loop(step_fn, steps, warmup, stream, world, dist, dev, torch, uuid, before_step=None):
    """Warm-up, then `steps` timed steps between CUDA events on the launching
    stream, bracketed by barrier + synchronize; returns (max-over-ranks ms,
    launches, clock summary)."""
    for _ in range(warmup):
        step_fn()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    launches = 0
    with ClockSampler(uuid) as clk:
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        start.record(stream)
        for k in range(steps):
            if before_step is not None:
                before_step(k)
            launches += step_fn()
        stop.record(stream)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
    t = torch.tensor([start.elapsed_time(stop)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item()), launches, clk.summary()


def run_pointwise(args, wl, world, rank, dev, torch, dist):
    from tikun_b200 import _native
    from tikun_b200.arena import Arena, LayoutPlan
    from tikun_b200.distributed import pieces_to_segments

    L = _native.lib()
    stream = torch.cuda.current_stream()
    s_handle = stream.cuda_stream
    if args.zero == "auto":
        args.zero = "fused"
    fused = world > 1 and args.zero != "allgather"
    plan = LayoutPlan(wl["sizes"], pad_to=16 * max(world, 1))
    hp_np, hg_np = make_host_state(wl)
    P, G = (Arena(plan, device=dev) for _ in range(2))
    for i in range(len(plan)):
        P.leaf(i).copy_(torch.from_numpy(hp_np[i]))
        G.leaf(i).copy_(torch.from_numpy(hg_np[i]))
    n_params = sum(wl["sizes"])
    hp = _native.TkHParams(HP["lr"], HP["b1"], HP["b2"], HP["eps"], HP["decay"])
    state = {"step": 0, "ev": None}
    clip = wl["max_norm"] > 0
    if world == 1:
        M, V = (Arena(plan, device=dev) for _ in range(2))
        leaves, n_leaves = _native.make_leaves(P.ptrs(), G.ptrs(), M.ptrs(), V.ptrs(), wl["sizes"])
        my_params = n_params
        scale_dev = torch.ones(1, dtype=torch.float32, device=dev)

        def one_step():
            state["step"] += 1
            ev = state["ev"]
            _native.check(L.tk_set_update_events(*(ev if ev else (None, None))))
            _native.check(L.tk_step_buffers_async(leaves, n_leaves, _native.TK_ADAMW,
                                                  ctypes.byref(hp), state["step"],
                                                  wl["max_norm"], scale_dev.data_ptr(), s_handle))
            return 2 if clip else 1
    else:
        # ZeRO-1 through the C ABI (tk_shard_*): the update kernel stores into
        # the peers' arenas (peers), or an all-gather follows it
        from tikun_b200.distributed import ShardedStep, ZeroHParams

        zp = ShardedStep(plan, P.flat, G.flat,
                         ZeroHParams(HP["lr"], HP["b1"], HP["b2"], HP["eps"], HP["decay"],
                                     wl["max_norm"]),
                         exchange={"fused": "peers", "copy": "copy"}.get(args.zero, "allgather"))
        my_params = sum(n for _, _, n in pieces_to_segments(plan, zp.lo, zp.hi))

        def one_step():
            ev = state["ev"]
            _native.check(L.tk_set_update_events(*(ev if ev else (None, None))))
            zp.step()
            return 4 if clip else 1  # norm partials, norm reduce, clip scale, update

    ev_pairs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                for _ in range(args.steps)]
    for a, b in ev_pairs:  # torch creates the CUDA events on first record
        a.record(stream)
        b.record(stream)

    def before(k):  # the library records them around its update launches
        state["ev"] = (ev_pairs[k][0].cuda_event, ev_pairs[k][1].cuda_event)

    uuid = str(torch.cuda.get_device_properties(dev).uuid)
    ms_total, launches, clocks = timed_loop(one_step, args.steps, args.warmup, stream, world, dist,
                                            dev, torch, uuid, before)
    state["ev"] = None
    _native.check(L.tk_set_update_events(None, None))
    if world > 1:
        zp.close()
    upd_ms = sum(a.elapsed_time(b) for a, b in ev_pairs) / args.steps
    ms_step = ms_total / args.steps
    value = n_params / (ms_step / 1e3)
    peak, peak_kind = load_peaks()
    upd_bytes = 28 * my_params
    achieved = upd_bytes / (upd_ms / 1e3) / 1e9
    traffic = None
    tpath = os.path.join(REPO, "profiles", "traffic.json")
    if os.path.exists(tpath):
        with open(tpath) as f:
            tr = json.load(f).get(f"{args.workload}/update")
        if tr:
            traffic = tr["bytes_per_param"] * my_params

    e2e = None
    if not args.no_e2e:
        # pinned host leaves: the whole PyTree on one GPU (tk_step_buffers), or
        # each rank's ZeRO-1 slice of it (tk_step_buffers_sharded, the Tier-1
        # sum all-reduced over NCCL)
        if world == 1:
            segs = [(i, 0, n) for i, n in enumerate(wl["sizes"])]
        else:
            segs = pieces_to_segments(plan, zp.lo, zp.hi)
        hp_pin = [torch.from_numpy(hp_np[i][a:a + n]).pin_memory() for i, a, n in segs]
        hg_pin = [torch.from_numpy(hg_np[i][a:a + n]).pin_memory() for i, a, n in segs]
        hm_pin = [torch.zeros(n).pin_memory() for _, _, n in segs]
        hv_pin = [torch.zeros(n).pin_memory() for _, _, n in segs]
        hleaves, hn = _native.make_leaves([t.data_ptr() for t in hp_pin],
                                          [t.data_ptr() for t in hg_pin],
                                          [t.data_ptr() for t in hm_pin],
                                          [t.data_ptr() for t in hv_pin], [n for _, _, n in segs])
        out = ctypes.c_float()
        comm = None
        if world > 1:
            from tikun_b200.distributed import nccl_comm_ptr
            comm = nccl_comm_ptr(None, dev)

        def host_step(k):
            if comm is None:
                _native.check(L.tk_step_buffers(hleaves, hn, _native.TK_ADAMW, ctypes.byref(hp),
                                                k, wl["max_norm"], ctypes.byref(out), s_handle))
            else:
                _native.check(L.tk_step_buffers_sharded(hleaves, hn, _native.TK_ADAMW,
                                                        ctypes.byref(hp), k, wl["max_norm"],
                                                        ctypes.byref(out), comm, s_handle))

        e2e_steps = max(3, min(args.steps, 10))
        for k in range(3):
            host_step(k + 1)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for k in range(e2e_steps):
            host_step(k + 4)
        e1.record(stream)
        torch.cuda.synchronize()
        e_ms = e0.elapsed_time(e1) / e2e_steps
        if world > 1:
            t = torch.tensor([e_ms], dtype=torch.float64, device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            e_ms = float(t.item())
        e2e = {"value": n_params / (e_ms / 1e3), "unit": "params/s", "ms_per_step": e_ms,
               "h2d_bytes_per_step": 16 * n_params, "d2h_bytes_per_step": 12 * n_params + 4 * world,
               "steps": e2e_steps, "host_memory": "pinned",
               "api": ("tk_step_buffers" if world == 1 else
                       f"tk_step_buffers_sharded on each of {world} ranks over its ZeRO-1 slice") +
                      " with pinned host leaves: g copied to HBM for the clip, p/m/v streamed "
                      "through the copy engines around the update kernel; bytes are whole-job"}
        del hp_pin, hg_pin, hm_pin, hv_pin

    cpu = None
    if not args.no_cpu_baseline and world == 1 and rank == 0:
        nthreads = os.cpu_count() or 1
        # a bounded sample: as many full steps as fit in about 10 s of host time
        cval, cms, cwarm, csteps = cpu_reference_run(wl, 100, 3, nthreads, budget_s=10.0)
        cpu = {"value": cval, "unit": "params/s", "cores": nthreads, "cpu_model": cpu_model(), "kind": "port",
               "sample": f"full workload, {csteps} timed steps after {cwarm} warm-up (about "
                         f"10 s), {nthreads} threads over leaves ({cms:.0f} ms/step)"}
        # not the reference's schedule: the same arithmetic with every leaf cut
        # into 1M-element pieces shared by all threads
        hval, hms, hwarm, hsteps = cpu_reference_run(wl, 100, 3, nthreads, budget_s=5.0,
                                                     chunk=1 << 20)
        cpu["all_cores_chunked"] = {
            "value": hval, "unit": "params/s", "cores": nthreads, "cpu_model": cpu_model(), "kind": "port, non-reference",
            "sample": f"full workload, leaves cut into 1M-element pieces over {nthreads} "
                      f"threads, {hsteps} timed steps after {hwarm} warm-up ({hms:.0f} ms/step)"}
    res = {
        "value": value, "ms_per_step": ms_step, "dtype": "f32", "scaling": "strong",
        "data": "synthetic (seeded N(0,0.02) params, N(0,%g) grads held fixed across steps)"
                % wl["g_std"],
        "config": pointwise_config(args.workload, wl),
        "parallelism": "single GPU" if world == 1 else
        f"zero1-dp{world} via tk_shard_step (" + {
            "fused": "update kernel stores into peer arenas over NVLink",
            "copy": "copy engines copy each updated chunk into peer arenas",
            "allgather": "ncclAllGather after the update"}[args.zero] + ")",
        "roofline": {"bound": "hbm", "kernel": "pointwise_kernel (AdamW update)",
                     "achieved": achieved, "peak": peak, "peak_kind": peak_kind, "unit": "GB/s",
                     "frac": achieved / peak, "traffic": traffic,
                     "algorithmic_bytes_per_launch": upd_bytes, "update_ms": upd_ms,
                     "step_GBps": (32 if clip else 28) * n_params / (ms_step / 1e3) / 1e9},
        "gpu_launches": launches, "clocks": clocks, "e2e": e2e, "cpu_baseline": cpu,
    }
    if fused:
        # the update kernel also writes 4 B per owned parameter to each peer
        # over NVLink and receives the peers' slices into its own HBM: its
        # target time is the slower of HBM and NVLink (measured 770 GB/s per
        # direction per GPU)
        nvl_bytes = 4 * my_params * (world - 1)
        hbm_bytes = upd_bytes + 4 * (n_params - my_params)
        target_ms = max(hbm_bytes / (peak * 1e9), nvl_bytes / 770e9) * 1e3
        res["roofline"]["fused_exchange"] = {
            "nvlink_bytes_per_launch": nvl_bytes, "nvlink_peak_GBps": 770,
            "hbm_bytes_per_launch": hbm_bytes, "target_ms": target_ms,
            "frac_of_target": target_ms / upd_ms}
    return res


def ns_scratch_bytes(m, n, split=False):
    """Newton-Schulz scratch of one m x n matrix (m <= n), as the library lays
    it out (rows padded to 64 elements, buffers 256-byte aligned): two X^T, A,
    A' and B in 16-bit (twice as wide with split f16 operands), the norm
    partials and the scale."""
    r64 = lambda x: (x + 63) // 64 * 64  # noqa: E731
    a256 = lambda x: (x + 255) // 256 * 256  # noqa: E731
    ldm = r64(m) * (2 if split else 1)
    nblk = max(1, min(256, (m * n + 16383) // 16384))
    return 2 * a256(n * ldm * 2) + 3 * a256(m * ldm * 2) + a256(8 * nblk) + a256(4) + 256


def muon_host_e2e(args, wl, world, dev, torch, dist, stream, mine, mats, hp, mhp, p_of, g_of,
                  p_aw, g_aw, plan, segs):
    """The Muon step end to end through the C ABI with host buffers, the
    reference's calling convention (MuonND hands NumPy buffers to the engine,
    python/tikun/muon_nd.py:96-126): this rank's matrices (bf16 p and g, f32
    momentum) and its AdamW slice (bf16 p and g, f32 m and v) live in host
    memory, page-locked with cudaHostRegister; each step is tk_muon_step over
    the host matrices (g, momentum and p stream in, p and momentum stream back,
    overlapped with the tensor-core work) and tk_step_buffers over the host
    AdamW leaves.  Both calls return when their results are back in host
    memory.  Returns the ``e2e`` record (params/s over all ranks, max-over-ranks
    time)."""
    from tikun_b200 import _native

    L = _native.lib()
    bf = torch.bfloat16
    s_handle = stream.cuda_stream
    sizes = {i: mats[i][0] * mats[i][1] for i in mine}
    n_mu = sum(sizes.values())
    n_aw = sum(c for _, _, c in segs)
    host = {"p": np.empty(max(n_mu, 1), np.int16), "g": np.empty(max(n_mu, 1), np.int16),
            "mom": np.zeros(max(n_mu, 1), np.float32),
            "ap": np.empty(max(n_aw, 1), np.int16), "ag": np.empty(max(n_aw, 1), np.int16),
            "am": np.zeros(max(n_aw, 1), np.float32), "av": np.zeros(max(n_aw, 1), np.float32)}
    cudart = torch.cuda.cudart()
    registered = []
    try:
        for a in host.values():
            torch.cuda.check_error(cudart.cudaHostRegister(a.ctypes.data, a.nbytes, 0))
            registered.append(a)
        t = {k: torch.from_numpy(a) for k, a in host.items()}
        hoff, at = {}, 0
        for i in mine:
            hoff[i] = at
            t["p"][at:at + sizes[i]].view(bf).copy_(p_of(i).view(-1))
            g = g_of(i)
            if g is not None:
                t["g"][at:at + sizes[i]].view(bf).copy_(g.view(-1))
            else:
                t["g"][at:at + sizes[i]].view(bf).normal_(0, 1e-3)
            at += sizes[i]
        at = 0
        for i, a, c in segs:
            o = plan.slots[i][0] + a
            t["ap"][at:at + c].view(bf).copy_(p_aw[o:o + c])
            t["ag"][at:at + c].view(bf).copy_(g_aw[o:o + c])
            at += c
        base = {k: a.ctypes.data for k, a in host.items()}
        arr = (_native.TkMuonLeaf * max(len(mine), 1))()
        for k, i in enumerate(mine):
            r, c = mats[i]
            arr[k] = _native.TkMuonLeaf(base["p"] + hoff[i] * 2, base["g"] + hoff[i] * 2,
                                        base["mom"] + hoff[i] * 4, 1, r, c, _native.TK_BF16,
                                        _native.TK_BF16)
        offs_aw = np.cumsum([0] + [c for _, _, c in segs])[:-1]
        aw = _native.make_leaves([base["ap"] + int(o) * 2 for o in offs_aw],
                                 [base["ag"] + int(o) * 2 for o in offs_aw],
                                 [base["am"] + int(o) * 4 for o in offs_aw],
                                 [base["av"] + int(o) * 4 for o in offs_aw],
                                 [c for _, _, c in segs], [_native.TK_BF16] * len(segs),
                                 [_native.TK_BF16] * len(segs))

        def host_step(k):
            _native.check(L.tk_muon_step(arr, len(mine), ctypes.byref(mhp), s_handle))
            _native.check(L.tk_step_buffers(aw[0], aw[1], _native.TK_ADAMW, ctypes.byref(hp), k,
                                            0.0, None, s_handle))

        host_step(1)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        steps = max(2, min(args.steps, 5))
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for k in range(steps):
            host_step(k + 2)
        e1.record(stream)
        torch.cuda.synchronize()
        e_ms = e0.elapsed_time(e1) / steps
        if world > 1:
            tt = torch.tensor([e_ms], dtype=torch.float64, device=dev)
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            e_ms = float(tt.item())
    finally:
        for a in registered:
            cudart.cudaHostUnregister(a.ctypes.data)
    n_all = sum(r * c for r, c in mats) + sum(wl["adamw"])
    return {"value": n_all / (e_ms / 1e3), "unit": "params/s", "ms_per_step": e_ms,
            # per Muon parameter 8 B in (g 2, momentum 4, p 2) and 6 B out (p, momentum);
            # per AdamW parameter 12 B in (p, g, m, v) and 10 B out (p, m, v); whole job
            "h2d_bytes_per_step": 8 * sum(r * c for r, c in mats) + 12 * sum(wl["adamw"]),
            "d2h_bytes_per_step": 6 * sum(r * c for r, c in mats) + 10 * sum(wl["adamw"]),
            "steps": steps, "host_memory": "page-locked (cudaHostRegister)",
            "api": "tk_muon_step over host matrices + tk_step_buffers over host AdamW leaves" +
                   ("" if world == 1 else f", each of {world} ranks over its own matrices and "
                                          "ZeRO-1 slice")}


def run_muon(args, wl, world, rank, dev, torch, dist):
    from tikun_b200 import _native
    from tikun_b200.arena import LayoutPlan, shard_bounds, shard_segments
    from tikun_b200.sharding import ns_dense_flops, ns_issued_flops, owner_major_layout

    L = _native.lib()
    stream = torch.cuda.current_stream()
    s_handle = stream.cuda_stream
    gen = torch.Generator(device=dev).manual_seed(1234 + rank)
    mats = wl["mats"]
    sizes = [r * c for r, c in mats]
    costs = [ns_dense_flops(r, c) for r, c in mats]
    bf = torch.bfloat16
    g_mu, mom = {}, {}
    if world == 1:
        # Muon parameters: one arena (bf16)
        owner = [0] * len(mats)
        offs, extent = owner_major_layout(sizes, owner, 1)
        p_mu = torch.empty(extent, dtype=bf, device=dev)
        p_mu.normal_(0, 0.02, generator=gen)
        mine = list(range(len(mats)))
        for i in mine:
            g_mu[i] = torch.empty(sizes[i], dtype=bf, device=dev).normal_(0, 1e-3, generator=gen)
            mom[i] = torch.zeros(sizes[i], dtype=torch.float32, device=dev)
    # AdamW leaves: one arena, ZeRO-1 slice per rank
    plan = LayoutPlan(wl["adamw"], pad_to=64 * max(world, 1))
    p_aw = torch.empty(plan.total, dtype=bf, device=dev).normal_(0, 0.02, generator=gen)
    g_aw = torch.empty(plan.total, dtype=bf, device=dev).normal_(0, 1e-3, generator=gen)
    m_aw = torch.zeros(plan.total, dtype=torch.float32, device=dev)
    v_aw = torch.zeros(plan.total, dtype=torch.float32, device=dev)
    lo, hi = shard_bounds(plan.total, world, rank)
    segs = shard_segments(plan, lo, hi)

    def aw_leaves(seg_list):
        return _native.make_leaves(
            [p_aw.data_ptr() + (plan.slots[i][0] + a) * 2 for i, a, c in seg_list],
            [g_aw.data_ptr() + (plan.slots[i][0] + a) * 2 for i, a, c in seg_list],
            [m_aw.data_ptr() + (plan.slots[i][0] + a) * 4 for i, a, c in seg_list],
            [v_aw.data_ptr() + (plan.slots[i][0] + a) * 4 for i, a, c in seg_list],
            [c for i, a, c in seg_list], [_native.TK_BF16] * len(seg_list),
            [_native.TK_BF16] * len(seg_list))

    hp = _native.TkHParams(HP["lr"], HP["b1"], HP["b2"], HP["eps"], HP["decay"])
    ns_prec = {"f16": _native.TK_NS_F16, "bf16": _native.TK_NS_BF16,
               "f16x3": _native.TK_NS_F16X3, "f16x2": _native.TK_NS_F16X2}[args.ns_precision]
    mhp = _native.TkMuonHParams(MUON_HP["lr"], MUON_HP["momentum"], 1, 5, ns_prec)

    def mu_leaves(idx):
        arr = (_native.TkMuonLeaf * max(len(idx), 1))()
        for k, i in enumerate(idx):
            r, c = mats[i]
            arr[k] = _native.TkMuonLeaf(p_mu.data_ptr() + offs[i] * 2, g_mu[i].data_ptr(),
                                        mom[i].data_ptr(), 1, r, c, _native.TK_BF16,
                                        _native.TK_BF16)
        return arr, len(idx)

    state = {"step": 0, "ns_ms": []}
    ns_ev, aw_ev = [], []
    exchange = {"fused": "peers", "copy": "copy", "auto": "copy"}.get(args.zero, "allgather")
    if world > 1:
        # Muon matrices LPT-assigned to ranks (MuonShard); AdamW leaves ZeRO-1;
        # with "peers" both update kernels store into every rank's arena over
        # NVLink, otherwise all-gathers follow them
        from tikun_b200.distributed import MuonShard, PeerArena

        ms = MuonShard(mats, bf, dev, MUON_HP["lr"], MUON_HP["momentum"], precision=ns_prec,
                       exchange=exchange)
        ms.params.normal_(0, 0.02, generator=gen)
        mine = ms.mine
        if not wl["inbackward"]:
            g_mu = {i: torch.empty(sizes[i], dtype=bf, device=dev).normal_(0, 1e-3,
                                                                          generator=gen)
                    for i in mine}
        aw_peer = PeerArena(p_aw) if exchange != "allgather" else None
        all_aw = aw_leaves(segs)
        barrier = torch.zeros(1, dtype=torch.float64, device=dev)

        if wl["inbackward"]:
            # layer l's grads come from a generator kernel on the main stream
            # (standing in for backward), in reverse layer order; the side
            # stream steps the rank's matrices of that layer as they appear
            side = torch.cuda.Stream(device=dev)
            per_layer = len(mats) // wl["layers"]
            layer_ev = [torch.cuda.Event() for _ in range(wl["layers"])]
            g_all = {i: torch.empty(sizes[i], dtype=bf, device=dev) for i in range(len(mats))}

            def one_step():
                state["step"] += 1
                e0, e1 = (torch.cuda.Event(enable_timing=True),
                          torch.cuda.Event(enable_timing=True))
                ms.step_begin(side)
                e0.record(side)
                for l in reversed(range(wl["layers"])):
                    for i in range(l * per_layer, (l + 1) * per_layer):
                        g_all[i].normal_(0, 1e-3, generator=gen)
                    layer_ev[l].record(stream)
                    side.wait_event(layer_ev[l])
                    ms.step_part(range(l * per_layer, (l + 1) * per_layer), g_all, side)
                # the AdamW leaves (embedding last in backward, then norms)
                if aw_peer is not None:
                    _native.check(L.tk_apply_pointwise_peers(
                        all_aw[0], all_aw[1], _native.TK_ADAMW, ctypes.byref(hp), state["step"],
                        None, aw_peer.deltas, aw_peer.n, side.cuda_stream))
                else:
                    _native.check(L.tk_apply_pointwise(all_aw[0], all_aw[1], _native.TK_ADAMW,
                                                       ctypes.byref(hp), state["step"], None,
                                                       side.cuda_stream))
                    with torch.cuda.stream(side):
                        dist.all_gather_into_tensor(p_aw, p_aw[lo:hi])
                ms.step_end(side)
                e1.record(side)
                ns_ev.append((e0, e1))
                stream.wait_stream(side)
                return -1
    if world > 1 and not wl["inbackward"]:

        def one_step():
            state["step"] += 1
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            ms.step(g_mu, events=(e0, e1))
            ns_ev.append((e0, e1))
            if aw_peer is not None:
                _native.check(L.tk_apply_pointwise_peers(all_aw[0], all_aw[1], _native.TK_ADAMW,
                                                         ctypes.byref(hp), state["step"], None,
                                                         aw_peer.deltas, aw_peer.n, s_handle))
                dist.all_reduce(barrier)
            else:
                _native.check(L.tk_apply_pointwise(all_aw[0], all_aw[1], _native.TK_ADAMW,
                                                   ctypes.byref(hp), state["step"], None,
                                                   s_handle))
                dist.all_gather_into_tensor(p_aw, p_aw[lo:hi])
            return -1  # counted below from the tile plan
    elif world == 1 and not wl["inbackward"]:
        all_mu = mu_leaves(mine)
        all_aw = aw_leaves(segs)

        def one_step():
            state["step"] += 1
            e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
            e0.record(stream)
            _native.check(L.tk_muon_step(all_mu[0], all_mu[1], ctypes.byref(mhp), s_handle))
            e1.record(stream)
            ns_ev.append((e0, e1))
            _native.check(L.tk_apply_pointwise(all_aw[0], all_aw[1], _native.TK_ADAMW,
                                               ctypes.byref(hp), state["step"], None, s_handle))
            e2.record(stream)
            aw_ev.append((e1, e2))
            return -1  # counted below from the tile plan
    elif world == 1:
        # in-backward (one GPU): layer l's grads are produced on the main stream
        # (a generator kernel standing in for backward), then its Muon and
        # AdamW steps run on a side stream, in reverse layer order; two side
        # streams take alternate layers, so one layer's step can overlap the
        # previous one's
        sides = [torch.cuda.Stream(device=dev) for _ in range(2)]
        per_layer = len(mats) // wl["layers"]
        layer_mu = [mu_leaves(list(range(l * per_layer, (l + 1) * per_layer)))
                    for l in range(wl["layers"])]
        # norms of layer l: the two leaves after the embedding for that layer
        layer_aw = [aw_leaves([s for s in segs if s[0] in (1 + 2 * l, 2 + 2 * l)])
                    for l in range(wl["layers"])]
        rest_aw = aw_leaves([s for s in segs if s[0] == 0 or s[0] == len(wl["adamw"]) - 1])
        layer_ev = [torch.cuda.Event() for _ in range(wl["layers"])]

        def one_step():
            state["step"] += 1
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for l in reversed(range(wl["layers"])):
                side = sides[l % 2]
                for i in range(l * per_layer, (l + 1) * per_layer):
                    g_mu[i].normal_(0, 1e-3, generator=gen)
                layer_ev[l].record(stream)
                side.wait_event(layer_ev[l])
                _native.check(L.tk_muon_step(layer_mu[l][0], layer_mu[l][1], ctypes.byref(mhp),
                                             side.cuda_stream))
                _native.check(L.tk_apply_pointwise(layer_aw[l][0], layer_aw[l][1],
                                                   _native.TK_ADAMW, ctypes.byref(hp),
                                                   state["step"], None, side.cuda_stream))
            _native.check(L.tk_apply_pointwise(rest_aw[0], rest_aw[1], _native.TK_ADAMW,
                                               ctypes.byref(hp), state["step"], None,
                                               side.cuda_stream))
            for sd in sides:
                stream.wait_stream(sd)
            e1.record(stream)
            ns_ev.append((e0, e1))
            return -1

    uuid = str(torch.cuda.get_device_properties(dev).uuid)
    ms_total, _, clocks = timed_loop(one_step, args.steps, args.warmup, stream, world, dist, dev,
                                     torch, uuid)
    assert _native.device_status() == 0, "a Newton-Schulz kernel reported a bounded-wait timeout"
    if world > 1:
        ms.close()
        if aw_peer is not None:
            aw_peer.close()
    ms_step = ms_total / args.steps
    n_params = sum(sizes) + sum(wl["adamw"])
    value = n_params / (ms_step / 1e3)
    ns_ms = sum(a.elapsed_time(b) for a, b in ns_ev[-args.steps:]) / args.steps
    my_dense = sum(costs[i] for i in mine)
    my_issued = sum(ns_issued_flops(*mats[i]) for i in mine)
    d = json.load(open(os.path.join(REPO, "MEASURED_PEAKS.json"))) if os.path.exists(
        os.path.join(REPO, "MEASURED_PEAKS.json")) else {}
    long_step = ms_step > 100
    peak = d.get("bf16_tflops_sustained" if long_step else "bf16_tflops", 1590.0)
    peak_kind = ("measured " + ("sustained" if long_step else "burst")) if d else "fallback"
    achieved = my_dense / (ns_ms / 1e3) / 1e12
    # launches per step: per call, shape group (m x n and n x m together) and
    # wave: 3 prologue kernels + 3 GEMMs x 5 iterations (+ the copy kernel when
    # the exchange is the copy kernel); plus the AdamW update launch(es)
    def ns_launches(idx):
        groups = {}
        for i in idx:
            key = (min(mats[i]), max(mats[i]))
            groups[key] = groups.get(key, 0) + 1
        n = 0
        for (m, nn), cnt in groups.items():
            per_wave = max(1, min(cnt, 256, (8 << 30) // ns_scratch_bytes(
                m, nn, args.ns_precision in ("f16x3", "f16x2"))))
            if world > 1 and exchange == "copy":  # at least three waves per group
                per_wave = max(1, min(per_wave, (cnt + 2) // 3))
            waves = -(-cnt // per_wave)
            n += waves * (3 + 15 + (1 if world > 1 and exchange == "copy" else 0))
        return n

    if wl["inbackward"]:
        per_layer = len(mats) // wl["layers"]
        calls = [[i for i in range(l * per_layer, (l + 1) * per_layer) if i in set(mine)]
                 for l in range(wl["layers"])]
        launches = sum(ns_launches(c) for c in calls) + (wl["layers"] + 1 if world == 1 else 1)
    else:
        launches = ns_launches(mine) + 1
    launches *= args.steps
    aw_params = sum(c for _, _, c in segs)
    aw_GBps = None
    if aw_ev:  # AdamW over bf16 p and g, f32 m and v: 22 B per parameter
        aw_ms = sum(a.elapsed_time(b) for a, b in aw_ev[-args.steps:]) / args.steps
        aw_GBps = 22 * aw_params / (aw_ms / 1e3) / 1e9

    e2e = None
    if not args.no_e2e:
        e2e = muon_host_e2e(args, wl, world, dev, torch, dist, stream, mine, mats, hp, mhp,
                            lambda i: (p_mu[offs[i]:offs[i] + sizes[i]] if world == 1
                                       else ms.params[ms.offs[i]:ms.offs[i] + sizes[i]]),
                            lambda i: g_mu[i] if i in g_mu else None,
                            p_aw, g_aw, plan, segs)

    cpu = None
    if not args.no_cpu_baseline and world == 1 and rank == 0:
        nthreads = os.cpu_count() or 1
        cval, cms, csample = cpu_muon_run(wl, nthreads, steps=3, warmup=1)
        cpu = {"value": cval, "unit": "params/s", "cores": nthreads, "cpu_model": cpu_model(),
               "kind": "port",
               "sample": f"3 timed samples after 1 warm-up, each: {csample} "
                         f"({cms:.0f} ms per full step, extrapolated)"}
    return {
        "value": value, "ms_per_step": ms_step,
        "dtype": "bf16 params, " + {"f16": "f16", "bf16": "bf16",
                                    "f16x3": "split f16 (hi+lo)",
                                    "f16x2": "f16, X as f16 pairs"}[args.ns_precision] +
                 " tensor-core operands",
        "scaling": "strong",
        "data": "synthetic (seeded N(0,0.02) bf16 params, N(0,1e-3) bf16 grads)",
        "config": muon_config(args.workload, wl),
        "parallelism": "single GPU" if world == 1 else
        f"muon-lpt{world}+zero1-dp{world}, " + (
            {"peers": "update kernels store into peer arenas over NVLink",
             "copy": "a copy kernel on 16 reserved SMs stores each finished Muon "
                     "batch into peer arenas during the next batch; the AdamW update "
                     "kernel stores into them",
             "allgather": "all-gathers after the updates"}[exchange]),
        "roofline": {"bound": "tensor", "kernel": "gemm_pair_kernel (m >= 1024) / gemm_tn_kernel (Newton-Schulz GEMMs)",
                     "achieved": achieved, "peak": peak, "peak_kind": peak_kind,
                     "unit": "TFLOP/s", "frac": achieved / peak, "traffic": None,
                     "flops": "dense-equivalent 5(4m^2n+2m^3) per matrix",
                     "ns_ms_per_step": ns_ms,
                     "issued_tflops": my_issued / (ns_ms / 1e3) / 1e12,
                     "issued_frac": my_issued / (ns_ms / 1e3) / 1e12 / peak,
                     "ns_dense_tflop_per_step_this_rank": my_dense / 1e12,
                     "adamw_GBps": aw_GBps,
                     "adamw_frac_of_hbm": None if aw_GBps is None else aw_GBps / load_peaks()[0]},
        "gpu_launches": launches, "clocks": clocks, "e2e": e2e, "cpu_baseline": cpu,
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="tikun", choices=["tikun", "reference"])
    ap.add_argument("--workload", default="muon-llama3-8b", choices=sorted(WORKLOADS) + sorted(MUON))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--ns-precision", default="f16", choices=["f16", "bf16", "f16x3", "f16x2"],
                    help="Newton-Schulz operands for the Muon workloads: f16 (default), bf16, "
                         "split f16 pairs (three times the tensor-core work, Newton-Schulz "
                         "within a few 1e-6 of f32), or X alone as f16 pairs (1.4 to 1.5 times the f16 time)")
    ap.add_argument("--zero", default="auto", choices=["auto", "fused", "copy", "allgather"],
                    help="multi-GPU exchange of updated parameters: peer stores from the update "
                         "kernel (fused), copies beside the next batch's work (copy: the copy "
                         "engines for AdamW chunks, a copy kernel on reserved SMs for Muon "
                         "batches), or all-gathers; auto = fused for AdamW, copy for Muon")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        if args.workload in WORKLOADS:
            run_reference(args, WORKLOADS[args.workload], rank)
        else:
            run_reference_muon(args, MUON[args.workload], rank)
        return

    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=300))
    if args.workload in WORKLOADS:
        res = run_pointwise(args, WORKLOADS[args.workload], world, rank, dev, torch, dist)
    else:
        res = run_muon(args, MUON[args.workload], world, rank, dev, torch, dist)
    if rank == 0:
        line = {"metric": METRIC, "value": res["value"], "unit": "params/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": res["ms_per_step"],
                "higher_is_better": True, "scaling": res["scaling"], "vs_baseline": None,
                "dtype": res["dtype"], "data": res["data"], "config": res["config"],
                "parallelism": res["parallelism"],
                "roofline": res["roofline"], "gpu_launches": res["gpu_launches"],
                "clocks": res["clocks"], "e2e": res["e2e"], "cpu_baseline": res["cpu_baseline"]}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
