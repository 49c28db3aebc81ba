"""Benchmark of the tikun optimizer step on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl tikun|reference]
                    [--workload gpt2-small-clip|flat-100m]

Default workload (the one the headline metric is quoted on at one GPU):
clipped AdamW (global-norm clip 1.0) over the GPT-2-small PyTree, 148 fp32
leaves, 124,439,808 parameters, lr 1e-3, betas (0.9, 0.999), eps 1e-8,
decay 0.01; params N(0, 0.02) with biases 0 and LayerNorm weights 1, grads
N(0, 1e-2) (seeded synthetic data).

One step = one full optimizer step over every leaf.  ``value`` is parameters
updated per second with all buffers resident in HBM (p, g, m, v: 1.99 GB, well
above the 126 MB L2, so no flush is needed between steps), timed with CUDA
events on the launching stream; at N GPUs the step is ZeRO-1 (each rank
updates its 1/N of the flat parameter space, f64 norm all-reduce, NCCL
all-gather of the updated fp32 parameters) and the time is the max over ranks.
``e2e`` is the same step through the C ABI with the leaves in pinned host
memory (the reference engine's calling convention), copies included.

``--impl reference`` times the reference's CPU algorithm (the oracle's
restatement of tikun-cpu; the Rust engine cannot be built here) on this host's
cores on the same workload.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
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
    """nvidia-smi samples every 200 ms for the GPU with the given UUID."""

    FIELDS = ("uuid,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, uuid: str):
        self.uuid = uuid
        self.rows = []
        self.proc = None
        self.thread = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9 and self.uuid and self.uuid in parts[0]:
                self.rows.append(parts)

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.thread.join(timeout=5)

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        sm = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows for i in range(4) if r[5 + i] == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(self.rows)}


# ------------------------------------------------------------------ workload
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


def cpu_reference_run(wl, steps, warmup, nthreads):
    """The oracle (tikun-cpu's algorithm, restated) on host cores, threads over
    leaves as tikun-cpu's rayon par_iter over leaves."""
    import oracle

    p, g = make_host_state(wl)
    m = [np.zeros_like(x) for x in p]
    v = [np.zeros_like(x) for x in p]
    for s in range(warmup):
        oracle.step_two_tier(p, g, m, v, oracle.ADAMW, HP["lr"], HP["b1"], HP["b2"], HP["eps"],
                             HP["decay"], s + 1, wl["max_norm"], nthreads)
    t0 = time.perf_counter()
    for s in range(steps):
        oracle.step_two_tier(p, g, m, v, oracle.ADAMW, HP["lr"], HP["b1"], HP["b2"], HP["eps"],
                             HP["decay"], warmup + s + 1, wl["max_norm"], nthreads)
    dt = time.perf_counter() - t0
    return sum(wl["sizes"]) * steps / dt, dt / steps * 1e3


def run_reference(args, wl, rank):
    if rank != 0:
        return
    nthreads = os.cpu_count() or 1
    # bounded: at most 10 timed steps of the full workload (about 1 s each)
    steps = max(1, min(args.steps, 10))
    warm = max(1, min(args.warmup, 3))
    value, ms = cpu_reference_run(wl, steps, warm, nthreads)
    sample = (f"full workload ({sum(wl['sizes']):,} params), {steps} timed steps after {warm} "
              f"warm-up, {nthreads} threads over leaves")
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": value, "unit": "params/s",
        "n_gpus": args.gpus, "steps": steps, "warmup": warm, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": {"workload": args.workload, "desc": wl["desc"]},
        "cpu_baseline": {"value": value, "unit": "params/s", "cores": nthreads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": "params/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="tikun", choices=["tikun", "reference"])
    ap.add_argument("--workload", default="gpt2-small-clip", choices=sorted(WORKLOADS))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    wl = WORKLOADS[args.workload]

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        run_reference(args, wl, rank)
        return

    import torch
    import torch.distributed as dist

    from tikun_b200 import _native
    from tikun_b200.arena import Arena, LayoutPlan, shard_bounds, shard_segments

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))
    stream = torch.cuda.current_stream()
    L = _native.lib()

    # --- state: one arena per array (p, g, m, v) -----------------------------
    plan = LayoutPlan(wl["sizes"], pad_to=16 * max(world, 1))
    hp_np, hg_np = make_host_state(wl)
    P, G, M, V = (Arena(plan, device=dev) for _ in range(4))
    for i in range(len(plan)):
        P.leaf(i).copy_(torch.from_numpy(hp_np[i]))
        G.leaf(i).copy_(torch.from_numpy(hg_np[i]))
    n_params = sum(wl["sizes"])
    lo, hi = shard_bounds(plan.total, world, rank)
    segs = shard_segments(plan, lo, hi)
    es = 4
    pp, gp, mp, vp = P.ptrs(), G.ptrs(), M.ptrs(), V.ptrs()
    leaves, n_leaves = _native.make_leaves(
        [pp[i] + a * es for i, a, c in segs], [gp[i] + a * es for i, a, c in segs],
        [mp[i] + a * es for i, a, c in segs], [vp[i] + a * es for i, a, c in segs],
        [c for i, a, c in segs])
    my_params = sum(c for _, _, c in segs)
    hp = _native.TkHParams(HP["lr"], HP["b1"], HP["b2"], HP["eps"], HP["decay"])
    scale_dev = torch.ones(1, dtype=torch.float32, device=dev)
    sumsq = torch.zeros(1, dtype=torch.float64, device=dev)
    s_handle = stream.cuda_stream
    state = {"step": 0}

    def one_step():
        state["step"] += 1
        if world == 1:
            _native.check(L.tk_step_buffers_async(leaves, n_leaves, _native.TK_ADAMW,
                                                  ctypes.byref(hp), state["step"],
                                                  wl["max_norm"], scale_dev.data_ptr(), s_handle))
            return 2 if wl["max_norm"] > 0 else 1
        launches = 0
        if wl["max_norm"] > 0:
            _native.check(L.tk_grad_sumsq(leaves, n_leaves, sumsq.data_ptr(), s_handle))
            dist.all_reduce(sumsq)
            _native.check(L.tk_clip_scale(sumsq.data_ptr(), wl["max_norm"], scale_dev.data_ptr(),
                                          s_handle))
            launches += 3
        _native.check(L.tk_set_update_events(*state["ev"]) if "ev" in state else 0)
        _native.check(L.tk_apply_pointwise(leaves, n_leaves, _native.TK_ADAMW, ctypes.byref(hp),
                                           state["step"],
                                           scale_dev.data_ptr() if wl["max_norm"] > 0 else None,
                                           s_handle))
        dist.all_gather_into_tensor(P.flat, P.flat[lo:hi])
        return launches + 1

    # --- timed region ----------------------------------------------------------
    for _ in range(args.warmup):
        one_step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ev_pairs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                for _ in range(args.steps)]
    for a, b in ev_pairs:  # torch creates the CUDA events on first record
        a.record(stream)
        b.record(stream)
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    uuid = str(torch.cuda.get_device_properties(dev).uuid)
    launches = 0
    with ClockSampler(uuid) as clk:
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        start.record(stream)
        for k in range(args.steps):
            a, b = ev_pairs[k]
            state["ev"] = (ctypes.c_void_p(a.cuda_event), ctypes.c_void_p(b.cuda_event))
            if world == 1:
                _native.check(L.tk_set_update_events(a.cuda_event, b.cuda_event))
            launches += one_step()
        stop.record(stream)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
    _native.check(L.tk_set_update_events(None, None))
    state.pop("ev", None)
    ms_total = start.elapsed_time(stop)
    upd_ms = sum(a.elapsed_time(b) for a, b in ev_pairs) / args.steps
    t = torch.tensor([ms_total], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_total = float(t.item())
    ms_step = ms_total / args.steps
    value = n_params / (ms_step / 1e3)

    # --- roofline of the update kernel: 28 B/param (read p, g, m, v; write p, m, v)
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

    # --- e2e: host (pinned) leaves through the C ABI, copies inside the region
    e2e = None
    if not args.no_e2e and world == 1:
        hp_pin = [torch.from_numpy(x).pin_memory() for x in hp_np]
        hg_pin = [torch.from_numpy(x).pin_memory() for x in hg_np]
        hm_pin = [torch.zeros(n).pin_memory() for n in wl["sizes"]]
        hv_pin = [torch.zeros(n).pin_memory() for n in wl["sizes"]]
        hleaves, hn = _native.make_leaves([t.data_ptr() for t in hp_pin],
                                          [t.data_ptr() for t in hg_pin],
                                          [t.data_ptr() for t in hm_pin],
                                          [t.data_ptr() for t in hv_pin], wl["sizes"])
        out = ctypes.c_float()
        e2e_steps = max(3, min(args.steps, 10))
        for s in range(3):
            _native.check(L.tk_step_buffers(hleaves, hn, _native.TK_ADAMW, ctypes.byref(hp), s + 1,
                                            wl["max_norm"], ctypes.byref(out), s_handle))
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for s in range(e2e_steps):
            _native.check(L.tk_step_buffers(hleaves, hn, _native.TK_ADAMW, ctypes.byref(hp), s + 4,
                                            wl["max_norm"], ctypes.byref(out), s_handle))
        e1.record(stream)
        torch.cuda.synchronize()
        e_ms = e0.elapsed_time(e1) / e2e_steps
        e2e = {"value": n_params / (e_ms / 1e3), "unit": "params/s", "ms_per_step": e_ms,
               "h2d_bytes_per_step": 16 * n_params, "d2h_bytes_per_step": 12 * n_params + 4,
               "steps": e2e_steps, "host_memory": "pinned"}
        del hp_pin, hg_pin, hm_pin, hv_pin

    # --- CPU baseline (rank 0, one GPU): the oracle on a bounded sample
    cpu = None
    if not args.no_cpu_baseline and world == 1 and rank == 0:
        nthreads = os.cpu_count() or 1
        cval, cms = cpu_reference_run(wl, 2, 1, nthreads)
        cpu = {"value": cval, "unit": "params/s", "cores": nthreads, "kind": "port",
               "sample": f"full workload, 2 timed steps after 1 warm-up, {nthreads} threads over "
                         f"leaves ({cms:.0f} ms/step)"}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "params/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded N(0,0.02) params, N(0,1e-2) grads held fixed across steps)",
            "config": {"workload": args.workload, "desc": wl["desc"], "params": n_params,
                       "leaves": len(wl["sizes"]),
                       "parallelism": "single GPU" if world == 1 else f"zero1-dp{world}",
                       "l2": "inputs (1.99 GB of p,g,m,v) larger than L2; no flush"},
            "roofline": {"bound": "hbm", "kernel": "pointwise_kernel (AdamW update)",
                         "achieved": achieved, "peak": peak, "peak_kind": peak_kind,
                         "unit": "GB/s", "frac": achieved / peak, "traffic": traffic,
                         "algorithmic_bytes_per_launch": upd_bytes,
                         "update_ms": upd_ms,
                         "step_GBps_32B_per_param": 32 * n_params / (ms_step / 1e3) / 1e9
                         if wl["max_norm"] > 0 else 28 * n_params / (ms_step / 1e3) / 1e9},
            "gpu_launches": launches,
            "clocks": clk.summary(),
            "e2e": e2e,
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
