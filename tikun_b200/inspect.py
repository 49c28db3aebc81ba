"""Execution-plan report and compilation schema of the B200 lowering.

The reference binds ``emit_inspect`` (crates/tikun-py/src/lib.rs:88-113, over
``HardwarePlan::report`` in crates/tikun-core/src/inspect.rs:10-99) and builds a
``CompilationSchema`` (crates/tikun-core/src/schema.rs:78-184) describing its
CPU/NEON schedule.  These are the same two views for the sm_100a engine: the
arguments are the reference's, the content describes what this engine runs --
leaf tables per launch, grids, bytes per parameter and the time that traffic
takes at the measured HBM bandwidth.
"""
from __future__ import annotations

import json
import os
from typing import Sequence

from . import _native

_REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
_SMS = 148
_LEAVES_PER_LAUNCH = 224  # kMaxLeavesPerLaunch: leaf table in kernel parameters
_UPDATE_CTAS_PER_SM = 2   # pointwise_kernel: 256 threads, 2 resident CTAs per SM

# the reference's fast-path schedule (tikun-py/src/lib.rs:48-51)
_NODES = [("Load", "load_p_g", 16), ("Compute", "fma_update", 16), ("Store", "store_p", 16)]

# algorithmic bytes per parameter of one Tier-2 pass, f32 p and g
_BYTES = {"AdamW": (16, 12), "Lion": (12, 8), "SGD": (12, 8)}
_FLOPS = {"AdamW": 14, "Lion": 8, "SGD": 5}


def _algorithm(name: str) -> str:
    # build_spec (tikun-py/src/lib.rs:56-60): "lion", "sgd", anything else AdamW
    return {"lion": "Lion", "sgd": "SGD"}.get(name.lower(), "AdamW")


def _hbm_peak() -> tuple[float, str]:
    path = os.path.join(_REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


def _table(header: Sequence[str], rows: Sequence[Sequence[str]]) -> str:
    widths = [max(len(str(x)) for x in col) for col in zip(header, *rows)]
    line = "+" + "+".join("-" * (w + 2) for w in widths) + "+"
    fmt = lambda r: "| " + " | ".join(str(x).ljust(w) for x, w in zip(r, widths)) + " |"  # noqa: E731
    return "\n".join([line, fmt(header), line] + [fmt(r) for r in rows] + [line])


def compilation_schema(param_ptrs: Sequence[int], lengths: Sequence[int], algorithm: str,
                       max_norm: float, lr: float, b1: float, b2: float, eps: float,
                       decay: float) -> dict:
    """The reference's CompilationSchema fields for the sm_100a lowering."""
    alg = _algorithm(algorithm)
    n = int(sum(lengths))
    rd, wr = _BYTES[alg]
    hyper = {"learning_rate": lr, "beta1": b1,
             "beta2": b2 if alg != "SGD" else None,
             "epsilon": eps if alg == "AdamW" else None,
             "weight_decay": decay, "max_norm": max_norm if max_norm > 0 else None}
    slots = [{"slot_id": i, "byte_offset": int(p), "num_elements": int(c), "byte_size": 4 * int(c),
              "cache_aligned": int(p) % 64 == 0} for i, (p, c) in enumerate(zip(param_ptrs, lengths))]
    passes = []
    if max_norm > 0:
        passes.append({"pass_id": 0, "pass_name": "sumsq_partials", "pass_role": "Reduce",
                       "target_hardware_unit": "sm_100a LSU, 128-bit loads, f64 FMA"})
    for role, name, _ in _NODES:
        passes.append({"pass_id": len(passes), "pass_name": name, "pass_role": role,
                       "target_hardware_unit": "sm_100a pointwise_kernel (" +
                       {"Load": "128-bit global loads", "Compute": "IEEE f32 FMUL/FADD/FDIV/FSQRT",
                        "Store": "128-bit global stores"}[role] + ")"})
    read = n * rd + (4 * n if max_norm > 0 else 0)
    written = n * wr
    return {
        "schema_version": "tikun.ir.v1.0",
        "target_architecture": "NVIDIA B200 (sm_100a)",
        "optimizer": {"algorithm": alg, "precision": "float32 (IEEE, separately rounded)",
                      "hyperparameters": hyper},
        "memory_topography": {"total_parameters": n, "total_allocated_bytes": 4 * n,
                              "cache_line_size_bytes": 128,
                              "is_cache_aligned": all(int(p) % 64 == 0 for p in param_ptrs),
                              "slots": slots},
        "execution_schedule": {"leaves_per_launch": _LEAVES_PER_LAUNCH,
                               "launches": -(-len(lengths) // _LEAVES_PER_LAUNCH) if lengths else 0,
                               "ctas": _SMS * _UPDATE_CTAS_PER_SM, "threads_per_cta": 256,
                               "vector_width_bytes": 16, "passes": passes},
        "performance_metrics": {"bytes_read_per_step": read, "bytes_written_per_step": written,
                                "total_memory_traffic_bytes": read + written,
                                "arithmetic_intensity_flop_per_byte":
                                    _FLOPS[alg] / float(rd + wr)},
    }


def emit_schema(*args, **kwargs) -> str:
    """compilation_schema as pretty JSON (CompilationSchema::to_json)."""
    return json.dumps(compilation_schema(*args, **kwargs), indent=2)


def emit_inspect(param_ptrs: Sequence[int], lengths: Sequence[int], algorithm: str,
                 max_norm: float, lr: float, b1: float, b2: float, eps: float, decay: float,
                 tile_kb: int | None = None, unroll: int | None = None,
                 prefetch: int | None = None, workers: int | None = None) -> str:
    """The reference's ``emit_inspect`` report (same arguments; ``tile_kb``,
    ``unroll``, ``prefetch`` and ``workers`` describe a CPU schedule and are
    shown as given) for the sm_100a lowering."""
    if len(param_ptrs) != len(lengths):
        raise _native.TikunValueError(_native.TK_ERR_INVALID,
                                      "param_ptrs and lengths must have the same length")
    sc = compilation_schema(param_ptrs, lengths, algorithm, max_norm, lr, b1, b2, eps, decay)
    peak, kind = _hbm_peak()
    mem = sc["memory_topography"]
    perf = sc["performance_metrics"]
    ex = sc["execution_schedule"]
    est_us = perf["total_memory_traffic_bytes"] / (peak * 1e9) * 1e6
    out = ["", "--- Hardware Execution Plan (B200, sm_100a) ---"]
    out.append(_table(["Property", "Value"], [
        ["Algorithm", sc["optimizer"]["algorithm"]],
        ["Target", sc["target_architecture"]],
        ["Active Memory", f"{mem['total_allocated_bytes'] / 2**20:.2f} MB "
                          f"({mem['total_parameters']} floats)"],
        ["Cache Alignment", "64-Byte Aligned" if mem["is_cache_aligned"] else "Unaligned"],
        ["Global Norm Clip", f"max_norm {max_norm}" if max_norm > 0 else "off"],
        ["Launches", f"{ex['launches']} x pointwise_kernel ({ex['leaves_per_launch']} leaves each)"
                     + (" + sumsq_partials" if max_norm > 0 else "")],
        ["Grid", f"{ex['ctas']} CTAs x {ex['threads_per_cta']} threads, equal slices of "
                 f"4-element groups"],
        ["Traffic", f"{perf['total_memory_traffic_bytes'] / 1e6:.1f} MB per step"],
        ["HBM Estimate", f"{est_us:.1f} us at {peak:.0f} GB/s ({kind})"],
        ["CPU Schedule Args", f"tile {tile_kb or 512} KB, unroll {unroll or 4}x, "
                              f"prefetch {prefetch or 128} B, {workers or 12} workers"],
    ]))
    out.append("")
    out.append("Schedule Nodes:")
    out.append(_table(["Role", "Op Name", "Tile Size", "Unroll", "Width", "Prefetch"],
                      [[r, nm, f"{t} B", "1x", "16 lanes", "0 B"] for r, nm, t in _NODES]))
    out.append("")
    out.append("Memory Layout:")
    rows = [[f"{s['slot_id']:02d}", f"0x{s['byte_offset']:08x}", str(s["num_elements"]),
             f"{s['byte_size'] / 2**20:.2f} MB",
             "64-B Aligned" if s["cache_aligned"] else "Unaligned"] for s in mem["slots"][:8]]
    out.append(_table(["Slot", "Offset", "Elements", "Size", "Alignment"], rows))
    if len(mem["slots"]) > 8:
        out.append(f"... and {len(mem['slots']) - 8} additional parameter slots")
    return "\n".join(out) + "\n"
