"""tikun oracle — TEST INFRASTRUCTURE ONLY.

CPU restatement of the reference engine's optimizer-step arithmetic, used as the
checker for the CUDA path and as the timed CPU baseline.  Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py`` (its ``cpu_baseline`` leg and its
``--impl reference`` arm) may import this package; the product package
``tikun_b200`` never does.

Two layers:

* ``libtikun_oracle.so`` (``tikun_oracle.c``): the bit-faithful C restatement of
  tikun-cpu's x86 scalar path — Tier-1 norm (crates/tikun-cpu/src/lib.rs:79-125),
  Tier-2 AdamW/Lion/SGD (lib.rs:144-428), the f32 Newton-Schulz polar step
  (crates/tikun-cpu/src/tensor_engine.rs:12-77) and LayoutPlan::from_shapes
  (crates/tikun-core/src/arena.rs:34-57).
* numpy restatements of the same Newton-Schulz algorithm with BLAS matmuls
  (summation order differs from the naive loops; used for large parity cases
  where the naive loops take minutes) and of the MuonND 2-D update
  (python/tikun/muon_nd.py:104-126).

Parity status: pinned against the reference's own checks — torch AdamW over 10
steps (examples/verify_exact_math_parity.py:16-72), the reference's torch
Newton-Schulz (python/tikun/muon.py:10-32), the 4x4 polar identity test
(tensor_engine.rs:198-210) and slot alignment (arena.rs:109-118).
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from typing import Sequence

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "libtikun_oracle.so")
_lib = None

ADAMW, LION, SGD, CUSTOM = 0, 1, 2, 3
F32, BF16 = 0, 1


class _Leaf(ctypes.Structure):
    _fields_ = [
        ("p", ctypes.c_void_p),
        ("g", ctypes.c_void_p),
        ("m", ctypes.c_void_p),
        ("v", ctypes.c_void_p),
        ("n", ctypes.c_uint64),
        ("p_dtype", ctypes.c_int32),
        ("g_dtype", ctypes.c_int32),
    ]


class _HParams(ctypes.Structure):
    _fields_ = [(k, ctypes.c_float) for k in ("lr", "beta1", "beta2", "eps", "decay")]


def build() -> str:
    """Compile the C restatement (idempotent)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        L.tko_powi.restype = ctypes.c_float
        L.tko_powi.argtypes = [ctypes.c_float, ctypes.c_int32]
        L.tko_clip_scale.restype = ctypes.c_float
        L.tko_clip_scale.argtypes = [ctypes.c_double, ctypes.c_float]
        L.tko_leaf_sumsq.restype = ctypes.c_double
        L.tko_leaf_sumsq.argtypes = [ctypes.POINTER(_Leaf)]
        L.tko_step_two_tier.restype = ctypes.c_float
        L.tko_step_two_tier.argtypes = [
            ctypes.POINTER(_Leaf), ctypes.c_size_t, ctypes.c_int32, ctypes.POINTER(_HParams),
            ctypes.c_uint64, ctypes.c_float, ctypes.c_int]
        L.tko_pointwise_leaf.restype = None
        L.tko_pointwise_leaf.argtypes = [ctypes.POINTER(_Leaf), ctypes.c_int32,
                                         ctypes.POINTER(_HParams), ctypes.c_uint64,
                                         ctypes.c_float]
        L.tko_polar_step.restype = None
        L.tko_polar_step.argtypes = [ctypes.c_void_p, ctypes.c_uint64, ctypes.c_uint64,
                                     ctypes.c_uint64, ctypes.c_int]
        L.tko_polar_batched.restype = None
        L.tko_polar_batched.argtypes = [ctypes.c_void_p, ctypes.c_uint64, ctypes.c_uint64,
                                        ctypes.c_uint64, ctypes.c_uint64, ctypes.c_int]
        L.tko_layout_from_shapes.restype = None
        L.tko_layout_from_shapes.argtypes = [ctypes.POINTER(ctypes.c_uint64), ctypes.c_size_t,
                                             ctypes.POINTER(ctypes.c_uint64),
                                             ctypes.POINTER(ctypes.c_uint64)]
        _lib = L
    return _lib


def _dtype_code(a: np.ndarray) -> int:
    if a.dtype == np.float32:
        return F32
    if a.dtype == np.uint16:  # bf16 bit patterns
        return BF16
    raise TypeError(f"oracle leaves hold float32 or bf16-as-uint16, got {a.dtype}")


def opt_kind(name: str) -> int:
    """tikun-py/src/lib.rs:194-214: "lion", "sgd", anything else is AdamW."""
    return {"lion": LION, "sgd": SGD}.get(name, ADAMW)


def step_two_tier(params: Sequence[np.ndarray], grads: Sequence[np.ndarray],
                  m1: Sequence[np.ndarray], m2: Sequence[np.ndarray] | None,
                  kind: int, lr: float, b1: float, b2: float, eps: float, decay: float,
                  step: int, max_norm: float, nthreads: int = 1) -> float:
    """In-place two-tier step over numpy leaves; returns the clip scale."""
    n = len(params)
    leaves = (_Leaf * max(n, 1))()
    for i in range(n):
        p, g, m = params[i], grads[i], m1[i]
        v = m2[i] if m2 else None
        for a in (p, g, m) + ((v,) if v is not None else ()):
            assert a.flags.c_contiguous
        assert m.dtype == np.float32 and (v is None or v.dtype == np.float32)
        assert p.size == g.size == m.size and (v is None or v.size == p.size)
        leaves[i] = _Leaf(p.ctypes.data, g.ctypes.data, m.ctypes.data,
                          v.ctypes.data if v is not None else 0, p.size,
                          _dtype_code(p), _dtype_code(g))
    hp = _HParams(lr, b1, b2, eps, decay)
    return float(lib().tko_step_two_tier(leaves, n, kind, ctypes.byref(hp), step,
                                         max_norm, nthreads))


def pointwise_leaf(p: np.ndarray, g: np.ndarray, m: np.ndarray, v: np.ndarray | None,
                   kind: int, lr: float, b1: float, b2: float, eps: float, decay: float,
                   step: int, clip_scale: float) -> None:
    """Tier 2 over one numpy leaf with a given clip scale, in place
    (crates/tikun-cpu/src/lib.rs:143-428)."""
    for a in (p, g, m) + ((v,) if v is not None else ()):
        assert a.flags.c_contiguous
    leaf = _Leaf(p.ctypes.data, g.ctypes.data, m.ctypes.data,
                 v.ctypes.data if v is not None else 0, p.size, _dtype_code(p), _dtype_code(g))
    hp = _HParams(lr, b1, b2, eps, decay)
    lib().tko_pointwise_leaf(ctypes.byref(leaf), kind, ctypes.byref(hp), step, clip_scale)


def step_fast_buffers(param_ptrs, grad_ptrs, m1_ptrs, m2_ptrs, lengths, max_norm,
                      opt_kind_name, step_count, lr, b1, b2, eps, decay,
                      nthreads: int = 1) -> float:
    """The reference's PyO3 ``step_fast_buffers`` (tikun-py/src/lib.rs:155-222)
    over raw f32 host pointers, computed by the oracle."""
    n = len(param_ptrs)
    leaves = (_Leaf * max(n, 1))()
    for i in range(n):
        leaves[i] = _Leaf(param_ptrs[i], grad_ptrs[i], m1_ptrs[i],
                          0 if len(m2_ptrs) == 0 else m2_ptrs[i], lengths[i], F32, F32)
    hp = _HParams(lr, b1, b2, eps, decay)
    return float(lib().tko_step_two_tier(leaves, n, opt_kind(opt_kind_name), ctypes.byref(hp),
                                         step_count, max_norm, nthreads))


def native_stub():
    """A stand-in for the reference's ``_tikun`` extension whose three hot-path
    functions run on the oracle.  Lets the reference's own Python front-ends
    (python/tikun/*.py) run here to produce golden vectors."""
    import types

    m = types.ModuleType("_tikun")
    m.step_fast_buffers = step_fast_buffers
    m.newton_schulz_2d_ffi = lambda ptr, rows, cols, steps: lib().tko_polar_step(
        ptr, rows, cols, steps, os.cpu_count() or 1)
    m.newton_schulz_3d_ffi = lambda ptr, heads, hout, hin, steps: lib().tko_polar_batched(
        ptr, heads, hout, hin, steps, os.cpu_count() or 1)
    return m


def powi(a: float, b: int) -> float:
    return float(lib().tko_powi(a, b))


def clip_scale(total_sumsq: float, max_norm: float) -> float:
    return float(lib().tko_clip_scale(total_sumsq, max_norm))


def polar_step(x: np.ndarray, steps: int = 5, nthreads: int = 1) -> np.ndarray:
    """Reference-loop f32 Newton-Schulz on a 2-D float32 array, in place."""
    assert x.dtype == np.float32 and x.flags.c_contiguous and x.ndim == 2
    lib().tko_polar_step(x.ctypes.data, x.shape[0], x.shape[1], steps, nthreads)
    return x


def polar_batched(x: np.ndarray, steps: int = 5, nthreads: int = 1) -> np.ndarray:
    assert x.dtype == np.float32 and x.flags.c_contiguous and x.ndim == 3
    lib().tko_polar_batched(x.ctypes.data, x.shape[0], x.shape[1], x.shape[2], steps, nthreads)
    return x


def layout_from_shapes(shapes: Sequence[int]) -> tuple[list[int], int]:
    n = len(shapes)
    arr = (ctypes.c_uint64 * max(n, 1))(*shapes)
    offs = (ctypes.c_uint64 * max(n, 1))()
    total = ctypes.c_uint64()
    lib().tko_layout_from_shapes(arr, n, offs, ctypes.byref(total))
    return list(offs)[:n], int(total.value)


# ---------------------------------------------------------------------------
# numpy restatements
# ---------------------------------------------------------------------------
NS_ABC = (np.float32(3.4445), np.float32(-4.7750), np.float32(2.0315))


def polar_step_np(x: np.ndarray, steps: int = 5) -> np.ndarray:
    """tensor_engine.rs:12-77 with BLAS float32 matmuls (returns a new array).

    Same algorithm and constants; only the GEMM summation order differs from
    the naive loops, which changes results at the 1e-6 relative level.
    """
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows, cols = x.shape
    if rows == 0 or cols == 0:
        return x.copy()
    if rows > cols:
        return np.ascontiguousarray(polar_step_np(np.ascontiguousarray(x.T), steps).T)
    a, b, c = NS_ABC
    s = float(np.sum(x.astype(np.float64) ** 2))
    inv = np.float32(1.0) / np.float32(max(np.float32(np.sqrt(s)), np.float32(1e-7)))
    x = x * inv
    eye = np.eye(rows, dtype=np.float32)
    for _ in range(steps):
        A = x @ x.T
        B = A @ A
        P = a * eye + b * A + c * B
        x = P @ x
    return x.astype(np.float32)


def polar_batched_np(x: np.ndarray, steps: int = 5) -> np.ndarray:
    return np.stack([polar_step_np(x[h], steps) for h in range(x.shape[0])])


def muon_momentum(buf: np.ndarray, grad: np.ndarray, momentum: float,
                  nesterov: bool = True) -> np.ndarray:
    """python/tikun/muon_nd.py:112-116 with NumPy's float32 arithmetic.

    Updates ``buf`` in place and returns the float32 matrix handed to
    Newton-Schulz.  (1 - momentum) is formed in double and rounded once to
    float32, as the reference's Python expression is.
    """
    mu = np.float32(momentum)
    om = np.float32(1.0 - momentum)
    buf *= mu
    buf += om * grad
    if nesterov:
        return (mu * buf + om * grad).astype(np.float32)
    return buf.copy()


def muon_update_scale(rows: int, cols: int) -> float:
    """muon_nd.py:122: sqrt(max(1, rows/cols))."""
    return max(1.0, rows / cols) ** 0.5


def bf16_to_f32(a: np.ndarray) -> np.ndarray:
    return (a.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(a: np.ndarray) -> np.ndarray:
    """Round to nearest even (NaN kept quiet); returns uint16 bit patterns."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r
