"""ctypes binding of ``libtikun_cuda.so`` (the C ABI in include/tikun_cuda.h).

Re-exports the reference's native entry points with their argument lists
(crates/tikun-py/src/lib.rs:155-254):

* ``step_fast_buffers(param_ptrs, grad_ptrs, m1_ptrs, m2_ptrs, lengths,
  max_norm, opt_kind, step_count, lr, b1, b2, eps, decay) -> clip_scale``
* ``newton_schulz_2d_ffi(matrix_ptr, rows, cols, steps)``
* ``newton_schulz_3d_ffi(tensor_ptr, num_heads, head_dim_out, head_dim_in, steps)``

Pointers may be CUDA device pointers (``tensor.data_ptr()``) or host pointers
(numpy ``ctypes.data``).  The library must have been built
(``python -m tikun_b200.build``); there is no CPU fallback, and loading fails
with an error if it is missing.
"""
from __future__ import annotations

import ctypes
import os
import sys
from typing import Sequence

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "lib", "libtikun_cuda.so")

# status codes, dtypes, kinds (include/tikun_cuda.h)
TK_OK, TK_ERR_INVALID, TK_ERR_VERIFY, TK_ERR_CUDA, TK_ERR_ALLOC, TK_ERR_UNSUPPORTED, TK_ERR_DEVICE = range(7)
TK_F32, TK_BF16, TK_F16 = 0, 1, 2
TK_ADAMW, TK_LION, TK_SGD, TK_CUSTOM = 0, 1, 2, 3
TK_ROLE_LOAD, TK_ROLE_COMPUTE, TK_ROLE_STORE = 0, 1, 2
TK_NS_F16, TK_NS_BF16, TK_NS_F16X3, TK_NS_F16X2 = 0, 1, 2, 3


class TkLeaf(ctypes.Structure):
    _fields_ = [
        ("p", ctypes.c_void_p),
        ("g", ctypes.c_void_p),
        ("m", ctypes.c_void_p),
        ("v", ctypes.c_void_p),
        ("n", ctypes.c_uint64),
        ("p_dtype", ctypes.c_int32),
        ("g_dtype", ctypes.c_int32),
    ]


class TkHParams(ctypes.Structure):
    _fields_ = [(k, ctypes.c_float) for k in ("lr", "beta1", "beta2", "eps", "decay")]


class TkMuonLeaf(ctypes.Structure):
    _fields_ = [
        ("p", ctypes.c_void_p),
        ("g", ctypes.c_void_p),
        ("momentum", ctypes.c_void_p),
        ("heads", ctypes.c_int64),
        ("rows", ctypes.c_int64),
        ("cols", ctypes.c_int64),
        ("p_dtype", ctypes.c_int32),
        ("g_dtype", ctypes.c_int32),
    ]


class TkMuonHParams(ctypes.Structure):
    _fields_ = [
        ("lr", ctypes.c_double),
        ("momentum", ctypes.c_double),
        ("nesterov", ctypes.c_int32),
        ("ns_steps", ctypes.c_int32),
        ("precision", ctypes.c_int32),
    ]


class TkScheduleNode(ctypes.Structure):
    _fields_ = [
        ("name", ctypes.c_char_p),
        ("role", ctypes.c_int32),
        ("tile_size", ctypes.c_uint64),
        ("unroll_factor", ctypes.c_uint64),
        ("vector_width", ctypes.c_uint64),
        ("prefetch_distance", ctypes.c_uint64),
    ]


class TkPipeline(ctypes.Structure):
    _fields_ = [
        ("nodes", ctypes.POINTER(TkScheduleNode)),
        ("n_nodes", ctypes.c_size_t),
        ("max_norm", ctypes.c_float),
    ]


class TikunError(RuntimeError):
    """A C-ABI call returned a non-zero status."""

    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status


class TikunValueError(TikunError, ValueError):
    """Invalid arguments (null or overlapping buffers, bad sizes or dtypes)."""


_lib = None
_P = ctypes.c_void_p
_SZ = ctypes.c_size_t
_U64 = ctypes.c_uint64
_I32 = ctypes.c_int32
_I64 = ctypes.c_int64
_F = ctypes.c_float

# name -> argtypes; every entry point returns int
_SIGNATURES = {
    "tk_abi_version": [],
    "tk_verify": [ctypes.POINTER(TkPipeline)],
    "tk_layout_from_shapes": [ctypes.POINTER(_U64), _SZ, ctypes.POINTER(_U64), ctypes.POINTER(_U64)],
    "tk_step_two_tier": [ctypes.POINTER(TkPipeline), ctypes.POINTER(TkLeaf), _SZ, _I32,
                         ctypes.POINTER(TkHParams), _U64, ctypes.POINTER(_F), _P],
    "tk_step_buffers": [ctypes.POINTER(TkLeaf), _SZ, _I32, ctypes.POINTER(TkHParams), _U64, _F,
                        ctypes.POINTER(_F), _P],
    "tk_step_buffers_async": [ctypes.POINTER(TkLeaf), _SZ, _I32, ctypes.POINTER(TkHParams), _U64,
                              _F, _P, _P],
    "tk_step_arena": [ctypes.POINTER(TkPipeline), _P, _P, _P, _P, _U64, ctypes.POINTER(_U64),
                      ctypes.POINTER(_U64), _SZ, _I32, ctypes.POINTER(TkHParams), _U64,
                      ctypes.POINTER(_F), _P],
    "tk_grad_sumsq": [ctypes.POINTER(TkLeaf), _SZ, _P, _P],
    "tk_clip_scale": [_P, _F, _P, _P],
    "tk_apply_pointwise": [ctypes.POINTER(TkLeaf), _SZ, _I32, ctypes.POINTER(TkHParams), _U64,
                           _P, _P],
    "tk_set_update_events": [_P, _P],
    "tk_set_reserved_sms": [ctypes.c_int],
    "tk_apply_pointwise_peers": [ctypes.POINTER(TkLeaf), _SZ, _I32, ctypes.POINTER(TkHParams),
                                 _U64, _P, ctypes.POINTER(_I64), ctypes.c_int, _P],
    "tk_ipc_export": [_P, _P, ctypes.POINTER(_U64)],
    "tk_ipc_import": [_P, _U64, ctypes.POINTER(_P)],
    "tk_ipc_close": [_P],
    "tk_muon_step_peers": [ctypes.POINTER(TkMuonLeaf), _SZ, ctypes.POINTER(TkMuonHParams),
                           ctypes.POINTER(_I64), ctypes.c_int, _P],
    "tk_muon_step_copy": [ctypes.POINTER(TkMuonLeaf), _SZ, ctypes.POINTER(TkMuonHParams),
                          ctypes.POINTER(_I64), ctypes.c_int, _P],
    "tk_muon_step_copy_deferred": [ctypes.POINTER(TkMuonLeaf), _SZ,
                                   ctypes.POINTER(TkMuonHParams), ctypes.POINTER(_I64),
                                   ctypes.c_int, _P],
    "tk_muon_copy_join": [_P],
    "tk_step_buffers_sharded": [ctypes.POINTER(TkLeaf), _SZ, _I32, ctypes.POINTER(TkHParams), _U64,
                                ctypes.c_float, ctypes.POINTER(ctypes.c_float), _P, _P],
    "tk_shard_init": [_P, _P, _P, _U64, ctypes.POINTER(_U64), ctypes.POINTER(_U64), _SZ, _I32,
                      _I32, _P, ctypes.POINTER(_P)],
    "tk_shard_step": [_P, ctypes.POINTER(TkHParams), _U64, ctypes.c_float,
                      ctypes.POINTER(ctypes.c_float), _P],
    "tk_shard_info": [_P, ctypes.POINTER(_U64), ctypes.POINTER(_U64), ctypes.POINTER(_P),
                      ctypes.POINTER(_P)],
    "tk_shard_destroy": [_P, _P],
    "tk_muon_layout": [_SZ, ctypes.POINTER(_I64), ctypes.POINTER(_I64), ctypes.c_int,
                       ctypes.POINTER(_I32), ctypes.POINTER(_U64), ctypes.POINTER(_U64)],
    "tk_muon_shard_init": [_P, _SZ, ctypes.POINTER(_I64), ctypes.POINTER(_I64), _P, _I32,
                           ctypes.POINTER(TkMuonHParams), _I32, _P, ctypes.POINTER(_P)],
    "tk_muon_shard_info": [_P, ctypes.POINTER(_I32), ctypes.POINTER(_U64), ctypes.POINTER(_U64)],
    "tk_muon_shard_step": [_P, ctypes.POINTER(_P), _I32, _P],
    "tk_muon_shard_destroy": [_P, _P],
    "tk_nccl_unique_id": [_P],
    "tk_nccl_comm_init": [_P, ctypes.c_int, ctypes.c_int, ctypes.POINTER(_P)],
    "tk_nccl_comm_destroy": [_P],
    "tk_nccl_comm_async_error": [_P, ctypes.POINTER(_I32)],
    "tk_nccl_comm_abort": [_P],
    "tk_stream_wait_deadline": [_P, _I32, _P],
    "tk_step_buffers_noalloc": [ctypes.POINTER(TkLeaf), _SZ, _I32, ctypes.POINTER(TkHParams),
                                _U64, _F, ctypes.POINTER(_F), _P],
    "tk_newton_schulz_2d": [_P, _I64, _I64, _I32, _I32, _I32, _P],
    "tk_newton_schulz_3d": [_P, _I64, _I64, _I64, _I32, _I32, _I32, _P],
    "tk_muon_step": [ctypes.POINTER(TkMuonLeaf), _SZ, ctypes.POINTER(TkMuonHParams), _P],
    "tk_device_status": [ctypes.POINTER(ctypes.c_int)],
    "tk_testing_bounded_wait": [ctypes.c_int, _P],
    "tk_testing_gemm_tn": [_P, _P, _P, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                           _I64, _I64, _I64, _F, ctypes.c_int, _P],
}

# Newton-Schulz operand type used when the caller does not choose: f16 with a
# power-of-two pre-scale (same tensor-core rate as bf16, 8x smaller rounding).
DEFAULT_NS_PRECISION = TK_NS_F16


def lib() -> ctypes.CDLL:
    """Loads the CUDA library (once).  Raises if it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"tikun_b200 CUDA library not found at {LIB_PATH}; build it with "
                "`python -m tikun_b200.build` (there is no CPU fallback)")
        L = ctypes.CDLL(LIB_PATH)
        L.tk_last_error.restype = ctypes.c_char_p
        L.tk_last_error.argtypes = []
        for name, args in _SIGNATURES.items():
            fn = getattr(L, name, None)
            if fn is None:
                continue  # reported by exported_symbols() checks
            fn.restype = ctypes.c_int
            fn.argtypes = args
        _lib = L
    return _lib


def check(status: int) -> None:
    if status == TK_OK:
        return
    msg = (lib().tk_last_error() or b"").decode("utf-8", "replace")
    if status == TK_ERR_VERIFY:
        raise TikunError(status, msg)
    if status == TK_ERR_INVALID:
        raise TikunValueError(status, msg)
    raise TikunError(status, msg or f"tikun_b200 call failed with status {status}")


def current_stream() -> int:
    """torch's current CUDA stream if torch has initialised CUDA, else 0."""
    torch = sys.modules.get("torch")
    if torch is not None and torch.cuda.is_available() and torch.cuda.is_initialized():
        return torch.cuda.current_stream().cuda_stream
    return 0


def opt_kind(name: str) -> int:
    """tikun-py/src/lib.rs:194-214: "lion" and "sgd" by exact name, else AdamW."""
    return {"lion": TK_LION, "sgd": TK_SGD}.get(name, TK_ADAMW)


def make_leaves(param_ptrs: Sequence[int], grad_ptrs: Sequence[int], m1_ptrs: Sequence[int],
                m2_ptrs: Sequence[int], lengths: Sequence[int],
                p_dtypes: Sequence[int] | None = None,
                g_dtypes: Sequence[int] | None = None):
    n = len(param_ptrs)
    if len(grad_ptrs) != n or len(m1_ptrs) != n or len(lengths) != n or (
            len(m2_ptrs) not in (0, n)):
        raise TikunValueError(TK_ERR_INVALID,
                              "param_ptrs, grad_ptrs, m1_ptrs, m2_ptrs (or empty) and lengths "
                              "must have the same length")
    arr = (TkLeaf * max(n, 1))()
    for i in range(n):
        arr[i] = TkLeaf(param_ptrs[i], grad_ptrs[i], m1_ptrs[i],
                        m2_ptrs[i] if len(m2_ptrs) else 0, lengths[i],
                        p_dtypes[i] if p_dtypes is not None else TK_F32,
                        g_dtypes[i] if g_dtypes is not None else TK_F32)
    return arr, n


def step_fast_buffers(param_ptrs, grad_ptrs, m1_ptrs, m2_ptrs, lengths, max_norm, opt_kind_name,
                      step_count, lr, b1, b2, eps, decay, *, p_dtypes=None, g_dtypes=None,
                      stream: int | None = None) -> float:
    """The reference's ``step_fast_buffers`` on the B200 engine; returns the
    clip scale (1.0 without clipping)."""
    leaves, n = make_leaves(param_ptrs, grad_ptrs, m1_ptrs, m2_ptrs, lengths, p_dtypes, g_dtypes)
    hp = TkHParams(lr, b1, b2, eps, decay)
    out = ctypes.c_float(1.0)
    check(lib().tk_step_buffers(leaves, n, opt_kind(opt_kind_name), ctypes.byref(hp),
                                int(step_count), max_norm, ctypes.byref(out),
                                current_stream() if stream is None else stream))
    return float(out.value)


def step_fast_buffers_async(param_ptrs, grad_ptrs, m1_ptrs, m2_ptrs, lengths, max_norm,
                            opt_kind_name, step_count, lr, b1, b2, eps, decay, *,
                            clip_scale_ptr: int = 0, p_dtypes=None, g_dtypes=None,
                            stream: int | None = None) -> None:
    """Device-buffer variant that does not wait; the clip scale goes to
    ``clip_scale_ptr`` (device f32) when given."""
    leaves, n = make_leaves(param_ptrs, grad_ptrs, m1_ptrs, m2_ptrs, lengths, p_dtypes, g_dtypes)
    hp = TkHParams(lr, b1, b2, eps, decay)
    check(lib().tk_step_buffers_async(leaves, n, opt_kind(opt_kind_name), ctypes.byref(hp),
                                      int(step_count), max_norm, clip_scale_ptr or None,
                                      current_stream() if stream is None else stream))


def newton_schulz_2d_ffi(matrix_ptr: int, rows: int, cols: int, steps: int, *,
                         dtype: int = TK_F32, precision: int | None = None,
                         stream: int | None = None) -> None:
    """The reference's ``newton_schulz_2d_ffi``: in-place polar step of a
    row-major rows x cols matrix (f32 by default, as the reference takes)."""
    check(lib().tk_newton_schulz_2d(matrix_ptr, rows, cols, steps, dtype,
                                    DEFAULT_NS_PRECISION if precision is None else precision,
                                    current_stream() if stream is None else stream))


def newton_schulz_3d_ffi(tensor_ptr: int, num_heads: int, head_dim_out: int, head_dim_in: int,
                         steps: int, *, dtype: int = TK_F32, precision: int | None = None,
                         stream: int | None = None) -> None:
    """The reference's ``newton_schulz_3d_ffi``: polar step of each head."""
    check(lib().tk_newton_schulz_3d(tensor_ptr, num_heads, head_dim_out, head_dim_in, steps,
                                    dtype, DEFAULT_NS_PRECISION if precision is None else precision,
                                    current_stream() if stream is None else stream))


def muon_step(leaves: Sequence[tuple], lr: float, momentum: float, nesterov: bool = True,
              ns_steps: int = 5, precision: int | None = None, stream: int | None = None) -> None:
    """Fused Muon update over (p_ptr, g_ptr, mom_ptr, heads, rows, cols, p_dtype,
    g_dtype) leaves.  Device leaves: enqueued on the stream, does not wait.
    Host leaves (all of them; the reference's convention): streamed through
    device memory, returns when the results are back in host memory."""
    arr = (TkMuonLeaf * max(len(leaves), 1))()
    for i, L in enumerate(leaves):
        arr[i] = TkMuonLeaf(*L)
    hp = TkMuonHParams(lr, momentum, 1 if nesterov else 0, ns_steps,
                       DEFAULT_NS_PRECISION if precision is None else precision)
    check(lib().tk_muon_step(arr, len(leaves), ctypes.byref(hp),
                             current_stream() if stream is None else stream))


def device_status() -> int:
    out = ctypes.c_int(0)
    check(lib().tk_device_status(ctypes.byref(out)))
    return int(out.value)


def verify(nodes: Sequence[tuple], max_norm: float = 0.0) -> None:
    """Verifier::verify over (name, role, tile, unroll, width, prefetch) nodes."""
    arr = (TkScheduleNode * max(len(nodes), 1))()
    names = []
    for i, (name, role, tile, unroll, width, prefetch) in enumerate(nodes):
        b = name.encode()
        names.append(b)
        arr[i] = TkScheduleNode(b, role, tile, unroll, width, prefetch)
    pl = TkPipeline(arr, len(nodes), max_norm)
    check(lib().tk_verify(ctypes.byref(pl)))


def layout_from_shapes(shapes: Sequence[int]) -> tuple[list[int], int]:
    n = len(shapes)
    a = (_U64 * max(n, 1))(*shapes)
    o = (_U64 * max(n, 1))()
    t = _U64()
    check(lib().tk_layout_from_shapes(a, n, o, ctypes.byref(t)))
    return list(o)[:n], int(t.value)
