"""tk_step_buffers_noalloc: the clipped two-tier step for callers that cannot
allocate device memory (an application that owns a fixed memory budget, or a
host runtime whose allocator must not be re-entered from an optimizer hook).

It must give the same results as tk_step_buffers, which takes its scratch from
a memory pool.  Checked through the C ABI on two calls in a row (the second
call reuses the fixed scratch the first one left behind), with the same
bit-identity bar as the other pointwise tests.  This file is collected last so
that a run stopping at the first failure has already run every other test; it
also passes on its own in a fresh process.
"""
import ctypes

import pytest
import torch

from helpers import Leaves, assert_bitexact, gpt2_small_sizes, to_np
from tikun_b200 import _native

pytestmark = pytest.mark.gpu


def _call(fn_name, L, step, max_norm, kind=_native.TK_ADAMW, want_scale=True):
    leaves, n = _native.make_leaves(
        [t.data_ptr() for t in L.p], [t.data_ptr() for t in L.g], [t.data_ptr() for t in L.m],
        [t.data_ptr() for t in L.v], [t.numel() for t in L.p],
        [_native.TK_BF16 if t.dtype == torch.bfloat16 else _native.TK_F32 for t in L.p],
        [_native.TK_BF16 if t.dtype == torch.bfloat16 else _native.TK_F32 for t in L.g])
    hp = _native.TkHParams(1e-3, 0.9, 0.99 if kind == _native.TK_LION else 0.999, 1e-8, 0.01)
    out = ctypes.c_float(-1.0)
    fn = getattr(_native.lib(), fn_name)
    _native.check(fn(leaves, n, kind, ctypes.byref(hp), step, max_norm,
                     ctypes.byref(out) if want_scale else None,
                     torch.cuda.current_stream().cuda_stream))
    return out.value


@pytest.mark.parametrize("max_norm", [1.0, 0.0], ids=["clip", "no_clip"])
def test_noalloc_matches_pooled_step_on_two_calls(max_norm):
    sizes = gpt2_small_sizes(d=128, vocab=1000, ctx=256)
    dts = [torch.bfloat16 if i % 7 == 3 else torch.float32 for i in range(len(sizes))]
    A = Leaves(sizes, p_dtypes=dts, g_dtypes=dts, seed=21)
    B = Leaves(sizes, p_dtypes=dts, g_dtypes=dts, seed=21)
    for step in (1, 2):
        A.new_grads(1e-2)
        B.g = [g.clone() for g in A.g]
        s_pool = _call("tk_step_buffers", A, step, max_norm)
        s_fixed = _call("tk_step_buffers_noalloc", B, step, max_norm)
        assert s_fixed == s_pool
        if max_norm > 0:
            assert s_pool < 1.0, "the clip must trigger"
        for i in range(len(sizes)):
            assert_bitexact(to_np(B.p[i]), to_np(A.p[i]), f"step {step} leaf {i} p")
            assert_bitexact(to_np(B.m[i]), to_np(A.m[i]), f"step {step} leaf {i} m")
            assert_bitexact(to_np(B.v[i]), to_np(A.v[i]), f"step {step} leaf {i} v")


def test_noalloc_rejects_more_leaves_than_its_limit():
    t = [torch.zeros(4, device="cuda") for _ in range(4 * 225)]
    leaves, n = _native.make_leaves([x.data_ptr() for x in t[0:225]],
                                    [x.data_ptr() for x in t[225:450]],
                                    [x.data_ptr() for x in t[450:675]],
                                    [x.data_ptr() for x in t[675:900]], [4] * 225)
    hp = _native.TkHParams(1e-3, 0.9, 0.999, 1e-8, 0.01)
    st = _native.lib().tk_step_buffers_noalloc(leaves, n, _native.TK_ADAMW, ctypes.byref(hp), 1,
                                               1.0, None, None)
    assert st == _native.TK_ERR_INVALID
    assert b"at most 224 leaves" in _native.lib().tk_last_error()


@pytest.mark.parametrize("kind", [_native.TK_LION, _native.TK_SGD], ids=["lion", "sgd"])
def test_noalloc_lion_and_sgd_match_pooled_step(kind):
    """Lion and SGD read no second moment (m2 may be anything) and use their own
    constants; the fixed-scratch step still gives the pooled step's bytes."""
    sizes = [1, 17, 4097, 65536 + 5, 300]
    A = Leaves(sizes, seed=5, kind="lion" if kind == _native.TK_LION else "sgd")
    B = Leaves(sizes, seed=5, kind="lion" if kind == _native.TK_LION else "sgd")
    for step in (1, 2):
        A.new_grads(0.05)
        B.g = [g.clone() for g in A.g]
        assert _call("tk_step_buffers_noalloc", B, step, 0.5, kind) == \
            _call("tk_step_buffers", A, step, 0.5, kind)
        for i in range(len(sizes)):
            assert_bitexact(to_np(B.p[i]), to_np(A.p[i]), f"step {step} leaf {i} p")
            assert_bitexact(to_np(B.m[i]), to_np(A.m[i]), f"step {step} leaf {i} m")


def test_noalloc_without_scale_out_is_stream_ordered():
    """With clip_scale_out NULL the call only enqueues; after a stream
    synchronisation the results equal the pooled step's."""
    sizes = [4099, 768, 65536]
    A = Leaves(sizes, seed=8)
    B = Leaves(sizes, seed=8)
    A.new_grads(0.05)
    B.g = [g.clone() for g in A.g]
    _call("tk_step_buffers", A, 1, 1.0)
    _call("tk_step_buffers_noalloc", B, 1, 1.0, want_scale=False)
    torch.cuda.current_stream().synchronize()
    for i in range(len(sizes)):
        assert_bitexact(to_np(B.p[i]), to_np(A.p[i]), f"leaf {i} p")
        assert_bitexact(to_np(B.v[i]), to_np(A.v[i]), f"leaf {i} v")


def test_noalloc_rejects_host_leaves():
    p, g, m, v = (torch.zeros(64).pin_memory() for _ in range(4))
    leaves, n = _native.make_leaves([p.data_ptr()], [g.data_ptr()], [m.data_ptr()],
                                    [v.data_ptr()], [64])
    hp = _native.TkHParams(1e-3, 0.9, 0.999, 1e-8, 0.01)
    st = _native.lib().tk_step_buffers_noalloc(leaves, n, _native.TK_ADAMW, ctypes.byref(hp), 1,
                                               1.0, None, None)
    assert st == _native.TK_ERR_INVALID
    assert b"device buffers only" in _native.lib().tk_last_error()


_FRESH_PROCESS = r"""
import ctypes, sys
sys.path.insert(0, sys.argv[1])
import torch
from tikun_b200 import _native
L = _native.lib()
ps = [torch.randn(n, device="cuda") * 0.02 for n in (4099, 65536, 1)]
gs = [torch.randn(n, device="cuda") * 0.05 for n in (4099, 65536, 1)]
ms = [torch.zeros(n, device="cuda") for n in (4099, 65536, 1)]
vs = [torch.zeros(n, device="cuda") for n in (4099, 65536, 1)]
leaves, n = _native.make_leaves([t.data_ptr() for t in ps], [t.data_ptr() for t in gs],
                                [t.data_ptr() for t in ms], [t.data_ptr() for t in vs],
                                [t.numel() for t in ps])
hp = _native.TkHParams(1e-3, 0.9, 0.999, 1e-8, 0.01)
out = ctypes.c_float(0.0)
for step in (1, 2, 3):
    _native.check(L.tk_step_buffers_noalloc(leaves, n, _native.TK_ADAMW, ctypes.byref(hp), step,
                                            1.0, ctypes.byref(out), None))
held = ctypes.c_uint64(1)
_native.check(L.tk_testing_library_device_bytes(ctypes.byref(held)))
print("scale", out.value, "library_device_bytes", held.value)
assert 0.0 < out.value < 1.0 and held.value == 0
"""


def test_noalloc_allocates_nothing_in_a_fresh_process():
    """In a process that calls only the fixed-scratch step, the library never
    creates its scratch pool or its status word: it held no device memory of
    its own after three clipped calls."""
    import os
    import subprocess
    import sys

    repo = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    r = subprocess.run([sys.executable, "-c", _FRESH_PROCESS, repo], capture_output=True,
                       text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "library_device_bytes 0" in r.stdout
