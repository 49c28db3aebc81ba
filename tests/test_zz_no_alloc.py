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


def _call(fn_name, L, step, max_norm):
    leaves, n = _native.make_leaves(
        [t.data_ptr() for t in L.p], [t.data_ptr() for t in L.g], [t.data_ptr() for t in L.m],
        [t.data_ptr() for t in L.v], [t.numel() for t in L.p],
        [_native.TK_BF16 if t.dtype == torch.bfloat16 else _native.TK_F32 for t in L.p],
        [_native.TK_BF16 if t.dtype == torch.bfloat16 else _native.TK_F32 for t in L.g])
    hp = _native.TkHParams(1e-3, 0.9, 0.999, 1e-8, 0.01)
    out = ctypes.c_float(-1.0)
    fn = getattr(_native.lib(), fn_name)
    _native.check(fn(leaves, n, _native.TK_ADAMW, ctypes.byref(hp), step, max_norm,
                     ctypes.byref(out), torch.cuda.current_stream().cuda_stream))
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
