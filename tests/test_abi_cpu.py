"""C-ABI checks that need no GPU: the library loads, exports every entry point
include/*.h declares, and the host-only entry points (verifier, layout plan)
behave like the reference's."""
import glob
import os
import re

import pytest

from tikun_b200 import _native
from tikun_b200.universal import _flatten_pytree, _extract_pointer_and_len

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    names = set()
    for h in glob.glob(os.path.join(REPO, "include", "*.h")):
        src = open(h).read()
        names.update(re.findall(r"TK_API\s+[\w\s\*]*?\b(tk_\w+)\s*\(", src))
    return sorted(names)


def test_library_exports_every_declared_symbol():
    lib = _native.lib()
    syms = declared_symbols()
    assert "tk_step_buffers" in syms and "tk_last_error" in syms
    missing = [s for s in syms if not hasattr(lib, s)]
    assert not missing, missing


def test_abi_version():
    assert _native.lib().tk_abi_version() == 1


def test_library_is_the_in_tree_build():
    assert os.path.realpath(_native.LIB_PATH).startswith(os.path.join(REPO, "tikun_b200"))


# -- verifier: crates/tikun-core/src/verifier.rs:14-45 ----------------------
def test_verify_accepts_reference_pipeline():
    nodes = [("load_g", 0, 64, 4, 8, 2), ("fma_opt", 1, 64, 4, 8, 2), ("store_p", 2, 64, 4, 8, 2)]
    _native.verify(nodes)


def test_verify_empty_pipeline():
    with pytest.raises(_native.TikunError) as e:
        _native.verify([])
    assert str(e.value) == "Static verification failed: [EmptyPipeline]"
    assert e.value.status == _native.TK_ERR_VERIFY


def test_verify_reports_every_violation_in_order():
    nodes = [("a", 0, 100, 4, 3, 2), ("b", 1, 64, 4, 8, 2), ("c", 2, 128, 4, 2, 2)]
    with pytest.raises(_native.TikunError) as e:
        _native.verify(nodes)
    assert str(e.value) == (
        'Static verification failed: [MisalignedCacheLine { node_name: "a", tile_size: 100 }, '
        'InvalidVectorWidth { node_name: "a", width: 3 }, '
        'InvalidVectorWidth { node_name: "c", width: 2 }]')


@pytest.mark.parametrize("width,ok", [(0, False), (1, False), (2, False), (4, True), (6, False),
                                      (8, True), (64, True), (1 << 20, True)])
def test_verify_vector_width_rule(width, ok):
    nodes = [("n", 1, 64, 4, width, 2)]
    if ok:
        _native.verify(nodes)
    else:
        with pytest.raises(_native.TikunError):
            _native.verify(nodes)


# -- layout: crates/tikun-core/src/arena.rs:34-57, tests :219-228 -------------
def test_layout_matches_oracle_and_alignment():
    import oracle

    for shapes in ([100, 513, 2048, 17], [1, 1, 1], [16, 16], [], [38597376, 786432, 768, 768]):
        offs, total = _native.layout_from_shapes(shapes)
        assert all(o % 64 == 0 for o in offs)
        assert (offs, total) == oracle.layout_from_shapes(shapes)


# -- host-side argument handling (no CUDA call is reached) ---------------------
def test_mismatched_list_lengths_raise_value_error():
    with pytest.raises(ValueError):
        _native.step_fast_buffers([1, 2], [3], [4, 5], [6, 7], [1, 1], 0.0, "adamw", 1, 1e-3,
                                  0.9, 0.999, 1e-8, 0.0)


def test_opt_kind_dispatch_matches_reference():
    # tikun-py/src/lib.rs:194-214: exact "lion"/"sgd", anything else AdamW
    assert _native.opt_kind("lion") == _native.TK_LION
    assert _native.opt_kind("sgd") == _native.TK_SGD
    assert _native.opt_kind("adamw") == _native.TK_ADAMW
    assert _native.opt_kind("Lion") == _native.TK_ADAMW
    assert _native.opt_kind("anything") == _native.TK_ADAMW


def test_pytree_flattening_order():
    import numpy as np

    a, b, c = np.zeros(3, np.float32), np.zeros(4, np.float32), np.zeros(5, np.float32)
    tree = {"x": a, "y": [b, (c,)], "raw": (1234, 7)}
    flat = _flatten_pytree(tree)
    assert flat[0] is a and flat[1] is b and flat[2] is c and flat[3] == (1234, 7)
    assert _extract_pointer_and_len(flat[3]) == (1234, 7)
    # strided views would be stepped as if contiguous: rejected
    import torch

    with pytest.raises(ValueError, match="strided"):
        _extract_pointer_and_len(torch.zeros(4, 6).t())
    with pytest.raises(ValueError, match="strided"):
        _extract_pointer_and_len(np.zeros(10, np.float32)[::2])
    t = torch.zeros(4, 6)
    assert _extract_pointer_and_len(t[1:3]) == (t[1:3].data_ptr(), 12)
    assert _extract_pointer_and_len(b) == (b.ctypes.data, 4)


# -- arena: crates/tikun-core/src/arena.rs:120-133 ----------------------------
def test_arena_leaf_views_alias_the_flat_buffer():
    import torch

    from tikun_b200.arena import Arena, LayoutPlan, shard_segments

    plan = LayoutPlan([128, 256, 17])
    a = Arena(plan, device="cpu")
    a.leaf(0)[0] = 42.0
    a.leaf(2)[16] = 7.0
    assert a.leaf(0)[0].item() == 42.0
    off2, _ = plan.slots[2]
    assert a.flat[off2 + 16].item() == 7.0
    # the padding between and after leaves stays zero-filled and belongs to no leaf
    mask = torch.zeros(plan.total, dtype=torch.bool)
    for off, n in plan.slots:
        mask[off:off + n] = True
    assert torch.count_nonzero(a.flat[~mask]) == 0
    assert [p - a.flat.data_ptr() for p in a.ptrs()] == [off * 4 for off, _ in plan.slots]
    assert plan.total % 16 == 0
    pieces = shard_segments(plan, 0, plan.total)
    assert pieces == [(i, 0, n) for i, n in enumerate(plan.sizes)]


# -- argument checks that return before any CUDA call --------------------------
def _err(status):
    return status, _native.lib().tk_last_error().decode()


def test_argument_checks_need_no_device():
    import ctypes

    L = _native.lib()
    I64 = ctypes.c_int64
    hp = _native.TkHParams(1e-3, 0.9, 0.999, 1e-8, 0.0)
    mhp = _native.TkMuonHParams()
    cases = [
        (lambda: L.tk_newton_schulz_2d(None, -1, 4, 5, _native.TK_F32, _native.TK_NS_F16, None),
         _native.TK_ERR_INVALID, "negative size"),
        (lambda: L.tk_newton_schulz_2d(None, 4, 4, 5, 7, _native.TK_NS_F16, None),
         _native.TK_ERR_INVALID, "not f32 or bf16"),
        (lambda: L.tk_newton_schulz_3d(None, 2, 4, 4, 5, _native.TK_F32, 9, None),
         _native.TK_ERR_INVALID, "unknown Newton-Schulz precision"),
        (lambda: L.tk_apply_pointwise_peers(None, 0, _native.TK_ADAMW, ctypes.byref(hp), 1, None,
                                            None, 8, None),
         _native.TK_ERR_INVALID, "n_peers must be 0..7"),
        (lambda: L.tk_apply_pointwise_peers(None, 0, _native.TK_ADAMW, ctypes.byref(hp), 1, None,
                                            (I64 * 1)(8), 1, None),
         _native.TK_ERR_INVALID, "not a multiple of 16 bytes"),
        (lambda: L.tk_muon_step_peers(None, 0, ctypes.byref(mhp), (I64 * 1)(24), 1, None),
         _native.TK_ERR_INVALID, "not a multiple of 16 bytes"),
        (lambda: L.tk_muon_step_copy(None, 0, ctypes.byref(mhp), None, 2, None),
         _native.TK_ERR_INVALID, "with a delta for each"),
        (lambda: L.tk_set_reserved_sms(-1), _native.TK_ERR_INVALID, "out of range"),
        (lambda: L.tk_set_update_events(ctypes.c_void_p(16), None),
         _native.TK_ERR_INVALID, "set both events or neither"),
        (lambda: L.tk_ipc_close(ctypes.c_void_p(4096)),
         _native.TK_ERR_INVALID, "was not returned by tk_ipc_import"),
        (lambda: L.tk_shard_init(None, None, None, 16, None, None, 0, _native.TK_ADAMW, 0, None,
                                 ctypes.byref(ctypes.c_void_p())),
         _native.TK_ERR_INVALID, "null communicator or arena"),
        (lambda: L.tk_muon_shard_init(None, 0, None, None, None, _native.TK_BF16,
                                      ctypes.byref(mhp), 0, None,
                                      ctypes.byref(ctypes.c_void_p())),
         _native.TK_ERR_INVALID, "null communicator"),
        (lambda: L.tk_shard_step(None, ctypes.byref(hp), 1, 0.0, None, None),
         _native.TK_ERR_INVALID, "null shard"),
        (lambda: L.tk_nccl_comm_init(ctypes.c_void_p(16), 2, 2, ctypes.byref(ctypes.c_void_p())),
         _native.TK_ERR_INVALID, "rank 2 of world 2"),
        (lambda: L.tk_muon_layout(0, None, None, 0, None, None, None),
         _native.TK_ERR_INVALID, "world 0"),
        (lambda: L.tk_step_buffers_noalloc(None, 0, _native.TK_ADAMW, None, 1, 0.0, None, None),
         _native.TK_ERR_INVALID, "hparams is NULL"),
        (lambda: L.tk_nccl_comm_async_error(None, ctypes.byref(ctypes.c_int32())),
         _native.TK_ERR_INVALID, "null argument"),
        (lambda: L.tk_stream_wait_deadline(None, -1, None),
         _native.TK_ERR_INVALID, "negative timeout"),
        (lambda: L.tk_step_arena(None, ctypes.c_void_p(256), ctypes.c_void_p(256),
                                 ctypes.c_void_p(256), None, 1024, (ctypes.c_uint64 * 1)(0),
                                 (ctypes.c_uint64 * 1)(16), 1, _native.TK_ADAMW,
                                 ctypes.byref(hp), 1, None, None),
         _native.TK_ERR_INVALID, "null arena"),
        (lambda: L.tk_step_arena(None, ctypes.c_void_p(256), ctypes.c_void_p(256),
                                 ctypes.c_void_p(256), ctypes.c_void_p(256), 1024,
                                 (ctypes.c_uint64 * 1)(66), (ctypes.c_uint64 * 1)(4), 1,
                                 _native.TK_ADAMW, ctypes.byref(hp), 1, None, None),
         _native.TK_ERR_INVALID, "not a multiple of 4"),
        (lambda: L.tk_step_arena(None, ctypes.c_void_p(256), ctypes.c_void_p(256),
                                 ctypes.c_void_p(256), None, 1024,
                                 (ctypes.c_uint64 * 2)(0, 960), (ctypes.c_uint64 * 2)(16, 17), 2,
                                 _native.TK_LION, ctypes.byref(hp), 1, None, None),
         _native.TK_ERR_INVALID, "does not fit an arena of 1024 bytes"),
    ]
    for call, code, text in cases:
        status, msg = _err(call())
        assert status == code and text in msg, (status, msg, text)
        # the next successful call clears the message
        assert _err(L.tk_newton_schulz_2d(None, 0, 0, 5, _native.TK_F32, _native.TK_NS_F16,
                                          None)) == (0, "")
    # releasing nothing succeeds
    assert L.tk_shard_destroy(None, None) == 0
    assert L.tk_muon_shard_destroy(None, None) == 0
    assert L.tk_nccl_comm_destroy(None) == 0
    assert L.tk_nccl_comm_abort(None) == 0
    assert L.tk_set_reserved_sms(0) == 0


def test_muon_frontend_rejects_strided_parameters_before_any_launch():
    import torch

    from tikun_b200.muon import Muon

    p = torch.nn.Parameter(torch.zeros(6, 4).t())  # a transposed (strided) weight
    p.grad = torch.zeros_like(p)
    opt = Muon([p], lr=0.02)
    with pytest.raises(ValueError, match="contiguous"):
        opt.step()


def test_torch_optimizer_adamw_shape_needs_no_device():
    """tikun_b200.optimizer.AdamW keeps the reference's torch.optim.Optimizer
    shape (python/tikun/optimizer.py:17-117): param_groups defaults under the
    reference's keys, and a missing gradient raises before any native call."""
    import torch

    from tikun_b200.optimizer import AdamW

    w = torch.nn.Parameter(torch.zeros(3, 4))
    opt = AdamW([w], lr=2e-3, betas=(0.8, 0.99), eps=1e-7, weight_decay=0.1, max_norm=1.0)
    g = opt.param_groups[0]
    assert (g["lr"], g["beta_one"], g["beta_two"], g["eps"], g["weight_decay"], g["max_norm"]) == \
        (2e-3, 0.8, 0.99, 1e-7, 0.1, 1.0)
    assert isinstance(opt, torch.optim.Optimizer) and opt.step_count == 0
    with pytest.raises(RuntimeError, match=r"Gradient for parameter with shape torch.Size\(\[3, 4\]\) is None."):
        opt.step()
