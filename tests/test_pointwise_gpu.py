"""Parity of the CUDA Tier 1 / Tier 2 step with the oracle (tikun-cpu's x86
scalar arithmetic), through the reference-facing C ABI.

Bar: max relative error <= 1e-6 per element on p, m, v after 10 steps (stated
in helpers.POINTWISE_RTOL); the kernels are written to be bit-identical and the
tests check bit-identity.
"""
import ctypes
import os

import numpy as np
import pytest
import torch

import oracle
from helpers import (POINTWISE_RTOL, Leaves, assert_bitexact, gpt2_small_init, gpt2_small_sizes,
                     max_rel_err, to_np)
from tikun_b200 import _native

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("n", [1_000_003, 100_000_000], ids=["1e6+3", "flat-1e8-full"])
def test_flat_adamw_ten_steps_no_clip(n):
    """Flat-buffer AdamW, fresh N(0, 1e-3) grads each step, lr 1e-3, betas
    (0.9, 0.999), eps 1e-8, decay 0.01, no clip, 10 steps: the flat-leaf
    workload at its full 100,000,000 elements and at 1e6+3 (ragged tail)."""
    L = Leaves([n])
    for step in range(1, 11):
        L.new_grads(1e-3)
        s_gpu = L.gpu_step(step, 0.0)
        s_ref = L.oracle_step(step, 0.0)
        assert s_gpu == s_ref == 1.0
    L.check("flat adamw")
    assert max_rel_err(to_np(L.p[0]), L.np_p[0]) <= POINTWISE_RTOL


@pytest.mark.parametrize("scale_down", [True, False], ids=["d128", "gpt2-small-full"])
def test_gpt2_clipped_adamw(scale_down):
    """Clipped AdamW (global norm 1.0) over the GPT-2-small leaf table: 148
    leaves; grads N(0, 1e-2) so the clip triggers; 10 steps.  Full size is the
    124,439,808-parameter table."""
    d, vocab, ctx = (128, 1000, 256) if scale_down else (768, 50257, 1024)
    steps = 10
    sizes = gpt2_small_sizes(d=d, vocab=vocab, ctx=ctx)
    assert len(sizes) == 148
    if not scale_down:
        assert sum(sizes) == 124_439_808
    L = Leaves(sizes)
    L.p = gpt2_small_init(sizes, d)
    L.np_p = [to_np(t) for t in L.p]
    for step in range(1, steps + 1):
        L.new_grads(1e-2)
        s_gpu = L.gpu_step(step, 1.0)
        s_ref = L.oracle_step(step, 1.0)
        assert s_ref < 1.0, "clip must trigger"
        assert s_gpu == s_ref
    L.check("gpt2 clip")


@pytest.mark.parametrize("kind", ["adamw", "lion", "sgd"])
def test_mixed_dtypes_and_ragged_sizes(kind):
    sizes = [1, 3, 15, 17, 4097, 0, 65536 + 5, 777]
    pdt = [torch.float32, torch.bfloat16, torch.float32, torch.bfloat16, torch.bfloat16,
           torch.float32, torch.float32, torch.bfloat16]
    gdt = [torch.float32, torch.bfloat16, torch.bfloat16, torch.float32, torch.bfloat16,
           torch.float32, torch.float32, torch.bfloat16]
    L = Leaves(sizes, pdt, gdt, kind=kind)
    for step in range(1, 6):
        L.new_grads(0.05)
        kw = dict(lr=1e-2, b1=0.9, b2=0.99 if kind == "lion" else 0.999, decay=0.01)
        s_gpu = L.gpu_step(step, 0.5, **kw)
        s_ref = L.oracle_step(step, 0.5, **kw)
        assert s_gpu == s_ref
    L.check(kind)


def test_unaligned_views_take_the_scalar_path():
    base = [torch.randn(5000, device="cuda") * 0.02 for _ in range(4)]
    L = Leaves([4999, 4998])
    # offsets of 1 and 2 floats: not 16-byte aligned
    L.p = [base[0][1:], base[1][2:]]
    L.m = [torch.zeros(5000, device="cuda")[1:], torch.zeros(5000, device="cuda")[2:]]
    L.v = [torch.zeros(5001, device="cuda")[2:], torch.zeros(5001, device="cuda")[3:]]
    L.np_p = [to_np(t) for t in L.p]
    L.np_m = [to_np(t) for t in L.m]
    L.np_v = [to_np(t) for t in L.v]
    for step in range(1, 4):
        L.new_grads(1e-2)
        L.g = [torch.cat([torch.zeros(1, device="cuda"), g])[1:] for g in L.g]
        assert L.gpu_step(step, 1.0) == L.oracle_step(step, 1.0)
    L.check("unaligned")


def test_many_leaves_span_several_launches():
    rng = np.random.default_rng(0)
    sizes = [int(x) for x in rng.integers(1, 3000, size=500)]
    L = Leaves(sizes)
    for step in range(1, 4):
        L.new_grads(0.1)
        assert L.gpu_step(step, 1.0) == L.oracle_step(step, 1.0)
    L.check("500 leaves")


def test_nonfinite_gradients_follow_reference_clip_rule():
    for bad, want in ((float("nan"), 1.0), (float("inf"), 0.0)):
        L = Leaves([1000, 33])
        L.new_grads(0.1)
        L.g[0][17] = bad
        L.np_g[0][17] = bad
        s_gpu = L.gpu_step(1, 1.0)
        s_ref = L.oracle_step(1, 1.0)
        assert s_gpu == s_ref == want
        L.check(f"nonfinite {bad}")


def test_step_zero_is_clamped_to_one():
    L = Leaves([4096])
    L.new_grads()
    L.gpu_step(0, 0.0)
    L.oracle_step(0, 0.0)
    L.check("step 0")


def test_empty_call_returns_unit_scale():
    assert _native.step_fast_buffers([], [], [], [], [], 1.0, "adamw", 1, 1e-3, 0.9, 0.999,
                                     1e-8, 0.0) == 1.0


def test_host_buffers_are_staged():
    """numpy (pageable) leaves through the same entry point, as a caller of the
    CPU engine would pass them."""
    rng = np.random.default_rng(3)
    sizes = [10000, 17, 4096]
    p = [(rng.standard_normal(n) * 0.02).astype(np.float32) for n in sizes]
    m = [np.zeros(n, np.float32) for n in sizes]
    v = [np.zeros(n, np.float32) for n in sizes]
    rp, rm, rv = [x.copy() for x in p], [x.copy() for x in m], [x.copy() for x in v]
    for step in range(1, 4):
        g = [(rng.standard_normal(n) * 0.1).astype(np.float32) for n in sizes]
        s = _native.step_fast_buffers([a.ctypes.data for a in p], [a.ctypes.data for a in g],
                                      [a.ctypes.data for a in m], [a.ctypes.data for a in v],
                                      sizes, 1.0, "adamw", step, 1e-3, 0.9, 0.999, 1e-8, 0.01)
        r = oracle.step_two_tier(rp, g, rm, rv, oracle.ADAMW, 1e-3, 0.9, 0.999, 1e-8, 0.01,
                                 step, 1.0)
        assert s == r
    for a, b in zip(p + m + v, rp + rm + rv):
        assert_bitexact(a, b, "host")


@pytest.mark.parametrize("kind,max_norm", [("adamw", 1.0), ("adamw", 0.0), ("lion", 0.5)])
def test_pinned_host_buffers(kind, max_norm):
    """Pinned host leaves: the update kernel works on them in place over the
    host link (g is copied to the device first when clipping)."""
    sizes = [1 << 16, 17, 3000]
    p = [(torch.randn(n) * 0.02).pin_memory() for n in sizes]
    m = [torch.zeros(n).pin_memory() for n in sizes]
    v = [torch.zeros(n).pin_memory() for n in sizes]
    rp = [t.numpy().copy() for t in p]
    rm = [t.numpy().copy() for t in m]
    rv = [t.numpy().copy() for t in v]
    for step in (1, 2, 3):
        g = [(torch.randn(n) * 0.1).pin_memory() for n in sizes]
        s = _native.step_fast_buffers([t.data_ptr() for t in p], [t.data_ptr() for t in g],
                                      [t.data_ptr() for t in m], [t.data_ptr() for t in v], sizes,
                                      max_norm, kind, step, 1e-3, 0.9, 0.99, 1e-8, 0.01)
        r = oracle.step_two_tier(rp, [t.numpy().copy() for t in g], rm, rv, oracle.opt_kind(kind),
                                 1e-3, 0.9, 0.99, 1e-8, 0.01, step, max_norm)
        assert s == r
    for a, b in zip(p + m + v, rp + rm + rv):
        assert_bitexact(a.numpy(), b, "pinned")


@pytest.mark.parametrize("kind,max_norm", [("adamw", 1.0), ("sgd", 0.5), ("lion", 0.0)])
def test_pinned_host_many_small_leaves(kind, max_norm):
    """Small pinned leaves are gathered into one staging block with zero
    padding between them; ragged sizes and two large leaves around them must
    still match the oracle bit for bit, and no byte outside the leaves moves."""
    rng = np.random.default_rng(11)
    sizes = [int(x) for x in rng.integers(1, 5000, size=40)] + [70000, 1 << 17]
    sizes.insert(7, 65536)  # the largest staged size
    perm = rng.permutation(len(sizes))
    sizes = [sizes[i] for i in perm]
    adam = kind == "adamw"
    # one pinned buffer per array with guard words around every leaf
    def arena(fill):
        n = sum(sizes) + 8 * (len(sizes) + 1)
        t = torch.full((n,), fill, dtype=torch.float32).pin_memory()
        views, at = [], 8
        for k in sizes:
            views.append(t[at:at + k])
            at += k + 8
        return t, views
    P, p = arena(7.0)
    M, m = arena(7.0)
    V, v = arena(7.0)
    for t in p:
        t.copy_(torch.randn(t.numel()) * 0.02)
    for t in m + v:
        t.zero_()
    rp = [t.numpy().copy() for t in p]
    rm = [t.numpy().copy() for t in m]
    rv = [t.numpy().copy() for t in v]
    guard = [P.numpy().copy(), M.numpy().copy(), V.numpy().copy()]
    for step in (1, 2):
        g = [(torch.randn(n) * 0.05).pin_memory() for n in sizes]
        s = _native.step_fast_buffers([t.data_ptr() for t in p], [t.data_ptr() for t in g],
                                      [t.data_ptr() for t in m],
                                      [t.data_ptr() for t in v] if adam else [], sizes,
                                      max_norm, kind, step, 1e-3, 0.9, 0.99, 1e-8, 0.01)
        r = oracle.step_two_tier(rp, [t.numpy().copy() for t in g], rm, rv if adam else None,
                                 oracle.opt_kind(kind), 1e-3, 0.9, 0.99, 1e-8, 0.01, step,
                                 max_norm)
        assert s == r
    for a, b in zip(p + m + (v if adam else []), rp + rm + (rv if adam else [])):
        assert_bitexact(a.numpy(), b, "staged")
    # the guard words between the leaves are untouched
    for T, before in zip((P, M, V), guard):
        mask = np.ones(T.numel(), bool)
        at = 8
        for k in sizes:
            mask[at:at + k] = False
            at += k + 8
        np.testing.assert_array_equal(T.numpy()[mask], before[mask])


def test_rejects_aliased_leaves():
    t = torch.zeros(100, device="cuda")
    g = torch.zeros(100, device="cuda")
    m1, m2 = torch.zeros(100, device="cuda"), torch.zeros(100, device="cuda")
    w1, w2 = torch.zeros(100, device="cuda"), torch.zeros(100, device="cuda")
    with pytest.raises(ValueError, match="overlap"):
        _native.step_fast_buffers([t.data_ptr(), t.data_ptr()], [g.data_ptr(), g.data_ptr()],
                                  [m1.data_ptr(), m2.data_ptr()], [w1.data_ptr(), w2.data_ptr()],
                                  [100, 100], 0.0, "adamw", 1, 1e-3, 0.9, 0.999, 1e-8, 0.0)
    with pytest.raises(ValueError, match="overlap"):  # p overlaps its own m
        _native.step_fast_buffers([t.data_ptr()], [g.data_ptr()], [t.data_ptr() + 200],
                                  [w1.data_ptr()], [100], 0.0, "adamw", 1, 1e-3, 0.9, 0.999,
                                  1e-8, 0.0)


def test_adamw_without_second_moment_is_an_error():
    t, g, m = (torch.zeros(10, device="cuda") for _ in range(3))
    with pytest.raises(ValueError, match="second-moment"):
        _native.step_fast_buffers([t.data_ptr()], [g.data_ptr()], [m.data_ptr()], [], [10], 0.0,
                                  "adamw", 1, 1e-3, 0.9, 0.999, 1e-8, 0.0)
    # Lion and SGD take an empty m2 list (tikun-py/src/lib.rs:178)
    _native.step_fast_buffers([t.data_ptr()], [g.data_ptr()], [m.data_ptr()], [], [10], 0.0,
                              "sgd", 1, 1e-3, 0.9, 0.999, 1e-8, 0.0)


def test_mixed_host_and_device_is_an_error():
    t, m, v = (torch.zeros(10, device="cuda") for _ in range(3))
    g = np.zeros(10, np.float32)
    with pytest.raises(ValueError, match="mixed"):
        _native.step_fast_buffers([t.data_ptr()], [g.ctypes.data], [m.data_ptr()],
                                  [v.data_ptr()], [10], 0.0, "adamw", 1, 1e-3, 0.9, 0.999, 1e-8, 0.0)


def test_step_two_tier_runs_the_verifier():
    t, g, m, v = (torch.zeros(10, device="cuda") for _ in range(4))
    leaves, n = _native.make_leaves([t.data_ptr()], [g.data_ptr()], [m.data_ptr()],
                                    [v.data_ptr()], [10])
    nodes = (_native.TkScheduleNode * 1)(_native.TkScheduleNode(b"bad", 1, 65, 4, 8, 2))
    pl = _native.TkPipeline(nodes, 1, 0.0)
    hp = _native.TkHParams(1e-3, 0.9, 0.999, 1e-8, 0.0)
    out = ctypes.c_float()
    st = _native.lib().tk_step_two_tier(ctypes.byref(pl), leaves, n, 0, ctypes.byref(hp), 1,
                                        ctypes.byref(out), None)
    assert st == _native.TK_ERR_VERIFY
    assert _native.lib().tk_last_error().decode() == (
        'Static verification failed: [MisalignedCacheLine { node_name: "bad", tile_size: 65 }]')


def test_sharded_pieces_compose_to_the_full_step():
    """tk_grad_sumsq -> tk_clip_scale -> tk_apply_pointwise gives the same bits
    as tk_step_buffers (the ZeRO-1 path all-reduces the sum in between)."""
    sizes = [12345, 678, 90000]
    A = Leaves(sizes, seed=9)
    B = Leaves(sizes, seed=9)
    A.new_grads(0.1)
    B.g = [g.clone() for g in A.g]
    sA = A.gpu_step(1, 1.0)
    leaves, n = _native.make_leaves([t.data_ptr() for t in B.p], [t.data_ptr() for t in B.g],
                                    [t.data_ptr() for t in B.m], [t.data_ptr() for t in B.v],
                                    sizes)
    ss = torch.zeros(1, dtype=torch.float64, device="cuda")
    sc = torch.zeros(1, dtype=torch.float32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    L = _native.lib()
    _native.check(L.tk_grad_sumsq(leaves, n, ss.data_ptr(), stream))
    _native.check(L.tk_clip_scale(ss.data_ptr(), 1.0, sc.data_ptr(), stream))
    hp = _native.TkHParams(1e-3, 0.9, 0.999, 1e-8, 0.01)
    _native.check(L.tk_apply_pointwise(leaves, n, 0, ctypes.byref(hp), 1, sc.data_ptr(), stream))
    assert float(sc.item()) == sA
    ref_sum = sum(float(np.sum(t.astype(np.float64) ** 2)) for t in A.np_g)
    assert abs(float(ss.item()) - ref_sum) <= 1e-12 * ref_sum
    for a, b in zip(A.p + A.m + A.v, B.p + B.m + B.v):
        assert_bitexact(to_np(b), to_np(a), "sharded")


# -- front-end: the reference's Python optimizers on CUDA tensors ------------
@pytest.mark.parametrize("case", ["adamw_clip", "adamw", "lion", "sgd"])
def test_frontend_matches_reference_frontend(golden_dir, case):
    """tikun_b200.AdamW/Lion/SGD on CUDA tensors against the reference's own
    front-end (python/tikun/universal.py) run over the oracle: bit-identical."""
    import tikun_b200

    z = np.load(os.path.join(golden_dir, "frontend_reference.npz"))
    keys = ["w", "b", "ln", "emb"]
    params = {k: torch.tensor(z[f"{case}/init/{k}"], device="cuda", requires_grad=True)
              for k in keys}
    make = {
        "adamw_clip": lambda ps: tikun_b200.AdamW(ps, lr=1e-3, max_norm=1.0),
        "adamw": lambda ps: tikun_b200.AdamW(ps, lr=1e-3),
        "lion": lambda ps: tikun_b200.Lion(ps, lr=1e-4, max_norm=0.5),
        "sgd": lambda ps: tikun_b200.SGD(ps, lr=1e-2, momentum=0.9, weight_decay=0.01),
    }[case]
    opt = make(params)
    for s in range(3):
        for k in keys:
            params[k].grad = torch.tensor(z[f"{case}/grad{s}/{k}"], device="cuda")
        opt.step()
    torch.cuda.synchronize()
    for k in keys:
        assert_bitexact(to_np(params[k]), z[f"{case}/final/{k}"], f"{case}/{k}")


def test_inbackward_frontend_matches_reference(golden_dir):
    """In-backward AdamW (python/tikun/universal.py:97-137) on CUDA tensors:
    per-leaf steps from post-accumulate-grad hooks, per-leaf clip, and the
    reference's step numbering (the first two backward passes both use step 1).
    The loss has device-exact gradients, so the result must be bit-identical."""
    import tikun_b200

    z = np.load(os.path.join(golden_dir, "frontend_reference.npz"))
    w1 = torch.tensor(z["inbwd/init/w1"], device="cuda", requires_grad=True)
    w2 = torch.tensor(z["inbwd/init/w2"], device="cuda", requires_grad=True)
    c2 = torch.tensor(z["inbwd/c2"], device="cuda")
    opt = tikun_b200.AdamW([w1, w2], lr=1e-2, max_norm=1.0, in_backward=True)
    for _ in range(4):
        loss = (w1 * w1).sum() + (w2 * c2).sum()
        loss.backward()
        opt.step()
    torch.cuda.synchronize()
    assert w1.grad is None and w2.grad is None
    assert_bitexact(to_np(w1), z["inbwd/final/w1"], "w1")
    assert_bitexact(to_np(w2), z["inbwd/final/w2"], "w2")


def test_bulk_copy_kernel_opt_in():
    """The cp.async.bulk pipeline kernel (TIKUN_PW_BULK=1, read once per
    process) matches the oracle bit for bit on aligned and ragged f32 leaves;
    run in a child process so the switch is set before the library reads it."""
    import subprocess
    import sys
    import textwrap

    code = textwrap.dedent("""
        import sys, numpy as np, torch
        sys.path.insert(0, %r)
        import oracle
        from tikun_b200 import _native
        rng = np.random.default_rng(5)
        sizes = [1 << 20, 4099, 17, 3 * 1024 + 5, 1]
        hp = [(rng.standard_normal(n) * 0.02).astype(np.float32) for n in sizes]
        hm = [np.zeros(n, np.float32) for n in sizes]
        hv = [np.zeros(n, np.float32) for n in sizes]
        dp, dm, dv = ([torch.from_numpy(x).cuda() for x in a] for a in (hp, hm, hv))
        for step in (1, 2, 3):
            hg = [(rng.standard_normal(n) * 0.05).astype(np.float32) for n in sizes]
            dg = [torch.from_numpy(x).cuda() for x in hg]
            s = _native.step_fast_buffers([t.data_ptr() for t in dp], [t.data_ptr() for t in dg],
                                          [t.data_ptr() for t in dm], [t.data_ptr() for t in dv],
                                          sizes, 1.0, "adamw", step, 1e-3, 0.9, 0.999, 1e-8, 0.01)
            r = oracle.step_two_tier(hp, hg, hm, hv, oracle.ADAMW, 1e-3, 0.9, 0.999, 1e-8, 0.01,
                                     step, 1.0)
            assert s == r, (s, r)
        for d, h in zip(dp + dm + dv, hp + hm + hv):
            assert np.array_equal(d.cpu().numpy().view(np.uint32), h.view(np.uint32))
        assert _native.device_status() == 0
        print("bulk ok")
    """) % os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = dict(os.environ, TIKUN_PW_BULK="1")
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0 and "bulk ok" in r.stdout, r.stdout + r.stderr


def test_checkpoint_resume_is_bit_identical():
    """Save the optimizer state after 3 steps, restore it into a fresh
    optimizer over copies of the parameters, and take 2 more steps: the result
    equals 5 uninterrupted steps bit for bit."""
    import tikun_b200

    torch.manual_seed(3)
    shapes = [(64, 33), (17,), (4099,)]
    p0 = [torch.randn(*s, device="cuda") * 0.02 for s in shapes]
    grads = [[torch.randn(*s, device="cuda") * 1e-2 for s in shapes] for _ in range(5)]

    def run(params, opt, steps):
        for g in steps:
            for p, gg in zip(params, g):
                p.grad = gg.clone()
            opt.step()

    a = [t.clone() for t in p0]
    opt_a = tikun_b200.AdamW(a, lr=1e-3, max_norm=1.0)
    run(a, opt_a, grads)
    b = [t.clone() for t in p0]
    opt_b = tikun_b200.AdamW(b, lr=1e-3, max_norm=1.0)
    run(b, opt_b, grads[:3])
    saved = opt_b.state_dict()
    c = [t.clone() for t in b]
    opt_c = tikun_b200.AdamW(c, lr=1e-3, max_norm=1.0)
    opt_c.load_state_dict(saved)
    run(c, opt_c, grads[3:])
    torch.cuda.synchronize()
    for x, y in zip(a, c):
        assert torch.equal(x, y)
    assert "sm_100a" in opt_c.to_json()


def test_framework_agnostic_frontends_match_oracle():
    """examples/test_framework_agnostic.py:12-84 with assertions: a nested dict
    of NumPy arrays with grads passed to step (Lion), a bare NumPy array (SGD
    with momentum) and raw (pointer, length) leaves (AdamW) step through the
    host-buffer path and match the oracle bit for bit."""
    import tikun_b200

    def oracle_step(opt, ps, gs, m1, m2):
        return oracle.step_two_tier(ps, gs, m1, m2, oracle.opt_kind(opt.algorithm), opt.lr,
                                    opt.beta1, opt.beta2, opt.eps, opt.weight_decay,
                                    opt.step_count, opt.max_norm)

    rng = np.random.default_rng(9)
    # nested dict, Lion, grads given to step()
    params = {"encoder": {"w": np.ones((50, 50), np.float32), "b": np.zeros(50, np.float32)},
              "decoder": {"w": np.ones((50, 10), np.float32)}}
    leaves = [params["encoder"]["w"], params["encoder"]["b"], params["decoder"]["w"]]
    ref = [x.copy() for x in leaves]
    rm = [np.zeros(x.size, np.float32) for x in leaves]
    opt = tikun_b200.Lion(params, lr=1e-4)
    for _ in range(3):
        grads = {"encoder": {"w": rng.standard_normal((50, 50)).astype(np.float32) * 0.1,
                             "b": rng.standard_normal(50).astype(np.float32) * 0.05},
                 "decoder": {"w": rng.standard_normal((50, 10)).astype(np.float32) * 0.2}}
        opt.step(grads=grads)
        g = [grads["encoder"]["w"], grads["encoder"]["b"], grads["decoder"]["w"]]
        oracle_step(opt, [r.reshape(-1) for r in ref], [x.reshape(-1) for x in g], rm, None)
    for a, b in zip(leaves, ref):
        assert_bitexact(a, b, "dict/lion")
    # bare NumPy array, SGD with momentum
    p = np.ones(1000, np.float32)
    rp, rm1 = p.copy(), np.zeros(1000, np.float32)
    opt = tikun_b200.SGD(p, lr=0.01, momentum=0.9)
    for _ in range(3):
        g = rng.standard_normal(1000).astype(np.float32) * 0.05
        opt.step(grads=g)
        oracle_step(opt, [rp], [g], [rm1], None)
    assert_bitexact(p, rp, "numpy/sgd")
    # raw (pointer, length) leaves, AdamW
    p = np.ones(500, np.float32)
    rp, rm1, rm2 = p.copy(), np.zeros(500, np.float32), np.zeros(500, np.float32)
    opt = tikun_b200.AdamW([(p.ctypes.data, 500)], lr=1e-3)
    for _ in range(3):
        g = rng.standard_normal(500).astype(np.float32) * 0.1
        opt.step(grads=[(g.ctypes.data, 500)])
        oracle_step(opt, [rp], [g], [rm1], [rm2])
    assert_bitexact(p, rp, "raw/adamw")


# -- CustomDAG fallback rule and the arena-resident step ----------------------
def test_custom_dag_fallback_rule_matches_oracle():
    """PointwiseOp::CustomDAG (crates/tikun-cpu/src/lib.rs:429-440): the
    reference runs one fixed rule, m = 0.9 m + 0.1 g; p -= 1e-3 m, with g
    clip-scaled; bit-identical to the oracle over 5 clipped steps, mixed
    dtypes and ragged sizes, the second-moment buffers not passed."""
    sizes = [1, 3, 17, 4097, 65541, 0, 777]
    pdt = [torch.float32, torch.bfloat16, torch.float32, torch.bfloat16, torch.float32,
           torch.float32, torch.bfloat16]
    L = Leaves(sizes, pdt, pdt, seed=31)
    hp = _native.TkHParams(1e-3, 0.9, 0.999, 1e-8, 0.01)
    for step in range(1, 6):
        L.new_grads(0.05)
        leaves, n = _native.make_leaves(
            [t.data_ptr() for t in L.p], [t.data_ptr() for t in L.g], [t.data_ptr() for t in L.m],
            [], [t.numel() for t in L.p], [_native.TK_BF16 if t.dtype == torch.bfloat16 else
                                           _native.TK_F32 for t in L.p],
            [_native.TK_BF16 if t.dtype == torch.bfloat16 else _native.TK_F32 for t in L.g])
        out = ctypes.c_float()
        _native.check(_native.lib().tk_step_buffers(leaves, n, _native.TK_CUSTOM,
                                                    ctypes.byref(hp), step, 0.5,
                                                    ctypes.byref(out), None))
        ref = oracle.step_two_tier(L.np_p, L.np_g, L.np_m, [None] * len(sizes), oracle.CUSTOM,
                                   1e-3, 0.9, 0.999, 1e-8, 0.01, step, 0.5)
        assert out.value == ref
    for i in range(len(sizes)):
        assert_bitexact(to_np(L.p[i]), L.np_p[i], f"custom leaf {i} p")
        assert_bitexact(to_np(L.m[i]), L.np_m[i], f"custom leaf {i} m")


@pytest.mark.parametrize("kind", ["adamw", "lion"])
def test_step_arena_matches_oracle_and_leaves_padding_alone(kind):
    """CpuLowering::step_arena (crates/tikun-cpu/src/lib.rs:39-65) through
    tk_step_arena: four flat f32 device arenas at LayoutPlan::from_shapes
    offsets, the GPT-2-small table at d=128, 3 clipped steps bit-identical to
    the oracle stepping the same slots; the padding between slots keeps a NaN
    sentinel (it is never touched)."""
    from tikun_b200.arena import Arena, LayoutPlan

    d = 128
    sizes = gpt2_small_sizes(d=d, vocab=1000, ctx=256)
    offs, total_bytes = _native.layout_from_shapes(sizes)
    plan = LayoutPlan(sizes)
    P, G, M, V = (Arena(plan) for _ in range(4))
    P.flat.fill_(float("nan"))
    init = gpt2_small_init(sizes, d)
    for i, t in enumerate(init):
        P.leaf(i).copy_(t)
    np_p = [to_np(t) for t in init]
    np_m = [np.zeros(n, np.float32) for n in sizes]
    np_v = [np.zeros(n, np.float32) for n in sizes]
    gen = torch.Generator().manual_seed(3)
    hp = _native.TkHParams(1e-3, 0.9, 0.99 if kind == "lion" else 0.999, 1e-8, 0.01)
    code = oracle.opt_kind(kind)
    U64 = ctypes.c_uint64 * len(sizes)
    pipe = _native.TkPipeline((_native.TkScheduleNode * 3)(
        _native.TkScheduleNode(b"load_g", 0, 64, 4, 8, 2),
        _native.TkScheduleNode(b"fma_opt", 1, 64, 4, 8, 2),
        _native.TkScheduleNode(b"store_p", 2, 64, 4, 8, 2)), 3, 1.0)
    for step in range(1, 4):
        np_g = [(torch.randn(n, generator=gen) * 1e-2).numpy() for n in sizes]
        for i, g in enumerate(np_g):
            G.leaf(i).copy_(torch.from_numpy(g))
        out = ctypes.c_float()
        _native.check(_native.lib().tk_step_arena(
            ctypes.byref(pipe), P.flat.data_ptr(), G.flat.data_ptr(), M.flat.data_ptr(),
            V.flat.data_ptr(), P.flat.numel() * 4, U64(*offs), U64(*sizes), len(sizes),
            code, ctypes.byref(hp), step, ctypes.byref(out), None))
        ref = oracle.step_two_tier(np_p, np_g, np_m, np_v, code, 1e-3, 0.9,
                                   0.99 if kind == "lion" else 0.999, 1e-8, 0.01, step, 1.0)
        assert out.value == ref and ref < 1.0
    for i in range(len(sizes)):
        assert_bitexact(to_np(P.leaf(i)), np_p[i], f"slot {i} p")
        assert_bitexact(to_np(M.leaf(i)), np_m[i], f"slot {i} m")
    covered = torch.zeros(P.flat.numel(), dtype=torch.bool, device="cuda")
    for off, n in plan.slots:
        covered[off:off + n] = True
    assert torch.isnan(P.flat[~covered]).all(), "padding between slots was written"


def test_universal_optimizer_arena_mode_matches_oracle():
    """UniversalOptimizer(arena=True): parameters and gradients become views of
    flat device arenas, the leaf table is built once; 3 clipped AdamW steps over
    the GPT-2-small table at d=128 are bit-identical to the oracle, and
    zero_grad clears the gradient arena in place."""
    import tikun_b200

    d = 128
    sizes = gpt2_small_sizes(d=d, vocab=1000, ctx=256)
    params = [t.clone().requires_grad_(True) for t in gpt2_small_init(sizes, d)]
    np_p = [to_np(t) for t in params]
    np_m = [np.zeros(n, np.float32) for n in sizes]
    np_v = [np.zeros(n, np.float32) for n in sizes]
    opt = tikun_b200.AdamW(params, lr=1e-3, weight_decay=0.01, max_norm=1.0, arena=True)
    base = opt._arena.params.flat.data_ptr()
    span = opt._arena.params.flat.numel() * 4
    assert all(base <= p.data_ptr() < base + span for p in params)
    grad_ptrs = [p.grad.data_ptr() for p in params]
    gen = torch.Generator().manual_seed(5)
    for step in range(1, 4):
        np_g = [(torch.randn(n, generator=gen) * 1e-2).numpy() for n in sizes]
        with torch.no_grad():
            for p, g in zip(params, np_g):
                p.grad.copy_(torch.from_numpy(g))
        opt.step()
        ref = oracle.step_two_tier(np_p, np_g, np_m, np_v, oracle.ADAMW, 1e-3, 0.9, 0.999,
                                   1e-8, 0.01, step, 1.0)
        assert float(opt.clip_scale) == ref and ref < 1.0
    for i, p in enumerate(params):
        assert_bitexact(to_np(p.detach()), np_p[i], f"leaf {i} p")
        assert_bitexact(to_np(opt.m2_state[p.data_ptr()]), np_v[i], f"leaf {i} v")
    opt.zero_grad()
    assert [p.grad.data_ptr() for p in params] == grad_ptrs
    assert all(int(torch.count_nonzero(p.grad)) == 0 for p in params)


def test_arena_mode_gradients_accumulate_into_the_arena():
    """With the gradients as arena views, autograd accumulates into them in
    place: a small MLP trained 3 steps with the arena front-end ends
    bit-identical to the same model stepped by the per-leaf front-end."""
    import tikun_b200

    torch.manual_seed(0)
    net_a = torch.nn.Sequential(torch.nn.Linear(64, 96), torch.nn.ReLU(),
                                torch.nn.Linear(96, 10)).cuda()
    net_b = torch.nn.Sequential(torch.nn.Linear(64, 96), torch.nn.ReLU(),
                                torch.nn.Linear(96, 10)).cuda()
    net_b.load_state_dict(net_a.state_dict())
    opt_a = tikun_b200.AdamW(list(net_a.parameters()), lr=1e-2, arena=True)
    opt_b = tikun_b200.AdamW(list(net_b.parameters()), lr=1e-2)
    ptrs = [p.grad.data_ptr() for p in net_a.parameters()]
    x = torch.randn(32, 64, device="cuda")
    for _ in range(3):
        opt_a.zero_grad()
        opt_b.zero_grad()
        net_a(x).square().mean().backward()
        net_b(x).square().mean().backward()
        assert [p.grad.data_ptr() for p in net_a.parameters()] == ptrs
        opt_a.step()
        opt_b.step()
    for pa, pb in zip(net_a.parameters(), net_b.parameters()):
        assert torch.equal(pa.detach(), pb.detach())


def test_torch_optimizer_adamw_matches_oracle_and_resumes():
    """tikun_b200.optimizer.AdamW (the reference's torch.optim.Optimizer
    wrapper, python/tikun/optimizer.py:17-117): 3 clipped steps driven through
    step(closure) bit-identical to the oracle; state_dict() after 2 steps,
    loaded into a fresh optimizer, continues bit-identically."""
    from tikun_b200.optimizer import AdamW

    sizes = [4099, 768, 1, 65536]
    gen = torch.Generator().manual_seed(17)
    init = [(torch.randn(n, generator=gen) * 0.02) for n in sizes]
    params = [torch.nn.Parameter(t.clone().cuda()) for t in init]
    np_p = [t.numpy().copy() for t in init]
    np_m = [np.zeros(n, np.float32) for n in sizes]
    np_v = [np.zeros(n, np.float32) for n in sizes]
    opt = AdamW(params, lr=1e-3, weight_decay=0.01, max_norm=1.0)
    grads = [[(torch.randn(n, generator=gen) * 0.05) for n in sizes] for _ in range(3)]
    saved = None
    for step in range(1, 4):
        def closure():
            for p, g in zip(params, grads[step - 1]):
                p.grad = g.cuda()
            return torch.tensor(float(step))
        loss = opt.step(closure)
        assert float(loss) == step
        ref = oracle.step_two_tier(np_p, [g.numpy() for g in grads[step - 1]], np_m, np_v,
                                   oracle.ADAMW, 1e-3, 0.9, 0.999, 1e-8, 0.01, step, 1.0)
        assert float(opt.clip_scale) == ref
        if step == 2:
            import copy

            saved = (copy.deepcopy(opt.state_dict()), [p.detach().clone() for p in params])
    for i, p in enumerate(params):
        assert_bitexact(to_np(p.detach()), np_p[i], f"leaf {i} p")
    # resume from the step-2 checkpoint
    state, p2 = saved
    params_b = [torch.nn.Parameter(t.clone()) for t in p2]
    opt_b = AdamW(params_b, lr=1e-3, weight_decay=0.01, max_norm=1.0)
    opt_b.load_state_dict(state)
    assert opt_b.step_count == 2
    for p, g in zip(params_b, grads[2]):
        p.grad = g.cuda()
    opt_b.step()
    for a, b in zip(params, params_b):
        assert torch.equal(a.detach(), b.detach())


def test_step_arena_over_host_arenas():
    """The reference's MemoryArena is host memory (a Vec<f32>,
    crates/tikun-core/src/arena.rs:69-80): tk_step_arena over four NumPy
    arenas (staged through the device by the engine) gives the oracle's bytes
    for every slot, over 3 clipped AdamW steps, and leaves the padding alone."""
    sizes = [100, 513, 2048, 17, 4099]  # the reference's own alignment-test shapes and more
    offs, total_bytes = _native.layout_from_shapes(sizes)
    n_el = (total_bytes + 3) // 4
    rng = np.random.default_rng(77)
    P = np.full(n_el, np.nan, np.float32)
    G = np.zeros(n_el, np.float32)
    M = np.zeros(n_el, np.float32)
    V = np.zeros(n_el, np.float32)
    for o, n in zip(offs, sizes):
        P[o // 4:o // 4 + n] = rng.standard_normal(n).astype(np.float32) * 0.02
    ref_p = [P[o // 4:o // 4 + n].copy() for o, n in zip(offs, sizes)]
    ref_m = [np.zeros(n, np.float32) for n in sizes]
    ref_v = [np.zeros(n, np.float32) for n in sizes]
    hp = _native.TkHParams(1e-3, 0.9, 0.999, 1e-8, 0.01)
    U64 = ctypes.c_uint64 * len(sizes)
    pipe = _native.TkPipeline((_native.TkScheduleNode * 3)(
        _native.TkScheduleNode(b"load_g", 0, 64, 4, 8, 2),
        _native.TkScheduleNode(b"fma_opt", 1, 64, 4, 8, 2),
        _native.TkScheduleNode(b"store_p", 2, 64, 4, 8, 2)), 3, 1.0)
    for step in range(1, 4):
        g = [(rng.standard_normal(n) * 0.1).astype(np.float32) for n in sizes]
        for (o, n), gi in zip(zip(offs, sizes), g):
            G[o // 4:o // 4 + n] = gi
        out = ctypes.c_float()
        _native.check(_native.lib().tk_step_arena(
            ctypes.byref(pipe), P.ctypes.data, G.ctypes.data, M.ctypes.data, V.ctypes.data,
            n_el * 4, U64(*offs), U64(*sizes), len(sizes), _native.TK_ADAMW, ctypes.byref(hp),
            step, ctypes.byref(out), None))
        ref = oracle.step_two_tier(ref_p, g, ref_m, ref_v, oracle.ADAMW, 1e-3, 0.9, 0.999, 1e-8,
                                   0.01, step, 1.0)
        assert out.value == ref and ref < 1.0
    covered = np.zeros(n_el, bool)
    for i, (o, n) in enumerate(zip(offs, sizes)):
        assert_bitexact(P[o // 4:o // 4 + n], ref_p[i], f"slot {i} p")
        assert_bitexact(V[o // 4:o // 4 + n], ref_v[i], f"slot {i} v")
        covered[o // 4:o // 4 + n] = True
    assert np.isnan(P[~covered]).all(), "padding between slots was written"


def test_arena_mode_bf16_parameters_match_per_leaf_front_end():
    """UniversalOptimizer(arena=True) with bf16 parameters and gradients: the
    arenas are bf16 for p and g, f32 for the moments; 3 clipped steps give the
    same bytes as the per-leaf front-end."""
    import tikun_b200

    gen = torch.Generator().manual_seed(9)
    sizes = [(768, 64), (64,), (1000, 3), (5,)]
    init = [(torch.randn(*s, generator=gen) * 0.02).bfloat16() for s in sizes]
    pa = [t.clone().cuda().requires_grad_(True) for t in init]
    pb = [t.clone().cuda().requires_grad_(True) for t in init]
    oa = tikun_b200.AdamW(pa, lr=1e-2, max_norm=0.5, arena=True)
    ob = tikun_b200.AdamW(pb, lr=1e-2, max_norm=0.5)
    for _ in range(3):
        grads = [(torch.randn(*s, generator=gen) * 0.1).bfloat16().cuda() for s in sizes]
        with torch.no_grad():
            for p, g in zip(pa, grads):
                p.grad.copy_(g)
        for p, g in zip(pb, grads):
            p.grad = g.clone()
        oa.step()
        ob.step()
    torch.cuda.synchronize()
    assert float(oa.clip_scale) == float(ob.clip_scale) < 1.0
    for a, b in zip(pa, pb):
        assert torch.equal(a.detach().view(torch.int16), b.detach().view(torch.int16))
