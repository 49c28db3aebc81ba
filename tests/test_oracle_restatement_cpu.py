"""A second, independent restatement of tikun-cpu's x86 scalar update loops in
NumPy float32 (each operation rounded on its own, in the Rust source's order),
compared bit for bit with the C oracle.  The reference's own tests pin only
AdamW (against torch, to 1e-5); Lion and SGD-momentum rest on the restatement,
so two restatements written apart from each other must agree exactly.

Sources: AdamW crates/tikun-cpu/src/lib.rs:152-154 and :258-270, Lion
:347-358, SGD with momentum :419-427, the CustomDAG fallback rule :429-440;
clip scale :117-122; momentum is the b1 argument
(crates/tikun-py/src/lib.rs:201-205).
"""
import numpy as np
import pytest

import oracle

F = np.float32


def powi(a, n):
    # f32::powi by repeated squaring (the oracle's own copy is pinned in
    # test_oracle_pins.py; this one is written out again on purpose)
    r, a = F(1.0), F(a)
    while True:
        if n & 1:
            r = F(r * a)
        n >>= 1
        if n == 0:
            return r
        a = F(a * a)


def adamw(p, g, m, v, lr, b1, b2, eps, decay, step, scale):
    lr, b1, b2, eps, decay, scale = map(F, (lr, b1, b2, eps, decay, scale))
    one = F(1.0)
    bc1 = one - powi(b1, max(step, 1))
    bc2 = one - powi(b2, max(step, 1))
    g = g * scale
    m[:] = b1 * m + (one - b1) * g
    v[:] = b2 * v + ((one - b2) * g) * g
    m_hat = m / bc1
    v_hat = v / bc2
    upd = (m_hat / (np.sqrt(v_hat) + eps)) + (decay * p)
    p[:] = p - lr * upd


def lion(p, g, m, lr, b1, b2, decay, scale):
    lr, b1, b2, decay, scale = map(F, (lr, b1, b2, decay, scale))
    one = F(1.0)
    g = g * scale
    c = b1 * m + (one - b1) * g
    sign = np.where(c > 0, F(1.0), np.where(c < 0, F(-1.0), F(0.0))).astype(F)
    p[:] = p - lr * (sign + decay * p)
    m[:] = b2 * m + (one - b2) * g


def sgd(p, g, m, lr, mom, decay, scale):
    lr, mom, decay, scale = map(F, (lr, mom, decay, scale))
    g = g * scale
    m[:] = mom * m + g
    p[:] = p - lr * (m + decay * p)


def custom_dag(p, g, m, scale):
    g = g * F(scale)
    m[:] = F(0.9) * m + F(0.1) * g
    p[:] = p - F(1e-3) * m


def inputs(n, seed):
    rng = np.random.default_rng(seed)
    p = (rng.standard_normal(n) * 0.02).astype(F)
    g = (rng.standard_normal(n) * 0.05).astype(F)
    # special values: zeros of both signs, subnormals, large and tiny magnitudes
    special = np.array([0.0, -0.0, 1e-40, -1e-40, 1e-30, 3.0e4, -3.0e4, 1.0, -1.0], F)
    g[:len(special)] = special
    p[len(special):2 * len(special)] = special
    return p, g


@pytest.mark.parametrize("kind", ["adamw", "lion", "sgd", "custom"])
@pytest.mark.parametrize("scale", [1.0, 0.00897, 0.5])
def test_two_restatements_agree_bit_for_bit(kind, scale):
    n = 4099
    p, g = inputs(n, {"adamw": 1, "lion": 2, "sgd": 3, "custom": 4}[kind])
    m = np.zeros(n, F)
    v = np.zeros(n, F)
    pc, mc, vc = p.copy(), m.copy(), v.copy()
    hp = dict(lr=1e-3, b1=0.9, b2=0.999 if kind != "lion" else 0.99, eps=1e-8, decay=0.01)
    code = {"adamw": oracle.ADAMW, "lion": oracle.LION, "sgd": oracle.SGD,
            "custom": oracle.CUSTOM}[kind]
    for step in range(1, 6):
        gs = (g * F(1.0 + 0.1 * step)).astype(F)
        oracle.pointwise_leaf(pc, gs, mc, vc if kind == "adamw" else None, code, hp["lr"],
                              hp["b1"], hp["b2"], hp["eps"], hp["decay"], step, scale)
        if kind == "adamw":
            adamw(p, gs, m, v, hp["lr"], hp["b1"], hp["b2"], hp["eps"], hp["decay"], step, scale)
        elif kind == "lion":
            lion(p, gs, m, hp["lr"], hp["b1"], hp["b2"], hp["decay"], scale)
        elif kind == "sgd":
            sgd(p, gs, m, hp["lr"], hp["b1"], hp["decay"], scale)
        else:
            custom_dag(p, gs, m, scale)
        for a, b, name in ((pc, p, "p"), (mc, m, "m")) + (((vc, v, "v"),) if kind == "adamw" else ()):
            assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), (kind, step, name)


def test_step_zero_is_step_one():
    # crates/tikun-cpu/src/lib.rs:152: step_count.max(1)
    p, g = inputs(257, 9)
    m, v = np.zeros(257, F), np.zeros(257, F)
    p0, m0, v0 = p.copy(), m.copy(), v.copy()
    oracle.pointwise_leaf(p, g, m, v, oracle.ADAMW, 1e-3, 0.9, 0.999, 1e-8, 0.01, 0, 1.0)
    adamw(p0, g, m0, v0, 1e-3, 0.9, 0.999, 1e-8, 0.01, 1, 1.0)
    assert np.array_equal(p.view(np.uint32), p0.view(np.uint32))
