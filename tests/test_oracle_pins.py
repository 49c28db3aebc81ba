"""Pins the oracle against the reference's own known-answer checks.

* AdamW against torch.optim.AdamW over 10 steps, 1e-5 absolute: the reference's
  pass criterion in examples/verify_exact_math_parity.py:72.
* Newton-Schulz against the reference's torch restatement
  (python/tikun/muon.py:10-32) on seeded matrices.
* The 4x4 identity polar test (crates/tikun-cpu/src/tensor_engine.rs:198-210).
* LayoutPlan 64-byte alignment (crates/tikun-core/src/arena.rs:109-118).
* One AdamW step lowers p and raises m and v (crates/tikun-cpu/src/jit.rs:128-152).
"""
import os

import numpy as np
import pytest

import oracle


def test_powi_matches_repeated_squaring():
    for b in (0.9, 0.999, 0.95, 0.5):
        for step in (1, 2, 3, 7, 10, 100, 1000):
            ref = np.float32(1.0)
            a = np.float32(b)
            e = step
            while True:
                if e & 1:
                    ref = np.float32(ref * a)
                e >>= 1
                if e == 0:
                    break
                a = np.float32(a * a)
            assert oracle.powi(b, step) == float(ref)


def test_adamw_matches_torch_known_answer(golden_dir):
    z = np.load(os.path.join(golden_dir, "adamw_torch_parity.npz"))
    np.random.seed(42)
    p = np.random.randn(10000).astype(np.float32)
    g = np.random.randn(10000).astype(np.float32)
    assert np.array_equal(p, z["p_init"]) and np.array_equal(g, z["g"])
    m = np.zeros_like(p)
    v = np.zeros_like(p)
    k = 0
    for step in range(1, 11):
        oracle.step_two_tier([p], [g], [m], [v], oracle.ADAMW, 0.01, 0.9, 0.999, 1e-8, 0.01,
                             step, 0.0)
        if step in z["steps"]:
            diff = np.max(np.abs(p - z["torch_p"][k]))
            assert diff <= 1e-5, (step, diff)
            k += 1
    assert k == len(z["steps"])


@pytest.mark.parametrize("shape", [(64, 96), (96, 64), (128, 128), (32, 200), (200, 32), (17, 45)])
def test_ns_matches_reference_torch_ns(golden_dir, shape):
    z = np.load(os.path.join(golden_dir, "ns_reference_torch.npz"))
    r, c = shape
    x_in = z[f"ns_in_{r}x{c}"]
    ref = z[f"ns_out_{r}x{c}"].astype(np.float64)
    out_loops = oracle.polar_step(x_in.copy(), 5, nthreads=2).astype(np.float64)
    out_np = oracle.polar_step_np(x_in, 5).astype(np.float64)
    for out in (out_loops, out_np):
        rel = np.linalg.norm(out - ref) / np.linalg.norm(ref)
        assert rel < 1e-4, rel


def test_ns_orthogonality_known_answer(golden_dir):
    """examples/test_muon_core.py:16-37 on the oracle: the same relative
    Frobenius error of X X^T - I as the reference's torch NS produces."""
    import torch

    z = np.load(os.path.join(golden_dir, "ns_reference_torch.npz"))
    torch.manual_seed(42)
    G = torch.randn(768, 768, dtype=torch.float32).numpy()
    X = oracle.polar_step_np(G, 5).astype(np.float64)
    frob = np.linalg.norm(X @ X.T - np.eye(768)) / np.sqrt(768)
    assert abs(frob - float(z["ortho768_frob"])) < 1e-4 * max(1.0, float(z["ortho768_frob"]))


def test_polar_identity_4x4():
    mat = np.eye(4, dtype=np.float32)
    oracle.polar_step(mat, 5)
    gram = mat @ mat.T
    assert gram[0, 0] > 0.5


def test_polar_batched_shape():
    t = np.full((2, 4, 4), 0.5, dtype=np.float32)
    oracle.polar_batched(t, 5)
    assert t.shape == (2, 4, 4)


def test_layout_alignment():
    offs, total = oracle.layout_from_shapes([100, 513, 2048, 17])
    assert len(offs) == 4 and all(o % 64 == 0 for o in offs)
    assert offs == [0, 448, 2560, 10752] and total == 10752 + 68


def test_clip_scale_rule():
    # crates/tikun-cpu/src/lib.rs:117-122: scale only when the norm exceeds max_norm > 0
    assert oracle.clip_scale(4.0, 1.0) == np.float32(1.0) / (np.float32(2.0) + np.float32(1e-6))
    assert oracle.clip_scale(0.25, 1.0) == 1.0
    assert oracle.clip_scale(4.0, 0.0) == 1.0
    assert oracle.clip_scale(float("nan"), 1.0) == 1.0
    assert oracle.clip_scale(float("inf"), 1.0) == 0.0


def test_bf16_roundtrip_rne():
    x = np.array([1.0, 1.00390625, 1.01171875, -3.5, 1e-40, np.inf, -0.0], dtype=np.float32)
    h = oracle.f32_to_bf16(x)
    back = oracle.bf16_to_f32(h)
    assert back[0] == 1.0 and back[1] == 1.0 and back[2] == 1.015625 and back[3] == -3.5
    assert np.isinf(back[5]) and np.signbit(back[6])


def test_one_adamw_step_moves_p_down_and_moments_up():
    # crates/tikun-cpu/src/jit.rs:128-152: 16 ones, grads 0.1, one AdamW step at
    # lr 1e-3, betas 0.9/0.999, eps 1e-8, decay 0.01 -> p < 1, m > 0, v > 0.
    p = np.ones(16, np.float32)
    g = np.full(16, 0.1, np.float32)
    m = np.zeros(16, np.float32)
    v = np.zeros(16, np.float32)
    s = oracle.step_two_tier([p], [g], [m], [v], oracle.ADAMW, 1e-3, 0.9, 0.999, 1e-8, 0.01,
                             1, 0.0)
    assert s == 1.0
    assert np.all(p < 1.0) and np.all(m > 0.0) and np.all(v > 0.0)
    # first step of bias-corrected AdamW: m_hat = g, v_hat = g^2, so the step is
    # lr * (g / (|g| + eps) + decay * p) ~= 1e-3 * 1.01
    assert np.allclose(1.0 - p, 1e-3 * 1.01, rtol=1e-4)
