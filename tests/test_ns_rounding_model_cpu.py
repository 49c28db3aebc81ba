"""A CPU model of where the Newton-Schulz kernels round, checked against the
errors the B200 produced on the same inputs.

For m < 256 (or bf16 operands) one iteration of tikun_b200's Newton-Schulz is
three tensor-core GEMMs with 16-bit operands and f32 accumulation:

    A = round16(X X^T)
    B = round16(c (A A) + b A)          (the epilogue adds b A in f32)
    X = round16(B X + a X)              (the epilogue adds a X in f32)

with X = round16(x / ||x||) first (the f16 power-of-two pre-scale is exact
and changes nothing at these sizes) and the last iteration's f32 result as
the output.  The figures below are the relative Frobenius errors against the
oracle's f32 Newton-Schulz (crates/tikun-cpu/src/tensor_engine.rs:12-77) that
test_ns_gpu.py::test_ns_2d_matches_oracle measured on a B200 for these seeded
inputs; the model reproduces them to within 1 %, so a change of rounding
points can be judged on the CPU before it is built.
"""
import numpy as np
import pytest

import oracle

NS_A, NS_B, NS_C = 3.4445, -4.7750, 2.0315


def round16(x, fmt):
    x = np.asarray(x, np.float32)
    if fmt == "bf16":
        return oracle.bf16_to_f32(oracle.f32_to_bf16(x))
    return x.astype(np.float16).astype(np.float32)


def ns_model(x, fmt, steps=5):
    tall = x.shape[0] > x.shape[1]
    X = np.ascontiguousarray(x.T if tall else x)
    norm = max(np.sqrt(np.sum(X.astype(np.float64) ** 2)), 1e-7)
    X = round16(X / np.float32(norm), fmt)
    out = X
    for s in range(steps):
        A = round16(X @ X.T, fmt)
        B = round16(np.float32(NS_C) * (A @ A) + np.float32(NS_B) * A, fmt)
        out = (B @ X + np.float32(NS_A) * X).astype(np.float32)
        X = round16(out, fmt)
    return out.T if tall else out


# (rows, cols, operands) -> relative Frobenius error measured on a B200
MEASURED = {
    (1, 300, "f16"): 1.099e-3, (300, 1, "f16"): 3.268e-3, (1, 1, "f16"): 3.612e-3,
    (1, 300, "bf16"): 1.693e-2, (300, 1, "bf16"): 1.691e-2, (1, 1, "bf16"): 1.454e-2,
}


@pytest.mark.parametrize("rows,cols,fmt", sorted(MEASURED), ids=lambda v: str(v))
def test_model_reproduces_the_measured_error(rows, cols, fmt):
    # the inputs of test_ns_gpu.py::test_ns_2d_matches_oracle
    x = (np.random.default_rng(rows * 7 + cols).standard_normal((rows, cols)) * 0.01
         ).astype(np.float32)
    ref = oracle.polar_step_np(x, 5).astype(np.float64)
    got = ns_model(x, fmt).astype(np.float64)
    err = np.linalg.norm(got - ref) / np.linalg.norm(ref)
    assert abs(err - MEASURED[(rows, cols, fmt)]) <= 0.01 * MEASURED[(rows, cols, fmt)], err
