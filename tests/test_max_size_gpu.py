"""A single leaf of 2^31 + 4099 f32 elements (4 x 8.6 GB of p, g, m, v):
element indices past 2^31 and a norm over more than 2^31 squares.

The clipped AdamW step runs through step_fast_buffers on the whole leaf.  The
clip scale must equal the reference rule applied to the f64 sum of squares
(lib.rs:79-125; torch's f64 sum has another order, so one f32 ulp is allowed).
Three slices -- the start, across element 2^31 and the end -- must match the
oracle's Tier 2 (lib.rs:143-272) bit for bit with that scale: the update is
element-wise, so the slices stand for the whole leaf."""
import numpy as np
import pytest
import torch

import oracle
from helpers import assert_bitexact
from tikun_b200 import _native

pytestmark = pytest.mark.gpu

N = (1 << 31) + 4099
SLICES = [(0, 4096), ((1 << 31) - 2048, (1 << 31) + 2048), (N - 4096, N)]
HP = dict(lr=1e-3, b1=0.9, b2=0.999, eps=1e-8, decay=0.01)


def test_leaf_beyond_two_to_the_31_elements():
    torch.cuda.empty_cache()  # memory cached by earlier tests in this process
    free, _ = torch.cuda.mem_get_info()
    if free < 4 * N * 4 + (4 << 30):
        pytest.skip("needs about 40 GB of free device memory")
    gen = torch.Generator(device="cuda").manual_seed(31)
    p = torch.randn(N, device="cuda", generator=gen).mul_(0.02)
    g = torch.randn(N, device="cuda", generator=gen).mul_(1e-2)
    m = torch.randn(N, device="cuda", generator=gen).mul_(1e-3)
    v = torch.rand(N, device="cuda", generator=gen).mul_(1e-5)
    try:
        before = [[t[a:b].cpu().numpy().copy() for t in (p, g, m, v)] for a, b in SLICES]
        scale = _native.step_fast_buffers([p.data_ptr()], [g.data_ptr()], [m.data_ptr()],
                                          [v.data_ptr()], [N], 1.0, "adamw", 3, HP["lr"],
                                          HP["b1"], HP["b2"], HP["eps"], HP["decay"])
        torch.cuda.synchronize()
        ss = 0.0
        for a in range(0, N, 1 << 28):
            ss += float(g[a:a + (1 << 28)].double().square().sum())
        want = oracle.clip_scale(ss, 1.0)
        assert want < 1.0  # the clip engaged
        assert abs(scale - want) <= np.spacing(np.float32(want)), (scale, want)
        for (a, b), (p0, g0, m0, v0) in zip(SLICES, before):
            oracle.pointwise_leaf(p0, g0, m0, v0, oracle.ADAMW, HP["lr"], HP["b1"], HP["b2"],
                                  HP["eps"], HP["decay"], 3, scale)
            assert_bitexact(p[a:b].cpu().numpy(), p0, f"p[{a}:{b}]")
            assert_bitexact(m[a:b].cpu().numpy(), m0, f"m[{a}:{b}]")
            assert_bitexact(v[a:b].cpu().numpy(), v0, f"v[{a}:{b}]")
    finally:
        del p, g, m, v
        torch.cuda.empty_cache()
