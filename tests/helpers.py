"""Shared helpers for the parity tests: leaves as torch CUDA tensors with numpy
copies for the oracle, and element-wise comparison with the stated bar."""
from __future__ import annotations

import numpy as np
import torch

import oracle
from tikun_b200 import _native

# AdamW / pointwise parity bar: max relative error <= 1e-6 per element,
# relative error |a - b| / max(|b|, 1e-30); the kernels aim for (and the tests
# also check) bit-identity with the oracle.
POINTWISE_RTOL = 1e-6


def to_np(t: torch.Tensor) -> np.ndarray:
    t = t.detach().contiguous().cpu()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16).copy()
    return t.numpy().copy()


def as_f32(a: np.ndarray) -> np.ndarray:
    return oracle.bf16_to_f32(a) if a.dtype == np.uint16 else a


def tk_dtype(t: torch.Tensor) -> int:
    return _native.TK_BF16 if t.dtype == torch.bfloat16 else _native.TK_F32


def assert_bitexact(gpu: np.ndarray, ref: np.ndarray, what: str = ""):
    gpu, ref = np.asarray(gpu), np.asarray(ref)
    assert gpu.shape == ref.shape and gpu.dtype == ref.dtype, what
    gb = gpu.view(np.uint16 if gpu.dtype == np.uint16 else np.uint32)
    rb = ref.view(np.uint16 if ref.dtype == np.uint16 else np.uint32)
    bad = np.flatnonzero(gb != rb)
    if bad.size:
        g32, r32 = as_f32(gpu).ravel(), as_f32(ref).ravel()
        nan_both = np.isnan(g32[bad]) & np.isnan(r32[bad])
        bad = bad[~nan_both]
    if bad.size:
        g32, r32 = as_f32(gpu).ravel(), as_f32(ref).ravel()
        rel = np.abs(g32 - r32) / np.maximum(np.abs(r32), 1e-30)
        i = bad[0]
        raise AssertionError(f"{what}: {bad.size} elements differ from the oracle; first at {i}: "
                             f"gpu={g32[i]!r} oracle={r32[i]!r}; max rel err {rel[bad].max():.3e}")


def max_rel_err(gpu: np.ndarray, ref: np.ndarray) -> float:
    g, r = as_f32(gpu).astype(np.float64).ravel(), as_f32(ref).astype(np.float64).ravel()
    if g.size == 0:
        return 0.0
    return float(np.max(np.abs(g - r) / np.maximum(np.abs(r), 1e-30)))


class Leaves:
    """A leaf table on the GPU plus numpy mirrors stepped by the oracle."""

    def __init__(self, sizes, p_dtypes=None, g_dtypes=None, seed=1234, device="cuda",
                 p_std=0.02, kind="adamw"):
        gen = torch.Generator(device="cpu").manual_seed(seed)
        self.kind = kind
        self.sizes = list(sizes)
        self.p, self.g, self.m, self.v = [], [], [], []
        p_dtypes = p_dtypes or [torch.float32] * len(sizes)
        self.g_dtypes = g_dtypes or [torch.float32] * len(sizes)
        for n, pdt in zip(sizes, p_dtypes):
            self.p.append((torch.randn(n, generator=gen) * p_std).to(pdt).to(device))
            self.m.append(torch.zeros(n, device=device))
            self.v.append(torch.zeros(n, device=device))
            self.g.append(torch.zeros(n, device=device, dtype=torch.float32))
        self.np_p = [to_np(t) for t in self.p]
        self.np_m = [to_np(t) for t in self.m]
        self.np_v = [to_np(t) for t in self.v]
        self.gen = gen

    def new_grads(self, std=1e-3):
        self.g = [(torch.randn(n, generator=self.gen) * std).to(gdt).to(self.p[0].device)
                  for n, gdt in zip(self.sizes, self.g_dtypes)]
        self.np_g = [to_np(t) for t in self.g]

    def gpu_step(self, step, max_norm, lr=1e-3, b1=0.9, b2=0.999, eps=1e-8, decay=0.01):
        return _native.step_fast_buffers(
            [t.data_ptr() for t in self.p], [t.data_ptr() for t in self.g],
            [t.data_ptr() for t in self.m], [t.data_ptr() for t in self.v],
            [t.numel() for t in self.p], max_norm, self.kind, step, lr, b1, b2, eps, decay,
            p_dtypes=[tk_dtype(t) for t in self.p], g_dtypes=[tk_dtype(t) for t in self.g])

    def oracle_step(self, step, max_norm, lr=1e-3, b1=0.9, b2=0.999, eps=1e-8, decay=0.01,
                    nthreads=8):
        return oracle.step_two_tier(self.np_p, self.np_g, self.np_m, self.np_v,
                                    oracle.opt_kind(self.kind), lr, b1, b2, eps, decay, step,
                                    max_norm, nthreads)

    def check(self, what=""):
        for i in range(len(self.sizes)):
            assert_bitexact(to_np(self.p[i]), self.np_p[i], f"{what} leaf {i} p")
            assert_bitexact(to_np(self.m[i]), self.np_m[i], f"{what} leaf {i} m")
            if self.kind == "adamw":
                assert_bitexact(to_np(self.v[i]), self.np_v[i], f"{what} leaf {i} v")


def gpt2_small_sizes(d=768, vocab=50257, ctx=1024, layers=12):
    """Leaf sizes of the GPT-2-small PyTree, in the order a state dict lists them:
    wte, wpe, per layer {ln1 w/b, c_attn W/b, attn c_proj W/b, ln2 w/b, c_fc W/b,
    mlp c_proj W/b}, ln_f w/b (148 leaves, 124,439,808 params at full size)."""
    sizes = [vocab * d, ctx * d]
    for _ in range(layers):
        sizes += [d, d, d * 3 * d, 3 * d, d * d, d, d, d, d * 4 * d, 4 * d, 4 * d * d, d]
    sizes += [d, d]
    return sizes


def gpt2_small_init(sizes, d, seed=1234, device="cuda"):
    """Params ~N(0, 0.02), biases 0, LayerNorm weights 1 (in that leaf order)."""
    gen = torch.Generator(device="cpu").manual_seed(seed)
    out = []
    n_layers = (len(sizes) - 4) // 12
    kinds = ["w", "w"] + ["ln_w", "b", "w", "b", "w", "b", "ln_w", "b", "w", "b", "w", "b"] * n_layers + ["ln_w", "b"]
    for n, k in zip(sizes, kinds):
        if k == "w":
            out.append((torch.randn(n, generator=gen) * 0.02).to(device))
        elif k == "ln_w":
            out.append(torch.ones(n, device=device))
        else:
            out.append(torch.zeros(n, device=device))
    return out


def spectrum_input(m, n, kind, seed):
    """An m x n matrix U diag(s) V^T * 1e-3 with orthonormal U, V and the singular
    values of `kind`: "steep" falls as exp(-8 i / m); "rank16" is 16 ones over a
    floor of 1e-3 (a few strong directions over noise, as momentum of real
    gradients tends to be)."""
    rng = np.random.default_rng(seed)
    U, _ = np.linalg.qr(rng.standard_normal((m, m)))
    V, _ = np.linalg.qr(rng.standard_normal((n, m)))
    if kind == "steep":
        s = np.exp(-np.arange(m) / (m / 8))
    else:
        s = np.r_[np.ones(16), np.full(m - 16, 1e-3)]
    return (U @ np.diag(s) @ V.T * 1e-3).astype(np.float32)
