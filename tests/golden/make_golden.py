"""Regenerates the golden fixtures in this folder.

Run from the repository root in a container where the reference checkout is
present (this script is the only file that reads it; the fixtures it writes
travel with the repository):

    python tests/golden/make_golden.py /path/to/reference

Fixtures:

* ``adamw_torch_parity.npz`` — the reference's AdamW known-answer check
  (examples/verify_exact_math_parity.py:16-72): np.random.seed(42), n=10000
  randn params and one fixed randn gradient, torch.optim.AdamW(lr=0.01,
  betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01) for 10 steps.  Stores the
  torch params after steps 1, 2, 3, 5 and 10; the reference passes if it is within 1e-5
  absolute of torch at every step (:72).
* ``ns_reference_torch.npz`` — the reference's own torch Newton-Schulz
  (python/tikun/muon.py:10-32) on seeded matrices of several aspect ratios,
  plus the 768x768 orthogonality check of examples/test_muon_core.py:16-37.
* ``frontend_reference.npz`` — the reference's Python front-ends
  (python/tikun/__init__.py AdamW/Lion/SGD factories over UniversalOptimizer,
  and MuonND) stepped on small torch CPU PyTrees, with the native extension
  replaced by the oracle (oracle.native_stub()).  Pins the host-side
  orchestration: leaf flattening order, step counting, state handling, the
  Muon momentum/Nesterov/scale rule.
"""
from __future__ import annotations

import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

import oracle  # noqa: E402


def _import_reference(ref_root: str):
    sys.modules["_tikun"] = oracle.native_stub()
    sys.path.insert(0, os.path.join(ref_root, "python"))
    import tikun  # noqa: F401  (reference package)
    from tikun.muon import zeropower_via_newtonschulz5

    return tikun, zeropower_via_newtonschulz5


def adamw_torch_parity() -> dict:
    np.random.seed(42)
    n = 10000
    p_init = np.random.randn(n).astype(np.float32)
    g_init = np.random.randn(n).astype(np.float32)
    p_t = torch.tensor(p_init.copy(), requires_grad=True)
    p_t.grad = torch.tensor(g_init.copy())
    opt = torch.optim.AdamW([p_t], lr=0.01, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01)
    keep = (1, 2, 3, 5, 10)
    traj = []
    for step in range(1, 11):
        opt.step()
        if step in keep:
            traj.append(p_t.detach().numpy().copy())
    return {"p_init": p_init, "g": g_init, "steps": np.array(keep), "torch_p": np.stack(traj)}


def ns_reference(zp) -> dict:
    out = {}
    shapes = [(64, 96), (96, 64), (128, 128), (32, 200), (200, 32), (17, 45)]
    for i, (r, c) in enumerate(shapes):
        torch.manual_seed(100 + i)
        G = torch.randn(r, c, dtype=torch.float32) * 0.01
        X = zp(G, steps=5)
        out[f"ns_in_{r}x{c}"] = G.numpy().copy()
        out[f"ns_out_{r}x{c}"] = X.numpy().copy()
    torch.manual_seed(42)
    G = torch.randn(768, 768, dtype=torch.float32)
    X = zp(G, steps=5)
    I_approx = X @ X.T
    eye = torch.eye(768)
    out["ortho768_frob"] = np.float64(((I_approx - eye).norm() / eye.norm()).item())
    out["ortho768_diag_mean"] = np.float64(I_approx.diagonal().mean().item())
    return out


def _tree(seed: int):
    g = torch.Generator().manual_seed(seed)
    return {
        "w": torch.randn(48, 80, generator=g) * 0.02,
        "b": torch.zeros(80),
        "ln": torch.ones(37),
        "emb": torch.randn(4097, generator=g) * 0.02,
    }


def frontend_reference(tikun) -> dict:
    out = {}
    # Pointwise optimizers through UniversalOptimizer (tikun.AdamW/Lion/SGD).
    cases = {
        "adamw_clip": lambda ps: tikun.AdamW(ps, lr=1e-3, max_norm=1.0),
        "adamw": lambda ps: tikun.AdamW(ps, lr=1e-3),
        "lion": lambda ps: tikun.Lion(ps, lr=1e-4, max_norm=0.5),
        "sgd": lambda ps: tikun.SGD(ps, lr=1e-2, momentum=0.9, weight_decay=0.01),
    }
    for name, make in cases.items():
        tree = _tree(7)
        params = {k: v.clone().requires_grad_(True) for k, v in tree.items()}
        for k, v in params.items():
            out[f"{name}/init/{k}"] = v.detach().numpy().copy()
        opt = make(params)
        gg = torch.Generator().manual_seed(11)
        for s in range(3):
            for k, v in params.items():
                grad = torch.randn(v.shape, generator=gg) * (0.05 if name != "sgd" else 0.01)
                v.grad = grad
                out[f"{name}/grad{s}/{k}"] = grad.numpy().copy()
            opt.step()
        for k, v in params.items():
            out[f"{name}/final/{k}"] = v.detach().numpy().copy()

    # MuonND: 1-D -> AdamW (eps 1e-8, no clip), 2-D -> momentum/Nesterov + NS,
    # 3-D -> head-batched NS (python/tikun/muon_nd.py:94-160).
    g0 = torch.Generator().manual_seed(3)
    mparams = {
        "bias": torch.zeros(64),
        "w_wide": torch.randn(48, 80, generator=g0) * 0.02,
        "w_tall": torch.randn(96, 40, generator=g0) * 0.02,
        "heads": torch.randn(2, 16, 24, generator=g0) * 0.02,
    }
    mparams = {k: v.clone().requires_grad_(True) for k, v in mparams.items()}
    for k, v in mparams.items():
        out[f"muon_nd/init/{k}"] = v.detach().numpy().copy()
    opt = tikun.MuonND(mparams, lr=0.02, momentum=0.95, nesterov=True, ns_steps=5)
    gg = torch.Generator().manual_seed(5)
    for s in range(3):
        for k, v in mparams.items():
            grad = torch.randn(v.shape, generator=gg) * 1e-3
            v.grad = grad
            out[f"muon_nd/grad{s}/{k}"] = grad.numpy().copy()
        opt.step()
    for k, v in mparams.items():
        out[f"muon_nd/final/{k}"] = v.detach().numpy().copy()

    # In-backward AdamW (universal.py:97-137): each leaf steps from its
    # post-accumulate-grad hook, clip per leaf, step numbering read before
    # step() increments it.  The loss sum(w1^2) + sum(w2 * c2) has gradients
    # 2*w1 and c2, which every device computes exactly.
    g1 = torch.Generator().manual_seed(17)
    w1 = (torch.randn(37, generator=g1) * 0.5).requires_grad_(True)
    w2 = (torch.randn(5, 7, generator=g1) * 0.5).requires_grad_(True)
    c2 = torch.randn(5, 7, generator=g1)
    out["inbwd/init/w1"] = w1.detach().numpy().copy()
    out["inbwd/init/w2"] = w2.detach().numpy().copy()
    out["inbwd/c2"] = c2.numpy().copy()
    opt = tikun.AdamW([w1, w2], lr=1e-2, max_norm=1.0, in_backward=True)
    for _ in range(4):
        loss = (w1 * w1).sum() + (w2 * c2).sum()
        loss.backward()
        opt.step()
    out["inbwd/final/w1"] = w1.detach().numpy().copy()
    out["inbwd/final/w2"] = w2.detach().numpy().copy()

    # tikun.Muon (muon.py:34-102): EMA momentum without Nesterov, torch f32 NS,
    # scale sqrt(max(1, r/c)); AdamW (betas 0.9/0.95, decay 0.1) on the rest.
    g2 = torch.Generator().manual_seed(23)
    mw = (torch.randn(64, 96, generator=g2) * 0.02).requires_grad_(True)
    mt = (torch.randn(80, 48, generator=g2) * 0.02).requires_grad_(True)
    mb = torch.zeros(96).requires_grad_(True)
    for k, v in (("w", mw), ("t", mt), ("b", mb)):
        out[f"muon/init/{k}"] = v.detach().numpy().copy()
    opt = tikun.Muon(muon_params=[mw, mt], adamw_params=[mb], lr=0.02, momentum=0.95,
                     adamw_lr=1e-3)
    for s in range(3):
        for k, v in (("w", mw), ("t", mt), ("b", mb)):
            v.grad = torch.randn(v.shape, generator=g2) * 1e-3
            out[f"muon/grad{s}/{k}"] = v.grad.numpy().copy()
        opt.step()
    for k, v in (("w", mw), ("t", mt), ("b", mb)):
        out[f"muon/final/{k}"] = v.detach().numpy().copy()
    return out


def main(ref_root: str) -> None:
    tikun, zp = _import_reference(ref_root)
    np.savez_compressed(os.path.join(HERE, "adamw_torch_parity.npz"), **adamw_torch_parity())
    np.savez_compressed(os.path.join(HERE, "ns_reference_torch.npz"), **ns_reference(zp))
    np.savez_compressed(os.path.join(HERE, "frontend_reference.npz"), **frontend_reference(tikun))
    for f in sorted(os.listdir(HERE)):
        if f.endswith(".npz"):
            print(f, os.path.getsize(os.path.join(HERE, f)), "bytes")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py /path/to/reference")
    main(sys.argv[1])
