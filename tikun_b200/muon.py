"""Muon (2-D matrices) + AdamW (everything else) on the B200 engine.

Mirrors the reference's ``Muon`` (python/tikun/muon.py:34-102): the explicit
partition into ``muon_params`` and ``adamw_params``, EMA momentum without
Nesterov (muon.py:91), Newton-Schulz of the momentum, the update scaled by
sqrt(max(1, rows/cols)) (:97-98), and AdamW with betas (0.9, 0.95) and decay 0.1
by default for the rest (:45-48, :62-72).

The Newton-Schulz normalisation is the engine's (tensor_engine.rs:37-44:
divide by max(||X||, 1e-7)); the reference's torch restatement divides by
(||X|| + 1e-7), a difference of one part in 10^7 of the norm.  Momentum is
kept in f32 whatever the parameter type.
"""
from __future__ import annotations

import torch

from . import _native
from .muon_nd import MultiDimensionalMuon
from .universal import UniversalOptimizer, _tk_dtype


def zeropower_via_newtonschulz5(G: torch.Tensor, steps: int = 5, eps: float = 1e-7,
                                precision: int | None = None) -> torch.Tensor:
    """Polar factor of a 2-D CUDA tensor by the engine's Newton-Schulz
    (returns a new tensor of G's dtype)."""
    assert G.ndim == 2 and G.is_cuda
    X = G.detach().clone().contiguous()
    if X.dtype not in (torch.float32, torch.bfloat16):
        X = X.float()
    with torch.cuda.device(X.device):
        _native.newton_schulz_2d_ffi(X.data_ptr(), X.shape[0], X.shape[1], steps,
                                     dtype=_tk_dtype(X), precision=precision)
    return X.to(G.dtype)


class Muon(torch.optim.Optimizer):
    def __init__(self, muon_params, adamw_params=None, lr: float = 0.02, momentum: float = 0.95,
                 adamw_lr: float = 6e-4, adamw_betas: tuple = (0.9, 0.95), adamw_decay: float = 0.1,
                 precision: int | None = None):
        muon_params = list(muon_params)
        super().__init__(muon_params, dict(lr=lr, momentum=momentum))
        self.lr = lr
        self.momentum = momentum
        self.step_count = 0
        self.precision = _native.DEFAULT_NS_PRECISION if precision is None else precision
        self.state_momentum = [torch.zeros(p.shape, dtype=torch.float32, device=p.device)
                               for p in muon_params]
        self.adamw = None
        if adamw_params is not None:
            adamw_list = list(adamw_params)
            if adamw_list:
                self.adamw = UniversalOptimizer(adamw_list, algorithm="adamw", lr=adamw_lr,
                                                beta1=adamw_betas[0], beta2=adamw_betas[1],
                                                weight_decay=adamw_decay)

    @torch.no_grad()
    def step(self):
        """muon.py:79-102."""
        self.step_count += 1
        leaves = []
        for i, p in enumerate(self.param_groups[0]["params"]):
            if p.grad is None:
                continue
            if not (p.is_contiguous() and p.grad.is_contiguous()):
                raise ValueError("Muon parameters and gradients must be contiguous (the kernels "
                                 "take their first address and shape)")
            mom = self.state_momentum[i]
            leaves.append((p.data_ptr(), p.grad.data_ptr(), mom.data_ptr(), 1, p.shape[0],
                           p.shape[1], _tk_dtype(p), _tk_dtype(p.grad)))
        if leaves:
            _native.muon_step(leaves, self.lr, self.momentum, nesterov=False, ns_steps=5,
                              precision=self.precision)
        if self.adamw is not None:
            self.adamw.step()


__all__ = ["Muon", "MultiDimensionalMuon", "zeropower_via_newtonschulz5"]
