"""Dimension-aware Muon on the B200 engine.

Mirrors the reference's ``MultiDimensionalMuon`` (python/tikun/muon_nd.py:14-160)
with the same constructor arguments and leaf partition:

* ndim < 2 (biases, norms): AdamW through ``step_fast_buffers`` with eps 1e-8 and
  no clipping (muon_nd.py:64-91);
* ndim == 2: momentum ``buf = mu*buf + (1-mu)*g``, Nesterov ``U = mu*buf +
  (1-mu)*g``, ``U = NS5(U)``, ``p -= lr*sqrt(max(1, rows/cols))*U``
  (muon_nd.py:94-126);
* ndim >= 3: the same per ``shape[-2] x shape[-1]`` head (muon_nd.py:129-160).

The 2-D and N-D leaves of one step go to ``tk_muon_step`` in one call: the
momentum update, the Newton-Schulz iteration on the tensor cores and the
parameter update are fused, and same-shape matrices are batched.  Parameters,
gradients and the f32 momentum state stay on the GPU.

``precision`` selects the Newton-Schulz operands: ``_native.TK_NS_F16`` (the
default), ``TK_NS_BF16``, ``TK_NS_F16X2`` (X as f16 pairs: momentum with a
few strong directions over a noise floor stays within 1.5e-3 of f32, at 1.4
to 1.5 times the f16 time) or ``TK_NS_F16X3`` (all operands as f16 pairs:
within a few 1e-6, for bf16 parameters held to 1e-3 over many steps, at 3
times).
"""
from __future__ import annotations

import math

import numpy as np

from . import _native
from .universal import UniversalOptimizer, _extract_pointer_and_len, _flatten_pytree, _tk_dtype


def _ndim(p) -> int:
    return getattr(p, "ndim", len(p.shape) if hasattr(p, "shape") else 1)


class MultiDimensionalMuon:
    def __init__(self, params, lr: float = 0.02, momentum: float = 0.95, nesterov: bool = True,
                 ns_steps: int = 5, adamw_lr: float = 1e-3, adamw_betas: tuple = (0.9, 0.999),
                 adamw_decay: float = 0.01, precision: int | None = None):
        self.raw_params = _flatten_pytree(params)
        self.lr = lr
        self.momentum = momentum
        self.nesterov = nesterov
        self.ns_steps = ns_steps
        self.adamw_lr = adamw_lr
        self.adamw_b1, self.adamw_b2 = adamw_betas
        self.adamw_decay = adamw_decay
        self.precision = _native.DEFAULT_NS_PRECISION if precision is None else precision
        self.step_count = 0
        self.rank_1_params, self.rank_2_params, self.rank_nd_params = [], [], []
        self.momentum_state = {}
        for p in self.raw_params:
            nd = _ndim(p)
            if nd < 2:
                self.rank_1_params.append(p)
            elif nd == 2:
                self.rank_2_params.append(p)
            else:
                self.rank_nd_params.append(p)
        # the 1-D leaves' AdamW state lives in a UniversalOptimizer
        self._adamw = UniversalOptimizer(self.rank_1_params, algorithm="adamw", lr=adamw_lr,
                                         beta1=self.adamw_b1, beta2=self.adamw_b2, eps=1e-8,
                                         weight_decay=adamw_decay, max_norm=0.0)

    def zero_grad(self):
        for p in self.raw_params:
            if hasattr(p, "grad") and p.grad is not None:
                p.grad = None

    def _muon_leaf(self, p):
        import torch

        if not getattr(p, "is_cuda", False):
            raise TypeError("the B200 Muon path takes CUDA tensors for 2-D and N-D parameters")
        p_ptr, _ = _extract_pointer_and_len(p)
        if p_ptr not in self.momentum_state:
            self.momentum_state[p_ptr] = torch.zeros(p.shape, dtype=torch.float32, device=p.device)
        mom = self.momentum_state[p_ptr]
        g = p.grad
        if not (p.is_contiguous() and g.is_contiguous()):
            raise ValueError("Muon leaves must be contiguous")
        shape = tuple(p.shape)
        heads = int(np.prod(shape[:-2])) if len(shape) > 2 else 1
        return (p_ptr, g.data_ptr(), mom.data_ptr(), heads, shape[-2], shape[-1], _tk_dtype(p),
                _tk_dtype(g))

    def step(self):
        """muon_nd.py:94-160."""
        self.step_count += 1
        # 1. 1-D leaves: AdamW (eps 1e-8, no clip) with this optimizer's step count
        if self.rank_1_params:
            self._adamw.step_count = self.step_count - 1
            self._adamw.step()
        # 2./3. 2-D and N-D leaves: one fused Muon call
        leaves = [self._muon_leaf(p) for p in self.rank_2_params + self.rank_nd_params
                  if getattr(p, "grad", None) is not None]
        if leaves:
            _native.muon_step(leaves, self.lr, self.momentum, self.nesterov, self.ns_steps,
                              self.precision)


def update_scale(rows: int, cols: int) -> float:
    """muon_nd.py:122: sqrt(max(1, rows/cols))."""
    return math.sqrt(max(1.0, rows / cols))
