"""tikun_b200 — the tikun optimizer-step hot path on B200 (sm_100a).

Front-ends with the reference's names and arguments (python/tikun/__init__.py):
``Optimizer`` (UniversalOptimizer), ``AdamW``, ``Lion``, ``SGD``, ``Muon`` and
``MuonND`` (MultiDimensionalMuon).  The native
entry points of the reference's ``_tikun`` module are in ``tikun_b200._native``.
"""
from .universal import UniversalOptimizer as Optimizer
from .universal import UniversalOptimizer
from .muon_nd import MultiDimensionalMuon as MuonND
from .muon_nd import MultiDimensionalMuon


def AdamW(params, lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01, max_norm=0.0,
          in_backward=False, arena=False):
    """python/tikun/__init__.py:7-8 (``arena``: see UniversalOptimizer)."""
    return Optimizer(params, algorithm="adamw", lr=lr, beta1=betas[0], beta2=betas[1], eps=eps,
                     weight_decay=weight_decay, max_norm=max_norm, in_backward=in_backward,
                     arena=arena)


def Lion(params, lr=1e-4, betas=(0.9, 0.99), weight_decay=0.01, max_norm=0.0, in_backward=False,
         arena=False):
    """python/tikun/__init__.py:10-11 (``arena``: see UniversalOptimizer)."""
    return Optimizer(params, algorithm="lion", lr=lr, beta1=betas[0], beta2=betas[1],
                     weight_decay=weight_decay, max_norm=max_norm, in_backward=in_backward,
                     arena=arena)


def SGD(params, lr=1e-2, momentum=0.9, weight_decay=0.0, max_norm=0.0, in_backward=False,
        arena=False):
    """python/tikun/__init__.py:13-14 (``arena``: see UniversalOptimizer)."""
    return Optimizer(params, algorithm="sgd", lr=lr, beta1=momentum, weight_decay=weight_decay,
                     max_norm=max_norm, in_backward=in_backward, arena=arena)


def __getattr__(name):
    # Muon subclasses torch.optim.Optimizer: import torch only when it is asked for
    if name in ("Muon", "zeropower_via_newtonschulz5"):
        from . import muon

        return getattr(muon, name)
    raise AttributeError(name)


__all__ = ["Optimizer", "UniversalOptimizer", "AdamW", "Lion", "SGD", "Muon", "MuonND",
           "MultiDimensionalMuon", "zeropower_via_newtonschulz5"]
