"""``torch.optim.Optimizer`` form of the fused AdamW step.

Mirrors the reference's ``tikun.optimizer.AdamW`` (python/tikun/optimizer.py:
17-117): the same constructor arguments and ``param_groups`` defaults
(``lr``, ``beta_one``, ``beta_two``, ``eps``, ``weight_decay``, ``max_norm``),
a step counter incremented on every ``step()``, ``step(closure)`` evaluating
the closure with gradients enabled and returning its loss, a ``RuntimeError``
naming the shape of a parameter whose gradient is missing, and every
parameter that requires a gradient stepped in one call with the first
group's hyperparameters (as the reference does).

Differences, on the device side:

* CUDA parameters keep their moments in device memory (``self.state[p]``
  holds ``m1`` and ``m2``, so ``state_dict()`` / ``load_state_dict()`` save
  and restore them) and step without a host synchronisation; the clip scale
  of the last step stays on the device in ``clip_scale``.  CPU parameters
  step synchronously through the same C ABI, staged through device memory.
* bf16 parameters and gradients are accepted (moments stay f32).
"""
from __future__ import annotations

import torch

from . import _native
from .universal import leaf_address


class AdamW(torch.optim.Optimizer):
    """python/tikun/optimizer.py:17-117 on the B200 engine."""

    def __init__(self, params, lr: float = 1e-3, betas: tuple[float, float] = (0.9, 0.999),
                 eps: float = 1e-8, weight_decay: float = 0.01, max_norm: float = 0.0):
        defaults = dict(lr=lr, beta_one=betas[0], beta_two=betas[1], eps=eps,
                        weight_decay=weight_decay, max_norm=max_norm)
        super().__init__(params, defaults)
        self.step_count = 0
        self.clip_scale = None

    def state_dict(self) -> dict:
        """torch's state (m1 and m2 per parameter) plus the step counter."""
        sd = super().state_dict()
        sd["step_count"] = self.step_count
        return sd

    def load_state_dict(self, state_dict: dict) -> None:
        sd = dict(state_dict)
        self.step_count = int(sd.pop("step_count", 0))
        super().load_state_dict(sd)
        # torch casts floating state to the parameter's dtype; the moments are f32
        for st in self.state.values():
            for k in ("m1", "m2"):
                if k in st:
                    st[k] = st[k].to(torch.float32).contiguous()

    def _stepped(self) -> list[torch.Tensor]:
        return [p for g in self.param_groups for p in g["params"] if p.requires_grad]

    def _moments(self, p: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        st = self.state[p]
        if "m1" not in st:
            st["m1"] = torch.zeros(p.numel(), dtype=torch.float32, device=p.device)
            st["m2"] = torch.zeros(p.numel(), dtype=torch.float32, device=p.device)
        return st["m1"], st["m2"]

    @torch.no_grad()
    def step(self, closure=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        self.step_count += 1
        group = self.param_groups[0]  # optimizer.py:81-88: the first group's values for all
        params = self._stepped()
        for p in params:
            if p.grad is None:
                raise RuntimeError(f"Gradient for parameter with shape {p.shape} is None.")
        if not params:
            return loss
        p_ptrs, g_ptrs, m1_ptrs, m2_ptrs, lengths = [], [], [], [], []
        p_dt, g_dt = [], []
        for p in params:
            m1, m2 = self._moments(p)
            ptr, n = leaf_address(p)
            p_ptrs.append(ptr)
            g_ptrs.append(leaf_address(p.grad)[0])
            m1_ptrs.append(m1.data_ptr())
            m2_ptrs.append(m2.data_ptr())
            lengths.append(n)
            p_dt.append(_native.TK_BF16 if p.dtype == torch.bfloat16 else _native.TK_F32)
            g_dt.append(_native.TK_BF16 if p.grad.dtype == torch.bfloat16 else _native.TK_F32)
        args = (p_ptrs, g_ptrs, m1_ptrs, m2_ptrs, lengths, group["max_norm"], "adamw",
                self.step_count, group["lr"], group["beta_one"], group["beta_two"], group["eps"],
                group["weight_decay"])
        devices = {p.device for p in params}
        if len(devices) == 1 and params[0].is_cuda:
            dev = params[0].device
            if self.clip_scale is None or not isinstance(self.clip_scale, torch.Tensor) or \
                    self.clip_scale.device != dev:
                self.clip_scale = torch.ones((), dtype=torch.float32, device=dev)
            with torch.cuda.device(dev):
                _native.step_fast_buffers_async(*args, clip_scale_ptr=self.clip_scale.data_ptr(),
                                                p_dtypes=p_dt, g_dtypes=g_dt)
        else:
            self.clip_scale = _native.step_fast_buffers(*args, p_dtypes=p_dt, g_dtypes=g_dt,
                                                        stream=0)
        return loss
