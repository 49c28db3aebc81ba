"""Framework-agnostic pointwise optimizer front-end on the B200 engine.

Mirrors the reference's ``UniversalOptimizer`` (python/tikun/universal.py:61-225):
same constructor arguments, PyTree flattening (dict values in insertion order,
lists, tuples, iterables, ``(ptr, len)`` pairs), per-parameter first/second
moment state keyed by the parameter's address, a step counter incremented at
the top of ``step()``, and the ``in_backward`` mode that steps each leaf from a
post-accumulate-grad hook.

Differences, all on the device side:
* CUDA tensors keep their moment state in device memory (the reference holds
  it in NumPy) and step without a host sync; the clip scale of the last step
  stays on the device in ``clip_scale``.
* bf16 parameters and gradients are accepted (updated in f32, rounded to
  nearest even on store); moments are f32.
* NumPy arrays and raw host ``(ptr, len)`` pairs step synchronously through the
  same C ABI, staged through device memory.
* ``arena=True`` (CUDA tensors of one dtype on one device) moves the
  parameters, their gradients and the moments into four flat device arenas
  laid out by LayoutPlan::from_shapes (the reference's MemoryArena and
  CpuLowering::step_arena, crates/tikun-core/src/arena.rs:34-103,
  crates/tikun-cpu/src/lib.rs:39-65): each parameter's ``.data`` and ``.grad``
  become views of their arenas, so autograd accumulates into the gradient
  arena, the leaf table is built once and every ``step()`` is one launch
  sequence over it, and ``zero_grad()`` clears the gradient arena in place
  (the gradients stay views, where the reference sets them to None).
"""
from __future__ import annotations

from typing import Any

import numpy as np

from . import _native


def _is_address_pair(x) -> bool:
    """An (address, length) pair of ints stands for one raw f32 buffer."""
    return isinstance(x, (tuple, list)) and len(x) == 2 and isinstance(x[0], int) \
        and isinstance(x[1], int)


def _is_container(x) -> bool:
    if isinstance(x, (dict, list, tuple)):
        return True
    # any other iterable except a tensor, an array or a string
    return hasattr(x, "__iter__") and not hasattr(x, "data_ptr") and \
        not isinstance(x, (str, bytes, np.ndarray))


def flatten_leaves(tree) -> list:
    """The leaves of a PyTree, in the order the reference's front-end steps them
    (python/tikun/universal.py:37-59): depth first, dict values in insertion
    order, list/tuple/iterable items in order; an (address, length) pair of
    ints is one leaf, and so is anything that is not a container."""
    leaves = []
    pending = [tree]
    while pending:
        node = pending.pop()
        if _is_address_pair(node) or not _is_container(node):
            leaves.append(node)
            continue
        children = list(node.values()) if isinstance(node, dict) else list(node)
        pending.extend(reversed(children))  # leftmost child next
    return leaves


def leaf_address(leaf) -> tuple[int, int]:
    """(address, element count) of one leaf.  Accepts what the reference's
    front-end accepts (python/tikun/universal.py:22-35): a tensor with
    data_ptr()/numel(), a NumPy array, anything with __array__ (a JAX array),
    or an (address, length) pair.  A strided tensor or array (a transposed
    weight, a slice with a step) is rejected: its first address and element
    count do not describe its elements, and the step would write the memory
    between them."""
    if hasattr(leaf, "data_ptr") and hasattr(leaf, "numel"):
        if hasattr(leaf, "is_contiguous") and not leaf.is_contiguous():
            raise ValueError("tikun_b200 steps contiguous tensors only; got a strided view of "
                             f"shape {tuple(leaf.shape)}")
        return leaf.data_ptr(), leaf.numel()
    if isinstance(leaf, np.ndarray) or hasattr(leaf, "__array__"):
        arr = leaf if isinstance(leaf, np.ndarray) else np.asarray(leaf)
        if not arr.flags.c_contiguous:
            raise ValueError("tikun_b200 steps contiguous arrays only; got a strided view of "
                             f"shape {arr.shape}")
        return arr.ctypes.data, arr.size
    if isinstance(leaf, (tuple, list)) and len(leaf) == 2 and isinstance(leaf[0], int):
        return int(leaf[0]), int(leaf[1])
    raise TypeError(f"cannot step a leaf of type {type(leaf).__name__}: expected a PyTorch "
                    "tensor, a JAX or NumPy array, or an (address, length) pair")


# the reference's names for the two helpers (its MuonND imports them from here)
_extract_pointer_and_len = leaf_address
_flatten_pytree = flatten_leaves


def _tk_dtype(t) -> int:
    dt = getattr(t, "dtype", None)
    if dt is None:
        return _native.TK_F32  # raw (ptr, len): f32 as in the reference
    name = str(dt)
    if name in ("torch.float32", "float32"):
        return _native.TK_F32
    if name in ("torch.bfloat16", "bfloat16"):
        return _native.TK_BF16
    raise TypeError(f"tikun_b200 leaves are float32 or bfloat16, got {dt}")


def _is_cuda(t) -> bool:
    return bool(getattr(t, "is_cuda", False))


class UniversalOptimizer:
    """See the module docstring; arguments as python/tikun/universal.py:67-78."""

    def __init__(self, params, algorithm: str = "adamw", lr: float = 1e-3, beta1: float = 0.9,
                 beta2: float = 0.999, eps: float = 1e-8, weight_decay: float = 0.01,
                 max_norm: float = 0.0, in_backward: bool = False, arena: bool = False):
        self.params = _flatten_pytree(params)
        self.algorithm = algorithm.lower()
        self.lr = lr
        self.beta1 = beta1
        self.beta2 = beta2
        self.eps = eps
        self.weight_decay = weight_decay
        self.max_norm = max_norm
        self.step_count = 0
        self.in_backward = in_backward
        self.m1_state: dict[int, Any] = {}
        self.m2_state: dict[int, Any] = {}
        self.clip_scale = None  # device f32 tensor (CUDA params) or float (host params)
        self._arena = None
        if arena:
            if in_backward:
                raise ValueError("arena mode steps every leaf at once; in_backward steps them "
                                 "one by one")
            self._arena = _ArenaState(self.params)
            for p, (m1, m2) in zip(self.params, self._arena.moments()):
                ptr, _ = _extract_pointer_and_len(p)
                self.m1_state[ptr], self.m2_state[ptr] = m1, m2
        if self.in_backward:
            self._hooks = []
            for p in self.params:
                if hasattr(p, "register_post_accumulate_grad_hook"):
                    self._hooks.append(p.register_post_accumulate_grad_hook(
                        self._make_in_backward_hook(p)))

    # -- state ---------------------------------------------------------------
    def _state_for(self, p, p_ptr: int, length: int):
        if p_ptr not in self.m1_state:
            if _is_cuda(p):
                import torch

                self.m1_state[p_ptr] = torch.zeros(length, dtype=torch.float32, device=p.device)
                self.m2_state[p_ptr] = torch.zeros(length, dtype=torch.float32, device=p.device)
            else:
                self.m1_state[p_ptr] = np.zeros(length, dtype=np.float32)
                self.m2_state[p_ptr] = np.zeros(length, dtype=np.float32)
        m1, m2 = self.m1_state[p_ptr], self.m2_state[p_ptr]
        return _extract_pointer_and_len(m1)[0], _extract_pointer_and_len(m2)[0]

    def _call(self, p_ptrs, g_ptrs, m1_ptrs, m2_ptrs, lengths, p_dt, g_dt, step, on_device,
              device=None):
        if on_device:
            import torch

            if self.clip_scale is None or self.clip_scale.device != device:
                self.clip_scale = torch.ones((), dtype=torch.float32, device=device)
            with torch.cuda.device(device):
                _native.step_fast_buffers_async(
                    p_ptrs, g_ptrs, m1_ptrs, m2_ptrs, lengths, self.max_norm, self.algorithm,
                    step, self.lr, self.beta1, self.beta2, self.eps, self.weight_decay,
                    clip_scale_ptr=self.clip_scale.data_ptr(), p_dtypes=p_dt, g_dtypes=g_dt)
        else:
            self.clip_scale = _native.step_fast_buffers(
                p_ptrs, g_ptrs, m1_ptrs, m2_ptrs, lengths, self.max_norm, self.algorithm, step,
                self.lr, self.beta1, self.beta2, self.eps, self.weight_decay, p_dtypes=p_dt,
                g_dtypes=g_dt, stream=0)

    # -- in-backward ---------------------------------------------------------
    def _make_in_backward_hook(self, p):
        def _hook(param):
            if param.grad is None:
                return
            self._step_single_tensor(param)
            param.grad = None

        return _hook

    def _step_single_tensor(self, p):
        """universal.py:112-137: one leaf, with step max(1, step_count) —
        the count is read before step() increments it, so the first two
        backward passes both use step 1, exactly as the reference does."""
        p_ptr, length = _extract_pointer_and_len(p)
        g_ptr, _ = _extract_pointer_and_len(p.grad)
        m1, m2 = self._state_for(p, p_ptr, length)
        self._call([p_ptr], [g_ptr], [m1], [m2], [length], [_tk_dtype(p)], [_tk_dtype(p.grad)],
                   max(1, self.step_count), _is_cuda(p), getattr(p, "device", None))

    # -- step ----------------------------------------------------------------
    def step(self, grads=None):
        """universal.py:139-192."""
        self.step_count += 1
        if self.in_backward:
            return
        if self._arena is not None:
            self._arena.step(self, grads)
            return
        p_ptrs, g_ptrs, m1_ptrs, m2_ptrs, lengths, p_dt, g_dt = [], [], [], [], [], [], []
        flat_grads = _flatten_pytree(grads) if grads is not None else None
        cuda_flags = []
        device = None
        for i, p in enumerate(self.params):
            p_ptr, length = _extract_pointer_and_len(p)
            if flat_grads is not None:
                g = flat_grads[i]
            elif hasattr(p, "grad") and p.grad is not None:
                g = p.grad
            else:
                continue
            g_ptr, _ = _extract_pointer_and_len(g)
            m1, m2 = self._state_for(p, p_ptr, length)
            p_ptrs.append(p_ptr)
            g_ptrs.append(g_ptr)
            m1_ptrs.append(m1)
            m2_ptrs.append(m2)
            lengths.append(length)
            p_dt.append(_tk_dtype(p))
            g_dt.append(_tk_dtype(g))
            cuda_flags.append(_is_cuda(p))
            if _is_cuda(p):
                device = p.device
        if not p_ptrs:
            return
        on_device = all(cuda_flags)
        self._call(p_ptrs, g_ptrs, m1_ptrs, m2_ptrs, lengths, p_dt, g_dt, self.step_count,
                   on_device, device)

    def zero_grad(self):
        if self._arena is not None:  # the gradients stay views of the arena
            self._arena.grads.flat.zero_()
            return
        for p in self.params:
            if hasattr(p, "grad") and p.grad is not None:
                p.grad = None

    # -- checkpoint / resume ---------------------------------------------------
    # The reference keeps m1/m2 keyed by raw pointers and never serialises them
    # (python/tikun/universal.py:93-95, 116-121); here they can be saved and
    # restored in parameter order, so a resumed run continues bit-identically.
    def state_dict(self) -> dict:
        """The step counter and copies of m1/m2 in parameter order (None for a
        parameter not stepped yet)."""
        m1, m2 = [], []
        for p in self.params:
            ptr, _ = _extract_pointer_and_len(p)
            if ptr in self.m1_state:
                a, b = self.m1_state[ptr], self.m2_state[ptr]
                m1.append(a.clone() if hasattr(a, "clone") else a.copy())
                m2.append(b.clone() if hasattr(b, "clone") else b.copy())
            else:
                m1.append(None)
                m2.append(None)
        return {"step": self.step_count, "m1": m1, "m2": m2}

    def load_state_dict(self, state: dict) -> None:
        """Restores state_dict() output onto this optimizer's parameters (same
        order and sizes)."""
        if len(state["m1"]) != len(self.params):
            raise ValueError(f"state holds {len(state['m1'])} parameters, the optimizer "
                             f"{len(self.params)}")
        self.step_count = int(state["step"])
        for p, a, b in zip(self.params, state["m1"], state["m2"]):
            if a is None:
                continue
            ptr, n = _extract_pointer_and_len(p)
            size = a.numel() if hasattr(a, "numel") else a.size
            if size != n:
                raise ValueError("state and parameter sizes differ")
            self._state_for(p, ptr, n)
            for dst, src in ((self.m1_state[ptr], a), (self.m2_state[ptr], b)):
                if hasattr(dst, "copy_"):
                    dst.copy_(src)
                else:
                    dst[...] = np.asarray(src)

    # -- inspection (python/tikun/universal.py:199-225) -------------------------
    def to_json(self) -> str:
        """The execution-plan report for these parameters, as the reference's
        to_json returns its emit_inspect text."""
        from .inspect import emit_inspect

        ptrs = [_extract_pointer_and_len(p)[0] for p in self.params]
        lens = [_extract_pointer_and_len(p)[1] for p in self.params]
        return emit_inspect(ptrs, lens, self.algorithm, self.max_norm, self.lr, self.beta1,
                            self.beta2, self.eps, self.weight_decay)

    def inspect(self):
        print(self.to_json())

    def to_mlir(self) -> str:
        raise NotImplementedError("the MLIR text emitter (crates/tikun-core/src/mlir.rs) is "
                                  "not part of the B200 lowering; see to_json()")


class _ArenaState:
    """Four flat device arenas (p and g in the parameters' dtype, m1 and m2 in
    f32) at LayoutPlan offsets, the parameters and gradients re-pointed into
    them, and the leaf table of the C ABI built once."""

    def __init__(self, params):
        import torch

        from .arena import Arena, LayoutPlan

        if not params:
            raise ValueError("arena mode needs at least one parameter")
        dtypes = {p.dtype for p in params if isinstance(p, torch.Tensor)}
        devices = {p.device for p in params if isinstance(p, torch.Tensor)}
        if (len(dtypes) != 1 or len(devices) != 1 or
                not all(isinstance(p, torch.Tensor) and p.is_cuda for p in params)):
            raise ValueError("arena mode takes CUDA tensors of one dtype on one device")
        dtype, self.device = dtypes.pop(), devices.pop()
        if dtype not in (torch.float32, torch.bfloat16):
            raise ValueError(f"arena leaves are float32 or bfloat16, got {dtype}")
        for p in params:
            leaf_address(p)  # contiguous only
        self.plan = LayoutPlan([p.numel() for p in params])
        self.params = Arena(self.plan, dtype=dtype, device=self.device)
        self.grads = Arena(self.plan, dtype=dtype, device=self.device)
        self.m1 = Arena(self.plan, device=self.device)
        self.m2 = Arena(self.plan, device=self.device)
        with torch.no_grad():
            for i, p in enumerate(params):
                view = self.params.leaf(i).view(p.shape)
                view.copy_(p)
                gview = self.grads.leaf(i).view(p.shape)
                if p.grad is not None:
                    gview.copy_(p.grad)
                p.data = view
                p.grad = gview
        dt = _tk_dtype(params[0])
        n = len(params)
        self.leaves, self.n = _native.make_leaves(
            self.params.ptrs(), self.grads.ptrs(), self.m1.ptrs(), self.m2.ptrs(),
            [p.numel() for p in params], [dt] * n, [dt] * n)
        self.scale = torch.ones((), dtype=torch.float32, device=self.device)
        self.n_params = n

    def moments(self):
        return [(self.m1.leaf(i), self.m2.leaf(i)) for i in range(self.n_params)]

    def step(self, opt, grads=None):
        import ctypes

        import torch

        if grads is not None:  # explicit gradients: copied into the arena first
            flat = flatten_leaves(grads)
            if len(flat) != self.n_params:
                raise ValueError(f"{len(flat)} gradients for {self.n_params} parameters")
            with torch.no_grad():
                for i, g in enumerate(flat):
                    self.grads.leaf(i).copy_(torch.as_tensor(g, device=self.device).reshape(-1))
        hp = _native.TkHParams(opt.lr, opt.beta1, opt.beta2, opt.eps, opt.weight_decay)
        with torch.cuda.device(self.device):
            _native.check(_native.lib().tk_step_buffers_async(
                self.leaves, self.n, _native.opt_kind(opt.algorithm), ctypes.byref(hp),
                opt.step_count, opt.max_norm if opt.max_norm > 0 else 0.0,
                self.scale.data_ptr(), torch.cuda.current_stream().cuda_stream))
        opt.clip_scale = self.scale
