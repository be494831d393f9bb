"""Optimizers over parameter slots: Adam, AdamW, SGD.

Mirrors ``tynx.optim`` (``crates/tynx-python/python/tynx/optim/__init__.py``) and the
native engines it wraps: ``AdamEngine::step_parameters``
(``crates/tynx-train/src/optimizer/adam.rs:431-527``, coupled L2 for Adam, decoupled
decay for AdamW at 502-507, AMSGrad) and ``Sgd::step_parameters``
(``crates/tynx-train/src/optimizer.rs:310-356``).  One step is one multi-tensor kernel
launch; tensors without a gradient are skipped (``adam.rs:439-441``) and duplicate
parameters are stepped once (``adam.rs:709-715``).  Step counters live on the device so
a captured step replays with the right bias corrections.
"""

from __future__ import annotations

import ctypes as C
from typing import Iterable, Optional, Union

import numpy as np

from .. import _native as N
from .._core import Tensor
from .._native import lib
from ..imported import Parameter

_KIND = {"adam": 0, "adamw": 1, "sgd": 2}


def _collect(parameters) -> list[Parameter]:
    items = list(parameters)
    if not items:
        raise ValueError("optimizer requires at least one Parameter")
    out: list[Parameter] = []
    seen: set[int] = set()
    for item in items:
        if isinstance(item, dict):
            raise NotImplementedError("parameter groups are not supported on the CUDA optimizer")
        p = item[1] if isinstance(item, tuple) else item
        if not isinstance(p, Parameter):
            raise TypeError(f"expected a Parameter, got {type(p).__qualname__}")
        if id(p) not in seen:
            seen.add(id(p))
            out.append(p)
    return out


class _Optimizer:
    _kind = "adam"

    def __init__(self, parameters, **options):
        self._params = _collect(parameters)
        ctx = self._params[0].ctx
        for p in self._params:
            if p.ctx is not ctx:
                raise ValueError("all parameters of one optimizer must live on the same device")
        self._ctx = ctx
        self._cfg = N.OptimCfg()
        self._cfg.kind = _KIND[self._kind]
        self._options = dict(options)
        self._apply_options()
        handle = C.c_void_p()
        n = len(self._params)
        values = N.ptr_array([p.ptr for p in self._params])
        grads = N.ptr_array([p._grad_ptr for p in self._params])
        numel = N.i64_array([p.numel for p in self._params])
        ctx.check(lib.tx_optim_create(ctx.handle, C.byref(self._cfg), n, values, grads, numel,
                                      C.byref(handle)), "optimizer")
        self._handle = handle
        self._synced = dict(self._options)

    def _apply_options(self) -> None:
        o = self._options
        c = self._cfg
        c.lr = float(o["lr"])
        if self._kind == "sgd":
            c.momentum = float(o.get("momentum", 0.0))
            c.dampening = float(o.get("dampening", 0.0))
            c.nesterov = int(bool(o.get("nesterov", False)))
            c.weight_decay = float(o.get("weight_decay", 0.0))
            if c.nesterov and (c.momentum <= 0 or c.dampening != 0):
                raise ValueError("nesterov momentum requires momentum > 0 and zero dampening")
        else:
            b1, b2 = o.get("betas", (0.9, 0.999))
            c.beta1, c.beta2 = float(b1), float(b2)
            c.eps = float(o.get("eps", 1e-8))
            c.weight_decay = float(o.get("weight_decay", 0.0 if self._kind == "adam" else 0.01))
            c.amsgrad = int(bool(o.get("amsgrad", False)))
            if not (0.0 <= c.beta1 < 1.0 and 0.0 <= c.beta2 < 1.0):
                raise ValueError("betas must be in [0, 1)")
        for key in ("lr", "weight_decay"):
            value = float(o.get(key, 0.0))
            if not np.isfinite(value) or value < 0:
                raise ValueError(f"{key} must be a non-negative finite number")

    @property
    def lr(self) -> float:
        return float(self._options["lr"])

    @lr.setter
    def lr(self, value: float) -> None:
        self._options["lr"] = float(value)

    learning_rate = lr

    @property
    def param_groups(self) -> list[dict]:
        group = dict(self._options)
        group["params"] = list(self._params)
        return [group]

    @property
    def parameter_count(self) -> int:
        return len(self._params)

    def zero_grad(self) -> None:
        for p in self._params:
            p.zero_grad()

    def _sync(self) -> None:
        if self._options != self._synced:
            self._apply_options()
            self._ctx.check(lib.tx_optim_set_hparams(self._handle, C.byref(self._cfg)))
            self._synced = dict(self._options)

    def step(self) -> None:
        self._sync()
        active = (C.c_uint8 * len(self._params))(*[int(p.grad_defined) for p in self._params])
        self._ctx.check(lib.tx_optim_step(self._handle, active), "optimizer step")

    def state_dict(self) -> dict:
        steps = (C.c_int64 * len(self._params))()
        self._ctx.check(lib.tx_optim_get_steps(self._handle, steps))
        state = {}
        slots = (("first_moment", 0), ("second_moment", 1)) if self._kind != "sgd" else \
            (("momentum", 3),) if self._cfg.momentum != 0 else ()
        if self._kind != "sgd" and self._cfg.amsgrad:
            slots = slots + (("max_second_moment", 2),)
        for i, p in enumerate(self._params):
            entry = {"step": int(steps[i])}
            for key, which in slots:
                ptr = C.c_void_p()
                self._ctx.check(lib.tx_optim_state_ptr(self._handle, i, which, C.byref(ptr)))
                host = np.empty(p.shape, np.float32)
                self._ctx.check(lib.tx_d2h(self._ctx.handle, host.ctypes.data, ptr.value, host.nbytes))
                entry[key] = host
            state[getattr(p, "name", str(i))] = entry
        return {"kind": self._kind, "options": dict(self._options), "state": state}

    def load_state_dict(self, state: dict) -> None:
        self._options.update(state.get("options", {}))
        self._sync()
        entries = state.get("state", {})
        steps = (C.c_int64 * len(self._params))()
        for i, p in enumerate(self._params):
            entry = entries.get(getattr(p, "name", str(i)))
            if entry is None:
                continue
            steps[i] = int(entry["step"])
            for key, which in (("first_moment", 0), ("second_moment", 1), ("max_second_moment", 2),
                               ("momentum", 3)):
                if key in entry:
                    ptr = C.c_void_p()
                    self._ctx.check(lib.tx_optim_state_ptr(self._handle, i, which, C.byref(ptr)))
                    host = np.ascontiguousarray(entry[key], dtype=np.float32)
                    self._ctx.check(lib.tx_h2d(self._ctx.handle, ptr.value, host.ctypes.data, host.nbytes))
        self._ctx.check(lib.tx_optim_set_steps(self._handle, steps))

    def __del__(self):
        try:
            if self._handle:
                lib.tx_optim_destroy(self._handle)
                self._handle = None
        except Exception:
            pass


class Adam(_Optimizer):
    _kind = "adam"

    def __init__(self, parameters, lr: float = 1e-3, betas=(0.9, 0.999), eps: float = 1e-8,
                 weight_decay: float = 0.0, amsgrad: bool = False):
        super().__init__(parameters, lr=lr, betas=tuple(betas), eps=eps, weight_decay=weight_decay,
                         amsgrad=amsgrad)


class AdamW(_Optimizer):
    _kind = "adamw"

    def __init__(self, parameters, lr: float = 1e-3, betas=(0.9, 0.999), eps: float = 1e-8,
                 weight_decay: float = 0.01, amsgrad: bool = False):
        super().__init__(parameters, lr=lr, betas=tuple(betas), eps=eps, weight_decay=weight_decay,
                         amsgrad=amsgrad)


class SGD(_Optimizer):
    _kind = "sgd"

    def __init__(self, parameters, lr: float, momentum: float = 0.0, dampening: float = 0.0,
                 weight_decay: float = 0.0, nesterov: bool = False):
        super().__init__(parameters, lr=lr, momentum=momentum, dampening=dampening,
                         weight_decay=weight_decay, nesterov=nesterov)


__all__ = ["Adam", "AdamW", "SGD"]
