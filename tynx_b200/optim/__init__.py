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


def _collect(parameters) -> tuple[list[Parameter], Optional[list[str]]]:
    """Unique parameters in first-occurrence order, and their names when the
    optimizer was built from ``named_parameters()`` (the names key its state
    dictionary, ``crates/tynx-python/src/optimizer.rs:208-217``)."""
    items = list(parameters)
    if not items:
        raise ValueError("optimizer requires at least one Parameter")
    out: list[Parameter] = []
    names: list[str] = []
    named = all(isinstance(item, tuple) for item in items)
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
            if named:
                names.append(str(item[0]))
    return out, (names if named else None)


class _Optimizer:
    _kind = "adam"

    def __init__(self, parameters, **options):
        self._params, self._names = _collect(parameters)
        ctx = self._params[0].ctx
        for p in self._params:
            if p.ctx is not ctx:
                raise ValueError("all parameters of one optimizer must live on the same device")
        self._ctx = ctx
        self._cfg = N.OptimCfg()
        self._cfg.kind = _KIND[self._kind]
        self._options = dict(options)
        self._apply_options()
        self._handle = None
        self._create()

    def _create(self) -> None:
        """(Re)create the native optimizer with zero state for the current options."""
        if self._handle:
            lib.tx_optim_destroy(self._handle)
            self._handle = None
        handle = C.c_void_p()
        values = N.ptr_array([p.ptr for p in self._params])
        grads = N.ptr_array([p._grad_ptr for p in self._params])
        numel = N.i64_array([p.numel for p in self._params])
        self._ctx.check(lib.tx_optim_create(self._ctx.handle, C.byref(self._cfg), len(self._params),
                                            values, grads, numel, C.byref(handle)), "optimizer")
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

    # -- state dictionaries (crates/tynx-python/src/optimizer/state.rs) ------------------
    _STATE_VERSION = 1
    _TITLE = {"adam": "Adam", "adamw": "AdamW", "sgd": "SGD"}

    def _named(self) -> list[str]:
        if self._names is None:
            raise ValueError(f"{self._TITLE[self._kind]}.state_dict() requires construction from "
                             "model.named_parameters()")
        return self._names

    def _config_dict(self) -> dict:
        c = self._cfg
        if self._kind == "sgd":
            return {"lr": c.lr, "momentum": c.momentum, "dampening": c.dampening,
                    "weight_decay": c.weight_decay, "nesterov": bool(c.nesterov)}
        return {"lr": c.lr, "betas": (c.beta1, c.beta2), "eps": c.eps,
                "weight_decay": c.weight_decay, "amsgrad": bool(c.amsgrad)}

    def _slots(self) -> tuple:
        """(state key, native slot) pairs present under the current options."""
        if self._kind == "sgd":
            return (("momentum_buffer", 3),) if self._cfg.momentum != 0 else ()
        slots = (("exp_avg", 0), ("exp_avg_sq", 1))
        return slots + ((("max_exp_avg_sq", 2),) if self._cfg.amsgrad else ())

    def _state_tensor(self, index: int, which: int) -> Tensor:
        ptr = C.c_void_p()
        self._ctx.check(lib.tx_optim_state_ptr(self._handle, index, which, C.byref(ptr)))
        p = self._params[index]
        out = Tensor._empty(p.shape, "float32", self._ctx)
        self._ctx.check(lib.tx_d2d(self._ctx.handle, out.ptr, ptr.value, out.nbytes))
        return out

    def state_dict(self) -> dict:
        """Name-keyed configuration and adaptive state in the reference's layout:
        ``version``, ``optimizer``, ``parameter_names`` (sorted), ``config`` and a
        ``state`` entry (step + moments as Tensors) for every parameter that has
        been stepped (``adam.rs:339-354``, ``state.rs:71-114``)."""
        names = self._named()
        self._sync()
        steps = (C.c_int64 * len(self._params))()
        self._ctx.check(lib.tx_optim_get_steps(self._handle, steps))
        state = {}
        for i, name in enumerate(names):
            if steps[i] <= 0:
                continue
            entry: dict = {} if self._kind == "sgd" else {"step": int(steps[i])}
            for key, which in self._slots():
                entry[key] = self._state_tensor(i, which)
            if entry:
                state[name] = entry
        return {"version": self._STATE_VERSION, "optimizer": self._TITLE[self._kind],
                "parameter_names": sorted(names), "config": self._config_dict(), "state": state}

    def load_state_dict(self, state_dict: dict) -> None:
        """Restore configuration and state by parameter name; nothing changes
        unless the whole dictionary validates (``state.rs:116-160``,
        ``optimizer.rs:400-455``)."""
        title = self._TITLE[self._kind]
        names = self._named()
        if not isinstance(state_dict, dict):
            raise TypeError(f"{title} state_dict must be a dictionary")

        def required(d, key):
            if key not in d:
                raise ValueError(f"state_dict is missing field {key!r}")
            return d[key]

        version = required(state_dict, "version")
        if version != self._STATE_VERSION:
            raise ValueError(f"unsupported optimizer state_dict version {version}; "
                             f"expected {self._STATE_VERSION}")
        kind = required(state_dict, "optimizer")
        if kind != title:
            raise ValueError(f"cannot load {kind} state into {title} optimizer")
        config = required(state_dict, "config")
        entries = required(state_dict, "state")
        if not isinstance(config, dict) or not isinstance(entries, dict):
            raise TypeError("state_dict fields 'config' and 'state' must be dictionaries")
        saved = list(required(state_dict, "parameter_names"))
        if len(set(saved)) != len(saved) or any(not str(n).strip() for n in saved):
            raise ValueError(f"{title} parameter names must be unique and non-empty")
        missing = sorted(set(names) - set(saved))
        unexpected = sorted(set(saved) - set(names))
        if missing or unexpected:
            raise ValueError(f"{title} parameter names do not match: missing={missing!r}, "
                             f"unexpected={unexpected!r}")
        for name in entries:
            if name not in set(saved):
                raise ValueError(f"{title} state for unknown parameter name {name!r}")
        options = dict(self._options)
        if self._kind == "sgd":
            for key in ("lr", "momentum", "dampening", "weight_decay", "nesterov"):
                options[key] = required(config, key)
        else:
            for key in ("lr", "betas", "eps", "weight_decay", "amsgrad"):
                options[key] = required(config, key)
            options["betas"] = tuple(options["betas"])
        index = {n: i for i, n in enumerate(names)}
        host: dict = {}
        for name, entry in entries.items():
            if not isinstance(entry, dict):
                raise TypeError(f"{title} state for {name!r} must be a dictionary")
            p = self._params[index[name]]
            step = 1 if self._kind == "sgd" else required(entry, "step")
            if self._kind != "sgd" and (not isinstance(step, int) or step <= 0):
                raise ValueError(f"{title} state step for {name!r} must be positive")
            arrays = {}
            keys = [k for k, _ in self._slots_for(options)]
            for key in keys:
                value = required(entry, key)
                array = value.numpy() if isinstance(value, Tensor) else np.asarray(value, np.float32)
                if tuple(array.shape) != tuple(p.shape):
                    raise ValueError(f"{title} state {key!r} for {name!r} has shape {array.shape}, "
                                     f"expected {tuple(p.shape)}")
                arrays[key] = np.ascontiguousarray(array, dtype=np.float32)
            host[name] = (int(step), arrays)
        # everything validated: publish
        previous = dict(self._options)
        self._options = options
        try:
            self._apply_options()
        except Exception:
            self._options = previous
            self._apply_options()
            raise
        self._create()
        steps = (C.c_int64 * len(self._params))()
        for name, (step, arrays) in host.items():
            i = index[name]
            steps[i] = step
            for key, which in self._slots():
                ptr = C.c_void_p()
                self._ctx.check(lib.tx_optim_state_ptr(self._handle, i, which, C.byref(ptr)))
                a = arrays[key]
                self._ctx.check(lib.tx_h2d(self._ctx.handle, ptr.value, a.ctypes.data, a.nbytes))
        self._ctx.check(lib.tx_optim_set_steps(self._handle, steps))

    def _slots_for(self, options: dict) -> tuple:
        if self._kind == "sgd":
            return (("momentum_buffer", 3),) if float(options.get("momentum", 0.0)) != 0 else ()
        slots = (("exp_avg", 0), ("exp_avg_sq", 1))
        return slots + ((("max_exp_avg_sq", 2),) if options.get("amsgrad") else ())

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
