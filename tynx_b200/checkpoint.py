"""Resumable model + optimizer checkpoints on ``Device("cuda")``.

The file format is the reference's ``tynx.training`` version 1 JSON payload
(``crates/tynx-python/python/tynx/checkpoint.py:22-23,87-114``), so that a
checkpoint written here loads in Tynx and the other way round:

* the root is ``{"format": "tynx.training", "version": 1, "model": ...,
  "optimizer": ..., "scheduler": ...}``;
* a tensor is ``{"__type__": "tensor", "data": nested lists, "dtype": ...,
  "shape": [...]}``, a tuple is ``{"__type__": "tuple", "items": [...]}``;
  dictionaries need string keys; ``NaN``/``inf`` are written as JSON allows
  (``allow_nan``), keys sorted, no whitespace;
* the write is atomic: a temporary file beside the target is written,
  fsynced and moved over the target with ``os.replace``.

Device tensors are copied to the host once for the write (one device-to-host
copy per tensor) and uploaded once on load.  ``load_checkpoint`` validates the
whole payload (model names, shapes and dtypes, the optimizer's own
validation) before it publishes anything, and rolls the model and optimizer
back if publishing fails part-way.

Both argument orders are accepted, as in the reference: ``(path, model[,
optimizer])`` and ``(model[, optimizer], path)``.
"""

from __future__ import annotations

import json
import os
import tempfile
from contextlib import suppress
from dataclasses import dataclass
from pathlib import Path
from typing import Any, Optional

import numpy as np

from ._core import Tensor

FORMAT = "tynx.training"
VERSION = 1


@dataclass(frozen=True)
class LoadStateResult:
    """Missing and unexpected names of a non-strict state load."""

    missing_keys: tuple
    unexpected_keys: tuple


# -- argument handling -------------------------------------------------------------------------

def _is_path(value) -> bool:
    return isinstance(value, (str, os.PathLike))


def _split_args(first, second, third, verb: str):
    if _is_path(first):
        path, model, optimizer = first, second, third
    elif _is_path(third):
        path, model, optimizer = third, first, second
    elif _is_path(second) and third is None:
        path, model, optimizer = second, first, None
    else:
        raise TypeError(f"{verb}_checkpoint expects (path, model[, optimizer]) or "
                        "(model[, optimizer], path)")
    if _is_path(model):
        raise TypeError(f"{verb}_checkpoint model must be a model object, not a path")
    if optimizer is not None:
        needed = ("state_dict",) if verb == "save" else ("state_dict", "load_state_dict")
        if not all(callable(getattr(optimizer, n, None)) for n in needed):
            what = " and ".join(f"{n}()" for n in needed)
            raise TypeError(f"{verb}_checkpoint optimizer must provide {what}")
    return Path(path), model, optimizer


def _check_scheduler(optimizer, scheduler) -> None:
    if scheduler is None:
        return
    if optimizer is None:
        raise ValueError("checkpointing a scheduler requires its optimizer")
    if not (callable(getattr(scheduler, "state_dict", None))
            and callable(getattr(scheduler, "load_state_dict", None))):
        raise TypeError("checkpoint scheduler must provide state_dict() and load_state_dict()")
    if getattr(scheduler, "optimizer", None) is not optimizer:
        raise ValueError("checkpoint scheduler must belong to the supplied optimizer")


# -- encoding ----------------------------------------------------------------------------------

def _encode(value) -> Any:
    if value is None or type(value) in (bool, int, float, str):
        return value
    if isinstance(value, Tensor):
        host = value.numpy()
        return {"__type__": "tensor", "data": host.tolist(), "dtype": value.dtype,
                "shape": [int(d) for d in value.shape]}
    if type(value) is tuple:
        return {"__type__": "tuple", "items": [_encode(v) for v in value]}
    if type(value) is list:
        return [_encode(v) for v in value]
    if type(value) is dict:
        out = {}
        for key, item in value.items():
            if not isinstance(key, str):
                raise TypeError(f"checkpoint dictionaries require string keys, got "
                                f"{type(key).__qualname__}")
            out[key] = _encode(item)
        return out
    raise TypeError(f"checkpoint cannot serialize {type(value).__qualname__}")


def _nested_shape_ok(data, shape) -> bool:
    if not shape:
        return not isinstance(data, list)
    if not isinstance(data, list) or len(data) != shape[0]:
        return False
    return all(_nested_shape_ok(item, shape[1:]) for item in data)


def _decode(value) -> Any:
    if isinstance(value, list):
        return [_decode(v) for v in value]
    if not isinstance(value, dict):
        return value
    marker = value.get("__type__")
    if marker == "tensor":
        dtype, shape = value.get("dtype"), value.get("shape")
        if not isinstance(dtype, str) or not isinstance(shape, list) or not shape or \
                not all(type(d) is int and d >= 0 for d in shape):
            raise ValueError("invalid tensor metadata in Tynx checkpoint")
        if dtype not in ("float32", "int64", "bool"):
            raise ValueError(f"unsupported checkpoint tensor dtype {dtype!r}")
        data = _required(value, "data")
        if not _nested_shape_ok(data, shape):
            raise ValueError(f"checkpoint tensor data does not match declared shape {tuple(shape)}")
        np_dtype = {"float32": np.float32, "int64": np.int64, "bool": np.bool_}[dtype]
        array = np.asarray(data, dtype=np_dtype).reshape(shape)
        return Tensor(array, dtype=dtype)
    if marker == "tuple":
        items = _required(value, "items")
        if not isinstance(items, list):
            raise ValueError("checkpoint tuple items must be a list")
        return tuple(_decode(v) for v in items)
    if marker is not None:
        raise ValueError(f"unknown checkpoint value type {marker!r}")
    return {k: _decode(v) for k, v in value.items()}


def _required(d: dict, key: str):
    if key not in d:
        raise ValueError(f"checkpoint is missing field {key!r}")
    return d[key]


# -- model state -------------------------------------------------------------------------------

def _model_state(model) -> dict:
    state = model.state_dict()
    if not isinstance(state, dict):
        raise TypeError("model.state_dict() must return a dictionary")
    return state


def _targets(model) -> dict:
    """The model's live state tensors by name (parameters, then buffers)."""
    out = dict(model.named_parameters()) if hasattr(model, "named_parameters") else {}
    if hasattr(model, "named_buffers"):
        out.update(dict(model.named_buffers()))
    return out


def prepare_model_state(model, state: dict, strict: bool):
    """Validate a model state load without changing the model: names (strict
    or not), shapes and dtypes.  Returns the names to publish and the result."""
    if not isinstance(state, dict):
        raise TypeError(f"state_dict must be a mapping, got {type(state).__qualname__}")
    if type(strict) is not bool:
        raise TypeError(f"strict must be a bool, got {type(strict).__qualname__}")
    current = _model_state(model)
    for name, value in state.items():
        if not isinstance(name, str):
            raise TypeError(f"state_dict keys must be strings, got {type(name).__qualname__}")
        if not isinstance(value, Tensor):
            raise TypeError(f"state_dict value for {name!r} must be a Tensor, got "
                            f"{type(value).__qualname__}")
    missing = tuple(sorted(set(current) - set(state)))
    unexpected = tuple(sorted(set(state) - set(current)))
    if strict and (missing or unexpected):
        raise ValueError(f"state_dict key mismatch: missing={list(missing)!r}, "
                         f"unexpected={list(unexpected)!r}")
    names = sorted(set(current) & set(state))
    for name in names:
        src, dst = state[name], current[name]
        if tuple(src.shape) != tuple(dst.shape) or src.dtype != dst.dtype:
            raise ValueError(f"state_dict value for {name!r} has shape {tuple(src.shape)} and dtype "
                             f"{src.dtype}; expected shape {tuple(dst.shape)} and dtype {dst.dtype}")
    return names, LoadStateResult(missing, unexpected)


# -- public API --------------------------------------------------------------------------------

def save_checkpoint(path, model, optimizer=None, *, scheduler=None) -> None:
    """Atomically save model state and optional optimizer / scheduler state."""
    target, model, optimizer = _split_args(path, model, optimizer, "save")
    _check_scheduler(optimizer, scheduler)
    state = _model_state(model)
    if not state:
        raise ValueError("cannot save checkpoint: model has no parameters or buffers")
    payload = {
        "format": FORMAT,
        "version": VERSION,
        "model": _encode(dict(state)),
        "optimizer": _encode(None if optimizer is None else optimizer.state_dict()),
        "scheduler": _encode(None if scheduler is None else scheduler.state_dict()),
    }
    text = json.dumps(payload, allow_nan=True, separators=(",", ":"), sort_keys=True)
    fd, tmp = tempfile.mkstemp(dir=target.parent, prefix=f".{target.name}.", suffix=".tmp", text=True)
    try:
        with os.fdopen(fd, "w", encoding="utf-8") as f:
            f.write(text)
            f.flush()
            os.fsync(f.fileno())
        os.replace(tmp, target)
    except BaseException:
        with suppress(FileNotFoundError):
            os.unlink(tmp)
        raise


def _read(path: Path) -> dict:
    try:
        with path.open(encoding="utf-8") as f:
            payload = json.load(f)
    except json.JSONDecodeError as error:
        raise ValueError(f"invalid Tynx checkpoint JSON: {error}") from error
    if not isinstance(payload, dict):
        raise ValueError("Tynx checkpoint root must be a dictionary")
    if payload.get("format") != FORMAT:
        raise ValueError("file is not a Tynx training checkpoint")
    if payload.get("version") != VERSION:
        raise ValueError(f"unsupported Tynx checkpoint version {payload.get('version')!r}; "
                         f"expected {VERSION}")
    return payload


def load_checkpoint(path, model, optimizer=None, strict: bool = True, *,
                    scheduler=None) -> LoadStateResult:
    """Restore model (and optimizer / scheduler) state; nothing is published
    until every component has validated, and a failure while publishing puts
    the previous state back."""
    target, model, optimizer = _split_args(path, model, optimizer, "load")
    payload = _read(target)
    state = _decode(_required(payload, "model"))
    if not isinstance(state, dict) or not all(isinstance(v, Tensor) for v in state.values()):
        raise ValueError("checkpoint field 'model' must map names to Tynx Tensors")
    if not state:
        raise ValueError("cannot load checkpoint: model state is empty")
    encoded_opt = _required(payload, "optimizer")
    opt_state = None
    if optimizer is not None:
        if encoded_opt is None:
            raise ValueError("checkpoint does not contain optimizer state")
        opt_state = _decode(encoded_opt)
        if not isinstance(opt_state, dict):
            raise ValueError("checkpoint field 'optimizer' must be a dictionary")
    _check_scheduler(optimizer, scheduler)
    sched_state = None
    if scheduler is not None:
        sched_state = _decode(payload.get("scheduler"))
        if not isinstance(sched_state, dict):
            raise ValueError("checkpoint does not contain scheduler state")
    names, result = prepare_model_state(model, state, strict)
    previous_model = {k: v.clone() for k, v in _model_state(model).items()}
    previous_opt = None if optimizer is None else optimizer.state_dict()
    previous_sched = None if scheduler is None else scheduler.state_dict()
    try:
        if optimizer is not None:
            optimizer.load_state_dict(opt_state)
        if scheduler is not None:
            scheduler.load_state_dict(sched_state)
        current = _targets(model)
        for name in names:
            target_tensor = current.get(name)
            if target_tensor is None:
                raise ValueError(f"model has no state named {name!r}")
            target_tensor.copy_(state[name])
    except BaseException:
        current = _targets(model)
        for name, value in previous_model.items():
            if name in current:
                current[name].copy_(value)
        if optimizer is not None and previous_opt is not None:
            optimizer.load_state_dict(previous_opt)
        if scheduler is not None:
            scheduler.load_state_dict(previous_sched)
        raise
    return result


__all__ = ["LoadStateResult", "load_checkpoint", "save_checkpoint"]
