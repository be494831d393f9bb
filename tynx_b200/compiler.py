"""``tynx_b200.compile``: whole-function capture into a CUDA graph.

Same contract as ``tynx.compile`` (``crates/tynx-python/python/tynx/compiler.py:131-205``):
the first call with a new exact signature (Tensor shapes and dtypes plus the
static arguments) runs the Python body once while every kernel it issues is
recorded; later calls with that signature copy the new inputs into the
recorded input buffers and replay the graph with no Python dispatch.  Where
the reference replays its IR node by node (``Graph::run_values``,
``crates/tynx-capture/src/lib.rs:747-882``), here the replay is one
``cudaGraphLaunch`` of the forward, loss, backward and optimizer kernels.

Guards: the signature and the static arguments must match, and so must the
gradient state of every parameter slot whose state the captured body *read*
before writing it (whether a gradient exists decides overwrite versus
accumulate in backward and which tensors the optimizer steps).  A body that
starts with ``zero_grad()`` therefore depends on no prior state.  On a
mismatch a new graph is captured.  A body that reads device data on the host
(``.item()``, ``.numpy()``) cannot be captured: with ``fullgraph=True`` that
raises, otherwise the function falls back to eager execution, as in the
reference.
"""

from __future__ import annotations

import ctypes as C
import inspect
import threading
import warnings
from typing import Any, Callable, Iterable, Optional

from . import _native as N
from ._core import Tensor
from ._native import CaptureError, lib

# While a body is being captured: first access to each parameter's gradient
# flag, id(param) -> (param, "read" | "write", flag before the access).
_capture_log: Optional[dict] = None


def note_grad_flag(param, kind: str) -> None:
    """Record the first access of a capture to ``param``'s gradient flag."""
    log = _capture_log
    if log is not None and id(param) not in log:
        log[id(param)] = (param, kind, param._raw_grad_defined())


def register_model(model) -> None:  # kept for API symmetry; guards are per parameter
    return None


def _read_guard(log: dict) -> tuple:
    return tuple((key, flag) for key, (_p, kind, flag) in sorted(log.items()) if kind == "read")


def _params_of(log: dict) -> dict:
    return {key: p for key, (p, _kind, _flag) in log.items()}


def _current(params: dict, guard: tuple) -> tuple:
    return tuple((key, params[key]._raw_grad_defined()) for key, _flag in guard)


class _Captured:
    def __init__(self, static_key, signature, exec_handle, static_inputs, static_outputs, spec,
                 guard, params, post_flags, ctx):
        self.static_key = static_key
        self.signature = signature
        self.exec = exec_handle
        self.static_inputs = static_inputs
        self.static_outputs = static_outputs
        self.spec = spec
        self.guard = guard          # ((param id, flag the body read), ...)
        self.params = params        # param id -> Parameter (kept alive with the graph)
        self.post_flags = post_flags  # param id -> flag after one execution
        self.ctx = ctx
        kernels, total = C.c_int64(), C.c_int64()
        lib.tx_exec_node_count(exec_handle, C.byref(kernels), C.byref(total))
        self.kernel_count = kernels.value
        self.node_count = total.value

    def matches(self) -> bool:
        return _current(self.params, self.guard) == self.guard

    def apply_post_state(self) -> None:
        for key, flag in self.post_flags.items():
            self.params[key]._set_grad_defined(flag)

    def __del__(self):
        try:
            if self.exec:
                lib.tx_exec_destroy(self.exec)
                self.exec = None
        except Exception:
            pass


def _flatten(output) -> tuple[list[Tensor], Any]:
    if isinstance(output, Tensor):
        return [output], "t"
    if isinstance(output, (tuple, list)):
        tensors, specs = [], []
        for item in output:
            t, s = _flatten(item)
            tensors.extend(t)
            specs.append((len(t), s))
        return tensors, (type(output), specs)
    if isinstance(output, dict):
        tensors, specs = [], []
        for key, item in output.items():
            t, s = _flatten(item)
            tensors.extend(t)
            specs.append((key, len(t), s))
        return tensors, ("dict", specs)
    if output is None:
        return [], None
    raise TypeError(f"compiled functions may return Tensors, tuples, lists or dicts, got "
                    f"{type(output).__qualname__}")


def _restore(tensors: Iterable[Tensor], spec):
    it = iter(tensors)

    def build(s):
        if s == "t":
            return next(it)
        if s is None:
            return None
        kind, specs = s
        if kind == "dict":
            return {key: build(sub) for key, _n, sub in specs}
        return kind(build(sub) for _n, sub in specs)

    return build(spec)


def _copy_out(t: Tensor) -> Tensor:
    out = Tensor._empty(t.shape, t.dtype, t.ctx)
    t.ctx.check(lib.tx_d2d(t.ctx.handle, out.ptr, t.ptr, t.nbytes))
    return out


class CompiledFunction:
    """Callable exact-signature CUDA-graph cache returned by :func:`compile`."""

    def __init__(self, function: Callable, *, fullgraph: bool = False,
                 static_argnames: Iterable[str] = ()):
        if not callable(function):
            raise TypeError(f"compile expected a callable, got {type(function).__qualname__}")
        self._function = function
        self._signature = inspect.signature(function)
        self._fullgraph = fullgraph
        self._static = frozenset(static_argnames)
        unknown = self._static.difference(self._signature.parameters)
        if unknown:
            raise ValueError(f"static_argnames {sorted(unknown)} are not parameters of the function")
        self._owner = threading.current_thread()
        self._graphs: list[_Captured] = []
        self._fallback = False
        self.compile_count = 0
        self.replay_count = 0
        self.fallback_count = 0
        self.invalidation_count = 0
        self.last_fallback_reason: Optional[str] = None

    @property
    def graph_count(self) -> int:
        return len(self._graphs)

    def clear_cache(self) -> None:
        self._graphs.clear()
        self._fallback = False
        self.last_fallback_reason = None

    def _prepare(self, bound) -> tuple[list[Tensor], tuple] | str:
        tensors, static_key = [], []
        for name, value in bound.arguments.items():
            kind = self._signature.parameters[name].kind
            if kind in (inspect.Parameter.VAR_POSITIONAL, inspect.Parameter.VAR_KEYWORD):
                return "variadic Python arguments"
            if name in self._static:
                if isinstance(value, Tensor):
                    return f"Tensor argument {name!r} declared static"
                try:
                    hash((type(value), value))
                except TypeError:
                    return f"unhashable static argument {name!r}"
                static_key.append((name, type(value), value))
            elif isinstance(value, Tensor):
                tensors.append(value)
            else:
                return f"non-Tensor argument {name!r}; declare it with static_argnames"
        if not tensors:
            return "a function call without Tensor inputs"
        return tensors, tuple(static_key)

    def _disable(self, reason: str) -> None:
        self._fallback = True
        self.last_fallback_reason = reason
        warnings.warn(f"tynx_b200.compile fell back to eager execution for the whole function: "
                      f"{reason}", RuntimeWarning, stacklevel=3)

    def __call__(self, *args, **kwargs):
        if threading.current_thread() is not self._owner:
            raise RuntimeError("tynx_b200.compile objects are thread-confined")
        if self._fallback:
            self.fallback_count += 1
            return self._function(*args, **kwargs)
        bound = self._signature.bind(*args, **kwargs)
        bound.apply_defaults()
        prepared = self._prepare(bound)
        if isinstance(prepared, str):
            if self._fullgraph:
                raise RuntimeError(f"tynx_b200.compile(fullgraph=True) cannot capture {prepared}")
            self._disable(prepared)
            self.fallback_count += 1
            return self._function(*args, **kwargs)
        tensors, static_key = prepared
        signature = tuple((t.shape, t.dtype, t.requires_grad) for t in tensors)
        for entry in self._graphs:
            if entry.static_key == static_key and entry.signature == signature and \
                    entry.matches():
                return self._replay(entry, tensors)
        return self._capture(bound, tensors, static_key, signature)

    def _replay(self, entry: _Captured, tensors: list[Tensor]):
        ctx = entry.ctx
        for dst, src in zip(entry.static_inputs, tensors):
            ctx.check(lib.tx_d2d(ctx.handle, dst.ptr, src.ptr, src.nbytes))
        ctx.check(lib.tx_exec_launch(entry.exec), "graph replay")
        entry.apply_post_state()
        self.replay_count += 1
        return _restore((_copy_out(t) for t in entry.static_outputs), entry.spec)

    def launch_only(self, *args, **kwargs) -> None:
        """Replay the cached graph for these arguments without copying outputs out
        (inputs are still copied in); used to time the captured step itself."""
        bound = self._signature.bind(*args, **kwargs)
        bound.apply_defaults()
        tensors, static_key = self._prepare(bound)
        signature = tuple((t.shape, t.dtype, t.requires_grad) for t in tensors)
        for entry in self._graphs:
            if entry.static_key == static_key and entry.signature == signature and entry.matches():
                ctx = entry.ctx
                for dst, src in zip(entry.static_inputs, tensors):
                    if dst.ptr != src.ptr:
                        ctx.check(lib.tx_d2d(ctx.handle, dst.ptr, src.ptr, src.nbytes))
                ctx.check(lib.tx_exec_launch(entry.exec), "graph replay")
                entry.apply_post_state()
                self.replay_count += 1
                return
        raise RuntimeError("no captured graph matches these arguments; call the function first")

    def entry_for(self, *args, **kwargs) -> Optional[_Captured]:
        bound = self._signature.bind(*args, **kwargs)
        bound.apply_defaults()
        tensors, static_key = self._prepare(bound)
        signature = tuple((t.shape, t.dtype, t.requires_grad) for t in tensors)
        for entry in self._graphs:
            if entry.static_key == static_key and entry.signature == signature and entry.matches():
                return entry
        return None

    def _capture(self, bound, tensors, static_key, signature):
        global _capture_log
        ctx = tensors[0].ctx
        static_inputs = []
        for t in tensors:
            s = Tensor._empty(t.shape, t.dtype, ctx)
            ctx.check(lib.tx_d2d(ctx.handle, s.ptr, t.ptr, t.nbytes))
            s.requires_grad = t.requires_grad
            static_inputs.append(s)
        replaced = iter(static_inputs)
        arguments = {name: (next(replaced) if isinstance(value, Tensor) else value)
                     for name, value in bound.arguments.items()}
        call = inspect.BoundArguments(self._signature, arguments)
        ctx.check(lib.tx_capture_begin(ctx.handle), "capture")
        ctx.capturing = True
        log: dict = {}
        _capture_log = log

        def restore_flags() -> None:
            for _key, (param, _kind, flag) in log.items():
                param._set_grad_defined(flag)

        try:
            output = self._function(*call.args, **call.kwargs)
            outputs, spec = _flatten(output)
        except BaseException as error:
            _capture_log = None
            lib.tx_capture_abort(ctx.handle)
            ctx.capturing = False
            restore_flags()
            if isinstance(error, CaptureError) and not self._fullgraph:
                self._disable(str(error))
                self.fallback_count += 1
                return self._function(*bound.args, **bound.kwargs)
            if isinstance(error, CaptureError):
                raise RuntimeError(f"tynx_b200.compile(fullgraph=True) cannot capture: {error}") \
                    from error
            raise
        _capture_log = None
        handle = C.c_void_p()
        code = lib.tx_capture_end(ctx.handle, C.byref(handle))
        ctx.capturing = False
        if code != N.TX_OK:
            restore_flags()
            ctx.check(code, "capture")
        params = _params_of(log)
        post_flags = {key: p._raw_grad_defined() for key, p in params.items()}
        static_outputs = [o.detach() for o in outputs]
        entry = _Captured(static_key, signature, handle.value, static_inputs, static_outputs, spec,
                          _read_guard(log), params, post_flags, ctx)
        self._graphs.append(entry)
        self.compile_count += 1
        # the body only recorded work: run it once now
        ctx.check(lib.tx_exec_launch(entry.exec), "graph launch")
        return _restore((_copy_out(t) for t in static_outputs), spec)


def compile(function: Optional[Callable] = None, *, fullgraph: bool = False,
            static_argnames: Iterable[str] = ()):
    """Capture a whole step (forward, loss, backward, optimizer) as one CUDA graph."""
    if function is None:
        return lambda f: CompiledFunction(f, fullgraph=fullgraph, static_argnames=static_argnames)
    return CompiledFunction(function, fullgraph=fullgraph, static_argnames=static_argnames)


__all__ = ["CompiledFunction", "compile"]
