"""Device placement, device contexts and the eager ``Tensor`` with its tape.

Mirrors the reference's tensor surface (``crates/tynx-python/src/tensor.rs``:
``PyTensor``, ``backward`` at 1337-1417, ``log_softmax`` 1589, ``gather`` 1769,
``mean`` 1425) on the CUDA placement.  Every operation launches kernels from
``libtynx_cuda.so``; the tape records one backward closure per operation and
is walked in reverse topological order by :meth:`Tensor.backward`, with leaf
gradients accumulating (``crates/tynx-train/src/parameter.rs:300-333``).

Tensors live on the device; ``tolist()`` / ``numpy()`` / ``item()`` copy to
the host and synchronise.  Contexts are per device and confined to the thread
that created them, like Tynx tensors (``crates/tynx-python/src/tensor.rs:54-92``).
"""

from __future__ import annotations

import ctypes as C
import os
import threading
from contextlib import contextmanager
from typing import Iterable, Optional, Sequence, Union

import numpy as np

from . import _native as N
from ._native import check, lib

Number = Union[int, float]

# =============================================================================
# devices and contexts
# =============================================================================


class Device:
    """A placement.  ``Device("cuda")`` / ``Device("cuda:1")`` select a B200.

    ``"default"`` resolves to the process's GPU (``LOCAL_RANK`` under torchrun,
    else 0).  The reference's CPU kinds (``"cpu"``, ``"flex"``) are rejected:
    this engine has no CPU path (``crates/tynx-python/src/device.rs:50-61``).
    """

    __slots__ = ("kind", "index")

    def __init__(self, spec: Union[str, "Device"] = "default"):
        if isinstance(spec, Device):
            self.kind, self.index = spec.kind, spec.index
            return
        if not isinstance(spec, str):
            raise TypeError(f"Device expects a string, got {type(spec).__qualname__}")
        text = spec.strip().lower()
        if text in ("default", "cuda", "gpu"):
            self.kind, self.index = "cuda", _default_index()
        elif text.startswith("cuda:"):
            try:
                self.index = int(text.split(":", 1)[1])
            except ValueError as error:
                raise ValueError(f"invalid CUDA device {spec!r}") from error
            self.kind = "cuda"
        elif text in ("cpu", "flex"):
            raise ValueError(
                f"device {spec!r} is the Flex CPU backend; tynx_b200 runs on CUDA only "
                "(use the reference build for CPU training)"
            )
        else:
            raise ValueError(f"unknown device {spec!r}; expected 'cuda', 'cuda:N' or 'default'")

    def __repr__(self) -> str:
        return f"Device('cuda:{self.index}')"

    def __str__(self) -> str:
        return f"cuda:{self.index}"

    def __eq__(self, other) -> bool:
        return isinstance(other, Device) and other.index == self.index

    def __hash__(self) -> int:
        return hash(("cuda", self.index))

    @property
    def is_accelerated(self) -> bool:
        return True


def _default_index() -> int:
    try:
        return int(os.environ.get("LOCAL_RANK", "0"))
    except ValueError:
        return 0


class Context:
    """One ``tx_ctx`` (stream, allocator, latched error) per device."""

    def __init__(self, index: int):
        math = os.environ.get("TYNX_CUDA_MATH", "tf32").lower()
        if math not in N.TX_MATH:
            raise ValueError(f"TYNX_CUDA_MATH must be one of {sorted(N.TX_MATH)}, got {math!r}")
        handle = C.c_void_p()
        code = lib.tx_ctx_create(index, N.TX_MATH[math], C.byref(handle))
        if code != N.TX_OK:
            if code == N.TX_ERR_UNSUPPORTED:
                raise RuntimeError(f"cuda:{index} is not an sm_100 (Blackwell) device")
            raise RuntimeError(
                f"cannot create a CUDA context on cuda:{index} (code {code}); a B200 is required"
            )
        self.handle = handle
        self.index = index
        self.owner = threading.get_ident()
        self.capturing = False

    def check(self, code: int, what: str = "") -> None:
        if code != N.TX_OK:
            N.raise_for(code, self.handle, what)

    def alloc(self, nbytes: int) -> int:
        out = C.c_void_p()
        self.check(lib.tx_alloc(self.handle, max(int(nbytes), 1), C.byref(out)), "alloc")
        return out.value

    def free(self, ptr: int) -> None:
        lib.tx_free(self.handle, ptr)

    def sync(self, timeout_ms: int = 0) -> None:
        self.check(lib.tx_sync(self.handle, timeout_ms), "synchronize")

    @property
    def math(self) -> str:
        out = C.c_int()
        lib.tx_ctx_get_math(self.handle, C.byref(out))
        return {v: k for k, v in N.TX_MATH.items()}[out.value]

    @math.setter
    def math(self, mode: str) -> None:
        self.check(lib.tx_ctx_set_math(self.handle, N.TX_MATH[mode]))


_contexts: dict[int, Context] = {}
_lock = threading.Lock()


def context(device: Optional[Device] = None) -> Context:
    index = (device or Device("default")).index
    ctx = _contexts.get(index)
    if ctx is None:
        with _lock:
            ctx = _contexts.get(index)
            if ctx is None:
                ctx = Context(index)
                _contexts[index] = ctx
    return ctx


def get_default_device() -> Device:
    return Device("default")


def synchronize(device: Optional[Device] = None, timeout_ms: int = 0) -> None:
    """Wait for queued work and surface latched asynchronous device errors
    (``crates/tynx/src/device.rs:84-90``)."""
    context(device).sync(timeout_ms)


def set_math_mode(mode: str, device: Optional[Device] = None) -> None:
    """Select the fp32 contraction mode: ``"tf32"``, ``"3xtf32"`` or ``"fp32"``."""
    if mode not in N.TX_MATH:
        raise ValueError(f"math mode must be one of {sorted(N.TX_MATH)}")
    context(device).math = mode


# =============================================================================
# grad mode
# =============================================================================

_grad = threading.local()


def is_grad_enabled() -> bool:
    return getattr(_grad, "enabled", True)


@contextmanager
def no_grad():
    previous = is_grad_enabled()
    _grad.enabled = False
    try:
        yield
    finally:
        _grad.enabled = previous


# =============================================================================
# storage
# =============================================================================

_DTYPES = {"float32": (np.float32, 4), "int64": (np.int64, 8), "bool": (np.bool_, 1)}


class Storage:
    """A device allocation returned to the context allocator when dropped."""

    __slots__ = ("ctx", "ptr", "nbytes", "owned", "__weakref__")

    def __init__(self, ctx: Context, nbytes: int, ptr: Optional[int] = None, owned: bool = True):
        self.ctx = ctx
        self.nbytes = nbytes
        self.owned = owned and ptr is None
        self.ptr = ctx.alloc(nbytes) if ptr is None else ptr

    def __del__(self):
        if self.owned and self.ptr:
            try:
                lib.tx_free(self.ctx.handle, self.ptr)
            except Exception:  # interpreter shutdown
                pass
            self.ptr = 0


def _shape_tuple(shape) -> tuple:
    if isinstance(shape, int):
        return (shape,)
    return tuple(int(s) for s in shape)


def _numel(shape) -> int:
    n = 1
    for s in shape:
        n *= s
    return n


def _contig_strides(shape) -> list[int]:
    strides = [0] * len(shape)
    acc = 1
    for i in range(len(shape) - 1, -1, -1):
        strides[i] = acc
        acc *= shape[i]
    return strides


def _broadcast(a: tuple, b: tuple) -> tuple:
    n = max(len(a), len(b))
    out = []
    for i in range(n):
        da = a[i - (n - len(a))] if i >= n - len(a) else 1
        db = b[i - (n - len(b))] if i >= n - len(b) else 1
        if da != db and da != 1 and db != 1:
            raise ValueError(f"shapes {a} and {b} cannot be broadcast")
        out.append(db if da == 1 else da)
    return tuple(out)


def _bstrides(shape: tuple, out: tuple) -> list[int]:
    n = len(out)
    st = [0] * n
    stride = 1
    for i in range(n - 1, -1, -1):
        j = i - (n - len(shape))
        if j < 0:
            st[i] = 0
            continue
        st[i] = 0 if (shape[j] == 1 and out[i] != 1) else stride
        stride *= shape[j]
    return st


# =============================================================================
# tape
# =============================================================================


class Fn:
    """A recorded operation: parents, and a closure mapping output gradients to
    input gradients."""

    __slots__ = ("inputs", "backward", "n_out", "name", "release", "__weakref__")

    def __init__(self, name: str, inputs: Sequence[Optional["Tensor"]], backward, n_out: int = 1,
                 release=None):
        self.name = name
        self.inputs = list(inputs)
        self.backward = backward
        self.n_out = n_out
        self.release = release

    def free(self) -> None:
        self.inputs = []
        self.backward = None
        if self.release is not None:
            self.release()
            self.release = None


def _needs_grad(*tensors) -> bool:
    return is_grad_enabled() and any(isinstance(t, Tensor) and t.requires_grad for t in tensors)


class Tensor:
    """A dense device tensor (float32, int64 or bool) with an optional tape node."""

    __slots__ = ("_storage", "_offset", "shape", "dtype", "requires_grad", "_grad", "_fn",
                 "_out_index", "__weakref__")

    def __init__(self, data=None, *, dtype: Optional[str] = None, device: Optional[Device] = None,
                 requires_grad: bool = False):
        if data is None:
            raise TypeError("Tensor() needs data")
        if isinstance(data, Tensor):
            array = data.numpy()
        else:
            array = np.asarray(data)
        if dtype is None:
            if array.dtype == np.bool_:
                dtype = "bool"
            elif np.issubdtype(array.dtype, np.integer):
                dtype = "int64"
            else:
                dtype = "float32"
        if dtype not in _DTYPES:
            raise ValueError(f"unsupported dtype {dtype!r}; expected float32, int64 or bool")
        if dtype == "int64" and np.issubdtype(array.dtype, np.floating):
            raise TypeError("cannot create an int64 Tensor from floating-point data")
        array = np.ascontiguousarray(array, dtype=_DTYPES[dtype][0])
        ctx = context(device)
        storage = Storage(ctx, array.nbytes)
        # (during a capture the library stages the bytes in pinned memory owned by the graph)
        check(lib.tx_h2d(ctx.handle, storage.ptr, array.ctypes.data, array.nbytes), ctx.handle, "h2d")
        self._init(storage, 0, array.shape, dtype, requires_grad)
        if requires_grad and dtype != "float32":
            raise ValueError("only float32 tensors can require gradients")

    # -- construction helpers -----------------------------------------------------
    def _init(self, storage, offset, shape, dtype, requires_grad=False):
        self._storage = storage
        self._offset = offset
        self.shape = _shape_tuple(shape)
        self.dtype = dtype
        self.requires_grad = requires_grad
        self._grad = None
        self._fn = None
        self._out_index = 0

    @classmethod
    def _empty(cls, shape, dtype: str = "float32", ctx: Optional[Context] = None) -> "Tensor":
        ctx = ctx or context()
        shape = _shape_tuple(shape)
        t = object.__new__(cls)
        t._init(Storage(ctx, _numel(shape) * _DTYPES[dtype][1]), 0, shape, dtype)
        return t

    @classmethod
    def _view(cls, storage: Storage, offset: int, shape, dtype: str) -> "Tensor":
        t = object.__new__(cls)
        t._init(storage, offset, shape, dtype)
        return t

    # -- properties ------------------------------------------------------------------------
    @property
    def ptr(self) -> int:
        return self._storage.ptr + self._offset

    @property
    def ctx(self) -> Context:
        return self._storage.ctx

    @property
    def ndim(self) -> int:
        return len(self.shape)

    @property
    def numel(self) -> int:
        return _numel(self.shape)

    @property
    def itemsize(self) -> int:
        return _DTYPES[self.dtype][1]

    @property
    def nbytes(self) -> int:
        return self.numel * self.itemsize

    @property
    def device(self) -> Device:
        return Device(f"cuda:{self.ctx.index}")

    @property
    def grad(self) -> Optional["Tensor"]:
        return self._grad

    @grad.setter
    def grad(self, value: Optional["Tensor"]) -> None:
        self._grad = value

    @property
    def is_leaf(self) -> bool:
        return self._fn is None

    def __len__(self) -> int:
        if not self.shape:
            raise TypeError("len() of a 0-d tensor")
        return self.shape[0]

    def __repr__(self) -> str:
        try:
            values = self.numpy()
        except Exception:  # pragma: no cover
            values = "<unavailable>"
        return f"Tensor({values!r}, dtype={self.dtype}, device={self.device})"

    # -- host transfer ----------------------------------------------------------------------
    def numpy(self) -> np.ndarray:
        out = np.empty(self.shape, dtype=_DTYPES[self.dtype][0])
        if out.nbytes:
            self.ctx.check(lib.tx_d2h(self.ctx.handle, out.ctypes.data, self.ptr, out.nbytes), "d2h")
        return out

    def tolist(self):
        return self.numpy().tolist()

    def item(self) -> Number:
        if self.numel != 1:
            raise ValueError(f"item() requires a one-element tensor, got shape {self.shape}")
        return self.numpy().reshape(-1)[0].item()

    def __float__(self) -> float:
        return float(self.item())

    def detach(self) -> "Tensor":
        return Tensor._view(self._storage, self._offset, self.shape, self.dtype)

    def clone(self) -> "Tensor":
        out = Tensor._empty(self.shape, self.dtype, self.ctx)
        self.ctx.check(lib.tx_d2d(self.ctx.handle, out.ptr, self.ptr, self.nbytes))
        if _needs_grad(self):
            out._attach(Fn("clone", [self], lambda g: [g[0]]))
        return out

    def requires_grad_(self, flag: bool = True) -> "Tensor":
        if flag and self.dtype != "float32":
            raise ValueError("only float32 tensors can require gradients")
        self.requires_grad = flag
        return self

    def _attach(self, fn: Fn, index: int = 0) -> "Tensor":
        self._fn = fn
        self._out_index = index
        self.requires_grad = True
        return self

    # -- autograd -----------------------------------------------------------------------------
    def backward(self, gradient: Optional["Tensor"] = None, retain_graph: bool = False) -> None:
        """Reverse-mode sweep from this tensor (``PyTensor::backward``,
        ``crates/tynx-python/src/tensor.rs:1337-1417``)."""
        if not self.requires_grad:
            raise ValueError("backward() called on a tensor that does not require gradients")
        if gradient is None:
            if self.numel != 1:
                raise ValueError(
                    f"backward() without a gradient requires a one-element tensor, got {self.shape}"
                )
            gradient = full(self.shape, 1.0, ctx=self.ctx)
        run_backward([(self, gradient)], retain_graph=retain_graph)

    # -- shape ops ------------------------------------------------------------------------------
    def reshape(self, *shape) -> "Tensor":
        if len(shape) == 1 and isinstance(shape[0], (tuple, list)):
            shape = tuple(shape[0])
        shape = list(shape)
        if -1 in shape:
            known = _numel([s for s in shape if s != -1])
            shape[shape.index(-1)] = self.numel // known if known else 0
        shape = tuple(shape)
        if _numel(shape) != self.numel:
            raise ValueError(f"cannot reshape {self.shape} to {shape}")
        out = Tensor._view(self._storage, self._offset, shape, self.dtype)
        if _needs_grad(self):
            src = self.shape
            out._attach(Fn("reshape", [self], lambda g: [g[0].reshape(src)]))
        return out

    view = reshape

    def flatten(self) -> "Tensor":
        return self.reshape(self.numel)

    def squeeze(self, dim: Optional[int] = None) -> "Tensor":
        if dim is None:
            return self.reshape(tuple(s for s in self.shape if s != 1))
        dim = dim % self.ndim
        if self.shape[dim] != 1:
            return self
        return self.reshape(self.shape[:dim] + self.shape[dim + 1:])

    def unsqueeze(self, dim: int) -> "Tensor":
        dim = dim % (self.ndim + 1)
        return self.reshape(self.shape[:dim] + (1,) + self.shape[dim:])

    def expand(self, *shape) -> "Tensor":
        if len(shape) == 1 and isinstance(shape[0], (tuple, list)):
            shape = tuple(shape[0])
        shape = tuple(s if s != -1 else self.shape[i - (len(shape) - self.ndim)]
                      for i, s in enumerate(shape))
        if shape == self.shape:
            return self
        _broadcast(self.shape, shape)
        out = Tensor._empty(shape, self.dtype, self.ctx)
        st = _bstrides(self.shape, shape)
        self.ctx.check(lib.tx_strided_copy(self.ctx.handle, self.ptr, N.i64_array(st), out.ptr,
                                           N.i64_array(shape), len(shape), self.itemsize))
        if _needs_grad(self):
            src = self.shape
            out._attach(Fn("expand", [self], lambda g: [_sum_to(g[0], src)]))
        return out

    def transpose(self, a: int, b: int) -> "Tensor":
        perm = list(range(self.ndim))
        perm[a], perm[b] = perm[b], perm[a]
        return self.permute(*perm)

    def permute(self, *perm) -> "Tensor":
        if len(perm) == 1 and isinstance(perm[0], (tuple, list)):
            perm = tuple(perm[0])
        shape = tuple(self.shape[p] for p in perm)
        st = _contig_strides(self.shape)
        out = Tensor._empty(shape, self.dtype, self.ctx)
        self.ctx.check(lib.tx_strided_copy(self.ctx.handle, self.ptr, N.i64_array([st[p] for p in perm]),
                                           out.ptr, N.i64_array(shape), len(shape), self.itemsize))
        if _needs_grad(self):
            inv = [0] * len(perm)
            for i, p in enumerate(perm):
                inv[p] = i
            out._attach(Fn("permute", [self], lambda g: [g[0].permute(*inv)]))
        return out

    @property
    def T(self) -> "Tensor":
        return self.permute(*reversed(range(self.ndim)))

    # -- arithmetic -----------------------------------------------------------------------------
    def __add__(self, other):
        return _binary("add", self, other)

    def __radd__(self, other):
        return _binary("add", other, self)

    def __sub__(self, other):
        return _binary("sub", self, other)

    def __rsub__(self, other):
        return _binary("sub", other, self)

    def __mul__(self, other):
        return _binary("mul", self, other)

    def __rmul__(self, other):
        return _binary("mul", other, self)

    def __truediv__(self, other):
        return _binary("div", self, other)

    def __rtruediv__(self, other):
        return _binary("div", other, self)

    def __neg__(self):
        return _unary("neg", self)

    def __pow__(self, exponent):
        if isinstance(exponent, (int, float)):
            if exponent == 2:
                return self * self
            return _unary("pow", self, float(exponent))
        return _binary("pow", self, exponent)

    def __rpow__(self, base):
        # base ** x = exp(x ln base) for a positive python scalar base
        # (ReversePowerScalar of the capture IR)
        if not isinstance(base, (int, float)):
            return _binary("pow", base, self)
        if base <= 0:
            raise ValueError("a scalar base of a tensor power must be positive")
        return _unary("exp", _scale(self, float(np.log(base)), 0.0))

    def __getitem__(self, index) -> "Tensor":
        return _getitem(self, index)

    def repeat(self, *sizes) -> "Tensor":
        """Tile along each axis (leading sizes add axes), as torch.Tensor.repeat."""
        if len(sizes) == 1 and isinstance(sizes[0], (tuple, list)):
            sizes = tuple(sizes[0])
        inter, tiled, final = _repeat_plan(tuple(self.shape), tuple(sizes))
        return self.reshape(inter).expand(tiled).reshape(final)

    def erf(self):
        return _unary("erf", self)

    def reciprocal(self):
        return _unary("reciprocal", self)

    def softplus(self):
        return _unary("softplus", self)

    def softsign(self):
        return _unary("softsign", self)

    def leaky_relu(self, negative_slope: float = 0.01):
        return _unary("leakyrelu", self, float(negative_slope))

    def elu(self, alpha: float = 1.0):
        return _unary("elu", self, float(alpha))

    def hardsigmoid(self, alpha: float = 1.0 / 6.0, beta: float = 0.5):
        return _unary("hardsigmoid", self, float(alpha), float(beta))

    def __matmul__(self, other):
        return matmul(self, other)

    def exp(self):
        return _unary("exp", self)

    def log(self):
        return _unary("log", self)

    def relu(self):
        return _unary("relu", self)

    def tanh(self):
        return _unary("tanh", self)

    def sigmoid(self):
        return _unary("sigmoid", self)

    def gelu(self):
        return _unary("gelu", self)

    def sqrt(self):
        return _unary("sqrt", self)

    def abs(self):
        return _unary("abs", self)

    def clamp(self, min: Optional[float] = None, max: Optional[float] = None):
        lo = -np.inf if min is None else float(min)
        hi = np.inf if max is None else float(max)
        return _unary("clamp", self, lo, hi)

    clip = clamp

    def sum(self, dim=None, keepdim: bool = False):
        return _reduce(self, dim, keepdim, mean=False)

    def mean(self, dim=None, keepdim: bool = False):
        return _reduce(self, dim, keepdim, mean=True)

    def softmax(self, dim: int = -1):
        return _softmax(self, dim, log=False)

    def log_softmax(self, dim: int = -1):
        return _softmax(self, dim, log=True)

    def gather(self, dim: int, index: "Tensor"):
        return _gather(self, dim, index)




# =============================================================================
# kernels behind the tensor ops
# =============================================================================


def _as_tensor(value, like: Tensor) -> Tensor:
    if isinstance(value, Tensor):
        return value
    return Tensor(np.asarray(value, dtype=np.float32), device=like.device)


def full(shape, value: float, *, ctx: Optional[Context] = None, dtype: str = "float32") -> Tensor:
    out = Tensor._empty(shape, dtype, ctx)
    if dtype == "float32":
        out.ctx.check(lib.tx_fill_f32(out.ctx.handle, out.ptr, out.numel, C.c_float(value)))
    else:
        if value != 0:
            array = np.full(out.shape, value, dtype=_DTYPES[dtype][0])
            out.ctx.check(lib.tx_h2d(out.ctx.handle, out.ptr, array.ctypes.data, array.nbytes))
        else:
            out.ctx.check(lib.tx_memset(out.ctx.handle, out.ptr, 0, out.nbytes))
    return out


def _sum_to(g: Tensor, shape: tuple) -> Tensor:
    """Reduce a broadcast gradient back to ``shape``."""
    shape = tuple(shape)
    if g.shape == shape:
        return g
    padded = (1,) * (g.ndim - len(shape)) + shape
    if _numel(padded) == g.numel:
        return g.reshape(shape)
    out = Tensor._empty(shape, "float32", g.ctx)
    g.ctx.check(lib.tx_reduce_to(g.ctx.handle, g.ptr, N.i64_array(g.shape), out.ptr,
                                 N.i64_array(padded), g.ndim, 0, 0))
    return out


def _check_float(*ts):
    for t in ts:
        if isinstance(t, Tensor) and t.dtype != "float32":
            raise TypeError(f"operation requires float32 tensors, got {t.dtype}")


def _unary(op: str, x: Tensor, a: float = 0.0, b: float = 0.0) -> Tensor:
    _check_float(x)
    out = Tensor._empty(x.shape, "float32", x.ctx)
    x.ctx.check(lib.tx_unary(x.ctx.handle, N.UN[op], x.ptr, out.ptr, x.numel, C.c_float(a), C.c_float(b)))
    if _needs_grad(x):
        uses_out = op in ("exp", "tanh", "sigmoid", "relu")
        saved = out.detach() if uses_out else x.detach()

        def backward(g, op=op, a=a, b=b, saved=saved):
            dx = Tensor._empty(saved.shape, "float32", saved.ctx)
            saved.ctx.check(lib.tx_unary_bwd(saved.ctx.handle, N.UN[op], saved.ptr, g[0].ptr, dx.ptr,
                                             dx.numel, C.c_float(a), C.c_float(b), 0))
            return [dx]

        out._attach(Fn(op, [x], backward))
    return out


def _scale(x: Tensor, a: float, b: float) -> Tensor:
    """a*x + b for python scalars (one rounding: exact for a=1 or b=0)."""
    out = Tensor._empty(x.shape, "float32", x.ctx)
    x.ctx.check(lib.tx_unary(x.ctx.handle, N.UN["scale"], x.ptr, out.ptr, x.numel, C.c_float(a),
                             C.c_float(b)))
    if _needs_grad(x):
        out._attach(Fn("scale", [x], lambda g, a=a: [_scale(g[0], a, 0.0) if a != 1.0 else g[0]]))
    return out


def _binary_raw(op: str, a: Tensor, b: Tensor, shape: tuple) -> Tensor:
    out = Tensor._empty(shape, "float32", a.ctx)
    a.ctx.check(lib.tx_binary(a.ctx.handle, N.BIN[op], a.ptr, N.i64_array(_bstrides(a.shape, shape)),
                              b.ptr, N.i64_array(_bstrides(b.shape, shape)), out.ptr,
                              N.i64_array(shape), len(shape)))
    return out


def _binary(op: str, a, b) -> Tensor:
    like = a if isinstance(a, Tensor) else b
    # scalar fast paths with a single rounding, matching add_scalar / mul_scalar
    if isinstance(b, (int, float)) and isinstance(a, Tensor):
        _check_float(a)
        if op == "add":
            return _scale(a, 1.0, float(b))
        if op == "sub":
            return _scale(a, 1.0, -float(b))
        if op == "mul":
            return _scale(a, float(b), 0.0)
    if isinstance(a, (int, float)) and isinstance(b, Tensor):
        _check_float(b)
        if op == "add":
            return _scale(b, 1.0, float(a))
        if op == "mul":
            return _scale(b, float(a), 0.0)
        if op == "sub":
            return _scale(b, -1.0, float(a))
    a = _as_tensor(a, like)
    b = _as_tensor(b, like)
    _check_float(a, b)
    shape = _broadcast(a.shape, b.shape)
    out = _binary_raw(op, a, b, shape)
    if _needs_grad(a, b):
        A, B = a.detach(), b.detach()
        need_a, need_b = a.requires_grad, b.requires_grad
        Y = out.detach()

        def backward(g, op=op):
            g = g[0]
            ga = gb = None
            if op == "add":
                ga = _sum_to(g, A.shape) if need_a else None
                gb = _sum_to(g, B.shape) if need_b else None
            elif op == "sub":
                ga = _sum_to(g, A.shape) if need_a else None
                gb = _sum_to(_unary_nograd("neg", g), B.shape) if need_b else None
            elif op == "mul":
                ga = _sum_to(_binary_raw("mul", g, B, g.shape), A.shape) if need_a else None
                gb = _sum_to(_binary_raw("mul", g, A, g.shape), B.shape) if need_b else None
            elif op == "div":
                ga = _sum_to(_binary_raw("div", g, B, g.shape), A.shape) if need_a else None
                if need_b:
                    t = _binary_raw("mul", g, Y, g.shape)
                    t = _binary_raw("div", t, B, g.shape)
                    gb = _sum_to(_unary_nograd("neg", t), B.shape)
            elif op in ("min", "max"):
                # ties go to the first operand
                mask = _binary_raw("le" if op == "min" else "ge", A, B, g.shape)
                if need_a:
                    ga = _sum_to(_binary_raw("mul", g, mask, g.shape), A.shape)
                if need_b:
                    inv = _scale_nograd(mask, -1.0, 1.0)
                    gb = _sum_to(_binary_raw("mul", g, inv, g.shape), B.shape)
            elif op == "pow":
                # d(a^b)/da = b a^(b-1), d(a^b)/db = a^b ln a
                if need_a:
                    t = _binary_raw("pow", A, _scale_nograd(B, 1.0, -1.0), g.shape)
                    t = _binary_raw("mul", t, B, g.shape)
                    ga = _sum_to(_binary_raw("mul", g, t, g.shape), A.shape)
                if need_b:
                    t = _binary_raw("mul", Y, _unary_nograd("log", A), g.shape)
                    gb = _sum_to(_binary_raw("mul", g, t, g.shape), B.shape)
            return [ga, gb]

        out._attach(Fn(op, [a, b], backward))
    return out


def _unary_nograd(op: str, x: Tensor) -> Tensor:
    out = Tensor._empty(x.shape, "float32", x.ctx)
    x.ctx.check(lib.tx_unary(x.ctx.handle, N.UN[op], x.ptr, out.ptr, x.numel, C.c_float(0), C.c_float(0)))
    return out


def _scale_nograd(x: Tensor, a: float, b: float) -> Tensor:
    out = Tensor._empty(x.shape, "float32", x.ctx)
    x.ctx.check(lib.tx_unary(x.ctx.handle, N.UN["scale"], x.ptr, out.ptr, x.numel, C.c_float(a),
                             C.c_float(b)))
    return out


def _repeat_plan(shape: tuple, sizes: tuple) -> tuple:
    """Tensor.repeat as reshape -> expand -> reshape: each axis of size s gets
    a unit axis before it that broadcasts to its repeat count r (leading sizes
    add axes of size 1 first); returns the three shapes."""
    if len(sizes) < len(shape):
        raise ValueError("repeat needs at least one size per axis")
    if any(not isinstance(r, (int, np.integer)) or r < 0 for r in sizes):
        raise ValueError("repeat sizes must be non-negative integers")
    full_shape = (1,) * (len(sizes) - len(shape)) + tuple(shape)
    inter, tiled = [], []
    for r, s in zip(sizes, full_shape):
        inter += [1, s]
        tiled += [int(r), s]
    return tuple(inter), tuple(tiled), tuple(int(r) * s for r, s in zip(sizes, full_shape))


def _index_plan(shape: tuple, index) -> tuple:
    """Basic indexing of a contiguous tensor of `shape` (integers, slices with
    any step, Ellipsis, None) as a strided view: (element offset of the first
    element, view shape, view strides in elements, result shape with the
    inserted unit axes)."""
    if not isinstance(index, tuple):
        index = (index,)
    if any(isinstance(i, (Tensor, list, np.ndarray)) for i in index):
        raise NotImplementedError("advanced indexing is not supported; use gather")
    ndim = len(shape)
    n_real = sum(1 for i in index if i is not None and i is not Ellipsis)
    if n_real > ndim:
        raise IndexError(f"too many indices for a tensor of rank {ndim}")
    if sum(1 for i in index if i is Ellipsis) > 1:
        raise IndexError("an index can only have a single ellipsis")
    expanded = []
    for i in index:
        if i is Ellipsis:
            expanded += [slice(None)] * (ndim - n_real)
        else:
            expanded.append(i)
    if Ellipsis not in index:
        expanded += [slice(None)] * (ndim - n_real)
    st = _contig_strides(shape)
    offset, vshape, strides, out_shape = 0, [], [], []
    axis = 0
    for i in expanded:
        if i is None:
            out_shape.append(1)
            continue
        dim = shape[axis]
        if isinstance(i, (int, np.integer)) and not isinstance(i, bool):
            k = int(i) + (dim if i < 0 else 0)
            if not 0 <= k < dim:
                raise IndexError(f"index {int(i)} is out of bounds for axis {axis} with size {dim}")
            offset += k * st[axis]
        elif isinstance(i, slice):
            start, stop, step = i.indices(dim)
            length = len(range(start, stop, step))
            offset += start * st[axis] if length else 0
            vshape.append(length)
            strides.append(step * st[axis])
            out_shape.append(length)
        else:
            raise TypeError(f"unsupported index {i!r}")
        axis += 1
    return offset, tuple(vshape), tuple(strides), tuple(out_shape)


def _getitem(x: Tensor, index) -> Tensor:
    """Basic indexing: integers, slices (any step), Ellipsis and None; a
    strided copy forward, a strided scatter into zeros backward (the Slice of
    the capture IR)."""
    offset, shape, strides, out_shape = _index_plan(tuple(x.shape), index)
    out = Tensor._empty(shape, x.dtype, x.ctx)
    if out.numel:
        x.ctx.check(lib.tx_strided_copy(x.ctx.handle, x.ptr + offset * x.itemsize, N.i64_array(strides), out.ptr,
                                        N.i64_array(shape), len(shape), x.itemsize))
    if _needs_grad(x):
        src_shape, base = x.shape, offset

        def backward(g, shape=shape, strides=strides):
            dx = full(src_shape, 0.0, ctx=g[0].ctx)
            if g[0].numel:
                g[0].ctx.check(lib.tx_strided_scatter(g[0].ctx.handle, g[0].ptr, dx.ptr + base * 4,
                                                      N.i64_array(strides), N.i64_array(shape), len(shape), 1))
            return [dx]

        out._attach(Fn("getitem", [x], backward))
    return out.reshape(out_shape) if out_shape != shape else out


def minimum(a, b) -> Tensor:
    return _binary("min", a, b)


def maximum(a, b) -> Tensor:
    return _binary("max", a, b)


def _reduce(x: Tensor, dim, keepdim: bool, mean: bool) -> Tensor:
    _check_float(x)
    if dim is None:
        axes = list(range(x.ndim))
    else:
        axes = [d % x.ndim for d in ([dim] if isinstance(dim, int) else dim)]
    keep = tuple(1 if i in axes else s for i, s in enumerate(x.shape))
    if dim is None:
        out_shape = (1,) if not keepdim else keep
    else:
        out_shape = keep if keepdim else tuple(s for i, s in enumerate(x.shape) if i not in axes)
    out = Tensor._empty(out_shape, "float32", x.ctx)
    x.ctx.check(lib.tx_reduce_to(x.ctx.handle, x.ptr, N.i64_array(x.shape), out.ptr, N.i64_array(keep),
                                 x.ndim, int(mean), 0))
    if _needs_grad(x):
        src = x.shape
        count = _numel(src) // max(_numel(keep), 1)

        def backward(g, keep=keep, src=src, count=count):
            gk = g[0].reshape(keep)
            scale = 1.0 / count if mean else 1.0
            out_g = Tensor._empty(src, "float32", gk.ctx)
            st = _bstrides(keep, src)
            # broadcast then scale (the copy kernel broadcasts; scale separately)
            gk.ctx.check(lib.tx_strided_copy(gk.ctx.handle, gk.ptr, N.i64_array(st), out_g.ptr,
                                             N.i64_array(src), len(src), 4))
            if scale != 1.0:
                out_g = _scale_nograd(out_g, scale, 0.0)
            return [out_g]

        out._attach(Fn("mean" if mean else "sum", [x], backward))
    return out


def _softmax(x: Tensor, dim: int, log: bool) -> Tensor:
    _check_float(x)
    dim = dim % x.ndim
    if dim != x.ndim - 1:
        moved = x.transpose(dim, x.ndim - 1)
        return _softmax(moved, -1, log).transpose(dim, x.ndim - 1)
    cols = x.shape[-1]
    rows = x.numel // cols if cols else 0
    out = Tensor._empty(x.shape, "float32", x.ctx)
    x.ctx.check(lib.tx_softmax_fwd(x.ctx.handle, x.ptr, out.ptr, rows, cols, int(log)))
    if _needs_grad(x):
        Y = out.detach()

        def backward(g, Y=Y):
            dx = Tensor._empty(Y.shape, "float32", Y.ctx)
            Y.ctx.check(lib.tx_softmax_bwd(Y.ctx.handle, Y.ptr, g[0].ptr, dx.ptr, rows, cols, int(log), 0))
            return [dx]

        out._attach(Fn("log_softmax" if log else "softmax", [x], backward))
    return out


def _gather(x: Tensor, dim: int, index: Tensor) -> Tensor:
    """``Tensor.gather(dim, index)`` for the last axis with one index per row."""
    if index.dtype != "int64":
        raise TypeError("gather index must be int64")
    dim = dim % x.ndim
    if dim != x.ndim - 1 or index.shape != x.shape[:-1] + (1,):
        raise NotImplementedError(
            "gather on CUDA supports the last axis with one index per row"
        )
    cols = x.shape[-1]
    rows = x.numel // cols
    out = Tensor._empty(index.shape, "float32", x.ctx)
    x.ctx.check(lib.tx_take_last(x.ctx.handle, x.ptr, index.ptr, out.ptr, rows, cols))
    if _needs_grad(x):
        idx = index.detach()
        src = x.shape

        def backward(g, idx=idx, src=src):
            dx = Tensor._empty(src, "float32", idx.ctx)
            idx.ctx.check(lib.tx_take_last_bwd(idx.ctx.handle, idx.ptr, g[0].ptr, dx.ptr, rows, cols, 0))
            return [dx]

        out._attach(Fn("gather", [x], backward))
    return out


def matmul(a: Tensor, b: Tensor) -> Tensor:
    """Rank-2 matmul on the tensor-core path (``DynTensor::matmul``, tensor.rs:1715)."""
    _check_float(a, b)
    if a.ndim != 2 or b.ndim != 2 or a.shape[1] != b.shape[0]:
        raise ValueError(f"matmul needs [M,K] x [K,N], got {a.shape} x {b.shape}")
    M, K = a.shape
    N_ = b.shape[1]
    out = Tensor._empty((M, N_), "float32", a.ctx)
    gemm(a.ctx, M, N_, K, a.ptr, K, False, b.ptr, N_, False, out.ptr, N_)
    if _needs_grad(a, b):
        A, B = a.detach(), b.detach()
        need_a, need_b = a.requires_grad, b.requires_grad

        def backward(g):
            g = g[0]
            ga = gb = None
            if need_a:
                ga = Tensor._empty((M, K), "float32", g.ctx)
                gemm(g.ctx, M, K, N_, g.ptr, N_, False, B.ptr, N_, True, ga.ptr, K)
            if need_b:
                gb = Tensor._empty((K, N_), "float32", g.ctx)
                gemm(g.ctx, K, N_, M, A.ptr, K, True, g.ptr, N_, False, gb.ptr, N_)
            return [ga, gb]

        out._attach(Fn("matmul", [a, b], backward))
    return out


def gemm(ctx: Context, M, N_, K, A, lda, ta, B, ldb, tb, Cp, ldc, *, alpha=1.0, beta=0.0,
         bias=None, bias_scale=1.0, act="none", flags=0, preact=None, ld_preact=0) -> None:
    d = N.GemmDesc()
    d.M, d.N, d.K = M, N_, K
    d.A, d.lda, d.trans_a = A, lda, int(ta)
    d.B, d.ldb, d.trans_b = B, ldb, int(tb)
    d.C, d.ldc = Cp, ldc
    d.alpha, d.beta = alpha, beta
    d.bias, d.bias_scale = bias, bias_scale
    d.act = N.ACT[act]
    d.batch = 1
    d.flags = flags
    if preact is not None:
        d.preact, d.ld_preact = preact, ld_preact or N_
    ctx.check(lib.tx_gemm(ctx.handle, C.byref(d)), "gemm")


# =============================================================================
# backward engine
# =============================================================================


def _accumulate(store: dict, key, g: Tensor) -> None:
    current = store.get(key)
    if current is None:
        store[key] = g
    else:
        store[key] = _binary_raw("add", current, g, current.shape)


def run_backward(roots: list, retain_graph: bool = False) -> None:
    """Walk the tape from ``roots`` = [(tensor, gradient)]."""
    order: list[Fn] = []
    seen: set[int] = set()
    stack = [(t._fn, False) for t, _ in roots if t._fn is not None]
    while stack:
        fn, done = stack.pop()
        if done:
            order.append(fn)
            continue
        if id(fn) in seen:
            continue
        seen.add(id(fn))
        stack.append((fn, True))
        for parent in fn.inputs:
            if parent is not None and parent._fn is not None and id(parent._fn) not in seen:
                stack.append((parent._fn, False))
    grads: dict = {}
    for t, g in roots:
        if t._fn is None:
            _accumulate_leaf(t, g)
        else:
            _accumulate(grads, (id(t._fn), t._out_index), g)
    for fn in reversed(order):
        outs = [grads.pop((id(fn), i), None) for i in range(fn.n_out)]
        if all(o is None for o in outs) or fn.backward is None:
            continue
        in_grads = fn.backward(outs)
        for parent, g in zip(fn.inputs, in_grads):
            if parent is None or g is None or not parent.requires_grad:
                continue
            if parent._fn is None:
                _accumulate_leaf(parent, g)
            else:
                _accumulate(grads, (id(parent._fn), parent._out_index), g)
        if not retain_graph:
            fn.free()


def _accumulate_leaf(t: Tensor, g: Tensor) -> None:
    if g.shape != t.shape:
        g = _sum_to(g, t.shape)
    accumulate = getattr(t, "_accumulate_grad", None)
    if accumulate is not None:
        accumulate(g)
        return
    if t._grad is None:
        t._grad = g.detach()
    else:
        t._grad = _binary_raw("add", t._grad, g, t.shape)


# =============================================================================
# factories
# =============================================================================


class _Pinned:
    __slots__ = ("ptr",)

    def __init__(self, nbytes: int):
        out = C.c_void_p()
        if lib.tx_host_alloc(max(nbytes, 1), C.byref(out)) != N.TX_OK:
            raise MemoryError("pinned host allocation failed")
        self.ptr = out.value

    def __del__(self):
        try:
            lib.tx_host_free(self.ptr)
        except Exception:
            pass


def pinned(array) -> np.ndarray:
    """Copy ``array`` into page-locked host memory (for fast, async H2D copies)."""
    src = np.ascontiguousarray(array)
    holder = _Pinned(src.nbytes)
    raw = (C.c_uint8 * max(src.nbytes, 1)).from_address(holder.ptr)
    out = np.frombuffer(raw, dtype=src.dtype, count=src.size).reshape(src.shape)
    out[...] = src
    _PINNED_OWNERS[id(out)] = holder
    return out


_PINNED_OWNERS: dict = {}


class _RingStorage(Storage):
    """A buffer of a Prefetcher ring: not owned; keeps the ring alive."""

    __slots__ = ("ring",)

    def __init__(self, ctx: Context, nbytes: int, ptr: int, ring: "Prefetcher"):
        super().__init__(ctx, nbytes, ptr=ptr, owned=False)
        self.ring = ring


class Prefetcher:
    """Uploads input batches on a copy stream beside the compute stream.

    ``Prefetcher(*like, depth=3)`` sets up, for each array of a batch (shaped
    and typed like ``like``), ``depth`` device buffers.  ``put(*arrays)`` queues
    one batch's upload and returns at once; ``get()`` returns the oldest queued
    batch as Tensors, and device work issued after it waits for that upload.
    A training loop keeps ``depth - 1`` batches in flight::

        pf.put(*batch[0]); pf.put(*batch[1])
        for i in range(steps):
            x, y = pf.get()
            loss = step(x, y)
            if i + 2 < steps:
                pf.put(*batch[i + 2])
            loss.item()

    so the uploads run while the steps do.  Sources should be page-locked
    (``pinned``) and must stay alive and unchanged until their upload has run.
    A batch from ``get`` stays valid for the device work issued before the
    next ``get``: after that call its buffer may be refilled by a ``put``, so
    keep a copy (``clone()``) of anything needed longer.
    """

    def __init__(self, *like, depth: int = 3, device: Optional[Device] = None):
        if depth < 2:
            raise ValueError("Prefetcher needs depth >= 2")
        self._ctx = context(device)
        self._rings: list = []
        self._specs: list = []
        for a in like:
            a = np.asarray(a)
            dtype = _dtype_of(a)
            nbytes = a.size * _DTYPES[dtype][1]
            h = C.c_void_p()
            check(lib.tx_prefetch_create(self._ctx.handle, max(nbytes, 1), depth, C.byref(h)),
                  self._ctx.handle, "prefetcher")
            self._rings.append(h.value)
            self._specs.append((a.shape, dtype, nbytes))

    def put(self, *arrays) -> None:
        if len(arrays) != len(self._specs):
            raise ValueError(f"expected {len(self._specs)} arrays, got {len(arrays)}")
        for (shape, dtype, _), a in zip(self._specs, arrays):
            if not isinstance(a, np.ndarray) or a.shape != shape or a.dtype != _DTYPES[dtype][0] \
                    or not a.flags["C_CONTIGUOUS"]:
                raise TypeError(f"put expects a C-contiguous {dtype} array of shape {shape}")
        for ring, (_, _, nbytes), a in zip(self._rings, self._specs, arrays):
            check(lib.tx_prefetch_put(ring, a.ctypes.data, nbytes), self._ctx.handle, "prefetch put")

    def get(self) -> tuple:
        out = []
        for ring, (shape, dtype, nbytes) in zip(self._rings, self._specs):
            d = C.c_void_p()
            check(lib.tx_prefetch_get(ring, C.byref(d)), self._ctx.handle, "prefetch get")
            out.append(Tensor._view(_RingStorage(self._ctx, nbytes, d.value, self), 0, shape, dtype))
        return tuple(out)

    def close(self) -> None:
        for ring in self._rings:
            lib.tx_prefetch_destroy(ring)
        self._rings = []

    def __del__(self):
        try:
            self.close()
        except Exception:  # interpreter shutdown
            pass


def _dtype_of(array: np.ndarray) -> str:
    if array.dtype == np.bool_:
        return "bool"
    if np.issubdtype(array.dtype, np.integer):
        return "int64"
    return "float32"


def tensor(data, *, dtype: Optional[str] = None, device: Optional[Device] = None,
           requires_grad: bool = False) -> Tensor:
    return Tensor(data, dtype=dtype, device=device, requires_grad=requires_grad)


def zeros(*shape, dtype: str = "float32", device: Optional[Device] = None) -> Tensor:
    shape = shape[0] if len(shape) == 1 and isinstance(shape[0], (tuple, list)) else shape
    return full(shape, 0.0, ctx=context(device), dtype=dtype)


def ones(*shape, dtype: str = "float32", device: Optional[Device] = None) -> Tensor:
    shape = shape[0] if len(shape) == 1 and isinstance(shape[0], (tuple, list)) else shape
    return full(shape, 1.0, ctx=context(device), dtype=dtype)


def zeros_like(t: Tensor) -> Tensor:
    return full(t.shape, 0.0, ctx=t.ctx, dtype=t.dtype)


def ones_like(t: Tensor) -> Tensor:
    return full(t.shape, 1.0, ctx=t.ctx, dtype=t.dtype)


def full_like(t: Tensor, value: float) -> Tensor:
    return full(t.shape, value, ctx=t.ctx, dtype=t.dtype)


def randn(*shape, seed: Optional[int] = None, device: Optional[Device] = None) -> Tensor:
    shape = shape[0] if len(shape) == 1 and isinstance(shape[0], (tuple, list)) else shape
    rng = np.random.default_rng(seed)
    return Tensor(rng.standard_normal(shape).astype(np.float32), device=device)


def rand(*shape, seed: Optional[int] = None, device: Optional[Device] = None) -> Tensor:
    shape = shape[0] if len(shape) == 1 and isinstance(shape[0], (tuple, list)) else shape
    rng = np.random.default_rng(seed)
    return Tensor(rng.random(shape, dtype=np.float32), device=device)


def arange(n: int, device: Optional[Device] = None) -> Tensor:
    return Tensor(np.arange(n, dtype=np.int64), device=device)


def cat(tensors: Iterable[Tensor], dim: int = 0) -> Tensor:
    tensors = list(tensors)
    return Tensor(np.concatenate([t.numpy() for t in tensors], axis=dim), device=tensors[0].device)
