"""CPU oracle: a numpy restatement of Tynx's Flex training semantics.

TEST INFRASTRUCTURE ONLY.  Nothing in the product imports this module; only
``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg use
it, and only as the checker or the timed CPU reference.

What it restates (the reference delegates all arithmetic to Burn, which is not
vendored: ``burn-flex`` / ``burn-autodiff`` 0.22.0-pre.1 at rev 78f10aec,
``Cargo.lock:348-700``; the algorithms below are the mathematical definitions
of those operators as Tynx composes them):

* the imported-model executor (``crates/tynx-train/src/imported_model/executor.rs:107-161``),
  with Gemm alpha/beta/trans semantics (``executor.rs:499-524``, ``add_bias`` 606-613),
  ONNX/numpy MatMul (``crates/tynx/src/interpreter/matrix.rs:238-318``),
  NCHW Conv (``crates/tynx/src/tensor.rs:1080-1180``), Gather
  (``crates/tynx/src/interpreter/gather.rs:18-58``, negative-index normalisation
  ``tensor.rs:2504``), LayerNormalization composed from mean / centre / mean of
  squares / ``powf(-0.5)`` (``crates/tynx/src/interpreter/normalization.rs:135-190``),
  exact-erf GELU (``crates/tynx/src/interpreter/unary.rs:234-237``), stable
  softmax / log-softmax (``crates/tynx/src/interpreter/softmax.rs:9-17``);
* reverse-mode autodiff with per-parameter gradient accumulation
  (``crates/tynx-train/src/autograd.rs:56-95``, ``parameter.rs:300-333``);
* losses: cross entropy as ``-mean(log_softmax(z)[y])``
  (``crates/tynx-python/python/tynx/nn/functional.py:133-145``), MSE
  (``crates/tynx-train/src/loss.rs:10-23``), Categorical log-prob / entropy
  (``crates/tynx-python/python/tynx/distributions.py:47-104``);
* Adam / AdamW with f64 bias corrections folded into f32 ops in the same order
  (``crates/tynx-train/src/optimizer/adam.rs:431-527``) and SGD with momentum /
  dampening / nesterov (``crates/tynx-train/src/optimizer.rs:310-356``).

All tensors are float32 (int64 for indices), as in Flex.  Scalars that Burn
receives as f64 (``mul_scalar(f64)``) are rounded to float32 before use.
"""

from __future__ import annotations

import math
from contextlib import contextmanager
from typing import Callable, Optional

import numpy as np

try:  # scipy ships in the image; the fallback keeps the oracle importable without it
    from scipy.special import erf as _erf
except Exception:  # pragma: no cover
    _erf = np.vectorize(math.erf)

F32 = np.float32  # the working precision; `precision(np.float64)` switches it for checks


def f32(x) -> np.float32:
    return F32(x)


@contextmanager
def precision(dtype):
    """Run the oracle in another floating precision (float64 gives the exact
    reference that fp32 implementations are measured against)."""
    global F32
    previous = F32
    F32 = dtype
    try:
        yield
    finally:
        F32 = previous


# =============================================================================
# reverse-mode tape
# =============================================================================


class T:
    """An oracle tensor: numpy value + optional gradient tape node."""

    __slots__ = ("data", "grad", "requires_grad", "_parents", "_backward", "name")

    def __init__(self, data, requires_grad: bool = False, name: str = ""):
        arr = np.asarray(data)
        if arr.dtype.kind == "f" and arr.dtype != F32:
            arr = arr.astype(F32)
        self.data = arr
        self.grad: Optional[np.ndarray] = None
        self.requires_grad = requires_grad
        self._parents: tuple = ()
        self._backward: Optional[Callable[[np.ndarray], tuple]] = None
        self.name = name

    # -- plumbing ---------------------------------------------------------------
    @property
    def shape(self):
        return self.data.shape

    def numpy(self) -> np.ndarray:
        return self.data

    def item(self) -> float:
        return float(self.data.reshape(-1)[0])

    def detach(self) -> "T":
        return T(self.data)

    def __repr__(self) -> str:  # pragma: no cover
        return f"T({self.data!r})"

    def backward(self, grad: Optional[np.ndarray] = None) -> None:
        """Walk the tape from this tensor; leaves accumulate into ``.grad``."""
        if grad is None:
            if self.data.size != 1:
                raise ValueError("backward() without a gradient requires a one-element tensor")
            grad = np.ones_like(self.data, dtype=F32)
        order: list[T] = []
        seen: set[int] = set()

        def visit(node: T) -> None:
            stack = [(node, False)]
            while stack:
                current, done = stack.pop()
                if done:
                    order.append(current)
                    continue
                if id(current) in seen:
                    continue
                seen.add(id(current))
                stack.append((current, True))
                for parent in current._parents:
                    if parent is not None and parent.requires_grad:
                        stack.append((parent, False))

        visit(self)
        grads: dict[int, np.ndarray] = {id(self): grad.astype(F32)}
        for node in reversed(order):
            g = grads.pop(id(node), None)
            if g is None:
                continue
            if node._backward is None:  # leaf
                node.grad = g.copy() if node.grad is None else (node.grad + g).astype(F32)
                continue
            parent_grads = node._backward(g)
            for parent, pg in zip(node._parents, parent_grads):
                if parent is None or not parent.requires_grad or pg is None:
                    continue
                pg = np.asarray(pg, dtype=F32).reshape(parent.data.shape)
                if id(parent) in grads:
                    grads[id(parent)] = grads[id(parent)] + pg
                else:
                    grads[id(parent)] = pg

    # -- operators --------------------------------------------------------------
    def __add__(self, other):
        return add(self, _wrap(other, self))

    __radd__ = __add__

    def __sub__(self, other):
        return sub(self, _wrap(other, self))

    def __rsub__(self, other):
        return sub(_wrap(other, self), self)

    def __mul__(self, other):
        return mul(self, _wrap(other, self))

    __rmul__ = __mul__

    def __truediv__(self, other):
        return div(self, _wrap(other, self))

    def __neg__(self):
        return neg(self)


def _wrap(value, like: T) -> T:
    if isinstance(value, T):
        return value
    return T(np.asarray(value, dtype=like.data.dtype if like.data.dtype == F32 else F32))


def _node(data: np.ndarray, parents: tuple, backward) -> T:
    out = T(data)
    if any(p is not None and p.requires_grad for p in parents):
        out.requires_grad = True
        out._parents = parents
        out._backward = backward
    return out


def _unbroadcast(grad: np.ndarray, shape: tuple) -> np.ndarray:
    """Sum a broadcast gradient back down to ``shape``."""
    if grad.shape == tuple(shape):
        return grad
    extra = grad.ndim - len(shape)
    if extra > 0:
        grad = grad.sum(axis=tuple(range(extra)), dtype=F32)
    axes = tuple(i for i, (g, s) in enumerate(zip(grad.shape, shape)) if s == 1 and g != 1)
    if axes:
        grad = grad.sum(axis=axes, keepdims=True, dtype=F32)
    return grad.reshape(shape)


# -- elementwise ---------------------------------------------------------------


def add(a: T, b: T) -> T:
    return _node((a.data + b.data).astype(a.data.dtype), (a, b),
                 lambda g: (_unbroadcast(g, a.shape), _unbroadcast(g, b.shape)))


def sub(a: T, b: T) -> T:
    return _node((a.data - b.data).astype(a.data.dtype), (a, b),
                 lambda g: (_unbroadcast(g, a.shape), _unbroadcast(-g, b.shape)))


def mul(a: T, b: T) -> T:
    return _node((a.data * b.data).astype(F32), (a, b),
                 lambda g: (_unbroadcast(g * b.data, a.shape), _unbroadcast(g * a.data, b.shape)))


def div(a: T, b: T) -> T:
    out = (a.data / b.data).astype(F32)
    return _node(out, (a, b),
                 lambda g: (_unbroadcast(g / b.data, a.shape),
                            _unbroadcast(-g * a.data / (b.data * b.data), b.shape)))


def neg(a: T) -> T:
    return _node(-a.data, (a,), lambda g: (-g,))


def exp(a: T) -> T:
    out = np.exp(a.data).astype(F32)
    return _node(out, (a,), lambda g: (g * out,))


def log(a: T) -> T:
    return _node(np.log(a.data).astype(F32), (a,), lambda g: (g / a.data,))


def relu(a: T) -> T:
    mask = a.data > 0
    return _node(np.where(mask, a.data, F32(0)), (a,), lambda g: (np.where(mask, g, F32(0)),))


def tanh(a: T) -> T:
    out = np.tanh(a.data).astype(F32)
    return _node(out, (a,), lambda g: (g * (F32(1) - out * out),))


def sigmoid(a: T) -> T:
    out = (1.0 / (1.0 + np.exp(-a.data.astype(np.float64)))).astype(F32)
    return _node(out, (a,), lambda g: (g * out * (F32(1) - out),))


def gelu(a: T) -> T:
    """Exact GELU x * Phi(x); ONNX ``approximate`` is ignored like the reference."""
    x = a.data.astype(np.float64)
    cdf = 0.5 * (1.0 + _erf(x / math.sqrt(2.0)))
    out = (x * cdf).astype(F32)
    pdf = np.exp(-0.5 * x * x) / math.sqrt(2.0 * math.pi)
    dgelu = (cdf + x * pdf).astype(F32)
    return _node(out, (a,), lambda g: (g * dgelu,))


def clamp(a: T, lo: Optional[float], hi: Optional[float]) -> T:
    out = a.data
    inside = np.ones(a.shape, dtype=bool)
    if lo is not None:
        inside &= a.data >= F32(lo)
        out = np.maximum(out, F32(lo))
    if hi is not None:
        inside &= a.data <= F32(hi)
        out = np.minimum(out, F32(hi))
    return _node(out.astype(F32), (a,), lambda g: (np.where(inside, g, F32(0)),))


def minimum(a: T, b: T) -> T:
    take_a = a.data <= b.data
    out = np.where(take_a, a.data, b.data).astype(F32)
    return _node(out, (a, b), lambda g: (_unbroadcast(np.where(take_a, g, F32(0)), a.shape),
                                         _unbroadcast(np.where(take_a, F32(0), g), b.shape)))


def maximum(a: T, b: T) -> T:
    take_a = a.data >= b.data
    out = np.where(take_a, a.data, b.data).astype(F32)
    return _node(out, (a, b), lambda g: (_unbroadcast(np.where(take_a, g, F32(0)), a.shape),
                                         _unbroadcast(np.where(take_a, F32(0), g), b.shape)))


def prelu(a: T, slope: T) -> T:
    pos = a.data >= 0
    out = np.where(pos, a.data, a.data * slope.data).astype(F32)
    return _node(out, (a, slope),
                 lambda g: (np.where(pos, g, g * slope.data),
                            _unbroadcast(np.where(pos, F32(0), g * a.data), slope.shape)))


# -- reductions / shape ----------------------------------------------------------


def sum_(a: T, axes=None, keepdims: bool = False) -> T:
    if axes is None:
        out = np.asarray(a.data.sum(dtype=F32)).reshape(1) if not keepdims else \
            a.data.sum(keepdims=True, dtype=F32)
        return _node(out, (a,), lambda g: (np.broadcast_to(g.reshape(-1)[0], a.shape),))
    axes = tuple(ax % a.data.ndim for ax in np.atleast_1d(axes))
    out = a.data.sum(axis=axes, keepdims=keepdims, dtype=F32)

    def back(g):
        if not keepdims:
            g = np.expand_dims(g, axes)
        return (np.broadcast_to(g, a.shape),)

    return _node(out, (a,), back)


def mean(a: T, axes=None, keepdims: bool = False) -> T:
    if axes is None:
        n = a.data.size
        out = np.asarray(a.data.mean(dtype=F32), dtype=F32).reshape(1)
        return _node(out, (a,), lambda g: (np.full(a.shape, g.reshape(-1)[0] / F32(n), dtype=F32),))
    axes = tuple(ax % a.data.ndim for ax in np.atleast_1d(axes))
    n = int(np.prod([a.data.shape[ax] for ax in axes]))
    out = a.data.mean(axis=axes, keepdims=keepdims, dtype=F32)

    def back(g):
        if not keepdims:
            g = np.expand_dims(g, axes)
        return (np.broadcast_to(g / F32(n), a.shape),)

    return _node(out, (a,), back)


def reshape(a: T, shape) -> T:
    return _node(a.data.reshape(shape), (a,), lambda g: (g.reshape(a.shape),))


def transpose(a: T, perm) -> T:
    inverse = np.argsort(perm)
    return _node(np.ascontiguousarray(a.data.transpose(perm)), (a,),
                 lambda g: (g.transpose(inverse),))


def expand(a: T, shape) -> T:
    return _node(np.broadcast_to(a.data, shape).copy(), (a,),
                 lambda g: (_unbroadcast(g, a.shape),))


def softmax(a: T, axis: int) -> T:
    x = a.data
    shifted = x - x.max(axis=axis, keepdims=True)
    e = np.exp(shifted)
    out = (e / e.sum(axis=axis, keepdims=True, dtype=F32)).astype(F32)
    return _node(out, (a,),
                 lambda g: (out * (g - (g * out).sum(axis=axis, keepdims=True, dtype=F32)),))


def log_softmax(a: T, axis: int) -> T:
    x = a.data
    shifted = x - x.max(axis=axis, keepdims=True)
    lse = np.log(np.exp(shifted).sum(axis=axis, keepdims=True, dtype=F32))
    out = (shifted - lse).astype(F32)
    soft = np.exp(out)
    return _node(out, (a,), lambda g: (g - soft * g.sum(axis=axis, keepdims=True, dtype=F32),))


def take_along(a: T, axis: int, index: np.ndarray) -> T:
    """``Tensor.gather(dim, index)`` (PyTorch-style gather along one axis)."""
    idx = np.asarray(index, dtype=np.int64)
    out = np.take_along_axis(a.data, idx, axis=axis)

    def back(g):
        full = np.zeros(a.shape, dtype=F32)
        np.put_along_axis(full, idx, 0, axis=axis)  # shape check only
        grid = list(np.indices(idx.shape, sparse=True))
        grid[axis] = idx
        np.add.at(full, tuple(grid), g)
        return (full,)

    return _node(out, (a,), back)


def normalize_indices(indices: np.ndarray, size: int) -> np.ndarray:
    """Negative indices wrap once; anything outside ``[-size, size)`` is an error
    (``DynInt::normalize_indices``, ``crates/tynx/src/tensor.rs:2504``)."""
    idx = np.asarray(indices, dtype=np.int64)
    if idx.size and (idx.min() < -size or idx.max() >= size):
        raise IndexError(f"index out of range for axis of size {size}")
    return np.where(idx < 0, idx + size, idx)


def gather(data: T, indices: np.ndarray, axis: int) -> T:
    """ONNX Gather (``np.take``); backward scatter-adds repeated rows."""
    axis = axis % data.data.ndim
    idx = normalize_indices(indices, data.shape[axis])
    out = np.take(data.data, idx, axis=axis)

    def back(g):
        full = np.zeros(data.shape, dtype=F32)
        moved = np.moveaxis(full, axis, 0)
        gm = g.reshape(data.shape[:axis] + (idx.size,) + data.shape[axis + 1:])
        np.add.at(moved, idx.reshape(-1), np.moveaxis(gm, axis, 0))
        return (full,)

    return _node(out, (data,), back)


def matmul(a: T, b: T) -> T:
    """ONNX/numpy MatMul including rank-1 promotion and batch broadcasting."""
    A, B = a.data, b.data
    a1, b1 = A.ndim == 1, B.ndim == 1
    A2 = A[None, :] if a1 else A
    B2 = B[:, None] if b1 else B
    out = np.matmul(A2, B2).astype(F32)
    res = out
    if a1:
        res = res[..., 0, :]
    if b1:
        res = res[..., 0]

    def back(g):
        G = g
        if a1:
            G = np.expand_dims(G, -2)
        if b1:
            G = np.expand_dims(G, -1)
        ga = np.matmul(G, np.swapaxes(B2, -1, -2))
        gb = np.matmul(np.swapaxes(A2, -1, -2), G)
        ga = _unbroadcast(ga, A2.shape)
        gb = _unbroadcast(gb, B2.shape)
        return (ga.reshape(A.shape), gb.reshape(B.shape))

    return _node(np.ascontiguousarray(res), (a, b), back)


# -- convolution -------------------------------------------------------------------


def _im2col(x: np.ndarray, kh, kw, sh, sw, dh, dw, oh, ow) -> np.ndarray:
    """[N, C, Hp, Wp] -> [N, OH, OW, C, KH, KW] strided view."""
    n, c, _, _ = x.shape
    s = x.strides
    return np.lib.stride_tricks.as_strided(
        x,
        shape=(n, oh, ow, c, kh, kw),
        strides=(s[0], s[2] * sh, s[3] * sw, s[1], s[2] * dh, s[3] * dw),
        writeable=False,
    )


def conv2d(x: T, w: T, b: Optional[T], strides, pads, dilations, group: int = 1) -> T:
    """NCHW convolution as an implicit GEMM over im2col columns.

    ``pads`` is ONNX order ``[top, left, bottom, right]``.
    """
    X, W = x.data, w.data
    n, c, h, wd = X.shape
    oc, cpg, kh, kw = W.shape
    sh, sw = strides
    dh, dw = dilations
    pt, pl, pb, pr = pads
    if c != cpg * group or oc % group:
        raise ValueError("Conv channel/group mismatch")
    Xp = np.pad(X, ((0, 0), (0, 0), (pt, pb), (pl, pr)))
    oh = (h + pt + pb - dh * (kh - 1) - 1) // sh + 1
    ow = (wd + pl + pr - dw * (kw - 1) - 1) // sw + 1
    ocg = oc // group
    outs = []
    cols_g = []
    for gi in range(group):
        cols = _im2col(np.ascontiguousarray(Xp[:, gi * cpg:(gi + 1) * cpg]), kh, kw, sh, sw, dh,
                       dw, oh, ow).reshape(n * oh * ow, cpg * kh * kw)
        Wg = W[gi * ocg:(gi + 1) * ocg].reshape(ocg, -1)
        outs.append(cols @ Wg.T)
        cols_g.append(cols)
    Y = np.concatenate(outs, axis=1).reshape(n, oh, ow, oc).transpose(0, 3, 1, 2)
    if b is not None:
        Y = Y + b.data.reshape(1, oc, 1, 1)
    Y = np.ascontiguousarray(Y, dtype=F32)

    def back(g):
        G = g.transpose(0, 2, 3, 1).reshape(n * oh * ow, oc)
        dW = np.zeros_like(W)
        dXp = np.zeros(Xp.shape, dtype=F32)
        for gi in range(group):
            Gg = G[:, gi * ocg:(gi + 1) * ocg]
            dW[gi * ocg:(gi + 1) * ocg] = (Gg.T @ cols_g[gi]).reshape(ocg, cpg, kh, kw)
            dcols = (Gg @ W[gi * ocg:(gi + 1) * ocg].reshape(ocg, -1)).reshape(
                n, oh, ow, cpg, kh, kw)
            for i in range(kh):
                for j in range(kw):
                    dXp[:, gi * cpg:(gi + 1) * cpg,
                        i * dh: i * dh + sh * (oh - 1) + 1: sh,
                        j * dw: j * dw + sw * (ow - 1) + 1: sw] += \
                        dcols[:, :, :, :, i, j].transpose(0, 3, 1, 2)
        dX = dXp[:, :, pt:pt + h, pl:pl + wd]
        db = G.sum(axis=0, dtype=F32) if b is not None else None
        return (dX, dW, db)

    return _node(Y, (x, w, b), back)


# =============================================================================
# ONNX interpreter over a TrainingGraph (executor.rs:107-161)
# =============================================================================


class OracleModel:
    """Slot-backed imported model: parameters are persistent leaves."""

    def __init__(self, graph):
        self.graph = graph
        self.params: dict[str, T] = {
            name: T(value.copy(), requires_grad=True, name=name)
            for name, value in graph.parameters.items()
        }

    def named_parameters(self) -> list[tuple[str, T]]:
        return list(self.params.items())

    def zero_grad(self) -> None:
        for p in self.params.values():
            p.grad = None

    def _value(self, env: dict, name: str):
        if name in env:
            return env[name]
        if name in self.graph.parameter_of_value:
            return self.params[self.graph.parameter_of_value[name]]
        if name in self.graph.constants:
            return T(self.graph.constants[name])
        raise KeyError(f"value {name!r} is not defined")

    def __call__(self, *inputs, **named):
        env: dict[str, T] = {}
        for info, value in zip(self.graph.inputs, inputs):
            env[info.name] = value if isinstance(value, T) else T(value)
        for key, value in named.items():
            env[key] = value if isinstance(value, T) else T(value)
        for op in self.graph.ops:
            vals = [self._value(env, i) if i else None for i in op.inputs]
            outs = run_op(op, vals)
            for name, out in zip(op.outputs, outs):
                env[name] = out
        results = [env[o] for o in self.graph.outputs]
        return results[0] if len(results) == 1 else {o: env[o] for o in self.graph.outputs}


def _const_ints(value: Optional[T]) -> list[int]:
    return [] if value is None else [int(v) for v in np.asarray(value.data).reshape(-1)]


def run_op(op, vals: list) -> list:
    t = op.op_type
    a = op.attrs
    x = vals[0] if vals else None
    if t == "Gemm":
        A, B = vals[0], vals[1]
        if a["transA"]:
            A = transpose(A, (1, 0))
        if a["transB"]:
            B = transpose(B, (1, 0))
        y = matmul(A, B) * T(np.asarray(a["alpha"], dtype=F32))
        if len(vals) > 2 and vals[2] is not None:
            y = y + vals[2] * T(np.asarray(a["beta"], dtype=F32))
        return [y]
    if t == "MatMul":
        return [matmul(vals[0], vals[1])]
    if t == "Add":
        return [vals[0] + vals[1]]
    if t == "Sub":
        return [vals[0] - vals[1]]
    if t == "Mul":
        return [vals[0] * vals[1]]
    if t == "Div":
        return [vals[0] / vals[1]]
    if t == "Relu":
        return [relu(x)]
    if t == "Tanh":
        return [tanh(x)]
    if t == "Sigmoid":
        return [sigmoid(x)]
    if t == "Gelu":
        return [gelu(x)]
    if t == "Exp":
        return [exp(x)]
    if t == "Log":
        return [log(x)]
    if t == "Neg":
        return [neg(x)]
    if t == "Identity":
        return [x]
    if t == "PRelu":
        return [prelu(x, vals[1])]
    if t == "Clip":
        lo = float(vals[1].data.reshape(-1)[0]) if len(vals) > 1 and vals[1] is not None else a.get("min")
        hi = float(vals[2].data.reshape(-1)[0]) if len(vals) > 2 and vals[2] is not None else a.get("max")
        return [clamp(x, lo, hi)]
    if t == "Softmax":
        return [softmax(x, a["axis"])]
    if t == "LogSoftmax":
        return [log_softmax(x, a["axis"])]
    if t == "LayerNormalization":
        return layer_norm(x, vals[1], vals[2] if len(vals) > 2 else None, a["axis"],
                          a["epsilon"], len(op.outputs))
    if t == "Gather":
        return [gather(x, vals[1].data, a["axis"])]
    if t == "Reshape":
        shape = _const_ints(vals[1])
        target = [x.shape[i] if s == 0 and not a.get("allowzero", 0) else s
                  for i, s in enumerate(shape)]
        return [reshape(x, target)]
    if t == "Transpose":
        perm = a.get("perm") or list(reversed(range(x.data.ndim)))
        return [transpose(x, perm)]
    if t == "Flatten":
        axis = a["axis"] % max(x.data.ndim, 1) if a["axis"] < 0 else a["axis"]
        lead = int(np.prod(x.shape[:axis])) if axis else 1
        return [reshape(x, (lead, -1))]
    if t in ("Squeeze", "Unsqueeze"):
        axes = a.get("axes") or _const_ints(vals[1] if len(vals) > 1 else None)
        if t == "Squeeze":
            if not axes:
                axes = [i for i, s in enumerate(x.shape) if s == 1]
            nd = x.data.ndim
            axes = sorted(ax % nd for ax in axes)
            shape = [s for i, s in enumerate(x.shape) if i not in axes]
        else:
            nd = x.data.ndim + len(axes)
            axes = sorted(ax % nd for ax in axes)
            shape = list(x.shape)
            for ax in axes:
                shape.insert(ax, 1)
        return [reshape(x, shape)]
    if t in ("ReduceMean", "ReduceSum"):
        axes = a.get("axes") or _const_ints(vals[1] if len(vals) > 1 else None)
        axes = axes or list(range(x.data.ndim))
        fn = mean if t == "ReduceMean" else sum_
        return [fn(x, tuple(axes), keepdims=bool(a["keepdims"]))]
    if t == "GlobalAveragePool":
        return [mean(x, tuple(range(2, x.data.ndim)), keepdims=True)]
    if t == "Conv":
        W = vals[1]
        nd = W.data.ndim - 2
        strides = a.get("strides") or [1] * nd
        dil = a.get("dilations") or [1] * nd
        pads = a.get("pads") or [0] * (2 * nd)
        if nd == 1:
            x4 = reshape(x, (x.shape[0], x.shape[1], 1, x.shape[2]))
            w4 = reshape(W, (W.shape[0], W.shape[1], 1, W.shape[2]))
            y = conv2d(x4, w4, vals[2] if len(vals) > 2 else None, (1, strides[0]),
                       (0, pads[0], 0, pads[1]), (1, dil[0]), a["group"])
            return [reshape(y, (y.shape[0], y.shape[1], y.shape[3]))]
        if nd != 2:
            raise NotImplementedError("oracle Conv supports 1-D and 2-D kernels")
        return [conv2d(x, W, vals[2] if len(vals) > 2 else None, strides, pads, dil, a["group"])]
    if t == "BatchNormalization":
        return [batch_norm(x, vals[1], vals[2], vals[3], vals[4], a["epsilon"])]
    if t == "InstanceNormalization":
        return [group_norm(x, vals[1], vals[2], x.shape[1], a["epsilon"])]
    if t == "GroupNormalization":
        return [group_norm(x, vals[1], vals[2], int(a["num_groups"]), a["epsilon"])]
    if t == "MaxPool":
        return [max_pool(x, a)]
    if t in _UNARY_RULES:
        return [_unary(x, t, a)]
    if t == "Pow":
        if vals[1].data.size == 1:
            return [power(x, float(vals[1].data.reshape(-1)[0]))]
        return [pow_(x, vals[1])]
    if t in ("Max", "Min"):
        out = vals[0]
        for v in vals[1:]:
            out = maximum(out, v) if t == "Max" else minimum(out, v)
        return [out]
    if t == "Concat":
        return [concat(vals, a["axis"])]
    if t == "Slice":
        if len(vals) > 1:
            starts, ends = _const_ints(vals[1]), _const_ints(vals[2])
            axes = _const_ints(vals[3]) if len(vals) > 3 and vals[3] is not None else list(range(len(starts)))
            steps = _const_ints(vals[4]) if len(vals) > 4 and vals[4] is not None else [1] * len(starts)
        else:
            starts, ends = list(a["starts"]), list(a["ends"])
            axes = list(a.get("axes") or range(len(starts)))
            steps = [1] * len(starts)
        return [slice_(x, starts, ends, axes, steps)]
    if t == "Split":
        sizes = a.get("split") or (_const_ints(vals[1]) if len(vals) > 1 and vals[1] is not None else None)
        axis = a["axis"] % x.data.ndim
        if not sizes:
            n_out = len(op.outputs)
            part = -(-x.shape[axis] // n_out)
            sizes = [min(part, x.shape[axis] - part * i) for i in range(n_out)]
        outs, at = [], 0
        for size in sizes:
            outs.append(slice_(x, [at], [at + size], [axis], [1]))
            at += size
        return outs
    if t == "Expand":
        target = _const_ints(vals[1])
        shape = np.broadcast_shapes(tuple(x.shape), tuple(target))
        return [expand(x, shape)]
    if t == "AveragePool":
        return [avg_pool(x, a)]
    if t in ("ReduceMax", "ReduceMin", "GlobalMaxPool"):
        if t == "GlobalMaxPool":
            axes, keep = list(range(2, x.data.ndim)), True
        else:
            axes = a.get("axes") or _const_ints(vals[1] if len(vals) > 1 else None)
            axes, keep = axes or list(range(x.data.ndim)), bool(a["keepdims"])
        return [extremum(x, axes, keep, t != "ReduceMin")]
    if t == "Dropout":
        return [x]
    raise NotImplementedError(f"oracle has no rule for {t}")


# -- the inference arms of interpreter/unary.rs, pow.rs, concat.rs, slice.rs,
# split.rs, expand.rs, pooling.rs and reduction.rs (forward) with the
# derivatives backward_support.rs validates --------------------------------------

def _erf_np(x: np.ndarray) -> np.ndarray:
    return np.vectorize(math.erf, otypes=[np.float64])(x)


def _unary_leaky(x, a):
    alpha = F32(a["alpha"])
    return np.where(x >= 0, x, alpha * x), np.where(x >= 0, F32(1), alpha)


def _unary_softplus(x, a):
    xd = x.astype(np.float64)
    y = np.where(xd > 20, xd, np.log1p(np.exp(np.minimum(xd, 20))))
    return y, 1.0 / (1.0 + np.exp(-xd))


def _unary_elu(x, a):
    alpha = float(a["alpha"])
    xd = x.astype(np.float64)
    return np.where(xd > 0, xd, alpha * (np.exp(xd) - 1)), np.where(xd > 0, 1.0, alpha * np.exp(xd))


def _unary_hardsigmoid(x, a):
    al, be = F32(a["alpha"]), F32(a["beta"])
    t = al * x + be
    return np.clip(t, 0, 1), np.where((t > 0) & (t < 1), al, F32(0))


def _unary_softsign(x, a):
    d = F32(1) + np.abs(x)
    return x / d, F32(1) / (d * d)


_UNARY_RULES = {
    "Sqrt": lambda x, a: (np.sqrt(x), F32(0.5) / np.sqrt(x)),
    "Abs": lambda x, a: (np.abs(x), np.sign(x)),
    "Reciprocal": lambda x, a: (F32(1) / x, -F32(1) / (x * x)),
    "Erf": lambda x, a: (_erf_np(x.astype(np.float64)), 2.0 / math.sqrt(math.pi) * np.exp(-x.astype(np.float64) ** 2)),
    "LeakyRelu": _unary_leaky,
    "Softplus": _unary_softplus,
    "Elu": _unary_elu,
    "HardSigmoid": _unary_hardsigmoid,
    "Softsign": _unary_softsign,
}


def _unary(x: T, t: str, a: dict) -> T:
    y, dy = _UNARY_RULES[t](x.data, a)
    y, dy = np.asarray(y, dtype=F32), np.asarray(dy, dtype=F32)
    return _node(y, (x,), lambda g: (g * dy,))


def pow_(a: T, b: T) -> T:
    out = np.power(a.data, b.data).astype(F32)
    return _node(out, (a, b),
                 lambda g: (_unbroadcast(g * b.data * np.power(a.data, b.data - F32(1)), a.shape),
                            _unbroadcast(g * out * np.log(a.data), b.shape)))


def concat(vals: list, axis: int) -> T:
    axis = axis % vals[0].data.ndim
    out = np.concatenate([v.data for v in vals], axis=axis).astype(F32)
    bounds = np.cumsum([0] + [v.shape[axis] for v in vals])

    def back(g):
        return tuple(np.take(g, np.arange(bounds[i], bounds[i + 1]), axis=axis) for i in range(len(vals)))

    return _node(out, tuple(vals), back)


def slice_(x: T, starts, ends, axes, steps) -> T:
    index = [slice(None)] * x.data.ndim
    for s, e, ax, st in zip(starts, ends, axes, steps):
        ax = ax % x.data.ndim
        dim = x.shape[ax]
        s, e = int(s), int(e)
        if s < 0:
            s += dim
        if e < 0:
            e += dim
        if st > 0:
            s, e = min(max(s, 0), dim), min(max(e, 0), dim)
        else:
            s, e = min(max(s, 0), dim - 1), min(max(e, -1), dim - 1)
        index[ax] = slice(s, e if e >= 0 else None, int(st))
    index = tuple(index)
    out = np.ascontiguousarray(x.data[index])

    def back(g):
        dx = np.zeros(x.shape, dtype=F32)
        dx[index] = g
        return (dx,)

    return _node(out, (x,), back)


def avg_pool(x: T, a: dict) -> T:
    """AveragePool: the mean of each window's taps inside the input (with
    count_include_pad, of those inside the explicitly padded input)."""
    k = list(a["kernel_shape"])
    st, dil, pads = list(a["strides"]), list(a["dilations"]), list(a["pads"])
    data = x.data
    one_d = len(k) == 1
    if one_d:
        data = data[:, :, None, :]
        k, st, dil, pads = [1] + k, [1] + st, [1] + dil, [0, pads[0], 0, pads[1]]
    n, c, h, w = data.shape
    auto, ceil = a.get("auto_pad", "NOTSET"), bool(a.get("ceil_mode", 0))
    pt, oh = _pool_axis(h, k[0], st[0], dil[0], pads[0], pads[2], auto, ceil)
    pl, ow = _pool_axis(w, k[1], st[1], dil[1], pads[1], pads[3], auto, ceil)
    pb = pads[2] if auto == "NOTSET" else max((oh - 1) * st[0] + (k[0] - 1) * dil[0] + 1 - h - pt, 0)
    pr = pads[3] if auto == "NOTSET" else max((ow - 1) * st[1] + (k[1] - 1) * dil[1] + 1 - w - pl, 0)
    if auto == "VALID":
        pb = pr = 0
    inc = bool(a.get("count_include_pad", 0))
    total = np.zeros((n, c, oh, ow), dtype=np.float64)
    rows = np.arange(oh) * st[0] - pt
    cols = np.arange(ow) * st[1] - pl
    lo_h, hi_h = (-pt, h + pb) if inc else (0, h)
    lo_w, hi_w = (-pl, w + pr) if inc else (0, w)
    cnt_h = sum(((rows + kh * dil[0] >= lo_h) & (rows + kh * dil[0] < hi_h)).astype(np.int64) for kh in range(k[0]))
    cnt_w = sum(((cols + kw * dil[1] >= lo_w) & (cols + kw * dil[1] < hi_w)).astype(np.int64) for kw in range(k[1]))
    cnt = (cnt_h[:, None] * cnt_w[None, :]).astype(np.float64)
    taps = []
    for kh in range(k[0]):
        hh = rows + kh * dil[0]
        vh = (hh >= 0) & (hh < h)
        for kw in range(k[1]):
            ww = cols + kw * dil[1]
            vw = (ww >= 0) & (ww < w)
            valid = vh[:, None] & vw[None, :]
            tap = data[:, :, np.clip(hh, 0, h - 1)[:, None], np.clip(ww, 0, w - 1)[None, :]]
            total += np.where(valid, tap, 0)
            taps.append((np.clip(hh, 0, h - 1), np.clip(ww, 0, w - 1), valid))
    safe = np.where(cnt > 0, cnt, 1)
    out = np.where(cnt > 0, total / safe, 0).astype(F32)

    def back(g):
        g4 = (g[:, :, None, :] if one_d else g).astype(np.float64) / safe
        dx = np.zeros((n, c, h, w), dtype=np.float64)
        for hh, ww, valid in taps:
            contrib = np.where(valid & (cnt > 0), g4, 0)
            np.add.at(dx, (slice(None), slice(None), hh[:, None], ww[None, :]), contrib)
        dx = dx.astype(F32)
        return (dx[:, :, 0, :] if one_d else dx,)

    return _node(np.ascontiguousarray(out[:, :, 0, :] if one_d else out), (x,), back)


def extremum(x: T, axes, keepdims: bool, is_max: bool) -> T:
    """ReduceMax / ReduceMin; the gradient goes to the first extremal element."""
    nd = x.data.ndim
    axes = sorted(ax % nd for ax in axes)
    keep = [i for i in range(nd) if i not in axes]
    moved = np.transpose(x.data, keep + axes)
    flat = moved.reshape(moved.shape[:len(keep)] + (-1,))
    idx = (np.argmax if is_max else np.argmin)(flat, axis=-1)
    val = np.take_along_axis(flat, idx[..., None], axis=-1)[..., 0].astype(F32)
    out_shape = [1 if i in axes else x.shape[i] for i in range(nd)] if keepdims else [x.shape[i] for i in keep]

    def back(g):
        gf = np.zeros(flat.shape, dtype=F32)
        np.put_along_axis(gf, idx[..., None], np.asarray(g, dtype=F32).reshape(idx.shape)[..., None], axis=-1)
        dx_moved = gf.reshape(moved.shape)
        inv = np.argsort(keep + axes)
        return (np.ascontiguousarray(np.transpose(dx_moved, inv)),)

    return _node(val.reshape(out_shape), (x,), back)


def sqrt_(a: T) -> T:
    out = np.sqrt(a.data).astype(F32)
    return _node(out, (a,), lambda g: (g / (F32(2) * out),))


def _channel(p: T, rank: int) -> T:
    """A [C] tensor reshaped to broadcast over axis 1 of a rank-`rank` input."""
    shape = [1] * rank
    shape[1] = p.shape[0]
    return reshape(p, shape)


def batch_norm(x: T, scale: T, bias: T, mean_: T, var: T, eps: float) -> T:
    """BatchNormalization with fixed running statistics, composed as
    ``crates/tynx-train/src/imported_model/executor.rs:441-445``:
    ((x - mean) / sqrt(var + eps)) * scale + bias.  mean / var are buffers."""
    r = x.data.ndim
    m = T(_channel(mean_, r).data)
    v = T(_channel(var, r).data)
    sd = sqrt_(v + T(np.asarray(eps, dtype=F32)))
    return (x - m) / sd * _channel(scale, r) + _channel(bias, r)


def group_norm(x: T, scale: T, bias: T, groups: int, eps: float) -> T:
    """Group normalization (InstanceNormalization is groups == C), composed as
    ``crates/tynx/src/interpreter/normalization.rs:73-106, 213-273``: mean and
    biased variance of each (sample, group) over its channels and positions,
    centred / sqrt(var + eps), then the per-channel affine."""
    shape = x.shape
    n, c = shape[0], shape[1]
    grouped = reshape(x, [n, groups, c // groups] + list(shape[2:]))
    axes = tuple(range(2, grouped.data.ndim))
    mu = mean(grouped, axes, keepdims=True)
    centred = grouped - mu
    var = mean(centred * centred, axes, keepdims=True)
    normal = reshape(centred / sqrt_(var + T(np.asarray(eps, dtype=F32))), shape)
    r = len(shape)
    return normal * _channel(scale, r) + _channel(bias, r)


def _pool_axis(size: int, k: int, s: int, d: int, begin: int, end: int, auto_pad: str,
               ceil: bool) -> tuple[int, int]:
    """Start padding and output length of one pooled axis
    (``crates/tynx/src/interpreter/spatial.rs:102-151``)."""
    eff = (k - 1) * d + 1
    if auto_pad == "VALID":
        begin = end = 0
    elif auto_pad in ("SAME_UPPER", "SAME_LOWER"):
        out = -(-size // s)
        total = max((out - 1) * s + eff - size, 0)
        small, large = total // 2, total - total // 2
        begin, end = (large, small) if auto_pad == "SAME_LOWER" else (small, large)
    padded = size + begin + end
    if padded < eff:
        raise ValueError("MaxPool window larger than its padded input")
    out = (padded - eff) // s + 1
    if ceil:
        out = -(-(padded - eff) // s) + 1
        if out > 0 and (out - 1) * s >= size + begin:
            out -= 1
    return begin, out


def max_pool(x: T, a: dict) -> T:
    """MaxPool over the -inf padded input (``pooling.rs:360-426``); the gradient
    goes to the first maximal tap in window order."""
    k = list(a["kernel_shape"])
    st, dil, pads = list(a["strides"]), list(a["dilations"]), list(a["pads"])
    data = x.data
    one_d = len(k) == 1
    if one_d:
        data = data[:, :, None, :]
        k, st, dil, pads = [1] + k, [1] + st, [1] + dil, [0, pads[0], 0, pads[1]]
    n, c, h, w = data.shape
    auto, ceil = a.get("auto_pad", "NOTSET"), bool(a.get("ceil_mode", 0))
    pt, oh = _pool_axis(h, k[0], st[0], dil[0], pads[0], pads[2], auto, ceil)
    pl, ow = _pool_axis(w, k[1], st[1], dil[1], pads[1], pads[3], auto, ceil)
    best = np.full((n, c, oh, ow), -np.inf, dtype=F32)
    arg = np.full((n, c, oh, ow), -1, dtype=np.int64)
    rows = np.arange(oh) * st[0] - pt
    cols = np.arange(ow) * st[1] - pl
    for kh in range(k[0]):
        hh = rows + kh * dil[0]
        vh = (hh >= 0) & (hh < h)
        for kw in range(k[1]):
            ww = cols + kw * dil[1]
            vw = (ww >= 0) & (ww < w)
            valid = vh[:, None] & vw[None, :]
            tap = data[:, :, np.clip(hh, 0, h - 1)[:, None], np.clip(ww, 0, w - 1)[None, :]]
            take = valid & ((tap > best) | (arg < 0))
            best = np.where(take, tap, best).astype(F32)
            pos = np.clip(hh, 0, h - 1)[:, None] * w + np.clip(ww, 0, w - 1)[None, :]
            arg = np.where(take, pos, arg)
    out = best[:, :, 0, :] if one_d else best

    def back(g):
        g4 = g[:, :, None, :] if one_d else g
        dx = np.zeros((n * c, h * w), dtype=F32)
        flat = arg.reshape(n * c, -1)
        src = g4.reshape(n * c, -1)
        ok = flat >= 0
        rows_ = np.repeat(np.arange(n * c)[:, None], flat.shape[1], axis=1)
        np.add.at(dx, (rows_[ok], flat[ok]), src[ok])
        dx = dx.reshape(n, c, h, w)
        return (dx[:, :, 0, :] if one_d else dx,)

    return _node(np.ascontiguousarray(out), (x,), back)


def layer_norm(x: T, scale: T, bias: Optional[T], axis: int, eps: float, n_out: int):
    """Composed LayerNormalization (``normalization.rs:135-190``)."""
    rank = x.data.ndim
    axis = axis % rank
    axes = tuple(range(axis, rank))
    mu = mean(x, axes, keepdims=True)
    centered = x - mu
    var = mean(centered * centered, axes, keepdims=True)
    inv_std = power(var + T(np.asarray(eps, dtype=F32)), -0.5)
    y = centered * inv_std * scale
    if bias is not None:
        y = y + bias
    return [y, mu, inv_std][:n_out]


def power(a: T, p: float) -> T:
    out = np.power(a.data, F32(p)).astype(F32)
    return _node(out, (a,), lambda g: (g * F32(p) * np.power(a.data, F32(p - 1)),))


# =============================================================================
# losses (functional.py:126-145, distributions.py:47-104, loss.rs:10-23)
# =============================================================================


def cross_entropy(logits: T, labels: np.ndarray) -> T:
    labels = np.asarray(labels, dtype=np.int64)
    selected = take_along(log_softmax(logits, 1), 1, labels[:, None])
    return mean(neg(reshape(selected, (labels.shape[0],))))


def mse_loss(pred: T, target) -> T:
    target = target if isinstance(target, T) else T(np.asarray(target, dtype=F32))
    diff = pred - target
    return mean(diff * diff)


class Categorical:
    def __init__(self, logits: T):
        self.logits = log_softmax(logits, -1)
        self.probs = exp(self.logits)

    def log_prob(self, actions: np.ndarray) -> T:
        idx = np.asarray(actions, dtype=np.int64)[..., None]
        return reshape(take_along(self.logits, -1, idx), idx.shape[:-1])

    def entropy(self) -> T:
        return neg(sum_(self.probs * self.logits, axes=-1))


def ppo_loss(logits: T, values: T, actions, old_log_prob, advantages, returns,
             clip: float = 0.2, value_coef: float = 0.5, entropy_coef: float = 0.01) -> T:
    """Clipped-surrogate PPO loss as composed in the reference's PPO test
    (``crates/tynx-python/tests/test_ppo.py:53-64``)."""
    policy = Categorical(logits)
    ratio = exp(policy.log_prob(actions) - T(np.asarray(old_log_prob, dtype=F32)))
    adv = T(np.asarray(advantages, dtype=F32))
    policy_loss = neg(mean(minimum(ratio * adv, clamp(ratio, 1 - clip, 1 + clip) * adv)))
    value_loss = mse_loss(reshape(values, (values.shape[0],)), returns)
    return policy_loss + value_loss * T(np.asarray(value_coef, dtype=F32)) - \
        mean(policy.entropy()) * T(np.asarray(entropy_coef, dtype=F32))


# =============================================================================
# optimizers
# =============================================================================


class Adam:
    """Adam / AdamW (``adam.rs:431-527``); f64 host scalars rounded to f32."""

    def __init__(self, params, lr: float, betas=(0.9, 0.999), eps: float = 1e-8,
                 weight_decay: float = 0.0, amsgrad: bool = False, decoupled: bool = False):
        self.params = [p for _, p in params] if params and isinstance(params[0], tuple) else \
            list(params)
        self.lr, self.betas, self.eps = lr, betas, eps
        self.weight_decay, self.amsgrad, self.decoupled = weight_decay, amsgrad, decoupled
        self.state: dict[int, dict] = {}

    def zero_grad(self) -> None:
        for p in self.params:
            p.grad = None

    def step(self) -> None:
        b1, b2 = self.betas
        for p in self.params:
            if p.grad is None:
                continue
            w = p.data
            d = p.grad
            if not self.decoupled and self.weight_decay != 0.0:
                d = (d + w * f32(self.weight_decay)).astype(F32)
            st = self.state.setdefault(id(p), {
                "step": 0, "m": np.zeros_like(w), "v": np.zeros_like(w),
                "vmax": np.zeros_like(w) if self.amsgrad else None})
            st["step"] += 1
            t = st["step"]
            m = (st["m"] * f32(b1) + d * f32(1.0 - b1)).astype(F32)
            v = (st["v"] * f32(b2) + (d * d) * f32(1.0 - b2)).astype(F32)
            denom = v
            if self.amsgrad:
                st["vmax"] = np.maximum(st["vmax"], v)
                denom = st["vmax"]
            bc1 = 1.0 - b1 ** float(t)
            bc2 = 1.0 - b2 ** float(t)
            m_hat = (m / f32(bc1)).astype(F32)
            v_hat = (denom / f32(bc2)).astype(F32)
            upd = ((m_hat / (np.sqrt(v_hat) + f32(self.eps))) * f32(self.lr)).astype(F32)
            if self.decoupled and self.weight_decay != 0.0:
                w = (w * f32(1.0 - self.lr * self.weight_decay)).astype(F32)
            p.data = (w - upd).astype(F32)
            st["m"], st["v"] = m, v


class SGD:
    """SGD with momentum/dampening/nesterov (``optimizer.rs:310-356``)."""

    def __init__(self, params, lr: float, momentum: float = 0.0, dampening: float = 0.0,
                 weight_decay: float = 0.0, nesterov: bool = False):
        self.params = [p for _, p in params] if params and isinstance(params[0], tuple) else \
            list(params)
        self.lr, self.momentum, self.dampening = lr, momentum, dampening
        self.weight_decay, self.nesterov = weight_decay, nesterov
        self.buffers: dict[int, np.ndarray] = {}

    def zero_grad(self) -> None:
        for p in self.params:
            p.grad = None

    def step(self) -> None:
        for p in self.params:
            if p.grad is None:
                continue
            d = p.grad
            if self.weight_decay != 0.0:
                d = (d + p.data * f32(self.weight_decay)).astype(F32)
            if self.momentum != 0.0:
                prev = self.buffers.get(id(p))
                buf = d if prev is None else \
                    (prev * f32(self.momentum) + d * f32(1.0 - self.dampening)).astype(F32)
                self.buffers[id(p)] = buf
                d = (d + buf * f32(self.momentum)).astype(F32) if self.nesterov else buf
            p.data = (p.data - d * f32(self.lr)).astype(F32)
