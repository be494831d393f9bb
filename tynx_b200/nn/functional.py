"""Loss functions on CUDA (``tynx.nn.functional``).

``cross_entropy`` keeps the reference's contract
(``crates/tynx-python/python/tynx/nn/functional.py:133-145``: rank-2 float32 logits,
rank-1 int64 targets, ``-mean(log_softmax(z)[y])``) but runs as one fused
softmax-cross-entropy kernel forward and one backward kernel instead of the five
taped operations.  ``mse_loss`` follows ``loss.rs:10-23`` / ``functional.py:126-130``.
"""

from __future__ import annotations

import ctypes as C

from .. import _native as N
from .._core import Fn, Tensor, _needs_grad, maximum
from .._native import lib


def cross_entropy(input: Tensor, target: Tensor, reduction: str = "mean") -> Tensor:
    """Cross entropy for rank-2 logits and rank-1 int64 class targets."""
    if input.dtype != "float32" or input.ndim != 2:
        raise ValueError(
            f"cross_entropy input must be rank-2 float32 logits, got {input.dtype} {input.shape}"
        )
    if target.dtype != "int64" or target.shape != (input.shape[0],):
        raise ValueError(
            "cross_entropy target must be a rank-1 int64 Tensor with one class index per row, "
            f"got {target.dtype} {target.shape}"
        )
    if reduction != "mean":
        selected = input.log_softmax(1).gather(1, target.unsqueeze(1)).squeeze(1)
        return -selected if reduction == "none" else (-selected).sum()
    rows, cols = input.shape
    ctx = input.ctx
    loss = Tensor._empty((1,), "float32", ctx)
    ctx.check(lib.tx_softmax_xent_fwd(ctx.handle, input.ptr, target.ptr, rows, cols, loss.ptr),
              "cross_entropy")
    if _needs_grad(input):
        logits, labels = input.detach(), target.detach()

        def backward(g):
            dz = Tensor._empty((rows, cols), "float32", ctx)
            ctx.check(lib.tx_softmax_xent_bwd(ctx.handle, logits.ptr, labels.ptr, rows, cols,
                                              g[0].ptr, dz.ptr, 0), "cross_entropy backward")
            return [dz]

        loss._attach(Fn("cross_entropy", [input], backward))
    return loss


def mse_loss(input: Tensor, target: Tensor, reduction: str = "mean") -> Tensor:
    """Elementwise, mean, or summed squared error for exactly matching shapes."""
    if input.shape != target.shape:
        raise ValueError(
            f"mse_loss requires exactly matching shapes, got {input.shape} and {target.shape}"
        )
    error = input - target
    squared = error * error
    if reduction == "none":
        return squared
    if reduction == "mean":
        return squared.mean()
    if reduction == "sum":
        return squared.sum()
    raise ValueError(f"reduction must be 'none', 'mean', or 'sum', got {reduction!r}")


def ppo_loss(logits: Tensor, values: Tensor, actions: Tensor, old_log_prob: Tensor, advantages: Tensor,
             returns: Tensor, *, clip: float = 0.2, value_coef: float = 0.5,
             entropy_coef: float = 0.01) -> Tensor:
    """The clipped-surrogate PPO objective as one fused kernel forward and one
    backward: ``-mean(min(r*A, clamp(r, 1-clip, 1+clip)*A)) + value_coef *
    mse(values, returns) - entropy_coef * mean(entropy)`` with ``r =
    exp(log_softmax(logits)[actions] - old_log_prob)``.  The same value, and
    the same gradients for ``logits`` and ``values``, as that objective
    composed from ``distributions.Categorical``, ``minimum``, ``clamp`` and
    ``mse_loss`` (the reference's ``crates/tynx-python/tests/test_ppo.py:53-64``),
    without its twenty intermediate tensors.  ``values`` is [rows] or
    [rows, 1]; the other per-row inputs are [rows]."""
    if logits.dtype != "float32" or logits.ndim != 2:
        raise ValueError(f"ppo_loss logits must be rank-2 float32, got {logits.dtype} {logits.shape}")
    rows, cols = logits.shape
    if values.shape not in ((rows,), (rows, 1)):
        raise ValueError(f"ppo_loss values must be [rows] or [rows, 1], got {values.shape}")
    if actions.dtype != "int64" or actions.shape != (rows,):
        raise ValueError(f"ppo_loss actions must be a rank-1 int64 Tensor of {rows} rows")
    for name, t in (("old_log_prob", old_log_prob), ("advantages", advantages), ("returns", returns)):
        if t.dtype != "float32" or t.shape != (rows,):
            raise ValueError(f"ppo_loss {name} must be a rank-1 float32 Tensor of {rows} rows")
    ctx = logits.ctx
    scalars = (C.c_float(clip), C.c_float(value_coef), C.c_float(entropy_coef))

    def inputs(z, v, a, o, adv, ret):
        return (z.ptr, rows, cols, v.ptr, a.ptr, o.ptr, adv.ptr, ret.ptr) + scalars

    loss = Tensor._empty((1,), "float32", ctx)
    ctx.check(lib.tx_ppo_loss_fwd(ctx.handle, *inputs(logits, values, actions, old_log_prob, advantages,
                                                      returns), loss.ptr), "ppo_loss")
    if _needs_grad(logits, values):
        # detached views keep the inputs' storage alive until this node is freed
        saved = tuple(t.detach() for t in (logits, values, actions, old_log_prob, advantages, returns))
        want_v = values.requires_grad

        def backward(g):
            dz = Tensor._empty((rows, cols), "float32", ctx)
            dv = Tensor._empty(values.shape, "float32", ctx) if want_v else None
            ctx.check(lib.tx_ppo_loss_bwd(ctx.handle, *inputs(*saved), g[0].ptr, dz.ptr,
                                          dv.ptr if dv is not None else None, 0, 0), "ppo_loss backward")
            return [dz, dv]

        loss._attach(Fn("ppo_loss", [logits, values], backward))
    return loss


def relu(input: Tensor) -> Tensor:
    return input.relu()


def binary_cross_entropy_with_logits(input: Tensor, target: Tensor, reduction: str = "mean"):
    if input.shape != target.shape:
        raise ValueError("binary_cross_entropy_with_logits requires exactly matching shapes")
    absolute = maximum(input, -input)
    loss = maximum(input, 0.0) - input * target + ((-absolute).exp() + 1.0).log()
    return mse_reduce(loss, reduction)


def mse_reduce(t: Tensor, reduction: str) -> Tensor:
    if reduction == "none":
        return t
    if reduction == "mean":
        return t.mean()
    if reduction == "sum":
        return t.sum()
    raise ValueError(f"reduction must be 'none', 'mean', or 'sum', got {reduction!r}")


__all__ = ["binary_cross_entropy_with_logits", "cross_entropy", "mse_loss", "ppo_loss", "relu"]
