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


__all__ = ["binary_cross_entropy_with_logits", "cross_entropy", "mse_loss", "relu"]
