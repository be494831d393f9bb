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


def _pair(v, name: str, positive: bool) -> tuple:
    pair = (v, v) if isinstance(v, int) else tuple(v)
    if len(pair) != 2 or any(not isinstance(x, int) for x in pair):
        raise TypeError(f"{name} must be an int or a pair of ints")
    if any(x <= 0 if positive else x < 0 for x in pair):
        raise ValueError(f"{name} must be {'positive' if positive else 'non-negative'}")
    return pair


def _pool_out(size: int, k: int, s: int, p: int, d: int, ceil: bool) -> int:
    eff = d * (k - 1) + 1
    if size + 2 * p < eff:
        raise ValueError("pooling window larger than its padded input")
    if ceil:
        out = -(-(size + 2 * p - eff) // s) + 1
        if (out - 1) * s >= size + p:
            out -= 1
        return out
    return (size + 2 * p - eff) // s + 1


def _pool_geom(input: Tensor, kernel, stride, padding, dilation, ceil: bool):
    if input.ndim != 4 or input.dtype != "float32":
        raise ValueError(f"pooling expects a float32 NCHW input, got {input.dtype} {input.shape}")
    _, _, h, w = input.shape
    oh = _pool_out(h, kernel[0], stride[0], padding[0], dilation[0], ceil)
    ow = _pool_out(w, kernel[1], stride[1], padding[1], dilation[1], ceil)
    geom = [kernel[0], kernel[1], stride[0], stride[1], padding[0], padding[1], dilation[0], dilation[1], oh, ow,
            padding[0], padding[1]]
    return geom, oh, ow


def max_pool2d(input: Tensor, kernel_size, stride=None, padding=0, dilation=1, ceil_mode: bool = False) -> Tensor:
    """Two-dimensional max pooling of an NCHW input over the -inf padded
    input; the gradient goes to the first maximal tap of each window."""
    kernel = _pair(kernel_size, "kernel_size", True)
    geom, oh, ow = _pool_geom(input, kernel, kernel if stride is None else _pair(stride, "stride", True),
                              _pair(padding, "padding", False), _pair(dilation, "dilation", True), bool(ceil_mode))
    n, c, h, w = input.shape
    out = Tensor._empty((n, c, oh, ow), "float32", input.ctx)
    arg = Tensor._empty((n, c, oh, ow), "int64", input.ctx)  # int32 indices in the first half
    g = N.i64_array(geom)
    input.ctx.check(lib.tx_maxpool2d_fwd(input.ctx.handle, input.ptr, out.ptr, arg.ptr, n * c, h, w, g))
    if _needs_grad(input):
        x_shape, ctx = input.shape, input.ctx

        def backward(grads):
            dx = Tensor._empty(x_shape, "float32", ctx)
            ctx.check(lib.tx_maxpool2d_bwd(ctx.handle, grads[0].ptr, arg.ptr, dx.ptr, n * c, h, w,
                                           N.i64_array(geom), 0))
            return [dx]

        out._attach(Fn("max_pool2d", [input], backward))
    return out


def avg_pool2d(input: Tensor, kernel_size, stride=None, padding=0, ceil_mode: bool = False,
               count_include_pad: bool = True, divisor_override=None) -> Tensor:
    """Two-dimensional average pooling of an NCHW input (torch semantics:
    count_include_pad counts the padding, not a ceil-mode overhang)."""
    if divisor_override is not None:
        raise NotImplementedError("avg_pool2d divisor_override is not supported")
    kernel = _pair(kernel_size, "kernel_size", True)
    geom, oh, ow = _pool_geom(input, kernel, kernel if stride is None else _pair(stride, "stride", True),
                              _pair(padding, "padding", False), (1, 1), bool(ceil_mode))
    n, c, h, w = input.shape
    out = Tensor._empty((n, c, oh, ow), "float32", input.ctx)
    inc = int(bool(count_include_pad))
    input.ctx.check(lib.tx_avgpool2d_fwd(input.ctx.handle, input.ptr, out.ptr, n * c, h, w, N.i64_array(geom), inc))
    if _needs_grad(input):
        x_shape, ctx = input.shape, input.ctx

        def backward(grads):
            dx = Tensor._empty(x_shape, "float32", ctx)
            ctx.check(lib.tx_avgpool2d_bwd(ctx.handle, grads[0].ptr, dx.ptr, n * c, h, w, N.i64_array(geom), inc, 0))
            return [dx]

        out._attach(Fn("avg_pool2d", [input], backward))
    return out


def adaptive_avg_pool2d(input: Tensor, output_size) -> Tensor:
    """Average pooling to an exact spatial size.  Windows are the uniform
    k = size / out ones when the sizes divide (the global pool included); other
    sizes need uneven windows and are not supported."""
    oh, ow = _pair(output_size, "output_size", True)
    _, _, h, w = input.shape
    if h % oh or w % ow:
        raise NotImplementedError("adaptive_avg_pool2d needs output sizes that divide the input's")
    return avg_pool2d(input, (h // oh, w // ow), (h // oh, w // ow))


def embedding(input: Tensor, weight: Tensor, padding_idx=None, max_norm=None, norm_type: float = 2.0,
              scale_grad_by_freq: bool = False, sparse: bool = False) -> Tensor:
    """Rows of a dense [rows, width] table for int64 indices; the gradient is
    a scatter-add into the table (the padding row's stays zero)."""
    if max_norm is not None or norm_type != 2.0 or scale_grad_by_freq or sparse:
        raise NotImplementedError("embedding supports the dense lookup only")
    if input.dtype != "int64":
        raise TypeError(f"embedding input must be int64, got {input.dtype}")
    if weight.dtype != "float32" or weight.ndim != 2:
        raise ValueError(f"embedding weight must be rank-2 float32, got {weight.dtype} {weight.shape}")
    rows, width = weight.shape
    if padding_idx is not None:
        if not -rows <= padding_idx < rows:
            raise ValueError("padding_idx must be within the table")
        padding_idx %= rows
    out = Tensor._empty(tuple(input.shape) + (width,), "float32", weight.ctx)
    weight.ctx.check(lib.tx_gather_rows(weight.ctx.handle, weight.ptr, rows, width, input.ptr, input.numel, out.ptr))
    if _needs_grad(weight):
        idx, ctx = input.detach(), weight.ctx

        def backward(grads):
            from .._core import full

            dw = full((rows, width), 0.0, ctx=ctx)
            ctx.check(lib.tx_scatter_add_rows(ctx.handle, dw.ptr, rows, width, idx.ptr, idx.numel, grads[0].ptr))
            if padding_idx is not None:
                ctx.check(lib.tx_fill_f32(ctx.handle, dw.ptr + padding_idx * width * 4, width, C.c_float(0.0)))
            return [None, dw]

        out._attach(Fn("embedding", [input, weight], backward))
    return out


def dropout(input: Tensor, p: float = 0.5, training: bool = True, inplace: bool = False, *,
            seed: int = 0) -> Tensor:
    """Training-mode dropout on a device random stream that advances with every
    call (a compiled step draws a new mask on every replay); the identity when
    not training or p == 0."""
    if not 0.0 <= p < 1.0:
        raise ValueError("dropout probability must be in [0, 1)")
    if not training or p == 0.0:
        return input
    mask = Tensor._empty(input.shape, "float32", input.ctx)
    out = Tensor._empty(input.shape, "float32", input.ctx)
    input.ctx.check(lib.tx_dropout_fwd(input.ctx.handle, input.ptr, out.ptr, mask.ptr, input.numel, C.c_float(p),
                                       C.c_uint64(seed & 0xFFFFFFFFFFFFFFFF), None))
    if _needs_grad(input):
        m = mask

        def backward(grads):
            return [grads[0] * m]

        out._attach(Fn("dropout", [input], backward))
    return out


__all__ = ["adaptive_avg_pool2d", "avg_pool2d", "binary_cross_entropy_with_logits", "cross_entropy", "dropout",
           "embedding", "max_pool2d", "mse_loss", "ppo_loss", "relu"]
