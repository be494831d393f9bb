"""Eager Tensor operations of the capture IR beyond the configurations' losses
(crates/tynx-capture/src/lib.rs:125-263: Sqrt, the smooth unary operations,
PowerScalar / ReversePowerScalar, Power, Slice, Repeat, MaxPool2d,
AvgPool2d, AdaptiveAvgPool2d, Dropout, plus embedding) on Device("cuda"):
forward and gradient against numpy / the oracle, and a compiled step built
from them that replays like the eager one (dropout drawing a new mask on
every replay from its device stream).
"""

import numpy as np
import pytest

from oracle import flex_oracle as fo

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def tx():
    import tynx_b200 as tx

    tx.set_math_mode("fp32")
    yield tx
    tx.set_math_mode("tf32")


def _rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def _grad_check(tx, fn_tx, fn_np, x_np, tol=1e-5):
    """fn_tx on a leaf Tensor against fn_np on a float64 array (gradient by
    central differences of sum(w * f(x)) in float64)."""
    x = tx.Tensor(x_np, requires_grad=True)
    y = fn_tx(x)
    ref = fn_np(x_np.astype(np.float64))
    assert tuple(y.shape) == ref.shape, (y.shape, ref.shape)
    assert _rel(y.numpy(), ref) <= tol
    w = np.random.default_rng(3).standard_normal(ref.shape)
    (y * tx.Tensor(w.astype(np.float32))).sum().backward()
    num = np.zeros_like(x_np, dtype=np.float64)
    flat = x_np.astype(np.float64).reshape(-1)
    h = 1e-6
    for i in range(flat.size):
        p, m = flat.copy(), flat.copy()
        p[i] += h
        m[i] -= h
        num.reshape(-1)[i] = (np.sum(w * fn_np(p.reshape(x_np.shape))) -
                              np.sum(w * fn_np(m.reshape(x_np.shape)))) / (2 * h)
    assert _rel(x.grad.numpy(), num) <= 1e-4, _rel(x.grad.numpy(), num)


def test_unary_methods(tx):
    rng = np.random.default_rng(0)
    x = (rng.standard_normal((3, 7)) * 1.5).astype(np.float32)
    from math import erf

    cases = [
        (lambda t: t.erf(), np.vectorize(erf)),
        (lambda t: t.softplus(), lambda v: np.log1p(np.exp(v))),
        (lambda t: t.softsign(), lambda v: v / (1 + np.abs(v))),
        (lambda t: t.leaky_relu(0.2), lambda v: np.where(v >= 0, v, 0.2 * v)),
        (lambda t: t.elu(0.8), lambda v: np.where(v > 0, v, 0.8 * (np.exp(v) - 1))),
        (lambda t: t.hardsigmoid(), lambda v: np.clip(v / 6 + 0.5, 0, 1)),
    ]
    for fn_tx, fn_np in cases:
        _grad_check(tx, fn_tx, fn_np, x)
    pos = np.abs(x) + 0.5
    _grad_check(tx, lambda t: t.reciprocal(), lambda v: 1 / v, pos)
    _grad_check(tx, lambda t: t.sqrt(), np.sqrt, pos)


def test_powers(tx):
    rng = np.random.default_rng(1)
    a = (np.abs(rng.standard_normal((4, 5))) + 0.5).astype(np.float32)
    e = rng.uniform(0.5, 2.0, (4, 5)).astype(np.float32)
    _grad_check(tx, lambda t: t ** 1.5, lambda v: v ** 1.5, a)
    _grad_check(tx, lambda t: 2.5 ** t, lambda v: 2.5 ** v, a)
    _grad_check(tx, lambda t: t ** tx.Tensor(e), lambda v: v ** e.astype(np.float64), a)
    _grad_check(tx, lambda t: tx.Tensor(a) ** t, lambda v: a.astype(np.float64) ** v, e)


@pytest.mark.parametrize("index", [
    (slice(1, 4),),
    (slice(None), slice(None, None, 2)),
    (Ellipsis, slice(5, 1, -2)),
    (1, slice(2, None)),
    (slice(None), None, -1),
    (slice(-2, None), Ellipsis, slice(None, None, 3)),
])
def test_getitem(tx, index):
    rng = np.random.default_rng(2)
    x = rng.standard_normal((5, 6, 7)).astype(np.float32)
    _grad_check(tx, lambda t: t[index], lambda v: v[index], x)


def test_repeat(tx):
    rng = np.random.default_rng(4)
    x = rng.standard_normal((2, 3)).astype(np.float32)
    _grad_check(tx, lambda t: t.repeat(2, 1, 3), lambda v: np.tile(v, (2, 1, 3)), x)


@pytest.mark.parametrize("kw", [{"kernel_size": 2}, {"kernel_size": 3, "stride": 2, "padding": 1},
                                {"kernel_size": 3, "stride": 2, "ceil_mode": True},
                                {"kernel_size": (3, 2), "stride": (1, 2), "dilation": (2, 1)}])
def test_max_pool2d(tx, kw):
    rng = np.random.default_rng(5)
    x_np = rng.standard_normal((2, 3, 11, 9)).astype(np.float32)
    x = tx.Tensor(x_np, requires_grad=True)
    y = tx.nn.functional.max_pool2d(x, **kw)
    k = kw["kernel_size"] if isinstance(kw["kernel_size"], tuple) else (kw["kernel_size"],) * 2
    s = kw.get("stride", k)
    s = s if isinstance(s, tuple) else (s, s)
    p = kw.get("padding", 0)
    d = kw.get("dilation", (1, 1))
    attrs = {"kernel_shape": list(k), "strides": list(s), "pads": [p, p, p, p], "dilations": list(d),
             "ceil_mode": int(kw.get("ceil_mode", False)), "auto_pad": "NOTSET"}
    xr = fo.T(x_np.copy(), requires_grad=True)
    yr = fo.max_pool(xr, attrs)
    assert _rel(y.numpy(), yr.data) == 0.0
    w = np.random.default_rng(6).standard_normal(yr.shape).astype(np.float32)
    (y * tx.Tensor(w)).sum().backward()
    fo.sum_(yr * fo.T(w)).backward()
    assert _rel(x.grad.numpy(), xr.grad) <= 1e-6


@pytest.mark.parametrize("kw", [{"kernel_size": 2}, {"kernel_size": 3, "stride": 2, "padding": 1},
                                {"kernel_size": 3, "stride": 2, "padding": 1, "count_include_pad": False},
                                {"kernel_size": 3, "stride": 2, "ceil_mode": True}])
def test_avg_pool2d(tx, kw):
    rng = np.random.default_rng(7)
    x_np = rng.standard_normal((2, 3, 11, 9)).astype(np.float32)
    x = tx.Tensor(x_np, requires_grad=True)
    y = tx.nn.functional.avg_pool2d(x, **kw)
    k = kw["kernel_size"]
    s = kw.get("stride", k)
    p = kw.get("padding", 0)
    attrs = {"kernel_shape": [k, k], "strides": [s, s], "pads": [p, p, p, p], "dilations": [1, 1],
             "ceil_mode": int(kw.get("ceil_mode", False)), "auto_pad": "NOTSET",
             "count_include_pad": int(kw.get("count_include_pad", True))}
    xr = fo.T(x_np.copy(), requires_grad=True)
    yr = fo.avg_pool(xr, attrs)
    assert _rel(y.numpy(), yr.data) <= 1e-6
    w = np.random.default_rng(8).standard_normal(yr.shape).astype(np.float32)
    (y * tx.Tensor(w)).sum().backward()
    fo.sum_(yr * fo.T(w)).backward()
    assert _rel(x.grad.numpy(), xr.grad) <= 1e-6


def test_adaptive_avg_pool2d_and_embedding(tx):
    rng = np.random.default_rng(9)
    x_np = rng.standard_normal((2, 3, 8, 6)).astype(np.float32)
    y = tx.nn.functional.adaptive_avg_pool2d(tx.Tensor(x_np), (4, 3)).numpy()
    ref = x_np.reshape(2, 3, 4, 2, 3, 2).mean(axis=(3, 5))
    assert _rel(y, ref) <= 1e-6
    table = rng.standard_normal((10, 4)).astype(np.float32)
    idx = np.array([[1, 3, 3], [0, 9, 1]], np.int64)
    w = tx.Tensor(table, requires_grad=True)
    out = tx.nn.functional.embedding(tx.Tensor(idx, dtype="int64"), w, padding_idx=3)
    np.testing.assert_array_equal(out.numpy(), table[idx])
    out.sum().backward()
    expect = np.zeros_like(table)
    np.add.at(expect, idx.reshape(-1), 1.0)
    expect[3] = 0.0
    np.testing.assert_array_equal(w.grad.numpy(), expect)


def test_dropout_stream(tx):
    x = tx.Tensor(np.ones((4096, 64), np.float32), requires_grad=True)
    y1 = tx.nn.functional.dropout(x, 0.25)
    y2 = tx.nn.functional.dropout(x, 0.25)
    a, b = y1.numpy(), y2.numpy()
    assert set(np.unique(a)) <= {0.0, np.float32(1 / 0.75)}
    keep = (a != 0).mean()
    assert abs(keep - 0.75) < 0.01, keep
    assert (a != b).any()  # the stream advanced between the calls
    y1.sum().backward()
    np.testing.assert_array_equal(x.grad.numpy(), a)
    assert tx.nn.functional.dropout(x, 0.25, training=False) is x


def test_compiled_step_with_capture_ops_replays(tx):
    """A loss built from slicing, repeat, pooling, powers and dropout, compiled
    into one CUDA graph: replays equal the eager function without dropout, and
    with dropout draw a fresh mask each replay."""
    rng = np.random.default_rng(10)
    w = tx.Tensor(rng.standard_normal((3, 3)).astype(np.float32) * 0.5, requires_grad=True)

    def loss_fn(x, drop):
        h = x[:, :, 1:, :].repeat(1, 1, 1, 2)
        h = tx.nn.functional.avg_pool2d(h, 2) + tx.nn.functional.max_pool2d(h, 2)
        h = (h.softplus() ** 1.5).mean(dim=(2, 3))
        h = h @ w
        if drop:
            h = tx.nn.functional.dropout(h, 0.5, seed=7)
        return (h * h).mean()

    @tx.compile(fullgraph=True)
    def step(x):
        return loss_fn(x, False)

    @tx.compile(fullgraph=True)
    def step_drop(x):
        return loss_fn(x, True)

    xs = [tx.Tensor(rng.standard_normal((4, 3, 9, 6)).astype(np.float32)) for _ in range(3)]
    for x in xs:
        assert abs(step(x).item() - loss_fn(x, False).item()) <= 1e-6 * max(1.0, abs(loss_fn(x, False).item()))
    vals = {round(step_drop(xs[0]).item(), 7) for _ in range(4)}
    assert len(vals) > 1, vals
