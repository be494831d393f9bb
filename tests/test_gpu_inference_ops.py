"""Operators beyond the five configurations on Device("cuda"), for the
inference Session and for training through them: the smooth unary
operations, Pow / Max / Min, Concat / Slice / Split / Expand, AveragePool,
ReduceMax / ReduceMin / GlobalMaxPool and inference Dropout (the arms of
crates/tynx/src/interpreter/{unary,pow,extrema,concat,slice,split,expand,
pooling,reduction,dropout}.rs, differentiable per
crates/tynx-train/src/backward_support.rs:70-100).

Each one-node model runs forward and backward in fp32 mode against the
oracle (rel 1e-5; the elementwise forwards that are one rounded fp32
expression are compared at 1e-6), and a small multi-operator model runs as an
inference Session.
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


def _model(op, x_shape, inits=(), consts=(), n_out=1, opset=13, extra_inputs=(), **attrs):
    """One node: inputs x, then initializer (trainable) or constant inputs in order."""
    from tynx_b200.onnx import proto

    names = ["x"] + [n for n, _ in inits] + [n for n, _ in consts] + list(extra_inputs)
    outs = [f"y{i}" for i in range(n_out)]
    nodes = [proto.encode_node(op, names, outs, name="op", **attrs)]
    enc = [proto.encode_tensor(n, a) for n, a in list(inits) + list(consts)]
    return proto.encode_model(nodes, enc, [proto.encode_value_info("x", proto.FLOAT, list(x_shape))],
                              [proto.encode_value_info(o, proto.FLOAT, None) for o in outs], opset=opset)


def _rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def _check(tx, data, x_np, tol=1e-5):
    from tynx_b200.onnx import ir

    model = tx.load(data, trainable="auto", simplify=False)
    ref = fo.OracleModel(ir.load_training_graph(data))
    x = tx.Tensor(x_np, requires_grad=True)
    ys = model(x)
    xr = fo.T(x_np.copy(), requires_grad=True)
    yrs = ref(xr)
    if not isinstance(ys, (list, tuple, dict)):
        ys, yrs = [ys], [yrs]
    if isinstance(ys, dict):
        ys, yrs = list(ys.values()), list(yrs.values())
    total, total_r = None, None
    for i, (y, yr) in enumerate(zip(ys, yrs)):
        assert tuple(y.shape) == tuple(yr.shape), (y.shape, yr.shape)
        assert _rel(y.numpy(), yr.data) <= tol, ("forward", i, _rel(y.numpy(), yr.data))
        w = np.random.default_rng(7 + i).standard_normal(yr.shape).astype(np.float32)
        term, term_r = (y * tx.Tensor(w)).sum(), fo.sum_(yr * fo.T(w))
        total = term if total is None else total + term
        total_r = term_r if total_r is None else total_r + term_r
    total.backward()
    total_r.backward()
    assert _rel(x.grad.numpy(), xr.grad) <= tol, ("dx", _rel(x.grad.numpy(), xr.grad))
    params = dict(model.named_parameters())
    for n, q in ref.named_parameters():
        assert _rel(params[n].grad.numpy(), q.grad) <= tol, (n, _rel(params[n].grad.numpy(), q.grad))


UNARY = [("Sqrt", {}, "positive"), ("Abs", {}, "any"), ("Reciprocal", {}, "positive"), ("Erf", {}, "any"),
         ("LeakyRelu", {"alpha": 0.1}, "any"), ("Softplus", {}, "any"), ("Elu", {"alpha": 0.7}, "any"),
         ("HardSigmoid", {"alpha": 0.3, "beta": 0.4}, "any"), ("Softsign", {}, "any")]


@pytest.mark.parametrize("op,attrs,domain", UNARY)
def test_unary_ops_match_oracle(tx, op, attrs, domain):
    rng = np.random.default_rng(1)
    x = (rng.standard_normal((6, 33)) * 2).astype(np.float32)
    if domain == "positive":
        x = np.abs(x) + 0.25
    _check(tx, _model(op, x.shape, **attrs), x)


def test_pow_by_constant_and_by_tensor(tx):
    rng = np.random.default_rng(2)
    x = (np.abs(rng.standard_normal((5, 8))) + 0.5).astype(np.float32)
    _check(tx, _model("Pow", x.shape, consts=[("e", np.array(1.7, np.float32))]), x)
    e = rng.uniform(0.5, 2.0, (1, 8)).astype(np.float32)
    _check(tx, _model("Pow", x.shape, inits=[("e", e)]), x)


@pytest.mark.parametrize("op", ["Max", "Min"])
def test_max_min_broadcast_with_parameter(tx, op):
    rng = np.random.default_rng(3)
    x = rng.standard_normal((4, 6, 5)).astype(np.float32)
    other = rng.standard_normal((6, 1)).astype(np.float32)
    _check(tx, _model(op, x.shape, inits=[("b", other)]), x)


def test_concat_with_parameter(tx):
    rng = np.random.default_rng(4)
    x = rng.standard_normal((3, 4, 5)).astype(np.float32)
    _check(tx, _model("Concat", x.shape, inits=[("p", rng.standard_normal((3, 2, 5)).astype(np.float32))], axis=1), x)
    _check(tx, _model("Concat", x.shape, inits=[("p", rng.standard_normal((3, 4, 7)).astype(np.float32))],
                      axis=-1), x)


@pytest.mark.parametrize("starts,ends,axes,steps", [
    ([1], [4], [1], [1]),
    ([0, -3], [2, 100], [0, 2], [1, 1]),
    ([5, 0], [-9, 7], [2, 1], [-2, 3]),
])
def test_slice_matches_oracle(tx, starts, ends, axes, steps):
    rng = np.random.default_rng(5)
    x = rng.standard_normal((3, 8, 9)).astype(np.float32)
    consts = [("s", np.array(starts, np.int64)), ("e", np.array(ends, np.int64)),
              ("a", np.array(axes, np.int64)), ("t", np.array(steps, np.int64))]
    _check(tx, _model("Slice", x.shape, consts=consts), x)


@pytest.mark.parametrize("sizes,n_out", [([2, 5, 1], 3), (None, 3), (None, 2)])
def test_split_matches_oracle(tx, sizes, n_out):
    rng = np.random.default_rng(6)
    x = rng.standard_normal((4, 8, 3)).astype(np.float32)
    consts = [("sp", np.array(sizes, np.int64))] if sizes else []
    _check(tx, _model("Split", x.shape, consts=consts, n_out=n_out, axis=1), x)


def test_expand_matches_oracle(tx):
    rng = np.random.default_rng(7)
    x = rng.standard_normal((3, 1, 5)).astype(np.float32)
    _check(tx, _model("Expand", x.shape, consts=[("s", np.array([2, 3, 4, 5], np.int64))]), x)


@pytest.mark.parametrize("attrs", [
    {"kernel_shape": [2, 2], "strides": [2, 2]},
    {"kernel_shape": [3, 3], "strides": [2, 2], "pads": [1, 1, 1, 1]},
    {"kernel_shape": [3, 3], "strides": [2, 2], "pads": [1, 1, 1, 1], "count_include_pad": 1},
    {"kernel_shape": [3, 3], "strides": [2, 2], "ceil_mode": 1, "pads": [0, 1, 1, 0]},
    {"kernel_shape": [3, 2], "strides": [1, 2], "auto_pad": "SAME_UPPER", "count_include_pad": 1},
    {"kernel_shape": [3], "strides": [2], "pads": [1, 1]},
])
def test_average_pool_matches_oracle(tx, attrs):
    rng = np.random.default_rng(8)
    shape = (3, 5, 13, 11) if len(attrs["kernel_shape"]) == 2 else (3, 5, 21)
    x = rng.standard_normal(shape).astype(np.float32)
    _check(tx, _model("AveragePool", x.shape, **attrs), x)


@pytest.mark.parametrize("op,axes,keepdims", [("ReduceMax", [1], 1), ("ReduceMin", [2, 3], 0),
                                              ("ReduceMax", None, 0), ("ReduceMin", [-1], 1)])
def test_reduce_max_min_match_oracle(tx, op, axes, keepdims):
    rng = np.random.default_rng(9)
    x = rng.standard_normal((3, 4, 5, 6)).astype(np.float32)
    kw = {"keepdims": keepdims}
    if axes is not None:
        kw["axes"] = axes
    _check(tx, _model(op, x.shape, **kw), x)


def test_global_max_pool_and_dropout(tx):
    rng = np.random.default_rng(10)
    x = rng.standard_normal((2, 3, 7, 5)).astype(np.float32)
    _check(tx, _model("GlobalMaxPool", x.shape), x)
    _check(tx, _model("Dropout", x.shape, ratio=0.3), x)


def test_inference_session_runs_a_mixed_graph(tx):
    """A Session (no tape) over Conv, AveragePool, Concat, Slice, Softplus,
    ReduceMax and Pow equals the oracle's forward."""
    from tynx_b200.onnx import ir, proto

    rng = np.random.default_rng(11)
    w = (rng.standard_normal((4, 3, 3, 3)) * 0.3).astype(np.float32)
    nodes = [proto.encode_node("Conv", ["x", "w"], ["c"], name="conv", kernel_shape=[3, 3], pads=[1, 1, 1, 1]),
             proto.encode_node("AveragePool", ["c"], ["p"], name="pool", kernel_shape=[2, 2], strides=[2, 2]),
             proto.encode_node("Softplus", ["p"], ["s"], name="sp"),
             proto.encode_node("Concat", ["s", "p"], ["cat"], name="cat", axis=1),
             proto.encode_node("Slice", ["cat", "st", "en", "ax"], ["sl"], name="slice"),
             proto.encode_node("ReduceMax", ["sl"], ["m"], name="rmax", axes=[2, 3], keepdims=0),
             proto.encode_node("Pow", ["m", "two"], ["y"], name="pow")]
    inits = [proto.encode_tensor("w", w), proto.encode_tensor("st", np.array([1], np.int64)),
             proto.encode_tensor("en", np.array([7], np.int64)), proto.encode_tensor("ax", np.array([1], np.int64)),
             proto.encode_tensor("two", np.array(2.0, np.float32))]
    data = proto.encode_model(nodes, inits, [proto.encode_value_info("x", proto.FLOAT, [2, 3, 8, 8])],
                              [proto.encode_value_info("y", proto.FLOAT, None)], opset=13)
    session = tx.load(data)
    x = rng.standard_normal((2, 3, 8, 8)).astype(np.float32)
    y = session(tx.Tensor(x)).numpy()
    ref = fo.OracleModel(ir.load_training_graph(data))(x)
    assert _rel(y, ref.data) <= 1e-5
