"""Trainable operators beyond the five configurations on Device("cuda"):
BatchNormalization with fixed statistics, PRelu, Instance / GroupNormalization
and MaxPool (the training registry of crates/tynx-train/src/backward_support.rs:106-179).

* the reference's own known answers for each (tests.rs:447-644 of
  crates/tynx-train/src/imported_model, normalization.rs:408-545 of
  crates/tynx/src/interpreter), through ``tx.load`` and backward;
* forward, input gradient and parameter gradients of each operator on seeded
  random data against the oracle (fp32 arithmetic on both sides: these are
  elementwise and reduction kernels, checked at rel 1e-5; the forwards that are
  single rounded f32 expressions are checked bit for bit);
* a CNN that chains them (Conv, BatchNorm, Relu, MaxPool, Conv, InstanceNorm,
  PRelu, GroupNorm, global average pool, Gemm) trains in step with the oracle.
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


def _load(tx, new_op_models, name):
    data, names = new_op_models[name]
    return tx.load(data, trainable="auto", simplify=False, initializer_names=names)


def test_batch_norm_trains_affine_state_with_frozen_statistics(tx, new_op_models):
    model = _load(tx, new_op_models, "batch_norm")
    assert sorted(n for n, _ in model.named_buffers()) == ["norm.running_mean", "norm.running_var"]
    buffers = {n: b.numpy().copy() for n, b in model.named_buffers()}
    x = tx.Tensor(np.array([[3, 8], [5, 11]], np.float32))
    y = model(x)
    assert y.flatten().tolist() == [2.5, 5.0, 4.5, 8.0]
    y.sum().backward()
    p = dict(model.named_parameters())
    assert sorted(p) == ["norm.bias", "norm.weight"]
    assert p["norm.weight"].grad.tolist() == [3.0, 5.0]
    assert p["norm.bias"].grad.tolist() == [2.0, 2.0]
    tx.optim.SGD(model.named_parameters(), lr=0.1).step()
    for n, b in model.named_buffers():
        np.testing.assert_array_equal(b.numpy(), buffers[n])
    state = model.state_dict()
    assert sorted(state) == ["norm.bias", "norm.running_mean", "norm.running_var", "norm.weight"]


def test_batch_norm_reads_its_buffers_live(tx, new_op_models):
    model = _load(tx, new_op_models, "batch_norm")
    state = model.state_dict()
    state["norm.running_mean"] = tx.Tensor(np.array([3, 8], np.float32))
    model.load_state_dict(state)
    y = model(tx.Tensor(np.array([[3, 8], [5, 11]], np.float32)))
    # ((x - [3, 8]) / [2, 3]) * [2, 3] + [0.5, -1]
    assert y.flatten().tolist() == [0.5, -1.0, 2.5, 2.0]


def test_prelu_trains_its_slope(tx, new_op_models):
    model = _load(tx, new_op_models, "prelu")
    x = tx.Tensor(np.array([-2.0, 3.0], np.float32))
    y = model(x)
    assert y.tolist() == [-0.5, 3.0]
    y.sum().backward()
    slope = dict(model.named_parameters())["activation.weight"]
    assert slope.grad.tolist() == [-2.0]
    tx.optim.SGD(model.named_parameters(), lr=0.1).step()
    assert model(x).tolist() == pytest.approx([-0.9, 3.0], rel=1e-6)


@pytest.mark.parametrize("name,x", [("instance_norm", [[[1, 3], [2, 6]]]),
                                    ("group_norm", [[[1, 3], [2, 6], [-1, 1], [4, 8]]])])
def test_instance_and_group_norm_train_affine_slots(tx, new_op_models, name, x):
    model = _load(tx, new_op_models, name)
    data, names = new_op_models[name]
    from tynx_b200.onnx import ir

    ref = fo.OracleModel(ir.load_training_graph(data, initializer_names=names))
    xs = np.asarray(x, np.float32)
    y = model(tx.Tensor(xs))
    yr = ref(xs)
    np.testing.assert_allclose(y.numpy(), yr.data, rtol=1e-6, atol=1e-6)
    before = y.numpy().copy()
    (y * y).sum().backward()
    (fo.sum_(yr * yr)).backward()
    y2 = model(tx.Tensor(xs))
    y2.sum().backward()
    fo.sum_(ref(xs)).backward()
    p = dict(model.named_parameters())
    assert sorted(p) == ["norm.bias", "norm.weight"]
    for n, q in ref.named_parameters():
        np.testing.assert_allclose(p[n].grad.numpy(), q.grad, rtol=1e-5, atol=1e-6, err_msg=n)
    tx.optim.SGD(model.named_parameters(), lr=0.05).step()
    assert not np.array_equal(model(tx.Tensor(xs)).numpy(), before)


def test_instance_norm_custom_epsilon(tx):
    from tynx_b200.onnx import proto

    nodes = [proto.encode_node("InstanceNormalization", ["x", "scale", "bias"], ["y"], name="n",
                               epsilon=1e-3)]
    inits = [proto.encode_tensor("scale", np.array([2, 0.5], np.float32)),
             proto.encode_tensor("bias", np.array([1, -1], np.float32))]
    model = tx.load(proto.encode_model(nodes, inits, [proto.encode_value_info("x", proto.FLOAT, [1, 2, 2])],
                                       [proto.encode_value_info("y", proto.FLOAT, [1, 2, 2])], opset=13),
                    trainable="auto", simplify=False)
    y = model(tx.Tensor(np.array([1, 3, 2, 6], np.float32).reshape(1, 2, 2)))
    first, second = 1 / np.sqrt(np.float32(1.001)), 2 / np.sqrt(np.float32(4.001))
    np.testing.assert_allclose(y.numpy().reshape(-1),
                               [1 - 2 * first, 1 + 2 * first, -1 - 0.5 * second, -1 + 0.5 * second],
                               atol=1e-5)


# -- seeded random parity against the oracle -----------------------------------------------------

def _one_op(op, x_shape, inits, opset=13, **attrs):
    from tynx_b200.onnx import proto

    names = ["x"] + [n for n, _ in inits]
    nodes = [proto.encode_node(op, names, ["y"], name="op", **attrs)]
    enc = [proto.encode_tensor(n, a) for n, a in inits]
    return proto.encode_model(nodes, enc, [proto.encode_value_info("x", proto.FLOAT, list(x_shape))],
                              [proto.encode_value_info("y", proto.FLOAT, None)], opset=opset)


def _check_op(tx, model_bytes, x_np, exact_forward=False, tol=1e-5):
    from tynx_b200.onnx import ir

    model = tx.load(model_bytes, trainable="auto", simplify=False)
    ref = fo.OracleModel(ir.load_training_graph(model_bytes))
    x = tx.Tensor(x_np, requires_grad=True)
    y = model(x)
    xr = fo.T(x_np.copy(), requires_grad=True)
    yr = ref(xr)
    if exact_forward:
        np.testing.assert_array_equal(y.numpy(), yr.data)
    else:
        np.testing.assert_allclose(y.numpy(), yr.data, rtol=tol, atol=tol)
    w = np.random.default_rng(5).standard_normal(yr.shape).astype(np.float32)
    (y * tx.Tensor(w)).sum().backward()
    fo.sum_(yr * fo.T(w)).backward()

    def rel(a, b):
        a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
        return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))

    assert rel(x.grad.numpy(), xr.grad) <= tol, rel(x.grad.numpy(), xr.grad)
    p = dict(model.named_parameters())
    for n, q in ref.named_parameters():
        assert rel(p[n].grad.numpy(), q.grad) <= tol, (n, rel(p[n].grad.numpy(), q.grad))


def test_batch_norm_matches_oracle(tx):
    rng = np.random.default_rng(0)
    C = 24
    inits = [("s", rng.standard_normal(C).astype(np.float32)), ("b", rng.standard_normal(C).astype(np.float32)),
             ("m", rng.standard_normal(C).astype(np.float32)),
             ("v", rng.uniform(0.5, 2.0, C).astype(np.float32))]
    for shape in ((16, C, 9, 7), (64, C)):
        x = rng.standard_normal(shape).astype(np.float32)
        _check_op(tx, _one_op("BatchNormalization", shape, inits, epsilon=1e-5), x, exact_forward=True)


@pytest.mark.parametrize("op,groups", [("InstanceNormalization", None), ("GroupNormalization", 4),
                                       ("GroupNormalization", 1)])
def test_group_and_instance_norm_match_oracle(tx, op, groups):
    rng = np.random.default_rng(1)
    C = 16
    inits = [("s", rng.standard_normal(C).astype(np.float32)), ("b", rng.standard_normal(C).astype(np.float32))]
    kw = {"num_groups": groups} if groups else {}
    x = (rng.standard_normal((6, C, 11, 13)) * 3 + 1).astype(np.float32)
    _check_op(tx, _one_op(op, x.shape, inits, opset=18 if groups else 13, **kw), x)


@pytest.mark.parametrize("slope_shape", [(1,), (12, 1, 1), (12, 5, 6)])
def test_prelu_matches_oracle(tx, slope_shape):
    rng = np.random.default_rng(2)
    slope = rng.uniform(-0.5, 0.5, slope_shape).astype(np.float32)
    x = rng.standard_normal((4, 12, 5, 6)).astype(np.float32)
    _check_op(tx, _one_op("PRelu", x.shape, [("slope", slope)]), x, exact_forward=True)


@pytest.mark.parametrize("attrs", [
    {"kernel_shape": [2, 2], "strides": [2, 2]},
    {"kernel_shape": [3, 3], "strides": [2, 2], "pads": [1, 1, 1, 1]},
    {"kernel_shape": [3, 3], "strides": [2, 2], "ceil_mode": 1},
    {"kernel_shape": [3, 2], "strides": [1, 2], "dilations": [2, 1], "pads": [2, 0, 1, 1]},
    {"kernel_shape": [3, 3], "strides": [2, 2], "auto_pad": "SAME_UPPER"},
    {"kernel_shape": [3], "strides": [2], "pads": [1, 1]},
])
def test_maxpool_matches_oracle(tx, attrs):
    rng = np.random.default_rng(3)
    shape = (3, 5, 17, 14) if len(attrs["kernel_shape"]) == 2 else (3, 5, 21)
    x = rng.standard_normal(shape).astype(np.float32)
    _check_op(tx, _one_op("MaxPool", shape, [], **attrs), x, exact_forward=True)


def _registry_cnn(seed=0, batch=8):
    from tynx_b200.onnx import proto

    rng = np.random.default_rng(seed)
    f = np.float32
    n = lambda *a, **k: proto.encode_node(*a, **k)  # noqa: E731
    inits = [
        ("c1.w", (rng.standard_normal((16, 3, 3, 3)) * 0.3).astype(f)), ("c1.b", np.zeros(16, f)),
        ("bn.s", rng.uniform(0.5, 1.5, 16).astype(f)), ("bn.b", (rng.standard_normal(16) * 0.1).astype(f)),
        ("bn.m", (rng.standard_normal(16) * 0.1).astype(f)), ("bn.v", rng.uniform(0.5, 1.5, 16).astype(f)),
        ("c2.w", (rng.standard_normal((32, 16, 3, 3)) * 0.1).astype(f)), ("c2.b", np.zeros(32, f)),
        ("in.s", np.ones(32, f)), ("in.b", np.zeros(32, f)),
        ("pr.a", np.full((32, 1, 1), 0.2, f)),
        ("gn.s", np.ones(32, f)), ("gn.b", np.zeros(32, f)),
        ("fc.w", (rng.standard_normal((10, 32)) * 0.2).astype(f)), ("fc.b", np.zeros(10, f)),
    ]
    nodes = [
        n("Conv", ["x", "c1.w", "c1.b"], ["c1"], name="c1", kernel_shape=[3, 3], pads=[1, 1, 1, 1]),
        n("BatchNormalization", ["c1", "bn.s", "bn.b", "bn.m", "bn.v"], ["bn"], name="bn", epsilon=1e-5),
        n("Relu", ["bn"], ["r1"], name="r1"),
        n("MaxPool", ["r1"], ["p1"], name="p1", kernel_shape=[2, 2], strides=[2, 2]),
        n("Conv", ["p1", "c2.w", "c2.b"], ["c2"], name="c2", kernel_shape=[3, 3], pads=[1, 1, 1, 1]),
        n("InstanceNormalization", ["c2", "in.s", "in.b"], ["in"], name="in", epsilon=1e-5),
        n("PRelu", ["in", "pr.a"], ["pr"], name="pr"),
        n("GroupNormalization", ["pr", "gn.s", "gn.b"], ["gn"], name="gn", num_groups=8, epsilon=1e-5),
        n("GlobalAveragePool", ["gn"], ["gap"], name="gap"),
        n("Flatten", ["gap"], ["feat"], name="flat", axis=1),
        n("Gemm", ["feat", "fc.w", "fc.b"], ["logits"], name="fc", transB=1),
    ]
    model = proto.encode_model(nodes, [proto.encode_tensor(k, v) for k, v in inits],
                               [proto.encode_value_info("x", proto.FLOAT, ["batch", 3, 16, 16])],
                               [proto.encode_value_info("logits", proto.FLOAT, ["batch", 10])], opset=18)
    data = np.random.default_rng(100 + seed)
    batches = [(data.standard_normal((batch, 3, 16, 16)).astype(f), data.integers(0, 10, batch))
               for _ in range(5)]
    return model, batches


@pytest.mark.parametrize("math", ["fp32", "3xtf32"])
def test_registry_cnn_trains_with_the_oracle(tx, math):
    """Five Adam steps of the chained-operator CNN: the loss at every step within
    rel 1e-5 of the oracle's, every gradient of the first step within 1e-4
    (relative L2; Relu and MaxPool selections flip where a value lies within
    rounding of its neighbour, the fp32 oracle's own float64 distance is allowed)."""
    from tynx_b200.onnx import ir

    tx.set_math_mode(math)
    try:
        model_bytes, batches = _registry_cnn()
        model = tx.load(model_bytes, trainable="auto")
        opt = tx.optim.Adam(model.named_parameters(), lr=1e-3)
        graph = ir.load_training_graph(model_bytes)
        ref = fo.OracleModel(graph)
        ref_opt = fo.Adam(ref.named_parameters(), lr=1e-3)
        with fo.precision(np.float64):
            ref64 = fo.OracleModel(graph)
        for i, (x, y) in enumerate(batches):
            opt.zero_grad()
            loss = tx.nn.functional.cross_entropy(model(tx.Tensor(x)), tx.Tensor(y))
            loss.backward()
            grads = {n: p.grad.numpy() for n, p in model.named_parameters()}
            opt.step()
            ref_opt.zero_grad()
            ref_loss = fo.cross_entropy(ref(x), y)
            ref_loss.backward()
            if i == 0:
                with fo.precision(np.float64):
                    l64 = fo.cross_entropy(ref64(x), y)
                    l64.backward()
                for n, q in ref.named_parameters():
                    g64 = dict(ref64.named_parameters())[n].grad
                    err = np.linalg.norm(grads[n] - g64) / np.linalg.norm(g64)
                    err32 = np.linalg.norm(q.grad - g64) / np.linalg.norm(g64)
                    assert err <= max(1e-4, 2 * err32), (n, err, err32)
            ref_opt.step()
            assert abs(loss.item() - ref_loss.item()) <= 1e-5 * max(1.0, abs(ref_loss.item())), \
                (i, loss.item(), ref_loss.item())
    finally:
        tx.set_math_mode("fp32")
