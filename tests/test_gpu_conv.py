"""Convolutions on Device("cuda") against the oracle over the geometries the
implicit-GEMM path takes (activation tiles gathered by shifted TMA boxes, the
data gradient split by the phases of the stride) and the ones it hands to
the explicit im2col columns (channel counts that are not multiples of 32,
grids whose rows do not tile 128 pixels, strides that leave a phase without
taps), with the reference's NCHW semantics of executor.rs:315-350 /
tensor.rs:1080-1180 (asymmetric padding, stride, dilation, bias).

Each model is Conv -> Relu -> 1x1 Conv, so the second convolution reads a
channels-last input and applies the Relu derivative in its data gradient.
The forward output and the gradients of the input and of every parameter are
compared with the oracle: at rel 2e-5 in 3xTF32 (fp32-class products) and at
rel 3e-3 in TF32 (11-bit operands).
"""

import numpy as np
import pytest

from oracle import flex_oracle as fo

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def tx():
    import tynx_b200 as tx

    yield tx
    tx.set_math_mode("tf32")


def _conv_model(rng, x_shape, cout, k, strides, pads, dil, cout2=32):
    from tynx_b200.onnx import proto

    cin = x_shape[1]
    kh, kw = k
    w1 = (rng.standard_normal((cout, cin, kh, kw)) / np.sqrt(cin * kh * kw)).astype(np.float32)
    b1 = (rng.standard_normal(cout) * 0.1).astype(np.float32)
    w2 = (rng.standard_normal((cout2, cout, 1, 1)) / np.sqrt(cout)).astype(np.float32)
    b2 = (rng.standard_normal(cout2) * 0.1).astype(np.float32)
    nodes = [proto.encode_node("Conv", ["x", "w1", "b1"], ["c1"], name="conv1", kernel_shape=[kh, kw],
                               strides=list(strides), pads=list(pads), dilations=list(dil)),
             proto.encode_node("Relu", ["c1"], ["r1"], name="relu1"),
             proto.encode_node("Conv", ["r1", "w2", "b2"], ["y"], name="conv2", kernel_shape=[1, 1])]
    inits = [proto.encode_tensor(n, a) for n, a in (("w1", w1), ("b1", b1), ("w2", w2), ("b2", b2))]
    return proto.encode_model(nodes, inits, [proto.encode_value_info("x", proto.FLOAT, list(x_shape))],
                              [proto.encode_value_info("y", proto.FLOAT, None)], opset=13)


def _rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def _check(tx, model_bytes, x_np, tol):
    from tynx_b200.onnx import ir

    model = tx.load(model_bytes, trainable="auto", simplify=False)
    ref = fo.OracleModel(ir.load_training_graph(model_bytes))
    x = tx.Tensor(x_np, requires_grad=True)
    y = model(x)
    xr = fo.T(x_np.copy(), requires_grad=True)
    yr = ref(xr)
    assert y.shape == tuple(yr.shape)
    assert _rel(y.numpy(), yr.data) <= tol, ("y", _rel(y.numpy(), yr.data))
    w = np.random.default_rng(5).standard_normal(yr.shape).astype(np.float32)
    (y * tx.Tensor(w)).sum().backward()
    fo.sum_(yr * fo.T(w)).backward()
    errs = {"x": _rel(x.grad.numpy(), xr.grad)}
    p = dict(model.named_parameters())
    for n, q in ref.named_parameters():
        errs[n] = _rel(p[n].grad.numpy(), q.grad)
    bad = {n: e for n, e in errs.items() if not e <= tol}
    assert not bad, (bad, errs)


# (cin, cout, input h x w, kernel, strides, pads [top, left, bottom, right], dilations, batch)
GEOMETRIES = {
    # implicit forward, weight gradient and data gradient
    "s1_16x16": (32, 64, (16, 16), (3, 3), (1, 1), (1, 1, 1, 1), (1, 1), 4),
    "s2_32x32_cnn_conv2": (32, 64, (32, 32), (3, 3), (2, 2), (1, 1, 1, 1), (1, 1), 3),
    "s2_16x16_cnn_conv3": (64, 128, (16, 16), (3, 3), (2, 2), (1, 1, 1, 1), (1, 1), 3),
    "k5_8x8_two_images_per_tile": (32, 32, (8, 8), (5, 5), (1, 1), (2, 2, 2, 2), (1, 1), 3),
    "dilated_asymmetric_pads": (32, 64, (16, 16), (3, 3), (1, 1), (1, 2, 3, 2), (2, 2), 2),
    "rows_of_64": (32, 32, (64, 64), (3, 3), (1, 1), (1, 1, 1, 1), (1, 1), 2),
    "k2_s2_unpadded": (32, 64, (32, 32), (2, 2), (2, 2), (0, 0, 0, 0), (1, 1), 2),
    # implicit forward, explicit data gradient (phases without taps / odd input)
    "k1_s2_phase_without_taps": (32, 64, (16, 16), (1, 1), (2, 2), (0, 0, 0, 0), (1, 1), 4),
    "s2_odd_input": (32, 64, (15, 15), (3, 3), (2, 2), (1, 1, 1, 1), (1, 1), 4),
    # explicit columns
    "three_channels": (3, 32, (32, 32), (3, 3), (1, 1), (1, 1, 1, 1), (1, 1), 4),
    "rows_of_12": (32, 32, (12, 12), (3, 3), (1, 1), (1, 1, 1, 1), (1, 1), 3),
    "48_out_channels": (32, 48, (16, 16), (3, 3), (2, 2), (1, 1, 1, 1), (1, 1), 2),
    "s2_unpadded_odd_grid": (32, 64, (31, 31), (3, 3), (2, 2), (0, 0, 0, 0), (1, 1), 2),
}


@pytest.mark.parametrize("name", sorted(GEOMETRIES))
def test_conv_matches_oracle_3xtf32(tx, name):
    cin, cout, (h, w), k, s, pads, dil, batch = GEOMETRIES[name]
    rng = np.random.default_rng(sorted(GEOMETRIES).index(name))
    tx.set_math_mode("3xtf32")
    x = rng.standard_normal((batch, cin, h, w)).astype(np.float32)
    _check(tx, _conv_model(rng, x.shape, cout, k, s, pads, dil), x, 2e-5)


@pytest.mark.parametrize("name", ["s1_16x16", "s2_32x32_cnn_conv2", "s2_16x16_cnn_conv3", "three_channels"])
def test_conv_matches_oracle_tf32(tx, name):
    cin, cout, (h, w), k, s, pads, dil, batch = GEOMETRIES[name]
    rng = np.random.default_rng(sorted(GEOMETRIES).index(name))
    tx.set_math_mode("tf32")
    x = rng.standard_normal((batch, cin, h, w)).astype(np.float32)
    _check(tx, _conv_model(rng, x.shape, cout, k, s, pads, dil), x, 3e-3)


def test_conv_gradient_accumulates_across_backward_calls(tx):
    """Two backward passes without zero_grad: the input's gradient (written
    through the phase views, then added into the NCHW leaf) and the
    parameters' gradients accumulate, equal to the oracle's two passes."""
    from tynx_b200.onnx import ir

    rng = np.random.default_rng(11)
    tx.set_math_mode("3xtf32")
    data = _conv_model(rng, (2, 32, 16, 16), 64, (3, 3), (2, 2), (1, 1, 1, 1), (1, 1))
    x_np = rng.standard_normal((2, 32, 16, 16)).astype(np.float32)
    model = tx.load(data, trainable="auto", simplify=False)
    ref = fo.OracleModel(ir.load_training_graph(data))
    x = tx.Tensor(x_np, requires_grad=True)
    xr = fo.T(x_np.copy(), requires_grad=True)
    for _ in range(2):
        model(x).sum().backward()
        fo.sum_(ref(xr)).backward()
    assert _rel(x.grad.numpy(), xr.grad) <= 2e-5
    p = dict(model.named_parameters())
    for n, q in ref.named_parameters():
        assert _rel(p[n].grad.numpy(), q.grad) <= 2e-5, n


def _single_conv(rng, x_shape, cout, k, group=1, **attrs):
    from tynx_b200.onnx import proto

    cin = x_shape[1]
    w = (rng.standard_normal((cout, cin // group) + tuple(k)) / np.sqrt(cin // group * np.prod(k))).astype(np.float32)
    b = (rng.standard_normal(cout) * 0.1).astype(np.float32)
    nodes = [proto.encode_node("Conv", ["x", "w", "b"], ["y"], name="conv", kernel_shape=list(k), group=group,
                               **attrs)]
    inits = [proto.encode_tensor("w", w), proto.encode_tensor("b", b)]
    return proto.encode_model(nodes, inits, [proto.encode_value_info("x", proto.FLOAT, list(x_shape))],
                              [proto.encode_value_info("y", proto.FLOAT, None)], opset=13)


# grouped and 1-D convolutions (the explicit columns, one product per group):
# (input shape, out channels, kernel, group, attributes)
VARIANTS = {
    "grouped_2": ((3, 16, 12, 10), 32, (3, 3), 2, {"pads": [1, 1, 1, 1]}),
    "grouped_4_strided": ((2, 32, 15, 15), 64, (3, 3), 4, {"pads": [1, 0, 1, 2], "strides": [2, 2]}),
    "depthwise": ((4, 8, 9, 9), 8, (3, 3), 8, {"pads": [1, 1, 1, 1]}),
    "depthwise_multiplier_2": ((2, 6, 11, 7), 12, (3, 2), 6, {"dilations": [2, 1]}),
    "conv1d": ((4, 8, 40), 16, (5,), 1, {"pads": [2, 1], "strides": [2]}),
    "conv1d_dilated_grouped": ((3, 12, 33), 24, (3,), 3, {"dilations": [3], "pads": [3, 3]}),
}


@pytest.mark.parametrize("math,tol", [("3xtf32", 2e-5), ("fp32", 2e-5), ("tf32", 3e-3)])
@pytest.mark.parametrize("name", sorted(VARIANTS))
def test_grouped_and_1d_conv_match_oracle(tx, name, math, tol):
    shape, cout, k, group, attrs = VARIANTS[name]
    rng = np.random.default_rng(100 + sorted(VARIANTS).index(name))
    tx.set_math_mode(math)
    x = rng.standard_normal(shape).astype(np.float32)
    _check(tx, _single_conv(rng, shape, cout, k, group, **attrs), x, tol)
