"""Pin the CPU oracle to the reference's own known answers (CPU only).

Each case reproduces an assertion from the reference's tests, recorded with its
file:line in ``tests/golden/expected.json``.
"""

import math

import numpy as np
import pytest

from oracle import flex_oracle as fo
from tynx_b200.onnx import ir


def _model(fixtures, name, **kw):
    return fo.OracleModel(ir.load_training_graph(fixtures[name], **kw))


def test_gemm_forward_backward(fixtures, expected):
    case = expected["gemm_forward_backward"]
    model = _model(fixtures, case["model"],
                   initializer_names={"weight": "head.weight", "bias": "head.bias"})
    x = fo.T(np.asarray(case["input"], np.float32), requires_grad=True)
    y = model(x)
    fo.sum_(y).backward()
    np.testing.assert_allclose(y.data.reshape(-1), case["output"], rtol=1e-6)
    np.testing.assert_allclose(x.grad.reshape(-1), case["input_grad"], rtol=1e-6)
    params = dict(model.named_parameters())
    assert sorted(params) == ["head.bias", "head.weight"]
    np.testing.assert_allclose(params["head.weight"].grad.reshape(-1), case["weight_grad"])
    np.testing.assert_allclose(params["head.bias"].grad.reshape(-1), case["bias_grad"])


def test_gemm_sgd_next_forward(fixtures, expected):
    case = expected["gemm_sgd_next_forward"]
    model = _model(fixtures, case["model"])
    opt = fo.SGD(model.named_parameters(), lr=case["lr"])
    x = np.asarray(case["input"], np.float32)
    fo.sum_(model(x)).backward()
    opt.step()
    np.testing.assert_allclose(model(x).data.reshape(-1), case["next_output"], rtol=1e-6)


def test_clip_gemm(fixtures, expected):
    case = expected["clip_gemm"]
    model = _model(fixtures, case["model"])
    y = model(np.asarray(case["input"], np.float32))
    fo.sum_(y).backward()
    np.testing.assert_allclose(y.data.reshape(-1), case["output"])
    p = dict(model.named_parameters())
    np.testing.assert_allclose(p["weight"].grad.reshape(-1), case["weight_grad"])
    np.testing.assert_allclose(p["bias"].grad.reshape(-1), case["bias_grad"])


def test_gather_accumulation(fixtures, expected):
    case = expected["gather_accumulation"]
    model = _model(fixtures, case["model"])
    idx = np.asarray(case["indices"], np.int64)
    y = model(idx)
    assert y.data.tolist() == case["output"]
    fo.sum_(y).backward()
    w = dict(model.named_parameters())["embedding.weight"]
    assert w.grad.tolist() == case["weight_grad"]
    fo.SGD(model.named_parameters(), lr=case["lr"]).step()
    np.testing.assert_allclose(model(idx).data.reshape(-1), case["next_output"], rtol=1e-6)


def test_layer_norm(fixtures, expected):
    case = expected["layer_norm"]
    model = _model(fixtures, case["model"])
    x = np.asarray(case["input"], np.float32)
    y = model(x)
    np.testing.assert_allclose(y.data.reshape(-1), case["output"], atol=case["abs"])
    fo.sum_(y).backward()
    p = dict(model.named_parameters())
    np.testing.assert_allclose(p["norm.weight"].grad.reshape(-1), case["weight_grad"],
                               atol=case["abs"])
    np.testing.assert_allclose(p["norm.bias"].grad.reshape(-1), case["bias_grad"],
                               atol=case["abs"])
    fo.SGD(model.named_parameters(), lr=case["lr"]).step()
    np.testing.assert_allclose(model(x).data.reshape(-1), case["next_output"], atol=case["abs"])


def test_batched_matmul(fixtures, expected):
    case = expected["batched_matmul"]
    model = _model(fixtures, case["model"])
    y = model(np.asarray(case["input"], np.float32))
    assert y.shape == (2, 2, 2)
    np.testing.assert_allclose(y.data.reshape(-1), case["output"])
    fo.sum_(y).backward()
    w = dict(model.named_parameters())["projection.weight"]
    np.testing.assert_allclose(w.grad.reshape(-1), case["weight_grad"])


def _scalar_param(value):
    return fo.T(np.asarray([value], np.float32), requires_grad=True)


def test_adam_constant_gradient(expected):
    case = expected["adam_constant_gradient"]
    p = _scalar_param(case["weight"])
    opt = fo.Adam([p], lr=case["lr"])
    for want in case["trajectory"]:
        p.grad = np.asarray([case["grad"]], np.float32)
        opt.step()
        assert abs(p.data[0] - want) < 1e-6


def test_adam_vs_adamw(expected):
    case = expected["adam_vs_adamw_decay"]
    for decoupled, want in ((False, case["adam"]), (True, case["adamw"])):
        p = _scalar_param(case["weight"])
        p.grad = np.asarray([case["grad"]], np.float32)
        fo.Adam([p], lr=case["lr"], betas=tuple(case["betas"]), eps=case["eps"],
                weight_decay=case["weight_decay"], decoupled=decoupled).step()
        assert abs(p.data[0] - want) < 1e-6


def test_amsgrad(expected):
    case = expected["amsgrad"]
    p = _scalar_param(case["weight"])
    opt = fo.Adam([p], lr=case["lr"], betas=tuple(case["betas"]), eps=case["eps"], amsgrad=True)
    for g in case["grads"]:
        p.grad = np.asarray([g], np.float32)
        opt.step()
    assert abs(p.data[0] - case["final"]) < 1e-6


def test_sgd_goldens(expected):
    """Plain SGD and coupled weight decay land exactly on the f32 values the
    reference asserts; momentum with dampening follows its two-step trajectory
    (the first step takes the gradient undamped)."""
    case = expected["sgd_goldens"]
    c = case["plain"]
    p = _scalar_param(case["weight"])
    p.grad = np.asarray([c["grad"]], np.float32)
    fo.SGD([p], lr=c["lr"]).step()
    assert p.data[0] == np.float32(c["after"])
    c = case["weight_decay"]
    p = _scalar_param(case["weight"])
    p.grad = np.asarray([c["grad"]], np.float32)
    fo.SGD([p], lr=c["lr"], weight_decay=c["weight_decay"]).step()
    assert p.data[0] == np.float32(c["after"])
    c = case["momentum"]
    p = _scalar_param(case["weight"])
    opt = fo.SGD([p], lr=c["lr"], momentum=c["momentum"], dampening=c["dampening"])
    for want in c["trajectory"]:
        p.grad = np.asarray([c["grad"]], np.float32)
        opt.step()
        assert abs(p.data[0] - want) < 1e-6


def test_softmax_and_log_softmax(expected):
    case = expected["softmax_axis0"]
    y = fo.softmax(fo.T(np.asarray(case["input"], np.float32)), case["axis"])
    np.testing.assert_allclose(y.data, case["output"], atol=case["abs"])
    case = expected["log_softmax_stable"]
    y = fo.log_softmax(fo.T(np.asarray(case["input"], np.float32)), 0)
    np.testing.assert_allclose(y.data, case["output"], atol=case["abs"])


def test_gelu_exact(expected):
    case = expected["gelu_exact_erf"]
    y = fo.gelu(fo.T(np.asarray(case["input"], np.float32)))
    np.testing.assert_allclose(y.data, case["output"], atol=case["abs"])


def test_mse(expected):
    case = expected["mse"]
    loss = fo.mse_loss(fo.T(np.asarray(case["prediction"], np.float32)), case["target"])
    assert abs(loss.item() - case["loss"]) < 1e-6


def test_ppo_trains(fixtures, expected):
    case = expected["ppo_training"]
    names = {"policy_weight": "policy.weight", "policy_bias": "policy.bias",
             "value_weight": "value.weight", "value_bias": "value.bias"}
    model = _model(fixtures, case["model"], initializer_names=names)
    obs = np.asarray(case["observations"], np.float32)
    actions = np.asarray(case["actions"], np.int64)
    ln, vn = model.graph.outputs
    out = model(obs)
    old = fo.Categorical(out[ln].detach()).log_prob(actions).data
    np.testing.assert_allclose(old, [expected["ppo_initial_log_prob"]["old_log_prob"]] * 4,
                               rtol=1e-6)

    def loss_fn():
        o = model(obs)
        loss = fo.ppo_loss(o[ln], o[vn], actions, old, case["advantages"], case["returns"])
        vl = fo.mse_loss(fo.reshape(o[vn], (4,)), case["returns"])
        return loss, vl

    l0, v0 = loss_fn()
    opt = fo.Adam(model.named_parameters(), lr=case["lr"])
    for _ in range(case["steps"]):
        opt.zero_grad()
        loss, _ = loss_fn()
        loss.backward()
        opt.step()
    l1, v1 = loss_fn()
    assert l1.item() < l0.item()
    assert v1.item() < v0.item() * case["final_value_loss_ratio_below"]
    probs = fo.Categorical(model(obs)[ln]).probs.data
    chosen = probs[np.arange(4), actions].mean()
    assert chosen > case["chosen_probability_above"]


@pytest.mark.parametrize("name", ["_CNN_MODEL", "_RECOMMENDER_MODEL", "_TRANSFORMER_MODEL"])
def test_composed_models_train(fixtures, expected, name):
    spec = expected["composed_training"]
    case = spec["cases"][name]
    graph = ir.load_training_graph(fixtures[name])
    assert graph.report.warnings == []
    assert sorted(graph.report.trainable_parameters) == case["trainable"]
    model = fo.OracleModel(graph)
    dtype = np.int64 if case.get("input_dtype") == "int64" else np.float32
    x = np.asarray(case["input"], dtype)
    target = np.asarray(case["target"], np.float32)
    opt = fo.Adam(model.named_parameters(), lr=spec["lr"])
    initial = fo.mse_loss(model(x), target).item()
    for _ in range(spec["steps"]):
        opt.zero_grad()
        loss = fo.mse_loss(model(x), target)
        loss.backward()
        opt.step()
    final = fo.mse_loss(model(x), target).item()
    assert final < initial * spec["final_ratio_below"]
    assert all(p.grad is not None for _, p in model.named_parameters())


def test_conv_finite_differences():
    """Central differences check the conv backward (as the reference's robustness
    test does for conv and LayerNorm, test_training_robustness.py:17-59).  The
    convolution is linear in each argument, so a large step is exact up to f32
    rounding."""
    rng = np.random.default_rng(0)
    x = fo.T(rng.standard_normal((2, 3, 6, 5)).astype(np.float32), requires_grad=True)
    w = fo.T(rng.standard_normal((4, 3, 3, 3)).astype(np.float32), requires_grad=True)
    b = fo.T(rng.standard_normal(4).astype(np.float32), requires_grad=True)
    probe = rng.standard_normal((2, 4, 3, 2)).astype(np.float32)

    def f():
        y = fo.conv2d(x, w, b, (2, 2), (1, 1, 1, 0), (1, 1))
        return float((y.data.astype(np.float64) * probe).sum()), y

    _, y = f()
    y.backward(probe)
    for tensor in (x, w, b):
        flat = tensor.data.reshape(-1)
        for i in rng.choice(flat.size, min(6, flat.size), replace=False):
            old = flat[i]
            flat[i] = old + np.float32(0.5)
            up, _ = f()
            flat[i] = old - np.float32(0.5)
            down, _ = f()
            flat[i] = old
            assert math.isclose(tensor.grad.reshape(-1)[i], (up - down) / 1.0, rel_tol=1e-3,
                                abs_tol=1e-3)


def test_gemm_learns_line(gemm_line_model, expected):
    """100 SGD steps on the mean squared error fit y = 2x + 1 through the
    imported Gemm; the first forward reads the zero initializers."""
    case = expected["gemm_learns_line"]
    model = fo.OracleModel(ir.load_training_graph(gemm_line_model,
                                                  initializer_names={"weight": "head.weight",
                                                                     "bias": "head.bias"}))
    x = np.asarray(case["input"], np.float32)
    target = np.asarray(case["target"], np.float32)
    assert model(x).data.reshape(-1).tolist() == case["output_before"]
    opt = fo.SGD(model.named_parameters(), lr=case["lr"])
    for _ in range(case["steps"]):
        opt.zero_grad()
        fo.mse_loss(model(x), target).backward()
        opt.step()
    params = dict(model.named_parameters())
    tol = case["tolerance"]
    assert abs(float(params["head.weight"].data.reshape(-1)[0]) - case["weight"]) < tol
    assert abs(float(params["head.bias"].data.reshape(-1)[0]) - case["bias"]) < tol
    np.testing.assert_allclose(model(x).data, target, atol=tol)


def test_reference_finite_difference_points(expected):
    """The reference's own central-difference checks, on its inputs: the
    conv2d input gradient at element 0 and the LayerNorm (unit scale, zero
    shift) input gradient of sum(y * coefficients) at element 1."""
    c = expected["conv2d_finite_difference"]
    w = fo.T(np.asarray(c["weight"], np.float32))

    def conv_sum(values):
        return float(fo.conv2d(fo.T(values), w, None, (1, 1), (0, 0, 0, 0), (1, 1)).data.sum())

    x0 = np.asarray(c["input"], np.float32)
    x = fo.T(x0.copy(), requires_grad=True)
    y = fo.conv2d(x, w, None, (1, 1), (0, 0, 0, 0), (1, 1))
    y.backward(np.ones_like(y.data))
    i, e = c["element"], c["epsilon"]
    up, down = x0.copy(), x0.copy()
    up.reshape(-1)[i] += np.float32(e)
    down.reshape(-1)[i] -= np.float32(e)
    numerical = (conv_sum(up) - conv_sum(down)) / (2 * e)
    assert x.grad.reshape(-1)[i] == pytest.approx(numerical, rel=c["rel"], abs=c["abs"])

    c = expected["layer_norm_finite_difference"]
    coef = np.asarray(c["coefficients"], np.float32)
    scale, shift = fo.T(np.ones(3, np.float32)), fo.T(np.zeros(3, np.float32))

    def ln_sum(values):
        (out,) = fo.layer_norm(fo.T(values), scale, shift, -1, c["eps"], 1)
        return float((out.data * coef).sum())

    x0 = np.asarray(c["input"], np.float32)
    x = fo.T(x0.copy(), requires_grad=True)
    (y,) = fo.layer_norm(x, scale, shift, -1, c["eps"], 1)
    y.backward(np.broadcast_to(coef, y.data.shape).copy())
    i, e = c["element"], c["epsilon"]
    up, down = x0.copy(), x0.copy()
    up.reshape(-1)[i] += np.float32(e)
    down.reshape(-1)[i] -= np.float32(e)
    numerical = (ln_sum(up) - ln_sum(down)) / (2 * e)
    assert x.grad.reshape(-1)[i] == pytest.approx(numerical, rel=c["rel"], abs=c["abs"])



def _new_op(new_op_models, name):
    data, names = new_op_models[name]
    return fo.OracleModel(ir.load_training_graph(data, initializer_names=names))


def test_batch_norm_trains_affine_state_with_frozen_statistics(new_op_models):
    """crates/tynx-train/src/imported_model/tests.rs:447-480."""
    model = _new_op(new_op_models, "batch_norm")
    graph = ir.load_training_graph(new_op_models["batch_norm"][0],
                                   initializer_names=new_op_models["batch_norm"][1])
    assert sorted(graph.buffers) == ["norm.running_mean", "norm.running_var"]
    y = model(np.array([[3, 8], [5, 11]], np.float32))
    np.testing.assert_array_equal(y.data.reshape(-1), [2.5, 5.0, 4.5, 8.0])
    fo.sum_(y).backward()
    p = dict(model.named_parameters())
    assert sorted(p) == ["norm.bias", "norm.weight"]
    np.testing.assert_array_equal(p["norm.weight"].grad, [3.0, 5.0])
    np.testing.assert_array_equal(p["norm.bias"].grad, [2.0, 2.0])


def test_batch_norm_uses_running_statistics():
    """crates/tynx/src/interpreter/normalization.rs:408-440 (epsilon 0)."""
    x = fo.T(np.array([1, 3, 2, 6], np.float32).reshape(1, 2, 2))
    y = fo.batch_norm(x, fo.T(np.array([2, 0.5], np.float32)), fo.T(np.array([1, -1], np.float32)),
                      fo.T(np.array([1, 2], np.float32)), fo.T(np.array([4, 1], np.float32)), 0.0)
    np.testing.assert_array_equal(y.data.reshape(-1), [1.0, 3.0, -1.0, 1.0])


def test_prelu_trains_its_slope(new_op_models):
    """crates/tynx-train/src/imported_model/tests.rs:527-568."""
    model = _new_op(new_op_models, "prelu")
    x = np.array([-2.0, 3.0], np.float32)
    y = model(x)
    np.testing.assert_array_equal(y.data, [-0.5, 3.0])
    fo.sum_(y).backward()
    slope = dict(model.named_parameters())["activation.weight"]
    np.testing.assert_array_equal(slope.grad, [-2.0])
    fo.SGD(model.named_parameters(), lr=0.1).step()
    np.testing.assert_allclose(model(x).data, [-0.9, 3.0], rtol=1e-6)


def test_instance_norm_custom_epsilon():
    """crates/tynx/src/interpreter/normalization.rs:505-545."""
    eps = 1e-3
    x = fo.T(np.array([1, 3, 2, 6], np.float32).reshape(1, 2, 2))
    y = fo.group_norm(x, fo.T(np.array([2, 0.5], np.float32)), fo.T(np.array([1, -1], np.float32)), 2, eps)
    first, second = 1 / np.sqrt(np.float32(1 + eps)), 2 / np.sqrt(np.float32(4 + eps))
    np.testing.assert_allclose(y.data.reshape(-1),
                               [1 - 2 * first, 1 + 2 * first, -1 - 0.5 * second, -1 + 0.5 * second],
                               atol=1e-5)


@pytest.mark.parametrize("name,x", [("instance_norm", [[[1, 3], [2, 6]]]),
                                    ("group_norm", [[[1, 3], [2, 6], [-1, 1], [4, 8]]])])
def test_instance_and_group_norm_train_affine_slots(new_op_models, name, x):
    """crates/tynx-train/src/imported_model/tests.rs:570-644: loss = sum(y^2) + sum(y)."""
    model = _new_op(new_op_models, name)
    x = np.asarray(x, np.float32)
    y = model(x)
    before = y.data.copy()
    (fo.sum_(y * y) + fo.sum_(y)).backward()
    p = dict(model.named_parameters())
    assert sorted(p) == ["norm.bias", "norm.weight"]
    assert all(q.grad is not None for q in p.values())
    fo.SGD(model.named_parameters(), lr=0.05).step()
    assert not np.array_equal(model(x).data, before)
