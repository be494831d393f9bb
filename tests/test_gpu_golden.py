"""The reference's own known answers, reproduced through the CUDA engine's public API.

Each case mirrors an assertion in the reference's tests (file:line recorded in
``tests/golden/expected.json``) and runs on ``Device("cuda")``.
"""

import math

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def tx():
    import tynx_b200 as tx

    tx.set_math_mode("fp32")  # the goldens are exact small-integer fp32 cases
    yield tx
    tx.set_math_mode("tf32")


def _load(tx, fixtures, name, **kw):
    return tx.load(fixtures[name], trainable="auto", simplify=False, **kw)


def test_gemm_forward_backward(tx, fixtures, expected):
    case = expected["gemm_forward_backward"]
    model = _load(tx, fixtures, case["model"],
                  initializer_names={"weight": "head.weight", "bias": "head.bias"})
    x = tx.Tensor(case["input"], requires_grad=True)
    y = model(x)
    y.sum().backward()
    assert y.flatten().tolist() == pytest.approx(case["output"])
    assert x.grad.flatten().tolist() == pytest.approx(case["input_grad"])
    params = dict(model.named_parameters())
    assert sorted(params) == ["head.bias", "head.weight"]
    assert params["head.weight"].grad.flatten().tolist() == pytest.approx(case["weight_grad"])
    assert params["head.bias"].grad.tolist() == pytest.approx(case["bias_grad"])


def test_gemm_sgd_next_forward(tx, fixtures, expected):
    case = expected["gemm_sgd_next_forward"]
    model = _load(tx, fixtures, case["model"])
    opt = tx.optim.SGD(model.named_parameters(), lr=case["lr"])
    x = tx.Tensor(case["input"])
    model(x).sum().backward()
    opt.step()
    assert model(x).flatten().tolist() == pytest.approx(case["next_output"])


def test_clip_gemm(tx, fixtures, expected):
    case = expected["clip_gemm"]
    model = _load(tx, fixtures, case["model"])
    y = model(tx.Tensor(case["input"]))
    assert y.flatten().tolist() == pytest.approx(case["output"])
    y.sum().backward()
    p = dict(model.named_parameters())
    assert p["weight"].grad.flatten().tolist() == pytest.approx(case["weight_grad"])
    assert p["bias"].grad.tolist() == pytest.approx(case["bias_grad"])


def test_gather_accumulates_repeated_rows(tx, fixtures, expected):
    case = expected["gather_accumulation"]
    model = _load(tx, fixtures, case["model"])
    idx = tx.Tensor(case["indices"], dtype="int64")
    y = model(idx)
    assert y.tolist() == case["output"]
    y.sum().backward()
    w = dict(model.named_parameters())["embedding.weight"]
    assert w.grad.tolist() == case["weight_grad"]
    tx.optim.SGD(model.named_parameters(), lr=case["lr"]).step()
    assert model(idx).flatten().tolist() == pytest.approx(case["next_output"])


def test_gather_out_of_range_raises_index_error(tx, fixtures):
    model = _load(tx, fixtures, "_GATHER_MODEL")
    with pytest.raises(IndexError):
        model(tx.Tensor([0, 3], dtype="int64")).tolist()


def test_layer_norm(tx, fixtures, expected):
    case = expected["layer_norm"]
    model = _load(tx, fixtures, case["model"])
    x = tx.Tensor(case["input"])
    y = model(x)
    assert y.flatten().tolist() == pytest.approx(case["output"], abs=case["abs"])
    y.sum().backward()
    p = dict(model.named_parameters())
    assert p["norm.weight"].grad.flatten().tolist() == pytest.approx(case["weight_grad"],
                                                                       abs=case["abs"])
    assert p["norm.bias"].grad.tolist() == pytest.approx(case["bias_grad"], abs=case["abs"])
    tx.optim.SGD(model.named_parameters(), lr=case["lr"]).step()
    assert model(x).flatten().tolist() == pytest.approx(case["next_output"], abs=case["abs"])


def test_batched_matmul(tx, fixtures, expected):
    case = expected["batched_matmul"]
    model = _load(tx, fixtures, case["model"])
    y = model(tx.Tensor(case["input"]))
    assert y.shape == (2, 2, 2)
    assert y.flatten().tolist() == pytest.approx(case["output"])
    y.sum().backward()
    w = dict(model.named_parameters())["projection.weight"]
    assert w.grad.flatten().tolist() == pytest.approx(case["weight_grad"])


def test_sgd_goldens(tx, fixtures, expected):
    """The reference's SGD known answers on a slot holding 2.0: plain and
    coupled weight decay exactly in f32, momentum with dampening over two
    steps (the first takes the gradient undamped) to 1e-6."""
    case = expected["sgd_goldens"]

    def weight():
        p = dict(_load(tx, fixtures, "_GEMM_MODEL").named_parameters())["weight"]
        assert p.item() == case["weight"]
        return p

    c = case["plain"]
    p = weight()
    p.grad = tx.Tensor([[c["grad"]]])
    tx.optim.SGD([p], lr=c["lr"]).step()
    assert np.float32(p.item()) == np.float32(c["after"])
    c = case["weight_decay"]
    p = weight()
    p.grad = tx.Tensor([[c["grad"]]])
    tx.optim.SGD([p], lr=c["lr"], weight_decay=c["weight_decay"]).step()
    assert np.float32(p.item()) == np.float32(c["after"])
    c = case["momentum"]
    p = weight()
    opt = tx.optim.SGD([p], lr=c["lr"], momentum=c["momentum"], dampening=c["dampening"])
    for want in c["trajectory"]:
        p.grad = tx.Tensor([[c["grad"]]])
        opt.step()
        assert p.item() == pytest.approx(want, abs=1e-6)


def test_adam_goldens(tx, fixtures, expected):
    model = _load(tx, fixtures, "_GEMM_MODEL")
    w = dict(model.named_parameters())["weight"]
    opt = tx.optim.Adam([w], lr=0.1)
    for want in expected["adam_constant_gradient"]["trajectory"]:
        w.grad = tx.Tensor([[2.0]])
        opt.step()
        assert w.item() == pytest.approx(want, abs=1e-6)
    case = expected["adam_vs_adamw_decay"]
    for cls, want in ((tx.optim.Adam, case["adam"]), (tx.optim.AdamW, case["adamw"])):
        m = _load(tx, fixtures, "_GEMM_MODEL")
        p = dict(m.named_parameters())["weight"]
        p.grad = tx.Tensor([[1.0]])
        cls([p], lr=0.1, betas=(0.0, 0.0), eps=0.0, weight_decay=0.5).step()
        assert p.item() == pytest.approx(want, abs=1e-6)
    case = expected["amsgrad"]
    m = _load(tx, fixtures, "_GEMM_MODEL")
    p = dict(m.named_parameters())["weight"]
    opt = tx.optim.Adam([p], lr=0.1, betas=(0.0, 0.0), eps=0.0, amsgrad=True)
    for g in case["grads"]:
        p.grad = tx.Tensor([[g]])
        opt.step()
    assert p.item() == pytest.approx(case["final"], abs=1e-6)


def test_softmax_gelu_mse_goldens(tx, expected):
    case = expected["softmax_axis0"]
    y = tx.Tensor(case["input"]).softmax(case["axis"])
    assert np.allclose(y.numpy(), case["output"], atol=case["abs"])
    case = expected["log_softmax_stable"]
    y = tx.Tensor(case["input"]).log_softmax(0)
    assert np.allclose(y.numpy(), case["output"], atol=case["abs"])
    case = expected["gelu_exact_erf"]
    assert np.allclose(tx.Tensor(case["input"]).gelu().numpy(), case["output"], atol=case["abs"])
    case = expected["mse"]
    loss = tx.nn.functional.mse_loss(tx.Tensor(case["prediction"]), tx.Tensor(case["target"]))
    assert loss.item() == pytest.approx(case["loss"], abs=1e-6)


def _ppo_setup(tx, fixtures):
    names = {"policy_weight": "policy.weight", "policy_bias": "policy.bias",
             "value_weight": "value.weight", "value_bias": "value.bias"}
    return _load(tx, fixtures, "_ACTOR_CRITIC_MODEL", initializer_names=names)


def test_ppo_trains_with_user_composed_loss(tx, fixtures, expected):
    case = expected["ppo_training"]
    model = _ppo_setup(tx, fixtures)
    ln, vn = model.outputs
    obs = tx.Tensor(case["observations"])
    actions = tx.Tensor(case["actions"], dtype="int64")
    returns = tx.Tensor(case["returns"])
    adv = tx.Tensor(case["advantages"])
    old = tx.distributions.Categorical(logits=model(obs)[ln]).log_prob(actions).detach()
    assert old.tolist() == pytest.approx([-math.log(2.0)] * 4)

    def ppo_loss():
        out = model(obs)
        policy = tx.distributions.Categorical(logits=out[ln])
        ratio = (policy.log_prob(actions) - old).exp()
        policy_loss = -tx.minimum(ratio * adv, ratio.clamp(0.8, 1.2) * adv).mean()
        value_loss = tx.nn.functional.mse_loss(out[vn].squeeze(1), returns)
        return policy_loss + value_loss * 0.5 - policy.entropy().mean() * 0.01, value_loss

    l0, v0 = ppo_loss()
    l0, v0 = l0.item(), v0.item()
    opt = tx.optim.Adam(model.named_parameters(), lr=case["lr"])
    for _ in range(case["steps"]):
        opt.zero_grad()
        loss, _ = ppo_loss()
        loss.backward()
        opt.step()
    l1, v1 = ppo_loss()
    assert l1.item() < l0
    assert v1.item() < v0 * case["final_value_loss_ratio_below"]
    probs = tx.distributions.Categorical(logits=model(obs)[ln]).probs
    chosen = probs.gather(1, actions.unsqueeze(1)).mean().item()
    assert chosen > case["chosen_probability_above"]


def test_captured_ppo_step_matches_eager(tx, fixtures):
    """Capture == eager within 1e-6 over 40 steps (test_ppo.py:95-194)."""
    eager, captured = _ppo_setup(tx, fixtures), _ppo_setup(tx, fixtures)
    eager_opt = tx.optim.Adam(eager.named_parameters(), lr=0.03)
    captured_opt = tx.optim.Adam(captured.named_parameters(), lr=0.03)
    ln, vn = eager.outputs
    calls = 0

    def update(model, opt, obs, actions, returns, adv, old):
        opt.zero_grad()
        out = model(obs)
        policy = tx.distributions.Categorical(logits=out[ln])
        ratio = (policy.log_prob(actions) - old).exp()
        policy_loss = -tx.minimum(ratio * adv, ratio.clamp(0.8, 1.2) * adv).mean()
        value_loss = tx.nn.functional.mse_loss(out[vn].squeeze(1), returns)
        loss = policy_loss + value_loss * 0.5 - policy.entropy().mean() * 0.01
        loss.backward()
        opt.step()
        return loss

    @tx.compile(fullgraph=True)
    def captured_update(obs, actions, returns, adv, old):
        nonlocal calls
        calls += 1
        return update(captured, captured_opt, obs, actions, returns, adv, old)

    obs = tx.Tensor([[1.0, 0.0], [0.0, 1.0], [1.0, 1.0], [-1.0, 1.0]])
    actions = tx.Tensor([0, 1, 0, 1], dtype="int64")
    returns = tx.Tensor([1.0, -1.0, 0.0, -2.0])
    adv = tx.Tensor([1.0, 1.0, 1.0, 1.0])
    old = tx.Tensor([-math.log(2.0)] * 4)
    for _ in range(40):
        le = update(eager, eager_opt, obs, actions, returns, adv, old)
        lc = captured_update(obs, actions, returns, adv, old)
        assert lc.item() == pytest.approx(le.item(), abs=1e-6)
    e, c = dict(eager.named_parameters()), dict(captured.named_parameters())
    for name in e:
        assert c[name].flatten().tolist() == pytest.approx(e[name].flatten().tolist(), abs=1e-6)
    assert calls == 1
    assert captured_update.compile_count == 1
    assert captured_update.replay_count == 39


@pytest.mark.parametrize("name", ["_CNN_MODEL", "_RECOMMENDER_MODEL", "_TRANSFORMER_MODEL"])
def test_composed_models_converge(tx, fixtures, expected, name):
    spec = expected["composed_training"]
    case = spec["cases"][name]
    model = tx.load(fixtures[name], trainable="auto", simplify=False)
    report = model.require_trainable()
    assert report.warnings == []
    assert sorted(report.trainable_parameters) == case["trainable"]
    x = tx.Tensor(case["input"], dtype=case.get("input_dtype", "float32"))
    target = tx.Tensor(case["target"])
    opt = tx.optim.Adam(model.named_parameters(), lr=spec["lr"])
    initial = tx.nn.functional.mse_loss(model(x), target).item()
    for _ in range(spec["steps"]):
        opt.zero_grad()
        loss = tx.nn.functional.mse_loss(model(x), target)
        loss.backward()
        opt.step()
    final = tx.nn.functional.mse_loss(model(x), target).item()
    assert final < initial * spec["final_ratio_below"]
    assert all(p.grad is not None for _, p in model.named_parameters())


def test_gemm_learns_line(tx, gemm_line_model, expected):
    """100 SGD steps on the mean squared error fit y = 2x + 1 through the
    imported Gemm on the GPU; the first forward reads the zero initializers,
    the next forward the updated slots; the final slots agree with the oracle
    run of the same steps."""
    from oracle import flex_oracle as fo
    from tynx_b200.onnx import ir

    case = expected["gemm_learns_line"]
    names = {"weight": "head.weight", "bias": "head.bias"}
    model = tx.load(gemm_line_model, trainable="auto", simplify=False, initializer_names=names)
    x, target = tx.Tensor(case["input"]), tx.Tensor(case["target"])
    assert model(x).flatten().tolist() == case["output_before"]
    opt = tx.optim.SGD(model.named_parameters(), lr=case["lr"])
    ref = fo.OracleModel(ir.load_training_graph(gemm_line_model, initializer_names=names))
    ref_opt = fo.SGD(ref.named_parameters(), lr=case["lr"])
    xs, ts = np.asarray(case["input"], np.float32), np.asarray(case["target"], np.float32)
    for _ in range(case["steps"]):
        opt.zero_grad()
        tx.nn.functional.mse_loss(model(x), target).backward()
        opt.step()
        ref_opt.zero_grad()
        fo.mse_loss(ref(xs), ts).backward()
        ref_opt.step()
    p = {n: float(v.numpy().reshape(-1)[0]) for n, v in model.named_parameters()}
    r = {n: float(v.data.reshape(-1)[0]) for n, v in ref.named_parameters()}
    tol = case["tolerance"]
    assert abs(p["head.weight"] - case["weight"]) < tol
    assert abs(p["head.bias"] - case["bias"]) < tol
    for n in r:
        assert abs(p[n] - r[n]) <= 1e-5 * max(1.0, abs(r[n])), (n, p[n], r[n])
    np.testing.assert_allclose(model(x).numpy(), ts, atol=tol)


def _one_node_model(op, x_shape, y_shape, inits, **attrs):
    from tynx_b200.onnx import proto

    names = [n for n, _ in inits]
    return proto.encode_model(
        [proto.encode_node(op, ["x", *names], ["y"], name="layer", **attrs)],
        [proto.encode_tensor(n, np.asarray(v, np.float32)) for n, v in inits],
        [proto.encode_value_info("x", proto.FLOAT, list(x_shape))],
        [proto.encode_value_info("y", proto.FLOAT, list(y_shape))], opset=17)


def _central_difference(f, x0, i, e):
    up, down = x0.copy(), x0.copy()
    up.reshape(-1)[i] += np.float32(e)
    down.reshape(-1)[i] -= np.float32(e)
    return (f(up) - f(down)) / (2 * e)


def test_reference_finite_difference_points(tx, expected):
    """The reference's central-difference checks on its inputs, through
    one-node imported graphs on the GPU: the Conv input gradient at element 0
    and the LayerNormalization input gradient of sum(y * coefficients) at
    element 1."""
    c = expected["conv2d_finite_difference"]
    x0 = np.asarray(c["input"], np.float32)
    w = np.asarray(c["weight"], np.float32)
    conv = tx.load(_one_node_model("Conv", x0.shape, (1, 1, 1, 1), [("w", w)]), trainable="auto",
                   simplify=False)
    x = tx.Tensor(x0, requires_grad=True)
    conv(x).sum().backward()
    numerical = _central_difference(lambda v: conv(tx.Tensor(v)).sum().item(), x0, c["element"], c["epsilon"])
    assert x.grad.flatten().tolist()[c["element"]] == pytest.approx(numerical, rel=c["rel"], abs=c["abs"])

    c = expected["layer_norm_finite_difference"]
    x0 = np.asarray(c["input"], np.float32)
    coef = tx.Tensor(c["coefficients"])
    ln = tx.load(_one_node_model("LayerNormalization", x0.shape, x0.shape,
                                 [("scale", np.ones(3)), ("shift", np.zeros(3))], axis=-1,
                                 epsilon=c["eps"]), trainable="auto", simplify=False)
    x = tx.Tensor(x0, requires_grad=True)
    (ln(x) * coef).sum().backward()
    numerical = _central_difference(lambda v: (ln(tx.Tensor(v)) * coef).sum().item(), x0, c["element"],
                                    c["epsilon"])
    assert x.grad.flatten().tolist()[c["element"]] == pytest.approx(numerical, rel=c["rel"], abs=c["abs"])


_HEAD = {"weight": "head.weight", "bias": "head.bias"}


def test_model_report_output_selection_and_strict_state_dict(tx, fixtures):
    """The model's structured, output-specific trainability report and its
    strict state_dict (test_imported_model.py:369-419)."""
    model = _load(tx, fixtures, "_GEMM_MODEL", initializer_names=_HEAD)
    report = model.trainability_report()
    out = model.outputs[0]
    assert isinstance(report, tx.TrainabilityReport)
    assert report.is_trainable is True
    assert report.selected_outputs == [out]
    assert sorted(report.trainable_parameters) == ["head.bias", "head.weight"]
    assert sorted(report.output_parameters[out]) == ["head.bias", "head.weight"]
    assert report.backward_issues == []
    assert {entry["role"] for entry in report.initializers} >= {"parameter"}
    assert "Trainable parameters" in str(report)
    report.require_trainable()
    assert model.require_trainable(outputs=[out]).selected_outputs == [out]
    with pytest.raises(ValueError, match=r"requested output.*not a declared"):
        model.require_trainable(outputs=["missing"])
    state = model.state_dict()
    assert sorted(state) == ["head.bias", "head.weight"]
    with pytest.raises(ValueError, match="state_dict key mismatch"):
        model.load_state_dict({"head.weight": state["head.weight"]})


def test_simplified_model_keeps_declared_output_names(tx, fixtures):
    """test_imported_model.py:422-438."""
    model = tx.load(fixtures["_GEMM_MODEL"], trainable="auto", simplify=True, initializer_names=_HEAD)
    assert model.outputs == ["y"]
    report = model.trainability_report()
    assert report.selected_outputs == ["y"] and "y" in report.output_parameters
    selected = model.require_trainable(outputs=["y"])
    assert selected.selected_outputs == ["y"] and "y" in selected.output_parameters


@pytest.mark.parametrize("simplify", [False, True])
def test_matmul_initializer_keeps_its_onnx_name(tx, fixtures, simplify):
    """test_imported_model.py:441-453."""
    model = tx.load(fixtures["_MATMUL_MODEL"], trainable="auto", simplify=simplify)
    assert [name for name, _ in model.named_parameters()] == ["encoder.weight"]
    report = model.trainability_report()
    assert report.trainable_parameters == ["encoder.weight"]
    assert report.initializers[0]["synthetic_name"] is False
    assert model(tx.Tensor([[3.0], [4.0]])).flatten().tolist() == [6.0, 8.0]


def test_no_grad_call_is_detached_and_plain_load_is_inference(tx, fixtures):
    """test_imported_model.py:378-398."""
    model = tx.load(fixtures["_GEMM_MODEL"], trainable=True, simplify=False, initializer_names=_HEAD)
    with tx.no_grad():
        output = model(tx.Tensor([[2.0], [-1.0]], requires_grad=True))
    assert output.requires_grad is False
    session = tx.load(fixtures["_GEMM_MODEL"], simplify=False)
    assert isinstance(session, tx.Session)
    x = tx.Tensor([[2.0], [-1.0]], requires_grad=True)
    positional, named = session(x), session.run(x=x)
    assert isinstance(positional, tx.Tensor) and isinstance(named, tx.Tensor)
    assert positional.flatten().tolist() == pytest.approx([5.0, -1.0])
    assert named.flatten().tolist() == pytest.approx([5.0, -1.0])


def test_model_binds_named_inputs_and_returns_named_outputs(tx, fixtures):
    """Two inputs, two outputs (test_imported_model.py:456-487): positional and
    named binding, a dict of outputs in declaration order, input gradients,
    and the binding errors."""
    model = _load(tx, fixtures, "_MULTI_MODEL")
    first = tx.Tensor([[1.0], [2.0]], requires_grad=True)
    second = tx.Tensor([[3.0], [4.0]], requires_grad=True)
    positional = model(first, second)
    assert isinstance(positional, dict) and list(positional) == model.outputs
    assert positional[model.outputs[0]].flatten().tolist() == pytest.approx([4.0, 6.0])
    assert positional[model.outputs[1]].flatten().tolist() == pytest.approx([3.0, 8.0])
    named = model(**{model.inputs[1]: second, model.inputs[0]: first})
    (named[model.outputs[0]].sum() + named[model.outputs[1]].sum()).backward()
    assert first.grad.flatten().tolist() == pytest.approx([4.0, 5.0])
    assert second.grad.flatten().tolist() == pytest.approx([2.0, 3.0])
    with pytest.raises(TypeError, match="missing required inputs"):
        model(first)
    with pytest.raises(TypeError, match="unexpected input"):
        model(first, unknown=second)
    with pytest.raises(TypeError, match="multiple values"):
        model(first, **{model.inputs[0]: second, model.inputs[1]: second})


def test_conv_weights_and_bias_train_in_place(tx, fixtures):
    """800 SGD steps fit the imported convolution to its target
    (test_imported_model.py:182-199)."""
    model = _load(tx, fixtures, "_CONV_MODEL")
    opt = tx.optim.SGD(model.named_parameters(), lr=0.05)
    x = tx.Tensor([[[[1.0, 2.0], [3.0, 4.0]]]])
    target = tx.Tensor([[[[3.0, 5.0], [7.0, 9.0]]]])
    for _ in range(800):
        opt.zero_grad()
        tx.nn.functional.mse_loss(model(x), target).backward()
        opt.step()
    assert model(x).flatten().tolist() == pytest.approx(target.flatten().tolist(), abs=1e-3)
    params = dict(model.named_parameters())
    assert params["weight"].grad is not None and params["bias"].grad is not None

