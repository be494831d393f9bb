"""Checkpoints on Device("cuda"): the ``tynx.training`` v1 JSON format, the
name-keyed Adam / SGD state dictionaries, and resumption that continues
bit-identically (``crates/tynx-python/python/tynx/checkpoint.py``,
``crates/tynx-python/src/optimizer/state.rs``, ``adam.rs:339-384``)."""

import json

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _policy(tx):
    from tynx_b200 import workloads

    wl = workloads.mlp_policy()
    model = tx.load(wl.onnx, trainable="auto")
    return wl, model


def _train(tx, wl, model, opt, steps, start=0):
    losses = []
    for i in range(start, start + steps):
        b = wl.make_batch(i)
        opt.zero_grad()
        loss = tx.nn.functional.cross_entropy(model(tx.Tensor(b["x"])), tx.Tensor(b["y"]))
        loss.backward()
        opt.step()
        losses.append(loss.item())
    return losses


@pytest.mark.parametrize("kind", ["Adam", "AdamW", "SGD"])
def test_resume_continues_bit_identically(tmp_path, kind):
    import tynx_b200 as tx

    make = {"Adam": lambda p: tx.optim.Adam(p, lr=3e-4, amsgrad=True),
            "AdamW": lambda p: tx.optim.AdamW(p, lr=3e-4),
            "SGD": lambda p: tx.optim.SGD(p, lr=1e-2, momentum=0.9, dampening=0.1)}[kind]
    wl, model = _policy(tx)
    opt = make(model.named_parameters())
    _train(tx, wl, model, opt, 5)
    path = tmp_path / "ckpt.json"
    tx.save_checkpoint(path, model, opt)
    straight = _train(tx, wl, model, opt, 5, start=5)
    final = {n: p.numpy() for n, p in model.named_parameters()}

    wl2, fresh = _policy(tx)
    opt2 = make(fresh.named_parameters())
    result = tx.load_checkpoint(fresh, opt2, path)  # PyTorch-shaped argument order
    assert result.missing_keys == () and result.unexpected_keys == ()
    resumed = _train(tx, wl2, fresh, opt2, 5, start=5)
    assert resumed == straight
    for n, p in fresh.named_parameters():
        np.testing.assert_array_equal(p.numpy(), final[n], err_msg=n)


def test_file_format_and_adam_state_layout(tmp_path):
    import tynx_b200 as tx

    wl, model = _policy(tx)
    opt = tx.optim.Adam(model.named_parameters(), lr=3e-4)
    _train(tx, wl, model, opt, 2)
    path = tmp_path / "c.json"
    tx.save_checkpoint(model, opt, path)
    payload = json.loads(path.read_text())
    assert payload["format"] == "tynx.training" and payload["version"] == 1
    assert payload["scheduler"] is None
    w = payload["model"]["fc0.weight"]
    assert w["__type__"] == "tensor" and w["dtype"] == "float32" and w["shape"] == [256, 64]
    np.testing.assert_array_equal(np.asarray(w["data"], np.float32),
                                  dict(model.named_parameters())["fc0.weight"].numpy())
    state = payload["optimizer"]
    assert state["optimizer"] == "Adam" and state["version"] == 1
    assert state["parameter_names"] == sorted(n for n, _ in model.named_parameters())
    assert state["config"]["betas"] == {"__type__": "tuple", "items": [0.9, 0.999]}
    entry = state["state"]["fc2.bias"]
    assert entry["step"] == 2 and set(entry) == {"step", "exp_avg", "exp_avg_sq"}
    # no temporary file is left beside the target
    assert [p.name for p in tmp_path.iterdir()] == ["c.json"]


def test_state_dict_validation(tmp_path):
    import tynx_b200 as tx

    wl, model = _policy(tx)
    opt = tx.optim.Adam(model.named_parameters(), lr=3e-4)
    _train(tx, wl, model, opt, 1)
    state = opt.state_dict()
    with pytest.raises(ValueError, match="cannot load Adam state into AdamW optimizer"):
        tx.optim.AdamW(model.named_parameters()).load_state_dict(state)
    bad = dict(state, parameter_names=state["parameter_names"][1:])
    with pytest.raises(ValueError, match="parameter names do not match"):
        opt.load_state_dict(bad)
    with pytest.raises(ValueError, match="requires construction from model.named_parameters"):
        tx.optim.Adam(model.parameters()).state_dict()
    with pytest.raises(ValueError, match="unsupported optimizer state_dict version"):
        opt.load_state_dict(dict(state, version=2))
    # a failed load leaves the optimizer as it was
    assert opt.state_dict()["state"]["fc0.weight"]["step"] == 1

    path = tmp_path / "m.json"
    tx.save_checkpoint(path, model)
    from tynx_b200 import workloads

    other = tx.load(workloads.cnn(batch=2).onnx, trainable="auto")
    with pytest.raises(ValueError, match="state_dict key mismatch"):
        tx.load_checkpoint(path, other)
    result = tx.load_checkpoint(path, model, strict=True)
    assert result.missing_keys == ()
    with pytest.raises(ValueError, match="checkpoint does not contain optimizer state"):
        tx.load_checkpoint(path, model, opt)
