"""Training-step parity of the CUDA engine with the CPU oracle on every workload.

Per step, from identical parameters and seeded inputs: the loss, every
parameter gradient and every Adam-updated parameter are compared with the
oracle, with the error of a tensor measured as the relative L2 norm
||a - b|| / ||b||:
  * ``fp32`` math (SIMT FFMA contractions): 1e-5 (reduction order only)
  * ``tf32`` math (tcgen05 kind::tf32):      1e-3 (the stated TF32 tolerance)
The L2 norm is used because Adam's first step moves each weight by about
lr * sign(g): a gradient entry within rounding of zero can flip one element's
update, which a max-norm would report as a large error although every
gradient agrees to 1e-6.
Trajectories (each step's loss) must agree within the same relative bound.
"""

import numpy as np
import pytest

from oracle import flex_oracle as fo

pytestmark = pytest.mark.gpu

TOL = {"fp32": 1e-5, "tf32": 1e-3}
TRAJ_TOL = {"fp32": 1e-5, "tf32": 1e-3}


def _rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


CASES = [
    ("mlp_policy", {}),
    ("mlp_classifier", {}),
    ("ppo", {"minibatch": 1024, "rollout": 4096}),
    ("cnn", {"batch": 16}),
    ("transformer", {"batch": 4}),
]


def _engine_step(tx, model, opt, wl, batch, old_logp=None):
    ln = model.outputs[0]
    opt.zero_grad()
    if wl.loss == "ppo":
        obs = tx.Tensor(batch["obs"])
        out = model(obs)
        actions = tx.Tensor(batch["actions"], dtype="int64")
        policy = tx.distributions.Categorical(logits=out["logits"])
        ratio = (policy.log_prob(actions) - tx.Tensor(old_logp)).exp()
        adv = tx.Tensor(batch["advantages"])
        policy_loss = -tx.minimum(ratio * adv, ratio.clamp(0.8, 1.2) * adv).mean()
        value_loss = tx.nn.functional.mse_loss(out["value"].squeeze(1), tx.Tensor(batch["returns"]))
        loss = policy_loss + value_loss * 0.5 - policy.entropy().mean() * 0.01
    else:
        key = "ids" if "ids" in batch else "x"
        x = tx.Tensor(batch[key], dtype="int64" if key == "ids" else "float32")
        loss = tx.nn.functional.cross_entropy(model(x), tx.Tensor(batch["y"]))
    loss.backward()
    grads = {n: p.grad.numpy() for n, p in model.named_parameters()}
    opt.step()
    return loss.item(), grads


def _oracle_step(model, opt, wl, batch, old_logp=None):
    opt.zero_grad()
    if wl.loss == "ppo":
        out = model(batch["obs"])
        loss = fo.ppo_loss(out["logits"], out["value"], batch["actions"], old_logp,
                           batch["advantages"], batch["returns"])
    else:
        key = "ids" if "ids" in batch else "x"
        loss = fo.cross_entropy(model(batch[key]), batch["y"])
    loss.backward()
    grads = {n: p.grad.copy() for n, p in model.named_parameters()}
    opt.step()
    return loss.item(), grads


@pytest.mark.parametrize("math", ["fp32", "tf32"])
@pytest.mark.parametrize("name,kw", CASES, ids=[c[0] for c in CASES])
def test_step_parity(name, kw, math):
    import tynx_b200 as tx
    from tynx_b200 import workloads
    from tynx_b200.onnx import ir

    tx.set_math_mode(math)
    try:
        wl = workloads.WORKLOADS[name](**kw)
        model = tx.load(wl.onnx, trainable="auto")
        opt = tx.optim.Adam(model.named_parameters(), lr=wl.lr)
        ref = fo.OracleModel(ir.load_training_graph(wl.onnx))
        ref_opt = fo.Adam(ref.named_parameters(), lr=wl.lr)
        old = None
        if wl.loss == "ppo":
            b0 = wl.make_batch(0)
            old = fo.Categorical(ref(b0["obs"])["logits"].detach()).log_prob(b0["actions"]).data
        tol = TOL[math]
        steps = 3 if name in ("transformer", "cnn") else 10
        for step in range(steps):
            batch = wl.make_batch(step)
            if old is not None:
                batch_old = fo.Categorical(ref(batch["obs"])["logits"].detach()).log_prob(batch["actions"]).data
            else:
                batch_old = None
            loss, grads = _engine_step(tx, model, opt, wl, batch, batch_old)
            ref_loss, ref_grads = _oracle_step(ref, ref_opt, wl, batch, batch_old)
            assert abs(loss - ref_loss) <= TRAJ_TOL[math] * max(1.0, abs(ref_loss)), (step, loss, ref_loss)
            if step == 0:
                # identical starting state: gradients and updated parameters
                for n, g in ref_grads.items():
                    assert _rel(grads[n], g) < tol, (n, _rel(grads[n], g))
                for n, p in ref.named_parameters():
                    got = dict(model.named_parameters())[n].numpy()
                    assert _rel(got, p.data) < tol, (n, _rel(got, p.data))
    finally:
        tx.set_math_mode("tf32")
