"""Training-step parity of the CUDA engine with the CPU oracle on every workload.

From identical parameters and seeded inputs, one training step (forward, loss,
backward, Adam) is compared: the loss and every parameter gradient against
the oracle, and every updated parameter exactly against the oracle's Adam
applied to the GPU's gradients.  Gradients use the relative L2 error
||a - b|| / ||b||:

* against the oracle evaluated in float64 (the exact result of the same
  arithmetic), the GPU error must be at most
  ``max(TOL[math], 2 * error of the fp32 oracle)``.  The second term matters
  because fp32 rounding alone moves some gradients (a ReLU mask flips where a
  pre-activation is within rounding of zero): the fp32 CPU restatement of Flex
  is itself ~7e-5 away from float64 on the MLP classifier's first layers, so
  no fp32 implementation can be held to 1e-5 there;
* ``TOL``: 1e-3 for TF32 contractions (the stated TF32 tolerance), 1e-5 for the
  fp32-class modes (SIMT fp32 and 3xTF32).

* gradients behind hard activation masks are not continuous in the weights:
  in exact float64 arithmetic a 1e-6 relative perturbation of the weights
  already moves the CNN's first-layer weight gradient by ~3e-3 (a ReLU mask
  flips where a pre-activation is within rounding of zero, and global average
  pooling spreads that position's gradient over a whole channel).  The bound
  therefore also admits the float64 oracle's own sensitivity: the change of
  its gradients under a random relative weight perturbation of the size of the
  mode's rounding (1e-6 for the fp32-class modes, 2^-11 for TF32).  For the
  smooth networks (tanh, GELU) that sensitivity is ~1e-6 and the stated
  tolerance is what binds.

The per-step loss over a short trajectory must agree with the fp32 oracle
within rel 1e-3.
The L2 norm is used because Adam's first step moves each weight by about
lr * sign(g): a gradient entry within rounding of zero flips one element's
update, which a max-norm would report as a large error.
"""

import numpy as np
import pytest

from oracle import flex_oracle as fo

pytestmark = pytest.mark.gpu

TOL = {"fp32": 1e-5, "3xtf32": 1e-5, "tf32": 1e-3}
ROUNDING = {"fp32": 1e-6, "3xtf32": 1e-6, "tf32": 2.0 ** -11}


def _sensitivity(graph, wl, batch, old, eps):
    """Relative change of the float64 oracle's gradients and updated parameters
    under a random relative weight perturbation of size eps."""
    def run(noise):
        rng = np.random.default_rng(123)
        with fo.precision(np.float64):
            m, o = _oracle_pair(graph, wl.lr)
            for p in m.params.values():
                p.data = p.data * (1 + noise * rng.standard_normal(p.data.shape))
            _, g = _oracle_step(m, o, wl, batch, old)
            return g, {n: p.data.copy() for n, p in m.named_parameters()}

    g0, p0 = run(0.0)
    g1, p1 = run(eps)
    return ({n: _rel(g1[n], g0[n]) for n in g0}, {n: _rel(p1[n], p0[n]) for n in p0})


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
    opt.zero_grad()
    if wl.loss == "ppo":
        out = model(tx.Tensor(batch["obs"]))
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


def _oracle_pair(graph, lr):
    m32 = fo.OracleModel(graph)
    o32 = fo.Adam(m32.named_parameters(), lr=lr)
    return m32, o32


@pytest.mark.parametrize("math", ["fp32", "3xtf32", "tf32"])
@pytest.mark.parametrize("name,kw", CASES, ids=[c[0] for c in CASES])
def test_step_parity(name, kw, math):
    import tynx_b200 as tx
    from tynx_b200 import workloads
    from tynx_b200.onnx import ir

    tx.set_math_mode(math)
    try:
        wl = workloads.WORKLOADS[name](**kw)
        graph = ir.load_training_graph(wl.onnx)
        model = tx.load(wl.onnx, trainable="auto")
        opt = tx.optim.Adam(model.named_parameters(), lr=wl.lr)
        ref, ref_opt = _oracle_pair(graph, wl.lr)
        with fo.precision(np.float64):
            ref64, ref64_opt = _oracle_pair(graph, wl.lr)
        tol = TOL[math]
        steps = 3 if name in ("transformer", "cnn") else 8
        params = dict(model.named_parameters())
        for step in range(steps):
            batch = wl.make_batch(step)
            old = None
            if wl.loss == "ppo":  # behaviour policy: the current parameters
                old = fo.Categorical(ref(batch["obs"])["logits"].detach()).log_prob(
                    batch["actions"]).data
            start = {n: p.numpy() for n, p in params.items()}
            loss, grads = _engine_step(tx, model, opt, wl, batch, old)
            ref_loss, ref_grads = _oracle_step(ref, ref_opt, wl, batch, old)
            if step == 0:
                with fo.precision(np.float64):
                    loss64, grads64 = _oracle_step(ref64, ref64_opt, wl, batch, old)
                gap = abs(ref_loss - loss64)
                assert abs(loss - loss64) <= max(tol * max(1.0, abs(loss64)), 2 * gap), \
                    (loss, ref_loss, loss64)
                sens_g, _ = _sensitivity(graph, wl, batch, old, ROUNDING[math])
                for n, g64 in grads64.items():
                    err, err_ref = _rel(grads[n], g64), _rel(ref_grads[n], g64)
                    assert err <= max(tol, 2 * err_ref, 2 * sens_g[n]), (n, err, err_ref, sens_g[n])
                # The update itself is checked exactly: Adam applied by the oracle
                # to the GPU's own gradients from the same start.  (Comparing the
                # updated parameters with the float64 run instead is ill-posed:
                # Adam's first step moves each weight by lr * sign(g), so one
                # gradient entry within rounding of zero -- common for
                # zero-initialised biases -- flips a whole update.)
                upd = [fo.T(start[n].copy(), requires_grad=True) for n in start]
                for t, n in zip(upd, start):
                    t.grad = grads[n]
                fo.Adam(upd, lr=wl.lr).step()
                for t, n in zip(upd, start):
                    np.testing.assert_allclose(params[n].numpy(), t.data, rtol=2e-7, atol=1e-9,
                                               err_msg=n)
            else:
                # trajectory: each step's loss against the fp32 oracle, which has
                # taken the same steps from the same start (rel 1e-3)
                assert abs(loss - ref_loss) <= 1e-3 * max(1.0, abs(ref_loss)), \
                    (step, loss, ref_loss)
    finally:
        tx.set_math_mode("tf32")


@pytest.mark.parametrize("math", ["tf32", "3xtf32"])
def test_hundred_step_loss_trajectory(math):
    """MLP policy (64->256->256->8, batch 256, Adam 3e-4): the 100-step loss
    trajectory matches the oracle within rel 1e-3 at every step."""
    import tynx_b200 as tx
    from tynx_b200 import workloads
    from tynx_b200.onnx import ir

    tx.set_math_mode(math)
    try:
        wl = workloads.mlp_policy()
        model = tx.load(wl.onnx, trainable="auto")
        opt = tx.optim.Adam(model.named_parameters(), lr=wl.lr)
        ref, ref_opt = _oracle_pair(ir.load_training_graph(wl.onnx), wl.lr)

        @tx.compile(fullgraph=True)
        def step(x, y):
            opt.zero_grad()
            loss = tx.nn.functional.cross_entropy(model(x), y)
            loss.backward()
            opt.step()
            return loss

        worst = 0.0
        for i in range(100):
            batch = wl.make_batch(i)
            loss = step(tx.Tensor(batch["x"]), tx.Tensor(batch["y"])).item()
            ref_loss, _ = _oracle_step(ref, ref_opt, wl, batch)
            worst = max(worst, abs(loss - ref_loss) / max(1.0, abs(ref_loss)))
        assert worst <= 1e-3, worst
        assert step.compile_count == 1 and step.replay_count == 99
    finally:
        tx.set_math_mode("tf32")
