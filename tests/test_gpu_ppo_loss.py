"""The fused PPO objective (``tx.nn.functional.ppo_loss``, C ABI
``tx_ppo_loss_fwd`` / ``tx_ppo_loss_bwd``) against the same objective composed
from Categorical, minimum, clamp and mse_loss (the reference's
``crates/tynx-python/tests/test_ppo.py:53-64``) and against the oracle:
equal loss and equal gradients for the logits and the value head on an
8192-row minibatch, index errors for bad actions, and a captured training
step that issues fewer kernels and follows the composed one's trajectory."""

import numpy as np
import pytest

from oracle import flex_oracle as fo

pytestmark = pytest.mark.gpu


def _batch(rows=8192, cols=16, seed=0):
    rng = np.random.default_rng(seed)
    return {"logits": (rng.standard_normal((rows, cols)) * 2).astype(np.float32),
            "values": rng.standard_normal((rows, 1)).astype(np.float32),
            "actions": rng.integers(0, cols, rows).astype(np.int64),
            "old": (rng.standard_normal(rows) * 0.5 - 2.8).astype(np.float32),
            "adv": rng.standard_normal(rows).astype(np.float32),
            "ret": rng.standard_normal(rows).astype(np.float32)}


def _composed(tx, logits, values, actions, old, adv, ret):
    policy = tx.distributions.Categorical(logits=logits)
    ratio = (policy.log_prob(actions) - old).exp()
    policy_loss = -tx.minimum(ratio * adv, ratio.clamp(0.8, 1.2) * adv).mean()
    value_loss = tx.nn.functional.mse_loss(values.squeeze(1), ret)
    return policy_loss + value_loss * 0.5 - policy.entropy().mean() * 0.01


def _rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.mark.parametrize("cols", [16, 7, 40])
def test_fused_matches_composed_and_oracle(cols):
    import tynx_b200 as tx

    b = _batch(cols=cols)
    grads = []
    for fused in (True, False):
        z = tx.Tensor(b["logits"], requires_grad=True)
        v = tx.Tensor(b["values"], requires_grad=True)
        args = (tx.Tensor(b["actions"], dtype="int64"), tx.Tensor(b["old"]), tx.Tensor(b["adv"]),
                tx.Tensor(b["ret"]))
        if fused:
            loss = tx.nn.functional.ppo_loss(z, v, *args)
        else:
            loss = _composed(tx, z, v, *args)
        loss.backward()
        grads.append((loss.item(), z.grad.numpy(), v.grad.numpy()))
    (lf, zf, vf), (lc, zc, vc) = grads
    zo = fo.T(b["logits"], requires_grad=True)
    vo = fo.T(b["values"], requires_grad=True)
    lo = fo.ppo_loss(zo, vo, b["actions"], b["old"], b["adv"], b["ret"])
    lo.backward()
    assert abs(lf - lo.item()) <= 1e-6 * max(1.0, abs(lo.item()))
    assert abs(lf - lc) <= 1e-6 * max(1.0, abs(lc))
    assert _rel(zf, zo.grad) < 1e-5 and _rel(zf, zc) < 1e-5
    assert _rel(vf, vo.grad) < 1e-6 and _rel(vf, vc) < 1e-6


def test_bad_action_raises_index_error():
    import tynx_b200 as tx

    b = _batch(rows=64)
    b["actions"][5] = 16
    with pytest.raises(IndexError):
        loss = tx.nn.functional.ppo_loss(tx.Tensor(b["logits"]), tx.Tensor(b["values"]),
                                         tx.Tensor(b["actions"], dtype="int64"), tx.Tensor(b["old"]),
                                         tx.Tensor(b["adv"]), tx.Tensor(b["ret"]))
        loss.item()
    tx.synchronize()  # the context stays usable


def test_captured_step_with_fused_loss_follows_composed_trajectory():
    """Eight captured PPO minibatch updates of the actor-critic (minibatch
    1024): the fused objective's losses equal the composed objective's within
    rel 1e-5 at every step, with fewer kernels per replayed step."""
    import tynx_b200 as tx
    from tynx_b200 import workloads
    from tynx_b200.distributions import Categorical

    wl = workloads.ppo(minibatch=1024, rollout=8192)
    runs = []
    for fused in (True, False):
        model = tx.load(wl.onnx, trainable="auto")
        opt = tx.optim.Adam(model.named_parameters(), lr=wl.lr)

        @tx.compile(fullgraph=True)
        def step(obs, actions, old, adv, ret):
            opt.zero_grad()
            out = model(obs)
            if fused:
                loss = tx.nn.functional.ppo_loss(out["logits"], out["value"], actions, old, adv, ret)
            else:
                policy = Categorical(logits=out["logits"])
                ratio = (policy.log_prob(actions) - old).exp()
                policy_loss = -tx.minimum(ratio * adv, ratio.clamp(0.8, 1.2) * adv).mean()
                value_loss = tx.nn.functional.mse_loss(out["value"].squeeze(1), ret)
                loss = policy_loss + value_loss * 0.5 - policy.entropy().mean() * 0.01
            loss.backward()
            opt.step()
            return loss

        losses = []
        for i in range(8):
            b = wl.make_batch(i)
            old = np.full(wl.batch, -2.77, np.float32)
            losses.append(step(tx.Tensor(b["obs"]), tx.Tensor(b["actions"], dtype="int64"), tx.Tensor(old),
                               tx.Tensor(b["advantages"]), tx.Tensor(b["returns"])).item())
        entry = step.entry_for(tx.Tensor(b["obs"]), tx.Tensor(b["actions"], dtype="int64"), tx.Tensor(old),
                               tx.Tensor(b["advantages"]), tx.Tensor(b["returns"]))
        runs.append((losses, entry.kernel_count))
    (lf, kf), (lc, kc) = runs
    assert kf < kc, (kf, kc)
    for a, c in zip(lf, lc):
        assert abs(a - c) <= 1e-5 * max(1.0, abs(c)), (lf, lc)
