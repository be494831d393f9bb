"""Write tests/golden/trajectories.json: the oracle's loss trajectory of every
configured workload at its full size.

Each workload trains from its seeded initial parameters on its seeded batch
stream (``tynx_b200.workloads``) with Adam for the configured number of steps
(MLP policy and classifier 100, PPO one rollout of 8 minibatches x 4 epochs,
CNN and transformer 50), in float32 like the Flex CPU backend.  The GPU
trajectory tests compare their per-step losses with these values at rel 1e-3;
the fixture spares the GPU box the CPU time of the full-size oracle (the
transformer's step takes ~13 s of numpy on eight cores).

PPO: the behaviour log-probabilities are those of the initial policy over the
whole rollout, and each minibatch step minimises the clipped surrogate (eps
0.2) + 0.5 value MSE - 0.01 entropy.

    python tests/golden/make_trajectories.py [workload ...]
"""

from __future__ import annotations

import json
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from oracle import flex_oracle as fo  # noqa: E402
from tynx_b200 import workloads  # noqa: E402
from tynx_b200.onnx import ir  # noqa: E402

OUT = Path(__file__).resolve().parent / "trajectories.json"
STEPS = {"mlp_policy": 100, "mlp_classifier": 100, "ppo": 32, "cnn": 50, "transformer": 50}


def ppo_old_log_probs(model, wl) -> np.ndarray:
    """Log-probabilities of every rollout action under the initial policy."""
    obs = wl.notes["rollout_obs"]
    actions = np.empty(obs.shape[0], np.int64)
    for j in range(obs.shape[0] // wl.batch):
        b = wl.make_batch(j)
        actions[b["index"]] = b["actions"]
    logits = model(obs)["logits"].detach()
    return fo.Categorical(logits).log_prob(actions).data.astype(np.float32)


def trajectory(name: str) -> list[float]:
    wl = workloads.WORKLOADS[name]()
    model = fo.OracleModel(ir.load_training_graph(wl.onnx))
    opt = fo.Adam(model.named_parameters(), lr=wl.lr)
    old_all = ppo_old_log_probs(model, wl) if wl.loss == "ppo" else None
    losses = []
    for step in range(STEPS[name]):
        b = wl.make_batch(step)
        opt.zero_grad()
        if wl.loss == "ppo":
            out = model(b["obs"])
            loss = fo.ppo_loss(out["logits"], out["value"], b["actions"], old_all[b["index"]],
                               b["advantages"], b["returns"])
        else:
            key = "ids" if "ids" in b else "x"
            loss = fo.cross_entropy(model(b[key]), b["y"])
        loss.backward()
        opt.step()
        losses.append(float(loss.item()))
    return losses


def main(names) -> None:
    data = json.loads(OUT.read_text()) if OUT.exists() else {}
    for name in names:
        t0 = time.time()
        data[name] = {"steps": STEPS[name], "precision": "float32", "loss": trajectory(name)}
        print(f"{name}: {STEPS[name]} steps in {time.time() - t0:.0f} s", flush=True)
        OUT.write_text(json.dumps(data, indent=1) + "\n")


if __name__ == "__main__":
    main(sys.argv[1:] or list(STEPS))
