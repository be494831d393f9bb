"""Regenerate ``tests/golden/*.json`` from the reference's own test fixtures.

Run in a container where the reference checkout is mounted (its path is the
first argument, default ``/root/reference``)::

    python tests/golden/make_golden.py /root/reference

Two files are written next to this script:

* ``onnx_fixtures.json`` -- the hex-encoded ONNX models the reference's Python
  tests and examples embed (``crates/tynx-python/tests/test_imported_model.py``,
  ``test_imported_composed_models.py``, ``test_ppo.py``,
  ``examples/models/*.onnx.hex``), extracted verbatim as data.
* ``expected.json`` -- the known answers those tests assert, transcribed below
  with the file:line of each assertion.  These pin the oracle and the CUDA path.

The GPU box never reads the reference: tests load only the committed JSON.
"""

from __future__ import annotations

import json
import re
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent

_HEX_BLOCK = re.compile(r"(_[A-Z0-9_]+_MODEL) = bytes\.fromhex\(\n((?:\s+\"[0-9a-f]+\"\n)+)\)")

SOURCES = {
    "test_imported_model": "crates/tynx-python/tests/test_imported_model.py",
    "test_imported_composed_models": "crates/tynx-python/tests/test_imported_composed_models.py",
    "test_ppo": "crates/tynx-python/tests/test_ppo.py",
}

# Known answers asserted by the reference's tests (file:line of the assertion).
EXPECTED = {
    "gemm_forward_backward": {
        "source": "crates/tynx-python/tests/test_imported_model.py:153-170",
        "model": "_GEMM_MODEL",
        "input": [[2.0], [-1.0]],
        "output": [5.0, -1.0],
        "input_grad": [2.0, 2.0],
        "weight_grad": [1.0],
        "bias_grad": [2.0],
    },
    "gemm_sgd_next_forward": {
        "source": "crates/tynx-python/tests/test_imported_model.py:173-181",
        "model": "_GEMM_MODEL",
        "input": [[2.0], [-1.0]],
        "lr": 0.1,
        "next_output": [4.6, -1.1],
    },
    "clip_gemm": {
        "source": "crates/tynx-python/tests/test_imported_model.py:205-217",
        "model": "_CLIPPED_GEMM_MODEL",
        "input": [[-1.0], [2.0]],
        "output": [0.0, 2.0],
        "weight_grad": [2.0],
        "bias_grad": [1.0],
    },
    "gather_accumulation": {
        "source": "crates/tynx-python/tests/test_imported_model.py:220-237",
        "model": "_GATHER_MODEL",
        "indices": [0, 2, 0],
        "output": [[1.0, 2.0], [5.0, 6.0], [1.0, 2.0]],
        "weight_grad": [[2.0, 2.0], [0.0, 0.0], [1.0, 1.0]],
        "lr": 0.1,
        "next_output": [0.8, 1.8, 4.9, 5.9, 0.8, 1.8],
    },
    "layer_norm": {
        "source": "crates/tynx-python/tests/test_imported_model.py:240-268",
        "model": "_LAYER_NORM_MODEL",
        "input": [[1.0, 3.0], [2.0, 6.0]],
        "output": [-0.999995, 0.999995, -0.999999, 0.999999],
        "weight_grad": [-1.999994, 1.999994],
        "bias_grad": [2.0, 2.0],
        "lr": 0.1,
        "next_output": [-1.399994, 0.599996, -1.399998, 0.599999],
        "abs": 1e-5,
    },
    "batched_matmul": {
        "source": "crates/tynx-python/tests/test_imported_model.py:271-292",
        "model": "_BATCHED_MATMUL_MODEL",
        "input": [[[1.0, 2.0, 3.0], [4.0, 5.0, 6.0]], [[7.0, 8.0, 9.0], [10.0, 11.0, 12.0]]],
        "output": [4.0, 5.0, 10.0, 11.0, 16.0, 17.0, 22.0, 23.0],
        "weight_grad": [22.0, 22.0, 26.0, 26.0, 30.0, 30.0],
    },
    "adam_constant_gradient": {
        "source": "crates/tynx-train/src/optimizer/adam.rs:800-814",
        "weight": 2.0,
        "grad": 2.0,
        "lr": 0.1,
        "trajectory": [1.9, 1.8],
    },
    "adam_vs_adamw_decay": {
        "source": "crates/tynx-train/src/optimizer/adam.rs:932-957",
        "weight": 2.0,
        "grad": 1.0,
        "lr": 0.1,
        "betas": [0.0, 0.0],
        "eps": 0.0,
        "weight_decay": 0.5,
        "adam": 1.9,
        "adamw": 1.8,
    },
    "amsgrad": {
        "source": "crates/tynx-train/src/optimizer/adam.rs:961-978",
        "weight": 2.0,
        "grads": [2.0, 0.5],
        "lr": 0.1,
        "betas": [0.0, 0.0],
        "eps": 0.0,
        "final": 1.875,
    },
    "softmax_axis0": {
        "source": "crates/tynx/src/interpreter/softmax.rs:33-64",
        "input": [[0.0, 0.0], [1.0, 2.0]],
        "axis": 0,
        "output": [[0.26894143, 0.11920292], [0.7310586, 0.880797]],
        "abs": 1e-5,
    },
    "log_softmax_stable": {
        "source": "crates/tynx/src/interpreter/softmax.rs:66-94",
        "input": [10000.0, 10001.0],
        "output": [-1.3132616, -0.31326166],
        "abs": 1e-4,
    },
    "gelu_exact_erf": {
        "source": "crates/tynx/src/interpreter/unary.rs:1314-1339",
        "input": [-1.0, 0.0, 1.0],
        "output": [-0.15865526, 0.0, 0.8413447],
        "abs": 1e-6,
    },
    "mse": {
        "source": "crates/tynx-train/src/loss.rs:37-48",
        "prediction": [[1.0, 2.0], [3.0, 4.0]],
        "target": [[1.0, 4.0], [2.0, 3.0]],
        "loss": 1.5,
    },
    "ppo_initial_log_prob": {
        "source": "crates/tynx-python/tests/test_ppo.py:47-50",
        "model": "_ACTOR_CRITIC_MODEL",
        "observations": [[1.0, 0.0], [0.0, 1.0], [1.0, 1.0], [-1.0, 1.0]],
        "actions": [0, 1, 0, 1],
        "old_log_prob": -0.6931471805599453,
    },
    "ppo_training": {
        "source": "crates/tynx-python/tests/test_ppo.py:23-93",
        "model": "_ACTOR_CRITIC_MODEL",
        "observations": [[1.0, 0.0], [0.0, 1.0], [1.0, 1.0], [-1.0, 1.0]],
        "actions": [0, 1, 0, 1],
        "returns": [1.0, -1.0, 0.0, -2.0],
        "advantages": [1.0, 1.0, 1.0, 1.0],
        "lr": 0.03,
        "steps": 120,
        "final_value_loss_ratio_below": 0.01,
        "chosen_probability_above": 0.55,
    },
    "composed_training": {
        "source": "crates/tynx-python/tests/test_imported_composed_models.py:78-148",
        "lr": 0.03,
        "steps": 80,
        "final_ratio_below": 1e-3,
        "cases": {
            "_CNN_MODEL": {
                "input": [[[[1.0, 2.0], [3.0, 4.0]]]],
                "target": [[1.5]],
                "trainable": ["conv.bias", "conv.weight", "head.bias", "head.weight"],
            },
            "_RECOMMENDER_MODEL": {
                "input": [0, 1, 0],
                "input_dtype": "int64",
                "target": [[1.0], [-1.0], [1.0]],
                "trainable": ["embedding.weight", "head.bias", "head.weight"],
            },
            "_TRANSFORMER_MODEL": {
                "input": [[0, 1]],
                "input_dtype": "int64",
                "target": [[2.0]],
                "trainable": [
                    "classifier.bias",
                    "classifier.weight",
                    "norm.bias",
                    "norm.weight",
                    "projection.weight",
                    "token_embedding.weight",
                ],
            },
        },
    },
    # One scalar parameter (2.0) with a set gradient; "after" values are
    # asserted exactly in f32 by the reference, the momentum trajectory to 1e-6.
    "sgd_goldens": {
        "source": "crates/tynx-train/src/optimizer.rs:487-535",
        "weight": 2.0,
        "plain": {"grad": 3.0, "lr": 0.1, "after": 1.7},
        "weight_decay": {"grad": 3.0, "lr": 0.1, "weight_decay": 0.5, "after": 1.6},
        "momentum": {"grad": 2.0, "lr": 0.1, "momentum": 0.9, "dampening": 0.5, "trajectory": [1.8, 1.52]},
    },
    # A one-node Gemm (x [4, 1], weight [1, 1] and bias [1] initializers, both
    # zero; opset 13, no transpose attributes) built in the test code, not a
    # hex fixture: the tests build the same model with the package's encoder.
    "gemm_learns_line": {
        "source": "crates/tynx-train/src/imported_model/tests.rs:62-140 (model: :647-657, :844-863)",
        "input": [[-1.0], [0.0], [1.0], [2.0]],
        "target": [[-1.0], [1.0], [3.0], [5.0]],
        "lr": 0.1,
        "steps": 100,
        "output_before": [0.0, 0.0, 0.0, 0.0],
        "weight": 2.0,
        "bias": 1.0,
        "tolerance": 1e-3,
    },
    # Central differences of one input element (the graphs are one Conv / one
    # LayerNormalization node; the reference builds them with its eager API).
    "conv2d_finite_difference": {
        "source": "crates/tynx-python/tests/test_training_robustness.py:17-36",
        "input": [[[[0.2, -0.4], [0.7, 1.1]]]],
        "weight": [[[[0.5, -0.25], [0.75, 0.1]]]],
        "element": 0,
        "epsilon": 1e-3,
        "rel": 2e-3,
        "abs": 2e-3,
    },
    "layer_norm_finite_difference": {
        "source": "crates/tynx-python/tests/test_training_robustness.py:39-59",
        "input": [[0.5, -1.0, 2.0]],
        "coefficients": [0.25, -0.5, 1.5],
        "eps": 1e-5,
        "element": 1,
        "epsilon": 1e-3,
        "rel": 3e-3,
        "abs": 3e-3,
    },
}


def extract(reference: Path) -> dict[str, str]:
    fixtures: dict[str, str] = {}
    for relative in SOURCES.values():
        text = (reference / relative).read_text()
        for match in _HEX_BLOCK.finditer(text):
            fixtures[match.group(1)] = "".join(re.findall(r"\"([0-9a-f]+)\"", match.group(2)))
    for path in sorted((reference / "examples" / "models").glob("*.onnx.hex")):
        fixtures["examples/" + path.name] = path.read_text().strip()
    return fixtures


def main() -> None:
    reference = Path(sys.argv[1] if len(sys.argv) > 1 else "/root/reference")
    fixtures = extract(reference)
    (HERE / "onnx_fixtures.json").write_text(json.dumps(fixtures, indent=1, sort_keys=True) + "\n")
    (HERE / "expected.json").write_text(json.dumps(EXPECTED, indent=1) + "\n")
    print(f"wrote {len(fixtures)} ONNX fixtures and {len(EXPECTED)} expected cases")


if __name__ == "__main__":
    main()
