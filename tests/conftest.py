"""Shared pytest configuration.

Tests marked ``gpu`` run the CUDA path on a B200 and compare it with the CPU
oracle; everything else runs on the CPU-only host (oracle vs golden vectors,
host-side load logic, C-ABI symbol exports, multi-rank host logic over gloo).
"""

import json
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = Path(__file__).resolve().parent / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def fixtures() -> dict:
    return {k: bytes.fromhex(v) for k, v in json.loads((GOLDEN / "onnx_fixtures.json").read_text()).items()}


@pytest.fixture(scope="session")
def expected() -> dict:
    return json.loads((GOLDEN / "expected.json").read_text())


@pytest.fixture(scope="session")
def gemm_line_model() -> bytes:
    """The one-node Gemm of the reference's line-fitting test: y = x W + b with
    x [4, 1], W [1, 1] and b [1] initializers, both zero (opset 13)."""
    import numpy as np

    from tynx_b200.onnx import proto

    nodes = [proto.encode_node("Gemm", ["x", "weight", "bias"], ["y"], name="layer")]
    inits = [proto.encode_tensor("weight", np.zeros((1, 1), np.float32)),
             proto.encode_tensor("bias", np.zeros(1, np.float32))]
    return proto.encode_model(nodes, inits, [proto.encode_value_info("x", proto.FLOAT, [4, 1])],
                              [proto.encode_value_info("y", proto.FLOAT, [4, 1])],
                              graph_name="imported_training_test", opset=13)


def _one_node_model(op, inputs, inits, x_shape, y_shape, opset, graph_name, **attrs):
    import numpy as np  # noqa: F401

    from tynx_b200.onnx import proto

    nodes = [proto.encode_node(op, inputs, ["y"], name="norm" if "Norm" in op else
                               "activation" if op == "PRelu" else "node", **attrs)]
    encoded = [proto.encode_tensor(name, array) for name, array in inits]
    return proto.encode_model(nodes, encoded, [proto.encode_value_info("x", proto.FLOAT, x_shape)],
                              [proto.encode_value_info("y", proto.FLOAT, y_shape)],
                              graph_name=graph_name, opset=opset)


@pytest.fixture(scope="session")
def new_op_models() -> dict:
    """The one-node models of the reference's trainable-operator tests
    (crates/tynx-train/src/imported_model/tests.rs:671-700, 772-831): BatchNorm
    with fixed statistics, PRelu with a scalar slope, Instance- and
    GroupNormalization with unit scale and zero bias."""
    import numpy as np

    f = np.float32
    return {
        "batch_norm": (_one_node_model(
            "BatchNormalization", ["x", "scale", "bias", "mean", "variance"],
            [("scale", np.array([2, 3], f)), ("bias", np.array([0.5, -1], f)),
             ("mean", np.array([1, 2], f)), ("variance", np.array([4, 9], f))],
            [2, 2], [2, 2], 13, "imported_batch_norm_test"),
            {"scale": "norm.weight", "bias": "norm.bias", "mean": "norm.running_mean",
             "variance": "norm.running_var"}),
        "prelu": (_one_node_model("PRelu", ["x", "slope"], [("slope", np.array([0.25], f))],
                                  [2], [2], 13, "unsupported_slot_report"),
                  {"slope": "activation.weight"}),
        "instance_norm": (_one_node_model(
            "InstanceNormalization", ["x", "scale", "bias"],
            [("scale", np.ones(2, f)), ("bias", np.zeros(2, f))], [1, 2, 2], [1, 2, 2], 13,
            "imported_InstanceNormalization_test"),
            {"scale": "norm.weight", "bias": "norm.bias"}),
        "group_norm": (_one_node_model(
            "GroupNormalization", ["x", "scale", "bias"],
            [("scale", np.ones(4, f)), ("bias", np.zeros(4, f))], [1, 4, 2], [1, 4, 2], 18,
            "imported_GroupNormalization_test", num_groups=2),
            {"scale": "norm.weight", "bias": "norm.bias"}),
    }
