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
