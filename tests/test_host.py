"""Host-side checks that need no GPU: the C ABI library, the header, lowering."""

import ctypes as C
import re
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent


def test_library_exports_every_declared_symbol():
    header = (ROOT / "include" / "tynx_cuda.h").read_text()
    declared = set(re.findall(r"^int (tx_\w+)\(", header, re.M))
    from tynx_b200 import _native

    lib = _native.lib
    missing = [name for name in declared if not hasattr(lib, name)]
    assert not missing, missing
    assert declared == set(_native.SIGNATURES), declared ^ set(_native.SIGNATURES)
    assert lib.tx_abi_version() == 2


def test_no_gpu_calls_fail_cleanly_without_a_device():
    from tynx_b200 import _native

    if _native.device_count() > 0:
        pytest.skip("a GPU is present")
    handle = C.c_void_p()
    assert _native.lib.tx_ctx_create(0, 0, C.byref(handle)) != 0
    assert not handle.value


def test_cpu_devices_are_rejected():
    from tynx_b200 import Device

    with pytest.raises(ValueError, match="CUDA only"):
        Device("cpu")
    assert str(Device("cuda:3")) == "cuda:3"


def test_workload_graphs_lower_and_match_parameter_counts():
    from tynx_b200 import workloads
    from tynx_b200.imported import lower
    from tynx_b200.onnx import ir

    expected = {"mlp_policy": 84488, "mlp_classifier": 1863690, "ppo": 337425, "cnn": 94538,
                "transformer": 5280258}
    for name, make in workloads.WORKLOADS.items():
        kw = {"minibatch": 64, "rollout": 256} if name == "ppo" else {}
        wl = make(**kw)
        graph = ir.load_training_graph(wl.onnx)
        assert graph.report.warnings == [] and graph.report.errors == []
        assert graph.report.backward_issues == []
        assert sum(p.size for p in graph.parameters.values()) == expected[name]
        values, nodes, outputs, *_ = lower(graph)
        assert len(outputs) == len(graph.outputs)
        assert all(n.op > 0 for n in nodes)


def test_reference_fixtures_lower(fixtures):
    from tynx_b200.imported import lower
    from tynx_b200.onnx import ir

    for name in ["_GEMM_MODEL", "_GATHER_MODEL", "_LAYER_NORM_MODEL", "_BATCHED_MATMUL_MODEL",
                 "_CLIPPED_GEMM_MODEL", "_CNN_MODEL", "_RECOMMENDER_MODEL", "_TRANSFORMER_MODEL",
                 "_ACTOR_CRITIC_MODEL", "_CONV_MODEL", "_MATMUL_MODEL"]:
        lower(ir.load_training_graph(fixtures[name]))


def test_onnx_codec_round_trip():
    from tynx_b200.onnx import proto

    w = np.arange(6, dtype=np.float32).reshape(2, 3)
    data = proto.encode_model(
        [proto.encode_node("Gemm", ["x", "w"], ["y"], name="g", transB=1, alpha=0.5)],
        [proto.encode_tensor("w", w)],
        [proto.encode_value_info("x", proto.FLOAT, ["batch", 3])],
        [proto.encode_value_info("y", proto.FLOAT, ["batch", 2])])
    model = proto.decode_model(data)
    node = model.graph.nodes[0]
    assert node.op_type == "Gemm" and node.attr("transB") == 1
    assert node.attr("alpha") == pytest.approx(0.5)
    np.testing.assert_array_equal(model.graph.initializers[0].array, w)
    assert model.graph.inputs[0].shape == ["batch", 3]


def test_trainability_roles_follow_consumers(fixtures):
    from tynx_b200.onnx import ir

    graph = ir.load_training_graph(fixtures["_GEMM_MODEL"],
                                   initializer_names={"weight": "head.weight", "bias": "head.bias"})
    assert sorted(graph.report.trainable_parameters) == ["head.bias", "head.weight"]
    assert graph.report.output_parameters["y"] == ["head.bias", "head.weight"]
    with pytest.raises(ValueError, match="not a declared"):
        ir.load_training_graph(fixtures["_GEMM_MODEL"], outputs=["missing"])
    # an initializer consumed by Add has no trainable role and stays constant with a warning
    from tynx_b200.onnx import proto

    data = proto.encode_model(
        [proto.encode_node("Add", ["x", "b"], ["y"], name="add")],
        [proto.encode_tensor("b", np.zeros(2, np.float32))],
        [proto.encode_value_info("x", proto.FLOAT, [2])],
        [proto.encode_value_info("y", proto.FLOAT, [2])])
    g = ir.load_training_graph(data)
    assert g.report.trainable_parameters == []
    assert any("no registered trainable role" in w for w in g.report.warnings)


def test_trainability_roles_by_operand():
    """Which initializers train, operand by operand, as the reference's
    trainability tests state it (trainability.rs:1243-1259, 1385-1432): a
    Gather trains its data table but not its indices; a Clip's bound
    initializers stay constant; a Linear weight in float16 is reported as an
    error, since training requires float32."""
    from tynx_b200.onnx import ir, proto

    def model(nodes, inits, inputs, outputs):
        return proto.encode_model(nodes, inits, inputs, outputs)

    g = ir.load_training_graph(model(
        [proto.encode_node("Gather", ["data", "idx"], ["y"], name="gather", axis=0)],
        [proto.encode_tensor("data", np.zeros((4, 2), np.float32)),
         proto.encode_tensor("idx", np.zeros(1, np.int64))],
        [], [proto.encode_value_info("y", proto.FLOAT, [1, 2])]))
    assert g.report.trainable_parameters == ["data"]

    g = ir.load_training_graph(model(
        [proto.encode_node("Clip", ["x", "lo", "hi"], ["y"], name="relu6")],
        [proto.encode_tensor("lo", np.zeros(1, np.float32)),
         proto.encode_tensor("hi", np.full(1, 6.0, np.float32))],
        [proto.encode_value_info("x", proto.FLOAT, [2, 2])],
        [proto.encode_value_info("y", proto.FLOAT, [2, 2])]))
    assert g.report.trainable_parameters == []

    g = ir.load_training_graph(model(
        [proto.encode_node("Gemm", ["x", "weight", "bias"], ["y"], name="linear")],
        [proto.encode_tensor("weight", np.zeros((2, 2), np.float16)),
         proto.encode_tensor("bias", np.zeros(2, np.float32))],
        [proto.encode_value_info("x", proto.FLOAT, [1, 2])],
        [proto.encode_value_info("y", proto.FLOAT, [1, 2])]))
    assert any("requires float32" in e for e in g.report.errors)


def test_selected_output_reports_influencing_blocked_and_unused_parameters():
    """Two branches from one input: policy = Relu(Gemm) trains, diagnostic =
    Ceil(Gemm) has no backward rule (trainability.rs:1434-1475).  Selecting
    policy leaves the diagnostic parameters unused; selecting diagnostic is
    not trainable, and the one issue names the Ceil node and the parameters it
    cuts off."""
    from tynx_b200.onnx import ir, proto

    z = lambda *shape: np.zeros(shape, np.float32)  # noqa: E731
    data = proto.encode_model(
        [proto.encode_node("Gemm", ["x", "policy.weight", "policy.bias"], ["policy_hidden"],
                           name="policy_linear"),
         proto.encode_node("Relu", ["policy_hidden"], ["policy"], name="policy_relu"),
         proto.encode_node("Gemm", ["x", "diagnostic.weight", "diagnostic.bias"], ["diagnostic_hidden"],
                           name="diagnostic_linear"),
         proto.encode_node("Ceil", ["diagnostic_hidden"], ["diagnostic"], name="diagnostic_round")],
        [proto.encode_tensor("policy.weight", z(2, 2)), proto.encode_tensor("policy.bias", z(2)),
         proto.encode_tensor("diagnostic.weight", z(2, 2)), proto.encode_tensor("diagnostic.bias", z(2))],
        [proto.encode_value_info("x", proto.FLOAT, [1, 2])],
        [proto.encode_value_info("policy", proto.FLOAT, [1, 2]),
         proto.encode_value_info("diagnostic", proto.FLOAT, [1, 2])])

    policy = ir.load_training_graph(data, outputs=["policy"]).report
    assert policy.is_trainable
    assert policy.output_parameters["policy"] == ["policy.bias", "policy.weight"]
    assert policy.backward_issues == []
    assert policy.unused_parameters == ["diagnostic.bias", "diagnostic.weight"]
    policy.require_trainable()

    diagnostic = ir.load_training_graph(data, outputs=["diagnostic"]).report
    assert not diagnostic.is_trainable
    assert len(diagnostic.backward_issues) == 1
    issue = diagnostic.backward_issues[0]
    assert "Ceil" in issue and "diagnostic_round" in issue
    assert "diagnostic.bias, diagnostic.weight" in issue
    with pytest.raises(ValueError, match="not trainable"):
        diagnostic.require_trainable()


def test_operator_without_backward_rule_is_reported_by_name():
    """A Det after a Gemm (trainability.rs:1477-1505): the model is not
    trainable and the printed report names the node, so the user can act."""
    from tynx_b200.onnx import ir, proto

    z = lambda *shape: np.zeros(shape, np.float32)  # noqa: E731
    data = proto.encode_model(
        [proto.encode_node("Gemm", ["x", "matrix.weight", "matrix.bias"], ["matrix_value"], name="matrix"),
         proto.encode_node("Det", ["matrix_value"], ["score"], name="determinant")],
        [proto.encode_tensor("matrix.weight", z(2, 2)), proto.encode_tensor("matrix.bias", z(2))],
        [proto.encode_value_info("x", proto.FLOAT, [1, 2])],
        [proto.encode_value_info("score", proto.FLOAT, [1])])
    report = ir.load_training_graph(data).report
    assert not report.is_trainable
    assert report.backward_issues and "Det" in report.backward_issues[0]
    assert "determinant" in str(report)


def test_trainability_report_entries_read_by_key(fixtures):
    """Report entries answer by key as the reference's Python report does
    (test_imported_model.py:401-454): roles, and synthetic_name False for an
    initializer that keeps its ONNX name."""
    import tynx_b200 as tx
    from tynx_b200.onnx import ir

    report = ir.load_training_graph(fixtures["_MATMUL_MODEL"]).report
    assert isinstance(report, tx.TrainabilityReport)
    assert report.trainable_parameters == ["encoder.weight"]
    assert report.initializers[0]["synthetic_name"] is False
    assert report.initializers[0]["role"] == report.initializers[0].role == "parameter"
    assert "Trainable parameters" in str(report)



def test_checkpoint_arguments_and_payload_validation(tmp_path):
    """Host-side checkpoint rules: both argument orders, and the payload checks
    of ``crates/tynx-python/python/tynx/checkpoint.py:314-331``."""
    import json

    from tynx_b200 import checkpoint as ck

    class Opt:
        def state_dict(self):
            return {}

        def load_state_dict(self, state):
            pass

    model, opt = object(), Opt()
    assert ck._split_args("a.json", model, opt, "save")[1:] == (model, opt)
    assert ck._split_args(model, opt, "a.json", "load")[1:] == (model, opt)
    assert ck._split_args(model, "a.json", None, "save")[1:] == (model, None)
    with pytest.raises(TypeError, match="expects"):
        ck._split_args(model, opt, None, "save")
    with pytest.raises(TypeError, match="must provide state_dict"):
        ck._split_args("a.json", model, object(), "save")
    with pytest.raises(ValueError, match="requires its optimizer"):
        ck._check_scheduler(None, object())
    path = tmp_path / "x.json"
    path.write_text("{not json")
    with pytest.raises(ValueError, match="invalid Tynx checkpoint JSON"):
        ck._read(path)
    path.write_text(json.dumps({"format": "other", "version": 1}))
    with pytest.raises(ValueError, match="not a Tynx training checkpoint"):
        ck._read(path)
    path.write_text(json.dumps({"format": "tynx.training", "version": 7}))
    with pytest.raises(ValueError, match="unsupported Tynx checkpoint version 7"):
        ck._read(path)
    assert ck._encode({"b": (1, 2.5), "a": [None, True]}) == \
        {"b": {"__type__": "tuple", "items": [1, 2.5]}, "a": [None, True]}
    with pytest.raises(TypeError, match="string keys"):
        ck._encode({1: 2})
    with pytest.raises(ValueError, match="unknown checkpoint value type"):
        ck._decode({"__type__": "set"})
    with pytest.raises(ValueError, match="does not match declared shape"):
        ck._decode({"__type__": "tensor", "dtype": "float32", "shape": [2], "data": [1.0]})


def test_rust_sys_crate_declares_every_header_function():
    """crates/tynx-cuda-sys/src/lib.rs (the FFI crate a Tynx integration
    compiles) declares every function of include/tynx_cuda.h with the same
    number of parameters, and its node descriptor matches the header's."""
    header = (ROOT / "include" / "tynx_cuda.h").read_text()
    header = re.sub(r"/\*.*?\*/", "", header, flags=re.S)
    rust = (ROOT / "crates" / "tynx-cuda-sys" / "src" / "lib.rs").read_text()
    c_funcs = {n: a for n, a in re.findall(r"^int (tx_\w+)\((.*?)\);", header, flags=re.S | re.M)}
    r_funcs = dict(re.findall(r"pub fn (tx_\w+)\((.*?)\) -> c_int;", rust))
    assert set(c_funcs) == set(r_funcs), set(c_funcs) ^ set(r_funcs)

    def count(args):
        args = " ".join(args.split())
        return 0 if args in ("", "void") else args.count(",") + 1

    for name, args in c_funcs.items():
        assert count(args) == count(r_funcs[name]), name
    assert "pub inp: [i32; 6]" in rust and "int32_t in[6], out[3];" in header
    assert re.search(r"TYNX_CUDA_ABI_VERSION: c_int = (\d+)", rust).group(1) == \
        re.search(r"#define TYNX_CUDA_ABI_VERSION (\d+)", header).group(1)
