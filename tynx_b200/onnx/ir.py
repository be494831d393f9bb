"""Load path: ONNX model -> normalized training graph + trainability report.

This is the host-side restatement of what the reference does between reading
the bytes and handing the graph to its executor:

* ``Session::from_bytes_with`` (``crates/tynx/src/session.rs:74-140``) parses
  with onnx-ir and keeps the declared names;
* ``analyze`` / ``role_proposal`` (``crates/tynx-train/src/trainability.rs:511-956``)
  give every initializer a role (parameter, buffer, constant) from the
  operator input that consumes it;
* ``analyze_backward_paths`` (``trainability.rs:684-826``) records which
  parameters each output depends on and which nodes on those paths have no
  backward rule;
* ``materialize_with_names`` (``crates/tynx-train/src/imported_state.rs:89-117``)
  turns parameter initializers into slots under their stable names.

The result, :class:`TrainingGraph`, is consumed by the CUDA engine (lowered to
the C node list in ``tynx_b200/engine.py``) and by the CPU oracle.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Optional

import numpy as np

from . import proto

PARAMETER = "parameter"
BUFFER = "buffer"
CONSTANT = "constant"
AMBIGUOUS = "ambiguous"

# Operators whose backward rule the engine implements (the training registry of
# crates/tynx-train/src/backward_support.rs:40-219 restricted to this build).
DIFFERENTIABLE = {
    "Gemm", "MatMul", "Conv", "Gather", "LayerNormalization", "Add", "Sub", "Mul", "Div",
    "Relu", "Tanh", "Gelu", "Sigmoid", "Exp", "Log", "Neg", "Softmax", "LogSoftmax",
    "ReduceMean", "ReduceSum", "GlobalAveragePool", "Reshape", "Transpose", "Flatten",
    "Squeeze", "Unsqueeze", "Identity", "Clip", "PRelu", "BatchNormalization",
    "InstanceNormalization", "GroupNormalization", "MaxPool",
    # smooth unary operations, extrema, layout and pooling (backward_support.rs:70-100)
    "Sqrt", "Abs", "Reciprocal", "Erf", "LeakyRelu", "Softplus", "Elu", "HardSigmoid", "Softsign",
    "Pow", "Max", "Min", "Concat", "Slice", "Split", "Expand", "AveragePool", "ReduceMax",
    "ReduceMin", "GlobalMaxPool", "Dropout",
}
# Operators that carry no gradient to their inputs but are allowed on a path.
NON_DIFFERENTIABLE_OK = {"Constant", "Shape"}


class LoadError(ValueError):
    """The model cannot be prepared for training."""


@dataclass
class RoleProposal:
    role: str
    reason: str
    recognized: bool


def role_proposal(op_type: str, input_index: int) -> RoleProposal:
    """Role an operator input proposes for an initializer it consumes.

    Follows ``role_proposal`` in ``crates/tynx-train/src/trainability.rs:889-956``.
    """
    parameter = RoleProposal(PARAMETER, "trainable weight, bias, or affine term", True)
    buffer = RoleProposal(BUFFER, "persistent normalization statistic", True)
    constant = RoleProposal(CONSTANT, "semantic metadata or fixed operator input", True)
    if op_type in ("Gemm", "Linear") and input_index in (1, 2):
        return parameter
    if op_type == "MatMul" and input_index in (0, 1):
        return parameter
    if op_type in ("Conv", "ConvTranspose") and input_index in (1, 2):
        return parameter
    if op_type == "BatchNormalization" and input_index in (1, 2):
        return parameter
    if op_type == "BatchNormalization" and input_index in (3, 4):
        return buffer
    if op_type in ("InstanceNormalization", "LayerNormalization", "GroupNormalization") and \
            input_index in (1, 2):
        return parameter
    if op_type == "PRelu" and input_index == 1:
        return parameter
    if op_type in ("Gather", "GatherElements", "GatherND") and input_index == 0:
        return parameter
    if op_type in ("Reshape", "Expand", "Tile", "Squeeze", "Unsqueeze") and input_index == 1:
        return constant
    if op_type in ("Gather", "GatherElements", "GatherND") and input_index == 1:
        return constant
    if op_type in ("Slice", "Resize", "Pad") and input_index >= 1:
        return constant
    if op_type in ("Clip", "OneHot") and input_index in (1, 2):
        return constant
    if op_type in ("TopK", "CumSum", "Trilu") and input_index == 1:
        return constant
    if op_type in ("Range", "ConstantOfShape"):
        return constant
    return RoleProposal(
        CONSTANT, "no trainable initializer role is registered for this consumer input", False
    )


@dataclass
class InitializerUse:
    node_name: str
    operator: str
    input_index: int
    proposed_role: str
    reason: str


@dataclass
class InitializerReport:
    """One initializer's entry in the report; read by attribute or, as the
    reference's Python report entries are, by key (``entry["role"]``).
    ``synthetic_name`` is True for a name the importer generated; names here
    are always the ONNX initializer's own or the caller's override."""

    name: str
    role: str
    dtype: str
    shape: tuple
    uses: list[InitializerUse] = field(default_factory=list)
    synthetic_name: bool = False

    def as_dict(self) -> dict:
        return {
            "name": self.name,
            "role": self.role,
            "dtype": self.dtype,
            "shape": list(self.shape),
            "uses": [u.__dict__ for u in self.uses],
            "synthetic_name": self.synthetic_name,
        }

    def __getitem__(self, key: str):
        return self.as_dict()[key]


@dataclass
class TrainabilityReport:
    """Structured trainability analysis (``trainability.rs:216-447``)."""

    initializers: list[InitializerReport] = field(default_factory=list)
    selected_outputs: list[str] = field(default_factory=list)
    output_parameters: dict[str, list[str]] = field(default_factory=dict)
    backward_issues: list[str] = field(default_factory=list)
    unused_parameters: list[str] = field(default_factory=list)
    warnings: list[str] = field(default_factory=list)
    errors: list[str] = field(default_factory=list)

    @property
    def trainable_parameters(self) -> list[str]:
        return [i.name for i in self.initializers if i.role == PARAMETER]

    @property
    def buffers(self) -> list[str]:
        return [i.name for i in self.initializers if i.role == BUFFER]

    @property
    def is_trainable(self) -> bool:
        return not self.errors and not self.backward_issues and bool(self.trainable_parameters)

    def require_trainable(self) -> "TrainabilityReport":
        if self.errors:
            raise ValueError("model is not trainable: " + "; ".join(self.errors))
        if self.backward_issues:
            raise ValueError("model is not trainable: " + "; ".join(self.backward_issues))
        if not self.trainable_parameters:
            raise ValueError("model is not trainable: no trainable parameters were found")
        return self

    def __str__(self) -> str:
        lines = [f"Trainable parameters ({len(self.trainable_parameters)}):"]
        for entry in self.initializers:
            if entry.role == PARAMETER:
                lines.append(f"  {entry.name} {list(entry.shape)} {entry.dtype}")
        if self.buffers:
            lines.append(f"Buffers ({len(self.buffers)}): " + ", ".join(self.buffers))
        for warning in self.warnings:
            lines.append(f"warning: {warning}")
        for error in self.errors:
            lines.append(f"error: {error}")
        for issue in self.backward_issues:
            lines.append(f"backward issue: {issue}")
        return "\n".join(lines)


@dataclass
class Op:
    """One normalized graph node."""

    op_type: str
    name: str
    inputs: list[str]  # "" for an absent optional input
    outputs: list[str]
    attrs: dict


@dataclass
class TrainingGraph:
    """Normalized graph plus initializer roles, ready for an executor."""

    ops: list[Op]
    inputs: list[proto.ValueInfo]
    outputs: list[str]
    parameters: dict[str, np.ndarray]  # stable name -> initial value (float32)
    parameter_of_value: dict[str, str]  # ONNX value name -> stable parameter name
    buffers: dict[str, np.ndarray]
    constants: dict[str, np.ndarray]  # ONNX value name -> constant array
    report: TrainabilityReport
    opset: int
    buffer_of_value: dict = field(default_factory=dict)  # ONNX value name -> stable buffer name


def _dtype_name(array: np.ndarray) -> str:
    return {np.float32: "float32", np.int64: "int64", np.bool_: "bool"}.get(
        array.dtype.type, str(array.dtype)
    )


def _normalize_attrs(node: proto.Node, opset: int) -> dict:
    """Resolve the ONNX defaults each supported operator relies on."""
    a = {name: attribute.value for name, attribute in node.attributes.items()}
    t = node.op_type
    if t == "Gemm":
        a.setdefault("alpha", 1.0)
        a.setdefault("beta", 1.0)
        a.setdefault("transA", 0)
        a.setdefault("transB", 0)
    elif t in ("Softmax", "LogSoftmax"):
        a.setdefault("axis", -1 if opset >= 13 else 1)
    elif t == "LayerNormalization":
        a.setdefault("axis", -1)
        a.setdefault("epsilon", 1e-5)
    elif t == "Gather":
        a.setdefault("axis", 0)
    elif t == "Flatten":
        a.setdefault("axis", 1)
    elif t in ("ReduceMean", "ReduceSum"):
        a.setdefault("keepdims", 1)
    elif t == "Conv":
        a.setdefault("group", 1)
        auto_pad = a.get("auto_pad", "NOTSET")
        if auto_pad not in ("NOTSET", ""):
            raise LoadError(f"Conv node {node.name!r}: auto_pad={auto_pad} is not supported")
    elif t == "Gelu":
        a.setdefault("approximate", "none")
    elif t == "BatchNormalization":
        # An absent epsilon adds nothing: the reference's imported BatchNorm
        # test (crates/tynx-train/src/imported_model/tests.rs:447-480) asserts
        # y == [2.5, 5.0, 4.5, 8.0] exactly for var [4, 9] with no epsilon
        # attribute, which holds in f32 only if var + eps == var.
        a.setdefault("epsilon", 0.0)
        if int(a.get("training_mode", 0)) or len(node.outputs) != 1:
            raise LoadError(f"BatchNormalization node {node.name!r}: training outputs are not "
                            "supported (the running statistics are fixed buffers)")
    elif t == "InstanceNormalization":
        a.setdefault("epsilon", 1e-5)
    elif t == "GroupNormalization":
        a.setdefault("epsilon", 1e-5)
        if "num_groups" not in a:
            raise LoadError(f"GroupNormalization node {node.name!r} has no num_groups attribute")
    elif t in ("ReduceMax", "ReduceMin"):
        a.setdefault("keepdims", 1)
    elif t == "LeakyRelu":
        a.setdefault("alpha", 0.01)
    elif t == "Elu":
        a.setdefault("alpha", 1.0)
    elif t == "HardSigmoid":
        a.setdefault("alpha", 0.2)
        a.setdefault("beta", 0.5)
    elif t in ("Concat", "Split"):
        a.setdefault("axis", 0)
        if t == "Concat" and "axis" not in node.attributes:
            raise LoadError(f"Concat node {node.name!r} has no axis attribute")
    elif t == "Dropout":
        # inference semantics: the identity; a mask output or a training flag
        # would need the random mask (backward_support.rs: Dropout is
        # differentiable only when inference-only)
        if len(node.outputs) > 1:
            raise LoadError(f"Dropout node {node.name!r}: the mask output is not supported")
    elif t == "AveragePool":
        if "kernel_shape" not in a:
            raise LoadError(f"AveragePool node {node.name!r} has no kernel_shape attribute")
        nd = len(a["kernel_shape"])
        a.setdefault("strides", [1] * nd)
        a.setdefault("dilations", [1] * nd)
        a.setdefault("pads", [0] * (2 * nd))
        a.setdefault("ceil_mode", 0)
        a.setdefault("auto_pad", "NOTSET")
        a.setdefault("count_include_pad", 0)
    elif t == "MaxPool":
        if "kernel_shape" not in a:
            raise LoadError(f"MaxPool node {node.name!r} has no kernel_shape attribute")
        nd = len(a["kernel_shape"])
        a.setdefault("strides", [1] * nd)
        a.setdefault("dilations", [1] * nd)
        a.setdefault("pads", [0] * (2 * nd))
        a.setdefault("ceil_mode", 0)
        a.setdefault("auto_pad", "NOTSET")
        if len(node.outputs) > 1:
            raise LoadError(f"MaxPool node {node.name!r}: the indices output is not supported "
                            "for training")
    return a


def build_training_graph(
    model: proto.Model,
    *,
    initializer_names: Optional[dict[str, str]] = None,
    outputs: Optional[list[str]] = None,
) -> TrainingGraph:
    """Normalize ``model`` and classify its initializers.

    ``initializer_names`` maps ONNX initializer names to stable public names
    (``imported_state.rs:89-117``); ``outputs`` selects a subset of the
    declared outputs (``imported_model.rs:48-71``).
    """
    graph = model.graph
    opset = model.opset.get("", model.opset.get("ai.onnx", 13))
    rename = dict(initializer_names or {})
    initializers = {t.name: t.array for t in graph.initializers}
    declared_outputs = [o.name for o in graph.outputs]
    if outputs is None:
        selected = declared_outputs
    else:
        for name in outputs:
            if name not in declared_outputs:
                raise ValueError(f"requested output {name!r} is not a declared model output")
        selected = list(outputs)

    ops: list[Op] = []
    constants: dict[str, np.ndarray] = {}
    constant_outputs: set[str] = set()
    for index, node in enumerate(graph.nodes):
        name = node.name or f"{node.op_type}_{index}"
        if node.op_type == "Constant":
            value = node.attr("value")
            if isinstance(value, proto.Tensor):
                array = value.array
            elif "value_float" in node.attributes:
                array = np.asarray(node.attr("value_float"), dtype=np.float32)
            elif "value_int" in node.attributes:
                array = np.asarray(node.attr("value_int"), dtype=np.int64)
            elif "value_floats" in node.attributes:
                array = np.asarray(node.attr("value_floats"), dtype=np.float32)
            elif "value_ints" in node.attributes:
                array = np.asarray(node.attr("value_ints"), dtype=np.int64)
            else:
                raise LoadError(f"Constant node {name!r} has no supported value attribute")
            constants[node.outputs[0]] = array
            constant_outputs.add(node.outputs[0])
            continue
        ops.append(Op(node.op_type, name, list(node.inputs), list(node.outputs),
                      _normalize_attrs(node, opset)))

    # --- initializer roles (trainability.rs:511-682) --------------------------------
    report = TrainabilityReport(selected_outputs=list(selected))
    uses: dict[str, list[tuple[InitializerUse, bool]]] = {}
    order: list[str] = []
    for op in ops:
        for input_index, value in enumerate(op.inputs):
            if value not in initializers:
                continue
            proposal = role_proposal(op.op_type, input_index)
            if value not in uses:
                uses[value] = []
                order.append(value)
            uses[value].append(
                (InitializerUse(op.name, op.op_type, input_index, proposal.role, proposal.reason),
                 proposal.recognized)
            )
    roles: dict[str, str] = {}
    for value in order:
        entry_roles = {u.proposed_role for u, _ in uses[value]}
        role = entry_roles.pop() if len(entry_roles) == 1 else AMBIGUOUS
        public = rename.get(value, value)
        if role == AMBIGUOUS:
            joined = ", ".join(
                f"{u.operator}:{u.node_name} input {u.input_index} -> {u.proposed_role}"
                for u, _ in uses[value]
            )
            report.warnings.append(
                f"initializer '{public}' has conflicting consumer roles ({joined}); "
                "add an explicit override"
            )
        for usage, recognized in uses[value]:
            if not recognized:
                report.warnings.append(
                    f"initializer '{public}' remains constant because {usage.operator} input "
                    f"{usage.input_index} has no registered trainable role"
                )
        array = initializers[value]
        if role == PARAMETER and array.dtype != np.float32:
            report.errors.append(
                f"initializer '{public}' is a trainable parameter with dtype {array.dtype}; "
                "training requires float32"
            )
        roles[value] = role
        report.initializers.append(
            InitializerReport(public, role, _dtype_name(array), tuple(array.shape),
                              [u for u, _ in uses[value]])
        )
    for key in rename:
        if key not in initializers:
            report.warnings.append(
                f"initializer override '{key}' did not match any processed graph initializer"
            )

    parameters: dict[str, np.ndarray] = {}
    parameter_of_value: dict[str, str] = {}
    buffers: dict[str, np.ndarray] = {}
    buffer_of_value: dict[str, str] = {}
    for value in order:
        array = initializers[value]
        public = rename.get(value, value)
        if roles[value] == PARAMETER:
            parameters[public] = np.array(array, dtype=np.float32, copy=True)
            parameter_of_value[value] = public
        elif roles[value] == BUFFER:
            buffers[public] = np.array(array, copy=True)
            constants[value] = buffers[public]
            buffer_of_value[value] = public
        else:
            constants[value] = np.array(array, copy=True)
    for value, array in initializers.items():
        if value not in uses:
            constants.setdefault(value, np.array(array, copy=True))

    # --- backward paths (trainability.rs:684-826) ----------------------------------
    producer = {out: op for op in ops for out in op.outputs}

    def upstream_parameters(values) -> list[str]:
        # every parameter that feeds these values, through any operator
        found, seen, stack = set(), set(), [v for v in values if v]
        while stack:
            value = stack.pop()
            if value in seen:
                continue
            seen.add(value)
            if value in parameter_of_value:
                found.add(parameter_of_value[value])
            elif value in producer:
                stack.extend(i for i in producer[value].inputs if i)
        return sorted(found)

    blocked: set[str] = set()
    for out in selected:
        reached: list[str] = []
        seen: set[str] = set()
        stack = [out]
        while stack:
            value = stack.pop()
            if value in seen:
                continue
            seen.add(value)
            if value in parameter_of_value:
                reached.append(parameter_of_value[value])
                continue
            op = producer.get(value)
            if op is None:
                continue
            if op.op_type not in DIFFERENTIABLE:
                touches = any(i in parameter_of_value or i in producer for i in op.inputs if i)
                if touches:
                    # the issue names the parameters it cuts off from the output
                    behind = upstream_parameters(op.inputs)
                    report.backward_issues.append(
                        f"{op.op_type} node '{op.name}' on the path to output '{out}' has no "
                        "backward rule" + (f" (blocks {', '.join(behind)})" if behind else "")
                    )
                    blocked.update(behind)
                continue
            stack.extend(i for i in op.inputs if i)
        report.output_parameters[out] = sorted(set(reached))
    used = {p for names in report.output_parameters.values() for p in names}
    report.unused_parameters = sorted(set(parameters) - used - blocked)

    return TrainingGraph(
        ops=ops,
        inputs=[i for i in graph.inputs if i.name not in initializers],
        outputs=selected,
        parameters=parameters,
        parameter_of_value=parameter_of_value,
        buffers=buffers,
        buffer_of_value=buffer_of_value,
        constants=constants,
        report=report,
        opset=opset,
    )


def load_training_graph(data: bytes, **kwargs) -> TrainingGraph:
    return build_training_graph(proto.decode_model(data), **kwargs)
