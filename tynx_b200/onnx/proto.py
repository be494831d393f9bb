"""Minimal ONNX protobuf codec (wire format) for the training-path load.

The image has no ``onnx`` package, so ONNX ``ModelProto`` bytes are decoded and
encoded here directly from the protobuf wire format.  Only the messages and
fields the training path reads are modelled: ``ModelProto`` (ir_version,
producer, opset_import, graph), ``GraphProto`` (node, name, initializer, input,
output, value_info), ``NodeProto``, ``AttributeProto``, ``TensorProto`` and
``ValueInfoProto`` with tensor types and static/dynamic dims.

Field numbers follow the public ``onnx.proto3`` schema.  The reference loads
models through onnx-ir (``crates/tynx/src/session.rs:74-140``); its tests embed
models as hex strings built with the protobuf crate
(``crates/tynx-train/src/imported_model/tests.rs``), and the same bytes decode
here.
"""

from __future__ import annotations

import struct
from dataclasses import dataclass, field
from typing import Optional, Union

import numpy as np

# TensorProto.DataType
FLOAT = 1
UINT8 = 2
INT8 = 3
INT32 = 6
INT64 = 7
STRING = 8
BOOL = 9
FLOAT16 = 10
DOUBLE = 11

_NP_OF = {
    FLOAT: np.float32,
    UINT8: np.uint8,
    INT8: np.int8,
    INT32: np.int32,
    INT64: np.int64,
    BOOL: np.bool_,
    FLOAT16: np.float16,
    DOUBLE: np.float64,
}
_DT_OF = {np.dtype(v): k for k, v in _NP_OF.items()}

# AttributeProto.AttributeType
A_FLOAT, A_INT, A_STRING, A_TENSOR, A_GRAPH = 1, 2, 3, 4, 5
A_FLOATS, A_INTS, A_STRINGS, A_TENSORS = 6, 7, 8, 9


class ProtoError(ValueError):
    """Malformed or unsupported ONNX protobuf bytes."""


# ----------------------------------------------------------------------------
# wire format
# ----------------------------------------------------------------------------


def _read_varint(buf: memoryview, pos: int) -> tuple[int, int]:
    result = 0
    shift = 0
    while True:
        if pos >= len(buf):
            raise ProtoError("truncated varint")
        byte = buf[pos]
        pos += 1
        result |= (byte & 0x7F) << shift
        if not byte & 0x80:
            return result, pos
        shift += 7
        if shift > 63:
            raise ProtoError("varint too long")


def _signed64(value: int) -> int:
    return value - (1 << 64) if value >= (1 << 63) else value


def _fields(buf: Union[bytes, memoryview]):
    """Yield ``(field_number, wire_type, value)``; length-delimited values are memoryviews."""
    view = memoryview(buf)
    pos = 0
    end = len(view)
    while pos < end:
        key, pos = _read_varint(view, pos)
        number, wire = key >> 3, key & 7
        if wire == 0:
            value, pos = _read_varint(view, pos)
        elif wire == 1:
            if pos + 8 > end:
                raise ProtoError("truncated fixed64")
            value = view[pos : pos + 8]
            pos += 8
        elif wire == 2:
            length, pos = _read_varint(view, pos)
            if pos + length > end:
                raise ProtoError("truncated length-delimited field")
            value = view[pos : pos + length]
            pos += length
        elif wire == 5:
            if pos + 4 > end:
                raise ProtoError("truncated fixed32")
            value = view[pos : pos + 4]
            pos += 4
        else:
            raise ProtoError(f"unsupported wire type {wire}")
        yield number, wire, value


def _packed_varints(wire: int, value) -> list[int]:
    if wire == 0:
        return [_signed64(value)]
    out = []
    pos = 0
    while pos < len(value):
        v, pos = _read_varint(value, pos)
        out.append(_signed64(v))
    return out


def _packed_floats(wire: int, value) -> list[float]:
    if wire == 5:
        return [struct.unpack("<f", bytes(value))[0]]
    return list(struct.unpack(f"<{len(value) // 4}f", bytes(value)))


def _packed_doubles(wire: int, value) -> list[float]:
    if wire == 1:
        return [struct.unpack("<d", bytes(value))[0]]
    return list(struct.unpack(f"<{len(value) // 8}d", bytes(value)))


def _text(value) -> str:
    return bytes(value).decode("utf-8")


# ----------------------------------------------------------------------------
# message model
# ----------------------------------------------------------------------------


@dataclass
class Tensor:
    name: str
    dims: list[int]
    data_type: int
    array: np.ndarray


@dataclass
class Attribute:
    name: str
    type: int
    value: object


@dataclass
class Node:
    op_type: str
    inputs: list[str]
    outputs: list[str]
    name: str = ""
    domain: str = ""
    attributes: dict[str, Attribute] = field(default_factory=dict)

    def attr(self, name: str, default=None):
        found = self.attributes.get(name)
        return default if found is None else found.value


@dataclass
class ValueInfo:
    name: str
    elem_type: int = 0
    # each dim is an int (static) or a str (symbolic) or None (unknown)
    shape: Optional[list[Union[int, str, None]]] = None


@dataclass
class Graph:
    name: str = ""
    nodes: list[Node] = field(default_factory=list)
    initializers: list[Tensor] = field(default_factory=list)
    inputs: list[ValueInfo] = field(default_factory=list)
    outputs: list[ValueInfo] = field(default_factory=list)
    value_info: list[ValueInfo] = field(default_factory=list)


@dataclass
class Model:
    ir_version: int = 8
    producer_name: str = ""
    opset: dict[str, int] = field(default_factory=dict)
    graph: Graph = field(default_factory=Graph)


# ----------------------------------------------------------------------------
# decode
# ----------------------------------------------------------------------------


def _decode_tensor(buf) -> Tensor:
    dims: list[int] = []
    data_type = 0
    name = ""
    raw = None
    floats: list[float] = []
    int32s: list[int] = []
    int64s: list[int] = []
    doubles: list[float] = []
    for number, wire, value in _fields(buf):
        if number == 1:
            dims.extend(_packed_varints(wire, value))
        elif number == 2:
            data_type = value
        elif number == 4:
            floats.extend(_packed_floats(wire, value))
        elif number == 5:
            int32s.extend(_packed_varints(wire, value))
        elif number == 7:
            int64s.extend(_packed_varints(wire, value))
        elif number == 8:
            name = _text(value)
        elif number == 9:
            raw = bytes(value)
        elif number == 10:
            doubles.extend(_packed_doubles(wire, value))
        elif number == 14 and value == 1:
            raise ProtoError(f"tensor {name!r} uses external data, which is not supported")
    if data_type not in _NP_OF:
        raise ProtoError(f"tensor {name!r} has unsupported data type {data_type}")
    dtype = np.dtype(_NP_OF[data_type])
    count = int(np.prod(dims)) if dims else 1
    if raw is not None:
        array = np.frombuffer(raw, dtype=dtype.newbyteorder("<")).astype(dtype)
    elif data_type == FLOAT:
        array = np.asarray(floats, dtype=np.float32)
    elif data_type == DOUBLE:
        array = np.asarray(doubles, dtype=np.float64)
    elif data_type == INT64:
        array = np.asarray(int64s, dtype=np.int64)
    elif data_type in (INT32, INT8, UINT8, BOOL):
        array = np.asarray(int32s, dtype=np.int64).astype(dtype)
    elif data_type == FLOAT16:
        array = np.asarray(int32s, dtype=np.uint16).view(np.float16)
    else:
        array = np.zeros(0, dtype=dtype)
    if array.size != count:
        raise ProtoError(
            f"tensor {name!r} holds {array.size} values but its dims {dims} need {count}"
        )
    return Tensor(name, dims, data_type, array.reshape(dims))


def _decode_attribute(buf) -> Attribute:
    name = ""
    atype = 0
    f = i = s = t = None
    floats: list[float] = []
    ints: list[int] = []
    strings: list[str] = []
    tensors: list[Tensor] = []
    for number, wire, value in _fields(buf):
        if number == 1:
            name = _text(value)
        elif number == 20:
            atype = value
        elif number == 2:
            f = _packed_floats(wire, value)[0]
        elif number == 3:
            i = _signed64(value)
        elif number == 4:
            s = bytes(value)
        elif number == 5:
            t = _decode_tensor(value)
        elif number == 7:
            floats.extend(_packed_floats(wire, value))
        elif number == 8:
            ints.extend(_packed_varints(wire, value))
        elif number == 9:
            strings.append(_text(value))
        elif number == 10:
            tensors.append(_decode_tensor(value))
    if atype == 0:  # proto2 writers may omit the type; infer it from the populated field
        atype = (
            A_FLOAT if f is not None else A_INT if i is not None else A_STRING if s is not None
            else A_TENSOR if t is not None else A_FLOATS if floats else A_INTS if ints
            else A_STRINGS if strings else A_TENSORS if tensors else 0
        )
    value: object = {
        A_FLOAT: f if f is not None else 0.0,
        A_INT: i if i is not None else 0,
        A_STRING: (s or b"").decode("utf-8", "replace"),
        A_TENSOR: t,
        A_FLOATS: floats,
        A_INTS: ints,
        A_STRINGS: strings,
        A_TENSORS: tensors,
    }.get(atype)
    return Attribute(name, atype, value)


def _decode_node(buf) -> Node:
    node = Node(op_type="", inputs=[], outputs=[])
    for number, _wire, value in _fields(buf):
        if number == 1:
            node.inputs.append(_text(value))
        elif number == 2:
            node.outputs.append(_text(value))
        elif number == 3:
            node.name = _text(value)
        elif number == 4:
            node.op_type = _text(value)
        elif number == 7:
            node.domain = _text(value)
        elif number == 5:
            attribute = _decode_attribute(value)
            node.attributes[attribute.name] = attribute
    return node


def _decode_value_info(buf) -> ValueInfo:
    info = ValueInfo(name="")
    for number, _wire, value in _fields(buf):
        if number == 1:
            info.name = _text(value)
        elif number == 2:  # TypeProto
            for tnum, _tw, tval in _fields(value):
                if tnum != 1:  # tensor_type
                    continue
                for fnum, _fw, fval in _fields(tval):
                    if fnum == 1:
                        info.elem_type = fval
                    elif fnum == 2:  # TensorShapeProto
                        info.shape = []
                        for dnum, _dw, dval in _fields(fval):
                            if dnum != 1:
                                continue
                            dim: Union[int, str, None] = None
                            for xnum, _xw, xval in _fields(dval):
                                if xnum == 1:
                                    dim = _signed64(xval)
                                elif xnum == 2:
                                    dim = _text(xval)
                            info.shape.append(dim)
    return info


def _decode_graph(buf) -> Graph:
    graph = Graph()
    for number, _wire, value in _fields(buf):
        if number == 1:
            graph.nodes.append(_decode_node(value))
        elif number == 2:
            graph.name = _text(value)
        elif number == 5:
            graph.initializers.append(_decode_tensor(value))
        elif number == 11:
            graph.inputs.append(_decode_value_info(value))
        elif number == 12:
            graph.outputs.append(_decode_value_info(value))
        elif number == 13:
            graph.value_info.append(_decode_value_info(value))
    return graph


def decode_model(data: bytes) -> Model:
    """Decode ONNX ``ModelProto`` bytes."""
    model = Model(ir_version=0)
    seen_graph = False
    for number, _wire, value in _fields(data):
        if number == 1:
            model.ir_version = value
        elif number == 2:
            model.producer_name = _text(value)
        elif number == 7:
            model.graph = _decode_graph(value)
            seen_graph = True
        elif number == 8:
            domain, version = "", 0
            for onum, _ow, oval in _fields(value):
                if onum == 1:
                    domain = _text(oval)
                elif onum == 2:
                    version = oval
            model.opset[domain] = version
    if not seen_graph:
        raise ProtoError("ModelProto has no graph")
    return model


# ----------------------------------------------------------------------------
# encode
# ----------------------------------------------------------------------------


def _varint(value: int) -> bytes:
    if value < 0:
        value += 1 << 64
    out = bytearray()
    while True:
        byte = value & 0x7F
        value >>= 7
        if value:
            out.append(byte | 0x80)
        else:
            out.append(byte)
            return bytes(out)


def _key(number: int, wire: int) -> bytes:
    return _varint((number << 3) | wire)


def _len_field(number: int, payload: bytes) -> bytes:
    return _key(number, 2) + _varint(len(payload)) + payload


def _str_field(number: int, text: str) -> bytes:
    return _len_field(number, text.encode("utf-8"))


def _int_field(number: int, value: int) -> bytes:
    return _key(number, 0) + _varint(value)


def encode_tensor(name: str, array: np.ndarray) -> bytes:
    array = np.ascontiguousarray(array)
    if array.dtype not in _DT_OF:
        raise ProtoError(f"cannot encode dtype {array.dtype}")
    out = b"".join(_int_field(1, int(d)) for d in array.shape)
    out += _int_field(2, _DT_OF[array.dtype])
    out += _str_field(8, name)
    out += _len_field(9, array.astype(array.dtype.newbyteorder("<"), copy=False).tobytes())
    return out


def encode_attribute(name: str, value) -> bytes:
    out = _str_field(1, name)
    if isinstance(value, bool) or isinstance(value, (int, np.integer)):
        out += _int_field(3, int(value)) + _int_field(20, A_INT)
    elif isinstance(value, float):
        out += _key(2, 5) + struct.pack("<f", value) + _int_field(20, A_FLOAT)
    elif isinstance(value, str):
        out += _len_field(4, value.encode()) + _int_field(20, A_STRING)
    elif isinstance(value, np.ndarray):
        out += _len_field(5, encode_tensor("", value)) + _int_field(20, A_TENSOR)
    elif isinstance(value, (list, tuple)) and all(isinstance(v, (int, np.integer)) for v in value):
        out += _len_field(8, b"".join(_varint(int(v)) for v in value)) + _int_field(20, A_INTS)
    elif isinstance(value, (list, tuple)):
        out += _len_field(7, struct.pack(f"<{len(value)}f", *value)) + _int_field(20, A_FLOATS)
    else:
        raise ProtoError(f"cannot encode attribute {name}={value!r}")
    return out


def encode_node(op_type: str, inputs, outputs, name: str = "", **attributes) -> bytes:
    out = b"".join(_str_field(1, i) for i in inputs)
    out += b"".join(_str_field(2, o) for o in outputs)
    if name:
        out += _str_field(3, name)
    out += _str_field(4, op_type)
    for key in sorted(attributes):
        out += _len_field(5, encode_attribute(key, attributes[key]))
    return out


def encode_value_info(name: str, elem_type: int, shape) -> bytes:
    """ValueInfoProto; ``shape`` None leaves the shape unstated."""
    tensor_type = _int_field(1, elem_type)
    if shape is not None:
        dims = b""
        for d in shape:
            dims += _len_field(1, _int_field(1, d) if isinstance(d, int) else _str_field(2, str(d)))
        tensor_type += _len_field(2, dims)
    return _str_field(1, name) + _len_field(2, _len_field(1, tensor_type))


def encode_model(
    nodes: list[bytes],
    initializers: list[bytes],
    inputs: list[bytes],
    outputs: list[bytes],
    *,
    graph_name: str = "graph",
    opset: int = 17,
    producer: str = "tynx_b200",
) -> bytes:
    graph = b"".join(_len_field(1, n) for n in nodes)
    graph += _str_field(2, graph_name)
    graph += b"".join(_len_field(5, t) for t in initializers)
    graph += b"".join(_len_field(11, i) for i in inputs)
    graph += b"".join(_len_field(12, o) for o in outputs)
    out = _int_field(1, 8) + _str_field(2, producer)
    out += _len_field(7, graph)
    out += _len_field(8, _str_field(1, "") + _int_field(2, opset))
    return out
