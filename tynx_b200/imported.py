"""Imported ONNX models on the CUDA engine: ``load``, ``ImportedModel``, ``Parameter``.

Mirrors the reference's training surface for imported graphs:

* ``tynx.load(path, trainable="auto", ...)`` (``crates/tynx-python/python/tynx/__init__.py:163-183``)
  -> ``PyImportedModel::new`` (``crates/tynx-python/src/imported_model.rs:225-257``);
* ``model(*inputs)`` -> ``PyImportedModel::__call__`` (``imported_model.rs:260-374``): a
  single Tensor for one output, a dict keyed by output name for several;
* ``named_parameters`` / ``state_dict`` / ``load_state_dict`` / ``trainability_report`` /
  ``require_trainable``.

The graph is normalized on the host (``tynx_b200.onnx.ir``) and lowered to the
C node list of ``tx_graph_create``; forward, backward and parameter storage are
native (``tynx_b200/csrc/engine.cu``).
"""

from __future__ import annotations

import ctypes as C
from os import PathLike
from pathlib import Path
from typing import Optional, Union

import numpy as np

from . import _native as N
from ._core import Context, Device, Fn, Storage, Tensor, context, is_grad_enabled
from ._native import lib
from .onnx import ir, proto

_OP_MAP = {
    "Gemm": "GEMM", "MatMul": "MATMUL", "Conv": "CONV", "Gather": "GATHER",
    "LayerNormalization": "LAYERNORM", "Add": "ADD", "Sub": "SUB", "Mul": "MUL", "Div": "DIV",
    "Relu": "RELU", "Tanh": "TANH", "Gelu": "GELU", "Sigmoid": "SIGMOID", "Exp": "EXP",
    "Log": "LOG", "Neg": "NEG", "Softmax": "SOFTMAX", "LogSoftmax": "LOGSOFTMAX",
    "ReduceMean": "REDUCEMEAN", "ReduceSum": "REDUCESUM", "GlobalAveragePool": "GAP",
    "Reshape": "RESHAPE", "Transpose": "TRANSPOSE", "Flatten": "FLATTEN", "Squeeze": "SQUEEZE",
    "Unsqueeze": "UNSQUEEZE", "Identity": "IDENTITY", "Clip": "CLIP", "PRelu": "PRELU",
    "BatchNormalization": "BATCHNORM", "InstanceNormalization": "GROUPNORM",
    "GroupNormalization": "GROUPNORM", "MaxPool": "MAXPOOL",
    "Sqrt": "UNARY", "Abs": "UNARY", "Reciprocal": "UNARY", "Erf": "UNARY", "LeakyRelu": "UNARY",
    "Softplus": "UNARY", "Elu": "UNARY", "HardSigmoid": "UNARY", "Softsign": "UNARY", "Pow": "BINARY",
    "Max": "BINARY", "Min": "BINARY", "Concat": "CONCAT", "Slice": "SLICE", "Split": "SPLIT",
    "Expand": "EXPAND", "AveragePool": "AVGPOOL", "ReduceMax": "REDUCEMAX", "ReduceMin": "REDUCEMIN",
    "GlobalMaxPool": "REDUCEMAX", "Dropout": "IDENTITY",
}
# the unary operators' kernel codes and their (a, b) from the attributes
_UNARY = {"Sqrt": ("sqrt", None), "Abs": ("abs", None), "Reciprocal": ("reciprocal", None),
          "Erf": ("erf", None), "LeakyRelu": ("leakyrelu", ("alpha",)), "Softplus": ("softplus", None),
          "Elu": ("elu", ("alpha",)), "HardSigmoid": ("hardsigmoid", ("alpha", "beta")),
          "Softsign": ("softsign", None)}
_AUTO_PAD = {"NOTSET": 0, "": 0, "VALID": 1, "SAME_UPPER": 2, "SAME_LOWER": 3}

_ELEM_TO_DTYPE = {proto.FLOAT: "float32", proto.INT64: "int64", proto.INT32: "int64",
                  proto.DOUBLE: "float32", proto.BOOL: "bool"}


class Parameter(Tensor):
    """A trainable slot backed by the engine's parameter storage.

    ``grad`` is ``None`` until a backward writes it, and again after
    ``zero_grad`` (``ParameterSlot::zero_grad``, ``crates/tynx-train/src/parameter.rs:155``).
    Values are updated in place by the optimizer, so the next forward sees them
    (``replace_values_atomic``, ``parameter.rs:227-257``).
    """

    __slots__ = ("name", "_graph", "_index", "_grad_ptr")

    @classmethod
    def _slot(cls, graph: "_Graph", index: int, name: str, shape, value_ptr: int, grad_ptr: int):
        p = object.__new__(cls)
        p._init(Storage(graph.ctx, _nbytes(shape), ptr=value_ptr, owned=False), 0, shape, "float32",
                True)
        p.name = name
        p._graph = graph
        p._index = index
        p._grad_ptr = grad_ptr
        return p

    def _raw_grad_defined(self) -> bool:
        out = C.c_int()
        lib.tx_graph_grad_defined(self._graph.handle, self._index, C.byref(out))
        return bool(out.value)

    @property
    def grad_defined(self) -> bool:
        _note(self, "read")
        return self._raw_grad_defined()

    def _set_grad_defined(self, flag: bool) -> None:
        lib.tx_graph_set_grad_defined(self._graph.handle, self._index, int(flag))

    def _write_grad_defined(self, flag: bool) -> None:
        _note(self, "write")
        self._set_grad_defined(flag)

    @property
    def grad(self) -> Optional[Tensor]:
        if not self.grad_defined:
            return None
        return Tensor._view(Storage(self.ctx, self.nbytes, ptr=self._grad_ptr, owned=False), 0,
                            self.shape, "float32")

    @grad.setter
    def grad(self, value: Optional[Tensor]) -> None:
        if value is None:
            self._write_grad_defined(False)
            return
        if tuple(value.shape) != self.shape:
            raise ValueError(f"gradient shape {value.shape} does not match parameter {self.shape}")
        self.ctx.check(lib.tx_d2d(self.ctx.handle, self._grad_ptr, value.ptr, self.nbytes))
        self._write_grad_defined(True)

    def zero_grad(self) -> None:
        self._write_grad_defined(False)

    def _accumulate_grad(self, g: Tensor) -> None:
        """Gradients reaching this slot through eager operations."""
        if self.grad_defined:
            shape = N.i64_array(self.shape)
            strides = N.i64_array([0] * 0 + _contig(self.shape))
            self.ctx.check(lib.tx_binary(self.ctx.handle, N.BIN["add"], self._grad_ptr, strides,
                                         g.ptr, strides, self._grad_ptr, shape, len(self.shape)))
        else:
            self.ctx.check(lib.tx_d2d(self.ctx.handle, self._grad_ptr, g.ptr, self.nbytes))
            self._write_grad_defined(True)

    def copy_(self, value) -> "Parameter":
        array = np.ascontiguousarray(np.asarray(value.numpy() if isinstance(value, Tensor) else value,
                                                dtype=np.float32))
        if array.shape != self.shape:
            raise ValueError(f"value shape {array.shape} does not match parameter {self.shape}")
        self.ctx.check(lib.tx_h2d(self.ctx.handle, self.ptr, array.ctypes.data, array.nbytes))
        self.ctx.sync()
        return self

    def __repr__(self) -> str:
        return f"Parameter({self.name!r}, shape={self.shape})"


class Buffer(Tensor):
    """Persistent non-trainable state of an imported model (the BatchNorm
    running statistics): a view of the engine's own storage, read by every
    forward and never touched by backward or the optimizer
    (``crates/tynx-train/src/backward_support.rs:165-167``)."""

    __slots__ = ("name", "_graph")

    @classmethod
    def _slot(cls, graph: "_Graph", name: str, shape, ptr: int, dtype: str = "float32"):
        b = object.__new__(cls)
        b._init(Storage(graph.ctx, _nbytes(shape) * (2 if dtype == "int64" else 1), ptr=ptr,
                        owned=False), 0, shape, dtype, False)
        b.name = name
        b._graph = graph
        return b

    def copy_(self, value) -> "Buffer":
        from ._core import _DTYPES

        array = np.ascontiguousarray(np.asarray(value.numpy() if isinstance(value, Tensor) else value,
                                                dtype=_DTYPES[self.dtype][0]))
        if array.shape != self.shape:
            raise ValueError(f"value shape {array.shape} does not match buffer {self.shape}")
        self.ctx.check(lib.tx_h2d(self.ctx.handle, self.ptr, array.ctypes.data, array.nbytes))
        self.ctx.sync()
        return self

    def __repr__(self) -> str:
        return f"Buffer({self.name!r}, shape={self.shape})"


def _note(param, kind: str) -> None:
    from . import compiler

    if compiler._capture_log is not None:
        compiler.note_grad_flag(param, kind)


def _nbytes(shape) -> int:
    n = 4
    for s in shape:
        n *= s
    return n


def _contig(shape) -> list[int]:
    out = [0] * len(shape)
    acc = 1
    for i in range(len(shape) - 1, -1, -1):
        out[i] = acc
        acc *= shape[i]
    return out


class _Record:
    """Saved activations of one tracked forward; freed with its tape node."""

    __slots__ = ("handle", "graph")

    def __init__(self, handle, graph):
        self.handle = handle
        self.graph = graph

    def free(self) -> None:
        if self.handle:
            lib.tx_record_free(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.free()
        except Exception:  # interpreter shutdown
            pass


class _Graph:
    """Owns a ``tx_graph`` handle."""

    def __init__(self, ctx: Context, handle):
        self.ctx = ctx
        self.handle = handle

    def __del__(self):
        try:
            if self.handle:
                lib.tx_graph_destroy(self.handle)
                self.handle = None
        except Exception:
            pass


# =============================================================================
# lowering
# =============================================================================


def _const_ints(graph: ir.TrainingGraph, name: str) -> list[int]:
    if name not in graph.constants:
        raise NotImplementedError(f"input {name!r} must be a constant for the CUDA engine")
    return [int(v) for v in np.asarray(graph.constants[name]).reshape(-1)]


def _const_float(graph: ir.TrainingGraph, name: str) -> float:
    if name not in graph.constants:
        raise NotImplementedError(f"input {name!r} must be a constant for the CUDA engine")
    return float(np.asarray(graph.constants[name]).reshape(-1)[0])


def lower(graph: ir.TrainingGraph):
    """TrainingGraph -> (value descs, node descs, output ids, bookkeeping)."""
    ids: dict[str, int] = {}
    values: list[N.ValueDesc] = []
    keep: list = []  # host arrays referenced by ValueDesc.h_data
    param_names: list[str] = []

    def add_value(name: str, kind: int, dtype: int, shape=None, data=None) -> int:
        desc = N.ValueDesc()
        desc.kind, desc.dtype = kind, dtype
        if shape is None:
            desc.ndim = -1
        else:
            if len(shape) > N.MAX_DIMS:
                raise NotImplementedError(f"value {name!r} has rank {len(shape)} > 8")
            desc.ndim = len(shape)
            for i, s in enumerate(shape):
                desc.shape[i] = int(s)
        if data is not None:
            keep.append(data)
            desc.h_data = data.ctypes.data
        ids[name] = len(values)
        values.append(desc)
        return ids[name]

    for info in graph.inputs:
        dtype = N.DT_I64 if _ELEM_TO_DTYPE.get(info.elem_type) == "int64" else N.DT_F32
        shape = None
        if info.shape is not None and all(isinstance(d, int) for d in info.shape):
            shape = info.shape
        add_value(info.name, N.VAL_INPUT, dtype, None if shape is None else shape)
        if shape is not None:  # only the rank is enforced; dims may vary (batch)
            pass
    for value, public in graph.parameter_of_value.items():
        array = np.ascontiguousarray(graph.parameters[public], dtype=np.float32)
        add_value(value, N.VAL_PARAM, N.DT_F32, array.shape, array)
        param_names.append(public)

    def const_id(name: str) -> int:
        if name in ids:
            return ids[name]
        array = np.asarray(graph.constants[name])
        if array.dtype.kind in "iub":
            array = np.ascontiguousarray(array, dtype=np.int64)
            dtype = N.DT_I64
        else:
            array = np.ascontiguousarray(array, dtype=np.float32)
            dtype = N.DT_F32
        return add_value(name, N.VAL_CONST, dtype, array.shape, array)

    def value_id(name: str) -> int:
        if name in ids:
            return ids[name]
        if name in graph.constants:
            return const_id(name)
        raise ValueError(f"value {name!r} is used before it is produced")

    nodes: list[N.NodeDesc] = []
    for op in graph.ops:
        kind = _OP_MAP.get(op.op_type)
        if kind is None:
            raise NotImplementedError(
                f"operator {op.op_type} (node {op.name!r}) is not supported by the CUDA engine"
            )
        a = op.attrs
        d = N.NodeDesc()
        d.op = N.OP[kind]
        ins = list(op.inputs)
        ints: list[int] = []
        t = op.op_type
        if t == "Gemm":
            d.iattr[0], d.iattr[1] = int(a["transA"]), int(a["transB"])
            d.fattr[0], d.fattr[1] = float(a["alpha"]), float(a["beta"])
        elif t == "Conv":
            W = graph.parameters.get(graph.parameter_of_value.get(ins[1], ""), None)
            if W is None and ins[1] in graph.constants:
                W = graph.constants[ins[1]]
            nd = (W.ndim - 2) if W is not None else 2
            strides = list(a.get("strides") or [1] * nd)
            pads = list(a.get("pads") or [0] * (2 * nd))
            dil = list(a.get("dilations") or [1] * nd)
            if nd == 1:  # 1-D convolution runs as 2-D over a unit height
                strides, dil, pads = [1] + strides, [1] + dil, [0, pads[0], 0, pads[1]]
            elif nd != 2:
                raise NotImplementedError(f"{nd}-D Conv is not supported by the CUDA engine")
            # ONNX pads are [x1_begin, x2_begin, x1_end, x2_end]
            ints = strides + [pads[0], pads[1], pads[2], pads[3]] + dil
            d.iattr[0] = int(a["group"])
        elif t == "Gather":
            d.iattr[0] = int(a["axis"])
        elif t == "BatchNormalization":
            d.fattr[0] = float(a["epsilon"])
        elif t in ("InstanceNormalization", "GroupNormalization"):
            # InstanceNormalization is group normalization with one group per channel
            d.iattr[0] = int(a["num_groups"]) if t == "GroupNormalization" else 0
            d.fattr[0] = float(a["epsilon"])
        elif t == "MaxPool":
            k, st, dil, pads = (list(a["kernel_shape"]), list(a["strides"]), list(a["dilations"]),
                                list(a["pads"]))
            if len(k) == 1:  # 1-D pooling runs as 2-D over a unit height
                k, st, dil, pads = [1] + k, [1] + st, [1] + dil, [0, pads[0], 0, pads[1]]
            if len(k) != 2:
                raise NotImplementedError(f"{len(k)}-D MaxPool is not supported by the CUDA engine")
            if a.get("auto_pad", "NOTSET") not in _AUTO_PAD:
                raise ValueError(f"MaxPool node {op.name!r}: unknown auto_pad {a['auto_pad']!r}")
            # ONNX pads are [x1_begin, x2_begin, x1_end, x2_end]
            ints = [k[0], k[1], st[0], st[1], pads[0], pads[1], pads[2], pads[3], dil[0], dil[1]]
            d.iattr[0] = int(a["ceil_mode"])
            d.iattr[1] = _AUTO_PAD[a.get("auto_pad", "NOTSET")]
        elif t == "LayerNormalization":
            d.iattr[0] = int(a["axis"])
            d.fattr[0] = float(a["epsilon"])
        elif t in ("Softmax", "LogSoftmax"):
            d.iattr[0] = int(a["axis"])
        elif t in ("ReduceMean", "ReduceSum"):
            axes = a.get("axes")
            if axes is None and len(ins) > 1 and ins[1]:
                axes = _const_ints(graph, ins[1])
            ins = ins[:1]
            ints = list(axes or [])
            d.iattr[0] = int(a["keepdims"])
            if not ints and a.get("noop_with_empty_axes", 0):
                raise NotImplementedError("ReduceMean noop_with_empty_axes")
        elif t == "Reshape":
            ints = _const_ints(graph, ins[1])
            ins = ins[:1]
            d.iattr[0] = int(a.get("allowzero", 0))
        elif t == "Transpose":
            ints = list(a.get("perm") or [])
        elif t == "Flatten":
            d.iattr[0] = int(a["axis"])
        elif t in ("Squeeze", "Unsqueeze"):
            axes = a.get("axes")
            if axes is None and len(ins) > 1 and ins[1]:
                axes = _const_ints(graph, ins[1])
            ints = list(axes or [])
            ins = ins[:1]
        elif t in _UNARY:
            code, names = _UNARY[t]
            d.iattr[0] = N.UN[code]
            for i, name in enumerate(names or ()):
                d.fattr[i] = float(a[name])
        elif t == "Pow":
            exponent = graph.constants.get(ins[1]) if len(ins) > 1 else None
            if exponent is not None and np.asarray(exponent).size == 1:
                # a constant scalar exponent: the unary power (its gradient
                # reaches the base only, as the reference's)
                d.op = N.OP["UNARY"]
                d.iattr[0] = N.UN["pow"]
                d.fattr[0] = float(np.asarray(exponent).reshape(-1)[0])
                ins = ins[:1]
            else:
                d.iattr[0] = N.BIN["pow"]
        elif t in ("Max", "Min"):
            if len(ins) == 1:
                d.op = N.OP["IDENTITY"]
            elif len(ins) != 2:
                raise NotImplementedError(f"{t} over {len(ins)} inputs is not supported by the CUDA engine")
            else:
                d.iattr[0] = N.BIN["max" if t == "Max" else "min"]
        elif t == "Concat":
            d.iattr[0] = int(a["axis"])
        elif t == "Slice":
            if len(ins) > 1:  # opset >= 10: starts, ends, axes, steps as inputs
                starts = _const_ints(graph, ins[1])
                ends = _const_ints(graph, ins[2])
                axes = _const_ints(graph, ins[3]) if len(ins) > 3 and ins[3] else list(range(len(starts)))
                steps = _const_ints(graph, ins[4]) if len(ins) > 4 and ins[4] else [1] * len(starts)
            else:
                starts, ends = list(a["starts"]), list(a["ends"])
                axes = list(a.get("axes") or range(len(starts)))
                steps = [1] * len(starts)
            if len(axes) > 3:
                raise NotImplementedError(f"Slice node {op.name!r} over more than 3 axes")
            big = (1 << 62)
            clip = [max(-big, min(big, int(v))) for v in ends]
            ints = [len(axes)] + list(axes) + list(starts) + clip + list(steps)
            ins = ins[:1]
        elif t == "Split":
            d.iattr[0] = int(a["axis"])
            sizes = a.get("split")
            if sizes is None and len(ins) > 1 and ins[1]:
                sizes = _const_ints(graph, ins[1])
            # no sizes: equal parts of the runtime extent (the engine's shapes),
            # the last one smaller when they do not divide it
            ints = list(sizes or [])
            ins = ins[:1]
        elif t == "Expand":
            ints = _const_ints(graph, ins[1])
            ins = ins[:1]
        elif t in ("ReduceMax", "ReduceMin", "GlobalMaxPool"):
            if t == "GlobalMaxPool":
                axes = "spatial"
            else:
                axes = a.get("axes")
                if axes is None and len(ins) > 1 and ins[1]:
                    axes = _const_ints(graph, ins[1])
                if not axes and a.get("noop_with_empty_axes", 0):
                    raise NotImplementedError(f"{t} noop_with_empty_axes")
            ints = [] if axes == "spatial" else list(axes or [])
            d.iattr[0] = 1 if t == "GlobalMaxPool" else int(a["keepdims"])
            d.iattr[1] = int(axes == "spatial")
            ins = ins[:1]
        elif t == "Dropout":
            if len(ins) > 2 and ins[2]:
                mode = graph.constants.get(ins[2])
                if mode is None or bool(np.asarray(mode).reshape(-1)[0]):
                    raise NotImplementedError(f"Dropout node {op.name!r} in training mode")
            ins = ins[:1]
        elif t == "AveragePool":
            k, st, dil, pads = (list(a["kernel_shape"]), list(a["strides"]), list(a["dilations"]),
                                list(a["pads"]))
            if len(k) == 1:  # 1-D pooling runs as 2-D over a unit height
                k, st, dil, pads = [1] + k, [1] + st, [1] + dil, [0, pads[0], 0, pads[1]]
            if len(k) != 2:
                raise NotImplementedError(f"{len(k)}-D AveragePool is not supported by the CUDA engine")
            if a.get("auto_pad", "NOTSET") not in _AUTO_PAD:
                raise ValueError(f"AveragePool node {op.name!r}: unknown auto_pad {a['auto_pad']!r}")
            ints = [k[0], k[1], st[0], st[1], pads[0], pads[1], pads[2], pads[3], dil[0], dil[1]]
            d.iattr[0] = int(a["ceil_mode"])
            d.iattr[1] = _AUTO_PAD[a.get("auto_pad", "NOTSET")]
            d.iattr[2] = int(a["count_include_pad"])
        elif t == "Clip":
            lo = a.get("min")
            hi = a.get("max")
            if len(ins) > 1 and ins[1]:
                lo = _const_float(graph, ins[1])
            if len(ins) > 2 and ins[2]:
                hi = _const_float(graph, ins[2])
            ins = ins[:1]
            d.iattr[0], d.iattr[1] = int(lo is not None), int(hi is not None)
            d.fattr[0] = float(lo) if lo is not None else 0.0
            d.fattr[1] = float(hi) if hi is not None else 0.0
        if len(ints) > 16:
            raise NotImplementedError(f"node {op.name!r} has too many list attributes")
        d.n_ints = len(ints)
        for i, v in enumerate(ints):
            d.ints[i] = int(v)
        if len(ins) > 6 or len(op.outputs) > 3:
            raise NotImplementedError(f"node {op.name!r} has too many inputs or outputs")
        d.n_in = len(ins)
        for i, name in enumerate(ins):
            d.inp[i] = value_id(name) if name else -1
        d.n_out = len(op.outputs)
        for i, name in enumerate(op.outputs):
            if name in ids:
                raise ValueError(f"value {name!r} is produced twice")
            add_value(name, N.VAL_ACT, N.DT_F32)
            d.out[i] = ids[name]
        nodes.append(d)
    # integer-valued activations (a Gather on int64 data) are not produced by the configs;
    # keep every produced value float32
    outputs = [value_id(o) for o in graph.outputs]
    return values, nodes, outputs, keep, param_names, ids


# =============================================================================
# model
# =============================================================================


class ImportedModel:
    """A callable slot-backed training model (``PyImportedModel``)."""

    def __init__(self, path: Union[str, PathLike, bytes], *, simplify: bool = True,
                 initializer_names: Optional[dict] = None, outputs: Optional[list] = None,
                 device: Optional[Device] = None, trainable: bool = True):
        data = path if isinstance(path, (bytes, bytearray)) else Path(path).read_bytes()
        self._graph_ir = ir.load_training_graph(bytes(data), initializer_names=initializer_names,
                                                outputs=outputs)
        if trainable and self._graph_ir.report.errors:
            raise ValueError("; ".join(self._graph_ir.report.errors))
        self._simplify = simplify
        self._ctx = context(device)
        values, nodes, out_ids, keep, param_names, ids = lower(self._graph_ir)
        handle = C.c_void_p()
        vals = (N.ValueDesc * len(values))(*values)
        nds = (N.NodeDesc * max(len(nodes), 1))(*nodes)
        outs = N.i32_array(out_ids)
        self._ctx.check(lib.tx_graph_create(self._ctx.handle, vals, len(values), nds, len(nodes),
                                            outs, len(out_ids), C.byref(handle)), "graph build")
        del keep
        self._graph = _Graph(self._ctx, handle)
        self._input_infos = list(self._graph_ir.inputs)
        self._input_dtypes = [
            "int64" if _ELEM_TO_DTYPE.get(i.elem_type) == "int64" else "float32"
            for i in self._input_infos
        ]
        self._input_ranks = [len(i.shape) if i.shape is not None else None
                             for i in self._input_infos]
        count = C.c_int()
        lib.tx_graph_param_count(handle, C.byref(count))
        self._params: dict[str, Parameter] = {}
        for i in range(count.value):
            vid, vptr, gptr, numel = C.c_int32(), C.c_void_p(), C.c_void_p(), C.c_int64()
            lib.tx_graph_param(handle, i, C.byref(vid), C.byref(vptr), C.byref(gptr), C.byref(numel))
            name = param_names[i]
            shape = tuple(self._graph_ir.parameters[name].shape)
            self._params[name] = Parameter._slot(self._graph, i, name, shape, vptr.value, gptr.value)
        self._buffers: dict[str, Buffer] = {}
        for value, public in self._graph_ir.buffer_of_value.items():
            if value not in ids:
                continue  # a buffer no node reads
            ptr = C.c_void_p()
            self._ctx.check(lib.tx_graph_value_ptr(handle, ids[value], C.byref(ptr)))
            array = self._graph_ir.buffers[public]
            dtype = "int64" if array.dtype.kind in "iu" else "float32"
            self._buffers[public] = Buffer._slot(self._graph, public, tuple(array.shape), ptr.value, dtype)
        self.training = True
        self._shape_cache: dict = {}
        from .compiler import register_model

        register_model(self)

    # -- introspection ------------------------------------------------------------------
    @property
    def outputs(self) -> list[str]:
        return list(self._graph_ir.outputs)

    @property
    def inputs(self) -> list[str]:
        return [i.name for i in self._input_infos]

    @property
    def device(self) -> Device:
        return Device(f"cuda:{self._ctx.index}")

    def named_parameters(self) -> list[tuple[str, Parameter]]:
        return list(self._params.items())

    def parameters(self) -> list[Parameter]:
        return list(self._params.values())

    def named_buffers(self) -> list[tuple[str, Buffer]]:
        return list(self._buffers.items())

    def buffers(self) -> list[Buffer]:
        return list(self._buffers.values())

    def state_dict(self) -> dict[str, Tensor]:
        """Detached copies of every parameter and buffer, by stable name."""
        state = {name: p.detach().clone() for name, p in self._params.items()}
        state.update({name: b.detach().clone() for name, b in self._buffers.items()})
        return state

    def load_state_dict(self, state: dict, strict: bool = True):
        """Copy tensors into the live parameters by name after validating every
        name, shape and dtype (``crates/tynx-python/python/tynx/nn/state.py``
        ``_prepare_state_dict_load``); returns the missing and unexpected names."""
        from .checkpoint import prepare_model_state

        names, result = prepare_model_state(self, state, strict)
        for name in names:
            (self._params.get(name) or self._buffers[name]).copy_(state[name])
        return result

    def trainability_report(self) -> ir.TrainabilityReport:
        return self._graph_ir.report

    def require_trainable(self, outputs: Optional[list] = None) -> ir.TrainabilityReport:
        report = self._graph_ir.report
        if outputs is not None:
            for name in outputs:
                if name not in self._graph_ir.outputs:
                    raise ValueError(f"requested output {name!r} is not a declared model output")
            selected = ir.TrainabilityReport(
                initializers=report.initializers, selected_outputs=list(outputs),
                output_parameters={o: report.output_parameters[o] for o in outputs},
                backward_issues=report.backward_issues, warnings=report.warnings,
                errors=report.errors)
            return selected.require_trainable()
        return report.require_trainable()

    def zero_grad(self) -> None:
        for p in self._params.values():
            p.zero_grad()

    def train(self, mode: bool = True) -> "ImportedModel":
        self.training = mode
        return self

    def eval(self) -> "ImportedModel":
        return self.train(False)

    def enable_data_parallel(self, bucket_mb: float = 8.0) -> None:
        """Average gradients across ranks inside backward (see ``tynx_b200.distributed``)."""
        self._ctx.check(lib.tx_graph_set_dp(self._graph.handle, 1, int(bucket_mb * (1 << 20))))

    # -- call ------------------------------------------------------------------------------
    def _bind(self, args, kwargs) -> list[Tensor]:
        """Positional inputs in declaration order, then named ones; the
        TypeErrors name what is missing, unexpected or given twice, in the
        reference's wording (test_imported_model.py:483-487)."""
        names = self.inputs
        if len(args) > len(names):
            raise TypeError(f"model takes {len(names)} inputs, got {len(args)}")
        bound: dict[str, object] = dict(zip(names, args))
        for key, value in kwargs.items():
            if key not in names:
                raise TypeError(f"unexpected input {key!r}; the model's inputs are {names}")
            if key in bound:
                raise TypeError(f"got multiple values for input {key!r}")
            bound[key] = value
        missing = [n for n in names if n not in bound]
        if missing:
            raise TypeError(f"missing required inputs {missing}")
        tensors = []
        for name, dtype, rank in zip(names, self._input_dtypes, self._input_ranks):
            value = bound[name]
            if not isinstance(value, Tensor):
                value = Tensor(np.asarray(value), dtype=dtype, device=self.device)
            if value.dtype != dtype:
                raise ValueError(f"input {name!r} must be {dtype}, got {value.dtype}")
            if rank is not None and value.ndim != rank:
                raise ValueError(f"input {name!r} must have rank {rank}, got shape {value.shape}")
            tensors.append(value)
        return tensors

    def _infer(self, inputs: list[Tensor]):
        key = tuple(t.shape for t in inputs)
        cached = self._shape_cache.get(key)
        if cached is not None:
            return cached
        shapes = [s for t in inputs for s in t.shape]
        ndims = [t.ndim for t in inputs]
        n_out = len(self._graph_ir.outputs)
        out_shapes = (C.c_int64 * (8 * n_out))()
        out_ndims = (C.c_int32 * n_out)()
        self._ctx.check(lib.tx_graph_infer(self._graph.handle, N.i64_array(shapes), N.i32_array(ndims),
                                           out_shapes, out_ndims), "shape inference")
        result, off = [], 0
        for i in range(n_out):
            nd = out_ndims[i]
            result.append(tuple(out_shapes[off:off + nd]))
            off += nd
        self._shape_cache[key] = result
        return result

    def __call__(self, *args, **kwargs):
        inputs = self._bind(args, kwargs)
        out_shapes = self._infer(inputs)
        outs = [Tensor._empty(s, "float32", self._ctx) for s in out_shapes]
        tracking = is_grad_enabled()
        rec = C.c_void_p()
        shapes = [s for t in inputs for s in t.shape]
        self._ctx.check(lib.tx_graph_forward(
            self._graph.handle, N.ptr_array([t.ptr for t in inputs]), N.i64_array(shapes),
            N.i32_array([t.ndim for t in inputs]), N.ptr_array([o.ptr for o in outs]),
            int(tracking), C.byref(rec) if tracking else None), "forward")
        if tracking:
            record = _Record(rec.value, self._graph)
            saved_in = [t.detach() for t in inputs]
            saved_out = [o.detach() for o in outs]
            need_in = [t.requires_grad and t.dtype == "float32" for t in inputs]
            graph = self._graph
            ctx = self._ctx

            params = list(self._params.values())

            def backward(grads, record=record, saved_in=saved_in, saved_out=saved_out):
                for p in params:  # backward decides overwrite/accumulate from these flags
                    _note(p, "read")
                d_out = [g.ptr if g is not None else None for g in grads]
                d_in = []
                results = []
                for t, need in zip(saved_in, need_in):
                    if need:
                        g = Tensor._empty(t.shape, "float32", ctx)
                        d_in.append(g.ptr)
                        results.append(g)
                    else:
                        d_in.append(None)
                        results.append(None)
                ctx.check(lib.tx_graph_backward(graph.handle, record.handle, N.ptr_array(d_out),
                                                N.ptr_array(d_in)), "backward")
                # keep outputs alive until here: the record reads them
                del saved_out
                return results

            fn = Fn("imported_model", list(inputs), backward, n_out=len(outs), release=record.free)
            for i, o in enumerate(outs):
                o._attach(fn, i)
        if len(outs) == 1:
            return outs[0]
        return dict(zip(self._graph_ir.outputs, outs))


class Session:
    """Inference-only session over the same engine (``tynx.load(path)``)."""

    def __init__(self, path, *, simplify: bool = True, device: Optional[Device] = None):
        self._model = ImportedModel(path, simplify=simplify, device=device, trainable=False)

    @property
    def outputs(self) -> list[str]:
        return self._model.outputs

    @property
    def inputs(self) -> list[str]:
        return self._model.inputs

    def __call__(self, *args, **kwargs):
        from ._core import no_grad

        with no_grad():
            return self._model(*[a.detach() if isinstance(a, Tensor) else a for a in args],
                               **{k: v.detach() if isinstance(v, Tensor) else v
                                  for k, v in kwargs.items()})

    def run(self, **inputs):
        return self(**inputs)


def load(path: Union[str, PathLike], *, trainable: Union[bool, str] = False, simplify: bool = True,
         initializer_names: Optional[dict] = None, outputs: Optional[list] = None,
         device: Optional[Device] = None):
    """Load an inference Session or a callable slot-backed training model."""
    if trainable is False:
        if initializer_names is not None or outputs is not None:
            raise ValueError("initializer_names and outputs are only valid for a trainable model")
        return Session(path, simplify=simplify, device=device)
    if trainable is not True and trainable != "auto":
        raise ValueError("trainable must be False, True, or 'auto'")
    return ImportedModel(path, simplify=simplify, initializer_names=initializer_names,
                         outputs=outputs, device=device)

