"""ctypes binding of ``libtynx_cuda.so`` (the C ABI in ``include/tynx_cuda.h``).

This is the Python counterpart of the ``tynx-cuda-sys`` crate: plain pointers
and sizes cross the boundary, status codes come back and are turned into the
exceptions the reference raises for the same conditions
(``crates/tynx-python/src/lib.rs:263-268``: shape/type problems -> ValueError,
out-of-range indices -> IndexError).

There is no CPU fallback: importing this module fails loudly when the library
is missing, and every call that needs a GPU fails with the driver's error when
there is none.
"""

from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

_LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libtynx_cuda.so"

TX_OK = 0
TX_ERR_INVALID = 1
TX_ERR_SHAPE = 2
TX_ERR_INDEX = 3
TX_ERR_OOM = 4
TX_ERR_CUDA = 5
TX_ERR_TIMEOUT = 6
TX_ERR_UNSUPPORTED = 7
TX_ERR_DEVICE = 8
TX_ERR_NCCL = 9
TX_ERR_CAPTURE = 10

TX_MATH = {"tf32": 0, "3xtf32": 1, "fp32": 2, "tf32trunc": 3}
MAX_DIMS = 8

ACT = {"none": 0, "relu": 1, "tanh": 2, "gelu": 3}
TX_GEMM_A_TF32, TX_GEMM_B_TF32, TX_GEMM_ROUND_OUT, TX_GEMM_EXACT, TX_GEMM_A_SHARED = 1, 2, 4, 8, 16
UN = {"neg": 0, "exp": 1, "log": 2, "relu": 3, "tanh": 4, "gelu": 5, "sigmoid": 6, "clamp": 7,
      "sqrt": 8, "abs": 9, "scale": 10, "pow": 11, "erf": 12, "leakyrelu": 13, "softplus": 14, "elu": 15,
      "hardsigmoid": 16, "softsign": 17, "reciprocal": 18}
BIN = {"add": 0, "sub": 1, "mul": 2, "div": 3, "min": 4, "max": 5, "le": 6, "ge": 7, "pow": 8}
OP = {name: i + 1 for i, name in enumerate([
    "GEMM", "MATMUL", "CONV", "GATHER", "LAYERNORM", "ADD", "SUB", "MUL", "DIV", "RELU", "TANH",
    "GELU", "SIGMOID", "EXP", "LOG", "NEG", "SOFTMAX", "LOGSOFTMAX", "REDUCEMEAN", "REDUCESUM",
    "GAP", "RESHAPE", "TRANSPOSE", "FLATTEN", "SQUEEZE", "UNSQUEEZE", "IDENTITY", "CLIP", "PRELU",
    "BATCHNORM", "GROUPNORM", "MAXPOOL", "UNARY", "BINARY", "CONCAT", "SLICE", "SPLIT", "EXPAND",
    "AVGPOOL", "REDUCEMAX", "REDUCEMIN"])}
VAL_INPUT, VAL_PARAM, VAL_CONST, VAL_ACT = 0, 1, 2, 3
DT_F32, DT_I64 = 0, 1


class CaptureError(RuntimeError):
    """An operation that cannot be recorded into a CUDA graph was attempted."""


class DeviceTimeoutError(TimeoutError):
    """A bounded device wait expired."""


class GemmDesc(C.Structure):
    _fields_ = [
        ("M", C.c_int64), ("N", C.c_int64), ("K", C.c_int64),
        ("A", C.c_void_p), ("lda", C.c_int64), ("trans_a", C.c_int32),
        ("B", C.c_void_p), ("ldb", C.c_int64), ("trans_b", C.c_int32),
        ("C", C.c_void_p), ("ldc", C.c_int64),
        ("alpha", C.c_float), ("beta", C.c_float),
        ("bias", C.c_void_p), ("bias_scale", C.c_float),
        ("act", C.c_int32),
        ("preact", C.c_void_p), ("ld_preact", C.c_int64),
        ("dact_src", C.c_void_p), ("ld_dact", C.c_int64), ("dact", C.c_int32),
        ("batch", C.c_int64), ("stride_a", C.c_int64), ("stride_b", C.c_int64),
        ("stride_c", C.c_int64), ("flags", C.c_int32),
        ("colsum", C.c_void_p), ("colsum_scale", C.c_float), ("colsum_acc", C.c_int32),
        ("B_lo", C.c_void_p),
    ]


class ValueDesc(C.Structure):
    _fields_ = [
        ("kind", C.c_int32), ("dtype", C.c_int32), ("ndim", C.c_int32),
        ("shape", C.c_int64 * MAX_DIMS), ("h_data", C.c_void_p),
    ]


class NodeDesc(C.Structure):
    _fields_ = [
        ("op", C.c_int32), ("n_in", C.c_int32), ("n_out", C.c_int32),
        ("inp", C.c_int32 * 6), ("out", C.c_int32 * 3),
        ("iattr", C.c_int64 * 8), ("fattr", C.c_double * 4),
        ("n_ints", C.c_int32), ("ints", C.c_int64 * 16),
    ]


class OptimCfg(C.Structure):
    _fields_ = [
        ("kind", C.c_int32), ("lr", C.c_double), ("beta1", C.c_double), ("beta2", C.c_double),
        ("eps", C.c_double), ("weight_decay", C.c_double), ("amsgrad", C.c_int32),
        ("momentum", C.c_double), ("dampening", C.c_double), ("nesterov", C.c_int32),
    ]


_vp = C.c_void_p
_i64 = C.c_int64
_i32 = C.c_int
_f = C.c_float
_p64 = C.POINTER(C.c_int64)
_p32 = C.POINTER(C.c_int32)

# name -> argtypes (every function returns int)
SIGNATURES = {
    "tx_abi_version": [],
    "tx_device_count": [C.POINTER(C.c_int)],
    "tx_ctx_create": [_i32, _i32, C.POINTER(_vp)],
    "tx_ctx_destroy": [_vp],
    "tx_ctx_set_math": [_vp, _i32],
    "tx_ctx_get_math": [_vp, C.POINTER(C.c_int)],
    "tx_last_error": [_vp, C.c_char_p, C.c_size_t],
    "tx_sync": [_vp, C.c_uint64],
    "tx_stream": [_vp, C.POINTER(_vp)],
    "tx_alloc": [_vp, C.c_size_t, C.POINTER(_vp)],
    "tx_free": [_vp, _vp],
    "tx_h2d": [_vp, _vp, _vp, C.c_size_t],
    "tx_prefetch_create": [_vp, C.c_size_t, C.c_int, C.POINTER(_vp)],
    "tx_prefetch_put": [_vp, _vp, C.c_size_t],
    "tx_prefetch_get": [_vp, C.POINTER(_vp)],
    "tx_prefetch_destroy": [_vp],
    "tx_d2h": [_vp, _vp, _vp, C.c_size_t],
    "tx_d2d": [_vp, _vp, _vp, C.c_size_t],
    "tx_memset": [_vp, _vp, _i32, C.c_size_t],
    "tx_fill_f32": [_vp, _vp, _i64, _f],
    "tx_host_alloc": [C.c_size_t, C.POINTER(_vp)],
    "tx_host_free": [_vp],
    "tx_mem_stats": [_vp, C.POINTER(C.c_uint64), C.POINTER(C.c_uint64)],
    "tx_capture_begin": [_vp],
    "tx_capture_end": [_vp, C.POINTER(_vp)],
    "tx_capture_abort": [_vp],
    "tx_capture_active": [_vp, C.POINTER(C.c_int)],
    "tx_exec_launch": [_vp],
    "tx_exec_destroy": [_vp],
    "tx_exec_node_count": [_vp, _p64, _p64],
    "tx_gemm": [_vp, C.POINTER(GemmDesc)],
    "tx_unary": [_vp, _i32, _vp, _vp, _i64, _f, _f],
    "tx_unary_bwd": [_vp, _i32, _vp, _vp, _vp, _i64, _f, _f, _i32],
    "tx_binary": [_vp, _i32, _vp, _p64, _vp, _p64, _vp, _p64, _i32],
    "tx_reduce_to": [_vp, _vp, _p64, _vp, _p64, _i32, _i32, _i32],
    "tx_strided_copy": [_vp, _vp, _p64, _vp, _p64, _i32, _i32],
    "tx_strided_scatter": [_vp, _vp, _vp, _p64, _p64, _i32, _i32],
    "tx_dropout_fwd": [_vp, _vp, _vp, _vp, _i64, C.c_float, C.c_uint64, _vp],
    "tx_softmax_fwd": [_vp, _vp, _vp, _i64, _i64, _i32],
    "tx_softmax_bwd": [_vp, _vp, _vp, _vp, _i64, _i64, _i32, _i32],
    "tx_softmax_xent_fwd": [_vp, _vp, _vp, _i64, _i64, _vp],
    "tx_softmax_xent_bwd": [_vp, _vp, _vp, _i64, _i64, _vp, _vp, _i32],
    "tx_softmax_xent_fwd_noalloc": [_vp, _vp, _vp, _i64, _i64, _vp],
    "tx_layernorm_fwd": [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _f],
    "tx_layernorm_bwd": [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i32, _i32],
    "tx_batchnorm_fwd": [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _f],
    "tx_batchnorm_bwd": [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _f, _i32, _i32],
    "tx_groupnorm_fwd": [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _f],
    "tx_groupnorm_bwd": [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i32, _i32],
    "tx_prelu_fwd": [_vp, _vp, _vp, _p64, _vp, _p64, _i32],
    "tx_prelu_bwd": [_vp, _vp, _vp, _p64, _vp, _vp, _vp, _p64, _i32, _i32],
    "tx_maxpool2d_fwd": [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _p64],
    "tx_maxpool2d_bwd": [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _p64, _i32],
    "tx_avgpool2d_fwd": [_vp, _vp, _vp, _i64, _i64, _i64, _p64, _i32],
    "tx_avgpool2d_bwd": [_vp, _vp, _vp, _i64, _i64, _i64, _p64, _i32, _i32],
    "tx_attention_fwd": [_vp, _vp, _vp, _vp, _i64, _vp, _i64, _i64, _i64, _i64, _i64, _f, _i32],
    "tx_attention_bwd": [_vp, _vp, _vp, _vp, _i64, _vp, _i64, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64,
                         _f, _i32],
    "tx_ppo_loss_fwd": [_vp, _vp, _i64, _i64, _vp, _vp, _vp, _vp, _vp, _f, _f, _f, _vp],
    "tx_ppo_loss_bwd": [_vp, _vp, _i64, _i64, _vp, _vp, _vp, _vp, _vp, _f, _f, _f, _vp, _vp, _vp, _i32,
                        _i32],
    "tx_gather_rows": [_vp, _vp, _i64, _i64, _vp, _i64, _vp],
    "tx_scatter_add_rows": [_vp, _vp, _i64, _i64, _vp, _i64, _vp],
    "tx_take_last": [_vp, _vp, _vp, _vp, _i64, _i64],
    "tx_take_last_bwd": [_vp, _vp, _vp, _vp, _i64, _i64, _i32],
    "tx_bias_grad": [_vp, _vp, _vp, _i64, _i64, _f, _i32],
    "tx_round_tf32": [_vp, _vp, _vp, _i64],
    "tx_split_tf32": [_vp, _vp, _vp, _vp, _i64],
    "tx_optim_create": [_vp, C.POINTER(OptimCfg), _i32, C.POINTER(_vp), C.POINTER(_vp), _p64,
                        C.POINTER(_vp)],
    "tx_optim_set_lr": [_vp, C.c_double],
    "tx_optim_set_hparams": [_vp, C.POINTER(OptimCfg)],
    "tx_optim_step": [_vp, C.POINTER(C.c_uint8)],
    "tx_optim_state_ptr": [_vp, _i32, _i32, C.POINTER(_vp)],
    "tx_optim_get_steps": [_vp, _p64],
    "tx_optim_set_steps": [_vp, _p64],
    "tx_optim_destroy": [_vp],
    "tx_graph_value_ptr": [_vp, _i32, C.POINTER(_vp)],
    "tx_graph_create": [_vp, C.POINTER(ValueDesc), _i32, C.POINTER(NodeDesc), _i32, _p32, _i32,
                        C.POINTER(_vp)],
    "tx_graph_destroy": [_vp],
    "tx_graph_param_count": [_vp, C.POINTER(C.c_int)],
    "tx_graph_param": [_vp, _i32, _p32, C.POINTER(_vp), C.POINTER(_vp), _p64],
    "tx_graph_grad_defined": [_vp, _i32, C.POINTER(C.c_int)],
    "tx_graph_set_grad_defined": [_vp, _i32, _i32],
    "tx_graph_infer": [_vp, _p64, _p32, _p64, _p32],
    "tx_graph_forward": [_vp, C.POINTER(_vp), _p64, _p32, C.POINTER(_vp), _i32, C.POINTER(_vp)],
    "tx_graph_backward": [_vp, _vp, C.POINTER(_vp), C.POINTER(_vp)],
    "tx_record_free": [_vp],
    "tx_dp_unique_id": [C.POINTER(C.c_uint8)],
    "tx_dp_init": [_vp, _i32, _i32, C.POINTER(C.c_uint8), C.c_uint64],
    "tx_dp_destroy": [_vp],
    "tx_graph_set_dp": [_vp, _i32, _i64],
    "tx_dp_allreduce": [_vp, _vp, _i64, _i32],
}


def _load() -> C.CDLL:
    if not _LIB_PATH.exists():
        raise ImportError(
            f"{_LIB_PATH} is missing: build it with `python -m tynx_b200.build` "
            "(the CUDA engine has no CPU fallback)"
        )
    lib = C.CDLL(str(_LIB_PATH), mode=os.RTLD_NOW | os.RTLD_GLOBAL)
    for name, argtypes in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = argtypes
        fn.restype = C.c_int
    return lib


lib = _load()

_EXC = {
    TX_ERR_INVALID: ValueError,
    TX_ERR_SHAPE: ValueError,
    TX_ERR_INDEX: IndexError,
    TX_ERR_OOM: MemoryError,
    TX_ERR_CUDA: RuntimeError,
    TX_ERR_TIMEOUT: DeviceTimeoutError,
    TX_ERR_UNSUPPORTED: NotImplementedError,
    TX_ERR_DEVICE: RuntimeError,
    TX_ERR_NCCL: RuntimeError,
    TX_ERR_CAPTURE: CaptureError,
}


def raise_for(code: int, ctx=None, what: str = "") -> None:
    if code == TX_OK:
        return
    message = ""
    if ctx is not None:
        buf = C.create_string_buffer(1024)
        latched = lib.tx_last_error(ctx, buf, 1024)
        message = buf.value.decode("utf-8", "replace")
        if latched and latched != code and not message:
            code = latched
    exc = _EXC.get(code, RuntimeError)
    text = message or f"tynx_cuda error {code}"
    if what:
        text = f"{what}: {text}"
    raise exc(text)


def check(code: int, ctx=None, what: str = "") -> None:
    if code != TX_OK:
        raise_for(code, ctx, what)


def i64_array(values) -> C.Array:
    values = list(values)
    return (C.c_int64 * max(len(values), 1))(*values)


def i32_array(values) -> C.Array:
    values = list(values)
    return (C.c_int32 * max(len(values), 1))(*values)


def ptr_array(values) -> C.Array:
    values = list(values)
    return (C.c_void_p * max(len(values), 1))(*values)


def device_count() -> int:
    n = C.c_int(0)
    lib.tx_device_count(C.byref(n))
    return n.value


def exported_symbols() -> list[str]:
    return sorted(SIGNATURES)
