"""tynx_b200: B200-native training-step engine for imported ONNX graphs.

A drop-in for Tynx's imported-model training surface
(``crates/tynx-python/python/tynx/__init__.py``) on ``Device("cuda")``:
``load(..., trainable="auto")``, ``Tensor``, ``loss.backward()``,
``optim.Adam(...).step()`` and ``compile`` capture/replay.  Forward, backward and
optimizer steps run on hand-written sm_100a kernels in ``libtynx_cuda.so``.
"""

from . import distributions, nn, optim
from ._core import (
    Device,
    Prefetcher,
    Tensor,
    arange,
    cat,
    full,
    full_like,
    get_default_device,
    is_grad_enabled,
    matmul,
    maximum,
    minimum,
    no_grad,
    ones,
    ones_like,
    pinned,
    rand,
    randn,
    set_math_mode,
    synchronize,
    tensor,
    zeros,
    zeros_like,
)
from .compiler import CompiledFunction, compile
from .imported import ImportedModel, Parameter, Session, load
from .onnx.ir import TrainabilityReport

__version__ = "0.1.0"

float32 = "float32"
int64 = "int64"
bool = "bool"  # noqa: A001  (mirrors tynx.bool)

__all__ = [
    "CompiledFunction", "Device", "ImportedModel", "Parameter", "Prefetcher", "Session", "Tensor",
    "TrainabilityReport", "arange", "cat", "compile", "distributions", "full", "full_like",
    "get_default_device", "is_grad_enabled", "load", "matmul", "maximum", "minimum", "nn",
    "no_grad", "ones", "ones_like", "optim", "pinned", "rand", "randn", "set_math_mode", "synchronize",
    "tensor", "zeros", "zeros_like",
]
