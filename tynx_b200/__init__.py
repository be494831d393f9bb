"""tynx_b200: B200-native training-step engine for imported ONNX graphs.

A drop-in for Tynx's imported-model training surface
(``crates/tynx-python/python/tynx/__init__.py``) on ``Device("cuda")``:
``load(..., trainable="auto")``, ``Tensor``, ``loss.backward()``,
``optim.Adam(...).step()`` and ``compile`` capture/replay.  Forward, backward and
optimizer steps run on hand-written sm_100a kernels in ``libtynx_cuda.so``.

The public names resolve on first use (module ``__getattr__``): importing a
host-only submodule (``tynx_b200.onnx``, ``tynx_b200.workloads``) does not map
the CUDA library, while the first use of any device-facing name (``load``,
``Tensor``, ``optim`` ...) loads it and fails loudly when it is missing.
"""

from __future__ import annotations

import importlib

__version__ = "0.1.0"

float32 = "float32"
int64 = "int64"
bool = "bool"  # noqa: A001  (mirrors tynx.bool)

_FROM = {
    "._core": ("Device", "Prefetcher", "Tensor", "arange", "cat", "full", "full_like",
               "get_default_device", "is_grad_enabled", "matmul", "maximum", "minimum", "no_grad",
               "ones", "ones_like", "pinned", "rand", "randn", "set_math_mode", "synchronize",
               "tensor", "zeros", "zeros_like"),
    ".compiler": ("CompiledFunction", "compile"),
    ".imported": ("Buffer", "ImportedModel", "Parameter", "Session", "load"),
    ".checkpoint": ("save_checkpoint", "load_checkpoint"),
    ".onnx.ir": ("TrainabilityReport",),
}
_SUBMODULES = ("distributions", "nn", "optim")
_LAZY = {name: module for module, names in _FROM.items() for name in names}

__all__ = sorted(list(_LAZY) + list(_SUBMODULES))


def __getattr__(name: str):
    if name in _SUBMODULES:
        value = importlib.import_module(f".{name}", __name__)
    elif name in _LAZY:
        value = getattr(importlib.import_module(_LAZY[name], __name__), name)
    else:
        raise AttributeError(f"module {__name__!r} has no attribute {name!r}")
    globals()[name] = value
    return value


def __dir__():
    return sorted(set(globals()) | set(__all__))
