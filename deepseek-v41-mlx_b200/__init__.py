"""B200-native (sm_100a) quantized-weight hot path of the DeepSeek-V4.1-Flash runtime.

Drop-in replacements for the reference's ``deepseek_v41_mlx.dequant``,
``deepseek_v41_mlx.moe`` and ``deepseek_v41_mlx.engram`` entry points, backed
by the C-ABI library ``libdsv41q.so`` built from ``csrc/`` (see ``build.py``).
Arrays are torch CUDA tensors; anything exposing ``__dlpack__`` is accepted
and converted with ``torch.from_dlpack``.  There is no CPU fallback: every
compute call raises if the CUDA library or a CUDA device is missing.
"""

from __future__ import annotations

from . import _lib  # noqa: F401
from ._lib import DSV41Error, lib_path  # noqa: F401

__all__ = ["dequant", "moe", "engram", "linear", "act_quant", "gemm", "ep", "release", "convert",
           "DSV41Error", "lib_path"]


def __getattr__(name):
    # submodules load lazily so that importing the package never touches CUDA
    if name in ("dequant", "moe", "engram", "linear", "act_quant", "gemm", "ep", "release",
                "convert"):
        import importlib
        return importlib.import_module(f"{__name__}.{name}")
    raise AttributeError(name)
