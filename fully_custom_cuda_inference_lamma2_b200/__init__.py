"""B200-native (sm_100a) varlen decode-attention path.

Drop-in for the decode-attention path of divakar-yadav/Fully_Custom_Cuda_Inference_Lamma2:
the pybind modules `attn_varlen` and `capture_decode_step` carry the reference's
names and signatures (custom_kernels/attn_varlen.cpp:47-49,
custom_kernels/capture_decode_step.cpp:312-325) and launch the hand-written
kernels of libfcci_decode.so. A server that imports the modules by name from
sys.path (case4_graph_generator_server_ipc.py:26-71) picks them up after
``sys.path.insert(0, dropin_path())``.

The native build is required: importing this package without it raises
ImportError; there is no CPU fallback.
"""
from __future__ import annotations

import os

import torch  # noqa: F401  (loads libc10/libtorch for the extension modules)

_PKG = os.path.dirname(os.path.abspath(__file__))


def dropin_path() -> str:
    """Directory holding the `attn_varlen` / `capture_decode_step` modules."""
    return _PKG


def library_path() -> str:
    """Path of the C-ABI library libfcci_decode.so."""
    return os.path.join(_PKG, "libfcci_decode.so")


try:
    from . import attn_varlen, capture_decode_step  # noqa: E402
except ImportError as exc:  # pragma: no cover - exercised only when unbuilt
    raise ImportError(
        "fully_custom_cuda_inference_lamma2_b200: native modules are not built; run "
        "`python fully_custom_cuda_inference_lamma2_b200/build.py`"
    ) from exc

from .arena import KVArena, decode_attention  # noqa: E402
from . import sharding  # noqa: E402

__all__ = [
    "attn_varlen",
    "capture_decode_step",
    "KVArena",
    "decode_attention",
    "sharding",
    "dropin_path",
    "library_path",
]
