"""gguf_onnx_ops_b200: B200-native (sm_100a) decode-time GGUF GEMV / MoE hot path of
tianleiwu/gguf_onnx_ops, as a drop-in libgguf_onnx_ops.so (C ABI in include/gguf_ops.h) plus a
host-side mirror of the reference's custom-op interface (``ops``)."""

from . import _lib  # noqa: F401
from ._lib import LIB_PATH, GgufOpsError, load  # noqa: F401
from .ops import (  # noqa: F401
    MoeRouteGGUF, MoeVerify, Nvfp4Gemv, Q4Gemv, Q8Gemv, dequantize, device_status, set_pdl,
)

__all__ = ["Q8Gemv", "Q4Gemv", "Nvfp4Gemv", "MoeRouteGGUF", "MoeVerify", "dequantize", "load", "LIB_PATH",
           "GgufOpsError", "set_pdl", "device_status"]
