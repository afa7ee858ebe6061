"""ctypes binding of libgguf_onnx_ops.so (the C ABI declared in include/gguf_ops.h).

The shared library is the product; this module only loads it and declares the entry points.
There is no CPU or PyTorch fallback: if the library cannot be loaded, every op raises.
"""

from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "lib", "libgguf_onnx_ops.so")

GGUF_OK = 0
GGUF_ERR_INVALID_ARGUMENT = 1
GGUF_ERR_CUDA = 2
GGUF_ERR_NOT_IMPLEMENTED = 3
GGUF_ERR_DEVICE = 4
GGUF_ERR_IO = 5

GGUF_TYPE_Q8_0 = 8
GGUF_TYPE_IQ2_XXS = 16
GGUF_TYPE_NVFP4 = 40

# legacy split layouts (include/gguf_ops.h GGUF_LAYOUT_*)
GGUF_LAYOUT_Q8_SPLIT, GGUF_LAYOUT_Q4_SPLIT, GGUF_LAYOUT_IQ2_CODES, GGUF_LAYOUT_IQ2_NATIVE, GGUF_LAYOUT_NVFP4_SPLIT = range(5)

# name -> (restype, argtypes); mirrors include/gguf_ops.h
_P, _I64, _I32, _F32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_float
SIGNATURES = {
    "gguf_version": (ctypes.c_char_p, []),
    "gguf_last_error": (ctypes.c_char_p, []),
    "gguf_q8_0_gemv": (_I32, [_P, _P, _P, _I64, _I64, _I64, _P]),
    "gguf_iq2_xxs_gemv": (_I32, [_P, _P, _P, _I64, _I64, _I64, _P]),
    "gguf_nvfp4_gemv": (_I32, [_P, _P, _P, _P, _I64, _I64, _I64, _P]),
    "gguf_gemv_legacy": (_I32, [_I32, _P, _P, _P, _P, _P, _I64, _I64, _I64, _P]),
    "gguf_moe_legacy": (_I32, [_I32] + [_P] * 11 + [_I64, _I64, _I64, _I64, _P]),
    "gguf_mamba_step": (_I32, [_P] * 5 + [_I32] + [_P] * 10 + [_I64] * 6 + [_F32, _F32, _P]),
    "gguf_q8_0_embed": (_I32, [_P, _P, _P, _I64, _I64, _I64, _P]),
    "gguf_rms_norm": (_I32, [_P, _P, _P, _P, _P, _I64, _I64, _F32, _P]),
    "gguf_rms_norm_iq2_xxs_gemv": (_I32, [_P, _P, _P, _F32, _P, _P, _P, _P, _I64, _I64, _P]),
    "gguf_moe_route": (_I32, [_P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _F32, _P]),
    "gguf_moe_route_bf16": (_I32, [_P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _F32, _P]),
    "gguf_relu2": (_I32, [_P, _P, _I64, _P]),
    "gguf_moe_verify_iq2_xxs": (_I32, [_P, _P, _P, _P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _P]),
    "gguf_moe_verify_iq2_xxs_noalloc": (_I32, [_P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _P]),
    "gguf_gemv_rowsplit": (_I32, [_I32, _P, _P, _P, _P, _I64, _I64, _I64, _P]),
    "gguf_moe_verify_iq2_xxs_ep": (_I32, [_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _P]),
    "gguf_ipc_get_handle": (_I32, [_P, _P, ctypes.POINTER(ctypes.c_int64)]),
    "gguf_ipc_open": (_I32, [_P, ctypes.POINTER(ctypes.c_void_p)]),
    "gguf_ipc_close": (_I32, [_P]),
    "gguf_dequantize": (_I32, [_I32, _P, _P, _I64, _I64, _P]),
    "gguf_device_status": (_I32, [ctypes.POINTER(ctypes.c_int)]),
    "gguf_set_pdl": (None, [_I32]),
    "gguf_set_fast_paths": (None, [_I32]),
    # include/gguf_file.h
    "gguf_file_open": (_I32, [ctypes.c_char_p, ctypes.POINTER(ctypes.c_void_p)]),
    "gguf_file_close": (None, [_P]),
    "gguf_file_header": (_I32, [_P, ctypes.POINTER(ctypes.c_int32), ctypes.POINTER(ctypes.c_int64),
                                ctypes.POINTER(ctypes.c_int64), ctypes.POINTER(ctypes.c_int64)]),
    "gguf_file_data": (_P, [_P]),
    "gguf_file_tensor_count": (_I64, [_P]),
    "gguf_file_tensor_info": (_I32, [_P, _I64, _P]),
    "gguf_file_find_tensor": (_I64, [_P, ctypes.c_char_p]),
    "gguf_file_kv_count": (_I64, [_P]),
    "gguf_file_kv": (_I32, [_P, _I64, _P]),
    "gguf_file_find_kv": (_I64, [_P, ctypes.c_char_p]),
    "gguf_type_size": (_I32, [ctypes.c_int32, ctypes.POINTER(ctypes.c_int64), ctypes.POINTER(ctypes.c_int64)]),
    "gguf_file_upload": (_I32, [_P, _P, _I64, _P]),
}


class GgufTensorInfo(ctypes.Structure):
    """Mirror of GgufTensorInfo (include/gguf_file.h)."""

    _fields_ = [("name", ctypes.c_char_p), ("type", ctypes.c_int32), ("n_dims", ctypes.c_int32),
                ("dims", ctypes.c_int64 * 4), ("offset", ctypes.c_int64), ("nbytes", ctypes.c_int64),
                ("block_elems", ctypes.c_int64), ("block_bytes", ctypes.c_int64), ("row_bytes", ctypes.c_int64)]


class GgufKv(ctypes.Structure):
    """Mirror of GgufKv (include/gguf_file.h)."""

    _fields_ = [("key", ctypes.c_char_p), ("type", ctypes.c_int32), ("elem_type", ctypes.c_int32),
                ("count", ctypes.c_int64), ("data", ctypes.c_void_p), ("nbytes", ctypes.c_int64)]


class GgufUploadItem(ctypes.Structure):
    """Mirror of GgufUploadItem (include/gguf_file.h)."""

    _fields_ = [("tensor", ctypes.c_int64), ("byte_offset", ctypes.c_int64), ("nbytes", ctypes.c_int64),
                ("dst", ctypes.c_void_p)]


class GgufPeerOut(ctypes.Structure):
    """Mirror of GgufPeerOut (include/gguf_ops.h)."""

    _fields_ = [("stage", (ctypes.c_void_p * 8) * 2), ("y", ctypes.c_void_p), ("state", ctypes.c_void_p),
                ("world", ctypes.c_int), ("rank", ctypes.c_int), ("n_total", ctypes.c_int64), ("row0", ctypes.c_int64),
                ("ctas", ctypes.c_int32), ("r_max", ctypes.c_int32)]


class GgufPeerReduce(ctypes.Structure):
    """Mirror of GgufPeerReduce (include/gguf_ops.h)."""

    _fields_ = [("slots", ctypes.c_void_p * 8), ("flags", ctypes.c_void_p * 8), ("state", ctypes.c_void_p),
                ("world", ctypes.c_int), ("rank", ctypes.c_int), ("r_max", ctypes.c_int64)]


class GgufOpsError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(msg)
        self.code = code


_lib = None


def load(path: str | None = None) -> ctypes.CDLL:
    """Load the library once (raises OSError with a clear message if it has not been built)."""
    global _lib
    if _lib is None:
        p = path or os.environ.get("GGUF_OPS_LIB", LIB_PATH)
        if not os.path.exists(p):
            raise OSError(f"{p} not found: build it with `python -m gguf_onnx_ops_b200.build` "
                          "(there is no CPU fallback)")
        lib = ctypes.CDLL(p)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def check(rc: int) -> None:
    if rc != GGUF_OK:
        msg = load().gguf_last_error().decode("utf-8", "replace")
        if rc == GGUF_ERR_INVALID_ARGUMENT:
            raise ValueError(msg)
        if rc == GGUF_ERR_NOT_IMPLEMENTED:
            raise NotImplementedError(msg)
        if rc == GGUF_ERR_IO:
            raise OSError(msg)
        raise GgufOpsError(rc, msg)


def device_status() -> tuple[int, int]:
    """(status, site) of kernel-side bounded waits on the current device; synchronises."""
    site = ctypes.c_int(0)
    rc = load().gguf_device_status(ctypes.byref(site))
    return rc, site.value
