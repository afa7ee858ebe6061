"""GGUF tensor-view loader: an unmodified ``.gguf`` file's tensors as device tensors the ops consume.

Host mirror of include/gguf_file.h.  The file is mapped and parsed by the native library (header,
metadata, tensor infos, with gguf-py 0.19.0 GGUFReader's accept / reject rules); tensor bytes go
to device memory through pinned staging buffers, whole or as a row range (one rank's shard of an
LM head, one expert of a stacked MoE tensor).  Each tensor is exposed in the default ONNX view of
docs/GGUF_ONNX_Custom_Ops.md:11-18: plain types (F32, F16, BF16, F64, I8..I64) as their element
type with the GGUF dims reversed; block-quantised types (Q8_0, IQ2_XXS, NVFP4, ...) as UINT8
``[..., (K / block) * type_size]`` -- exactly the ``w`` inputs of Q8Gemv / Q4Gemv / Nvfp4Gemv /
MoeVerify / Q8Embed.  This stands in for ONNX Runtime GenAI's ``gguf_initializers`` (the
reference's docs/GGUF_ONNX_Custom_Ops.md:5-7) for users outside ONNX Runtime.

    with GGUFFile("model.gguf") as f:
        emb = f.load("token_embd.weight", device="cuda")        # uint8 [vocab, (K/32)*34]
        y = ops.Q8Embed(emb, ids)
"""

from __future__ import annotations

import ctypes
from typing import NamedTuple

import numpy as np
import torch

from . import _lib
from ._lib import check, load

# ggml type id -> (name, torch dtype of the plain view or None for block-quantised bytes)
_PLAIN = {0: torch.float32, 1: torch.float16, 24: torch.int8, 25: torch.int16, 26: torch.int32, 27: torch.int64,
          28: torch.float64, 30: torch.bfloat16}
TYPE_NAMES = {0: "F32", 1: "F16", 2: "Q4_0", 3: "Q4_1", 6: "Q5_0", 7: "Q5_1", 8: "Q8_0", 9: "Q8_1", 10: "Q2_K",
              11: "Q3_K", 12: "Q4_K", 13: "Q5_K", 14: "Q6_K", 15: "Q8_K", 16: "IQ2_XXS", 17: "IQ2_XS", 18: "IQ3_XXS",
              19: "IQ1_S", 20: "IQ4_NL", 21: "IQ3_S", 22: "IQ2_S", 23: "IQ4_XS", 24: "I8", 25: "I16", 26: "I32",
              27: "I64", 28: "F64", 29: "IQ1_M", 30: "BF16", 34: "TQ1_0", 35: "TQ2_0", 39: "MXFP4", 40: "NVFP4",
              41: "Q1_0"}

# GGUF metadata value types (include/gguf_file.h GGUF_VAL_*) -> numpy scalar types
_VAL_NP = {0: np.uint8, 1: np.int8, 2: np.uint16, 3: np.int16, 4: np.uint32, 5: np.int32, 6: np.float32,
           7: np.bool_, 10: np.uint64, 11: np.int64, 12: np.float64}
VAL_STRING, VAL_ARRAY = 8, 9


class GGUFTensor(NamedTuple):
    index: int
    name: str
    type: int
    dims: tuple          # GGUF order: dims[0] innermost
    offset: int          # byte offset in the file
    nbytes: int
    block_elems: int
    block_bytes: int
    row_bytes: int

    @property
    def type_name(self) -> str:
        return TYPE_NAMES.get(self.type, str(self.type))

    @property
    def n_elements(self) -> int:
        return int(np.prod(self.dims))

    @property
    def rows(self) -> int:
        """Number of dims[0] rows (product of the outer dims)."""
        return int(np.prod(self.dims[1:])) if len(self.dims) > 1 else 1

    def onnx_view(self) -> tuple[torch.dtype, tuple]:
        """(dtype, shape) of the default ONNX view (docs/GGUF_ONNX_Custom_Ops.md:11-18)."""
        outer = tuple(reversed(self.dims[1:]))
        if self.type in _PLAIN:
            return _PLAIN[self.type], outer + (self.dims[0],)
        return torch.uint8, outer + (self.row_bytes,)


def _tensor_from(info: _lib.GgufTensorInfo, i: int) -> GGUFTensor:
    return GGUFTensor(i, info.name.decode("utf-8"), int(info.type), tuple(int(d) for d in info.dims[: info.n_dims]),
                      int(info.offset), int(info.nbytes), int(info.block_elems), int(info.block_bytes),
                      int(info.row_bytes))


def _walk_value(buf: memoryview, pos: int, t: int, out: list) -> int:
    """Decodes one value of type t starting at buf[pos]; appends it (arrays flattened, as
    GGUFReader's ReaderField.contents() does) and returns the next position."""
    if t in _VAL_NP:
        dt = np.dtype(_VAL_NP[t]).newbyteorder("<")
        out.append(np.frombuffer(buf, dt, 1, pos).tolist()[0])
        return pos + dt.itemsize
    if t == VAL_STRING:
        n = int(np.frombuffer(buf, "<u8", 1, pos)[0])
        out.append(bytes(buf[pos + 8: pos + 8 + n]).decode("utf-8"))
        return pos + 8 + n
    if t == VAL_ARRAY:
        et = int(np.frombuffer(buf, "<u4", 1, pos)[0])
        n = int(np.frombuffer(buf, "<u8", 1, pos + 4)[0])
        pos += 12
        if et in _VAL_NP:
            dt = np.dtype(_VAL_NP[et]).newbyteorder("<")
            out.extend(np.frombuffer(buf, dt, n, pos).tolist())
            return pos + n * dt.itemsize
        for _ in range(n):
            pos = _walk_value(buf, pos, et, out)
        return pos
    raise ValueError(f"GGUF: unknown metadata value type {t}")


class GGUFFile:
    """A parsed, mapped ``.gguf`` file.  ``tensors`` and ``metadata`` keep the file's order."""

    def __init__(self, path: str):
        lib = load()
        h = ctypes.c_void_p()
        check(lib.gguf_file_open(str(path).encode(), ctypes.byref(h)))
        self._h = h
        self.path = str(path)
        v, a, d, sz = ctypes.c_int32(), ctypes.c_int64(), ctypes.c_int64(), ctypes.c_int64()
        check(lib.gguf_file_header(h, ctypes.byref(v), ctypes.byref(a), ctypes.byref(d), ctypes.byref(sz)))
        self.version, self.alignment, self.data_offset, self.file_size = v.value, a.value, d.value, sz.value
        base = lib.gguf_file_data(h)
        self._buf = memoryview((ctypes.c_uint8 * self.file_size).from_address(base)).cast("B")
        self.tensors: dict[str, GGUFTensor] = {}
        info = _lib.GgufTensorInfo()
        for i in range(lib.gguf_file_tensor_count(h)):
            check(lib.gguf_file_tensor_info(h, i, ctypes.byref(info)))
            t = _tensor_from(info, i)
            self.tensors[t.name] = t
        self._kv_raw: dict[str, tuple[int, int, int]] = {}  # key -> (type, offset of the value, elem type)
        kv = _lib.GgufKv()
        for i in range(lib.gguf_file_kv_count(h)):
            check(lib.gguf_file_kv(h, i, ctypes.byref(kv)))
            hdr = 8 if kv.type == VAL_STRING else 12 if kv.type == VAL_ARRAY else 0
            self._kv_raw[kv.key.decode("utf-8")] = (int(kv.type), int(kv.data) - base - hdr, int(kv.elem_type))
        self._metadata: dict | None = None

    # ---- metadata ----
    @property
    def metadata(self) -> dict:
        """key -> value: scalars as Python numbers / bools, strings as str, arrays as flat lists."""
        if self._metadata is None:
            md = {}
            for k, (t, pos, _) in self._kv_raw.items():
                out: list = []
                _walk_value(self._buf, pos, t, out)
                md[k] = out if t == VAL_ARRAY else out[0]
            self._metadata = md
        return self._metadata

    def value_type(self, key: str) -> tuple[int, int]:
        """(GGUF value type, array element type or -1) of a metadata key."""
        t, _, et = self._kv_raw[key]
        return t, et

    # ---- tensors ----
    def __getitem__(self, name: str) -> GGUFTensor:
        return self.tensors[name]

    def __contains__(self, name: str) -> bool:
        return name in self.tensors

    def host_bytes(self, name: str) -> np.ndarray:
        """Zero-copy uint8 view of the tensor's bytes in the mapping, shaped [rows, row_bytes]."""
        t = self.tensors[name]
        return np.frombuffer(self._buf, np.uint8, t.nbytes, t.offset).reshape(t.rows, t.row_bytes)

    def load(self, name: str, device=None, rows: tuple[int, int] | None = None,
             out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
        """Copies a tensor (or rows [r0, r1) of its [rows, row] view) to device memory in the
        default ONNX view; a row range keeps the inner dim and flattens the outer ones."""
        t = self.tensors[name]
        dtype, shape = t.onnx_view()
        r0, r1 = (0, t.rows) if rows is None else rows
        if not 0 <= r0 <= r1 <= t.rows:
            raise ValueError(f"{name}: row range [{r0}, {r1}) outside [0, {t.rows})")
        if rows is not None:
            shape = (r1 - r0, shape[-1])
        nbytes = (r1 - r0) * t.row_bytes
        if out is None:
            dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
            out = torch.empty(shape, dtype=dtype, device=dev)
        elif out.dtype != dtype or tuple(out.shape) != tuple(shape) or not out.is_contiguous():
            raise ValueError(f"{name}: out must be a contiguous {dtype} tensor of shape {tuple(shape)}")
        self._upload([(t.index, r0 * t.row_bytes, nbytes, out.data_ptr())], out.device, stream)
        return out

    def load_many(self, names, device=None, stream=None) -> dict[str, torch.Tensor]:
        """Copies several whole tensors in one staged pass."""
        dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        outs = {}
        items = []
        for n in names:
            t = self.tensors[n]
            dtype, shape = t.onnx_view()
            outs[n] = torch.empty(shape, dtype=dtype, device=dev)
            items.append((t.index, 0, t.nbytes, outs[n].data_ptr()))
        self._upload(items, dev, stream)
        return outs

    def _upload(self, items, device, stream):
        if device.type != "cuda":
            raise ValueError("GGUFFile.load copies into CUDA device memory (use host_bytes for a host view)")
        arr = (_lib.GgufUploadItem * max(1, len(items)))()
        for i, (ti, off, nb, dst) in enumerate(items):
            arr[i].tensor, arr[i].byte_offset, arr[i].nbytes, arr[i].dst = ti, off, nb, dst
        with torch.cuda.device(device):
            s = stream if stream is not None else torch.cuda.current_stream()
            check(load().gguf_file_upload(self._h, arr, len(items), ctypes.c_void_p(s.cuda_stream)))

    # ---- lifetime ----
    def close(self) -> None:
        if getattr(self, "_h", None) is not None and self._h.value:
            self._buf = None
            load().gguf_file_close(self._h)
            self._h = ctypes.c_void_p()

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def type_size(type_id: int) -> tuple[int, int]:
    """(block elements, bytes per block) of a ggml type id, from the native table."""
    b, n = ctypes.c_int64(), ctypes.c_int64()
    check(load().gguf_type_size(type_id, ctypes.byref(b), ctypes.byref(n)))
    return b.value, n.value
