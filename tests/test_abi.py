"""The C-ABI library: it loads, exports every symbol include/gguf_ops.h declares, and rejects bad
arguments with the reference's error style -- all without touching a GPU."""

import ctypes
import os
import re

import pytest

from gguf_onnx_ops_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADERS = [os.path.join(ROOT, "include", h) for h in sorted(os.listdir(os.path.join(ROOT, "include")))
           if h.endswith(".h")]


def declared():
    src = "".join(open(h).read() for h in HEADERS)
    return re.findall(r"GGUF_OPS_API\s+[\w\s\*]+?\b(gguf_\w+)\s*\(", src)


def test_header_declares_the_hot_path():
    names = set(declared())
    for n in ("gguf_q8_0_gemv", "gguf_iq2_xxs_gemv", "gguf_nvfp4_gemv", "gguf_moe_route", "gguf_moe_verify_iq2_xxs",
              "gguf_dequantize", "gguf_last_error", "gguf_device_status", "gguf_q8_0_embed", "gguf_file_open",
              "gguf_file_upload"):
        assert n in names


def test_library_exports_every_declared_symbol(lib):
    for n in declared():
        assert hasattr(lib, n), n
        assert n in _lib.SIGNATURES, f"{n} has no ctypes signature"


def declared_arg_counts():
    """name -> number of parameters, from the prototypes in include/*.h."""
    src = "".join(open(h).read() for h in HEADERS)
    out = {}
    for m in re.finditer(r"GGUF_OPS_API\s+[\w\s\*]+?\b(gguf_\w+)\s*\(([^)]*)\)", src):
        args = m.group(2).strip()
        out[m.group(1)] = 0 if args in ("", "void") else args.count(",") + 1
    return out


def test_ctypes_signatures_match_header_arity():
    for name, n in declared_arg_counts().items():
        assert len(_lib.SIGNATURES[name][1]) == n, f"{name}: header has {n} parameters"


def test_version(lib):
    assert b"sm_100a" in lib.gguf_version()


FAKE = 0x10000  # 16-byte aligned, never dereferenced: validation fails before any CUDA call


@pytest.mark.parametrize("fn,args,msg", [
    ("gguf_q8_0_gemv", (FAKE, FAKE, FAKE, 17, 4096, 4096, None), "Q8Gemv gguf=1"),
    ("gguf_q8_0_gemv", (FAKE, FAKE, FAKE, 0, 4096, 4096, None), "1..16 rows"),
    ("gguf_q8_0_gemv", (FAKE, FAKE, FAKE, 1, 4096, 4000, None), "K % 64"),
    ("gguf_q8_0_gemv", (FAKE + 2, FAKE, FAKE, 1, 4096, 4096, None), "aligned"),
    ("gguf_q8_0_gemv", (None, FAKE, FAKE, 1, 4096, 4096, None), "null"),
    ("gguf_iq2_xxs_gemv", (FAKE, FAKE, FAKE, 1, 14336, 4000, None), "Q4Gemv iq2=3"),
    ("gguf_iq2_xxs_gemv", (FAKE, FAKE, FAKE, 99, 14336, 4096, None), "1..16 rows"),
    ("gguf_nvfp4_gemv", (FAKE, FAKE, None, FAKE, 1, 1024, 5120, None), "Nvfp4Gemv gguf=1"),
    ("gguf_nvfp4_gemv", (FAKE, FAKE, FAKE, FAKE, 1, 1024, 5000, None), "K % 64"),
    ("gguf_moe_route", (FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, 8, 1024, 513, 6, 1.0, None), "MoeRoute"),
    ("gguf_moe_route", (FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, 8, 1000, 128, 6, 1.0, None), "K % 256"),
    ("gguf_moe_route", (FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, 8, 1024, 128, 33, 1.0, None), "topk"),
    ("gguf_moe_verify_iq2_xxs", (FAKE,) * 9 + (9, 128, 1792, 6, None), "rows must be in [1,8]"),
    ("gguf_moe_verify_iq2_xxs", (FAKE,) * 9 + (8, 128, 1792, 17, None), "rows*topk <= 128"),
    ("gguf_moe_verify_iq2_xxs", (FAKE,) * 9 + (8, 128, 1800, 6, None), "inter size"),
])
def test_invalid_arguments_rejected(lib, fn, args, msg):
    rc = getattr(lib, fn)(*args)
    assert rc == _lib.GGUF_ERR_INVALID_ARGUMENT
    assert msg in lib.gguf_last_error().decode()


def test_unknown_dequant_type(lib):
    assert lib.gguf_dequantize(2, FAKE, FAKE, 4, 64, None) == _lib.GGUF_ERR_NOT_IMPLEMENTED


def test_check_raises_typed_errors(lib):
    lib.gguf_q8_0_gemv(FAKE, FAKE, FAKE, 17, 64, 64, None)
    with pytest.raises(ValueError, match="Q8Gemv"):
        _lib.check(_lib.GGUF_ERR_INVALID_ARGUMENT)


def test_no_silent_fallback_without_gpu(lib):
    """Valid arguments on a machine without a usable GPU must fail loudly (CUDA error), never compute."""
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    rc = lib.gguf_q8_0_gemv(FAKE, FAKE, FAKE, 1, 64, 64, None)
    assert rc == _lib.GGUF_ERR_CUDA
    assert lib.gguf_last_error()


def test_ops_validate_legacy_layouts_without_gpu():
    """Legacy attribute values are implemented: shapes are checked on the host before any launch,
    and host tensors are refused."""
    import torch

    from gguf_onnx_ops_b200 import ops

    x = torch.zeros(1, 64, dtype=torch.bfloat16)
    w = torch.zeros(8, 68, dtype=torch.uint8)
    with pytest.raises(ValueError, match="CUDA tensor"):
        ops.Q8Gemv(x, w, torch.zeros(8, 2, dtype=torch.bfloat16), gguf=0)
    with pytest.raises(ValueError):
        ops.Q4Gemv(x, w, None, iq2=2)
    with pytest.raises(NotImplementedError, match="unknown iq2"):
        ops.Q4Gemv(x, w, None, iq2=5)
    with pytest.raises(ValueError, match="CUDA tensor"):
        ops.Q8Gemv(x, w)


def test_legacy_entry_rejects_bad_layouts(lib):
    rc = lib.gguf_gemv_legacy(9, FAKE, FAKE, FAKE, None, FAKE, 1, 64, 64, None)
    assert rc == _lib.GGUF_ERR_INVALID_ARGUMENT and b"unknown layout" in lib.gguf_last_error()
    rc = lib.gguf_gemv_legacy(_lib.GGUF_LAYOUT_IQ2_NATIVE, FAKE, FAKE, FAKE, None, FAKE, 1, 64, 96, None)
    assert rc == _lib.GGUF_ERR_INVALID_ARGUMENT and b"K % 256" in lib.gguf_last_error()
    rc = lib.gguf_gemv_legacy(_lib.GGUF_LAYOUT_NVFP4_SPLIT, FAKE, FAKE, FAKE, None, FAKE, 1, 64, 64, None)
    assert rc == _lib.GGUF_ERR_INVALID_ARGUMENT and b"null" in lib.gguf_last_error()
    rc = lib.gguf_gemv_legacy(_lib.GGUF_LAYOUT_Q8_SPLIT, FAKE, FAKE, FAKE, None, FAKE, 17, 64, 64, None)
    assert rc == _lib.GGUF_ERR_INVALID_ARGUMENT and b"rows" in lib.gguf_last_error()


def test_missing_library_fails_loudly(tmp_path, monkeypatch):
    monkeypatch.setattr(_lib, "_lib", None)
    with pytest.raises(OSError, match="no CPU fallback"):
        _lib.load(str(tmp_path / "nope.so"))
    monkeypatch.setattr(_lib, "_lib", None)
    ctypes.CDLL  # noqa: B018
