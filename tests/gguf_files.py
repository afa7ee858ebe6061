"""GGUF test files written with gguf-py 0.19.0's GGUFWriter (the writer of the GGUF ecosystem; the
reader side under test is the repo's native parser, checked against gguf-py's GGUFReader)."""

from __future__ import annotations

import struct

import numpy as np

from oracle import inputs as I


def write_model_file(path, seed: int = 0, alignment: int | None = None):
    """A small model-shaped file: every metadata value type, and tensors of the path's formats
    (Q8_0 LM head + embedding, IQ2_XXS expert stack, NVFP4, F32 / F16 / BF16 / I32 plain tensors).
    Returns {name: raw bytes [rows, row_bytes] as written}."""
    from gguf import GGMLQuantizationType as Q
    from gguf import GGUFWriter

    g = I.rng(seed)
    w = GGUFWriter(str(path), "test")
    if alignment is not None:
        w.add_custom_alignment(alignment)
    w.add_uint8("t.u8", 7)
    w.add_int8("t.i8", -3)
    w.add_uint16("t.u16", 65000)
    w.add_int16("t.i16", -300)
    w.add_uint32("t.u32", 4000000000)
    w.add_int32("t.i32", -5)
    w.add_float32("t.f32", 1.5)
    w.add_bool("t.bool", True)
    w.add_string("t.str", "héllo")
    w.add_uint64("t.u64", 2 ** 63)
    w.add_int64("t.i64", -2 ** 40)
    w.add_float64("t.f64", 3.25)
    w.add_array("t.arr_i32", [1, 2, 3])
    w.add_array("t.arr_str", ["x", "yy", "", "ü"])
    w.add_array("t.arr_f32", [1.5, 2.5])
    w.add_array("t.arr_bool", [True, False, True])
    w.add_array("t.arr_nested", [[1, 2], [3]])
    w.add_array("t.arr_empty", [])
    raw = {}
    raw["token_embd.weight"] = I.q8_test_blocks(g, 96, 512)                  # Q8_0 [96, 512]
    raw["output.weight"] = I.q8_0_weights(g, 80, 1024)                        # Q8_0 LM head [80, 1024]
    raw["blk.0.ffn_up_exps.weight"] = I.iq2_test_blocks(g, (4, 64), 512).reshape(4 * 64, -1)  # IQ2 [4, 64, 512]
    raw["blk.0.nvfp4.weight"] = I.nvfp4_weights(g, 48, 640)                    # NVFP4 [48, 640]
    f32 = g.standard_normal((3, 5)).astype(np.float32)
    f16 = g.standard_normal((7,)).astype(np.float16)
    bf16 = g.integers(0, 65536, size=(2, 4), dtype=np.uint16)
    i32 = np.arange(-4, 4, dtype=np.int32).reshape(2, 4)
    w.add_tensor("token_embd.weight", raw["token_embd.weight"], raw_dtype=Q.Q8_0)
    w.add_tensor("output.weight", raw["output.weight"], raw_dtype=Q.Q8_0)
    w.add_tensor("blk.0.ffn_up_exps.weight", raw["blk.0.ffn_up_exps.weight"].reshape(4, 64, -1), raw_dtype=Q.IQ2_XXS)
    w.add_tensor("blk.0.nvfp4.weight", raw["blk.0.nvfp4.weight"], raw_dtype=Q.NVFP4)
    w.add_tensor("f32", f32)
    w.add_tensor("f16", f16)
    w.add_tensor("bf16", bf16.view(np.uint8), raw_dtype=Q.BF16)
    w.add_tensor("i32", i32)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    raw["f32"] = f32.view(np.uint8).reshape(3, -1)
    raw["f16"] = f16.view(np.uint8).reshape(1, -1)
    raw["bf16"] = bf16.view(np.uint8).reshape(2, -1)
    raw["i32"] = i32.view(np.uint8).reshape(2, -1)
    return raw


def gguf_string(s: bytes) -> bytes:
    return struct.pack("<Q", len(s)) + s


def handmade(version=3, kvs=(), tensors=(), alignment_pad=32, data=b"", magic=b"GGUF"):
    """Builds a GGUF file byte by byte (for malformed cases the writer refuses to make).
    kvs: (key bytes, type id, payload bytes); tensors: (name bytes, dims, type id, offset)."""
    out = bytearray(magic + struct.pack("<IQQ", version, len(tensors), len(kvs)))
    for k, t, payload in kvs:
        out += gguf_string(k) + struct.pack("<I", t) + payload
    for name, dims, t, off in tensors:
        out += gguf_string(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims)
        out += struct.pack("<IQ", t, off)
    out += b"\0" * ((-len(out)) % alignment_pad)
    return bytes(out + data)
