"""The native GGUF parser (include/gguf_file.h) against gguf-py 0.19.0's GGUFReader: same header,
metadata, tensor infos, data offsets and bytes; the same files rejected.  No GPU needed."""

import struct

import numpy as np
import pytest
import torch

from gguf_onnx_ops_b200.gguf_file import GGUFFile, type_size
from tests.gguf_files import gguf_string, handmade, write_model_file


@pytest.fixture(scope="module", params=[None, 64, 256])
def model_file(request, tmp_path_factory):
    p = tmp_path_factory.mktemp("gguf") / f"model_{request.param}.gguf"
    raw = write_model_file(p, seed=3, alignment=request.param)
    return p, raw


def test_header_and_tensors_match_gguf_reader(model_file):
    from gguf import GGUFReader

    p, raw = model_file
    r = GGUFReader(str(p))
    with GGUFFile(p) as f:
        assert f.version == int(r.fields["GGUF.version"].contents())
        assert f.alignment == r.alignment and f.data_offset == r.data_offset
        assert list(f.tensors) == [t.name for t in r.tensors]
        for t in r.tensors:
            mine = f[t.name]
            assert mine.type == int(t.tensor_type)
            assert mine.dims == tuple(int(d) for d in t.shape)
            assert mine.nbytes == t.n_bytes and mine.offset == t.data_offset
            assert np.array_equal(f.host_bytes(t.name).reshape(-1), np.asarray(t.data).view(np.uint8).reshape(-1))
            assert np.array_equal(f.host_bytes(t.name), raw[t.name])


def test_metadata_matches_gguf_reader(model_file):
    from gguf import GGUFReader

    p, _ = model_file
    r = GGUFReader(str(p))
    with GGUFFile(p) as f:
        expect = {k: v.contents() for k, v in r.fields.items() if not k.startswith("GGUF.")}
        assert list(f.metadata) == list(expect)
        for k, v in expect.items():
            got = f.metadata[k]
            if isinstance(v, float):
                assert got == pytest.approx(v, rel=0, abs=0), k
            else:
                assert got == v, k
            assert f.value_type(k)[0] == int(r.fields[k].types[0])


def test_onnx_views(model_file):
    p, _ = model_file
    with GGUFFile(p) as f:
        assert f["token_embd.weight"].onnx_view() == (torch.uint8, (96, 16 * 34))
        assert f["output.weight"].onnx_view() == (torch.uint8, (80, 32 * 34))
        assert f["blk.0.ffn_up_exps.weight"].onnx_view() == (torch.uint8, (4, 64, 2 * 66))
        assert f["blk.0.nvfp4.weight"].onnx_view() == (torch.uint8, (48, 10 * 36))
        assert f["f32"].onnx_view() == (torch.float32, (3, 5))
        assert f["f16"].onnx_view() == (torch.float16, (7,))
        assert f["bf16"].onnx_view() == (torch.bfloat16, (2, 4))
        assert f["i32"].onnx_view() == (torch.int32, (2, 4))
        assert f["blk.0.ffn_up_exps.weight"].rows == 256


def test_type_table_matches_gguf():
    from gguf import GGML_QUANT_SIZES

    for t, (blk, nbytes) in GGML_QUANT_SIZES.items():
        assert type_size(int(t)) == (blk, nbytes), t
    with pytest.raises(ValueError, match="unknown type"):
        type_size(31)


def test_every_truncation_is_rejected(model_file, tmp_path):
    p, _ = model_file
    data = p.read_bytes()
    with GGUFFile(p) as f:
        header_end = f.data_offset
        last_end = max(t.offset + t.nbytes for t in f.tensors.values())
    cuts = sorted(set(list(range(0, min(header_end, 400))) + list(range(400, header_end, 7)) +
                      [header_end, last_end - 1]))
    q = tmp_path / "cut.gguf"
    for n in cuts:
        q.write_bytes(data[:n])
        with pytest.raises(ValueError):
            GGUFFile(q)


def kv_u32(key, v):
    return (key, 4, struct.pack("<I", v))


@pytest.mark.parametrize("case,msg", [
    (dict(magic=b"GGUX"), "bad magic"),
    (dict(version=1), "unsupported version"),
    (dict(version=4), "unsupported version"),
    (dict(kvs=[kv_u32(b"general.alignment", 48)]), "alignment"),
    (dict(kvs=[kv_u32(b"general.alignment", 0)]), "alignment"),
    (dict(kvs=[(b"general.alignment", 10, struct.pack("<Q", 64))]), "general.alignment"),
    (dict(kvs=[kv_u32(b"k", 1), kv_u32(b"k", 2)]), "duplicate metadata key"),
    (dict(kvs=[(b"k", 13, b"\0" * 8)]), "unknown metadata value type"),
    (dict(tensors=[(b"t", [32], 8, 0), (b"t", [32], 8, 64)], data=b"\0" * 128), "duplicate tensor name"),
    (dict(tensors=[(b"t", [1, 1, 1, 1, 32], 8, 0)], data=b"\0" * 64), "dims"),
    (dict(tensors=[(b"t", [32], 31, 0)], data=b"\0" * 64), "unknown type"),
    (dict(tensors=[(b"t", [48], 8, 0)], data=b"\0" * 64), "whole blocks"),
    (dict(tensors=[(b"t", [64], 8, 0)], data=b"\0" * 67), "beyond the end"),
    (dict(tensors=[(b"t", [32], 8, 1 << 62)], data=b"\0" * 64), "beyond the end"),
    # 2^62 F32 elements: 2^64 bytes would wrap int64 to a small size that fits the file
    (dict(tensors=[(b"t", [1 << 31, 1 << 31], 0, 0)], data=b"\0" * 64), "too large"),
])
def test_malformed_files_rejected(tmp_path, case, msg):
    q = tmp_path / "bad.gguf"
    q.write_bytes(handmade(**case))
    with pytest.raises(ValueError, match=msg):
        GGUFFile(q)


def test_big_endian_rejected(tmp_path):
    q = tmp_path / "be.gguf"
    q.write_bytes(b"GGUF" + struct.pack(">IQQ", 3, 0, 0))
    with pytest.raises(ValueError, match="big-endian"):
        GGUFFile(q)


def test_handmade_file_matches_reader(tmp_path):
    """A minimal file with zero-sized padding rules and an empty tensor, against the reader."""
    from gguf import GGUFReader

    payload = np.arange(68, dtype=np.uint8).tobytes()
    q = tmp_path / "ok.gguf"
    q.write_bytes(handmade(version=2, kvs=[(b"s", 8, gguf_string(b"abc"))],
                           tensors=[(b"a", [32, 2], 8, 0), (b"empty", [0], 0, 96)], data=payload + b"\0" * 60))
    r = GGUFReader(str(q))
    with GGUFFile(q) as f:
        assert f.version == 2 and f.data_offset == r.data_offset
        assert f["a"].nbytes == 68 and f["a"].offset == r.tensors[0].data_offset
        assert f["empty"].nbytes == 0
        assert f.host_bytes("a").tobytes() == payload
        assert f.metadata == {"s": "abc"}


def test_missing_and_empty_files(tmp_path):
    with pytest.raises(OSError):
        GGUFFile(tmp_path / "nope.gguf")
    (tmp_path / "empty.gguf").write_bytes(b"")
    with pytest.raises(ValueError):
        GGUFFile(tmp_path / "empty.gguf")


def test_upload_rejects_bad_ranges_without_gpu(model_file):
    p, _ = model_file
    with GGUFFile(p) as f:
        with pytest.raises(ValueError):
            f.load("output.weight", rows=(0, 81), device="cuda")
        with pytest.raises(ValueError):
            f.load("output.weight", device="cpu")
