"""GGUF file -> HBM -> ops: the staged upload lands the file's bytes unchanged, row ranges give
the shard a rank would load, and the ops run on the loaded tensors with oracle parity."""

import numpy as np
import pytest
import torch

import oracle as O
from gguf_onnx_ops_b200 import ops
from gguf_onnx_ops_b200.gguf_file import GGUFFile
from oracle import inputs as I
from tests.gguf_files import write_model_file
from tests.util import bf16_t, rel

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def model(tmp_path_factory):
    p = tmp_path_factory.mktemp("gguf") / "model.gguf"
    raw = write_model_file(p, seed=5, alignment=64)
    f = GGUFFile(p)
    yield f, raw
    f.close()


def test_upload_bytes_exact(cuda, model):
    f, raw = model
    for name, t in f.tensors.items():
        d = f.load(name, device=cuda)
        dtype, shape = t.onnx_view()
        assert d.dtype == dtype and tuple(d.shape) == shape
        got = d.contiguous().view(torch.uint8).cpu().numpy().reshape(-1)
        assert np.array_equal(got, raw[name].reshape(-1)), name


def test_load_many_and_row_ranges(cuda, model):
    f, raw = model
    names = list(f.tensors)
    outs = f.load_many(names, device=cuda)
    for n in names:
        assert np.array_equal(outs[n].view(torch.uint8).cpu().numpy().reshape(-1), raw[n].reshape(-1))
    # a rank's shard of the LM head and one expert of the stacked IQ2 tensor
    shard = f.load("output.weight", rows=(16, 48), device=cuda)
    assert np.array_equal(shard.cpu().numpy(), raw["output.weight"][16:48])
    e2 = f.load("blk.0.ffn_up_exps.weight", rows=(128, 192), device=cuda)
    assert np.array_equal(e2.cpu().numpy(), raw["blk.0.ffn_up_exps.weight"][128:192])
    empty = f.load("output.weight", rows=(5, 5), device=cuda)
    assert tuple(empty.shape) == (0, 32 * 34)


def test_ops_on_loaded_tensors(cuda, model):
    f, raw = model
    g = I.rng(77)
    # LM head GEMV (Q8Gemv gguf=1) on the loaded weight
    w = f.load("output.weight", device=cuda)
    x = I.bf16_normal(g, (4, 1024))
    y = ops.Q8Gemv(bf16_t(x, cuda), w, gguf=1)
    ref = O.gemv_ref(x, O.dequant_q8_0(raw["output.weight"]))
    assert rel(y.float().cpu().numpy(), ref) < 5e-3
    # token embedding gather on the loaded table
    emb = f.load("token_embd.weight", device=cuda)
    ids = g.integers(-2, 100, size=(3, 7)).astype(np.int64)
    out = ops.Q8Embed(emb, torch.from_numpy(ids).to(cuda))
    expect = O.bf16_bits(O.embed_ref(raw["token_embd.weight"], ids))
    assert np.array_equal(out.cpu().view(torch.int16).numpy().view(np.uint16), expect)


def test_large_multi_chunk_upload(cuda, tmp_path):
    """A tensor larger than the staging ring (4 x 32 MiB) with a row range crossing chunk edges."""
    from gguf import GGMLQuantizationType as Q
    from gguf import GGUFWriter

    rows, row_bytes = 40000, 4352  # 174 MB of Q8_0 [40000, 4096]
    data = np.random.default_rng(1).integers(0, 256, size=(rows, row_bytes), dtype=np.uint8)
    p = tmp_path / "big.gguf"
    w = GGUFWriter(str(p), "test")
    w.add_tensor("big", data, raw_dtype=Q.Q8_0)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    with GGUFFile(p) as f:
        d = f.load("big", device=cuda)
        assert torch.equal(d.cpu(), torch.from_numpy(data))
        s = f.load("big", rows=(7711, 31000), device=cuda)
        assert torch.equal(s.cpu(), torch.from_numpy(data[7711:31000]))
