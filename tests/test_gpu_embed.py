"""Q8Embed (src/bolt_ops.cu:1645-1690): the device gather + dequantisation is bit-identical to the
oracle, including ids outside [0, vocab), empty and multi-dimensional id tensors."""

import numpy as np
import pytest
import torch

import oracle as O
from gguf_onnx_ops_b200 import ops
from oracle import inputs as I
from tests.golden.cases import embed_inputs
from tests.util import u8_t

pytestmark = pytest.mark.gpu


def bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.cpu().view(torch.int16).numpy().view(np.uint16)


def test_embed_golden_bit_exact(cuda, golden):
    blk, ids = embed_inputs()
    out = ops.Q8Embed(u8_t(blk, cuda), torch.from_numpy(ids).to(cuda))
    assert out.dtype == torch.bfloat16 and tuple(out.shape) == (2, 9, 1024)
    assert np.array_equal(bf16_bits(out), golden("embed.npz")["out_bf16"])


@pytest.mark.parametrize("V,K,shape", [(512, 4096, (1, 8)),      # the reference test's case
                                       (1000, 2048, (3, 77)),
                                       (37, 96, (5,)),           # K not a multiple of 128: partial 4-block group
                                       (7, 32, (2, 3, 4)),
                                       (300, 2080, (2, 50)),     # 65 blocks per row: scalar kernel
                                       (2000, 768, (4001,)),     # 3 units per row, 4 per warp, ragged tail
                                       (32000, 4096, (4, 2048))])
def test_embed_random_bit_exact(cuda, V, K, shape):
    g = I.rng(V * 31 + K)
    blk = I.q8_test_blocks(g, V, K)
    ids = g.integers(-3, V + 3, size=shape).astype(np.int64)
    out = ops.Q8Embed(u8_t(blk, cuda), torch.from_numpy(ids).to(cuda))
    assert tuple(out.shape) == shape + (K,)
    assert np.array_equal(bf16_bits(out), O.bf16_bits(O.embed_ref(blk, ids)))


def test_embed_empty_ids(cuda):
    blk, _ = embed_inputs()
    w = u8_t(blk, cuda)
    for shape in ((0,), (2, 0)):
        out = ops.Q8Embed(w, torch.zeros(shape, dtype=torch.int64, device=cuda))
        assert tuple(out.shape) == shape + (1024,)


def test_embed_rejects_bad_tables(cuda):
    with pytest.raises(ValueError, match="multiple of 34"):
        ops.Q8Embed(torch.zeros(4, 35, dtype=torch.uint8, device=cuda), torch.zeros(1, dtype=torch.int64, device=cuda))
    with pytest.raises(ValueError, match="invalid weight shape"):
        ops.Q8Embed(torch.zeros(0, 34, dtype=torch.uint8, device=cuda), torch.zeros(1, dtype=torch.int64, device=cuda))
