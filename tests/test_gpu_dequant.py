"""The device decoders (shared by the GEMVs) are bit-identical to gguf-py 0.19.0."""

import numpy as np
import pytest

import oracle as O
from gguf_onnx_ops_b200 import _lib, ops
from oracle import inputs as I
from tests.util import u8_t

pytestmark = pytest.mark.gpu

TYPES = {"q8": (_lib.GGUF_TYPE_Q8_0, O.dequant_q8_0, 32), "iq2": (_lib.GGUF_TYPE_IQ2_XXS, O.dequant_iq2_xxs, 256),
         "fp4": (_lib.GGUF_TYPE_NVFP4, O.dequant_nvfp4, 64), "fp4all": (_lib.GGUF_TYPE_NVFP4, O.dequant_nvfp4, 64)}


def device_deq(raw, t, K, dev):
    return ops.dequantize(u8_t(raw, dev), t, K).cpu().numpy()


def bits_equal(a, b):
    return np.array_equal(np.asarray(a, np.float32).view(np.uint32), np.asarray(b, np.float32).view(np.uint32))


@pytest.mark.parametrize("fmt", list(TYPES))
def test_dequant_golden_bit_exact(cuda, golden, fmt):
    d = golden("dequant.npz")
    t, _, _ = TYPES[fmt]
    raw = d[f"{fmt}_raw"]
    assert bits_equal(device_deq(raw, t, 1024, cuda), d[f"{fmt}_deq"])


@pytest.mark.parametrize("fmt,rows,K", [("q8", 257, 4096), ("q8", 3, 64), ("iq2", 129, 4096), ("iq2", 7, 1792),
                                        ("fp4", 101, 5120), ("fp4", 5, 64)])
def test_dequant_baseline_distributions_bit_exact(cuda, fmt, rows, K):
    t, fn, _ = TYPES[fmt]
    g = I.rng(rows * K)
    raw = {"q8": lambda: I.q8_0_weights(g, rows, K), "iq2": lambda: I.iq2_xxs_weights(g, (rows,), K),
           "fp4": lambda: I.nvfp4_weights(g, rows, K, 0, 255)}[fmt]()
    assert bits_equal(device_deq(raw, t, K, cuda), fn(raw))
