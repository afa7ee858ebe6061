"""The IQ2_XXS codebook compiled into the library equals the reference's (src/iq2xxs_grid.h)."""

import os
import re

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _array(src: str, name: str) -> np.ndarray:
    body = src[src.index(name):]
    body = body[:body.index("};")]
    return np.array([int(v, 16) for v in re.findall(r"0x([0-9a-f]{8})u", body)], dtype=np.uint32)


def test_generated_table_equals_reference_bf16_grid(golden):
    src = open(os.path.join(ROOT, "gguf_onnx_ops_b200", "csrc", "iq2xxs_tables.h")).read()
    vals = _array(src, "g_iq2_mag_bf16").reshape(256, 4)
    assert np.array_equal(vals, golden("iq2xxs_grid.npz")["grid_bf16x2"])


def test_byte_codebook_and_sign_masks(golden):
    """g_iq2_mag_u8 holds the same magnitudes as bytes; g_iq2_sign_mask[i] marks the negative
    elements of sign pattern i (7 bits + even-parity 8th bit)."""
    src = open(os.path.join(ROOT, "gguf_onnx_ops_b200", "csrc", "iq2xxs_tables.h")).read()
    bf = golden("iq2xxs_grid.npz")["grid_bf16x2"].astype(np.uint32)
    halves = np.stack([bf & 0xFFFF, bf >> 16], -1).reshape(256, 8).astype(np.uint32)
    mags = (halves << 16).view(np.float32).astype(np.uint32)  # bf16 -> float -> integer magnitude
    u8 = _array(src, "g_iq2_mag_u8").reshape(256, 2)
    got = np.stack([(u8[:, i // 4] >> (8 * (i % 4))) & 0xFF for i in range(8)], -1)
    assert np.array_equal(got, mags)
    masks = _array(src, "g_iq2_sign_mask").reshape(128, 2)
    for si in range(128):
        sb = si | ((bin(si).count("1") & 1) << 7)
        want = [0xFF if (sb >> q) & 1 else 0 for q in range(8)]
        have = [int((masks[si, q // 4] >> (8 * (q % 4))) & 0xFF) for q in range(8)]
        assert have == want, si


def test_generator_is_reproducible():
    from gguf_onnx_ops_b200.csrc import gen_tables

    src = open(os.path.join(ROOT, "gguf_onnx_ops_b200", "csrc", "iq2xxs_tables.h")).read()
    assert gen_tables.render(gen_tables.grid_bytes()) == src
