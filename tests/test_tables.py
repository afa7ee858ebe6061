"""The IQ2_XXS codebook compiled into the library equals the reference's (src/iq2xxs_grid.h)."""

import os
import re

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_generated_table_equals_reference_bf16_grid(golden):
    src = open(os.path.join(ROOT, "gguf_onnx_ops_b200", "csrc", "iq2xxs_tables.h")).read()
    vals = np.array([int(v, 16) for v in re.findall(r"0x([0-9a-f]{8})u", src)], dtype=np.uint32).reshape(256, 4)
    assert np.array_equal(vals, golden("iq2xxs_grid.npz")["grid_bf16x2"])


def test_generator_is_reproducible():
    from gguf_onnx_ops_b200.csrc import gen_tables

    src = open(os.path.join(ROOT, "gguf_onnx_ops_b200", "csrc", "iq2xxs_tables.h")).read()
    assert gen_tables.render(gen_tables.grid_bytes()) == src
