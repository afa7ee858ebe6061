"""Legacy split weight layouts (Q8Gemv gguf=0, Q4Gemv iq2=0/1/2, Nvfp4Gemv gguf=0) on the engine
against the oracle (the reference harness's dequantisation, tests/test_bolt_ops.py:70-100,
155-181, 210-240) followed by an fp64 matmul.  The weights enter the tensor cores exactly, so the
observed error is the bf16 rounding of y; the reference's own bars are rel < 1e-2 (Q8 / Q4 /
NVFP4) and 6e-3 (IQ2 codes)."""

import numpy as np
import pytest
import torch

import oracle as O
from gguf_onnx_ops_b200 import ops
from oracle import inputs as I
from tests.util import bf16_t, rel, u8_t

pytestmark = pytest.mark.gpu

TOL = 5e-3


def run_layout(layout, x, w, s, dev, g=0.37):
    xt = bf16_t(x, dev)
    N = w.shape[0]
    K = x.shape[1]
    if layout == "q8":
        return ops.Q8Gemv(xt, u8_t(w, dev).reshape(N, K // 32, 32), bf16_t(s, dev), gguf=0)
    if layout == "q4":
        return ops.Q4Gemv(xt, u8_t(w, dev).reshape(N, K // 32, 16), bf16_t(s, dev), iq2=0)
    if layout == "iq2c":
        return ops.Q4Gemv(xt, u8_t(w, dev).reshape(N, K // 32, 16), bf16_t(s, dev), iq2=1)
    if layout == "iq2n":
        return ops.Q4Gemv(xt, u8_t(w, dev), bf16_t(s, dev), iq2=2)
    return ops.Nvfp4Gemv(xt, u8_t(w, dev), u8_t(s, dev), torch.tensor([g], device=dev), gguf=0)


def deq(layout, w, s, g=0.37):
    if layout == "q8":
        return O.dequant_q8_split(w, s)
    if layout == "q4":
        return O.dequant_q4_split(w, s)
    if layout == "iq2c":
        return O.dequant_iq2_codes(w, s)
    if layout == "iq2n":
        return O.dequant_iq2_native(w, s)
    return O.dequant_nvfp4_split(w, s) * np.float32(g)


LAYOUTS = ["q8", "q4", "iq2c", "iq2n", "fp4"]


@pytest.mark.parametrize("layout", LAYOUTS)
@pytest.mark.parametrize("R", [1, 3, 8, 16])
def test_legacy_rows(cuda, layout, R):
    g = I.rng(R * 131 + len(layout))
    N, K = 200, 1024  # ragged N
    w, s = I.legacy_case(layout, g, N, K)
    x = I.bf16_normal(g, (R, K))
    y = run_layout(layout, x, w, s, cuda)
    assert rel(y.float().cpu().numpy(), O.gemv_ref(x, deq(layout, w, s))) < TOL


@pytest.mark.parametrize("layout,K", [("q8", 96), ("q8", 4096), ("q4", 160), ("q4", 4096), ("iq2c", 480),
                                      ("iq2c", 8192), ("iq2n", 256), ("iq2n", 4096), ("iq2n", 1280),
                                      ("fp4", 64), ("fp4", 5120), ("fp4", 8192)])
def test_legacy_k_staging_modes(cuda, layout, K):
    """K % 256 != 0 (whole-tile copies), K % 256 == 0 (tensor-map segments), long rows."""
    g = I.rng(K + len(layout))
    N = 72
    w, s = I.legacy_case(layout, g, N, K)
    x = I.bf16_normal(g, (4, K))
    y = run_layout(layout, x, w, s, cuda)
    assert rel(y.float().cpu().numpy(), O.gemv_ref(x, deq(layout, w, s))) < TOL


@pytest.mark.parametrize("R", [1, 3, 5, 8, 12, 16])
@pytest.mark.parametrize("N,K", [(37, 2048), (200, 4096), (61, 5120), (5000, 4096)])
def test_q8_split_few_row_kernel(cuda, R, N, K):
    """Q8Gemv gguf=0 through the few-row integer kernel (K = 2048 / 4096 / 5120; R > 8 at K = 4096
    only, 8 warps of two slices) against the oracle and the generic engine, ragged N; 5000 rows give
    every CTA several tiles (the staging ring wraps)."""
    g = I.rng(N + K + R)
    w, sc = I.legacy_case("q8", g, N, K)
    x = I.bf16_normal(g, (R, K), 2.0)
    y = run_layout("q8", x, w, sc, cuda).float().cpu().numpy()
    assert rel(y, O.gemv_ref(x, deq("q8", w, sc))) < TOL
    ops.set_fast_paths(False)
    try:
        y_gen = run_layout("q8", x, w, sc, cuda).float().cpu().numpy()
    finally:
        ops.set_fast_paths(True)
    assert rel(y, y_gen) < 2e-3


@pytest.mark.parametrize("R", [1, 3, 4, 5])
@pytest.mark.parametrize("N,K", [(37, 2048), (200, 4096), (61, 5120)])
def test_q4_split_few_row_kernel(cuda, R, N, K):
    """Q4Gemv iq2=0 through the few-row integer kernel (R <= 4; nibbles n as u8 weights, the -8 offset
    as the MMA's C input; K = 2048 / 4096 / 5120) against the oracle and the generic engine (R = 5
    takes the engine itself), ragged N."""
    g = I.rng(3 * N + K + R)
    w, sc = I.legacy_case("q4", g, N, K)
    x = I.bf16_normal(g, (R, K), 2.0)
    y = run_layout("q4", x, w, sc, cuda).float().cpu().numpy()
    assert rel(y, O.gemv_ref(x, deq("q4", w, sc))) < TOL
    ops.set_fast_paths(False)
    try:
        y_gen = run_layout("q4", x, w, sc, cuda).float().cpu().numpy()
    finally:
        ops.set_fast_paths(True)
    assert rel(y, y_gen) < 2e-3


@pytest.mark.parametrize("R", [2, 3, 8, 9])
@pytest.mark.parametrize("N,K", [(37, 2048), (200, 4096), (61, 5120)])
def test_fp4_split_few_row_kernel(cuda, R, N, K):
    """Nvfp4Gemv gguf=0 through the few-row NVFP4 kernel (2 <= R <= 8; R = 9 takes the engine) against
    the oracle and the generic engine, ragged N."""
    g = I.rng(5 * N + K + R)
    w, sc = I.legacy_case("fp4", g, N, K)
    x = I.bf16_normal(g, (R, K), 2.0)
    y = run_layout("fp4", x, w, sc, cuda).float().cpu().numpy()
    assert np.isfinite(y).all()
    assert rel(y, O.gemv_ref(x, deq("fp4", w, sc))) < TOL
    ops.set_fast_paths(False)
    try:
        y_gen = run_layout("fp4", x, w, sc, cuda).float().cpu().numpy()
    finally:
        ops.set_fast_paths(True)
    assert rel(y, y_gen) < 2e-3


def test_legacy_reference_shapes(cuda):
    """The harness's shapes: Nvfp4 4096x4096 R=1..8, Q8 / Q4 [N, K/32, 32|16] (tests/test_bolt_ops.py:452-470)."""
    for layout, R, N, K in (("fp4", 1, 4096, 4096), ("fp4", 8, 1024, 8192), ("q8", 2, 4096, 4096),
                            ("q4", 8, 4096, 4096), ("iq2c", 8, 2048, 4096), ("iq2n", 4, 2048, 4096)):
        g = I.rng(N + R)
        w, s = I.legacy_case(layout, g, N, K)
        x = I.bf16_normal(g, (R, K), 2.0)
        y = run_layout(layout, x, w, s, cuda)
        assert rel(y.float().cpu().numpy(), O.gemv_ref(x, deq(layout, w, s))) < TOL, (layout, R, N, K)


@pytest.mark.parametrize("R", [2, 8])
def test_fp4_split_few_row_f16_operands(cuda, R):
    """Nvfp4Gemv gguf=0 on launches of at least 4 tiles per SM (the few-row kernel's f16 operands)
    against the oracle and the generic engine."""
    import torch

    sms = torch.cuda.get_device_properties(0).multi_processor_count
    N, K = 16 * 4 * sms + 21, 4096
    g = I.rng(31 * R)
    w, sc = I.legacy_case("fp4", g, N, K)
    x = I.bf16_normal(g, (R, K), 2.0)
    y = run_layout("fp4", x, w, sc, cuda).float().cpu().numpy()
    assert np.isfinite(y).all()
    assert rel(y, O.gemv_ref(x, deq("fp4", w, sc))) < TOL
    ops.set_fast_paths(False)
    try:
        y_gen = run_layout("fp4", x, w, sc, cuda).float().cpu().numpy()
    finally:
        ops.set_fast_paths(True)
    assert rel(y, y_gen) < 2e-3


def test_fp4_every_scale_byte(cuda):
    """Every non-NaN e4m3fn scale byte (both signs, subnormals) decodes exactly."""
    g = I.rng(9)
    N, K = 16, 16 * 254
    w = g.integers(0, 256, size=(N, K // 2), dtype=np.uint8)
    codes = np.array([b for b in range(256) if (b & 0x7F) != 0x7F], dtype=np.uint8)
    s = np.tile(codes, (N, 1))
    x = I.bf16_normal(g, (2, K))
    y = run_layout("fp4", x, w, s, cuda, g=1.0)
    assert rel(y.float().cpu().numpy(), O.gemv_ref(x, deq("fp4", w, s, g=1.0))) < TOL


def test_iq2_native_matches_gguf_layout(cuda):
    """iq2=2 (records + d) and iq2=3 (GGUF blocks) hold the same weights: both match the oracle
    and each other to the bf16 rounding of y (the reference harness's vs_repack check, :241-242)."""
    g = I.rng(21)
    N, K = 256, 4096
    blk = I.iq2_test_blocks(g, (N,), K)
    rec, d = O.iq2_native_from_blocks(blk)
    x = I.bf16_normal(g, (3, K))
    y_native = run_layout("iq2n", x, rec, d, cuda).float().cpu().numpy()
    y_gguf = ops.Q4Gemv(bf16_t(x, cuda), u8_t(blk, cuda), iq2=3).float().cpu().numpy()
    ref = O.gemv_ref(x, O.dequant_iq2_xxs(blk))
    assert rel(y_native, ref) < TOL and rel(y_gguf, ref) < TOL and rel(y_native, y_gguf) < TOL


def test_legacy_graph_capture_and_status(cuda):
    g = I.rng(3)
    w, s = I.legacy_case("q4", g, 64, 512)
    x = bf16_t(I.bf16_normal(g, (2, 512)), cuda)
    wt, st = u8_t(w, cuda).reshape(64, 16, 16), bf16_t(s, cuda)
    y = torch.empty(2, 64, dtype=torch.bfloat16, device=cuda)
    from gguf_onnx_ops_b200 import _lib

    ops.gemv_legacy_into(_lib.GGUF_LAYOUT_Q4_SPLIT, x, wt, st, None, y, 2, 64, 512)
    ref = y.clone()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        ops.gemv_legacy_into(_lib.GGUF_LAYOUT_Q4_SPLIT, x, wt, st, None, y, 2, 64, 512)
    y.zero_()
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(y, ref)
    assert ops.device_status() == (0, 0)
