"""GPU parity of the GGUF GEMVs (through the C ABI) against the CPU oracle and the golden fixtures.

Tolerance: rel-L2 <= 5e-3 of the fp64 oracle (north-star bound for bf16 outputs); the kernels see
the exact dequantised weights, so the observed error is the bf16 rounding of y (~1e-3).
"""

import numpy as np
import pytest
import torch

import oracle as O
from gguf_onnx_ops_b200 import _lib, ops
from oracle import inputs as I
from tests.golden.cases import GEMV_CASES
from tests.util import bf16_t, np_f32, rel, u8_t

pytestmark = pytest.mark.gpu

TOL = 5e-3
DEQ = {"q8_0": O.dequant_q8_0, "iq2_xxs": O.dequant_iq2_xxs, "nvfp4": O.dequant_nvfp4}


def run_gemv(op, x, w, extra, dev):
    xt, wt = bf16_t(x, dev), u8_t(w, dev)
    if op == "q8_0":
        y = ops.Q8Gemv(xt, wt, gguf=1)
    elif op == "iq2_xxs":
        y = ops.Q4Gemv(xt, wt, iq2=3)
    else:
        y = ops.Nvfp4Gemv(xt, wt, None, torch.from_numpy(extra["gscale"]).to(dev), gguf=1)
    torch.cuda.synchronize()
    return np_f32(y)


def oracle_y(op, x, w, extra, rows=None):
    wsel = w if rows is None else w[rows]
    y = O.gemv_ref(x, DEQ[op](wsel))
    return y * (float(extra["gscale"][0]) if op == "nvfp4" else 1.0)


def assert_device_ok():
    rc, site = _lib.device_status()
    assert rc == 0, f"device-side error at site {site}"


@pytest.mark.parametrize("name", list(GEMV_CASES))
def test_golden_cases(cuda, golden, name):
    d = golden("gemv.npz")
    op, R, N, K, seed = GEMV_CASES[name]
    x, w = d[f"{name}_x"], d[f"{name}_w"]
    extra = {"gscale": np.array([1.0 / 448.0], np.float32)}
    y = run_gemv(op, x, w, extra, cuda)
    assert rel(y, d[f"{name}_y"]) < TOL
    assert rel(y, oracle_y(op, x, w, extra)) < TOL


@pytest.mark.parametrize("op", ["q8_0", "iq2_xxs", "nvfp4"])
@pytest.mark.parametrize("R", [1, 2, 3, 5, 7, 8, 9, 12, 16])
def test_all_row_counts(cuda, op, R):
    K = {"q8_0": 1024, "iq2_xxs": 1024, "nvfp4": 1280}[op]
    x, w, extra = I.gemv_case(op, R, 200, K, seed=100 + R)
    y = run_gemv(op, x, w, extra, cuda)
    assert rel(y, oracle_y(op, x, w, extra)) < TOL


@pytest.mark.parametrize("op,N,K", [
    ("q8_0", 1, 64), ("q8_0", 17, 320), ("q8_0", 33, 4160), ("q8_0", 5, 16384),  # contiguous + tail paths
    ("iq2_xxs", 1, 256), ("iq2_xxs", 23, 768), ("iq2_xxs", 31, 1792), ("iq2_xxs", 9, 8192),
    ("nvfp4", 1, 64), ("nvfp4", 19, 192), ("nvfp4", 45, 5120), ("nvfp4", 7, 16384),
])
def test_ragged_and_odd_shapes(cuda, op, N, K):
    x, w, extra = I.gemv_case(op, 3, N, K, seed=N * 7 + K)
    y = run_gemv(op, x, w, extra, cuda)
    assert rel(y, oracle_y(op, x, w, extra)) < TOL


@pytest.mark.parametrize("op", ["q8_0", "iq2_xxs", "nvfp4"])
def test_massive_activations(cuda, op):
    """Outlier activations (the reference's XSCALE=3000 case) must not overflow anything."""
    g = I.rng(77)
    K = 2048
    x = I.bf16_normal(g, (8, K), 3000.0)
    _, w, extra = I.gemv_case(op, 1, 96, K, seed=78)
    y = run_gemv(op, x, w, extra, cuda)
    assert np.isfinite(y).all()
    assert rel(y, oracle_y(op, x, w, extra)) < TOL


def test_nvfp4_all_scale_bytes(cuda, golden):
    d = golden("dequant.npz")
    w = d["fp4all_raw"]  # scale bytes 0x00..0xFF incl. 0x7F and >= 0x80 (gguf-py semantics)
    g = I.rng(3)
    x = I.bf16_normal(g, (2, 1024))
    extra = {"gscale": np.array([0.37], np.float32)}
    y = run_gemv("nvfp4", x, w, extra, cuda)
    ref = O.gemv_ref(x, d["fp4all_deq"]) * 0.37
    assert rel(y, ref) < TOL


# BASELINE configs at full size: oracle on a random subset of rows; every row against the
# bit-exact device dequantisation followed by an fp32 matmul.
CONFIG_CASES = [("C0", "q8_0", 1, 4096, 4096)] + [("C1", "iq2_xxs", R, 14336, 4096) for R in (1, 4, 8)] + \
               [("C2", "nvfp4", R, 13824, 5120) for R in (1, 8, 16)]


@pytest.mark.parametrize("cfg,op,R,N,K", CONFIG_CASES)
def test_baseline_configs(cuda, cfg, op, R, N, K):
    x, w, extra = I.gemv_case(op, R, N, K, seed=0)
    y = run_gemv(op, x, w, extra, cuda)
    rows = np.sort(I.rng(1).choice(N, size=512, replace=False))
    assert rel(y[:, rows], oracle_y(op, x, w, extra, rows)) < TOL
    gt = {"q8_0": _lib.GGUF_TYPE_Q8_0, "iq2_xxs": _lib.GGUF_TYPE_IQ2_XXS, "nvfp4": _lib.GGUF_TYPE_NVFP4}[op]
    deq = ops.dequantize(u8_t(w, cuda), gt, K)
    full = bf16_t(x, cuda).float() @ deq.T
    if op == "nvfp4":
        full = full * float(extra["gscale"][0])
    assert rel(y, np_f32(full)) < TOL
    assert_device_ok()


def test_lm_head_shape_r16(cuda):
    """C4 shape (N = 131072) at R=16, oracle on a row subset."""
    x, w, extra = I.gemv_case("q8_0", 16, 131072, 4096, seed=4)
    y = run_gemv("q8_0", x, w, extra, cuda)
    rows = np.sort(I.rng(2).choice(131072, size=256, replace=False))
    assert rel(y[:, rows], oracle_y("q8_0", x, w, extra, rows)) < TOL


@pytest.fixture(scope="module")
def c4_weights():
    """BASELINE config 4's LM head (Q8_0, N = 131072, K = 4096), built once for the R sweep."""
    _, w, extra = I.gemv_case("q8_0", 1, 131072, 4096, seed=0)
    return w, extra


@pytest.mark.parametrize("R", [1, 4, 8])
def test_lm_head_config_c4(cuda, c4_weights, R):
    """Config C4 at full size (N = 131072, K = 4096) for R = 1, 4, 8: the oracle on a 512-row sample,
    every row against the bit-exact device dequantisation followed by an fp32 matmul."""
    w, extra = c4_weights
    x = I.bf16_normal(I.rng(40 + R), (R, 4096))
    y = run_gemv("q8_0", x, w, extra, cuda)
    rows = np.sort(I.rng(R).choice(131072, size=512, replace=False))
    assert rel(y[:, rows], oracle_y("q8_0", x, w, extra, rows)) < TOL
    wt = u8_t(w, cuda)
    deq = ops.dequantize(wt, _lib.GGUF_TYPE_Q8_0, 4096)
    full = np_f32(bf16_t(x, cuda).float() @ deq.T)
    del deq, wt
    assert rel(y, full) < TOL
    assert_device_ok()


# The reference harness's own IQ2_XXS GEMV shapes (tests/test_bolt_ops.py:478, test_q4_iq2_native):
# K = 5376 is 21 super-blocks, an odd count between the K-specialised kernels (2048 / 4096 / 5120).
@pytest.mark.parametrize("R,N,K", [(8, 5376, 4096), (1, 4096, 5376), (3, 1024, 4096), (8, 4096, 5376)])
def test_harness_iq2_shapes(cuda, R, N, K):
    g = I.rng(21 + R + N + K)
    w = I.iq2_test_blocks(g, (N,), K)  # the harness's block builder (tests/test_bolt_ops.py:210-215)
    x = I.bf16_normal(g, (R, K))
    y = run_gemv("iq2_xxs", x, w, {}, cuda)
    assert rel(y, oracle_y("iq2_xxs", x, w, {})) < TOL
    assert_device_ok()


@pytest.mark.parametrize("op", ["q8_0", "iq2_xxs", "nvfp4"])
def test_chained_calls_with_pdl(cuda, op):
    """y of call i is x of call i+1 (N == K): programmatic dependent launch must still order the
    consumer's activation reads after the producer kernel; results equal the non-PDL chain."""
    K = 1024
    chain = [I.gemv_case(op, 4, K, K, seed=500 + i) for i in range(6)]
    x0 = bf16_t(chain[0][0], cuda)
    ws = [u8_t(c[1], cuda) for c in chain]
    gs = torch.tensor([1.0 / 64.0], device=cuda)

    def run(pdl):
        ops.set_pdl(pdl)
        x = x0
        for wt in ws:
            if op == "q8_0":
                x = ops.Q8Gemv(x, wt)
            elif op == "iq2_xxs":
                x = ops.Q4Gemv(x, wt)
            else:
                x = ops.Nvfp4Gemv(x, wt, None, gs)
        torch.cuda.synchronize()
        return x.clone()

    try:
        a = run(True)
        b = run(False)
    finally:
        ops.set_pdl(True)
    assert torch.equal(a, b)
    assert_device_ok()


def test_graph_capture_replay(cuda):
    x, w, _ = I.gemv_case("iq2_xxs", 4, 2048, 4096, seed=9)
    xt, wt = bf16_t(x, cuda), u8_t(w, cuda)
    y = torch.empty(4, 2048, dtype=torch.bfloat16, device=cuda)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        ops.iq2_xxs_gemv_into(xt, wt, y, 4, 2048, 4096)  # warm-up (sets kernel attributes)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        ops.iq2_xxs_gemv_into(xt, wt, y, 4, 2048, 4096)
    y.zero_()
    g.replay()
    torch.cuda.synchronize()
    assert rel(np_f32(y), oracle_y("iq2_xxs", x, w, {})) < TOL


def test_invalid_row_count_raises(cuda):
    x = torch.zeros(17, 256, dtype=torch.bfloat16, device=cuda)
    w = torch.zeros(16, 66, dtype=torch.uint8, device=cuda)
    with pytest.raises(ValueError, match="1..16 rows"):
        ops.Q4Gemv(x, w)


@pytest.mark.parametrize("op", ["q8_0", "iq2_xxs", "nvfp4"])
@pytest.mark.parametrize("N,K,xscale", [(1, 2048, 1.0), (37, 2048, 1.0), (200, 4096, 1.0), (4096, 4096, 1.0),
                                        (61, 5120, 1.0), (300, 4096, 3000.0), (50, 8192, 1.0)])
def test_single_row_fast_path(cuda, op, N, K, xscale):
    """The R=1 slice kernels (block-diagonal MMA columns, x resident in registers) against the oracle
    and against the generic engine; xscale=3000 exercises outlier activations (Q8's offset trick)."""
    if op == "nvfp4" and K % 64 or op == "iq2_xxs" and K % 256:
        pytest.skip("shape")
    _, w, extra = I.gemv_case(op, 1, N, K, seed=N + K)
    x = I.bf16_normal(I.rng(N * K), (1, K), xscale)
    y_fast = run_gemv(op, x, w, extra, cuda)
    rows = np.arange(N) if N <= 512 else np.sort(I.rng(3).choice(N, size=512, replace=False))
    assert rel(y_fast[:, rows], oracle_y(op, x, w, extra, rows)) < TOL
    ops.set_fast_paths(False)
    try:
        y_gen = run_gemv(op, x, w, extra, cuda)
        if op == "iq2_xxs":  # the other single-row kernels (modes 2, 3) against the default (mode 1)
            for mode in (2, 3):
                ops.set_fast_paths(mode)
                y_alt = run_gemv(op, x, w, extra, cuda)
                assert rel(y_fast, y_alt) < 2e-3, mode
    finally:
        ops.set_fast_paths(True)
    assert rel(y_fast, y_gen) < 2e-3
    assert_device_ok()


@pytest.mark.parametrize("N,K,xscale", [(2408, 4096, 1.0), (2650, 2048, 1.0), (2448, 5120, 1.0),
                                        (14336, 4096, 3000.0), (14331, 4096, 1.0), (3648, 4096, 1.0)])
def test_iq2_single_row_partial_last_round(cuda, N, K, xscale):
    """Single-row IQ2_XXS where the tiles leave a partial last round on 148 SMs (2408 rows: 151 tiles,
    the last of 8 rows; 14336 rows: 896 tiles = 6 x 148 + 8; 14331 rows: the last tile of 11 rows).
    3648 rows: 228 tiles = 148 + 80.
    Against the oracle on every row of the last tiles and a sample of the rest, against the generic
    engine, and bit-identical over 70 launches (fixed-order reductions, no state kept between calls)."""
    _, w, extra = I.gemv_case("iq2_xxs", 1, N, K, seed=N + K + 5)
    x = I.bf16_normal(I.rng(N + K), (1, K), xscale)
    x[:, 7] = O.bf16_bits(O.bf16_to_f32(x[:, 7]) * np.float32(300.0))  # bf16 bits: one outlier column
    y = run_gemv("iq2_xxs", x, w, extra, cuda)
    tail = np.arange(max(0, N - 200), N)  # the split tiles are the last ones
    rows = np.union1d(tail, np.sort(I.rng(4).choice(N, size=min(N, 300), replace=False)))
    assert rel(y[:, rows], oracle_y("iq2_xxs", x, w, extra, rows)) < TOL
    assert rel(y[:, tail], oracle_y("iq2_xxs", x, w, extra, tail)) < TOL
    xt, wt = bf16_t(x, cuda), u8_t(w, cuda)
    outs = [ops.Q4Gemv(xt, wt, iq2=3) for _ in range(70)]
    torch.cuda.synchronize()
    ref = outs[0].view(torch.int16)
    for o in outs[1:]:
        assert torch.equal(o.view(torch.int16), ref)
    assert np.array_equal(np_f32(outs[0]), y)
    ops.set_fast_paths(False)
    try:
        y_gen = run_gemv("iq2_xxs", x, w, extra, cuda)
    finally:
        ops.set_fast_paths(True)
    assert rel(y, y_gen) < 2e-3
    assert_device_ok()


@pytest.mark.parametrize("R", [2, 3, 4, 5, 8])
@pytest.mark.parametrize("N,K,xscale", [(37, 2048, 1.0), (200, 4096, 1.0), (1000, 4096, 3000.0), (61, 5120, 1.0)])
def test_iq2_few_row_integer_kernel(cuda, R, N, K, xscale):
    """The few-row IQ2_XXS kernel (2 <= R <= 8: activation rows x limbs as MMA columns; R > 4 at
    K = 4096 only, else the engine) against the oracle and the generic engine, ragged N, one outlier
    column per row and a x3000 scale."""
    _, w, _ = I.gemv_case("iq2_xxs", 1, N, K, seed=N + K + R)
    x = I.bf16_normal(I.rng(N * K + R), (R, K), xscale)
    x[:, 7] = O.bf16_bits(O.bf16_to_f32(x[:, 7]) * np.float32(300.0))  # bf16 bits: one outlier column
    y = run_gemv("iq2_xxs", x, w, {}, cuda)
    assert rel(y, oracle_y("iq2_xxs", x, w, {})) < TOL
    ops.set_fast_paths(False)
    try:
        y_gen = run_gemv("iq2_xxs", x, w, {}, cuda)
    finally:
        ops.set_fast_paths(True)
    assert rel(y, y_gen) < 2e-3
    assert_device_ok()


@pytest.mark.parametrize("R", [2, 3, 4, 5, 8, 12, 16])
@pytest.mark.parametrize("N,K,xscale", [(37, 2048, 1.0), (200, 4096, 1.0), (1000, 4096, 3000.0), (61, 5120, 1.0)])
def test_q8_few_row_integer_kernel(cuda, R, N, K, xscale):
    """The few-row Q8_0 kernel (2 <= R <= 16: the int8 quants as the MMA's A operand, activation rows x
    signed limbs as columns; R > 8 at K = 4096 only) against the oracle and the generic engine, ragged
    N and outliers."""
    _, w, _ = I.gemv_case("q8_0", 1, N, K, seed=N + K + R)
    x = I.bf16_normal(I.rng(N * K + R), (R, K), xscale)
    x[:, 7] = O.bf16_bits(O.bf16_to_f32(x[:, 7]) * np.float32(300.0))  # bf16 bits: one outlier column
    y = run_gemv("q8_0", x, w, {}, cuda)
    assert rel(y, oracle_y("q8_0", x, w, {})) < TOL
    ops.set_fast_paths(False)
    try:
        y_gen = run_gemv("q8_0", x, w, {}, cuda)
    finally:
        ops.set_fast_paths(True)
    assert rel(y, y_gen) < 2e-3
    assert_device_ok()


@pytest.mark.parametrize("R", [2, 3, 5, 8, 9, 12, 16])
@pytest.mark.parametrize("N,K", [(37, 2048), (200, 4096), (333, 5120), (4000, 5120)])
def test_nvfp4_few_row_kernel(cuda, R, N, K):
    """The few-row NVFP4 kernel (activation rows as the MMA columns, scales inside the exact bf16
    weights; R = 9..16 in one launch with a second set of 8 activation rows, whose fragments sit in
    shared memory) against the oracle and the generic engine, every scale byte present; 4000 rows
    give every CTA 2 stages' worth of tiles and a ragged last tile."""
    g = I.rng(K + 11 * R + N)
    w = I.nvfp4_weights(g, N, K, 0, 255)
    x = I.bf16_normal(g, (R, K), 2.0)
    extra = {"gscale": np.array([0.37], np.float32)}
    y = run_gemv("nvfp4", x, w, extra, cuda)
    assert np.isfinite(y).all()
    assert rel(y, oracle_y("nvfp4", x, w, extra, np.arange(N))) < TOL
    ops.set_fast_paths(False)
    try:
        y_gen = run_gemv("nvfp4", x, w, extra, cuda)
    finally:
        ops.set_fast_paths(True)
    assert rel(y, y_gen) < 2e-3
    assert_device_ok()


@pytest.mark.parametrize("R", [2, 5, 8])
@pytest.mark.parametrize("K", [4096, 5120])
def test_nvfp4_few_row_f16_operands(cuda, R, K):
    """Launches of at least 4 tiles per SM take the few-row NVFP4 kernel's f16 operands (hardware E2M1
    conversion, per-row power-of-two x scaling): against the oracle and the generic engine, with a
    ragged last tile, every scale byte present and a row of large and one of tiny activations."""
    import torch

    sms = torch.cuda.get_device_properties(0).multi_processor_count
    N = 16 * 4 * sms + 37
    g = I.rng(K + 7 * R)
    w = I.nvfp4_weights(g, N, K, 0, 255)
    x = I.bf16_normal(g, (R, K), 2.0)
    big = I.bf16_normal(g, (1, K), 3000.0)
    tiny = I.bf16_normal(g, (1, K), 2.0 ** -100)
    x[0], x[R - 1] = big[0], tiny[0]
    extra = {"gscale": np.array([0.37], np.float32)}
    y = run_gemv("nvfp4", x, w, extra, cuda)
    assert np.isfinite(y).all()
    ref = oracle_y("nvfp4", x, w, extra, np.arange(N))
    for r in range(R):  # each activation row on its own scale
        assert rel(y[r], ref[r]) < TOL, r
    ops.set_fast_paths(False)
    try:
        y_gen = run_gemv("nvfp4", x, w, extra, cuda)
    finally:
        ops.set_fast_paths(True)
    assert rel(y, y_gen) < 2e-3
    assert_device_ok()


@pytest.mark.parametrize("K", [2048, 4096, 5120, 6144, 8192])
def test_nvfp4_single_row_integer_kernel(cuda, K):
    """The single-row NVFP4 kernels (bf16 slice, the default, and the integer-decode variant, mode 4)
    against the oracle and the generic engine, with every scale byte present (gguf-py UE4M3: 0x7F -> 0,
    otherwise bit 7 ignored)."""
    N = 333
    g = I.rng(K + 7)
    w = I.nvfp4_weights(g, N, K, 0, 255)
    x = I.bf16_normal(g, (1, K), 2.0)
    extra = {"gscale": np.array([0.37], np.float32)}
    ref = oracle_y("nvfp4", x, w, extra, np.arange(N))
    y = run_gemv("nvfp4", x, w, extra, cuda)
    assert rel(y, ref) < TOL
    try:
        ops.set_fast_paths(4)
        y4 = run_gemv("nvfp4", x, w, extra, cuda)
        ops.set_fast_paths(False)
        y0 = run_gemv("nvfp4", x, w, extra, cuda)
    finally:
        ops.set_fast_paths(True)
    assert rel(y4, ref) < TOL and rel(y, y4) < 2e-3
    assert rel(y, y0) < 2e-3
    assert_device_ok()


@pytest.mark.parametrize("case", ["wide_range", "zero_groups", "subnormal", "outlier_per_group"])
def test_nvfp4_single_row_activation_ranges(cuda, case):
    """The integer NVFP4 path scales each 16-element sub-block of x by its maximum (as IQ2_XXS does
    per 32): wide ranges, zero / subnormal sub-blocks and outliers stay within the op tolerance."""
    N, K = 512, 5120
    _, w, extra = I.gemv_case("nvfp4", 1, N, K, seed=12)
    g = I.rng(98)
    xf = g.standard_normal(K).astype(np.float32)
    if case == "wide_range":
        xf *= np.exp2(g.integers(-24, 12, K)).astype(np.float32)
    elif case == "zero_groups":
        xf.reshape(-1, 16)[::3] = 0.0
    elif case == "subnormal":
        xf.reshape(-1, 16)[::2] *= np.float32(2.0 ** -130)
    else:
        xf.reshape(-1, 16)[:, 5] *= 3000.0
    x = O.bf16_bits(xf).reshape(1, K)
    y = run_gemv("nvfp4", x, w, extra, cuda)
    assert np.isfinite(y).all()
    assert rel(y, oracle_y("nvfp4", x, w, extra, np.arange(N))) < TOL
    assert_device_ok()


@pytest.mark.parametrize("case", ["wide_range", "zero_groups", "subnormal", "outlier_per_group"])
def test_iq2_single_row_activation_ranges(cuda, case):
    """Single-row IQ2_XXS carries each 32-element group of x as a 2-limb fixed-point integer scaled by
    the group maximum: exact within 2^7 of the maximum, 2^-14 of the maximum below.  Activations with
    a wide dynamic range inside groups, all-zero groups and subnormal groups stay within the op
    tolerance of the fp64 oracle."""
    N, K = 512, 4096
    _, w, extra = I.gemv_case("iq2_xxs", 1, N, K, seed=11)
    g = I.rng(99)
    xf = g.standard_normal(K).astype(np.float32)
    if case == "wide_range":
        xf *= np.exp2(g.integers(-24, 12, K)).astype(np.float32)
    elif case == "zero_groups":
        xf.reshape(-1, 32)[::3] = 0.0
    elif case == "subnormal":
        xf.reshape(-1, 32)[::2] *= np.float32(2.0 ** -130)
    else:
        xf.reshape(-1, 32)[:, 5] *= 3000.0
    x = O.bf16_bits(xf).reshape(1, K)
    y = run_gemv("iq2_xxs", x, w, extra, cuda)
    ref = oracle_y("iq2_xxs", x, w, extra, np.arange(N))
    assert np.isfinite(y).all()
    assert rel(y, ref) < TOL
    assert_device_ok()
