"""The CPU oracle pinned against the reference's CPU path (gguf-py 0.19.0 + torch), via the committed
golden fixtures and live gguf-py calls.  No GPU needed."""

import numpy as np
import pytest
import torch

import oracle as O
from oracle import inputs as I
from tests.golden.cases import GEMV_CASES, embed_inputs, mamba_inputs, moe_inputs, norm_inputs, route_inputs, sha
from tests.util import rel


def bits_equal(a, b):
    return np.array_equal(np.asarray(a, np.float32).view(np.uint32), np.asarray(b, np.float32).view(np.uint32))


@pytest.mark.parametrize("fmt", ["q8", "iq2", "fp4", "fp4all"])
def test_dequant_matches_golden(golden, fmt):
    d = golden("dequant.npz")
    fn = {"q8": O.dequant_q8_0, "iq2": O.dequant_iq2_xxs, "fp4": O.dequant_nvfp4, "fp4all": O.dequant_nvfp4}[fmt]
    assert bits_equal(fn(d[f"{fmt}_raw"]), d[f"{fmt}_deq"])


def test_dequant_matches_live_gguf():
    from gguf import GGMLQuantizationType as Q
    from gguf import quants

    g = I.rng(5)
    for raw, qt, fn in ((I.q8_0_weights(g, 33, 256), Q.Q8_0, O.dequant_q8_0),
                        (I.iq2_xxs_weights(g, (17,), 512), Q.IQ2_XXS, O.dequant_iq2_xxs),
                        (I.nvfp4_weights(g, 9, 320, 0, 255), Q.NVFP4, O.dequant_nvfp4)):
        ref = np.asarray(quants.dequantize(raw, qt), np.float32).reshape(raw.shape[0], -1)
        assert bits_equal(fn(raw), ref)


def test_quantize_q8_0_matches_gguf():
    from gguf import GGMLQuantizationType as Q
    from gguf import quants

    w = (I.rng(6).standard_normal((16, 512)) * 0.02).astype(np.float32)
    w[3, :32] = 0.0  # all-zero block: d = 0
    assert np.array_equal(O.quantize_q8_0(w), quants.quantize(w, Q.Q8_0))


def test_grid_matches_reference_codebook(golden):
    g = golden("iq2xxs_grid.npz")
    ref = g["grid_u64"].astype(np.uint64)
    ref_bytes = ((ref[:, None] >> (np.arange(8, dtype=np.uint64) * 8)[None, :]) & 0xFF).astype(np.uint8)
    assert np.array_equal(O.iq2xxs_grid(), ref_bytes)


def test_sign_byte_is_ksigns():
    from gguf.quants import IQ2_XXS

    assert np.array_equal(O.iq2xxs_sign_byte(np.arange(128)), np.frombuffer(IQ2_XXS.ksigns, dtype=np.uint8))


def test_ue4m3_table_semantics():
    t = O.ue4m3_table()
    assert t[0] == 0 and t[0x7F] == 0 and t[0x80] == 0
    assert t[0x38] == 0.5  # e4m3 1.0, halved (doubled nibble table)
    assert t[0xB8] == t[0x38]  # bit 7 ignored
    assert t[0xFF] == 240.0  # gguf-py quirk: 0xFF is not zeroed


@pytest.mark.parametrize("name", list(GEMV_CASES))
def test_gemv_ref_matches_golden(golden, name):
    d = golden("gemv.npz")
    op, R, N, K, seed = GEMV_CASES[name]
    x, w, extra = I.gemv_case(op, R, N, K, seed=seed)
    assert np.array_equal(x, d[f"{name}_x"]) and np.array_equal(w, d[f"{name}_w"]), "input builder drifted"
    deq = {"q8_0": O.dequant_q8_0, "iq2_xxs": O.dequant_iq2_xxs, "nvfp4": O.dequant_nvfp4}[op](w)
    y = O.gemv_ref(x, deq) * (float(extra["gscale"][0]) if op == "nvfp4" else 1.0)
    assert rel(y, d[f"{name}_y"]) < 1e-6


@pytest.mark.parametrize("name", ["c3", "harness"])
def test_route_ref_matches_golden(golden, name):
    d = golden("route.npz")
    x, gw, b, topk, scale = route_inputs(name)
    assert sha(x, gw, b) == str(d[f"{name}_sha"]), "input builder drifted"
    idx, wts, scores, near = O.route_ref(x, gw, b, topk, scale)
    # rows whose k-th / (k+1)-th bias-corrected scores are within 1e-6 may legitimately swap the
    # boundary expert under another summation order: compare their selected scores instead
    ok = ~near
    assert ok.sum() >= len(ok) - 1
    assert np.array_equal(idx[ok], d[f"{name}_idx"][ok])  # torch.topk order: descending value
    assert np.allclose(np.sort(wts[near], 1), np.sort(d[f"{name}_w"][near], 1), rtol=1e-5, atol=1e-6)
    assert rel(wts, d[f"{name}_w"]) < 1e-5
    assert rel(scores, d[f"{name}_scores"]) < 1e-6


def test_route_ref_ties_to_lower_index():
    x = np.zeros((1, 256), dtype=np.uint16)  # all-zero input: every score is sigmoid(0) = 0.5
    gw = np.ones((16, 256), dtype=np.float32)
    b = np.zeros(16, dtype=np.float32)
    idx, wts, _, near = O.route_ref(x, gw, b, 4, 2.0)
    assert idx.tolist() == [[0, 1, 2, 3]] and near.all()
    assert np.allclose(wts, 0.5)


def test_moe_ref_matches_golden(golden):
    d = golden("moe.npz")
    z, idx, w, b1, b2, (R, E, H, Idim, topk) = moe_inputs()
    assert sha(z, idx, w, b1, b2) == str(d["sha"]), "input builder drifted"
    d1 = O.dequant_iq2_xxs(b1.reshape(E * Idim, -1)).reshape(E, Idim, H)
    d2 = O.dequant_iq2_xxs(b2.reshape(E * H, -1)).reshape(E, H, Idim)
    out, h, part = O.moe_ref(z, idx, w, d1, d2)
    # fp64 vs torch fp32 sums may flip an occasional bf16 rounding of h / part
    assert rel(out, d["out"]) < 2e-3


def test_embed_ref_matches_golden(golden):
    d = golden("embed.npz")
    blk, ids = embed_inputs()
    assert sha(blk, ids) == str(d["sha"]), "input builder drifted"
    out = O.embed_ref(blk, ids)
    assert out.shape == (2, 9, 1024)
    assert np.array_equal(O.bf16_bits(out), d["out_bf16"])
    # ids outside [0, vocab) read row 0 (src/bolt_ops.cu:1680)
    assert np.array_equal(out[0, 3], out[1, 0]) and np.array_equal(out[1, 8], O.embed_ref(blk, np.array([0]))[0])


def test_embed_ref_empty_ids():
    blk, _ = embed_inputs()
    assert O.embed_ref(blk, np.zeros((0,), np.int64)).shape == (0, 1024)
    assert O.embed_ref(blk, np.zeros((3, 0), np.int64)).shape == (3, 0, 1024)


def bf16_ulps(a_bits, b_bits) -> np.ndarray:
    """Distance in bf16 ulps between two arrays of bf16 bit patterns (same-sign values)."""
    a = np.asarray(a_bits, np.uint16).astype(np.int32)
    b = np.asarray(b_bits, np.uint16).astype(np.int32)
    oa = np.where(a & 0x8000, 0x8000 - a, a)
    ob = np.where(b & 0x8000, 0x8000 - b, b)
    return np.abs(oa - ob)


@pytest.mark.parametrize("name", ["h4096", "h2048"])
def test_rms_norm_ref_matches_golden(golden, name):
    d = golden("norm.npz")
    x, skip, gamma, eps = norm_inputs(name)
    assert sha(x, skip, gamma) == str(d[f"{name}_sha"]), "input builder drifted"
    y, v = O.rms_norm_ref(x, gamma, eps)
    assert np.array_equal(O.bf16_bits(v), x)
    ys, s = O.rms_norm_ref(x, gamma, eps, skip=skip)
    assert np.array_equal(O.bf16_bits(s), d[f"{name}_sum"])  # bf16 add: exact
    for got, key in ((y, "rms"), (ys, "skip_rms")):
        # fp64 mean vs the harness's fp32 torch mean: at most one bf16 ulp apart, rarely
        u = bf16_ulps(O.bf16_bits(got), d[f"{name}_{key}"])
        assert u.max() <= 1 and u.mean() < 0.01
        assert rel(got, O.bf16_to_f32(d[f"{name}_{key}"])) < 1e-3


@pytest.mark.parametrize("layout", ["q8", "q4", "iq2c", "iq2n", "fp4"])
def test_legacy_dequant_matches_harness_expressions(layout):
    """The split-layout dequantisers against the reference harness's torch expressions."""
    g = I.rng(77)
    N, K = 24, 512
    w, s = I.legacy_case(layout, g, N, K)
    wt = torch.from_numpy(w)
    if layout in ("q8", "q4", "iq2c"):
        sc = torch.from_numpy(s.astype(np.int16)).view(torch.bfloat16).float()
    if layout == "q8":
        ref = ((wt.float() - 128).reshape(N, K // 32, 32) * sc.unsqueeze(-1)).reshape(N, K)
        got = O.dequant_q8_split(w, s)
    elif layout == "q4":
        q = wt.reshape(N, K // 32, 16)
        ref = ((torch.stack([(q & 15).float(), (q >> 4).float()], -1).reshape(N, K // 32, 32) - 8)
               * sc.unsqueeze(-1)).reshape(N, K)
        got = O.dequant_q4_split(w, s)
    elif layout == "iq2c":
        vals = torch.tensor([8, 25, 43, 0, -8, -25, -43, 0], dtype=torch.float32)
        code = torch.stack([wt & 15, wt >> 4], -1).reshape(N, K)
        ref = (vals[code.long()].reshape(N, K // 32, 32) * sc.unsqueeze(-1)).reshape(N, K)
        got = O.dequant_iq2_codes(w, s)
    elif layout == "iq2n":
        blk = np.concatenate([s.reshape(N, K // 256, 1).view(np.uint8), w.reshape(N, K // 256, 64)], axis=2)
        from gguf import GGMLQuantizationType as Q
        from gguf import quants

        ref = torch.from_numpy(np.asarray(quants.dequantize(blk.reshape(N, -1), Q.IQ2_XXS), np.float32).reshape(N, K))
        got = O.dequant_iq2_native(w, s)
    else:
        fp4 = torch.tensor([0, 0.5, 1, 1.5, 2, 3, 4, 6, -0.0, -0.5, -1, -1.5, -2, -3, -4, -6])
        deq = torch.stack([fp4[(wt & 15).long()], fp4[(wt >> 4).long()]], -1).reshape(N, K)
        ref = deq * torch.from_numpy(s).view(torch.float8_e4m3fn).float().repeat_interleave(16, 1)
        got = O.dequant_nvfp4_split(w, s)
    assert np.array_equal(got, ref.numpy())


def test_e4m3fn_table_matches_torch():
    ref = torch.arange(256, dtype=torch.uint8).view(torch.float8_e4m3fn).float().numpy()
    assert np.array_equal(O.e4m3fn_table(), ref, equal_nan=True)


def test_mamba_ref_matches_golden(golden):
    d = golden("mamba.npz")
    m = mamba_inputs()
    assert sha(*(m[k] for k in ("proj", "cst", "sst", "cw", "cb", "dtb", "an", "D", "nw"))) == str(d["sha"])
    y, xbc, ypre, conv_states, states = O.mamba_ref(m["proj"], m["cst"][0], m["sst"][0], m["cw"], m["cb"], m["dtb"],
                                                    m["an"], m["D"], m["nw"], m["heads"], m["n_groups"], m["eps"],
                                                    m["tmin"])
    assert rel(y, d["y"]) < 1e-5  # fp64 vs the harness's fp32 torch loop
    assert rel(states[-1], d["ssm"]) < 1e-6
    assert np.array_equal(O.bf16_bits(conv_states[-1].astype(np.float32)), d["conv"])


def test_bf16_round_matches_torch():
    v = (I.rng(9).standard_normal(4096) * 100).astype(np.float32)
    assert np.array_equal(O.bf16_round(v), torch.from_numpy(v).bfloat16().float().numpy())
