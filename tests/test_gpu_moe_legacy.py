"""MoeDecode and MoeVerify iq2 = 0 / 1 / 2 (legacy split expert layouts) against the oracle's
per-(row, expert) relu^2 loop on the split dequantisers (the reference harness's
test_moe_decode / test_moe_iq2 / test_moe_iq2_native, tests/test_bolt_ops.py:128-153, 183-207,
246-267).  Bars: out within rel-L2 5e-3 (the reference's: 1e-2), h / part elementwise close."""

import numpy as np
import pytest
import torch

import oracle as O
from gguf_onnx_ops_b200 import ops
from oracle import inputs as I
from tests.util import bf16_t, np_f32, rel, u8_t

pytestmark = pytest.mark.gpu


def experts(layout, g, E, I_, dev):
    """Per-expert fc1 [I, 1024] and fc2 [1024, I] in a split layout, device tensors and dequantised copies."""
    w1, s1 = I.legacy_case(layout, g, E * I_, 1024)
    w2, s2 = I.legacy_case(layout, g, E * 1024, I_)
    deq = {"q4": O.dequant_q4_split, "iq2c": O.dequant_iq2_codes, "iq2n": O.dequant_iq2_native}[layout]
    if layout == "iq2n":
        d1, d2 = deq(w1, s1).reshape(E, I_, 1024), deq(w2, s2).reshape(E, 1024, I_)
        t1 = u8_t(w1, dev).reshape(E, I_, 32, 8)
        t2 = u8_t(w2, dev).reshape(E, 1024, I_ // 32, 8)
    else:
        d1, d2 = deq(w1, s1).reshape(E, I_, 1024), deq(w2, s2).reshape(E, 1024, I_)
        t1 = u8_t(w1, dev).reshape(E, I_, 512)
        t2 = u8_t(w2, dev).reshape(E, 1024, I_ // 2)
    return t1, bf16_t(s1, dev), t2, bf16_t(s2, dev), d1, d2


def moe_inputs(g, R, E, topk):
    z = I.bf16_normal(g, (R, 1024), 0.5)
    idx = np.stack([g.permutation(E)[:topk] for _ in range(R)]).astype(np.int32)
    w = g.random((R, topk)).astype(np.float32)
    return z, idx, w


def check(out, h, part, z, idx, w, d1, d2):
    ref, h_ref, p_ref = O.moe_ref(z, idx, w, d1, d2)
    assert rel(np_f32(out), O.bf16_round(ref)) < 5e-3
    assert rel(np_f32(h), h_ref) < 5e-3
    assert rel(np_f32(part), p_ref) < 5e-3


@pytest.mark.parametrize("layout,iq2", [("q4", 0), ("iq2c", 1), ("iq2n", 2)])
@pytest.mark.parametrize("R,E,I_,topk", [(1, 16, 512, 6), (4, 16, 256, 9), (8, 12, 512, 6)])
def test_moe_verify_legacy(cuda, layout, iq2, R, E, I_, topk):
    g = I.rng(R * 100 + E + iq2)
    t1, s1, t2, s2, d1, d2 = experts(layout, g, E, I_, cuda)
    z, idx, w = moe_inputs(g, R, E, topk)
    out, h, part, meta = ops.MoeVerify(bf16_t(z, cuda), torch.from_numpy(idx).to(cuda), torch.from_numpy(w).to(cuda),
                                       t1, s1, t2, s2, topk=topk, iq2=iq2)
    check(out, h, part, z, idx, w, d1, d2)
    m = meta.cpu().numpy()
    U = len(dict.fromkeys(idx.reshape(-1).tolist()))
    assert m[0] == U and list(m[1:1 + U]) == list(dict.fromkeys(idx.reshape(-1).tolist()))


@pytest.mark.parametrize("R,E,I_,topk", [(1, 16, 512, 9), (8, 16, 512, 9), (21, 20, 256, 9), (40, 8, 128, 4)])
def test_moe_decode(cuda, R, E, I_, topk):
    """MoeDecode has no row limit: rows beyond 8 (or 128 pairs) run in groups."""
    g = I.rng(R * 7 + E)
    t1, s1, t2, s2, d1, d2 = experts("q4", g, E, I_, cuda)
    z, idx, w = moe_inputs(g, R, E, topk)
    out, h, part = ops.MoeDecode(bf16_t(z, cuda), torch.from_numpy(idx).to(cuda), torch.from_numpy(w).to(cuda),
                                 t1, s1, t2, s2, topk=topk)
    check(out, h, part, z, idx, w, d1, d2)


def test_moe_decode_equals_verify_iq2_0(cuda):
    """The same pairs computed grouped (MoeVerify) and in row groups (MoeDecode) agree exactly."""
    g = I.rng(5)
    t1, s1, t2, s2, _, _ = experts("q4", g, 16, 256, cuda)
    z, idx, w = moe_inputs(g, 6, 16, 6)
    args = (bf16_t(z, cuda), torch.from_numpy(idx).to(cuda), torch.from_numpy(w).to(cuda), t1, s1, t2, s2)
    o1, h1, p1, _ = ops.MoeVerify(*args, topk=6, iq2=0)
    o2, h2, p2 = ops.MoeDecode(*args, topk=6)
    assert torch.equal(o1, o2) and torch.equal(h1, h2) and torch.equal(p1, p2)
    assert ops.device_status() == (0, 0)
