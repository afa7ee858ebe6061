"""MoeRoute (bf16 gate) and Relu2 on the device.

MoeRoute: the reference's harness asserts MoeRoute(x, bf16(w), b) == MoeRouteGGUF(x, w, b) exactly
(tests/test_bolt_ops.py:314-319); the same holds here, plus oracle parity through MoeRouteGGUF's
tests.  Relu2: bit-exact against bf16(max(x, 0)^2) computed in fp32 (src/bolt_ops.cu:700-705)."""

import numpy as np
import pytest
import torch

import oracle as O
from gguf_onnx_ops_b200 import ops
from oracle import inputs as I
from tests.golden.cases import route_inputs
from tests.util import bf16_t

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("R,E,K,topk,scale", [(8, 240, 4096, 9, 5.0), (1, 128, 1024, 6, 1.0), (21, 128, 1024, 6, 1.0),
                                              (5, 512, 256, 32, 1.0), (2, 7, 256, 1, 1.0)])
def test_route_bf16_equals_gguf(cuda, R, E, K, topk, scale):
    g = I.rng(R * 17 + E)
    x = bf16_t(I.bf16_normal(g, (R, K)), cuda)
    gw = torch.from_numpy((g.standard_normal((E, K)) * 0.05).astype(np.float32)).to(cuda)
    b = torch.from_numpy((g.standard_normal(E) * 0.1).astype(np.float32)).to(cuda)
    i1, w1, s1 = ops.MoeRoute(x, gw.bfloat16(), b, topk, scale)
    i2, w2, s2 = ops.MoeRouteGGUF(x, gw, b, topk, scale)
    assert torch.equal(i1, i2) and torch.equal(w1, w2) and torch.equal(s1, s2)


@pytest.mark.parametrize("name", ["c3", "harness"])
def test_route_bf16_golden(cuda, golden, name):
    d = golden("route.npz")
    x, gw, b, topk, scale = route_inputs(name)
    idx, w, _ = ops.MoeRoute(bf16_t(x, cuda), torch.from_numpy(gw).to(cuda).bfloat16(), torch.from_numpy(b).to(cuda),
                             topk, scale)
    _, _, _, near = O.route_ref(x, gw, b, topk, scale)
    assert np.array_equal(idx.cpu().numpy()[~near], d[f"{name}_idx"][~near])
    assert O.rel_l2(w.cpu().numpy(), d[f"{name}_w"]) < 1e-5


def relu2_ref_bits(xb: np.ndarray) -> np.ndarray:
    v = O.bf16_to_f32(xb)
    r = np.where(v > 0, v, np.float32(0))  # fmaxf(x, 0): NaN -> 0
    r = np.nan_to_num(r, nan=0.0, posinf=np.inf)
    with np.errstate(over="ignore"):  # 3e38^2 -> inf, as the fp32 product on the device
        return O.bf16_bits((r * r).astype(np.float32))


@pytest.mark.parametrize("shape", [(1,), (7,), (8,), (3, 1000), (4, 4096), (2, 3, 17), (1 << 20,)])
def test_relu2_bit_exact(cuda, shape):
    g = I.rng(int(np.prod(shape)))
    xb = I.bf16_normal(g, shape, 50.0)
    y = ops.Relu2(bf16_t(xb, cuda))
    assert tuple(y.shape) == shape
    assert np.array_equal(y.cpu().view(torch.int16).numpy().view(np.uint16), relu2_ref_bits(xb))


def test_relu2_specials_and_offsets(cuda):
    vals = np.array([0.0, -0.0, 1.0, -1.0, 3e38, -3e38, np.inf, -np.inf, np.nan, 1e-40, 2.0 ** -70], np.float32)
    xb = O.bf16_bits(vals)
    y = ops.Relu2(bf16_t(xb, cuda))
    got = y.cpu().view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(got, relu2_ref_bits(xb))
    # unaligned sub-tensor (scalar kernel) equals the aligned result
    big = bf16_t(I.bf16_normal(I.rng(3), (1027,), 10.0), cuda)
    part = big[3:1027]
    out = torch.empty_like(part)
    ops.relu2_into(part, out, part.numel())
    assert torch.equal(out, ops.Relu2(part.clone()))
    assert ops.Relu2(torch.empty(0, dtype=torch.bfloat16, device=cuda)).numel() == 0
