"""MambaStep / MambaVerify (+ GGUF variants), src/bolt_ops.cu:68-378, against the golden fixture
(the reference harness's torch loop, tests/test_bolt_ops.py:389-413) and the fp64 oracle.  Bars:
y rel-L2 < 5e-3 (reference: 1e-2), states rel < 1e-5 (reference: 1e-4), conv state exact; Verify
equals chained Steps bit for bit; the GGUF ops equal the bf16 ops bit for bit on bf16-valued weights
(the reference asserts both, :340-372)."""

import numpy as np
import pytest
import torch

import oracle as O
from gguf_onnx_ops_b200 import ops
from tests.golden.cases import mamba_inputs
from tests.util import bf16_t, np_f32, rel

pytestmark = pytest.mark.gpu


def dev_inputs(m, dev, gguf=False):
    cw = torch.from_numpy(m["cw"]).to(dev)
    cb = torch.from_numpy(m["cb"]).to(dev)
    if not gguf:
        cw, cb = cw.bfloat16(), cb.bfloat16()
    return dict(proj=bf16_t(m["proj"], dev), conv_state=bf16_t(m["cst"], dev), ssm_state=torch.from_numpy(m["sst"]).to(dev),
                conv_w=cw, conv_b=cb, dt_bias=torch.from_numpy(m["dtb"]).to(dev), A_neg=torch.from_numpy(m["an"]).to(dev),
                D=torch.from_numpy(m["D"]).to(dev), norm_w=torch.from_numpy(m["nw"]).to(dev))


def attrs(m):
    return dict(heads=m["heads"], n_groups=m["n_groups"], epsilon=m["eps"], time_step_min=m["tmin"])


def bits(t):
    return t.cpu().view(torch.int16).numpy().view(np.uint16)


def test_mamba_golden(cuda, golden):
    d = golden("mamba.npz")
    m = mamba_inputs()
    y, cs, ss, xbc, ypre = ops.MambaStep(**dev_inputs(m, cuda), **attrs(m))
    assert rel(np_f32(y), d["y"]) < 5e-3
    assert rel(ss.cpu().numpy()[0], d["ssm"]) < 1e-5
    assert np.array_equal(bits(cs)[0], d["conv"])
    assert ops.device_status() == (0, 0)


@pytest.mark.parametrize("R,heads,ng", [(1, 128, 8), (2, 128, 8), (8, 128, 8), (16, 32, 4), (5, 4, 1), (3, 24, 3)])
def test_mamba_step_vs_oracle(cuda, R, heads, ng):
    m = mamba_inputs(R=R, heads=heads, n_groups=ng, seed=R * 31 + heads)
    y, cs, ss, xbc, ypre = ops.MambaStep(**dev_inputs(m, cuda), **attrs(m))
    y_ref, xbc_ref, ypre_ref, conv_states, states = O.mamba_ref(
        m["proj"], m["cst"][0], m["sst"][0], m["cw"], m["cb"], m["dtb"], m["an"], m["D"], m["nw"], heads, ng,
        m["eps"], m["tmin"])
    assert rel(np_f32(y), y_ref) < 5e-3
    xb = bits(xbc)
    xr = O.bf16_bits(xbc_ref)
    assert (xb != xr).mean() < 0.01  # fp32 conv vs fp64: an occasional bf16 rounding flip
    assert rel(np_f32(xbc), xbc_ref) < 1e-3
    assert rel(ypre.cpu().numpy(), ypre_ref) < 1e-3
    assert rel(ss.cpu().numpy()[0], states[-1]) < 1e-3
    assert np.array_equal(bits(cs)[0], O.bf16_bits(conv_states[-1].astype(np.float32)))


@pytest.mark.parametrize("R,sel", [(8, 3), (4, 0), (1, 0), (16, 15)])
def test_mamba_verify_equals_chained_steps(cuda, R, sel):
    m = mamba_inputs(R=R, heads=32, n_groups=4, rows_state=R, seed=7 + R)
    inp = dev_inputs(m, cuda)
    at = attrs(m)
    row = torch.tensor([sel], dtype=torch.int32, device=cuda)
    yv, csv, ssv, xbv, ypv = ops.MambaVerify(**inp, state_row=row, **at)
    cs, ss = inp["conv_state"][sel:sel + 1].clone(), inp["ssm_state"][sel:sel + 1].clone()
    for r in range(R):
        step = dict(inp, proj=inp["proj"][r:r + 1].contiguous(), conv_state=cs, ssm_state=ss)
        y, cs, ss, xb, yp = ops.MambaStep(**step, **at)
        assert torch.equal(y[0], yv[r]) and torch.equal(xb[0], xbv[r]) and torch.equal(yp[0], ypv[r]), r
        assert torch.equal(cs[0], csv[r]) and torch.equal(ss[0], ssv[r]), r


def test_mamba_gguf_equals_bf16(cuda):
    m = mamba_inputs(R=8, heads=32, n_groups=4, rows_state=8, seed=99)
    at = attrs(m)
    a = ops.MambaStep(**dev_inputs(m, cuda), **at)
    b = ops.MambaStepGGUF(**dev_inputs(m, cuda, gguf=True), **at)
    # Step writes state row 0 only (rows >= 1 of the state outputs are not written, as in the reference)
    a = (a[0], a[1][0], a[2][0], a[3], a[4])
    b = (b[0], b[1][0], b[2][0], b[3], b[4])
    assert all(torch.equal(x, y) for x, y in zip(a, b))
    row = torch.tensor([2], dtype=torch.int32, device=cuda)
    a = ops.MambaVerify(**dev_inputs(m, cuda), state_row=row, **at)
    b = ops.MambaVerifyGGUF(**dev_inputs(m, cuda, gguf=True), state_row=row, **at)
    assert all(torch.equal(x, y) for x, y in zip(a, b))


def test_mamba_bad_state_row_is_reported(cuda):
    """A device-side state row outside [0, Rs) is read as row 0 and reported (bounds-checked read)."""
    m = mamba_inputs(R=2, heads=4, n_groups=2, rows_state=2, seed=3)
    inp = dev_inputs(m, cuda)
    at = attrs(m)
    ref = ops.MambaVerify(**inp, state_row=torch.tensor([0], dtype=torch.int32, device=cuda), **at)
    assert ops.device_status() == (0, 0)
    bad = ops.MambaVerify(**inp, state_row=torch.tensor([7], dtype=torch.int32, device=cuda), **at)
    assert ops.device_status() == (4, 6)  # GGUF_ERR_DEVICE, the bad-state-row site
    assert all(torch.equal(x, y) for x, y in zip(ref, bad))


def test_mamba_rejects_bad_shapes(cuda):
    m = mamba_inputs(R=2, heads=4, n_groups=2, seed=1)
    inp = dev_inputs(m, cuda)
    with pytest.raises(ValueError, match="head_dim=64"):
        ops.MambaStep(**inp, **attrs(m), head_dim=32)
    with pytest.raises(ValueError, match="bad proj width"):
        ops.MambaStep(**dict(inp, proj=inp["proj"][:, 1:].contiguous()), **attrs(m))
    with pytest.raises(ValueError, match="state buffer"):
        ops.MambaVerify(**inp, state_row=torch.zeros(1, dtype=torch.int32, device=cuda), **attrs(m))
