"""RmsNorm / SkipRmsNorm (src/bolt_ops.cu:1692-1864) on the device against the reference test's
torch expressions (golden) and the oracle: sum bit-exact, y within one bf16 ulp (the reference's
own bar is rel < 1e-3, tests/test_bolt_ops.py:323-337)."""

import numpy as np
import pytest
import torch

import oracle as O
from gguf_onnx_ops_b200 import ops
from oracle import inputs as I
from tests.golden.cases import norm_inputs
from tests.test_oracle import bf16_ulps
from tests.util import bf16_t, rel

pytestmark = pytest.mark.gpu


def bits(t: torch.Tensor) -> np.ndarray:
    return t.cpu().view(torch.int16).numpy().view(np.uint16)


def check_close(got_bits, ref_bits, frac=0.01):
    u = bf16_ulps(got_bits, ref_bits)
    assert u.max() <= 1, f"max {u.max()} ulps"
    assert u.mean() < frac
    assert rel(O.bf16_to_f32(got_bits), O.bf16_to_f32(ref_bits)) < 1e-3


@pytest.mark.parametrize("name", ["h4096", "h2048"])
def test_norm_golden(cuda, golden, name):
    d = golden("norm.npz")
    x, skip, gamma, eps = norm_inputs(name)
    xt, st, gt = bf16_t(x, cuda), bf16_t(skip, cuda), torch.from_numpy(gamma).to(cuda)
    check_close(bits(ops.RmsNorm(xt, gt, eps)), d[f"{name}_rms"])
    y, s = ops.SkipRmsNorm(xt, st, gt, eps)
    assert np.array_equal(bits(s), d[f"{name}_sum"])
    check_close(bits(y), d[f"{name}_skip_rms"])
    (y_only,) = ops.SkipRmsNorm(xt, st, gt, eps, return_sum=False)  # optional 2nd output omitted
    assert torch.equal(y_only, y)


@pytest.mark.parametrize("R,H", [(1, 8), (3, 64), (1, 4096), (16, 4096), (1000, 4096), (5, 2048), (2, 5120),
                                 (7, 8192), (4, 12288), (3, 16384), (2, 20480), (3, 32776)])
@pytest.mark.parametrize("with_skip", [False, True])
def test_norm_shapes_vs_oracle(cuda, R, H, with_skip):
    g = I.rng(R * 7919 + H)
    x = I.bf16_normal(g, (R, H), 3.0)
    skip = I.bf16_normal(g, (R, H)) if with_skip else None
    gamma = (g.random(H) + 0.5).astype(np.float32)
    eps = 1e-6
    y_ref, v_ref = O.rms_norm_ref(x, gamma, eps, skip=skip)
    xt, gt = bf16_t(x, cuda), torch.from_numpy(gamma).to(cuda)
    if with_skip:
        y, s = ops.SkipRmsNorm(xt, bf16_t(skip, cuda), gt, eps)
        assert np.array_equal(bits(s), O.bf16_bits(v_ref))
    else:
        y = ops.RmsNorm(xt, gt, eps)
    check_close(bits(y), O.bf16_bits(y_ref))


def test_norm_extreme_rows(cuda):
    """Zero rows (rsqrt(eps)), tiny rows (mean underflows toward eps), one huge element per row."""
    H = 4096
    x = np.zeros((4, H), np.float32)
    x[1] = 1e-20
    x[2, 17] = 3e4
    x[2, 18:40] = -2.5
    x[3] = np.linspace(-100, 100, H)
    xb = O.bf16_bits(x)
    gamma = np.linspace(0.5, 1.5, H).astype(np.float32)
    y_ref, _ = O.rms_norm_ref(xb, gamma, 1e-5)
    y = ops.RmsNorm(bf16_t(xb, cuda), torch.from_numpy(gamma).to(cuda), 1e-5)
    check_close(bits(y), O.bf16_bits(y_ref))
    assert not torch.isnan(y.float()).any()


def test_norm_multi_dim_and_empty(cuda):
    g = I.rng(5)
    x = bf16_t(I.bf16_normal(g, (2, 3, 512)), cuda)
    gamma = torch.rand(512, device=cuda) + 0.5
    y = ops.RmsNorm(x, gamma)
    assert y.shape == x.shape
    assert torch.equal(y.reshape(6, 512), ops.RmsNorm(x.reshape(6, 512), gamma))
    e = ops.RmsNorm(torch.empty(0, 512, dtype=torch.bfloat16, device=cuda), gamma)
    assert e.shape == (0, 512)


def test_norm_deterministic_across_grid_sizes(cuda):
    """Rows processed by different CTAs / grid-stride passes normalise identically."""
    g = I.rng(11)
    row = I.bf16_normal(g, (1, 4096))
    x = np.repeat(row, 2000, axis=0)
    gamma = torch.rand(4096, device=cuda) + 0.5
    y = ops.RmsNorm(bf16_t(x, cuda), gamma)
    assert (y == y[0]).all()
    assert torch.equal(y[:1], ops.RmsNorm(bf16_t(row, cuda), gamma))


def test_norm_rejects_bad_shapes(cuda):
    x = torch.zeros(2, 12, dtype=torch.bfloat16, device=cuda)
    with pytest.raises(ValueError, match="multiple of 8"):
        ops.RmsNorm(x, torch.ones(12, device=cuda))
    x = torch.zeros(2, 16, dtype=torch.bfloat16, device=cuda)
    with pytest.raises(ValueError, match="gamma size mismatch"):
        ops.RmsNorm(x, torch.ones(8, device=cuda))
    with pytest.raises(ValueError, match="skip shape mismatch"):
        ops.SkipRmsNorm(x, torch.zeros(2, 8, dtype=torch.bfloat16, device=cuda), torch.ones(16, device=cuda))
    big = torch.zeros(2, 40, dtype=torch.bfloat16, device=cuda)
    with pytest.raises(ValueError, match="16-byte aligned"):
        ops.RmsNorm(big[:, 8:24].contiguous()[:, :].reshape(-1)[4:20].reshape(1, 16), torch.ones(16, device=cuda))
