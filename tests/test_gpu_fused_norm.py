"""(Skip)RmsNorm fused into the single-row IQ2_XXS GEMV: bit-identical to the standalone norm followed
by Q4Gemv iq2=3 (same reduction order and rounding points), and within the oracle tolerance."""

import numpy as np
import pytest
import torch

import oracle as O
from gguf_onnx_ops_b200 import ops
from oracle import inputs as I
from tests.util import bf16_t, np_f32, rel, u8_t

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("N", [14336, 200, 37])
@pytest.mark.parametrize("with_skip", [True, False])
def test_fused_equals_norm_then_gemv(cuda, N, with_skip):
    g = I.rng(N + with_skip)
    K = 4096
    w = I.iq2_xxs_weights(g, (N,), K)
    x = bf16_t(I.bf16_normal(g, (1, K), 2.0), cuda)
    skip = bf16_t(I.bf16_normal(g, (1, K)), cuda) if with_skip else None
    gamma = torch.from_numpy((g.random(K) + 0.5).astype(np.float32)).to(cuda)
    wt = u8_t(w, cuda)
    y, xn, s = ops.SkipRmsNormQ4Gemv(x, skip, gamma, wt, 1e-5)
    if with_skip:
        xn_ref, s_ref = ops.SkipRmsNorm(x, skip, gamma, 1e-5)
        assert torch.equal(s, s_ref)
    else:
        xn_ref = ops.RmsNorm(x, gamma, 1e-5)
        assert s is None
    assert torch.equal(xn, xn_ref)
    y_ref = ops.Q4Gemv(xn_ref, wt, iq2=3)
    assert torch.equal(y, y_ref)
    ref = O.gemv_ref(O.bf16_bits(np_f32(xn_ref)), O.dequant_iq2_xxs(w))
    assert rel(np_f32(y), ref) < 5e-3
    assert ops.device_status() == (0, 0)


def test_fused_rejects_other_k(cuda):
    w = torch.zeros(16, 8 * 66, dtype=torch.uint8, device=cuda)
    x = torch.zeros(1, 2048, dtype=torch.bfloat16, device=cuda)
    with pytest.raises(ValueError, match="K = 4096"):
        ops.SkipRmsNormQ4Gemv(x, None, torch.ones(2048, device=cuda), w)
