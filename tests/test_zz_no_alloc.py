"""gguf_moe_verify_iq2_xxs_noalloc (library-owned scratch) against gguf_moe_verify_iq2_xxs.

Some callers cannot allocate device memory for MoeVerify's scratch outputs (h, part, meta): a
cgo / JNI / FFI host that holds only the model's buffers and has no CUDA allocator, or a decode loop
that must not enter an allocator.  The no-alloc entry point keeps that scratch in a device array of
the library.  Collected last (file name) so that it also runs after every other test has used the
library on the same device.  Both entry points are called through the C ABI; the no-alloc one twice
in a row.  Both run the same deterministic kernels, so each no-alloc result must equal the
caller-scratch result bit for bit; the caller-scratch result is also checked against the oracle
(rel-L2 <= 5e-3, the MoeVerify tolerance).
"""

import ctypes

import numpy as np
import pytest
import torch

import oracle as O
from gguf_onnx_ops_b200 import _lib
from oracle import inputs as I
from tests.util import bf16_t, rel, u8_t


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def test_noalloc_rejects_sizes_beyond_its_scratch(lib):
    # validated before any device call
    rc = lib.gguf_moe_verify_iq2_xxs_noalloc(None, None, None, None, None, None, 2, 128, 4352, 6, None)
    assert rc == _lib.GGUF_ERR_INVALID_ARGUMENT
    assert b"I <= 4096" in lib.gguf_last_error()
    rc = lib.gguf_moe_verify_iq2_xxs_noalloc(None, None, None, None, None, None, 8, 128, 1792, 17, None)
    assert rc == _lib.GGUF_ERR_INVALID_ARGUMENT
    assert b"rows*topk <= 128" in lib.gguf_last_error()
    # the caller-visible argument checks run before the scratch lookup (no device call without a GPU)
    rc = lib.gguf_moe_verify_iq2_xxs_noalloc(None, None, None, None, None, None, 2, 128, 1792, 6, None)
    assert rc == _lib.GGUF_ERR_INVALID_ARGUMENT
    assert b"null tensor pointer" in lib.gguf_last_error()


@pytest.mark.gpu
@pytest.mark.parametrize("R,E,Iw,topk", [(1, 128, 1792, 6), (3, 40, 512, 9), (8, 24, 4096, 16)])
def test_noalloc_matches_caller_scratch(cuda, lib, R, E, Iw, topk):
    g = I.rng(7000 + R * 31 + Iw)
    H = 1024
    z = I.bf16_normal(g, (R, H))
    w1 = I.iq2_xxs_weights(g, (E, Iw), H)
    w2 = I.iq2_xxs_weights(g, (E, H), Iw)
    idx = np.stack([g.choice(E, topk, replace=False) for _ in range(R)]).astype(np.int32)
    wt = g.random((R, topk)).astype(np.float32)
    wt /= wt.sum(1, keepdims=True)

    dev = cuda
    zt, it, wtt = bf16_t(z, dev), torch.from_numpy(idx).to(dev), torch.from_numpy(wt).to(dev)
    w1t, w2t = u8_t(w1, dev), u8_t(w2, dev)
    P = R * topk
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)

    out_ref = torch.empty(R, H, dtype=torch.bfloat16, device=dev)
    h = torch.empty(P, Iw, dtype=torch.bfloat16, device=dev)
    part = torch.empty(P, H, dtype=torch.float32, device=dev)
    meta = torch.empty(1 + 9 * P, dtype=torch.int32, device=dev)
    _lib.check(lib.gguf_moe_verify_iq2_xxs(_p(zt), _p(it), _p(wtt), _p(w1t), _p(w2t), _p(out_ref), _p(h), _p(part),
                                           _p(meta), R, E, Iw, topk, stream))
    outs = []
    for _ in range(2):  # two calls in a row reuse the same library-owned scratch
        o = torch.empty(R, H, dtype=torch.bfloat16, device=dev)
        _lib.check(lib.gguf_moe_verify_iq2_xxs_noalloc(_p(zt), _p(it), _p(wtt), _p(w1t), _p(w2t), _p(o), R, E, Iw,
                                                       topk, stream))
        outs.append(o)
    torch.cuda.synchronize()
    assert _lib.device_status() == (0, 0)

    ref = out_ref.float().cpu().numpy()
    assert np.isfinite(ref).all() and np.abs(ref).max() > 0
    ref_bits = out_ref.cpu().view(torch.int16).numpy()
    for o in outs:
        assert np.array_equal(o.cpu().view(torch.int16).numpy(), ref_bits)
    used = sorted(set(idx.reshape(-1).tolist()))
    d1 = {e: O.dequant_iq2_xxs(w1[e]) for e in used}
    d2 = {e: O.dequant_iq2_xxs(w2[e]) for e in used}
    oref, _, _ = O.moe_ref(z, idx, wt, d1, d2)
    assert rel(ref, O.bf16_round(oref)) < 5e-3
