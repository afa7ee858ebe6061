"""Host-side mirror of the reference's ONNX Runtime custom-op interface for the hot path.

Each function takes the op's inputs (torch CUDA tensors, ``None`` for an omitted optional input
``""``) and attributes, validates them with the reference's constraints and messages, allocates
the outputs with the reference's shapes (as ``KernelContext::GetOutput`` would) and calls the
C ABI of libgguf_onnx_ops.so on the current torch CUDA stream.

    Q8Gemv(x, w, scales=None, gguf=1)                  -> y        src/bolt_ops.cu:1592-1643, :2018-2027
    Q4Gemv(x, w, scales=None, iq2=3)                   -> y        src/bolt_ops.cu:1592-1643, :2028-2037
    Nvfp4Gemv(x, w, w_scale, gscale, gguf=1)           -> y        src/bolt_ops.cu:1411-1469, :2004-2016
    Q8Embed(w, input_ids)                              -> out      src/bolt_ops.cu:1645-1690, :2038-2044
    RmsNorm(x, gamma, epsilon)                         -> y        src/bolt_ops.cu:1692-1864, :2045-2051
    SkipRmsNorm(x, skip, gamma, epsilon)               -> y, sum   src/bolt_ops.cu:1692-1864, :2052-2061
    Relu2(x)                                           -> y        src/bolt_ops.cu:700-726, :1997-2003
    MoeRouteGGUF(x, gate_w, bias, topk, scale)         -> idx, weights, scores    src/bolt_ops.cu:512-546
    MoeRoute(x, gate_w_bf16, bias, topk, scale)        -> idx, weights, scores    src/bolt_ops.cu:513-547, :1947
    MoeVerify(z, idx, w, fc1_w, fc1_s, fc2_w, fc2_s=None, topk, iq2=3) -> out, h, part, meta
                                                                   src/bolt_ops.cu:1327-1409, :1981-1996
    MoeDecode(z, idx, w, fc1_w, fc1_s, fc2_w, fc2_s, topk)            -> out, h, part
                                                                   src/bolt_ops.cu:664-699, :1967-1980
    MambaStep / MambaStepGGUF / MambaVerify / MambaVerifyGGUF       -> y, conv_state, ssm_state, xbc, ypre
                                                                   src/bolt_ops.cu:68-378, :1886-1946

Every weight layout of the GEMVs is implemented: the GGUF ones (``gguf=1`` / ``iq2=3``) and the
legacy split layouts (``gguf=0``, ``iq2`` in 0..2, through ``gguf_gemv_legacy``).  The lower-level
``*_into`` functions write into caller-provided outputs (no allocation), for graph capture and
benchmarking.
"""

from __future__ import annotations

import torch

from . import _lib
from ._lib import check, load

Q8_0_BYTES, IQ2_XXS_BYTES, NVFP4_BYTES = 34, 66, 36


def _stream(stream=None) -> int:
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _need(t, name, dtype, op):
    if t is None:
        raise ValueError(f"{op}: Missing required tensor input {name}")
    if not t.is_cuda:
        raise ValueError(f"{op}: {name} must be a CUDA tensor")
    if t.dtype != dtype:
        raise ValueError(f"{op}: {name} must be {dtype}, got {t.dtype}")
    if not t.is_contiguous():
        raise ValueError(f"{op}: {name} must be contiguous")


# ------------------------------------------------------------------------------------------------
# GEMVs
# ------------------------------------------------------------------------------------------------
def q8_0_gemv_into(x: torch.Tensor, w: torch.Tensor, y: torch.Tensor, R: int, N: int, K: int, stream=None) -> None:
    check(load().gguf_q8_0_gemv(_ptr(x), _ptr(w), _ptr(y), R, N, K, _stream(stream)))


def iq2_xxs_gemv_into(x: torch.Tensor, w: torch.Tensor, y: torch.Tensor, R: int, N: int, K: int, stream=None) -> None:
    check(load().gguf_iq2_xxs_gemv(_ptr(x), _ptr(w), _ptr(y), R, N, K, _stream(stream)))


def nvfp4_gemv_into(x, w, gscale, y, R: int, N: int, K: int, stream=None) -> None:
    check(load().gguf_nvfp4_gemv(_ptr(x), _ptr(w), _ptr(gscale), _ptr(y), R, N, K, _stream(stream)))


def _gemv_shapes(x: torch.Tensor, w: torch.Tensor):
    K = x.shape[-1]
    R = x.numel() // K if K else 0
    N = w.shape[0]
    return R, N, K


def gemv_legacy_into(layout: int, x, w, scales, gscale, y, R: int, N: int, K: int, stream=None) -> None:
    check(load().gguf_gemv_legacy(layout, _ptr(x), _ptr(w), _ptr(scales), _ptr(gscale), _ptr(y), R, N, K,
                                  _stream(stream)))


def _legacy(op, layout, x, w, scales, gscale=None):
    _need(x, "x", torch.bfloat16, op)
    _need(w, "w", torch.uint8, op)
    R, N, K = _gemv_shapes(x, w)
    y = torch.empty(*x.shape[:-1], N, dtype=torch.bfloat16, device=x.device)
    gemv_legacy_into(layout, x, w, scales, gscale, y, R, N, K)
    return y


def Q8Gemv(x: torch.Tensor, w: torch.Tensor, scales: torch.Tensor | None = None, gguf: int = 1) -> torch.Tensor:
    """y[..., N] = x[..., K] @ deq(W)^T.  gguf=1: raw GGUF Q8_0 blocks W [N, (K/32)*34]; gguf=0: the
    split layout W u8 [N, K/32, 32] = q + 128 with bf16 scales [N, K/32] (src/bolt_ops.cu:1617-1640)."""
    if gguf != 1:
        _need(w, "w", torch.uint8, "Q8Gemv")
        _need(scales, "scales", torch.bfloat16, "Q8Gemv")
        K = x.shape[-1]
        if K % 32 != 0 or w.dim() < 2 or w.shape[1] * 32 != K or w.numel() != w.shape[0] * K \
                or scales.numel() != w.shape[0] * (K // 32):
            raise ValueError("QGemv: K mismatch")
        return _legacy("Q8Gemv", _lib.GGUF_LAYOUT_Q8_SPLIT, x, w, scales)
    _need(x, "x", torch.bfloat16, "Q8Gemv")
    _need(w, "w", torch.uint8, "Q8Gemv")
    R, N, K = _gemv_shapes(x, w)
    if K % 64 != 0 or w.numel() != N * (K // 32) * Q8_0_BYTES or R < 1 or R > 16:
        raise ValueError("Q8Gemv gguf=1: needs B [N, (K/32)*34] and 1..16 rows")
    y = torch.empty(*x.shape[:-1], N, dtype=torch.bfloat16, device=x.device)
    q8_0_gemv_into(x, w, y, R, N, K)
    return y


def Q4Gemv(x: torch.Tensor, w: torch.Tensor, scales: torch.Tensor | None = None, iq2: int = 3) -> torch.Tensor:
    """y[..., N] = x[..., K] @ deq(W)^T.  iq2=3: raw GGUF IQ2_XXS super-blocks W [N, (K/256)*66];
    iq2=0: 4-bit W [N, K/32, 16] (n - 8) with bf16 scales [N, K/32]; iq2=1: 3-bit IQ2 codes in the
    same packing; iq2=2: IQ2_XXS records W [N, K/32, 8] with fp16 d bits [N, K/256] carried in a
    bf16-typed tensor (src/bolt_ops.cu:1593-1643)."""
    if iq2 != 3:
        if iq2 not in (0, 1, 2):
            raise NotImplementedError(f"Q4Gemv: unknown iq2={iq2}")
        _need(w, "w", torch.uint8, "Q4Gemv")
        _need(scales, "scales", torch.bfloat16, "Q4Gemv")
        K = x.shape[-1]
        N = w.shape[0]
        if iq2 == 2:
            if K % 256 != 0 or w.dim() != 3 or w.shape[1] * 32 != K or w.shape[2] != 8 or scales.numel() != N * (K // 256):
                raise ValueError("Q4Gemv iq2=2: needs B [N, K/32, 8] and 1..16 rows")
            layout = _lib.GGUF_LAYOUT_IQ2_NATIVE
        else:
            if K % 32 != 0 or w.dim() < 2 or w.shape[1] * 32 != K or w.numel() != N * K // 2 \
                    or scales.numel() != N * (K // 32):
                raise ValueError("QGemv: K mismatch")
            layout = _lib.GGUF_LAYOUT_IQ2_CODES if iq2 == 1 else _lib.GGUF_LAYOUT_Q4_SPLIT
        return _legacy("Q4Gemv", layout, x, w, scales)
    _need(x, "x", torch.bfloat16, "Q4Gemv")
    _need(w, "w", torch.uint8, "Q4Gemv")
    R, N, K = _gemv_shapes(x, w)
    if K % 256 != 0 or w.numel() != N * (K // 256) * IQ2_XXS_BYTES or R < 1 or R > 16:
        raise ValueError("Q4Gemv iq2=3: needs B [N, (K/256)*66] and 1..16 rows")
    y = torch.empty(*x.shape[:-1], N, dtype=torch.bfloat16, device=x.device)
    iq2_xxs_gemv_into(x, w, y, R, N, K)
    return y


def Nvfp4Gemv(x: torch.Tensor, w: torch.Tensor, w_scale: torch.Tensor | None, gscale: torch.Tensor,
              gguf: int = 1) -> torch.Tensor:
    """y[..., N] = gscale * (x[..., K] @ deq(W)^T).  gguf=1: raw GGUF NVFP4 blocks W [N, (K/64)*36];
    gguf=0: E2M1 nibbles W [N, K/2] with e4m3fn scales [N, K/16] (src/bolt_ops.cu:1411-1469)."""
    if gguf != 1:
        _need(w, "w", torch.uint8, "Nvfp4Gemv")
        _need(w_scale, "ws", torch.uint8, "Nvfp4Gemv")
        _need(gscale, "gscale", torch.float32, "Nvfp4Gemv")
        K = x.shape[-1]
        if K % 32 != 0 or w.dim() != 2 or w.shape[1] * 2 != K or w_scale.numel() != w.shape[0] * (K // 16):
            raise ValueError("Nvfp4Gemv: K mismatch (K % 32 required)")
        return _legacy("Nvfp4Gemv", _lib.GGUF_LAYOUT_NVFP4_SPLIT, x, w, w_scale, gscale)
    _need(x, "x", torch.bfloat16, "Nvfp4Gemv")
    _need(w, "w", torch.uint8, "Nvfp4Gemv")
    _need(gscale, "gscale", torch.float32, "Nvfp4Gemv")
    R, N, K = _gemv_shapes(x, w)
    if K % 64 != 0 or w.numel() != N * (K // 64) * NVFP4_BYTES or R < 1 or R > 16:
        raise ValueError("Nvfp4Gemv gguf=1: needs w [N, (K/64)*36] and 1..16 rows")
    y = torch.empty(*x.shape[:-1], N, dtype=torch.bfloat16, device=x.device)
    nvfp4_gemv_into(x, w, gscale, y, R, N, K)
    return y


# ------------------------------------------------------------------------------------------------
# Embedding
# ------------------------------------------------------------------------------------------------
def q8_0_embed_into(w, ids, out, vocab: int, row_bytes: int, R: int, stream=None) -> None:
    check(load().gguf_q8_0_embed(_ptr(w), _ptr(ids), _ptr(out), vocab, row_bytes, R, _stream(stream)))


def Q8Embed(w: torch.Tensor, input_ids: torch.Tensor) -> torch.Tensor:
    """Gather + dequantise rows of a raw GGUF Q8_0 table w [vocab, (K/32)*34] -> bf16 [..., K]
    (src/bolt_ops.cu:1645-1690, :2038-2044); out-of-range ids read row 0."""
    _need(w, "w", torch.uint8, "Q8Embed")
    _need(input_ids, "input_ids", torch.int64, "Q8Embed")
    vocab = w.shape[0]
    if vocab <= 0 or w.numel() % vocab != 0:
        raise ValueError("Q8Embed: invalid weight shape")
    row_bytes = w.numel() // vocab
    if row_bytes <= 0 or row_bytes % Q8_0_BYTES != 0:
        raise ValueError("Q8Embed: row_bytes must be a positive multiple of 34")
    K = row_bytes // Q8_0_BYTES * 32
    out = torch.empty(*input_ids.shape, K, dtype=torch.bfloat16, device=w.device)
    q8_0_embed_into(w, input_ids, out, vocab, row_bytes, input_ids.numel())
    return out


# ------------------------------------------------------------------------------------------------
# Norms
# ------------------------------------------------------------------------------------------------
def rms_norm_into(x, skip, gamma, y, sum_out, R: int, H: int, eps: float, stream=None) -> None:
    check(load().gguf_rms_norm(_ptr(x), _ptr(skip), _ptr(gamma), _ptr(y), _ptr(sum_out), R, H, eps, _stream(stream)))


def _norm_shapes(x, gamma, op):
    _need(x, "x", torch.bfloat16, op)
    _need(gamma, "gamma", torch.float32, op)
    if x.dim() < 1:
        raise ValueError(f"{op}: input must be at least 1D")
    H = x.shape[-1]
    if H <= 0 or H % 8 != 0:
        raise ValueError(f"{op}: hidden size H must be a positive multiple of 8")
    if gamma.numel() != H:
        raise ValueError(f"{op}: gamma size mismatch")
    return x.numel() // H, H


def RmsNorm(x: torch.Tensor, gamma: torch.Tensor, epsilon: float = 1e-5) -> torch.Tensor:
    """y = bf16(bf16(gamma) * x * rsqrt(mean(x^2) + eps)) over the last dim (src/bolt_ops.cu:1692-1864)."""
    R, H = _norm_shapes(x, gamma, "RmsNorm")
    y = torch.empty_like(x)
    rms_norm_into(x, None, gamma, y, None, R, H, epsilon)
    return y


def SkipRmsNorm(x: torch.Tensor, skip: torch.Tensor, gamma: torch.Tensor, epsilon: float = 1e-5,
                return_sum: bool = True):
    """sum = bf16(x + skip); y = RmsNorm(sum).  Returns (y, sum), or (y,) when the optional second
    output is not requested (src/bolt_ops.cu:1830-1856)."""
    R, H = _norm_shapes(x, gamma, "SkipRmsNorm")
    _need(skip, "skip", torch.bfloat16, "SkipRmsNorm")
    if skip.numel() != x.numel():
        raise ValueError("SkipRmsNorm: skip shape mismatch")
    y = torch.empty_like(x)
    s = torch.empty_like(x) if return_sum else None
    rms_norm_into(x, skip, gamma, y, s, R, H, epsilon)
    return (y, s) if return_sum else (y,)


def rms_norm_iq2_xxs_gemv_into(x, skip, gamma, eps, w, y, x_norm, sum_out, N: int, K: int, stream=None) -> None:
    check(load().gguf_rms_norm_iq2_xxs_gemv(_ptr(x), _ptr(skip), _ptr(gamma), eps, _ptr(w), _ptr(y), _ptr(x_norm),
                                            _ptr(sum_out), N, K, _stream(stream)))


def SkipRmsNormQ4Gemv(x: torch.Tensor, skip: torch.Tensor | None, gamma: torch.Tensor, w: torch.Tensor,
                      epsilon: float = 1e-5):
    """Fused decode step (an extension, not a reference op): y = Q4Gemv iq2=3(RmsNorm(x [+ skip])) for one
    row, K = 4096.  Returns (y [1, N], x_norm [1, K], sum [1, K] or None), bit-identical to SkipRmsNorm /
    RmsNorm followed by Q4Gemv."""
    _need(x, "x", torch.bfloat16, "SkipRmsNormQ4Gemv")
    _need(gamma, "gamma", torch.float32, "SkipRmsNormQ4Gemv")
    _need(w, "w", torch.uint8, "SkipRmsNormQ4Gemv")
    K = x.shape[-1]
    N = w.shape[0]
    if x.numel() != K or K != 4096 or gamma.numel() != K or w.numel() != N * (K // 256) * IQ2_XXS_BYTES:
        raise ValueError("SkipRmsNormQ4Gemv: needs one row of K = 4096 and w [N, (K/256)*66]")
    if skip is not None:
        _need(skip, "skip", torch.bfloat16, "SkipRmsNormQ4Gemv")
    y = torch.empty(1, N, dtype=torch.bfloat16, device=x.device)
    x_norm = torch.empty(1, K, dtype=torch.bfloat16, device=x.device)
    s = torch.empty(1, K, dtype=torch.bfloat16, device=x.device) if skip is not None else None
    rms_norm_iq2_xxs_gemv_into(x, skip, gamma, epsilon, w, y, x_norm, s, N, K)
    return y, x_norm, s


# ------------------------------------------------------------------------------------------------
# Router + MoE
# ------------------------------------------------------------------------------------------------
def moe_route_into(x, gate_w, bias, idx, weights, scores, R, K, E, topk, scale, stream=None) -> None:
    check(load().gguf_moe_route(_ptr(x), _ptr(gate_w), _ptr(bias), _ptr(idx), _ptr(weights), _ptr(scores),
                                R, K, E, topk, float(scale), _stream(stream)))


def MoeRouteGGUF(x: torch.Tensor, gate_w: torch.Tensor, bias: torch.Tensor, topk: int, scale: float):
    """Sigmoid router with F32 GGUF gate weights (rounded to bf16) and bias-corrected top-k."""
    _need(x, "x", torch.bfloat16, "MoeRouteGGUF")
    _need(gate_w, "gate_w", torch.float32, "MoeRouteGGUF")
    _need(bias, "bias", torch.float32, "MoeRouteGGUF")
    R, K = x.shape
    E = gate_w.shape[0]
    if E > 512 or K % 256 != 0 or topk > 32 or gate_w.shape[1] != K or bias.numel() != E:
        raise ValueError("MoeRoute: unsupported shape")
    idx = torch.empty(R, topk, dtype=torch.int32, device=x.device)
    wts = torch.empty(R, topk, dtype=torch.float32, device=x.device)
    scores = torch.empty(R, E, dtype=torch.float32, device=x.device)
    moe_route_into(x, gate_w, bias, idx, wts, scores, R, K, E, topk, scale)
    return idx, wts, scores


def moe_route_bf16_into(x, gate_w, bias, idx, wts, scores, R, K, E, topk, scale, stream=None) -> None:
    check(load().gguf_moe_route_bf16(_ptr(x), _ptr(gate_w), _ptr(bias), _ptr(idx), _ptr(wts), _ptr(scores), R, K, E,
                                     topk, scale, _stream(stream)))


def MoeRoute(x: torch.Tensor, gate_w: torch.Tensor, bias: torch.Tensor, topk: int, scale: float):
    """MoeRouteGGUF with bf16 gate weights (src/bolt_ops.cu:513-547, :1947-1956)."""
    _need(x, "x", torch.bfloat16, "MoeRoute")
    _need(gate_w, "gate_w", torch.bfloat16, "MoeRoute")
    _need(bias, "bias", torch.float32, "MoeRoute")
    R, K = x.shape
    E = gate_w.shape[0]
    if E > 512 or K % 256 != 0 or topk > 32 or gate_w.shape[1] != K or bias.numel() != E:
        raise ValueError("MoeRoute: unsupported shape")
    idx = torch.empty(R, topk, dtype=torch.int32, device=x.device)
    wts = torch.empty(R, topk, dtype=torch.float32, device=x.device)
    scores = torch.empty(R, E, dtype=torch.float32, device=x.device)
    moe_route_bf16_into(x, gate_w, bias, idx, wts, scores, R, K, E, topk, scale)
    return idx, wts, scores


def relu2_into(x, y, n: int, stream=None) -> None:
    check(load().gguf_relu2(_ptr(x), _ptr(y), n, _stream(stream)))


def Relu2(x: torch.Tensor) -> torch.Tensor:
    """y = bf16(max(x, 0)^2) elementwise (src/bolt_ops.cu:700-726)."""
    _need(x, "x", torch.bfloat16, "Relu2")
    y = torch.empty_like(x)
    relu2_into(x, y, x.numel())
    return y


def moe_verify_into(z, idx, w, fc1_w, fc2_w, out, h, part, meta, R, E, I, topk, stream=None) -> None:
    check(load().gguf_moe_verify_iq2_xxs(_ptr(z), _ptr(idx), _ptr(w), _ptr(fc1_w), _ptr(fc2_w), _ptr(out), _ptr(h),
                                         _ptr(part), _ptr(meta), R, E, I, topk, _stream(stream)))


def moe_legacy_into(layout, z, idx, w, fc1_w, fc1_s, fc2_w, fc2_s, out, h, part, meta, R, E, I, topk,
                    stream=None) -> None:
    check(load().gguf_moe_legacy(layout, _ptr(z), _ptr(idx), _ptr(w), _ptr(fc1_w), _ptr(fc1_s), _ptr(fc2_w),
                                 _ptr(fc2_s), _ptr(out), _ptr(h), _ptr(part), _ptr(meta), R, E, I, topk,
                                 _stream(stream)))


_MOE_LAYOUTS = {0: _lib.GGUF_LAYOUT_Q4_SPLIT, 1: _lib.GGUF_LAYOUT_IQ2_CODES, 2: _lib.GGUF_LAYOUT_IQ2_NATIVE}


def _moe_legacy(op, z, idx, w, fc1_w, fc1_s, fc2_w, fc2_s, topk, iq2, with_meta):
    for t, n, dt in ((z, "z", torch.bfloat16), (idx, "idx", torch.int32), (w, "weights", torch.float32),
                     (fc1_w, "fc1_w", torch.uint8), (fc1_s, "fc1_s", torch.bfloat16), (fc2_w, "fc2_w", torch.uint8),
                     (fc2_s, "fc2_s", torch.bfloat16)):
        _need(t, n, dt, op)
    R = z.shape[0]
    P = R * topk
    if with_meta and (R < 1 or R > 8 or P > 128):
        raise ValueError("MoeVerify: rows must be in [1,8] and rows*topk <= 128")
    if z.shape[1] != 1024:
        raise ValueError(f"{op}: latent size must be 1024")
    E, I = fc1_w.shape[0], fc1_w.shape[1]
    per32 = 8 if iq2 == 2 else 16
    gsz = 256 if iq2 == 2 else 32
    if I % gsz != 0 or fc1_w.numel() != E * I * 32 * per32 or fc2_w.numel() != E * 1024 * (I // 32) * per32 \
            or fc1_s.numel() != E * I * (1024 // gsz) or fc2_s.numel() != E * 1024 * (I // gsz):
        raise ValueError(f"{op}: bad inter size")
    out = torch.empty(R, 1024, dtype=torch.bfloat16, device=z.device)
    h = torch.empty(P, I, dtype=torch.bfloat16, device=z.device)
    part = torch.empty(P, 1024, dtype=torch.float32, device=z.device)
    meta = torch.empty(1 + P + P * 8, dtype=torch.int32, device=z.device) if with_meta else None
    moe_legacy_into(_MOE_LAYOUTS[iq2], z, idx, w, fc1_w, fc1_s, fc2_w, fc2_s, out, h, part, meta, R, E, I, topk)
    return (out, h, part, meta) if with_meta else (out, h, part)


def MoeDecode(z, idx, w, fc1_w, fc1_s, fc2_w, fc2_s, *, topk: int):
    """relu^2 MoE over 4-bit experts fc1_w [E, I, 512] / fc2_w [E, 1024, I/2] with bf16 scales per 32
    (src/bolt_ops.cu:664-699).  Returns (out [R,1024] bf16, h [R*topk, I] bf16, part [R*topk, 1024] f32)."""
    return _moe_legacy("MoeDecode", z, idx, w, fc1_w, fc1_s, fc2_w, fc2_s, topk, 0, False)


def MoeVerify(z, idx, w, fc1_w, fc1_s=None, fc2_w=None, fc2_s=None, *, topk: int, iq2: int = 3):
    """Expert-grouped relu^2 MoE.  iq2=3: raw GGUF IQ2_XXS expert tensors; iq2=0: 4-bit experts with
    bf16 scales (as MoeDecode); iq2=1: 3-bit IQ2 codes; iq2=2: IQ2_XXS records + fp16 d
    (src/bolt_ops.cu:1327-1409).

    Returns (out [R,1024] bf16, h [R*topk, I] bf16, part [R*topk, 1024] f32, meta [1 + 9*R*topk] i32).
    """
    if iq2 in (0, 1, 2):
        return _moe_legacy("MoeVerify", z, idx, w, fc1_w, fc1_s, fc2_w, fc2_s, topk, iq2, True)
    if iq2 != 3:
        raise NotImplementedError(f"MoeVerify: unknown iq2={iq2}")
    _need(z, "z", torch.bfloat16, "MoeVerify")
    _need(idx, "idx", torch.int32, "MoeVerify")
    _need(w, "weights", torch.float32, "MoeVerify")
    _need(fc1_w, "fc1_w", torch.uint8, "MoeVerify")
    _need(fc2_w, "fc2_w", torch.uint8, "MoeVerify")
    R = z.shape[0]
    P = R * topk
    if R < 1 or R > 8 or P > 128:
        raise ValueError("MoeVerify: rows must be in [1,8] and rows*topk <= 128")
    if z.shape[1] != 1024:
        raise ValueError("MoeVerify: latent size must be 1024")
    E, I = fc1_w.shape[0], fc1_w.shape[1]
    if I % 256 != 0 or fc1_w.numel() != E * I * (1024 // 256) * IQ2_XXS_BYTES \
            or fc2_w.numel() != E * 1024 * (I // 256) * IQ2_XXS_BYTES:
        raise ValueError("MoeVerify: inter size alignment mismatch")
    out = torch.empty(R, 1024, dtype=torch.bfloat16, device=z.device)
    h = torch.empty(P, I, dtype=torch.bfloat16, device=z.device)
    part = torch.empty(P, 1024, dtype=torch.float32, device=z.device)
    meta = torch.empty(1 + P + P * 8, dtype=torch.int32, device=z.device)
    moe_verify_into(z, idx, w, fc1_w, fc2_w, out, h, part, meta, R, E, I, topk)
    return out, h, part, meta


# ------------------------------------------------------------------------------------------------
# Mamba
# ------------------------------------------------------------------------------------------------
def mamba_step_into(proj, conv_state, ssm_state, conv_w, conv_b, dt_bias, a_neg, d_skip, norm_w, state_row, y,
                    conv_out, ssm_out, xbc, ypre, *, R, state_rows, heads, n_groups, eps, tmin, stream=None) -> None:
    f32w = 1 if conv_w.dtype == torch.float32 else 0
    check(load().gguf_mamba_step(_ptr(proj), _ptr(conv_state), _ptr(ssm_state), _ptr(conv_w), _ptr(conv_b), f32w,
                                 _ptr(dt_bias), _ptr(a_neg), _ptr(d_skip), _ptr(norm_w), _ptr(state_row), _ptr(y),
                                 _ptr(conv_out), _ptr(ssm_out), _ptr(xbc), _ptr(ypre), R, state_rows, heads, 64, 128,
                                 n_groups, eps, tmin, _stream(stream)))


def _mamba(op, proj, conv_state, ssm_state, conv_w, conv_b, dt_bias, a_neg, D, norm_w, state_row, *, heads, head_dim,
           d_state, n_groups, epsilon, time_step_min, gguf):
    wdt = torch.float32 if gguf else torch.bfloat16
    for t, n, dt in ((proj, "proj", torch.bfloat16), (conv_state, "conv_state", torch.bfloat16),
                     (ssm_state, "ssm_state", torch.float32), (conv_w, "conv_w", wdt), (conv_b, "conv_b", wdt),
                     (dt_bias, "dt_bias", torch.float32), (a_neg, "A_neg", torch.float32), (D, "D", torch.float32),
                     (norm_w, "norm_w", torch.float32)):
        _need(t, n, dt, op)
    if head_dim != 64 or d_state != 128:
        raise ValueError("MambaStep: only head_dim=64, d_state=128 are implemented")
    R = proj.shape[0]
    if R < 1 or R > 16:
        raise ValueError("MambaStep: rows must be in [1,16]")
    di = heads * head_dim
    cd = di + 2 * n_groups * d_state
    if proj.shape[1] != di + cd + heads:
        raise ValueError("MambaStep: bad proj width")
    if state_row is not None:
        _need(state_row, "state_row", torch.int32, op)
        if conv_state.shape[0] < R:
            raise ValueError("MambaVerify: state buffer needs >= R rows")
    dev = proj.device
    y = torch.empty(R, di, dtype=torch.bfloat16, device=dev)
    conv_out = torch.empty_like(conv_state)
    ssm_out = torch.empty_like(ssm_state)
    xbc = torch.empty(R, cd, dtype=torch.bfloat16, device=dev)
    ypre = torch.empty(R, di, dtype=torch.float32, device=dev)
    mamba_step_into(proj, conv_state, ssm_state, conv_w, conv_b, dt_bias, a_neg, D, norm_w, state_row, y, conv_out,
                    ssm_out, xbc, ypre, R=R, state_rows=conv_state.shape[0], heads=heads, n_groups=n_groups,
                    eps=epsilon, tmin=time_step_min)
    return y, conv_out, ssm_out, xbc, ypre


def MambaStep(proj, conv_state, ssm_state, conv_w, conv_b, dt_bias, A_neg, D, norm_w, *, heads, head_dim=64,
              d_state=128, n_groups, epsilon=1e-5, time_step_min=0.0):
    """One Mamba-2 mixer step (src/bolt_ops.cu:304-378).  Returns (y, conv_state_out, ssm_state_out,
    xbc_act, ypre)."""
    return _mamba("MambaStep", proj, conv_state, ssm_state, conv_w, conv_b, dt_bias, A_neg, D, norm_w, None,
                  heads=heads, head_dim=head_dim, d_state=d_state, n_groups=n_groups, epsilon=epsilon,
                  time_step_min=time_step_min, gguf=False)


def MambaStepGGUF(proj, conv_state, ssm_state, conv_w, conv_b, dt_bias, A_neg, D, norm_w, **attrs):
    """MambaStep with fp32 GGUF conv weights / bias (rounded to bf16 on use)."""
    return _mamba("MambaStepGGUF", proj, conv_state, ssm_state, conv_w, conv_b, dt_bias, A_neg, D, norm_w, None,
                  gguf=True, **{"head_dim": 64, "d_state": 128, "epsilon": 1e-5, "time_step_min": 0.0, **attrs})


def MambaVerify(proj, conv_state, ssm_state, conv_w, conv_b, dt_bias, A_neg, D, norm_w, state_row, **attrs):
    """MambaStep over R speculative tokens from state row *state_row; the state after token r is
    row r of the outputs (src/bolt_ops.cu:1915-1933)."""
    return _mamba("MambaVerify", proj, conv_state, ssm_state, conv_w, conv_b, dt_bias, A_neg, D, norm_w, state_row,
                  gguf=False, **{"head_dim": 64, "d_state": 128, "epsilon": 1e-5, "time_step_min": 0.0, **attrs})


def MambaVerifyGGUF(proj, conv_state, ssm_state, conv_w, conv_b, dt_bias, A_neg, D, norm_w, state_row, **attrs):
    """MambaVerify with fp32 GGUF conv weights / bias."""
    return _mamba("MambaVerifyGGUF", proj, conv_state, ssm_state, conv_w, conv_b, dt_bias, A_neg, D, norm_w,
                  state_row, gguf=True,
                  **{"head_dim": 64, "d_state": 128, "epsilon": 1e-5, "time_step_min": 0.0, **attrs})


# ------------------------------------------------------------------------------------------------
# Debug / parity
# ------------------------------------------------------------------------------------------------
def dequantize(w: torch.Tensor, gguf_type: int, K: int) -> torch.Tensor:
    """Raw GGUF rows [rows, row_bytes] -> f32 [rows, K] with the GEMV's device decoders."""
    rows = w.shape[0]
    out = torch.empty(rows, K, dtype=torch.float32, device=w.device)
    check(load().gguf_dequantize(gguf_type, _ptr(w), _ptr(out), rows, K, _stream()))
    return out


def set_pdl(enable: bool) -> None:
    load().gguf_set_pdl(1 if enable else 0)


def set_fast_paths(enable) -> None:
    """Enable / disable the shape-specialised kernels (the generic engine handles every shape).

    ``True`` / 1 = on (default), ``False`` / 0 = generic engine only, 2 = on, with the bf16 instead of
    the integer tensor-core kernel for single-row IQ2_XXS (a cross-check of the two decoders)."""
    load().gguf_set_fast_paths(int(enable) if not isinstance(enable, bool) else (1 if enable else 0))


def device_status():
    return _lib.device_status()
