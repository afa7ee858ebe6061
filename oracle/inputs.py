"""Seeded synthetic inputs with the shapes and value distributions of the BASELINE configs.

No public dataset is involved: every config is synthetic by definition.

* C0 / C4  Q8Gemv gguf=1: x ~ N(0,1) bf16; W ~ N(0, 0.02) fp32 quantised to Q8_0 (ggml rounding).
* C1       Q4Gemv iq2=3:  x ~ N(0,1) bf16; per 66-B super-block d = fp16(|N(0,1)| * 0.002) then
                          64 uniform random bytes.
* C2       Nvfp4Gemv:     x ~ N(0,1) bf16; per 36-B block 4 scale bytes uniform over the E4M3 codes
                          for [2^-4, 2^2] (0x18..0x48), then 32 uniform random bytes; gscale 1/448.
* C3       MoeRouteGGUF -> MoeVerify iq2=3: z, x ~ N(0,1) bf16 [R,1024]; gate_w ~ N(0, 0.02) fp32
                          [128,1024]; bias ~ N(0, 0.01) fp32; w1 [128,1792,264], w2 [128,1024,462]
                          built as C1; topk 6; scale 1.0.

Also the reference test's own builders (``tests/test_bolt_ops.py``), restated with numpy RNG:
``iq2_test_blocks`` (``:210-215``: uniform bytes, d = fp16(U(0.001, 0.021))) and
``q8_test_blocks`` (``:290-294``).
"""

from __future__ import annotations

import numpy as np

from .quants import IQ2_XXS_BYTES, NVFP4_BYTES, Q8_0_BYTES, bf16_bits, quantize_q8_0


def rng(seed: int) -> np.random.Generator:
    return np.random.Generator(np.random.PCG64(seed))


def bf16_normal(g: np.random.Generator, shape, scale: float = 1.0) -> np.ndarray:
    """N(0, scale) values rounded to bf16, returned as uint16 bit patterns."""
    return bf16_bits((g.standard_normal(shape) * scale).astype(np.float32))


def q8_0_weights(g: np.random.Generator, n: int, k: int, std: float = 0.02) -> np.ndarray:
    w = (g.standard_normal((n, k), dtype=np.float32) * np.float32(std)).astype(np.float32)
    return quantize_q8_0(w)


def iq2_xxs_weights(g: np.random.Generator, lead: tuple, k: int) -> np.ndarray:
    """[*lead, k/256*66] raw IQ2_XXS: d = fp16(|N(0,1)| * 0.002), then 64 uniform bytes."""
    nsb = k // 256
    blk = g.integers(0, 256, size=(*lead, nsb, IQ2_XXS_BYTES), dtype=np.uint8)
    d = (np.abs(g.standard_normal((*lead, nsb))) * 0.002).astype(np.float16)
    blk[..., :2] = d.view(np.uint8).reshape(*lead, nsb, 2)
    return blk.reshape(*lead, nsb * IQ2_XXS_BYTES)


def nvfp4_weights(g: np.random.Generator, n: int, k: int, lo: int = 0x18, hi: int = 0x48) -> np.ndarray:
    nb = k // 64
    blk = g.integers(0, 256, size=(n, nb, NVFP4_BYTES), dtype=np.uint8)
    blk[..., :4] = g.integers(lo, hi + 1, size=(n, nb, 4), dtype=np.uint8)
    return blk.reshape(n, nb * NVFP4_BYTES)


def iq2_test_blocks(g: np.random.Generator, lead: tuple, k: int) -> np.ndarray:
    """Reference test builder (``tests/test_bolt_ops.py:210-215``): uniform random bytes with
    d = fp16(U(0.001, 0.021))."""
    nsb = k // 256
    blk = g.integers(0, 256, size=(*lead, nsb, IQ2_XXS_BYTES), dtype=np.uint8)
    d = (g.random((*lead, nsb)) * 0.02 + 0.001).astype(np.float16)
    blk[..., :2] = d.view(np.uint8).reshape(*lead, nsb, 2)
    return blk.reshape(*lead, nsb * IQ2_XXS_BYTES)


def q8_test_blocks(g: np.random.Generator, n: int, k: int) -> np.ndarray:
    """Reference test builder (``tests/test_bolt_ops.py:290-294``): uniform int8 q, d = fp16(U(0.001, 0.021))."""
    nb = k // 32
    blk = g.integers(0, 256, size=(n, nb, Q8_0_BYTES), dtype=np.uint8)
    d = (g.random((n, nb)) * 0.02 + 0.001).astype(np.float16)
    blk[..., :2] = d.view(np.uint8).reshape(n, nb, 2)
    return blk.reshape(n, nb * Q8_0_BYTES)


def legacy_case(layout: str, g: np.random.Generator, n: int, k: int):
    """Weights + scales of a legacy split layout, as the reference harness builds them
    (tests/test_bolt_ops.py:70-75 NVFP4, :84-93 Q8 / Q4, :159-175 IQ2 codes, :210-223 IQ2 native).
    Returns (w u8, scales (bf16 bits u16 / e4m3fn u8 / fp16 bits u16))."""
    nb = k // 32
    if layout == "q8":
        w = g.integers(0, 256, size=(n, k), dtype=np.uint8)
    elif layout == "q4":
        w = g.integers(0, 256, size=(n, k // 2), dtype=np.uint8)
    elif layout == "iq2c":
        code = (g.integers(0, 3, size=(n, k)) + 4 * g.integers(0, 2, size=(n, k))).astype(np.uint8)
        w = (code[:, 0::2] | (code[:, 1::2] << 4)).astype(np.uint8)
    elif layout == "iq2n":
        from .quants import iq2_native_from_blocks

        return iq2_native_from_blocks(iq2_test_blocks(g, (n,), k))
    elif layout == "fp4":
        w = g.integers(0, 256, size=(n, k // 2), dtype=np.uint8)
        return w, g.integers(0x30, 0x48, size=(n, k // 16), dtype=np.uint8)
    else:
        raise ValueError(layout)
    from .quants import bf16_bits

    return w, bf16_bits((g.random((n, nb)) * 0.02).astype(np.float32))


# Shapes of the benchmark configurations C0..C4 (the GEMV / MoE decode calls being measured).
CONFIGS = {
    "C0": dict(op="q8_0", N=4096, K=4096, R=(1,)),
    "C1": dict(op="iq2_xxs", N=14336, K=4096, R=(1, 4, 8)),
    "C2": dict(op="nvfp4", N=13824, K=5120, R=(1, 8, 16), gscale=1.0 / 448.0),
    "C3": dict(op="moe", E=128, H=1024, I=1792, topk=6, scale=1.0, R=(1, 4, 8)),
    "C4": dict(op="q8_0", N=131072, K=4096, R=(1, 4, 8, 16)),
}


def gemv_case(op: str, R: int, N: int, K: int, seed: int = 0):
    """Returns (x bf16 bits [R,K], raw weights [N, row_bytes], extra dict)."""
    g = rng(seed)
    x = bf16_normal(g, (R, K))
    extra = {}
    if op == "q8_0":
        w = q8_0_weights(g, N, K)
    elif op == "iq2_xxs":
        w = iq2_xxs_weights(g, (N,), K)
    elif op == "nvfp4":
        w = nvfp4_weights(g, N, K)
        extra["gscale"] = np.array([1.0 / 448.0], dtype=np.float32)
    else:
        raise ValueError(op)
    return x, w, extra


def moe_case(R: int, E: int = 128, H: int = 1024, I: int = 1792, seed: int = 0):
    """Router + MoE inputs of config C3 (weights for all E experts)."""
    g = rng(seed)
    z = bf16_normal(g, (R, H))
    x = bf16_normal(g, (R, H))
    gate_w = (g.standard_normal((E, H)) * 0.02).astype(np.float32)
    bias = (g.standard_normal(E) * 0.01).astype(np.float32)
    w1 = iq2_xxs_weights(g, (E, I), H)
    w2 = iq2_xxs_weights(g, (E, H), I)
    return dict(z=z, x=x, gate_w=gate_w, bias=bias, w1=w1, w2=w2)
