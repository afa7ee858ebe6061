"""numpy restatement of the GGUF block dequantisers on the hot path (test infrastructure).

Each function follows the published algorithm of llama.cpp's gguf-py (``gguf`` 0.19.0,
``gguf/quants.py``), the third-party package that the reference's test harness calls as its
CPU oracle (``tests/test_bolt_ops.py:225-230``).  The fp32 operation order is kept identical
so that results are bit-identical; ``tests/test_oracle.py`` checks that against
``gguf.quants.dequantize`` and against the committed fixtures.

Block layouts (``docs/GGUF_ONNX_Custom_Ops.md:13-18``):

* Q8_0    (type 8):  34 B / 32 elements  = fp16 d, int8 q[32];           w = q * d
* IQ2_XXS (type 16): 66 B / 256 elements = fp16 d, 8 x (u8 grid[4], u32 aux)
* NVFP4   (type 40): 36 B / 64 elements  = u8 ue4m3 scale[4], 4 x u8 nibbles[8]
"""

from __future__ import annotations

import numpy as np

Q8_0_BLOCK, Q8_0_BYTES = 32, 34
IQ2_XXS_BLOCK, IQ2_XXS_BYTES = 256, 66
NVFP4_BLOCK, NVFP4_BYTES = 64, 36


# ----------------------------------------------------------------------------------------------
# bf16 helpers (round-to-nearest-even, as __float2bfloat16 and torch's .bfloat16() do)
# ----------------------------------------------------------------------------------------------
def bf16_bits(a) -> np.ndarray:
    """fp32 -> bf16 bit patterns (uint16), round to nearest even (finite inputs)."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    r = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return r.astype(np.uint16)


def bf16_round(a) -> np.ndarray:
    """fp32 values rounded to the nearest bf16, returned as fp32."""
    return (bf16_bits(a).astype(np.uint32) << 16).view(np.float32)


def bf16_to_f32(bits) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


# ----------------------------------------------------------------------------------------------
# Q8_0  (gguf-py quants.py:378-401 -- class Q8_0)
# ----------------------------------------------------------------------------------------------
def _roundf(n: np.ndarray) -> np.ndarray:
    """C roundf (half away from zero), as gguf-py's np_roundf (quants.py:43-47)."""
    a = np.abs(n)
    f = np.floor(a)
    return np.sign(n) * (f + np.floor(2 * (a - f)))


def quantize_q8_0(w: np.ndarray) -> np.ndarray:
    """fp32 [rows, K] -> raw Q8_0 bytes [rows, K/32*34] (ggml rounding: d = amax/127 in fp32,
    q = roundf(v * (1/d)), d stored as fp16)."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    rows, k = w.shape
    assert k % Q8_0_BLOCK == 0
    b = w.reshape(-1, Q8_0_BLOCK)
    d = np.abs(b).max(axis=1, keepdims=True) / np.float32(127)
    with np.errstate(divide="ignore"):
        inv = np.where(d == 0, np.float32(0), np.float32(1) / d).astype(np.float32)
    q = _roundf(b * inv).astype(np.int8)
    out = np.concatenate([d.astype(np.float16).view(np.uint8), q.view(np.uint8)], axis=1)
    return out.reshape(rows, k // Q8_0_BLOCK * Q8_0_BYTES)


def dequant_q8_0(raw: np.ndarray) -> np.ndarray:
    """raw Q8_0 [rows, nb*34] -> fp32 [rows, nb*32];  w = fp32(int8 q) * fp32(fp16 d)."""
    raw = np.ascontiguousarray(raw, dtype=np.uint8)
    rows = raw.shape[0]
    b = raw.reshape(-1, Q8_0_BYTES)
    d = b[:, :2].copy().view(np.float16).astype(np.float32)
    q = b[:, 2:].view(np.int8).astype(np.float32)
    return (q * d).reshape(rows, -1)


# ----------------------------------------------------------------------------------------------
# IQ2_XXS  (gguf-py quants.py:766-828 -- class IQ2_XXS; grid = ggml iq2xxs_grid)
# ----------------------------------------------------------------------------------------------
_GRID = None


def iq2xxs_grid() -> np.ndarray:
    """The 256 x 8 IQ2_XXS magnitude codebook (values 8, 25, 43) as uint8.

    The codebook is format data: it is taken from gguf 0.19.0 (``IQ2_XXS.grid_hex``: 2-bit
    codes mapping 0->0x08, 1->0x19, 2->0x2b, element j of entry i in bits 2*(j%4) of byte
    2*i + j//4) and checked against the reference's table ``src/iq2xxs_grid.h:6`` through
    the committed fixture ``tests/golden/iq2xxs_grid.npz``.
    """
    global _GRID
    if _GRID is None:
        from gguf.quants import IQ2_XXS  # pinned third-party dependency: gguf 0.19.0

        hexs = bytes(IQ2_XXS.grid_hex).decode("ascii")
        packed = np.frombuffer(bytes.fromhex(hexs), dtype=np.uint8)  # 512 bytes
        assert packed.size == 512
        codes = (packed[:, None] >> np.array([0, 2, 4, 6], dtype=np.uint8)[None, :]) & 3  # [512, 4]
        codes = codes.reshape(256, 8)
        _GRID = np.array([0x08, 0x19, 0x2B], dtype=np.uint8)[codes]
    return _GRID


def iq2xxs_sign_byte(si: np.ndarray) -> np.ndarray:
    """7-bit sign index -> 8 sign bits: bit 7 makes the parity even (equals ggml ksigns[si])."""
    si = np.asarray(si).astype(np.uint32) & 0x7F
    par = np.zeros_like(si)
    for b in range(7):
        par ^= (si >> b) & 1
    return (si | (par << 7)).astype(np.uint8)


def dequant_iq2_xxs(raw: np.ndarray) -> np.ndarray:
    """raw IQ2_XXS [rows, nsb*66] -> fp32 [rows, nsb*256].

    Per super-block: d = fp16; per 32-element sub-block (8-byte record): 4 grid indices and a
    u32 aux; db = d * (0.5 + (aux >> 28)) * 0.25; element = db * grid[idx][j] * sign, where the
    sign of element j of group g is bit j of the sign byte of the 7-bit index (aux >> 7g) & 127.
    """
    raw = np.ascontiguousarray(raw, dtype=np.uint8)
    rows = raw.shape[0]
    b = raw.reshape(-1, IQ2_XXS_BYTES)
    n = b.shape[0]
    d = b[:, :2].copy().view(np.float16).astype(np.float32)  # [n, 1]
    rec = b[:, 2:].copy().view(np.uint32).reshape(n, 8, 2)
    aux = rec[..., 1]
    db = d * (np.float32(0.5) + (aux >> 28).astype(np.float32)) * np.float32(0.25)  # [n, 8]
    si = (aux[..., None] >> np.array([0, 7, 14, 21], dtype=np.uint32)) & 0x7F  # [n, 8, 4]
    sb = iq2xxs_sign_byte(si)
    bits = (sb[..., None] >> np.arange(8, dtype=np.uint8)) & 1  # [n, 8, 4, 8]
    sign = np.where(bits == 0, np.float32(1), np.float32(-1))
    gidx = rec[..., 0].copy().view(np.uint8).reshape(n, 8, 4)
    grid = iq2xxs_grid().astype(np.float32)[gidx]  # [n, 8, 4, 8]
    out = db[..., None, None] * grid * sign
    return out.reshape(rows, -1)


# ----------------------------------------------------------------------------------------------
# NVFP4  (gguf-py quants.py:707-763 -- class NVFP4)
# ----------------------------------------------------------------------------------------------
# E2M1 values doubled (0, 0.5, ..., 6 -> 0, 1, ..., 12); the scale decode carries the 0.5.
_NVFP4_KVALUES = np.array([0, 1, 2, 3, 4, 6, 8, 12, 0, -1, -2, -3, -4, -6, -8, -12], dtype=np.float32)


def ue4m3_table() -> np.ndarray:
    """All 256 scale bytes -> fp32, exactly as gguf-py's ``NVFP4.ue4m3_to_fp32``: bit 7 is
    ignored (unsigned E4M3, bias 7), bytes 0x00 and 0x7F decode to 0, the result carries a
    factor 0.5 because the nibble table is doubled."""
    x = np.arange(256, dtype=np.uint8)
    exp = (x >> 3).astype(np.int32) & 0xF
    man = (x & 0x7).astype(np.float32)
    raw = np.where(exp == 0, man * np.float32(2.0 ** -9),
                   (np.float32(1.0) + man / np.float32(8.0)) * (np.float32(2.0) ** (exp.astype(np.float32) - np.float32(7))))
    return np.where((x == 0) | (x == 0x7F), np.float32(0.0), raw * np.float32(0.5)).astype(np.float32)


def dequant_nvfp4(raw: np.ndarray) -> np.ndarray:
    """raw NVFP4 [rows, nb*36] -> fp32 [rows, nb*64].  Sub-block s (16 elements) uses scale byte s;
    its element j < 8 is the low nibble of byte j of the 8-byte group, j >= 8 the high nibble of
    byte j - 8."""
    raw = np.ascontiguousarray(raw, dtype=np.uint8)
    rows = raw.shape[0]
    b = raw.reshape(-1, NVFP4_BYTES)
    n = b.shape[0]
    d = ue4m3_table()[b[:, :4]].reshape(n, 4, 1)
    qs = b[:, 4:].reshape(n, 4, 8)
    nib = np.concatenate([qs & 0x0F, qs >> 4], axis=-1)  # [n, 4, 16]
    vals = _NVFP4_KVALUES[nib]
    return (d * vals).reshape(rows, -1)


# ----------------------------------------------------------------------------------------------
# Split (pre-GGUF) layouts of the reference's legacy attribute values; expected values as the
# reference harness computes them (tests/test_bolt_ops.py:70-100, 155-181, 210-232).
# Nibble tensors: element 2i is the low nibble of byte i, element 2i+1 the high nibble.
# ----------------------------------------------------------------------------------------------
def _nibbles(w: np.ndarray) -> np.ndarray:
    w = np.ascontiguousarray(w, dtype=np.uint8)
    return np.stack([w & 0x0F, w >> 4], axis=-1).reshape(w.shape[0], -1)


def _group_scale(s_bits: np.ndarray, K: int) -> np.ndarray:
    """bf16 scale bits [N, K/32] -> fp32 per element [N, K]."""
    return np.repeat(bf16_to_f32(np.asarray(s_bits, np.uint16)), 32, axis=1).reshape(-1, K)


def dequant_q8_split(w: np.ndarray, s_bits: np.ndarray) -> np.ndarray:
    """Q8Gemv gguf=0: w u8 [N, K] holding q + 128, bf16 scales [N, K/32] -> (w - 128) * s
    (tests/test_bolt_ops.py:88-95)."""
    w = np.asarray(w, np.uint8)
    return (w.astype(np.float32) - np.float32(128)) * _group_scale(s_bits, w.shape[1])


def dequant_q4_split(w: np.ndarray, s_bits: np.ndarray) -> np.ndarray:
    """Q4Gemv iq2=0: nibbles n [N, K/2], bf16 scales [N, K/32] -> (n - 8) * s (:90-95)."""
    n = _nibbles(w)
    return (n.astype(np.float32) - np.float32(8)) * _group_scale(s_bits, n.shape[1])


IQ2_CODE_VALUES = np.array([8, 25, 43, 0, -8, -25, -43, 0], dtype=np.float32)  # tests/test_bolt_ops.py:156


def dequant_iq2_codes(w: np.ndarray, s_bits: np.ndarray) -> np.ndarray:
    """Q4Gemv iq2=1: 3-bit codes c = mag + 4 * negative in nibbles [N, K/2], bf16 scales [N, K/32]
    -> {8, 25, 43, 0}[mag] * sign * s (:155-181).  Bit 3 of a nibble is not part of the format and is
    ignored."""
    c = _nibbles(w) & 7
    return IQ2_CODE_VALUES[c] * _group_scale(s_bits, c.shape[1])


def iq2_native_from_blocks(blk: np.ndarray):
    """GGUF IQ2_XXS blocks [N, K/256 * 66] -> (records u8 [N, K/32, 8], fp16 d bits u16 [N, K/256]),
    the repacking of the reference harness's iq2_repack (tests/test_bolt_ops.py:218-223)."""
    blk = np.ascontiguousarray(blk, np.uint8)
    N = blk.shape[0]
    b = blk.reshape(N, -1, IQ2_XXS_BYTES)
    rec = np.ascontiguousarray(b[:, :, 2:]).reshape(N, -1, 8)
    d = np.ascontiguousarray(b[:, :, :2]).view(np.uint16).reshape(N, -1)
    return rec, d


def dequant_iq2_native(rec: np.ndarray, d_bits: np.ndarray) -> np.ndarray:
    """Q4Gemv iq2=2: records [N, K/32, 8] + fp16 d [N, K/256] -> the gguf-py IQ2_XXS values of the
    reassembled blocks (exact; the reference kernel rounds each weight to bf16, :237)."""
    rec = np.asarray(rec, np.uint8)
    N, g = rec.shape[0], rec.shape[1]
    d = np.asarray(d_bits, np.uint16).reshape(N, g // 8, 1).view(np.uint8)
    blk = np.concatenate([d, rec.reshape(N, g // 8, 64)], axis=2)
    return dequant_iq2_xxs(blk.reshape(N, -1))


_E2M1 = np.array([0, 0.5, 1, 1.5, 2, 3, 4, 6, -0.0, -0.5, -1, -1.5, -2, -3, -4, -6], dtype=np.float32)  # :67


def e4m3fn_table() -> np.ndarray:
    """All 256 bytes as torch.float8_e4m3fn values (signed, bias 7, subnormal for e == 0, 0x7F and
    0xFF NaN)."""
    x = np.arange(256, dtype=np.uint32)
    e = ((x >> 3) & 15).astype(np.float32)
    m = (x & 7).astype(np.float32)
    v = np.where(e == 0, m * np.float32(2.0 ** -9), (1 + m / 8) * np.float32(2.0) ** (e - 7)).astype(np.float32)
    v = np.where(x & 0x80, -v, v).astype(np.float32)
    return np.where((x & 0x7F) == 0x7F, np.float32(np.nan), v).astype(np.float32)


def dequant_nvfp4_split(w: np.ndarray, ws: np.ndarray) -> np.ndarray:
    """Nvfp4Gemv gguf=0: E2M1 nibbles [N, K/2], e4m3fn scales [N, K/16] -> E2M1 * scale (the
    global scale is applied by the caller) (tests/test_bolt_ops.py:70-79)."""
    n = _nibbles(w)
    s = np.repeat(e4m3fn_table()[np.asarray(ws, np.uint8)], 16, axis=1)
    return _E2M1[n] * s
