// GGUF block decoders shared by the tensor-core GEMV engine and the dequantise kernels.
//
// A "k-group" is 32 consecutive elements of one weight row: one Q8_0 block, one IQ2_XXS
// sub-block, or half an NVFP4 block.  In the engine a k-group is consumed by two
// mma.m16n8k16 steps; lane (g = lane/4, t = lane%4) owns rows g and g+8 of the 16-row tile and
// the 8 elements of the group listed below (any k permutation shared by the A and B operands
// is valid because the MMA sums over k):
//
//   Q8_0    : elements 4t..4t+3 and 16+4t..19+4t            (quad reads 4 consecutive words)
//   IQ2_XXS : elements 8t..8t+7 = grid entry t of the record (one codebook lookup per lane)
//   NVFP4   : per 16-element sub-block, bytes 2t and 2t+1 of its nibble group: low nibbles are
//             elements 2t, 2t+1 and high nibbles 8+2t, 9+2t -- exactly the m16n8k16 slots, so
//             the GGUF nibble order needs no shuffling.
//
// Weights reach the tensor cores EXACTLY equal to the gguf-py dequantised values:
//   Q8_0    : int8 q as bf16 (exact), the fp16 block scale d applied in fp32 after the MMA.
//   IQ2_XXS : +-{8,25,43} as bf16 (exact), db = d*(0.5+s)*0.25 applied in fp32 after the MMA.
//   NVFP4   : E2M1 bits placed in the bf16 exponent/mantissa field (value * 2^-126, subnormal
//             for 0.5) times the UE4M3 scale * 2^110 in bf16 -- a product of <= 6 significant
//             bits, exact; the epilogue multiplies by 2^16 (and gscale).
#pragma once

#include "common.cuh"
#include "iq2xxs_tables.h"

namespace gguf_b200 {

constexpr int kFmtQ8 = 0, kFmtIQ2 = 1, kFmtFP4 = 2;
// Split (pre-GGUF) layouts of the reference's legacy attribute values: weight bytes and scales in
// two tensors (src/bolt_ops.cu:840-848, tests/test_bolt_ops.py:70-100, 159-181, 210-240).
//   kFmtQ8S  : Q8Gemv gguf=0       u8 [N, K] = q + 128,             bf16 scale [N, K/32]
//   kFmtQ4S  : Q4Gemv iq2=0        u8 [N, K/2] nibbles (n - 8),     bf16 scale [N, K/32]
//   kFmtIQ2C : Q4Gemv iq2=1        u8 [N, K/2] 3-bit codes,         bf16 scale [N, K/32]
//   kFmtIQ2N : Q4Gemv iq2=2        u8 [N, K/32, 8] IQ2_XXS records, fp16 d bits [N, K/256]
//   kFmtFP4S : Nvfp4Gemv gguf=0    u8 [N, K/2] E2M1 nibbles,        e4m3fn scale [N, K/16]
// Byte i of a nibble-packed group holds element 2i in its low and 2i+1 in its high nibble.
constexpr int kFmtQ8S = 3, kFmtQ4S = 4, kFmtIQ2C = 5, kFmtIQ2N = 6, kFmtFP4S = 7;

template <int F>
struct FmtInfo;
// kSeg = smallest K granule whose byte size (and, for split layouts, whose scale bytes) is a
// multiple of 16 (segmented bulk copies).  kScDiv: weight elements per scale byte (0: the scales
// are inside the GGUF blocks).
template <>
struct FmtInfo<kFmtQ8> {
  static constexpr int kBlock = 32, kBytes = 34, kSeg = 256, kScDiv = 0;
};
template <>
struct FmtInfo<kFmtIQ2> {
  static constexpr int kBlock = 256, kBytes = 66, kSeg = 2048, kScDiv = 0;
};
template <>
struct FmtInfo<kFmtFP4> {
  static constexpr int kBlock = 64, kBytes = 36, kSeg = 256, kScDiv = 0;
};
template <>
struct FmtInfo<kFmtQ8S> {
  static constexpr int kBlock = 32, kBytes = 32, kSeg = 256, kScDiv = 16;
};
template <>
struct FmtInfo<kFmtQ4S> {
  static constexpr int kBlock = 32, kBytes = 16, kSeg = 256, kScDiv = 16;
};
template <>
struct FmtInfo<kFmtIQ2C> {
  static constexpr int kBlock = 32, kBytes = 16, kSeg = 256, kScDiv = 16;
};
template <>
struct FmtInfo<kFmtIQ2N> {
  static constexpr int kBlock = 32, kBytes = 8, kSeg = 2048, kScDiv = 128;
};
template <>
struct FmtInfo<kFmtFP4S> {
  static constexpr int kBlock = 32, kBytes = 16, kSeg = 256, kScDiv = 16;
};
constexpr bool is_split(int F) { return F >= kFmtQ8S; }

// ---------------------------------------------------------------------------------------------
// Unaligned (2-byte aligned) reads from a 4-byte aligned base (shared or global).
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t ld_u16(const uint8_t* base, uint32_t off) {
  return *reinterpret_cast<const uint16_t*>(base + off);
}
__device__ __forceinline__ uint32_t ld_u32_a2(const uint8_t* base, uint32_t off) {
  const uint32_t* w = reinterpret_cast<const uint32_t*>(base + (off & ~3u));
  return __funnelshift_r(w[0], w[1], (off & 2u) * 8u);
}
__device__ __forceinline__ uint2 ld_u64_a2(const uint8_t* base, uint32_t off) {
  const uint32_t* w = reinterpret_cast<const uint32_t*>(base + (off & ~3u));
  const uint32_t sh = (off & 2u) * 8u;
  const uint32_t w0 = w[0], w1 = w[1], w2 = w[2];
  return make_uint2(__funnelshift_r(w0, w1, sh), __funnelshift_r(w1, w2, sh));
}
// Exact-width variants for global memory: never touch a byte outside [off, off + 4/8).
__device__ __forceinline__ uint32_t ld_u32_a2_exact(const uint8_t* base, uint32_t off) {
  if ((off & 2u) == 0u) return *reinterpret_cast<const uint32_t*>(base + off);
  const uint16_t* h = reinterpret_cast<const uint16_t*>(base + off);
  return static_cast<uint32_t>(h[0]) | (static_cast<uint32_t>(h[1]) << 16);
}
__device__ __forceinline__ uint2 ld_u64_a2_exact(const uint8_t* base, uint32_t off) {
  return make_uint2(ld_u32_a2_exact(base, off), ld_u32_a2_exact(base, off + 4u));
}
__device__ __forceinline__ float fp16_bits_to_f32(uint32_t h) { return __half2float(__ushort_as_half(static_cast<unsigned short>(h))); }

// ---------------------------------------------------------------------------------------------
// Q8_0
// ---------------------------------------------------------------------------------------------
// 4 signed bytes -> two bf16x2 words (exact): (q0,q1), (q2,q3).
__device__ __forceinline__ void q8_to_bf16x4(uint32_t q, uint32_t& w01, uint32_t& w23) {
  const uint32_t u = q ^ 0x80808080u;  // q + 128 per byte
  // float with bits 0x4B0000uu = 2^23 + u; subtracting 2^23 + 128 yields q exactly.
  const float f0 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7540)) - 8388736.0f;
  const float f1 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7541)) - 8388736.0f;
  const float f2 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7542)) - 8388736.0f;
  const float f3 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7543)) - 8388736.0f;
  w01 = pack_bf16x2(f0, f1);
  w23 = pack_bf16x2(f2, f3);
}

// Group decode for one row: `row` points at the row's first byte of the staged K segment,
// grp = group index within that segment.  Outputs the lane's 4 A words and the block scale.
// kExact: read exactly the bytes of the block (global memory); otherwise a padded shared-memory
// stage is read with aligned words.
template <bool kExact = false>
__device__ __forceinline__ void q8_decode_row(const uint8_t* base, uint32_t row_off, int grp, int t, uint32_t (&a)[4],
                                              float& d) {
  const uint32_t bo = row_off + static_cast<uint32_t>(grp) * 34u;
  const uint32_t lo = kExact ? ld_u32_a2_exact(base, bo + 2u + 4u * t) : ld_u32_a2(base, bo + 2u + 4u * t);
  const uint32_t hi = kExact ? ld_u32_a2_exact(base, bo + 18u + 4u * t) : ld_u32_a2(base, bo + 18u + 4u * t);
  d = fp16_bits_to_f32(ld_u16(base, bo));
  q8_to_bf16x4(lo, a[0], a[1]);
  q8_to_bf16x4(hi, a[2], a[3]);
}

// ---------------------------------------------------------------------------------------------
// IQ2_XXS
// ---------------------------------------------------------------------------------------------
// Sign word for bf16x2 word p of an 8-element grid entry: bit 2p of the sign byte -> bit 15,
// bit 2p+1 -> bit 31 (sb * (2^(15-2p) + 2^(30-2p)), both products land without overlap).
__device__ __forceinline__ uint32_t iq2_sign_mask(uint32_t sb, int p) {
  const uint32_t k = (1u << (15 - 2 * p)) + (1u << (30 - 2 * p));
  return (sb * k) & 0x80008000u;
}

// Decodes grid entry t (8 elements) of a record (gw = 4 grid bytes, aux = 4 x 7-bit sign indices
// + 4-bit scale) into 4 bf16x2 words of signed magnitudes.  `mag` = 4 bf16x2 magnitude words of
// the entry (from the codebook).
__device__ __forceinline__ void iq2_apply_signs(uint4 mag, uint32_t aux, uint32_t t7, uint32_t (&w)[4]) {
  const uint32_t si = (aux >> t7) & 0x7Fu;
  const uint32_t sb = si | ((__popc(si) & 1u) << 7);  // even parity: the ggml ksigns table
  w[0] = mag.x ^ iq2_sign_mask(sb, 0);
  w[1] = mag.y ^ iq2_sign_mask(sb, 1);
  w[2] = mag.z ^ iq2_sign_mask(sb, 2);
  w[3] = mag.w ^ iq2_sign_mask(sb, 3);
}
// db = d * (0.5 + s) * 0.25 in the fp32 order of gguf-py (exact: <= 16 significant bits).
__device__ __forceinline__ float iq2_db(float d, uint32_t aux) {
  return d * (0.5f + static_cast<float>(aux >> 28)) * 0.25f;
}

// ---------------------------------------------------------------------------------------------
// NVFP4
// ---------------------------------------------------------------------------------------------
// Scale byte -> bf16 bits of (gguf-py raw UE4M3 value) * 2^110; gguf-py semantics: bit 7 ignored,
// 0x00 and 0x7F decode to zero.  raw = (1 + m/8) 2^(e-7) for e > 0, m 2^-9 for e == 0.
__device__ __forceinline__ uint32_t fp4_scale_bf16_bits(uint32_t b) {
  if (b == 0u || b == 0x7Fu) return 0u;
  const uint32_t e = (b >> 3) & 15u, m = b & 7u;
  if (e != 0u) return ((e + 230u) << 7) | (m << 4);
  return __float_as_uint(static_cast<float>(m) * 0x1p101f) >> 16;
}
// Two nibble bytes (byte0 | byte1 << 8) -> bf16x2 bit patterns of E2M1 * 2^-126:
// lo = (low nibble of byte0, low nibble of byte1), hi = (high nibbles).
__device__ __forceinline__ void fp4_patterns(uint32_t v, uint32_t& lo, uint32_t& hi) {
  const uint32_t v2 = (v & 0xFFu) | ((v & 0xFF00u) << 8);
  lo = ((v2 & 0x00070007u) << 6) | ((v2 & 0x00080008u) << 12);
  hi = ((v2 & 0x00700070u) << 2) | ((v2 & 0x00800080u) << 8);
}
__device__ __forceinline__ uint32_t hmul2_bits(uint32_t a, uint32_t b) {
  __nv_bfloat162 r = __hmul2(*reinterpret_cast<__nv_bfloat162*>(&a), *reinterpret_cast<__nv_bfloat162*>(&b));
  return *reinterpret_cast<uint32_t*>(&r);
}

// ---------------------------------------------------------------------------------------------
// Split layouts: lane t of a k-group owns elements 8t..8t+7 (nibble formats: bytes 4t..4t+3 of the
// group; Q8S: elements 4t..4t+3 and 16+4t..19+4t as Q8_0).  Each helper returns the 4 A words
// (bf16x2, exact) of one row for the two m16n8k16 steps: (w[0], w[1]) step 0, (w[2], w[3]) step 1.
// ---------------------------------------------------------------------------------------------
// Q4S: nibble n -> bf16(128 + n) = 0x4300 | n exactly; minus 136 gives n - 8 (exact).
__device__ __forceinline__ void q4s_words(uint32_t v, uint32_t (&w)[4]) {
  const __nv_bfloat162 zp = __floats2bfloat162_rn(136.f, 136.f);
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    const uint32_t x = (v >> (8 * p)) & 0xFFu;
    uint32_t u = 0x43004300u | (x & 0xFu) | ((x & 0xF0u) << 12);
    __nv_bfloat162 r = __hsub2(*reinterpret_cast<__nv_bfloat162*>(&u), zp);
    w[p] = *reinterpret_cast<uint32_t*>(&r);
  }
}
// IQ2C: code c (low 3 bits; bit 3 ignored) -> {8, 25, 43, 0} by c & 3, negative when c & 4.
// bf16 patterns of the magnitudes in two words: bytes 0-1 = 8, 2-3 = 25, 4-5 = 43, 6-7 = 0.
__device__ __forceinline__ void iq2c_words(uint32_t v, uint32_t (&w)[4]) {
  constexpr uint32_t kP0 = 0x41C84100u, kP1 = 0x0000422Cu;
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    const uint32_t x = (v >> (8 * p)) & 0xFFu;
    const uint32_t m0 = x & 3u, m1 = (x >> 4) & 3u;
    const uint32_t sel = (m0 * 0x22u + 0x10u) | ((m1 * 0x22u + 0x10u) << 8);
    w[p] = __byte_perm(kP0, kP1, sel) | ((x & 0x04u) << 13) | ((x & 0x40u) << 25);
  }
}
// FP4S: nibble -> bf16 pattern of E2M1 * 2^-126 (as fp4_patterns), pairs (low, high) of each byte.
__device__ __forceinline__ void fp4s_words(uint32_t v, uint32_t (&w)[4]) {
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    const uint32_t x = (v >> (8 * p)) & 0xFFu;
    w[p] = ((x & 0x07u) << 6) | ((x & 0x08u) << 12) | ((x & 0x70u) << 18) | ((x & 0x80u) << 24);
  }
}
// e4m3fn byte (torch.float8_e4m3fn: signed, 0x7F / 0xFF NaN, subnormal for e == 0) -> bf16 bits of
// value * 2^110 (exact: 4 significant bits, exponent within bf16's normal range).
__device__ __forceinline__ uint32_t e4m3fn_bf16_bits_x2p110(uint32_t b) {
  const uint32_t sign = (b & 0x80u) << 8;
  if ((b & 0x7Fu) == 0x7Fu) return sign | 0x7FC0u;
  const uint32_t e = (b >> 3) & 15u, m = b & 7u;
  if (e != 0u) return sign | ((e + 230u) << 7) | (m << 4);
  if (m == 0u) return sign;
  return sign | (__float_as_uint(static_cast<float>(m) * 0x1p101f) >> 16);
}

// IQ2_XXS codebook (bf16x2) replicated 8x into shared memory: entry e, copy c at e*128 + c*16, so
// the 8 lanes of each quarter-warp read distinct bank groups whatever entries they pick.  Called by
// threads 0..kThreads-1; each issues all of its (L2-resident) loads before its first store, so the
// fill costs one L2 round trip instead of one per iteration.
template <int kThreads>
__device__ __forceinline__ void fill_iq2_lut_bf16(uint8_t* smem, int tid) {
  constexpr int kN = 256 * 8, kIt = (kN + kThreads - 1) / kThreads;
  const uint4* src = reinterpret_cast<const uint4*>(&g_iq2_mag_bf16[0][0]);
  uint4 v[kIt];
#pragma unroll
  for (int j = 0; j < kIt; ++j) {
    const int i = tid + j * kThreads;
    v[j] = i < kN ? __ldg(src + (i >> 3)) : make_uint4(0u, 0u, 0u, 0u);
  }
#pragma unroll
  for (int j = 0; j < kIt; ++j) {
    const int i = tid + j * kThreads;
    if (i < kN) reinterpret_cast<uint4*>(smem)[i] = v[j];
  }
}

}  // namespace gguf_b200
