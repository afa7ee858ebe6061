// Single-activation-row IQ2_XXS GEMV (R = 1) on the integer tensor cores: mma.sync m16n8k32 with
// u8 weight magnitudes against the activation row carried as two 8-bit limbs.
//
// Weights.  An IQ2_XXS weight is s * m with m in {8, 25, 43} (the grid) and s = +-1, times the
// sub-block scale d * (0.5 + s4) * 0.25.  The tensor cores see A = 64 + s * m, an exact u8 in
// [21, 107]: one shared table gives, per 8-weight grid entry, the bytes 64 + m (indexed by the grid
// byte), a second one byte masks 0x3F / 0x00 marking the negative weights (indexed by the 7-bit sign
// index; the table holds the parity bit of the 8th sign), and per 4 weights
// A = X - 2 * (X & mask) (one LOP3 + one IMAD, no borrow between bytes).  The offset is removed in
// the epilogue: sum(w * x) = sum(A * x) - 64 * sum(x).  Both tables are replicated 16x
// (replica = lane & 15), so the 8-byte lookups of a half-warp never share a bank.
//
// Activations.  Each 32-element group of x (the sub-block the weight scale belongs to) is converted
// once per launch to integers x_int = x * 2^(14 - E), E = the exponent of the group's largest
// |x|, |x_int| <= 32640, split as x_int = 256 * hi + lo (hi s8, lo u8).  The conversion (exact
// power-of-two products, then a round-to-integer by adding 1.5 * 2^23) is exact for every element
// within a factor 2^7 of the group maximum (the bf16 significand then fits); smaller elements are
// rounded (nearest, ties to even) to a step of 2^(E - 14), i.e. 2^-14 of the group maximum.  Products and sums are exact in s32; the epilogue applies 2^(E - 14) and the weight scale
// in fp32.
//
// MMA layout (block-diagonal B, as in the bf16 slice kernel): k-slots 4t..4t+3 belong to group t
// and 4t+16..4t+19 to group t+4; MMA step j (0..7) takes elements 4j..4j+3 of every group, so the
// eight groups of a 256-element slice stay in separate C columns.  Lane (g, t) decodes groups t and
// t+4 of rows g and g+8 and supplies the x limbs of group t (if g == t) or t+4 (if g == t+4).
// Two s32 accumulators per slice: A . x_hi and A . x_lo.
#pragma once

#include "engine.cuh"
#include "rms_norm.cuh"
#include "slice_r1.cuh"

namespace gguf_b200 {

// Shared-memory tables: 256-byte slot e holds the 16 replicas (8 bytes each, replica = lane & 15) of
// codebook entry e as 64 + magnitude bytes (slot bytes 0..127) and, for e < 128, of sign pattern e
// as 0x3F per negative byte (slot bytes 128..255).  With a 256-byte slot the magnitude address of
// grid byte k of a record word is one byte-permute: [lane_off, byte k, 0, 0].
constexpr int kI8Lut = 256 * 256;

__device__ __forceinline__ uint32_t i8_mag_addr(uint32_t grid_word, int e, uint32_t lane_off) {
  return __byte_perm(grid_word, lane_off, 0x5504u | (static_cast<uint32_t>(e) << 4));
}
// Sign field e (bits 7e..7e+6 of the aux word) * 256 + 128 + lane_off; lane_off128 = lane_off | 128.
__device__ __forceinline__ uint32_t i8_sgn_addr(uint32_t aux, int e, uint32_t lane_off128) {
  const uint32_t f = e == 0 ? (aux << 8) : (e == 1 ? (aux << 1) : (aux >> (7 * e - 8)));
  return (f & 0x7F00u) | lane_off128;
}

__device__ __forceinline__ void imma_u8s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                          uint32_t b1) {
  asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void imma_u8u8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                          uint32_t b1) {
  asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.u8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// atomic add on a shared-memory counter with acquire-release semantics at CTA scope: publishes the
// caller's (and, through a preceding __syncwarp, its warp's) shared-memory writes and, for the
// last arriver, makes every earlier arriver's writes visible.
__device__ __forceinline__ int atom_add_acq_rel_cta(int* p, int v) {
  int old;
  asm volatile("atom.acq_rel.cta.shared::cta.add.s32 %0, [%1], %2;" : "=r"(old) : "r"(smem_u32(p)), "r"(v) : "memory");
  return old;
}

// bf16 bits -> (sign, significand with the implicit bit, effective biased exponent)
__device__ __forceinline__ void bf16_parts(uint32_t b, int& neg, int& sig, int& ex) {
  neg = (b >> 15) & 1;
  const int e = (b >> 7) & 0xFF;
  sig = (b & 0x7F) | (e ? 0x80 : 0);
  ex = e ? e : 1;
}

// x_int = x * 2^(14 - E) for an element with parts (neg, sig, ex) in a group whose largest
// effective exponent is emax: sig * 2^(ex - emax + 7), rounded to nearest (ties away) below 2^0.
__device__ __forceinline__ int bf16_to_fixed(int neg, int sig, int ex, int emax) {
  const int sh = ex - emax + 7;  // <= 7
  int v;
  if (sh >= 0) {
    v = sig << sh;
  } else {
    const int n = -sh;
    v = n > 9 ? 0 : ((sig + (1 << (n - 1))) >> n);
  }
  return neg ? -v : v;
}

// ---------------------------------------------------------------------------------------------
// Building blocks shared by the single-row GEMV and the single-row MoE kernel
// ---------------------------------------------------------------------------------------------
// B fragments of one 256-element activation slice (block-diagonal; see the header comment).
struct I8XFrag {
  uint32_t bh0[8], bl0[8], bh1[8], bl1[8];
  float xs0, xs1;    // 2^(E - 14) of the lane's C columns (groups 2t, 2t+1)
  int xoff0, xoff1;  // 64 * sum(x_int) of those columns
};

// Converts the 8 activations xv (elements 8l..8l+7 of the slice, l = lane) into the warp's
// fragments: lane l handles group l >> 2; the group's scale and sum are reduced over the quad.
template <bool kLibPow2 = false>
__device__ __forceinline__ void i8_x_frag(const uint4 xv, I8XFrag& f) {
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const bool dlo = (g == t), dhi = (g == t + 4);
  const uint32_t wv[4] = {xv.x, xv.y, xv.z, xv.w};
  // largest |x| of the group: bf16 magnitudes order like their bit patterns
  uint32_t mb = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) mb = max(mb, max(wv[i] & 0x7FFFu, (wv[i] >> 16) & 0x7FFFu));
  mb = max(mb, __shfl_xor_sync(0xffffffffu, mb, 1));
  mb = max(mb, __shfl_xor_sync(0xffffffffu, mb, 2));
  const int emax = max(1, static_cast<int>(mb >> 7));  // effective biased exponent of the maximum
  // x_int = x * 2^(14 - E) without branches: two exact power-of-two products (the first 2^64 for
  // groups below 2^-63), then adding 1.5 * 2^23 rounds to an integer (nearest, ties to even) whose
  // low 16 bits are x_int: byte 1 = the high limb x_int >> 8 (s8), byte 0 = the low limb (u8).
  const bool tiny = emax < 64;
  const float s1 = tiny ? 18446744073709551616.0f : 1.0f;  // 2^64
  const float s2 = __uint_as_float(static_cast<uint32_t>(268 - emax - (tiny ? 64 : 0)) << 23);  // 2^(141 - emax) / s1
  uint32_t r[8], rsum = 0u;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float v = __uint_as_float(i & 1 ? (wv[i >> 1] & 0xFFFF0000u) : (wv[i >> 1] << 16));
    r[i] = __float_as_uint((v * s1) * s2 + 12582912.0f);
    rsum += r[i];
  }
  uint32_t hw[2], lw[2];
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    hw[k] = __byte_perm(__byte_perm(r[4 * k], r[4 * k + 1], 0x0051u), __byte_perm(r[4 * k + 2], r[4 * k + 3], 0x0051u), 0x5410u);
    lw[k] = __byte_perm(__byte_perm(r[4 * k], r[4 * k + 1], 0x0040u), __byte_perm(r[4 * k + 2], r[4 * k + 3], 0x0040u), 0x5410u);
  }
  int xsum = static_cast<int>(rsum - 8u * 0x4B400000u);  // sum of x_int (mod 2^32, exact)
  xsum += __shfl_xor_sync(0xffffffffu, xsum, 1);
  xsum += __shfl_xor_sync(0xffffffffu, xsum, 2);
  // owner of group c: lane (g = c, t = c) for c < 4, lane (g = c, t = c - 4) for c >= 4.  Step j of
  // group c = elements 4j..4j+3 = word (j & 1) of lane 4c + (j >> 1).
  const int c = dlo ? t : (dhi ? t + 4 : 0);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int src = 4 * c + (j >> 1);
    const uint32_t h = __shfl_sync(0xffffffffu, hw[j & 1], src);
    const uint32_t l = __shfl_sync(0xffffffffu, lw[j & 1], src);
    f.bh0[j] = dlo ? h : 0u;
    f.bl0[j] = dlo ? l : 0u;
    f.bh1[j] = dhi ? h : 0u;
    f.bl1[j] = dhi ? l : 0u;
  }
  const int e0 = __shfl_sync(0xffffffffu, emax, 4 * (2 * t)), e1 = __shfl_sync(0xffffffffu, emax, 4 * (2 * t + 1));
  f.xoff0 = 64 * __shfl_sync(0xffffffffu, xsum, 4 * (2 * t));
  f.xoff1 = 64 * __shfl_sync(0xffffffffu, xsum, 4 * (2 * t + 1));
  // kLibPow2: ldexpf instead of the bit-built power (the single-row MoE kernel, whose register
  // allocation spilled more with the latter and measured 0.65 µs slower per call)
  f.xs0 = kLibPow2 ? ldexpf(1.0f, e0 - 141) : pow2i(e0 - 141);  // 2^(E - 14), E = emax - 127
  f.xs1 = kLibPow2 ? ldexpf(1.0f, e1 - 141) : pow2i(e1 - 141);
}

// B fragments of one 256-element activation slice with permuted columns: column 2t of the
// block-diagonal B carries group t and column 2t + 1 group t + 4, so the C cells lane (g, t) holds
// (rows g, g + 8 x groups t, t + 4) are exactly the records it decodes and the sub-block scales need
// no shuffles.  Lane (g, t)'s b0 is non-zero for g = 2t, b1 for g = 2t + 1.  Conversion as
// i8_x_frag: x_int = x * 2^(14 - E) per 32-element group, split into a signed high and an unsigned
// low byte.  xs0 / xoff0 belong to the lane's column 2t (group t), xs1 / xoff1 to column 2t + 1.
__device__ __forceinline__ void perm_x_frag(const uint4 xv, I8XFrag& f) {
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const bool dlo = (g == 2 * t), dhi = (g == 2 * t + 1);
  const uint32_t wv[4] = {xv.x, xv.y, xv.z, xv.w};
  uint32_t mb = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) mb = max(mb, max(wv[i] & 0x7FFFu, (wv[i] >> 16) & 0x7FFFu));
  mb = max(mb, __shfl_xor_sync(0xffffffffu, mb, 1));
  mb = max(mb, __shfl_xor_sync(0xffffffffu, mb, 2));
  const int emax = max(1, static_cast<int>(mb >> 7));
  const bool tiny = emax < 64;
  const float s1 = tiny ? 18446744073709551616.0f : 1.0f;  // 2^64
  const float s2 = __uint_as_float(static_cast<uint32_t>(268 - emax - (tiny ? 64 : 0)) << 23);
  uint32_t r[8], rsum = 0u;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float v = __uint_as_float(i & 1 ? (wv[i >> 1] & 0xFFFF0000u) : (wv[i >> 1] << 16));
    r[i] = __float_as_uint((v * s1) * s2 + 12582912.0f);
    rsum += r[i];
  }
  uint32_t hw[2], lw[2];
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    hw[k] = __byte_perm(__byte_perm(r[4 * k], r[4 * k + 1], 0x0051u), __byte_perm(r[4 * k + 2], r[4 * k + 3], 0x0051u), 0x5410u);
    lw[k] = __byte_perm(__byte_perm(r[4 * k], r[4 * k + 1], 0x0040u), __byte_perm(r[4 * k + 2], r[4 * k + 3], 0x0040u), 0x5410u);
  }
  int xsum = static_cast<int>(rsum - 8u * 0x4B400000u);
  xsum += __shfl_xor_sync(0xffffffffu, xsum, 1);
  xsum += __shfl_xor_sync(0xffffffffu, xsum, 2);
  // the group this lane's non-zero B column carries; step j of group c = word (j & 1) of lane 4c + (j >> 1)
  const int c = dlo ? t : (dhi ? t + 4 : 0);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int src = 4 * c + (j >> 1);
    const uint32_t h = __shfl_sync(0xffffffffu, hw[j & 1], src);
    const uint32_t l = __shfl_sync(0xffffffffu, lw[j & 1], src);
    f.bh0[j] = dlo ? h : 0u;
    f.bl0[j] = dlo ? l : 0u;
    f.bh1[j] = dhi ? h : 0u;
    f.bl1[j] = dhi ? l : 0u;
  }
  const int e0 = __shfl_sync(0xffffffffu, emax, 4 * t), e1 = __shfl_sync(0xffffffffu, emax, 4 * (t + 4));
  f.xoff0 = 64 * __shfl_sync(0xffffffffu, xsum, 4 * t);
  f.xoff1 = 64 * __shfl_sync(0xffffffffu, xsum, 4 * (t + 4));
  f.xs0 = pow2i(e0 - 141);  // 2^(E - 14)
  f.xs1 = pow2i(e1 - 141);
}

// The records of one slice for lane (g, t): grid bytes + sign/scale words of rows g, g+8 x groups
// t, t+4 (rc[0..3] = [g, t], [g, t+4], [g+8, t], [g+8, t+4]) and the two super-block scales.
// r0 / r1: byte offsets of rows g / g+8 in the stage; so: the slice's byte offset in a row (its
// records are 4-byte aligned iff `al`).
__device__ __forceinline__ void i8_records(const uint8_t* st, uint32_t r0, uint32_t r1, uint32_t so, bool al,
                                           uint2 (&rc)[4], uint32_t& dbits) {
  const uint32_t t = threadIdx.x & 3;
  rc[0] = lds8(st, r0 + so + 2u + 8u * t, al);
  rc[1] = lds8(st, r0 + so + 34u + 8u * t, al);
  rc[2] = lds8(st, r1 + so + 2u + 8u * t, al);
  rc[3] = lds8(st, r1 + so + 34u + 8u * t, al);
  dbits = ld_u16(st, r0 + so) | (ld_u16(st, r1 + so) << 16);
}
// The same for rows whose byte offsets may differ in alignment from lane to lane (odd row sizes):
// every 8-byte record is read as three aligned words and funnel-shifted (a shift of 0 when aligned).
__device__ __forceinline__ uint2 lds8_any(const uint8_t* base, uint32_t off) {
  const uint32_t* w = reinterpret_cast<const uint32_t*>(base + (off & ~3u));
  const uint32_t sh = (off & 2u) * 8u, w0 = w[0], w1 = w[1], w2 = w[2];
  return make_uint2(__funnelshift_r(w0, w1, sh), __funnelshift_r(w1, w2, sh));
}
__device__ __forceinline__ void i8_records_any(const uint8_t* st, uint32_t r0, uint32_t r1, uint32_t so, uint2 (&rc)[4],
                                               uint32_t& dbits) {
  const uint32_t t = threadIdx.x & 3;
  rc[0] = lds8_any(st, r0 + so + 2u + 8u * t);
  rc[1] = lds8_any(st, r0 + so + 34u + 8u * t);
  rc[2] = lds8_any(st, r1 + so + 2u + 8u * t);
  rc[3] = lds8_any(st, r1 + so + 34u + 8u * t);
  dbits = ld_u16(st, r0 + so) | (ld_u16(st, r1 + so) << 16);
}

// One 16-row x 256-column slice: decode (tables at shared offset 0), 16 MMAs, fp32 epilogue.  Gives
// the lane's partial sums of rows g (acc0) and g+8 (acc1) over its C columns; the caller reduces
// them over the quad (shuffles by 1 and 2).
__device__ __forceinline__ void i8_slice(const uint8_t* smem, const uint2 (&rc)[4], uint32_t dbits, const I8XFrag& f,
                                         float& acc0, float& acc1) {
  const int lane = threadIdx.x & 31, t = lane & 3;
  const uint32_t lane_off = static_cast<uint32_t>(lane & 15) * 8u, lane_off128 = lane_off | 128u;
  const int q0 = (lane & ~3) | ((2 * t) & 3), q1 = (lane & ~3) | ((2 * t + 1) & 3);
  const int sel_sh = t >= 2 ? 4 : 0;
  int ch[4] = {0, 0, 0, 0}, cl[4] = {0, 0, 0, 0};
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    uint32_t A[4][2];
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const uint2 X = *reinterpret_cast<const uint2*>(smem + i8_mag_addr(rc[r].x, e, lane_off));
      const uint2 M = *reinterpret_cast<const uint2*>(smem + i8_sgn_addr(rc[r].y, e, lane_off128));
      A[r][0] = X.x - 2u * (X.x & M.x);  // 64 + s*m per byte, no borrow between bytes
      A[r][1] = X.y - 2u * (X.y & M.y);
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int j = 2 * e + h;
      imma_u8s8(ch, A[0][h], A[2][h], A[1][h], A[3][h], f.bh0[j], f.bh1[j]);
      imma_u8u8(cl, A[0][h], A[2][h], A[1][h], A[3][h], f.bl0[j], f.bl1[j]);
    }
  }
  // exact s32 dot products of the lane's four (row, group) cells: sum(A x) - 64 sum(x)
  const float f0 = static_cast<float>(ch[0] * 256 + cl[0] - f.xoff0);
  const float f1 = static_cast<float>(ch[1] * 256 + cl[1] - f.xoff1);
  const float f2 = static_cast<float>(ch[2] * 256 + cl[2] - f.xoff0);
  const float f3 = static_cast<float>(ch[3] * 256 + cl[3] - f.xoff1);
  const uint32_t mine = (rc[0].y >> 28) | ((rc[1].y >> 28) << 4) | ((rc[2].y >> 28) << 8) | ((rc[3].y >> 28) << 12);
  const uint32_t p0 = __shfl_sync(0xffffffffu, mine, q0) >> sel_sh, p1 = __shfl_sync(0xffffffffu, mine, q1) >> sel_sh;
  const float d0s = fp16_bits_to_f32(dbits & 0xFFFFu) * 0.25f, d1s = fp16_bits_to_f32(dbits >> 16) * 0.25f;
  // 0.5 + s exactly: float(2^23 + s) - (2^23 - 0.5)
  const float h00 = __uint_as_float((p0 & 15u) | 0x4B000000u) - 8388607.5f;
  const float h01 = __uint_as_float((p1 & 15u) | 0x4B000000u) - 8388607.5f;
  const float h10 = __uint_as_float(((p0 >> 8) & 15u) | 0x4B000000u) - 8388607.5f;
  const float h11 = __uint_as_float(((p1 >> 8) & 15u) | 0x4B000000u) - 8388607.5f;
  acc0 = (f0 * (f.xs0 * h00) + f1 * (f.xs1 * h01)) * d0s;
  acc1 = (f2 * (f.xs0 * h10) + f3 * (f.xs1 * h11)) * d1s;
}

// 16 replicas of each 8-byte table entry at shared offset 0 (64 + magnitudes and sign masks in the
// 256-byte slots described at kI8Lut), two replicas per 16-byte store; called by threads
// 0..kThreads-1, each issuing all of its loads before its first store (one L2 round trip).  With
// kSign8 the sign half of every slot e (not only e < 128) holds sign pattern e & 127, so that an
// 8-bit field of the aux word whose top bit belongs to the next field indexes it directly.
template <int kThreads, bool kSign8 = false>
__device__ __forceinline__ void i8_fill_tables(uint8_t* smem, int tid) {
  constexpr int kSigns = kSign8 ? 256 : 128;
  constexpr int kStores = (256 + kSigns) * 8, kIters = (kStores + kThreads - 1) / kThreads;
  uint2 v[kIters];
#pragma unroll
  for (int j = 0; j < kIters; ++j) {
    const int i = tid + j * kThreads, ent = i >> 3;
    v[j] = i >= kStores ? make_uint2(0u, 0u)
                        : (ent < 256 ? __ldg(reinterpret_cast<const uint2*>(&g_iq2_mag_u8[ent][0]))
                                     : __ldg(reinterpret_cast<const uint2*>(&g_iq2_sign_mask[(ent - 256) & 127][0])));
    // magnitudes -> 64 + m (m < 64), sign masks -> 0x3F per negative byte
    const uint32_t op = ent < 256 ? 0x40404040u : 0u, and_ = ent < 256 ? 0xFFFFFFFFu : 0x3F3F3F3Fu;
    v[j] = make_uint2((v[j].x & and_) | op, (v[j].y & and_) | op);
  }
#pragma unroll
  for (int j = 0; j < kIters; ++j) {
    const int i = tid + j * kThreads;
    const int ent = i >> 3, slot = ent < 256 ? ent * 256 : (ent - 256) * 256 + 128;
    if (i < kStores) *reinterpret_cast<uint4*>(smem + slot + (i & 7) * 16) = make_uint4(v[j].x, v[j].y, v[j].x, v[j].y);
  }
}

// Stage = one 16-row tile (one bulk copy, see `fill`).  There is no dedicated producer warp (a 17th
// warp would cap every thread at 96 registers) and no CTA-wide barrier per tile: each warp writes
// its 16 partial row sums into the stage's reduction slot and increments the stage's counter
// (acquire-release); the warp that arrives last sums the slot in warp order (deterministic), stores
// y, resets the counter and refills the stage with the tile `stages` rounds ahead.  Every warp read
// the stage's records before incrementing, so the refill cannot overwrite data still in use, and a
// slot is rewritten only after its stage has been refilled, i.e. after it was summed.
template <int kW>
__global__ void __launch_bounds__(kW * 32, 1) slice_iq2_i8_kernel(const __grid_constant__ SliceArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + a.off_bar);
  uint8_t* stages = smem + a.off_stage;
  float* red = reinterpret_cast<float*>(smem + a.off_red);  // [stages][kW][16]
  int* cnt = reinterpret_cast<int*>(red + a.stages * kW * 16);  // [stages]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < a.stages; ++s) {
      mbar_init(&full[s], 1);
      cnt[s] = 0;
    }
    fence_mbar_init();
  }
  __syncthreads();
  pdl_launch_dependents();

  // stage s <- tile `tile` (lane 0 of the calling warp): one copy per tile (the copy engine's
  // throughput per SM is bounded by copies in flight, not bytes: 1 KB row copies would cap a GPU
  // near 2.4 TB/s).  Either one 2-D tensor box at the padded pitch a.stride (row bytes a multiple of
  // 32, see attach_slice_tmap) or one bulk copy with the rows contiguous (pitch = row bytes); there a
  // tail of < 16 bytes (rows * row bytes not a multiple of 16) is copied with plain loads before the
  // arrive, whose release orders it for the consumers.
  auto fill = [&](int s, int tile) {
    if (lane == 0 && a.use_tmap) {  // one 2-D box at the padded pitch a.stride (see attach_slice_tmap)
      mbar_arrive_expect_tx(&full[s], 16u * static_cast<uint32_t>(a.stride));
      tma_load_2d(stages + s * a.stage_bytes, &a.tmap, 0, tile * 16, &full[s]);
    } else if (lane == 0) {
      const int rv = min(16, a.N - tile * 16);
      const uint32_t bytes = static_cast<uint32_t>(rv * a.row_bytes), main = bytes & ~15u;
      const uint8_t* src = a.w + static_cast<int64_t>(tile) * 16 * a.row_bytes;
      uint8_t* dst = stages + s * a.stage_bytes;
      for (uint32_t b = main; b < bytes; ++b) dst[b] = src[b];
      mbar_arrive_expect_tx(&full[s], main);
      if (main) bulk_g2s(dst, src, main, &full[s]);
    }
  };
  // Two stages are requested before the dependency wait, the rest once every warp has issued its load
  // of x: behind all eight stages' bulk copies that load returned late (C1: 10.22 -> 9.83 µs).
  const int pre = min(a.stages, 2);
  if (warp == 0)
    for (int j = 0; j < pre; ++j) {
      const int tile = blockIdx.x + j * gridDim.x;
      if (tile < a.tiles) fill(j, tile);
    }

  // ---------------- tables, built while the first tiles are in flight ----------------
  i8_fill_tables<kW * 32>(smem, threadIdx.x);
  __syncthreads();

  const int g = lane >> 2, t = lane & 3;
  Gamma8 gm;  // fused norm: gamma is a weight, fetched before the dependency wait
  if (a.gamma != nullptr) gm = load_gamma8(a.gamma, warp * 32 + lane);
  pdl_wait();  // x is produced by the previous kernel

  // ---- x fragments of this warp's slice: lane l converts elements 8l..8l+7 (group l >> 2) ----
  uint4 xv = ldg128(a.x + warp * 256 + 8 * lane);
  if (pre < a.stages) {
    __syncthreads();  // every warp's x load is issued before the remaining stages' copies
    if (warp == 0)
      for (int j = pre; j < a.stages; ++j) {
        const int tile = blockIdx.x + j * gridDim.x;
        if (tile < a.tiles) fill(j, tile);
      }
  }
  if (a.gamma != nullptr) {
    // fused (Skip)RmsNorm: thread t holds chunk t of the 4096-element row, the layout of the
    // standalone kernel's 512 threads, so the mean of squares (and every output bit) is the same
    // (the host enables it for K = 4096 only, where kW = 16 warps = 512 threads)
    if (a.skip != nullptr) {
      xv = bf16x8_add(xv, ldg128(a.skip + warp * 256 + 8 * lane));
      if (blockIdx.x == 0 && a.sum_out != nullptr)
        *reinterpret_cast<uint4*>(a.sum_out + warp * 256 + 8 * lane) = xv;
    }
    const float rs = rsqrtf(norm_block_sum(norm_accumulate(0.f, xv, 1.0f / static_cast<float>(a.K)), red) + a.eps);
    xv = norm_scale8(xv, gm, rs);
    if (blockIdx.x == 0 && a.x_norm_out != nullptr)
      *reinterpret_cast<uint4*>(a.x_norm_out + warp * 256 + 8 * lane) = xv;
  }
  I8XFrag xf;
  i8_x_frag(xv, xf);
  const bool al = (warp & 1) != 0;  // odd super-block: records 4-byte aligned
  const uint32_t so = static_cast<uint32_t>(warp) * 66u;
  const uint32_t r0 = static_cast<uint32_t>(g * a.stride), r1 = static_cast<uint32_t>((g + 8) * a.stride);
  int s = 0;        // stage of this round
  uint32_t ph = 0;  // parity of the stage's current use
  // Records are software-pipelined: a round decodes the records loaded during the previous round
  // and loads the next round's, so their shared-memory latency overlaps the decode.
  uint2 rc[4];
  uint32_t dbits;
  if (static_cast<int>(blockIdx.x) < a.tiles) {
    mbar_wait(&full[0], 0u, kSiteFullWait);
    i8_records(stages, r0, r1, so, al, rc, dbits);
  }
  for (int tile = blockIdx.x; tile < a.tiles; tile += gridDim.x) {
    const int sn = s + 1 == a.stages ? 0 : s + 1;
    const uint32_t phn = sn == 0 ? ph ^ 1u : ph;
    uint2 rcn[4];
    uint32_t dbitsn = 0;
    if (tile + static_cast<int>(gridDim.x) < a.tiles) {
      mbar_wait(&full[sn], phn, kSiteFullWait);
      i8_records(stages + sn * a.stage_bytes, r0, r1, so, al, rcn, dbitsn);
    }

    float acc0, acc1;
    i8_slice(smem, rc, dbits, xf, acc0, acc1);

    acc0 += __shfl_xor_sync(0xffffffffu, acc0, 1);
    acc0 += __shfl_xor_sync(0xffffffffu, acc0, 2);
    acc1 += __shfl_xor_sync(0xffffffffu, acc1, 1);
    acc1 += __shfl_xor_sync(0xffffffffu, acc1, 2);
    float* rb = red + s * kW * 16;
    if (t == 0) {
      rb[warp * 16 + g] = acc0;
      rb[warp * 16 + g + 8] = acc1;
    }
    __syncwarp();  // orders the lanes' slot writes before lane 0's release below
    int last = 0;
    if (lane == 0) last = atom_add_acq_rel_cta(&cnt[s], 1) == kW - 1;
    if (__shfl_sync(0xffffffffu, last, 0)) {  // every warp's partials of this tile are in the slot
      if (lane < 16) {
        float v[4] = {0.f, 0.f, 0.f, 0.f};  // fixed summation order: 4 strided partial sums, then a tree
#pragma unroll
        for (int w2 = 0; w2 < kW; ++w2) v[w2 & 3] += rb[w2 * 16 + lane];
        const int row = tile * 16 + lane;
        if (row < a.N) a.y[row] = __float2bfloat16((v[0] + v[1]) + (v[2] + v[3]));
      }
      __syncwarp();
      if (lane == 0) cnt[s] = 0;
      const int next = tile + a.stages * static_cast<int>(gridDim.x);
      if (next < a.tiles) {
        fence_proxy_async_smem();  // the warps' generic reads of the stage before the copy engine's writes
        fill(s, next);
      }
    }
    s = sn;
    ph = phn;
#pragma unroll
    for (int r = 0; r < 4; ++r) rc[r] = rcn[r];
    dbits = dbitsn;
  }
}

}  // namespace gguf_b200
