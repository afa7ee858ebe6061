// Single-activation-row GEMV (R = 1, the decode case) for Q8_0, IQ2_XXS and NVFP4.
//
// Each of the kW consumer warps owns kSPW fixed 256-element K slices of every 16-row weight tile,
// so its B fragments (x) stay in registers for the whole kernel.  With one activation row seven
// of the eight MMA columns of m16n8k16 would be idle; they are used instead to separate eight
// "groups" of 32 (or 16) elements: column c of the B operand holds x restricted to group c (a
// block-diagonal B), so C[row, c] is the row's dot product with group c alone and a per-group
// scale is applied once in fp32 after the MMAs.
//
// k-slot mapping: MMA slots (2t, 2t+1) <-> group t, slots (2t+8, 2t+9) <-> group t+4, each MMA
// taking one element pair of every group.  Lane (g, t) therefore decodes groups t and t+4 of rows
// g and g+8 ("records" 0..3 = [g, t], [g, t+4], [g+8, t], [g+8, t+4]) and supplies x[group t] as
// b0 when g == t and x[group t+4] as b1 when g == t+4 (zero otherwise).  Its C registers hold
// columns 2t and 2t+1 of rows g and g+8.
//
//   IQ2_XXS : slice = one super-block, group = 32-element sub-block.  A = exact signed grid
//             magnitudes (codebook in shared memory, 8x replicated); per-group scale
//             d*(0.5+s)*0.25 in the epilogue.  16 MMAs per slice.
//   Q8_0    : slice = 8 blocks, group = block.  Each byte u = q + 128 is split into nibbles and
//             each nibble pair becomes an exact bf16x2 with one LOP3:
//             (v & 0x000F000F) | 0x43004300 = bf16(128 + lo), the high nibble gives bf16(2048 + 16 hi)
//             (0x4500 | hi).  The MMA then sums (2176 + u) x = (q + 2304) x over the group; the
//             epilogue subtracts 2304 * sum(x of the group) and scales by d.  32 MMAs per slice.
//   NVFP4   : slice = 4 blocks = two halves of 8 sub-blocks of 16 (group = sub-block).  f16 operands:
//             each nibble byte (element j low, j + 8 high) goes through sm_100's E2M1 converter
//             (cvt.rn.f16x2.e2m1x2), one instruction per element pair; x is scaled per slice by 2^s
//             (max |x| 2^s < 2^15, exact in f16).  The block-diagonal B puts each sub-block in its own
//             C column, so the UE4M3 scales are applied to the C cells in fp32 after each half's
//             MMAs (a 256-entry float table), and the epilogue multiplies by 2^-s and gscale.  16 MMAs
//             per slice.  (Before: the bf16 patterns (n * 0x1040) & 0x81C0 times scale * 2^110, four
//             instructions per pair, C2 R = 1 12.45 µs; the converter with an f16x2 scale multiply per
//             pair, 10.80 µs; now 10.07 µs.)
//
// Stage = one 16-row tile with the full K (per-row bulk copies into a padded stride).  The kW
// partial sums of a tile are combined through a double-buffered shared-memory array (one named
// barrier per tile).
#pragma once

#include "decode.cuh"

namespace gguf_b200 {

struct SliceArgs {
  const uint8_t* w;
  const bf16* x;
  const float* gscale;  // NVFP4 only
  bf16* y;
  int N, K, row_bytes, tiles;
  int R;  // activation rows (slice_iq2_i8_rows_kernel; the single-row kernels ignore it)
  int stride, stage_bytes, stages;
  int off_stage, off_red, off_bar;
  PeerOut po;  // npeer > 0: row-split shard, y stored into every GPU of the group (slice_r1_kernel)
  // fused (Skip)RmsNorm prologue (slice_iq2_i8_kernel, K = 4096): x <- RmsNorm(x [+ skip]) with the
  // standalone op's arithmetic (rms_norm.cuh); CTA 0 writes the normalised row / the sum if asked
  const float* gamma;  // null: no norm
  const bf16* skip;
  bf16* x_norm_out;
  bf16* sum_out;
  float eps;
  // slice_iq2_i8_rows_kernel: when use_tmap, a stage is one 2-D box of 16 rows x `stride` bytes
  // (the row bytes plus a 16-byte pad, zero-filled past the row end) instead of one bulk copy
  CUtensorMap tmap;
  int use_tmap;
  // slice_q8_i8_rows_kernel, split layout (Q8Gemv gguf=0): bf16 scales [N, K/32], sc_row_bytes = K/16,
  // staged after the 16 weight rows at stage offset sc_off
  const uint8_t* sc;
  int sc_row_bytes, sc_off;
  // slice_fp4_rows_kernel with two activation sets: byte offset of the per-warp fragment areas
  int off_x2;
};

template <int F>
struct SliceFmt;
template <>
struct SliceFmt<kFmtIQ2> {
  static constexpr int kSliceBytes = 66, kLut = 256 * 8 * 16;
};
template <>
struct SliceFmt<kFmtQ8> {
  static constexpr int kSliceBytes = 8 * 34, kLut = 0;
};
template <>
struct SliceFmt<kFmtFP4> {
  static constexpr int kSliceBytes = 4 * 36, kLut = 1024;
};

// 8 bytes at a 2-byte aligned offset; `al` = offset is 4-byte aligned (warp-uniform)
__device__ __forceinline__ uint2 lds8(const uint8_t* base, uint32_t off, bool al) {
  const uint32_t* w = reinterpret_cast<const uint32_t*>(base + (off & ~3u));
  if (al) return make_uint2(w[0], w[1]);
  const uint32_t w0 = w[0], w1 = w[1], w2 = w[2];
  return make_uint2(__funnelshift_r(w0, w1, 16), __funnelshift_r(w1, w2, 16));
}
// 32 bytes at a 2-byte aligned offset (alignment may differ per lane; branch free)
__device__ __forceinline__ void lds32b(const uint8_t* base, uint32_t off, uint32_t (&q)[8]) {
  const uint32_t* w = reinterpret_cast<const uint32_t*>(base + (off & ~3u));
  const uint32_t sh = (off & 2u) * 8u;
  uint32_t prev = w[0];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint32_t nxt = w[i + 1];
    q[i] = __funnelshift_r(prev, nxt, sh);
    prev = nxt;
  }
}
// c ^ (a & m): a masked field merged into constant bits c (c may overlap the field: XOR there)
__device__ __forceinline__ uint32_t lop_xm(uint32_t a, uint32_t m, uint32_t c) {
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0x6A;" : "=r"(r) : "r"(a), "r"(m), "r"(c));
  return r;
}
__device__ __forceinline__ uint32_t pair_lo(uint32_t w0, uint32_t w1) { return __byte_perm(w0, w1, 0x5410); }  // (w0.lo, w1.lo)
__device__ __forceinline__ uint32_t pair_hi(uint32_t w0, uint32_t w1) { return __byte_perm(w0, w1, 0x7632); }  // (w0.hi, w1.hi)


// E2M1 pairs -> f16x2 on the hardware converter: byte k of v (low nibble element j, high nibble
// element j + 8) -> d[k] = (element j in the low half, element j + 8 in the high half)
__device__ __forceinline__ void e2m1x4_to_f16x2(uint32_t v, uint32_t (&d)[4]) {
  asm("{\n .reg .b8 b0, b1, b2, b3;\n mov.b32 {b0, b1, b2, b3}, %4;\n cvt.rn.f16x2.e2m1x2 %0, b0;\n"
      " cvt.rn.f16x2.e2m1x2 %1, b1;\n cvt.rn.f16x2.e2m1x2 %2, b2;\n cvt.rn.f16x2.e2m1x2 %3, b3;\n}"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3]) : "r"(v));
}
__device__ __forceinline__ uint32_t hmul2_f16_bits(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
// A bf16 pair times sc (a power of two) as an f16 pair: exact while the products stay in f16's normal range.
__device__ __forceinline__ uint32_t f16x2_scaled(uint32_t w, float sc) {
  const float lo = __uint_as_float(w << 16) * sc, hi = __uint_as_float(w & 0xFFFF0000u) * sc;
  uint32_t d;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
  return d;
}
__device__ __forceinline__ void mma_f16_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                              uint32_t b0, uint32_t b1, const float (&c)[4]) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%11,%12,%13};\n"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(c[0]), "f"(c[1]), "f"(c[2]), "f"(c[3]));
}

template <int F, int kW, int kSPW>
__global__ void __launch_bounds__((kW + 1) * 32, 1) slice_r1_kernel(const SliceArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + a.off_bar);
  uint64_t* empty = full + a.stages;
  uint8_t* stages = smem + a.off_stage;
  float* red = reinterpret_cast<float*>(smem + a.off_red);  // [2][kW][16]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __shared__ uint32_t s_call;  // row-split: this launch's call number (its tag)

  if (threadIdx.x == 0) {
    for (int s = 0; s < a.stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kW);
    }
    fence_mbar_init();
    if (a.po.npeer) s_call = peer_call(a.po);  // before launch_dependents: see peer_call
  }
  __syncthreads();
  pdl_launch_dependents();

  if (warp == kW) {
    // ---------------- producer warp: one 16-row tile per stage, one bulk copy per row ----------------
    // Two stages are requested at once, the rest after the consumers have built their x fragments
    // (named barrier 2): a load of x issued behind the whole ring's copies into this SM returns late
    // (Q8 R = 1 at 4096 x 2048: 4.06 -> 3.97 µs; NVFP4 C2 R = 1: 12.51 -> 12.46 µs).
    constexpr uint32_t kPreStages = 2;
    uint32_t it = 0;
    bool released = false;
    for (int tile = blockIdx.x; tile < a.tiles; tile += gridDim.x, ++it) {
      if (it == kPreStages) {
        named_bar_sync(2, (kW + 1) * 32);
        released = true;
      }
      const int s = static_cast<int>(it % a.stages);
      const int rv = min(16, a.N - tile * 16);
      if (lane == 0) {
        if (it >= static_cast<uint32_t>(a.stages)) mbar_wait(&empty[s], ((it / a.stages) - 1) & 1, kSiteEmptyWait);
        mbar_arrive_expect_tx(&full[s], static_cast<uint32_t>(rv * a.row_bytes));
      }
      __syncwarp();
      if (lane < rv)
        bulk_g2s(stages + s * a.stage_bytes + lane * a.stride, a.w + (static_cast<int64_t>(tile) * 16 + lane) * a.row_bytes,
                 a.row_bytes, &full[s]);
    }
    if (!released) named_bar_sync(2, (kW + 1) * 32);  // every arrival of the consumers is matched
    if (lane == 0) {
      const uint32_t total = it;
      const uint32_t first = total > static_cast<uint32_t>(a.stages) ? total - a.stages : 0u;
      for (uint32_t j = first; j < total; ++j) mbar_wait(&full[j % a.stages], (j / a.stages) & 1, kSiteDrainWait);
    }
    return;
  }

  // ---------------- consumers ----------------
  // format tables, built while the first tiles are in flight
  if constexpr (F == kFmtIQ2) {  // codebook replicated 8x: conflict-free 16-byte lookups
    fill_iq2_lut_bf16<kW * 32>(smem, threadIdx.x);
  } else if constexpr (F == kFmtFP4) {
    // UE4M3 scale byte -> its value (the bf16 pattern of scale * 2^110, times 2^-110: exact)
    float* slf = reinterpret_cast<float*>(smem);
    for (int i = threadIdx.x; i < 256; i += kW * 32) slf[i] = __uint_as_float(fp4_scale_bf16_bits(i) << 16) * 0x1p-110f;
  }
  if constexpr (SliceFmt<F>::kLut > 0) named_bar_sync(1, kW * 32);

  const int g = lane >> 2, t = lane & 3;
  const bool dlo = (g == t), dhi = (g == t + 4);
  pdl_wait();  // x is produced by the previous kernel

  // ---- B fragments of this warp's slices, in MMA order ----
  uint32_t xa[kSPW][16], xb[kSPW][16];
  float xoff[kSPW][2];  // Q8: 2304 * sum(x) of the lane's C columns (groups 2t, 2t+1)
  float xinv[kSPW];     // NVFP4: 2^-s of the slice's x scaling
#pragma unroll
  for (int j = 0; j < kSPW; ++j) {
    const bf16* xs = a.x + (warp * kSPW + j) * 256;
    if constexpr (F == kFmtFP4) {
      // f16 operands: x scaled by 2^s per slice (max |x| * 2^s < 2^15, exact), pairs (e_j, e_j+8)
      uint4 vv[2][4];
      uint32_t mb = 0;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint4 v0 = make_uint4(0, 0, 0, 0), v1 = v0, u0 = v0, u1 = v0;
        if (dlo) v0 = ldg128(xs + h * 128 + 16 * t), v1 = ldg128(xs + h * 128 + 16 * t + 8);
        if (dhi) u0 = ldg128(xs + h * 128 + 16 * (t + 4)), u1 = ldg128(xs + h * 128 + 16 * (t + 4) + 8);
        vv[h][0] = v0; vv[h][1] = v1; vv[h][2] = u0; vv[h][3] = u1;
      }
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint4 u = vv[h][q];
          const uint32_t w4[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
          for (int i = 0; i < 4; ++i) mb = max(mb, max(w4[i] & 0x7FFFu, (w4[i] >> 16) & 0x7FFFu));
        }
      mb = __reduce_max_sync(0xffffffffu, mb);
      const int sx = min(127, 141 - static_cast<int>(mb >> 7));
      const float sc = pow2i(sx);
      xinv[j] = pow2i(-sx);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const uint32_t A[8] = {vv[h][0].x, vv[h][0].y, vv[h][0].z, vv[h][0].w, vv[h][1].x, vv[h][1].y, vv[h][1].z, vv[h][1].w};
        const uint32_t B[8] = {vv[h][2].x, vv[h][2].y, vv[h][2].z, vv[h][2].w, vv[h][3].x, vv[h][3].y, vv[h][3].z, vv[h][3].w};
        uint32_t* oa = &xa[j][8 * h];
        uint32_t* ob = &xb[j][8 * h];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          oa[2 * q] = f16x2_scaled(pair_lo(A[q], A[q + 4]), sc);
          oa[2 * q + 1] = f16x2_scaled(pair_hi(A[q], A[q + 4]), sc);
          ob[2 * q] = f16x2_scaled(pair_lo(B[q], B[q + 4]), sc);
          ob[2 * q + 1] = f16x2_scaled(pair_hi(B[q], B[q + 4]), sc);
        }
      }
    } else {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint4 va = make_uint4(0, 0, 0, 0), vb = va;
        if (dlo) va = ldg128(xs + 32 * t + 8 * q);
        if (dhi) vb = ldg128(xs + 32 * (t + 4) + 8 * q);
        if constexpr (F == kFmtQ8) {  // pairs (e0,e2) (e1,e3) (e4,e6) (e5,e7) of these 8 elements
          xa[j][4 * q + 0] = pair_lo(va.x, va.y); xa[j][4 * q + 1] = pair_hi(va.x, va.y);
          xa[j][4 * q + 2] = pair_lo(va.z, va.w); xa[j][4 * q + 3] = pair_hi(va.z, va.w);
          xb[j][4 * q + 0] = pair_lo(vb.x, vb.y); xb[j][4 * q + 1] = pair_hi(vb.x, vb.y);
          xb[j][4 * q + 2] = pair_lo(vb.z, vb.w); xb[j][4 * q + 3] = pair_hi(vb.z, vb.w);
        } else {  // IQ2: natural pairs (e0,e1) ... (e6,e7)
          xa[j][4 * q + 0] = va.x; xa[j][4 * q + 1] = va.y; xa[j][4 * q + 2] = va.z; xa[j][4 * q + 3] = va.w;
          xb[j][4 * q + 0] = vb.x; xb[j][4 * q + 1] = vb.y; xb[j][4 * q + 2] = vb.z; xb[j][4 * q + 3] = vb.w;
        }
      }
    }
    if constexpr (F == kFmtQ8) {
      float sa = 0.f, sb = 0.f;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        sa += bf16_lo(xa[j][i]) + bf16_hi(xa[j][i]);
        sb += bf16_lo(xb[j][i]) + bf16_hi(xb[j][i]);
      }
      // group c's sum is on lane (g = c, t = c & 3): sa for c < 4, sb for c >= 4
      const float mine = dlo ? sa : (dhi ? sb : 0.f);
      const int c0 = 2 * t, c1 = 2 * t + 1;
      xoff[j][0] = 2304.0f * __shfl_sync(0xffffffffu, mine, c0 * 4 + (c0 & 3));
      xoff[j][1] = 2304.0f * __shfl_sync(0xffffffffu, mine, c1 * 4 + (c1 & 3));
    } else {
      xoff[j][0] = xoff[j][1] = 0.f;
    }
  }
  named_bar_arrive(2, (kW + 1) * 32);  // x fragments built: the producer may request the other stages
  float post = 1.0f;
  if constexpr (F == kFmtFP4) post = __ldg(a.gscale);
  const uint32_t lut_lane = static_cast<uint32_t>(lane & 7) * 16u;
  const uint16_t* fp4lut = reinterpret_cast<const uint16_t*>(smem);
  const int q0 = (lane & ~3) | ((2 * t) & 3), q1 = (lane & ~3) | ((2 * t + 1) & 3);
  const int sel_sh = t >= 2 ? 4 : 0;

  uint32_t it = 0;
  for (int tile = blockIdx.x; tile < a.tiles; tile += gridDim.x, ++it) {
    const int s = static_cast<int>(it % a.stages);
    mbar_wait(&full[s], (it / a.stages) & 1, kSiteFullWait);
    const uint8_t* st = stages + s * a.stage_bytes;
    const uint32_t r0 = static_cast<uint32_t>(g * a.stride), r1 = static_cast<uint32_t>((g + 8) * a.stride);
    float acc0 = 0.f, acc1 = 0.f;  // rows g, g+8
#pragma unroll
    for (int j = 0; j < kSPW; ++j) {
      const int sl = warp * kSPW + j;
      const uint32_t so = static_cast<uint32_t>(sl) * SliceFmt<F>::kSliceBytes;
      float c[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
      if constexpr (F == kFmtIQ2) {
        const bool al = (sl & 1) != 0;  // odd super-block: records 4-byte aligned
        uint2 rc[4];
        rc[0] = lds8(st, r0 + so + 2u + 8u * t, al);
        rc[1] = lds8(st, r0 + so + 34u + 8u * t, al);
        rc[2] = lds8(st, r1 + so + 2u + 8u * t, al);
        rc[3] = lds8(st, r1 + so + 34u + 8u * t, al);
        const uint32_t dbits = ld_u16(st, r0 + so) | (ld_u16(st, r1 + so) << 16);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          uint4 m[4];
#pragma unroll
          for (int r = 0; r < 4; ++r) m[r] = *reinterpret_cast<const uint4*>(smem + lut_lane + (((rc[r].x >> (8 * e)) & 0xFFu) << 7));
          uint32_t A[4][4];
#pragma unroll
          for (int r = 0; r < 4; ++r) {
            const uint32_t si = (rc[r].y >> (7 * e)) & 0x7Fu;
            const uint32_t sb = si + (__popc(si) << 7);  // bits above bit 7 never reach bits 15 / 31 below
            A[r][0] = m[r].x ^ ((sb * 0x40008000u) & 0x80008000u);
            A[r][1] = m[r].y ^ ((sb * 0x10002000u) & 0x80008000u);
            A[r][2] = m[r].z ^ ((sb * 0x04000800u) & 0x80008000u);
            A[r][3] = m[r].w ^ ((sb * 0x01000200u) & 0x80008000u);
          }
#pragma unroll
          for (int wd = 0; wd < 4; ++wd) {
            const int i = 4 * e + wd;
            mma_bf16_16816(c[i & 1], A[0][wd], A[2][wd], A[1][wd], A[3][wd], xa[j][i], xb[j][i], c[i & 1]);
          }
        }
        const uint32_t mine = (rc[0].y >> 28) | ((rc[1].y >> 28) << 4) | ((rc[2].y >> 28) << 8) | ((rc[3].y >> 28) << 12);
        const uint32_t p0 = __shfl_sync(0xffffffffu, mine, q0) >> sel_sh, p1 = __shfl_sync(0xffffffffu, mine, q1) >> sel_sh;
        const float d0s = fp16_bits_to_f32(dbits & 0xFFFFu) * 0.25f, d1s = fp16_bits_to_f32(dbits >> 16) * 0.25f;
        // 0.5 + s exactly: float(2^23 + s) - (2^23 - 0.5)
        acc0 = fmaf(d0s * (__uint_as_float((p0 & 15u) | 0x4B000000u) - 8388607.5f), c[0][0] + c[1][0], acc0);
        acc0 = fmaf(d0s * (__uint_as_float((p1 & 15u) | 0x4B000000u) - 8388607.5f), c[0][1] + c[1][1], acc0);
        acc1 = fmaf(d1s * (__uint_as_float(((p0 >> 8) & 15u) | 0x4B000000u) - 8388607.5f), c[0][2] + c[1][2], acc1);
        acc1 = fmaf(d1s * (__uint_as_float(((p1 >> 8) & 15u) | 0x4B000000u) - 8388607.5f), c[0][3] + c[1][3], acc1);
      } else if constexpr (F == kFmtQ8) {
#pragma unroll
        for (int half = 0; half < 2; ++half) {  // payload words 4*half .. 4*half+3 of each block
          uint32_t q[4][4];
#pragma unroll
          for (int r = 0; r < 4; ++r) {
            const uint32_t off = (r < 2 ? r0 : r1) + so + 34u * static_cast<uint32_t>(t + 4 * (r & 1)) + 2u + 16u * half;
            const uint32_t* w = reinterpret_cast<const uint32_t*>(st + (off & ~3u));
            const uint32_t sh = (off & 2u) * 8u;
            const uint32_t w0 = w[0], w1 = w[1], w2 = w[2], w3 = w[3], w4 = w[4];
            q[r][0] = __funnelshift_r(w0, w1, sh);
            q[r][1] = __funnelshift_r(w1, w2, sh);
            q[r][2] = __funnelshift_r(w2, w3, sh);
            q[r][3] = __funnelshift_r(w3, w4, sh);
          }
#pragma unroll
          for (int wq = 0; wq < 4; ++wq) {
            const int w = 4 * half + wq;  // payload word index: elements 4w..4w+3
            uint32_t A[4][4];
#pragma unroll
            for (int r = 0; r < 4; ++r) {
              const uint32_t v = q[r][wq];
              A[r][0] = lop_xm(v, 0x000F000Fu, 0x43004300u);                   // (e0, e2) low nibbles: 128 + lo
              A[r][1] = lop_xm(v >> 4, 0x000F000Fu, 0x45084508u);              // (e0, e2) high: 2048 + 16 (hi ^ 8)
              A[r][2] = lop_xm(v >> 8, 0x000F000Fu, 0x43004300u);              // (e1, e3) low
              A[r][3] = lop_xm(v >> 12, 0x000F000Fu, 0x45084508u);             // (e1, e3) high
            }
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const int bi = 2 * w + (k >> 1);
              mma_bf16_16816(c[k & 1], A[0][k], A[2][k], A[1][k], A[3][k], xa[j][bi], xb[j][bi], c[k & 1]);
            }
          }
        }
        // scales of the lane's C columns: blocks 2t, 2t+1 of rows g, g+8
        const float d00 = fp16_bits_to_f32(ld_u16(st, r0 + so + 34u * (2 * t)));
        const float d01 = fp16_bits_to_f32(ld_u16(st, r0 + so + 34u * (2 * t + 1)));
        const float d10 = fp16_bits_to_f32(ld_u16(st, r1 + so + 34u * (2 * t)));
        const float d11 = fp16_bits_to_f32(ld_u16(st, r1 + so + 34u * (2 * t + 1)));
        acc0 = fmaf(d00, (c[0][0] + c[1][0]) - xoff[j][0], acc0);
        acc0 = fmaf(d01, (c[0][1] + c[1][1]) - xoff[j][1], acc0);
        acc1 = fmaf(d10, (c[0][2] + c[1][2]) - xoff[j][0], acc1);
        acc1 = fmaf(d11, (c[0][3] + c[1][3]) - xoff[j][1], acc1);
      } else {  // NVFP4
        // bare E2M1 values into the MMA; C column c of half h is one sub-block (block 2h + (c >> 2),
        // sub-block c & 3), so lane (g, t)'s cells (columns 2t, 2t+1) take the scales of block
        // 2h + (t >> 1), sub-blocks 2 (t & 1) and 2 (t & 1) + 1, applied in fp32 after the half's MMAs
        const float* slf = reinterpret_cast<const float*>(smem);
        float y0 = 0.f, y1 = 0.f;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          uint2 nb[4];
#pragma unroll
          for (int r = 0; r < 4; ++r) {
            const uint32_t bo = (r < 2 ? r0 : r1) + so + 36u * static_cast<uint32_t>(2 * h + (r & 1));
            const uint32_t* w = reinterpret_cast<const uint32_t*>(st + bo + 4u + 8u * t);
            nb[r] = make_uint2(w[0], w[1]);
          }
          const uint32_t sbo = so + 36u * static_cast<uint32_t>(2 * h + (t >> 1)) + 2u * static_cast<uint32_t>(t & 1);
          const uint32_t sb0 = ld_u16(st, r0 + sbo), sb1 = ld_u16(st, r1 + sbo);
          float ch[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
          for (int ui = 0; ui < 2; ++ui) {
            uint32_t A[4][4];
#pragma unroll
            for (int r = 0; r < 4; ++r) e2m1x4_to_f16x2(ui ? nb[r].y : nb[r].x, A[r]);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const int bi = 8 * h + 4 * ui + k;
              mma_f16_16816(ch[k & 1], A[0][k], A[2][k], A[1][k], A[3][k], xa[j][bi], xb[j][bi], ch[k & 1]);
            }
          }
          y0 = fmaf(ch[0][0] + ch[1][0], slf[sb0 & 0xFFu], y0);
          y0 = fmaf(ch[0][1] + ch[1][1], slf[sb0 >> 8], y0);
          y1 = fmaf(ch[0][2] + ch[1][2], slf[sb1 & 0xFFu], y1);
          y1 = fmaf(ch[0][3] + ch[1][3], slf[sb1 >> 8], y1);
        }
        acc0 += y0 * xinv[j];
        acc1 += y1 * xinv[j];
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);  // this warp no longer reads the stage
    acc0 += __shfl_xor_sync(0xffffffffu, acc0, 1);
    acc0 += __shfl_xor_sync(0xffffffffu, acc0, 2);
    acc1 += __shfl_xor_sync(0xffffffffu, acc1, 1);
    acc1 += __shfl_xor_sync(0xffffffffu, acc1, 2);
    // double-buffered partials: buffer (it & 1) is read by warp 0 after this tile's barrier and
    // rewritten only after the barrier of the tile after next, which warp 0 reaches once done.
    float* rb = red + (it & 1) * kW * 16;
    if (t == 0) {
      rb[warp * 16 + g] = acc0;
      rb[warp * 16 + g + 8] = acc1;
    }
    named_bar_sync(1, kW * 32);
    if (threadIdx.x < 16) {
      float v = 0.f;
#pragma unroll
      for (int w2 = 0; w2 < kW; ++w2) v += rb[w2 * 16 + threadIdx.x];
      const int row = tile * 16 + threadIdx.x;
      if (row < a.N) {
        if (a.po.npeer) peer_store(a.po, s_call, 0, row, __float2bfloat16(v * post));
        else a.y[row] = __float2bfloat16(v * post);
      }
    }
  }
  if (a.po.npeer) peer_gather(a.po, s_call, 1, threadIdx.x, kW * 32);  // the whole y, from the staging buffer
}

}  // namespace gguf_b200
