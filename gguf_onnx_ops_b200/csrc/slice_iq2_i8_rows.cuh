// Few-row IQ2_XXS GEMV on the integer tensor cores: the single-row kernel's exact u8 weights
// (64 + s * m, from the same shared tables, slice_iq2_i8.cuh) against 4 * kNR activation rows per
// launch (kNR = 1 for 2 <= R <= 4, kNR = 2 for 5 <= R <= 8 at K = 4096).
//
// MMA layout (mma.sync m16n8k32, u8 x s8 -> s32).  One MMA covers one 32-element group of a 16-row
// tile: its k-slots 4t..4t+3 / 4t+16..4t+19 hold elements 8t..8t+3 / 8t+4..8t+7 of the group, so lane
// (g, t) decodes grid entry t of the group's records for rows g and g+8 (one magnitude and one sign
// lookup each), and its 8 columns are four activation rows x two limbs: column 2i = the high limb of
// activation row i, column 2i+1 = the low limb.  Every column carries data (the single-row kernel's
// block-diagonal B uses one in eight), so one decoded tile serves four activation rows per MMA;
// activation rows 4..7 take a second MMA on the same A fragments.  C column pair (2t, 2t+1) of lane
// (g, t) is activation row t: its full 32-element sums for weight rows g and g+8, no quad shuffles.
//
// Activations.  Per (activation row, group) x_int = x * 2^(13 - E), E = the exponent of the group's
// largest |x|, |x_int| <= 16320, split into two signed limbs x_int = 256 * hi + lo with
// hi = (x_int + 128) >> 8 in [-64, 64] and lo in [-128, 127] (both s8, so one MMA type serves both
// columns of a row).  Exact for every element within a factor 2^6 of the group maximum; smaller
// elements are rounded to a step of 2^-13 of it.  The weight offset is removed in the epilogue:
// sum((64 + s m) x) = 256 C_hi + C_lo - 64 sum(x_int), then scaled by 2^(E - 13) and the sub-block
// scale d * (0.5 + s4) / 4 in fp32.
#pragma once

#include "slice_iq2_i8.cuh"

namespace gguf_b200 {

// D = A . B + C with C in separate registers (the per-group offset enters as C, no init moves).
__device__ __forceinline__ void imma_u8s8_c(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                            uint32_t b0, uint32_t b1, int c0, int c1) {
  asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%11,%10,%11};\n"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(c0), "r"(c1));
}

// B fragments and per-(activation row, group) constants of one 256-element slice (kOff: with the
// offset sums that an unsigned A operand needs).
template <int kNR, bool kOff = true>
struct I8RowsX {
  uint32_t b[kNR][8][2];           // [MMA set][group][k-slots 4t.. / 4t+16..]
  float xs[kNR][8];                // 2^(E - 13) of activation row 4m + t, group j (this lane's C columns)
  int nxoff[kOff ? kNR : 1][8];    // -64 * sum(x_int) of the same (the low-limb column's C input)
};

// Lane (g, t), MMA set m: B column g = activation row 4m + (g >> 1), limb g & 1, k-slots of elements
// 8t..8t+7 of each group of that row.  The two lanes of a column pair (g even: high limb, g odd: low
// limb, lanes l and l ^ 4) share the conversion: the even lane converts elements 8t..8t+3, the odd
// one 8t+4..8t+7, each forms both limbs of its four and one shuffle swaps the word the other needs.
// Group maximum and sum are reduced over the eight lanes of the column pair's two quads.  Rows >= R
// read as zeros.
//
// Conversion without branches: p = x * 2^(13 - E) as two exact power-of-two products (the first is
// 2^64 for groups below 2^-63, so that neither factor leaves the normal range), then
// r = p + (1.5 * 2^23 + 128) rounds p to an integer (nearest, ties to even) whose low 16 bits are
// those of x_int + 128: byte 1 is the high limb (x_int + 128) >> 8 and byte 0 ^ 0x80 the low limb
// x_int mod 256.
// The load half: the lane's activation words (issued at once; i8_rows_x_cvt consumes them).
template <int kNR>
__device__ __forceinline__ void i8_rows_x_load(const bf16* x, int R, int K, int slice, uint2 (&xv)[kNR][8]) {
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const bool odd = (g & 1) != 0;
#pragma unroll
  for (int m = 0; m < kNR; ++m) {
    const int xr = 4 * m + (g >> 1);
#pragma unroll
    for (int j = 0; j < 8; ++j)
      xv[m][j] = xr < R ? __ldg(reinterpret_cast<const uint2*>(x + static_cast<int64_t>(xr) * K + slice * 256 + 32 * j +
                                                               8 * t + (odd ? 4 : 0)))
                        : make_uint2(0u, 0u);
  }
}
template <int kNR, bool kOff = true>
__device__ __forceinline__ void i8_rows_x_cvt(const uint2 (&xv)[kNR][8], I8RowsX<kNR, kOff>& f);
template <int kNR, bool kOff = true>
__device__ __forceinline__ void i8_rows_x(const bf16* x, int R, int K, int slice, I8RowsX<kNR, kOff>& f) {
  uint2 xv[kNR][8];
  i8_rows_x_load<kNR>(x, R, K, slice, xv);
  i8_rows_x_cvt<kNR, kOff>(xv, f);
}
// The conversion half.
template <int kNR, bool kOff>
__device__ __forceinline__ void i8_rows_x_cvt(const uint2 (&xv)[kNR][8], I8RowsX<kNR, kOff>& f) {
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const bool odd = (g & 1) != 0;
  const float magic = 12582912.0f + 128.0f;
#pragma unroll
  for (int m = 0; m < kNR; ++m) {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint32_t wv[2] = {xv[m][j].x, xv[m][j].y};
      // largest |x| of the group: bf16 magnitudes order like their bit patterns
      const uint32_t m2 = __vmaxu2(wv[0] & 0x7FFF7FFFu, wv[1] & 0x7FFF7FFFu);
      uint32_t mb = max(m2 & 0xFFFFu, m2 >> 16);
      mb = max(mb, __shfl_xor_sync(0xffffffffu, mb, 4));
      mb = max(mb, __shfl_xor_sync(0xffffffffu, mb, 1));
      mb = max(mb, __shfl_xor_sync(0xffffffffu, mb, 2));
      const int emax = max(1, static_cast<int>(mb >> 7));  // biased exponent of the maximum, E = emax - 127
      const bool tiny = emax < 64;
      const float s1 = tiny ? 18446744073709551616.0f : 1.0f;  // 2^64
      const float s2 = __uint_as_float(static_cast<uint32_t>(267 - emax - (tiny ? 64 : 0)) << 23);  // 2^(140 - emax) / s1
      uint32_t r[4], rsum = 0u;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float v = __uint_as_float(i & 1 ? (wv[i >> 1] & 0xFFFF0000u) : (wv[i >> 1] << 16));
        r[i] = __float_as_uint((v * s1) * s2 + magic);
        rsum += r[i];
      }
      const uint32_t hi = __byte_perm(__byte_perm(r[0], r[1], 0x0051u), __byte_perm(r[2], r[3], 0x0051u), 0x5410u);
      const uint32_t lo = __byte_perm(__byte_perm(r[0], r[1], 0x0040u), __byte_perm(r[2], r[3], 0x0040u), 0x5410u) ^ 0x80808080u;
      const uint32_t other = __shfl_xor_sync(0xffffffffu, odd ? hi : lo, 4);  // partner's word for my column
      f.b[m][j][0] = odd ? other : hi;  // elements 8t..8t+3
      f.b[m][j][1] = odd ? lo : other;  // elements 8t+4..8t+7
      // this lane's C columns (2t, 2t+1) are activation row 4m + t, converted by quads 2t, 2t + 1 (lane 8t)
      f.xs[m][j] = pow2i(__shfl_sync(0xffffffffu, emax, 8 * t) - 140);  // 2^(E - 13), E = emax - 127
      if constexpr (kOff) {
        int xsum = static_cast<int>(rsum - 4u * (0x4B400000u + 128u));  // sum of x_int (mod 2^32, exact)
        xsum += __shfl_xor_sync(0xffffffffu, xsum, 4);
        xsum += __shfl_xor_sync(0xffffffffu, xsum, 1);
        xsum += __shfl_xor_sync(0xffffffffu, xsum, 2);
        f.nxoff[m][j] = -64 * __shfl_sync(0xffffffffu, xsum, 8 * t);
      }
    }
  }
}

// One 16-row x 256-column slice against the kNR MMA sets: acc[m][0 / 1] += the slice's dot products
// of weight rows g / g+8 with activation row 4m + t.  Tables at shared offset 0 (sign halves filled
// for 8-bit indices); st = the stage, r0 / r1 = byte offsets of rows g / g+8, so = the slice's byte
// offset in a row (its records are 4-byte aligned iff `al`).
template <int kNR>
__device__ __forceinline__ void i8_rows_slice(const uint8_t* smem, const uint8_t* st, uint32_t r0, uint32_t r1,
                                              uint32_t so, bool al, const I8RowsX<kNR>& f, float (&acc)[kNR][2]) {
  const int lane = threadIdx.x & 31, t = lane & 3;
  const uint32_t lane_off = static_cast<uint32_t>(lane & 15) * 8u, lane_off128 = lane_off | 128u;
  const uint32_t sel = 0x5504u | (static_cast<uint32_t>(t) << 4);  // [lane_off, grid byte t, 0, 0]
  const uint32_t sh = 7u * static_cast<uint32_t>(t);                 // sign field t of the aux word
  const float d0 = fp16_bits_to_f32(ld_u16(st, r0 + so)) * 0.25f, h0 = 0.5f * d0;
  const float d1 = fp16_bits_to_f32(ld_u16(st, r1 + so)) * 0.25f, h1 = 0.5f * d1;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const uint2 q0 = lds8(st, r0 + so + 2u + 8u * j, al), q1 = lds8(st, r1 + so + 2u + 8u * j, al);
    const uint2 X0 = *reinterpret_cast<const uint2*>(smem + __byte_perm(q0.x, lane_off, sel));
    const uint2 M0 = *reinterpret_cast<const uint2*>(smem + __byte_perm(q0.y >> sh, lane_off128, 0x5504u));
    const uint2 X1 = *reinterpret_cast<const uint2*>(smem + __byte_perm(q1.x, lane_off, sel));
    const uint2 M1 = *reinterpret_cast<const uint2*>(smem + __byte_perm(q1.y >> sh, lane_off128, 0x5504u));
    // 64 + s*m per byte (no borrow between bytes): rows g / g+8, elements 8t..8t+3 / 8t+4..8t+7
    const uint32_t a0 = X0.x - 2u * (X0.x & M0.x), a2 = X0.y - 2u * (X0.y & M0.y);
    const uint32_t a1 = X1.x - 2u * (X1.x & M1.x), a3 = X1.y - 2u * (X1.y & M1.y);
    // sub-block scales d * (0.5 + s) / 4 (one rounding)
    const float w0 = fmaf(d0, static_cast<float>(q0.y >> 28), h0);
    const float w1 = fmaf(d1, static_cast<float>(q1.y >> 28), h1);
#pragma unroll
    for (int m = 0; m < kNR; ++m) {
      int cc[4];
      imma_u8s8_c(cc, a0, a1, a2, a3, f.b[m][j][0], f.b[m][j][1], 0, f.nxoff[m][j]);
      const float p = f.xs[m][j];
      acc[m][0] = fmaf(static_cast<float>(cc[0] * 256 + cc[1]), p * w0, acc[m][0]);
      acc[m][1] = fmaf(static_cast<float>(cc[2] * 256 + cc[3]), p * w1, acc[m][1]);
    }
  }
}

// Staging and the cross-warp reduction follow slice_iq2_i8_kernel: warp w owns slice w of K for the
// whole launch, a stage holds one 16-row tile, the last warp to finish a tile sums the stage's
// reduction slot in warp order, stores y [R, N] and refills the stage.  The tile arrives as one bulk
// copy (rows contiguous, pitch = row bytes) or, where that pitch would put rows g and g+4 on the same
// shared-memory banks (row bytes = 0 mod 32 words), as one 2-D tensor box with a 16-byte row pad:
// the record loads of the eight quads (rows 0..7, then 8..15) then hit eight distinct bank pairs.
template <int kW, int kNR>
__global__ void __launch_bounds__(kW * 32, 1) slice_iq2_i8_rows_kernel(const __grid_constant__ SliceArgs a) {
  constexpr int kRX = 4 * kNR;  // activation rows per launch (padded)
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + a.off_bar);
  uint8_t* stages = smem + a.off_stage;
  float* red = reinterpret_cast<float*>(smem + a.off_red);  // [stages][kW][kRX][16]
  int* cnt = reinterpret_cast<int*>(red + a.stages * kW * kRX * 16);  // [stages]
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

  auto fill = [&](int s, int tile) {
    if (lane == 0 && a.use_tmap) {
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
  if (warp == 0)
    for (int j = 0; j < a.stages; ++j) {
      const int tile = blockIdx.x + j * gridDim.x;
      if (tile < a.tiles) fill(j, tile);
    }

  i8_fill_tables<kW * 32, true>(smem, threadIdx.x);
  __syncthreads();
  pdl_wait();  // x is produced by the previous kernel

  I8RowsX<kNR> xf;
  i8_rows_x<kNR>(a.x, a.R, a.K, warp, xf);
  const int g = lane >> 2, t = lane & 3;
  const bool al = (warp & 1) != 0;  // odd super-block: records 4-byte aligned
  const uint32_t so = static_cast<uint32_t>(warp) * 66u;
  const uint32_t r0 = static_cast<uint32_t>(g * a.stride), r1 = static_cast<uint32_t>((g + 8) * a.stride);
  int s = 0;
  uint32_t ph = 0;
  for (int tile = blockIdx.x; tile < a.tiles; tile += gridDim.x) {
    mbar_wait(&full[s], ph, kSiteFullWait);
    float acc[kNR][2];
#pragma unroll
    for (int m = 0; m < kNR; ++m) acc[m][0] = acc[m][1] = 0.f;
    i8_rows_slice<kNR>(smem, stages + s * a.stage_bytes, r0, r1, so, al, xf, acc);

    float* rb = red + (s * kW + warp) * kRX * 16;
#pragma unroll
    for (int m = 0; m < kNR; ++m) {
      rb[(4 * m + t) * 16 + g] = acc[m][0];
      rb[(4 * m + t) * 16 + g + 8] = acc[m][1];
    }
    __syncwarp();  // orders the lanes' slot writes before lane 0's release below
    int last = 0;
    if (lane == 0) last = atom_add_acq_rel_cta(&cnt[s], 1) == kW - 1;
    if (__shfl_sync(0xffffffffu, last, 0)) {  // every warp's partials of this tile are in the slot
      const float* rs = red + s * kW * kRX * 16;
#pragma unroll
      for (int o = lane; o < kRX * 16; o += 32) {
        float v[4] = {0.f, 0.f, 0.f, 0.f};  // fixed summation order: 4 strided partial sums, then a tree
#pragma unroll
        for (int w2 = 0; w2 < kW; ++w2) v[w2 & 3] += rs[w2 * kRX * 16 + o];
        const int xr = o >> 4, row = tile * 16 + (o & 15);
        if (xr < a.R && row < a.N) a.y[static_cast<int64_t>(xr) * a.N + row] = __float2bfloat16((v[0] + v[1]) + (v[2] + v[3]));
      }
      __syncwarp();
      if (lane == 0) cnt[s] = 0;
      const int next = tile + a.stages * static_cast<int>(gridDim.x);
      if (next < a.tiles) {
        fence_proxy_async_smem();  // the warps' generic reads of the stage before the copy engine's writes
        fill(s, next);
      }
    }
    if (++s == a.stages) {
      s = 0;
      ph ^= 1u;
    }
  }
}

}  // namespace gguf_b200
