// Single-activation-row IQ2_XXS GEMV (R = 1) with row blocks owned by warp pairs.
//
// Same arithmetic as slice_iq2_i8.cuh (exact u8 operands 64 + s*m on the integer tensor cores, x as
// two 8-bit limbs per 32-element group, block-diagonal B), different work split: a 16-row block is
// owned by a pair of warps, each taking half of the K slices, so the only cross-warp step is one
// exchange of 16 partial row sums per block instead of a 16-warp reduction per 256-column slice.
// With one 16-row block per pair the decode of a whole block runs without any synchronisation.
//
//   * CTA = 16 warps = 8 pairs; pair p of CTA b takes blocks p * gridDim + b, + 8 * gridDim, ...
//   * Each pair has one stage (its block's rows, contiguous, one bulk copy) and a named barrier.
//   * The activation row is converted once per CTA into shared memory: per slice and group the
//     hi / lo limb words of the 8 MMA steps (64 bytes), the group scale 2^(E-14) and 64 * sum(x_int).
//     A warp loads its B fragments per slice (8 x 16-byte loads; lanes that supply no group read a
//     shared zero block).
#pragma once

#include "slice_iq2_i8.cuh"

namespace gguf_b200 {

struct RowBlockArgs {
  const uint8_t* w;
  const bf16* x;
  bf16* y;
  int N, K, row_bytes, blocks;
  int stage_bytes;
  int off_stage, off_x, off_red, off_bar;
};

constexpr int kRbPairs = 8, kRbWarps = 2 * kRbPairs;

__global__ void __launch_bounds__(kRbWarps * 32, 1) iq2_rowblock_kernel(const RowBlockArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + a.off_bar);  // [kRbPairs]
  uint8_t* xsm = smem + a.off_x;                                    // [slices][8 groups][64 B]
  float* xsc = reinterpret_cast<float*>(xsm + (a.K / 256) * 512);   // [slices][8] 2^(E-14)
  int* xof = reinterpret_cast<int*>(xsc + (a.K / 256) * 8);         // [slices][8] 64 * sum(x_int)
  const uint8_t* xzero = reinterpret_cast<const uint8_t*>(xof + (a.K / 256) * 8);  // 64 zero bytes
  float* red = reinterpret_cast<float*>(smem + a.off_red);          // [kRbPairs][16]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int pair = warp >> 1, half = warp & 1;
  const int slices = a.K / 256, my_slices = slices / 2, sl0 = half * my_slices;

  if (threadIdx.x == 0) {
    for (int p = 0; p < kRbPairs; ++p) mbar_init(&full[p], 1);
    fence_mbar_init();
  }
  if (threadIdx.x < 16) reinterpret_cast<uint32_t*>(const_cast<uint8_t*>(xzero))[threadIdx.x] = 0u;
  __syncthreads();
  pdl_launch_dependents();

  // this pair's first block: in flight before anything else
  auto fill = [&](int blk) {
    const int rv = min(16, a.N - blk * 16);
    const uint32_t bytes = static_cast<uint32_t>(rv * a.row_bytes), main = bytes & ~15u;
    const uint8_t* src = a.w + static_cast<int64_t>(blk) * 16 * a.row_bytes;
    uint8_t* dst = smem + a.off_stage + pair * a.stage_bytes;
    for (uint32_t b = main; b < bytes; ++b) dst[b] = src[b];
    mbar_arrive_expect_tx(&full[pair], main);
    if (main) bulk_g2s(dst, src, main, &full[pair]);
  };
  const int stride_blk = kRbPairs * static_cast<int>(gridDim.x);
  const int blk0 = pair * static_cast<int>(gridDim.x) + static_cast<int>(blockIdx.x);
  if (half == 0 && lane == 0 && blk0 < a.blocks) fill(blk0);

  i8_fill_tables<kRbWarps * 32>(smem, threadIdx.x);  // tables at offset 0 (kI8Lut bytes)

  pdl_wait();  // x is produced by the previous kernel
  // ---- x -> limbs: thread i converts elements 8i..8i+7 (group i >> 2 of slice i >> 5) ----
  for (int i = threadIdx.x; i < a.K / 8; i += kRbWarps * 32) {
    const uint4 v = ldg128(a.x + 8 * i);
    const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
    uint32_t mb = 0;
#pragma unroll
    for (int q = 0; q < 4; ++q) mb = max(mb, max(wv[q] & 0x7FFFu, (wv[q] >> 16) & 0x7FFFu));
    mb = max(mb, __shfl_xor_sync(0xffffffffu, mb, 1));
    mb = max(mb, __shfl_xor_sync(0xffffffffu, mb, 2));
    const int emax = max(1, static_cast<int>(mb >> 7));
    uint32_t hw[2] = {0u, 0u}, lw[2] = {0u, 0u};
    int xsum = 0;
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      int neg, sig, ex;
      bf16_parts(q & 1 ? (wv[q >> 1] >> 16) : (wv[q >> 1] & 0xFFFFu), neg, sig, ex);
      const int xi = bf16_to_fixed(neg, sig, ex, emax);
      xsum += xi;
      hw[q >> 2] |= (static_cast<uint32_t>(xi >> 8) & 0xFFu) << (8 * (q & 3));
      lw[q >> 2] |= (static_cast<uint32_t>(xi) & 0xFFu) << (8 * (q & 3));
    }
    xsum += __shfl_xor_sync(0xffffffffu, xsum, 1);
    xsum += __shfl_xor_sync(0xffffffffu, xsum, 2);
    const int grp = i >> 2, j0 = 2 * (i & 3);  // global group index (slice * 8 + group), first MMA step
    uint32_t* gw = reinterpret_cast<uint32_t*>(xsm + grp * 64);
    *reinterpret_cast<uint2*>(gw + j0) = make_uint2(hw[0], hw[1]);
    *reinterpret_cast<uint2*>(gw + 8 + j0) = make_uint2(lw[0], lw[1]);
    if ((i & 3) == 0) {
      xsc[grp] = pow2i(emax - 141);
      xof[grp] = 64 * xsum;
    }
  }
  __syncthreads();

  const int g = lane >> 2, t = lane & 3;
  const bool dlo = (g == t), dhi = (g == t + 4);
  const uint32_t lane_off = static_cast<uint32_t>(lane & 15) * 8u;
  const int q0 = (lane & ~3) | ((2 * t) & 3), q1 = (lane & ~3) | ((2 * t + 1) & 3);
  const int sel_sh = t >= 2 ? 4 : 0;
  uint8_t* st = smem + a.off_stage + pair * a.stage_bytes;
  uint32_t ph = 0;

  for (int blk = blk0; blk < a.blocks; blk += stride_blk) {
    mbar_wait(&full[pair], ph, kSiteFullWait);
    ph ^= 1u;
    const uint32_t r0 = static_cast<uint32_t>(g * a.row_bytes), r1 = static_cast<uint32_t>((g + 8) * a.row_bytes);
    float acc0 = 0.f, acc1 = 0.f;  // rows g, g+8
    for (int k = 0; k < my_slices; ++k) {
      const int sl = sl0 + k;
      // B fragments of this slice: b0 from group t (lanes g == t), b1 from group t + 4 (lanes
      // g == t + 4); every other lane reads the zero block (one broadcast address)
      uint32_t b0h[8], b0l[8], b1h[8], b1l[8];
      {
        const uint4* s0 = reinterpret_cast<const uint4*>(dlo ? xsm + (sl * 8 + t) * 64 : xzero);
        const uint4* s1 = reinterpret_cast<const uint4*>(dhi ? xsm + (sl * 8 + t + 4) * 64 : xzero);
        const uint4 u0 = s0[0], u1 = s0[1], u2 = s0[2], u3 = s0[3], v0 = s1[0], v1 = s1[1], v2 = s1[2], v3 = s1[3];
        b0h[0] = u0.x; b0h[1] = u0.y; b0h[2] = u0.z; b0h[3] = u0.w; b0h[4] = u1.x; b0h[5] = u1.y; b0h[6] = u1.z; b0h[7] = u1.w;
        b0l[0] = u2.x; b0l[1] = u2.y; b0l[2] = u2.z; b0l[3] = u2.w; b0l[4] = u3.x; b0l[5] = u3.y; b0l[6] = u3.z; b0l[7] = u3.w;
        b1h[0] = v0.x; b1h[1] = v0.y; b1h[2] = v0.z; b1h[3] = v0.w; b1h[4] = v1.x; b1h[5] = v1.y; b1h[6] = v1.z; b1h[7] = v1.w;
        b1l[0] = v2.x; b1l[1] = v2.y; b1l[2] = v2.z; b1l[3] = v2.w; b1l[4] = v3.x; b1l[5] = v3.y; b1l[6] = v3.z; b1l[7] = v3.w;
      }
      const float2 xs = *reinterpret_cast<const float2*>(xsc + sl * 8 + 2 * t);
      const int2 xo = *reinterpret_cast<const int2*>(xof + sl * 8 + 2 * t);
      const uint32_t so = static_cast<uint32_t>(sl) * 66u;
      const bool al = (sl & 1) != 0;  // odd super-block: records 4-byte aligned (row bytes % 4 == 0)
      uint2 rc[4];
      rc[0] = lds8(st, r0 + so + 2u + 8u * t, al);
      rc[1] = lds8(st, r0 + so + 34u + 8u * t, al);
      rc[2] = lds8(st, r1 + so + 2u + 8u * t, al);
      rc[3] = lds8(st, r1 + so + 34u + 8u * t, al);
      const uint32_t dbits = ld_u16(st, r0 + so) | (ld_u16(st, r1 + so) << 16);

      // one accumulator pair per grid entry: 4 independent chains of 2 MMAs instead of one chain of
      // 8 (the MMA latency, not its throughput, bounds a warp working through a block alone);
      // integer sums, so the regrouping is exact
      int ch4[4][4], cl4[4][4];
#pragma unroll
      for (int e = 0; e < 4; ++e)
#pragma unroll
        for (int q = 0; q < 4; ++q) ch4[e][q] = cl4[e][q] = 0;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        uint32_t A[4][2];
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          const uint2 X = *reinterpret_cast<const uint2*>(smem + i8_mag_addr(rc[r].x, e, lane_off));
          const uint2 M = *reinterpret_cast<const uint2*>(smem + i8_sgn_addr(rc[r].y, e, lane_off | 128u));
          A[r][0] = X.x - 2u * (X.x & M.x);
          A[r][1] = X.y - 2u * (X.y & M.y);
        }
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const int j = 2 * e + hh;
          imma_u8s8(ch4[e], A[0][hh], A[2][hh], A[1][hh], A[3][hh], b0h[j], b1h[j]);
          imma_u8u8(cl4[e], A[0][hh], A[2][hh], A[1][hh], A[3][hh], b0l[j], b1l[j]);
        }
      }
      int ch[4], cl[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        ch[q] = (ch4[0][q] + ch4[1][q]) + (ch4[2][q] + ch4[3][q]);
        cl[q] = (cl4[0][q] + cl4[1][q]) + (cl4[2][q] + cl4[3][q]);
      }
      const float f0 = static_cast<float>(ch[0] * 256 + cl[0] - xo.x);
      const float f1 = static_cast<float>(ch[1] * 256 + cl[1] - xo.y);
      const float f2 = static_cast<float>(ch[2] * 256 + cl[2] - xo.x);
      const float f3 = static_cast<float>(ch[3] * 256 + cl[3] - xo.y);
      const uint32_t mine = (rc[0].y >> 28) | ((rc[1].y >> 28) << 4) | ((rc[2].y >> 28) << 8) | ((rc[3].y >> 28) << 12);
      const uint32_t p0 = __shfl_sync(0xffffffffu, mine, q0) >> sel_sh, p1 = __shfl_sync(0xffffffffu, mine, q1) >> sel_sh;
      const float d0s = fp16_bits_to_f32(dbits & 0xFFFFu) * 0.25f, d1s = fp16_bits_to_f32(dbits >> 16) * 0.25f;
      const float h00 = __uint_as_float((p0 & 15u) | 0x4B000000u) - 8388607.5f;
      const float h01 = __uint_as_float((p1 & 15u) | 0x4B000000u) - 8388607.5f;
      const float h10 = __uint_as_float(((p0 >> 8) & 15u) | 0x4B000000u) - 8388607.5f;
      const float h11 = __uint_as_float(((p1 >> 8) & 15u) | 0x4B000000u) - 8388607.5f;
      acc0 = fmaf(d0s, f0 * (xs.x * h00) + f1 * (xs.y * h01), acc0);
      acc1 = fmaf(d1s, f2 * (xs.x * h10) + f3 * (xs.y * h11), acc1);
    }
    acc0 += __shfl_xor_sync(0xffffffffu, acc0, 1);
    acc0 += __shfl_xor_sync(0xffffffffu, acc0, 2);
    acc1 += __shfl_xor_sync(0xffffffffu, acc1, 1);
    acc1 += __shfl_xor_sync(0xffffffffu, acc1, 2);
    // pair exchange: the second half hands its 16 partial rows to the first, which stores y and
    // refills the pair's stage (both warps are past their reads of it at the barrier)
    float* rp = red + pair * 16;
    if (half == 1 && t == 0) {
      rp[g] = acc0;
      rp[g + 8] = acc1;
    }
    named_bar_sync(1 + pair, 64);
    if (half == 0) {
      if (t == 0) {
        const int row0 = blk * 16 + g, row1 = row0 + 8;
        if (row0 < a.N) a.y[row0] = __float2bfloat16(acc0 + rp[g]);
        if (row1 < a.N) a.y[row1] = __float2bfloat16(acc1 + rp[g + 8]);
      }
      const int next = blk + stride_blk;
      if (lane == 0 && next < a.blocks) {
        fence_proxy_async_smem();
        fill(next);
      }
    }
    named_bar_sync(1 + pair, 64);  // rp consumed before the next block's exchange
  }
}

}  // namespace gguf_b200
