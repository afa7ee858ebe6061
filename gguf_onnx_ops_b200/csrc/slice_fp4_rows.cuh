// Few-row NVFP4 GEMV (2 <= R <= 16) on the f16 tensor cores: the activation rows are the 8 columns
// of mma.sync m16n8k16, so one decoded tile serves every row (the single-row kernel, slice_r1.cuh,
// spends its columns on a block-diagonal B instead).
//
// Decode (as slice_r1.cuh): each nibble byte goes through sm_100's E2M1 converter
// (cvt.rn.f16x2.e2m1x2: low nibble to the low half) and one f16x2 multiply by the sub-block's scale
// (a 256-entry table of f16 scales in shared memory) makes the weight: exact, since E2M1 x UE4M3
// has at most 6 significant bits and stays above 2^-10.  Because the scale is inside A, the MMAs of
// a whole slice accumulate into one C: no per-sub-block epilogue.  The activations are f16 too:
// each activation row's slice is scaled by a power of two 2^s (its largest |x| times 2^s below
// 2^15, so every bf16 value converts exactly), and the epilogue multiplies column c by 2^-s(c) and
// gscale.  (The former bf16 decode, (n * 0x1040) & 0x81C0 times scale * 2^110, took four
// instructions per element pair.)
//
// k-slot mapping: lane (g, t) decodes sub-block t (elements 16t..16t+15) of every 64-element block
// of its slice, for rows g and g+8.  In GGUF NVFP4, element j < 8 of a sub-block is the low nibble
// of its byte j and element j + 8 the high nibble, so nibble byte j converts to the pair
// (j, j + 8); MMA q = 0..3 takes bytes 2q (k-slots 2t, 2t+1) and 2q+1 (k-slots 2t+8, 2t+9).  The B
// fragment of column g is activation row g at the same element pairs (rows >= R read as zeros),
// fixed for the launch; C column pair (2t, 2t+1) of lane (g, t) is activation rows 2t, 2t+1.
//
// Staging and reduction as the few-row Q8_0 kernel (slice_q8_i8_rows.cuh): 16 whole rows per stage,
// one bulk copy per row at a pitch of row bytes + 32 (with the row words = 0 or 16 mod 32 the eight
// quads' loads would share banks), the last warp to finish a tile sums the slot in warp order.
#pragma once

#include "slice_r1.cuh"
#include "slice_iq2_i8.cuh"

namespace gguf_b200 {

// kSplit: the legacy layout of Nvfp4Gemv gguf=0 (u8 [N, K/2] nibbles with element 2i the low nibble
// of byte i, e4m3fn scales [N, K/16] in a second tensor).  Its nibble byte i converts to the pair
// (2i, 2i + 1), so MMA q takes bytes q and q + 4; the scale table holds e4m3fn values, and a stage
// carries the tile's 16 scale rows after its 16 weight rows (lane t's nibbles: bytes 32 b + 8 t of
// the slice).
// kF16: f16 operands (hardware E2M1 conversion, one activation set only); otherwise the bf16 decode,
// whose lighter x prologue the host picks for short launches and for two activation sets (R = 9..16:
// 4096 x 4096 R = 16 6.59 against 7.89 µs, 13824 x 5120 21.34 against 21.44 µs; 4096 x 4096 R = 4
// 4.63 against 4.86 µs, where 13824 x 5120 R = 2 / 8 take 11.98 / 13.72 against 13.01 / 14.52 µs).
template <int kW, bool kSplit = false, int kNB = 1, bool kF16 = false>
__global__ void __launch_bounds__(kW * 32, 1) slice_fp4_rows_kernel(const __grid_constant__ SliceArgs a) {
  static_assert(kNB == 1 || (kNB == 2 && !kSplit), "two activation sets: GGUF layout only");
  static_assert(!kF16 || kNB == 1, "f16 operands: one activation set");
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + a.off_bar);
  uint8_t* stages = smem + a.off_stage;
  float* red = reinterpret_cast<float*>(smem + a.off_red);  // [stages][kW][8 kNB activation rows][16]
  int* cnt = reinterpret_cast<int*>(red + a.stages * kW * 8 * kNB * 16);  // [stages]
  const uint16_t* fp4lut = reinterpret_cast<const uint16_t*>(smem);  // [256] scale: f16 bits (kF16) or bf16 * 2^110
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < a.stages; ++s) {
      mbar_init(&full[s], 1);
      cnt[s] = 0;
    }
    fence_mbar_init();
  }
  for (int i = threadIdx.x; i < 256; i += kW * 32) {
    // kF16: the scale value (exact in f16) from its bf16 pattern times 2^110; else that pattern
    const uint32_t b = kSplit ? e4m3fn_bf16_bits_x2p110(i) : fp4_scale_bf16_bits(i);
    reinterpret_cast<uint16_t*>(smem)[i] =
        kF16 ? __half_as_ushort(__float2half_rn(__uint_as_float(b << 16) * 0x1p-110f)) : static_cast<uint16_t>(b);
  }
  __syncthreads();
  pdl_launch_dependents();

  // stage s <- tile `tile` (the calling warp): lane 0 announces the bytes, lanes < rows copy a row each
  auto fill = [&](int s, int tile) {
    const int rv = min(16, a.N - tile * 16);
    const uint32_t scb = kSplit ? static_cast<uint32_t>(rv * a.sc_row_bytes) : 0u;  // the tile's scale rows
    if (lane == 0) mbar_arrive_expect_tx(&full[s], static_cast<uint32_t>(rv * a.row_bytes) + scb);
    __syncwarp();
    if (lane < rv)
      bulk_g2s(stages + s * a.stage_bytes + lane * a.stride, a.w + (static_cast<int64_t>(tile) * 16 + lane) * a.row_bytes,
               static_cast<uint32_t>(a.row_bytes), &full[s]);
    if (kSplit && lane == 16)
      bulk_g2s(stages + s * a.stage_bytes + a.sc_off, a.sc + static_cast<int64_t>(tile) * 16 * a.sc_row_bytes, scb, &full[s]);
  };
  if (warp == 0)
    for (int j = 0; j < a.stages; ++j) {
      const int tile = blockIdx.x + j * gridDim.x;
      if (tile < a.tiles) fill(j, tile);
    }
  const float gs = __ldg(a.gscale);  // a weight: read before the wait
  pdl_wait();  // x is produced by the previous kernel

  const int g = lane >> 2, t = lane & 3;
  // ---- B fragments: activation row g, elements 16t..16t+15 of the slice's four blocks ----
  uint32_t xb[4][4][2];  // [block][MMA][b0 / b1] of activation rows 0..7
  // kNB = 2: the fragments of activation rows 8..15, packed once per launch into this warp's
  // [block][MMA][lane] area of shared memory (one 8-byte load per MMA, conflict-free)
  uint2* xs2 = reinterpret_cast<uint2*>(smem + a.off_x2) + warp * 16 * 32;
  float post[kNB][2];  // gscale (times 2^-s of the column's activation row, kF16; else 2^16)
  if constexpr (kF16) {
#pragma unroll
    for (int nb = 0; nb < kNB; ++nb) {
      uint4 u[4][2];
      uint32_t mb = 0;
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        u[b][0] = u[b][1] = make_uint4(0u, 0u, 0u, 0u);
        if (8 * nb + g < a.R) {
          const bf16* xp = a.x + static_cast<int64_t>(8 * nb + g) * a.K + warp * 256 + 64 * b + 16 * t;
          u[b][0] = ldg128(xp);
          u[b][1] = ldg128(xp + 8);
        }
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const uint32_t w4[4] = {u[b][h].x, u[b][h].y, u[b][h].z, u[b][h].w};
#pragma unroll
          for (int i = 0; i < 4; ++i) mb = max(mb, max(w4[i] & 0x7FFFu, (w4[i] >> 16) & 0x7FFFu));
        }
      }
      // the row's largest magnitude over its quad (the row's whole slice), its scale 2^s (s <= 127)
      mb = max(mb, __shfl_xor_sync(0xffffffffu, mb, 1));
      mb = max(mb, __shfl_xor_sync(0xffffffffu, mb, 2));
      const int sx = min(127, 141 - static_cast<int>(mb >> 7));
      const float sc = pow2i(sx);
      post[nb][0] = gs * pow2i(-__shfl_sync(0xffffffffu, sx, 4 * (2 * t)));
      post[nb][1] = gs * pow2i(-__shfl_sync(0xffffffffu, sx, 4 * (2 * t + 1)));
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const uint32_t lo[4] = {u[b][0].x, u[b][0].y, u[b][0].z, u[b][0].w};  // (x0, x1) .. (x6, x7)
        const uint32_t hi[4] = {u[b][1].x, u[b][1].y, u[b][1].z, u[b][1].w};  // (x8, x9) .. (x14, x15)
        uint32_t f[4][2];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          if constexpr (kSplit) {  // (x2q, x2q+1), (x2q+8, x2q+9)
            f[q][0] = f16x2_scaled(lo[q], sc);
            f[q][1] = f16x2_scaled(hi[q], sc);
          } else {  // (x2q, x2q+8), (x2q+1, x2q+9)
            f[q][0] = f16x2_scaled(pair_lo(lo[q], hi[q]), sc);
            f[q][1] = f16x2_scaled(pair_hi(lo[q], hi[q]), sc);
          }
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          if (nb == 0) {
            xb[b][q][0] = f[q][0];
            xb[b][q][1] = f[q][1];
          } else {
            xs2[(b * 4 + q) * 32 + lane] = make_uint2(f[q][0], f[q][1]);
          }
        }
      }
    }
  } else {
    post[0][0] = post[0][1] = post[kNB - 1][0] = post[kNB - 1][1] = 65536.0f * gs;
#pragma unroll
    for (int nb = 0; nb < kNB; ++nb) {
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        uint4 u0 = make_uint4(0u, 0u, 0u, 0u), u1 = u0;
        if (8 * nb + g < a.R) {
          const bf16* xp = a.x + static_cast<int64_t>(8 * nb + g) * a.K + warp * 256 + 64 * b + 16 * t;
          u0 = ldg128(xp);
          u1 = ldg128(xp + 8);
        }
        uint32_t f[4][2];
        if constexpr (kSplit) {
          f[0][0] = pair_lo(u0.x, u0.z);  // (x0, x4)
          f[0][1] = pair_hi(u0.x, u0.z);  // (x1, x5)
          f[1][0] = pair_lo(u0.y, u0.w);  // (x2, x6)
          f[1][1] = pair_hi(u0.y, u0.w);  // (x3, x7)
          f[2][0] = pair_lo(u1.x, u1.z);  // (x8, x12)
          f[2][1] = pair_hi(u1.x, u1.z);  // (x9, x13)
          f[3][0] = pair_lo(u1.y, u1.w);  // (x10, x14)
          f[3][1] = pair_hi(u1.y, u1.w);  // (x11, x15)
        } else {
          f[0][0] = pair_lo(u0.x, u0.y);  // (x0, x2)
          f[0][1] = pair_lo(u1.x, u1.y);  // (x8, x10)
          f[1][0] = pair_hi(u0.x, u0.y);  // (x1, x3)
          f[1][1] = pair_hi(u1.x, u1.y);  // (x9, x11)
          f[2][0] = pair_lo(u0.z, u0.w);  // (x4, x6)
          f[2][1] = pair_lo(u1.z, u1.w);  // (x12, x14)
          f[3][0] = pair_hi(u0.z, u0.w);  // (x5, x7)
          f[3][1] = pair_hi(u1.z, u1.w);  // (x13, x15)
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          if (nb == 0) {
            xb[b][q][0] = f[q][0];
            xb[b][q][1] = f[q][1];
          } else {
            xs2[(b * 4 + q) * 32 + lane] = make_uint2(f[q][0], f[q][1]);
          }
        }
      }
    }
  }
  if (kNB == 2) __syncwarp();  // each warp reads back only its own area
  const uint32_t so = static_cast<uint32_t>(warp) * (kSplit ? 128u : 144u);  // four blocks per slice
  const uint32_t sc0 = static_cast<uint32_t>(a.sc_off + g * a.sc_row_bytes) + 16u * warp;   // split: the slice's
  const uint32_t sc1 = static_cast<uint32_t>(a.sc_off + (g + 8) * a.sc_row_bytes) + 16u * warp;  // 16 scale bytes
  const uint32_t r0 = static_cast<uint32_t>(g * a.stride), r1 = static_cast<uint32_t>((g + 8) * a.stride);
  int s = 0;
  uint32_t ph = 0;
  for (int tile = blockIdx.x; tile < a.tiles; tile += gridDim.x) {
    mbar_wait(&full[s], ph, kSiteFullWait);
    const uint8_t* st = stages + s * a.stage_bytes;
    // two accumulator chains: the MMA parity (one activation set) or the set (kNB = 2)
    float c[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      uint32_t v0[2], v1[2], s0, s1;
      if constexpr (kSplit) {  // nibbles: 32 bytes per block, lane t's sub-block at 8 t; scales staged apart
        const uint2 n0 = *reinterpret_cast<const uint2*>(st + r0 + so + 32u * b + 8u * t);
        const uint2 n1 = *reinterpret_cast<const uint2*>(st + r1 + so + 32u * b + 8u * t);
        v0[0] = n0.x; v0[1] = n0.y; v1[0] = n1.x; v1[1] = n1.y;
        s0 = fp4lut[st[sc0 + 4u * b + t]];
        s1 = fp4lut[st[sc1 + 4u * b + t]];
      } else {
        const uint32_t bo0 = r0 + so + 36u * b, bo1 = r1 + so + 36u * b;  // block: 4 scale bytes, 32 nibble bytes
        const uint32_t* w0 = reinterpret_cast<const uint32_t*>(st + bo0 + 4u + 8u * t);
        const uint32_t* w1 = reinterpret_cast<const uint32_t*>(st + bo1 + 4u + 8u * t);
        v0[0] = w0[0]; v0[1] = w0[1]; v1[0] = w1[0]; v1[1] = w1[1];
        s0 = fp4lut[st[bo0 + t]];
        s1 = fp4lut[st[bo1 + t]];
      }
      const uint32_t S0 = s0 | (s0 << 16), S1 = s1 | (s1 << 16);
      if constexpr (kF16) {  // one activation set
        uint32_t d0[8], d1[8];  // the converted pairs of bytes 0..7 of rows g / g+8, times the scale
        e2m1x4_to_f16x2(v0[0], reinterpret_cast<uint32_t(&)[4]>(d0[0]));
        e2m1x4_to_f16x2(v0[1], reinterpret_cast<uint32_t(&)[4]>(d0[4]));
        e2m1x4_to_f16x2(v1[0], reinterpret_cast<uint32_t(&)[4]>(d1[0]));
        e2m1x4_to_f16x2(v1[1], reinterpret_cast<uint32_t(&)[4]>(d1[4]));
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          d0[i] = hmul2_f16_bits(d0[i], S0);
          d1[i] = hmul2_f16_bits(d1[i], S1);
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int i0 = kSplit ? q : 2 * q, i2 = kSplit ? q + 4 : 2 * q + 1;  // k-slots 2t.. / 2t+8..
          mma_f16_16816(c[q & 1], d0[i0], d1[i0], d0[i2], d1[i2], xb[b][q][0], xb[b][q][1], c[q & 1]);
        }
      } else {  // bf16 decode
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint32_t u0 = (q & 1) ? (v0[q >> 1] >> 8) : v0[q >> 1];
          const uint32_t u1 = (q & 1) ? (v1[q >> 1] >> 8) : v1[q >> 1];
          // low nibbles of bytes 0, 2 of the (shifted) word and their high nibbles -> exact bf16 pairs
          // of E2M1 * 2^-126, times the scale * 2^110
          const uint32_t a0 = hmul2_bits(((u0 & 0x000F000Fu) * 0x1040u) & 0x81C081C0u, S0);
          const uint32_t a2 = hmul2_bits(((u0 & 0x00F000F0u) * 0x104u) & 0x81C081C0u, S0);
          const uint32_t a1 = hmul2_bits(((u1 & 0x000F000Fu) * 0x1040u) & 0x81C081C0u, S1);
          const uint32_t a3 = hmul2_bits(((u1 & 0x00F000F0u) * 0x104u) & 0x81C081C0u, S1);
          if constexpr (kNB == 1) {
            mma_bf16_16816(c[q & 1], a0, a1, a2, a3, xb[b][q][0], xb[b][q][1], c[q & 1]);
          } else {
            const uint2 y2 = xs2[(b * 4 + q) * 32 + lane];
            mma_bf16_16816(c[0], a0, a1, a2, a3, xb[b][q][0], xb[b][q][1], c[0]);
            mma_bf16_16816(c[1], a0, a1, a2, a3, y2.x, y2.y, c[1]);
          }
        }
      }
    }
    // lane's C: rows g / g+8 x activation rows 2t, 2t+1
    float* rb = red + (s * kW + warp) * 8 * kNB * 16;
    if constexpr (kNB == 1) {
      rb[(2 * t) * 16 + g] = (c[0][0] + c[1][0]) * post[0][0];
      rb[(2 * t + 1) * 16 + g] = (c[0][1] + c[1][1]) * post[0][1];
      rb[(2 * t) * 16 + g + 8] = (c[0][2] + c[1][2]) * post[0][0];
      rb[(2 * t + 1) * 16 + g + 8] = (c[0][3] + c[1][3]) * post[0][1];
    } else {
#pragma unroll
      for (int nb = 0; nb < kNB; ++nb) {
        rb[(8 * nb + 2 * t) * 16 + g] = c[nb][0] * post[nb][0];
        rb[(8 * nb + 2 * t + 1) * 16 + g] = c[nb][1] * post[nb][1];
        rb[(8 * nb + 2 * t) * 16 + g + 8] = c[nb][2] * post[nb][0];
        rb[(8 * nb + 2 * t + 1) * 16 + g + 8] = c[nb][3] * post[nb][1];
      }
    }
    __syncwarp();  // orders the lanes' slot writes before lane 0's release below
    int last = 0;
    if (lane == 0) last = atom_add_acq_rel_cta(&cnt[s], 1) == kW - 1;
    if (__shfl_sync(0xffffffffu, last, 0)) {  // every warp's partials of this tile are in the slot
      const float* rs = red + s * kW * 8 * kNB * 16;
#pragma unroll
      for (int o = lane; o < 8 * kNB * 16; o += 32) {
        float v[4] = {0.f, 0.f, 0.f, 0.f};  // fixed summation order: 4 strided partial sums, then a tree
#pragma unroll
        for (int w2 = 0; w2 < kW; ++w2) v[w2 & 3] += rs[w2 * 8 * kNB * 16 + o];
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
