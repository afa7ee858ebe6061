// Single-row NVFP4 GEMV (Nvfp4Gemv gguf=1, R = 1) on the integer tensor cores.
//
// Weights: 2 * E2M1 magnitudes are the integers {0, 1, 2, 3, 4, 6, 8, 12}.  A prmt over the 8-byte
// table [0 1 2 3 4 6 8 12] turns four nibbles of a weight word into four u8 magnitudes in one
// instruction; a nibble whose sign bit (bit 3) is set selects prmt's sign-replicate mode, which
// yields 0 for these table bytes (all < 0x80).  So prmt(table, word) is the positive part A+ and
// prmt(table, word ^ 0x8888...) the negative part A- of four weights, and the slice is two u8
// MMAs whose int32 results subtract exactly: sum(A x) = sum(A+ x) - sum(A- x).
//
// Activations: each 16-element sub-block of x (one weight scale's span) is converted once per launch
// to integers x_int = x * 2^(14 - E) (E = exponent of the sub-block's largest |x|, the conversion of
// slice_iq2_i8.cuh), split into a signed high byte and an unsigned low byte; products are exact
// s32, scaled in fp32 by 2^(E - 14) * UE4M3(scale) after the MMA.
//
// MMA layout (m16n8k32, block-diagonal B): a slice = 128 elements = 2 NVFP4 blocks = 8 sub-blocks,
// one per MMA column; k-slots 4t..4t+3 belong to sub-block t (block 0) and 4t+16..4t+19 to sub-block
// t+4 (block 1).  Step j (0..3) takes half-word j of the sub-block's 8 nibble bytes, i.e. elements
// (2j, 2j+8, 2j+1, 2j+9) in k-slot order (low / high nibbles of bytes 2j and 2j+1 of the GGUF
// sub-block, where element e < 8 is the low nibble of byte e and e >= 8 the high nibble of byte
// e - 8); the activation fragments use the same order.  Lane (g, t) decodes rows g and g+8 of
// sub-blocks t and t+4 and supplies the x bytes of sub-block t (if g == t) or t+4 (if g == t+4).
//
// Skeleton as slice_iq2_i8.cuh (stage ring, no producer warp, each warp owns kSPW slices of every
// tile, cross-warp reduction through the last arriver of a per-stage counter, which also refills the
// stage), but rows are copied one bulk copy each into a padded pitch: the NVFP4 row sizes of the
// supported K are multiples of 128 bytes, which would put every other row on the same banks.
#pragma once

#include "slice_iq2_i8.cuh"

namespace gguf_b200 {

__device__ __forceinline__ uint32_t prmt_sign(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}
constexpr uint32_t kFp4MagLo = 0x03020100u, kFp4MagHi = 0x0C080604u;  // 2 * |E2M1| by code 0..7

__device__ __forceinline__ void imma_s8s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                          uint32_t b1) {
  asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void imma_s8u8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                          uint32_t b1) {
  asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.u8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// B fragments of one 128-element slice and the 2^(E - 14) factors of the lane's C columns.
struct F4XFrag {
  uint32_t bh0[4], bl0[4], bh1[4], bl1[4];
  float xs0, xs1;
};

// Lane l converts elements 16c + 4q .. + 3 of the slice (c = l >> 2, q = l & 3; xv = their 4 bf16).
__device__ __forceinline__ void f4_x_frag(const uint2 xv, F4XFrag& f) {
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const bool dlo = (g == t), dhi = (g == t + 4);
  const uint32_t wv[2] = {xv.x, xv.y};
  uint32_t mb = max(max(wv[0] & 0x7FFFu, (wv[0] >> 16) & 0x7FFFu), max(wv[1] & 0x7FFFu, (wv[1] >> 16) & 0x7FFFu));
  mb = max(mb, __shfl_xor_sync(0xffffffffu, mb, 1));
  mb = max(mb, __shfl_xor_sync(0xffffffffu, mb, 2));
  const int emax = max(1, static_cast<int>(mb >> 7));
  uint32_t hw = 0u, lw = 0u;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    int neg, sig, ex;
    bf16_parts(i & 1 ? (wv[i >> 1] >> 16) : (wv[i >> 1] & 0xFFFFu), neg, sig, ex);
    const int xi = bf16_to_fixed(neg, sig, ex, emax);
    hw |= (static_cast<uint32_t>(xi >> 8) & 0xFFu) << (8 * i);
    lw |= (static_cast<uint32_t>(xi) & 0xFFu) << (8 * i);
  }
  // column c's step j needs elements (2j, 2j+8, 2j+1, 2j+9): bytes 2h, 2h+1 (h = j & 1) of the
  // words of lanes 4c + (j >> 1) and 4c + 2 + (j >> 1)
  const int c = dlo ? t : (dhi ? t + 4 : 0);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int qa = 4 * c + (j >> 1), qb = qa + 2;
    const uint32_t ha = __shfl_sync(0xffffffffu, hw, qa), hb = __shfl_sync(0xffffffffu, hw, qb);
    const uint32_t la = __shfl_sync(0xffffffffu, lw, qa), lb = __shfl_sync(0xffffffffu, lw, qb);
    const uint32_t sel = (j & 1) ? 0x7362u : 0x5140u;  // [a.b2h, b.b2h, a.b2h+1, b.b2h+1]
    const uint32_t h = __byte_perm(ha, hb, sel), l = __byte_perm(la, lb, sel);
    f.bh0[j] = dlo ? h : 0u;
    f.bl0[j] = dlo ? l : 0u;
    f.bh1[j] = dhi ? h : 0u;
    f.bl1[j] = dhi ? l : 0u;
  }
  const int e0 = __shfl_sync(0xffffffffu, emax, 4 * (2 * t)), e1 = __shfl_sync(0xffffffffu, emax, 4 * (2 * t + 1));
  f.xs0 = pow2i(e0 - 141);  // 2^(E - 14), E = emax - 127
  f.xs1 = pow2i(e1 - 141);
}

// gguf-py's UE4M3 scale value times 0.5 (the factor of the doubled magnitudes), exact in fp32: byte
// 0x7F decodes to 0, otherwise bit 7 is ignored (so 0xFF is the largest scale, 0x00 / 0x80 are 0).
// Takes the byte in bits 0..7 of b.
__device__ __forceinline__ float f4_scale(uint32_t b) {
  b &= 0xFFu;
  if (b == 0x7Fu) return 0.f;
  const uint32_t e = (b >> 3) & 15u, m = b & 7u;
  return e ? __uint_as_float(((e + 119u) << 23) | (m << 20)) : static_cast<float>(m) * 0x1p-10f;
}

// One slice of the tile for lane (g, t): rows g / g+8 at stage offsets r0 / r1, slice at byte offset
// so of each row.  Returns the lane's partial sums of rows g and g+8 over its C columns.
__device__ __forceinline__ void f4_slice(const uint8_t* st, uint32_t r0, uint32_t r1, uint32_t so, const F4XFrag& f,
                                         float& acc0, float& acc1) {
  const uint32_t t = threadIdx.x & 3;
  // sub-block t of block 0 (bytes 4 + 8t .. of the slice: 4 mod 8, read as the upper / lower words
  // of two aligned 8-byte loads) and of block 1 (bytes 40 + 8t .., 8-byte aligned), rows g and g+8;
  // 8-byte loads over a row pitch of 32 mod 128 bytes put each half-warp on 16 distinct bank pairs
  const uint32_t o0 = so + 8u * t, o1 = so + 40u + 8u * t;
  const uint32_t a00 = reinterpret_cast<const uint2*>(st + r0 + o0)->y;
  const uint32_t a01 = reinterpret_cast<const uint2*>(st + r0 + o0 + 8u)->x;
  const uint32_t b00 = reinterpret_cast<const uint2*>(st + r1 + o0)->y;
  const uint32_t b01 = reinterpret_cast<const uint2*>(st + r1 + o0 + 8u)->x;
  const uint2 a1 = *reinterpret_cast<const uint2*>(st + r0 + o1);
  const uint2 b1 = *reinterpret_cast<const uint2*>(st + r1 + o1);
  const uint32_t so_sc = so + 36u * (t >> 1) + 2u * (t & 1);  // scale bytes of columns 2t, 2t+1
  const uint32_t sg = ld_u16(st, r0 + so_sc), sg8 = ld_u16(st, r1 + so_sc);
  // A operands in MMA order (row g sub t, row g+8 sub t, row g sub t+4, row g+8 sub t+4): steps 0 / 1
  // take the low / high half of the first nibble word, steps 2 / 3 of the second
  const uint32_t wlo[4] = {a00, b00, a1.x, b1.x}, whi[4] = {a01, b01, a1.y, b1.y};
  int ch[4] = {0, 0, 0, 0}, cl[4] = {0, 0, 0, 0};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint32_t a[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint32_t w = j < 2 ? wlo[q] : whi[q];
      const uint32_t sel = (j & 1) ? (w >> 16) : w;
      const uint32_t ap = prmt_sign(kFp4MagLo, kFp4MagHi, sel);           // positive weights, 0 for negative
      const uint32_t an = prmt_sign(kFp4MagLo, kFp4MagHi, sel ^ 0x8888u);  // negative weights, 0 for positive
      // signed bytes: -m per byte as (0x80 - m) ^ 0x80 (m < 0x80: no borrow between bytes), then merge
      a[q] = ap | ((0x80808080u - an) ^ 0x80808080u);
    }
    imma_s8s8(ch, a[0], a[1], a[2], a[3], f.bh0[j], f.bh1[j]);
    imma_s8u8(cl, a[0], a[1], a[2], a[3], f.bl0[j], f.bl1[j]);
  }
  // exact s32 dot products of the lane's (row, sub-block) cells
  const float v0 = static_cast<float>(ch[0] * 256 + cl[0]);
  const float v1 = static_cast<float>(ch[1] * 256 + cl[1]);
  const float v2 = static_cast<float>(ch[2] * 256 + cl[2]);
  const float v3 = static_cast<float>(ch[3] * 256 + cl[3]);
  acc0 = fmaf(v0, f.xs0 * f4_scale(sg), acc0);
  acc0 = fmaf(v1, f.xs1 * f4_scale(sg >> 8), acc0);
  acc1 = fmaf(v2, f.xs0 * f4_scale(sg8), acc1);
  acc1 = fmaf(v3, f.xs1 * f4_scale(sg8 >> 8), acc1);
}

template <int kW, int kSPW>
__global__ void __launch_bounds__(kW * 32, 1) slice_fp4_i8_kernel(const SliceArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + a.off_bar);
  uint8_t* stages = smem + a.off_stage;
  float* red = reinterpret_cast<float*>(smem + a.off_red);       // [stages][kW][16]
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

  // stage s <- tile `tile`: one bulk copy per row (lanes 0..15 of the calling warp) into a padded
  // row pitch (a.stride = 32 mod 128 bytes).  Row bytes are 16-byte multiples.
  auto fill = [&](int s, int tile) {
    const int rv = min(16, a.N - tile * 16);
    uint8_t* dst = stages + s * a.stage_bytes;
    if (lane == 0) mbar_arrive_expect_tx(&full[s], static_cast<uint32_t>(rv * a.row_bytes));
    __syncwarp();
    if (lane < rv)
      bulk_g2s(dst + lane * a.stride, a.w + (static_cast<int64_t>(tile) * 16 + lane) * a.row_bytes,
               static_cast<uint32_t>(a.row_bytes), &full[s]);
  };
  if (warp == 0)
    for (int j = 0; j < a.stages; ++j) {
      const int tile = blockIdx.x + j * gridDim.x;
      if (tile < a.tiles) fill(j, tile);
    }
  const float post = __ldg(a.gscale);
  const int g = lane >> 2, t = lane & 3;
  pdl_wait();  // x is produced by the previous kernel

  // slices w, w + kW, ... of every tile belong to this warp
  F4XFrag xf[kSPW];
#pragma unroll
  for (int i = 0; i < kSPW; ++i) {
    const int sl = warp + i * kW;
    f4_x_frag(ldg64(a.x + sl * 128 + 16 * (lane >> 2) + 4 * (lane & 3)), xf[i]);
  }
  const uint32_t r0 = static_cast<uint32_t>(g * a.stride), r1 = static_cast<uint32_t>((g + 8) * a.stride);
  int s = 0;
  uint32_t ph = 0;
  for (int tile = blockIdx.x; tile < a.tiles; tile += gridDim.x) {
    mbar_wait(&full[s], ph, kSiteFullWait);
    const uint8_t* st = stages + s * a.stage_bytes;
    float acc0 = 0.f, acc1 = 0.f;
#pragma unroll
    for (int i = 0; i < kSPW; ++i) f4_slice(st, r0, r1, static_cast<uint32_t>((warp + i * kW) * 72), xf[i], acc0, acc1);
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
        if (row < a.N) a.y[row] = __float2bfloat16(((v[0] + v[1]) + (v[2] + v[3])) * post);
      }
      __syncwarp();
      if (lane == 0) cnt[s] = 0;
      const int next = tile + a.stages * static_cast<int>(gridDim.x);
      if (next < a.tiles) {
        fence_proxy_async_smem();  // the warps' generic reads of the stage before the copy engine's writes
        fill(s, next);
      }
    }
    if (++s == a.stages) s = 0, ph ^= 1u;
  }
}

}  // namespace gguf_b200
