// IQ2_XXS GEMV specialised for one activation row (R = 1, the decode case of BASELINE config 1).
//
// With one activation row seven of the eight MMA columns of m16n8k16 would be wasted.  This
// kernel uses them to separate the 8 sub-blocks of a 256-element super-block: column c of the B
// operand holds x restricted to sub-block c (a block-diagonal B), so after the 16 MMAs of a
// super-block C[row, c] is the row's dot product with sub-block c alone.  The per-sub-block
// scale db = d*(0.5+s)*0.25 is then applied once per super-block in fp32 (4 FMAs per lane)
// instead of once per 32 elements, and the weights entering the MMA stay the exact signed grid
// magnitudes.
//
// k-slot mapping of MMA i (0..15) of a super-block: slots (2t, 2t+1) <-> sub-block t, elements
// (2i, 2i+1); slots (2t+8, 2t+9) <-> sub-block t+4, elements (2i, 2i+1).  Lane (g, t) therefore
// decodes, for rows g and g+8, the whole sub-blocks t and t+4 (4 records), entry e = i/4 and word
// i%4 feeding MMA i; and the B operand of lane (g, t) is x[sub t] when g == t, x[sub t+4] (as b1)
// when g == t+4, zero otherwise.
//
// Work split: one 16-row weight tile per stage (one bulk copy per row, padded stride); each of the
// kW consumer warps owns a fixed set of super-blocks of every row, so its x fragments are loaded
// into registers once per kernel.  The kW partial dot products of a tile are combined through
// shared memory.
#pragma once

#include "decode.cuh"

namespace gguf_b200 {

struct Iq2R1Args {
  const uint8_t* w;
  const bf16* x;
  bf16* y;
  int N, K, row_bytes, tiles;
  int stride, stage_bytes, stages;
  int off_stage, off_red, off_bar;
};

// Records of one (row, sub-block): 8 raw bytes at `off` (2-byte aligned; `odd` = super-block
// index is odd, so that the record is 4-byte aligned).
__device__ __forceinline__ uint2 iq2_record(const uint8_t* base, uint32_t off, bool aligned4) {
  const uint32_t* w = reinterpret_cast<const uint32_t*>(base + (off & ~3u));
  if (aligned4) return make_uint2(w[0], w[1]);
  const uint32_t w0 = w[0], w1 = w[1], w2 = w[2];
  return make_uint2(__funnelshift_r(w0, w1, 16), __funnelshift_r(w1, w2, 16));
}

template <int kW, int kSPW>  // kW consumer warps, kSPW super-blocks per warp (x fragments in registers)
__global__ void __launch_bounds__((kW + 1) * 32, 1) iq2_r1_kernel(const Iq2R1Args a) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + a.off_bar);
  uint64_t* empty = full + a.stages;
  uint8_t* stages = smem + a.off_stage;
  float* red = reinterpret_cast<float*>(smem + a.off_red);  // [2][kW][16]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < a.stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kW);
    }
    fence_mbar_init();
  }
  {
    uint4* lut = reinterpret_cast<uint4*>(smem);
    const uint4* src = reinterpret_cast<const uint4*>(&g_iq2_mag_bf16[0][0]);
    for (int i = threadIdx.x; i < 256 * 8; i += blockDim.x) lut[i] = src[i >> 3];
  }
  __syncthreads();
  pdl_launch_dependents();

  if (warp == kW) {
    // ---------------- producer: one 16-row tile per stage, one bulk copy per row ----------------
    uint32_t it = 0;
    for (int tile = blockIdx.x; tile < a.tiles; tile += gridDim.x, ++it) {
      const int s = static_cast<int>(it % a.stages);
      const int rv = min(16, a.N - tile * 16);
      if (lane == 0) {
        if (it >= static_cast<uint32_t>(a.stages)) mbar_wait(&empty[s], ((it / a.stages) - 1) & 1, kSiteEmptyWait);
        mbar_arrive_expect_tx(&full[s], static_cast<uint32_t>(rv * a.row_bytes));
      }
      __syncwarp();
      if (lane < rv)
        bulk_g2s(stages + s * a.stage_bytes + lane * a.stride,
                 a.w + (static_cast<int64_t>(tile) * 16 + lane) * a.row_bytes, a.row_bytes, &full[s]);
    }
    if (lane == 0) {
      const uint32_t total = it;
      const uint32_t first = total > static_cast<uint32_t>(a.stages) ? total - a.stages : 0u;
      for (uint32_t j = first; j < total; ++j) mbar_wait(&full[j % a.stages], (j / a.stages) & 1, kSiteDrainWait);
    }
    return;
  }

  // ---------------- consumers ----------------
  const int g = lane >> 2, t = lane & 3;
  const bool dlo = (g == t), dhi = (g == t + 4);
  pdl_wait();  // x is produced by the previous kernel

  // x fragments of this warp's super-blocks: xa (b0, sub t) on lanes g == t, xb (b1, sub t+4) on
  // lanes g == t+4, zero elsewhere.
  uint32_t xa[kSPW][16], xb[kSPW][16];
#pragma unroll
  for (int j = 0; j < kSPW; ++j) {
    const int sb = warp * kSPW + j;
    const bf16* xs = a.x + sb * 256;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint4 va = dlo ? ldg128(xs + 32 * t + 8 * q) : make_uint4(0, 0, 0, 0);
      const uint4 vb = dhi ? ldg128(xs + 32 * (t + 4) + 8 * q) : make_uint4(0, 0, 0, 0);
      xa[j][4 * q + 0] = va.x; xa[j][4 * q + 1] = va.y; xa[j][4 * q + 2] = va.z; xa[j][4 * q + 3] = va.w;
      xb[j][4 * q + 0] = vb.x; xb[j][4 * q + 1] = vb.y; xb[j][4 * q + 2] = vb.z; xb[j][4 * q + 3] = vb.w;
    }
  }
  const uint32_t lut_lane = static_cast<uint32_t>(lane & 7) * 16u;
  // quad lanes holding sub-blocks 2t and 2t+1 (see the scale exchange below)
  const int q0 = (lane & ~3) | ((2 * t) & 3), q1 = (lane & ~3) | ((2 * t + 1) & 3);
  const int nib_sh = t >= 2 ? 4 : 0;

  uint32_t it = 0;
  for (int tile = blockIdx.x; tile < a.tiles; tile += gridDim.x, ++it) {
    const int s = static_cast<int>(it % a.stages);
    mbar_wait(&full[s], (it / a.stages) & 1, kSiteFullWait);
    const uint8_t* st = stages + s * a.stage_bytes;
    const uint32_t r0 = static_cast<uint32_t>(g * a.stride), r1 = static_cast<uint32_t>((g + 8) * a.stride);
    float acc0 = 0.f, acc1 = 0.f;  // rows g, g+8
#pragma unroll
    for (int j = 0; j < kSPW; ++j) {
      const int sb = warp * kSPW + j;
      const uint32_t so = static_cast<uint32_t>(sb) * 66u;
      const bool al = (sb & 1) != 0;  // odd super-block: records 4-byte aligned (warp-uniform)
      // records: [row g, sub t], [row g, sub t+4], [row g+8, sub t], [row g+8, sub t+4]
      uint2 rc[4];
      rc[0] = iq2_record(st, r0 + so + 2u + 8u * t, al);
      rc[1] = iq2_record(st, r0 + so + 34u + 8u * t, al);
      rc[2] = iq2_record(st, r1 + so + 2u + 8u * t, al);
      rc[3] = iq2_record(st, r1 + so + 34u + 8u * t, al);
      const uint32_t dbits = ld_u16(st, r0 + so) | (ld_u16(st, r1 + so) << 16);
      float c[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        uint4 m[4];
#pragma unroll
        for (int r = 0; r < 4; ++r) {  // the four codebook rows first (independent loads)
          const uint32_t gi = (rc[r].x >> (8 * e)) & 0xFFu;
          m[r] = *reinterpret_cast<const uint4*>(smem + lut_lane + (gi << 7));
        }
        uint32_t A[4][4];
#pragma unroll
        for (int r = 0; r < 4; ++r) iq2_apply_signs(m[r], rc[r].y, 7u * e, A[r]);
#pragma unroll
        for (int wd = 0; wd < 4; ++wd) {
          const int i = 4 * e + wd;
          float (&cc)[4] = c[i & 1];
          mma_bf16_16816(cc, A[0][wd], A[2][wd], A[1][wd], A[3][wd], xa[j][i], xb[j][i], cc);
        }
      }
      if (j == kSPW - 1) {
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);  // stage no longer read by this warp
      }
      // scales: lane packs the s nibbles of its 4 records, gathers those of sub-blocks 2t, 2t+1
      const uint32_t mine = (rc[0].y >> 28) | ((rc[1].y >> 28) << 4) | ((rc[2].y >> 28) << 8) | ((rc[3].y >> 28) << 12);
      const uint32_t p0 = __shfl_sync(0xffffffffu, mine, q0) >> nib_sh, p1 = __shfl_sync(0xffffffffu, mine, q1) >> nib_sh;
      // (0.5 + s) exactly: float(2^23 + s) - (2^23 - 0.5)
      const float h00 = __uint_as_float((p0 & 15u) | 0x4B000000u) - 8388607.5f;
      const float h01 = __uint_as_float((p1 & 15u) | 0x4B000000u) - 8388607.5f;
      const float h10 = __uint_as_float(((p0 >> 8) & 15u) | 0x4B000000u) - 8388607.5f;
      const float h11 = __uint_as_float(((p1 >> 8) & 15u) | 0x4B000000u) - 8388607.5f;
      const float d0s = fp16_bits_to_f32(dbits & 0xFFFFu) * 0.25f, d1s = fp16_bits_to_f32(dbits >> 16) * 0.25f;
      // C[row g, col 2t] = sub 2t, [g, 2t+1] = sub 2t+1, [g+8, 2t], [g+8, 2t+1]
      acc0 = fmaf(d0s * h00, c[0][0] + c[1][0], acc0);
      acc0 = fmaf(d0s * h01, c[0][1] + c[1][1], acc0);
      acc1 = fmaf(d1s * h10, c[0][2] + c[1][2], acc1);
      acc1 = fmaf(d1s * h11, c[0][3] + c[1][3], acc1);
    }
    // quad reduction (the 4 lanes of a quad hold the 8 sub-block columns), then across warps
    acc0 += __shfl_xor_sync(0xffffffffu, acc0, 1);
    acc0 += __shfl_xor_sync(0xffffffffu, acc0, 2);
    acc1 += __shfl_xor_sync(0xffffffffu, acc1, 1);
    acc1 += __shfl_xor_sync(0xffffffffu, acc1, 2);
    // double-buffered partials: buffer (it & 1) is read by warp 0 after the barrier of this tile and
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
      if (row < a.N) a.y[row] = __float2bfloat16(v);
    }
  }
}

}  // namespace gguf_b200
