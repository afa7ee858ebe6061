// Few-row Q8_0 GEMV (1 <= R <= 4 * kNR) on the integer tensor cores (kSplit: the legacy split layout
// of Q8Gemv gguf=0, u8 q + 128 with bf16 scales per 32 in a second tensor).  A Q8_0 block is an fp16 scale
// d and 32 int8 quants, so the quants are the MMA's A operand as they are (s8, no decode step):
// the launch is bound by HBM and by the per-block epilogue, not by a codebook.
//
// MMA layout (mma.sync m16n8k32, s8 x s8 -> s32), as in the few-row IQ2_XXS kernel
// (slice_iq2_i8_rows.cuh): one MMA covers one 32-element block of a 16-row tile; lane (g, t) supplies
// quants 8t..8t+7 of rows g and g+8 (k-slots 4t..4t+3 and 4t+16..4t+19), the 8 columns are four
// activation rows x two signed limbs of x_int = x * 2^(13 - E) (i8_rows_x: E per 32-element group),
// and C column pair (2t, 2t+1) of lane (g, t) is activation row t.  Epilogue per (row, block):
// y += (256 C_hi + C_lo) * 2^(E - 13) * d, in fp32.  No offset term: the quants are signed.
//
// Row-split shards (a.po.npeer > 0): every y value goes to every GPU of the group as a tagged word
// (peer_store_tile16), and the launch ends once every GPU's shard is present (peer_gather).
//
// Staging: a tile is 16 whole rows (K / 32 * 34 bytes each), one bulk copy per row into a stage
// whose row pitch is the row bytes + 16, which keeps the eight quads' loads off a common bank (a
// pitch of 0 mod 32 words would put all eight rows on the same banks).  Rows are 17K/16 bytes, so a
// 16-row tile is large (K = 4096: 68 KB); two stages already hold ~140 KB of a GPU-wide ~20 MB in
// flight, and the per-tile compute is well below the tile's HBM time.
#pragma once

#include "slice_iq2_i8_rows.cuh"

namespace gguf_b200 {

__device__ __forceinline__ void imma_s8s8_c(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                            uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};\n"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}

// One 16-row x 256-column slice (8 blocks of 32 per row) against the kNR MMA sets; st = the stage,
// r0 / r1 = byte offsets of rows g / g+8, sl = the slice index.  Q8_0 (kSplit false): block j at
// 272 * sl + 34 j, fp16 d then the quants.  Split layout (Q8Gemv gguf=0, kSplit true): the quants as
// u8 q + 128 at 256 * sl + 32 j (8-byte aligned; q = u ^ 0x80 per byte), the bf16 scales of rows g /
// g+8 at sc0 / sc1 (stage offsets of their scale rows) + 2 (8 sl + j), read as one 16-byte load per
// row and slice (the scale rows are 256 bytes apart, so the eight quads' reads share banks).
//
// kLay: 0 = Q8_0, 1 = Q8Gemv gguf=0 (split), 2 = Q4Gemv iq2=0 (split: u8 [N, K/2] nibbles n, element
// 2i the low nibble of byte i, value n - 8, bf16 scales per 32).  Q4: lane t's 8 elements of block j
// are bytes 4t..4t+3 at 128 sl + 16 j; the nibbles become the u8 A operand n as they are (two LOP3,
// two byte-permutes per 8 elements) and the offset 8 sum(x_int) enters as the low-limb column's C.
constexpr int kLayQ8 = 0, kLayQ8S = 1, kLayQ4S = 2;

template <int kNR, int kLay = kLayQ8>
__device__ __forceinline__ void q8_rows_slice(const uint8_t* st, uint32_t r0, uint32_t r1, uint32_t sl, uint32_t sc0,
                                              uint32_t sc1, const I8RowsX<kNR, kLay == kLayQ4S>& f,
                                              float (&acc)[kNR][2]) {
  constexpr bool kSplit = kLay != kLayQ8;
  const uint32_t t = threadIdx.x & 3;
  uint32_t sv0[4] = {0u, 0u, 0u, 0u}, sv1[4] = {0u, 0u, 0u, 0u};
  if constexpr (kSplit) {  // the slice's 8 bf16 scales of rows g / g+8: one 16-byte load each
    const uint4 u0 = *reinterpret_cast<const uint4*>(st + sc0 + 16u * sl);
    const uint4 u1 = *reinterpret_cast<const uint4*>(st + sc1 + 16u * sl);
    sv0[0] = u0.x; sv0[1] = u0.y; sv0[2] = u0.z; sv0[3] = u0.w;
    sv1[0] = u1.x; sv1[1] = u1.y; sv1[2] = u1.z; sv1[3] = u1.w;
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    uint2 q0, q1;
    float d0, d1;
    if constexpr (kLay == kLayQ4S) {
      const uint32_t ob = 128u * sl + 16u * j + 4u * t;
      const uint32_t v0 = *reinterpret_cast<const uint32_t*>(st + r0 + ob), v1 = *reinterpret_cast<const uint32_t*>(st + r1 + ob);
      const uint32_t l0 = v0 & 0x0F0F0F0Fu, h0 = (v0 >> 4) & 0x0F0F0F0Fu, l1 = v1 & 0x0F0F0F0Fu, h1 = (v1 >> 4) & 0x0F0F0F0Fu;
      q0 = make_uint2(__byte_perm(l0, h0, 0x5140u), __byte_perm(l0, h0, 0x7362u));  // elements 8t..8t+3, 8t+4..8t+7
      q1 = make_uint2(__byte_perm(l1, h1, 0x5140u), __byte_perm(l1, h1, 0x7362u));
      d0 = __uint_as_float(j & 1 ? (sv0[j >> 1] & 0xFFFF0000u) : (sv0[j >> 1] << 16));
      d1 = __uint_as_float(j & 1 ? (sv1[j >> 1] & 0xFFFF0000u) : (sv1[j >> 1] << 16));
    } else if constexpr (kSplit) {
      const uint32_t ob = 256u * sl + 32u * j + 8u * t;
      q0 = *reinterpret_cast<const uint2*>(st + r0 + ob);
      q1 = *reinterpret_cast<const uint2*>(st + r1 + ob);
      q0 = make_uint2(q0.x ^ 0x80808080u, q0.y ^ 0x80808080u);
      q1 = make_uint2(q1.x ^ 0x80808080u, q1.y ^ 0x80808080u);
      d0 = __uint_as_float(j & 1 ? (sv0[j >> 1] & 0xFFFF0000u) : (sv0[j >> 1] << 16));
      d1 = __uint_as_float(j & 1 ? (sv1[j >> 1] & 0xFFFF0000u) : (sv1[j >> 1] << 16));
    } else {
      const uint32_t ob = 272u * sl + 34u * j;  // block j: d at ob, quants at ob + 2 (4-byte aligned iff j is odd)
      q0 = lds8(st, r0 + ob + 2u + 8u * t, (j & 1) != 0);
      q1 = lds8(st, r1 + ob + 2u + 8u * t, (j & 1) != 0);
      d0 = fp16_bits_to_f32(ld_u16(st, r0 + ob));
      d1 = fp16_bits_to_f32(ld_u16(st, r1 + ob));
    }
#pragma unroll
    for (int m = 0; m < kNR; ++m) {
      int cc[4];
      if constexpr (kLay == kLayQ4S)
        imma_u8s8_c(cc, q0.x, q1.x, q0.y, q1.y, f.b[m][j][0], f.b[m][j][1], 0, f.nxoff[m][j] >> 3);  // -8 sum(x_int)
      else
        imma_s8s8_c(cc, q0.x, q1.x, q0.y, q1.y, f.b[m][j][0], f.b[m][j][1]);
      const float p = f.xs[m][j];
      acc[m][0] = fmaf(static_cast<float>(cc[0] * 256 + cc[1]), p * d0, acc[m][0]);
      acc[m][1] = fmaf(static_cast<float>(cc[2] * 256 + cc[3]), p * d1, acc[m][1]);
    }
  }
}

// Warp w owns slices w * kSPW .. w * kSPW + kSPW - 1 of K for the whole launch; the last warp to
// finish a tile sums the stage's reduction slot in warp order (deterministic), stores y [R, N] and
// refills the stage (the last-arriver scheme of slice_iq2_i8_kernel).  kSPW = 2 halves the warps
// and with them the reduction slots, which leaves room for a third stage at eight activation rows.
template <int kW, int kNR, int kSPW = 1, int kLay = kLayQ8>
__global__ void __launch_bounds__(kW * 32, 1) slice_q8_i8_rows_kernel(const __grid_constant__ SliceArgs a) {
  constexpr bool kSplit = kLay != kLayQ8;
  constexpr int kRX = 4 * kNR;
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + a.off_bar);
  uint8_t* stages = smem + a.off_stage;
  float* red = reinterpret_cast<float*>(smem + a.off_red);  // [stages][kW][kRX][16]
  int* cnt = reinterpret_cast<int*>(red + a.stages * kW * kRX * 16);  // [stages]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __shared__ uint32_t s_call;  // row-split: this launch's call number (its tag)

  if (threadIdx.x == 0) {
    for (int s = 0; s < a.stages; ++s) {
      mbar_init(&full[s], 1);
      cnt[s] = 0;
    }
    fence_mbar_init();
    if (a.po.npeer) s_call = peer_call(a.po);  // before launch_dependents: see peer_call
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
  // Only the first stage (two for long launches) is requested before the dependency wait: a load of x
  // issued behind a full ring of bulk copies into this SM returns only after most of them (measured:
  // ~3 µs of x conversion at C0 with every stage in flight), so the other stages follow once every
  // warp has issued its x loads (C0 4096 x 4096: 6.36 -> 6.20 µs; 16384 rows: 15.24 -> 14.42 µs;
  // C4 131072 rows with two stages first: 94.0 -> 92.9 µs).
  const int pre = a.tiles > 16 * static_cast<int>(gridDim.x) ? 2 : 1;
  if (warp == 0)
    for (int j = 0; j < pre; ++j) {
      const int tile = blockIdx.x + j * gridDim.x;
      if (tile < a.tiles) fill(j, tile);
    }
  pdl_wait();  // x is produced by the previous kernel

  uint2 xv[kSPW][kNR][8];
#pragma unroll
  for (int j = 0; j < kSPW; ++j) i8_rows_x_load<kNR>(a.x, a.R, a.K, warp * kSPW + j, xv[j]);
  if (pre < a.stages) {
    __syncthreads();  // every warp's x loads are issued before the remaining stages' copies
    if (warp == 0)
      for (int j = pre; j < a.stages; ++j) {
        const int tile = blockIdx.x + j * gridDim.x;
        if (tile < a.tiles) fill(j, tile);
      }
  }
  I8RowsX<kNR, kLay == kLayQ4S> xf[kSPW];  // signed quants need no offset sums, Q4 nibbles (u8) do
#pragma unroll
  for (int j = 0; j < kSPW; ++j) i8_rows_x_cvt<kNR, kLay == kLayQ4S>(xv[j], xf[j]);
  const int g = lane >> 2, t = lane & 3;
  const uint32_t sl0 = static_cast<uint32_t>(warp * kSPW);
  const uint32_t r0 = static_cast<uint32_t>(g * a.stride), r1 = static_cast<uint32_t>((g + 8) * a.stride);
  const uint32_t sc0 = static_cast<uint32_t>(a.sc_off + g * a.sc_row_bytes), sc1 = static_cast<uint32_t>(a.sc_off + (g + 8) * a.sc_row_bytes);
  int s = 0;
  uint32_t ph = 0;
  for (int tile = blockIdx.x; tile < a.tiles; tile += gridDim.x) {
    mbar_wait(&full[s], ph, kSiteFullWait);
    float acc[kNR][2];
#pragma unroll
    for (int m = 0; m < kNR; ++m) acc[m][0] = acc[m][1] = 0.f;
#pragma unroll
    for (int j = 0; j < kSPW; ++j)
      q8_rows_slice<kNR, kLay>(stages + s * a.stage_bytes, r0, r1, sl0 + j, sc0, sc1, xf[j], acc);

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
      const bool vec = a.po.npeer && a.po.vec && tile * 16 + 16 <= a.N;  // full tile, aligned peer rows
#pragma unroll
      for (int o = lane; o < kRX * 16; o += 32) {
        float v[4] = {0.f, 0.f, 0.f, 0.f};  // fixed summation order: 4 strided partial sums, then a tree
#pragma unroll
        for (int w2 = 0; w2 < kW; ++w2) v[w2 & 3] += rs[w2 * kRX * 16 + o];
        const int xr = o >> 4, row = tile * 16 + (o & 15);
        const bf16 yv = __float2bfloat16((v[0] + v[1]) + (v[2] + v[3]));
        if (vec) {  // row-split shard: 16-byte stores into every GPU's y (warp-uniform branch)
          if (o - lane < 16 * a.R)  // the pass's first half holds an activation row < R
            peer_store_tile16(a.po, s_call, yv, xr < a.R, xr, tile * 16);
        } else if (xr < a.R && row < a.N) {
          if (a.po.npeer) peer_store(a.po, s_call, xr, row, yv);  // row-split shard: into every GPU's staging
          else a.y[static_cast<int64_t>(xr) * a.N + row] = yv;
        }
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
  if (a.po.npeer) peer_gather(a.po, s_call, a.R, threadIdx.x, blockDim.x);  // the whole y, from the staging buffer
}

}  // namespace gguf_b200
