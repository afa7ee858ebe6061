// Persistent skinny-GEMM engine for raw GGUF weights on sm_100a.
//
//   y[col, row] = sum_k x[col, k] * W[row, k]      (col < R <= 16, row < rows)
//
// Work unit = a 16-row weight tile (MMA M side).  One CTA per SM (<= half of the SM's shared
// memory, so that the next kernel on the stream can co-reside and prefetch under programmatic
// dependent launch) loops over tiles blockIdx.x, blockIdx.x + gridDim.x, ...
//
//   warp KW (producer) : one lane streams each tile's raw bytes into a ring of `stages` shared-
//                        memory stages with 1-D bulk async copies (TMA engine), completion
//                        tracked by a "full" mbarrier per stage; it refills a stage once the KW
//                        consumer warps have arrived on its "empty" mbarrier.  A stage holds
//                        16 rows x kc elements (one bulk copy per row into a padded row stride,
//                        or one contiguous copy of the whole tile when rows are not 16-byte
//                        multiples).  Weight prefetch does not depend on the previous kernel.
//   warps 0..KW-1      : after griddepcontrol.wait, split the stage's k-groups, decode each group
//                        in registers (decode.cuh) and issue two mma.m16n8k16 per group per 8
//                        activation rows; then reduce the KW partial tiles through shared memory
//                        and store.
//
// MODE kDense: y = bf16(acc * post) for the dense GEMVs.
// MODE kMoe1 / kMoe2: expert-grouped MoE phases over IQ2_XXS expert tensors (MoeVerify); the
// unique-expert grouping of idx is recomputed by every CTA in shared memory.
#pragma once

#include "decode.cuh"

namespace gguf_b200 {

constexpr int kModeDense = 0, kModeMoe1 = 1, kModeMoe2 = 2;
constexpr int kMaxPairs = 128;

struct EngineArgs {
  // Segmented staging through a 2-D tensor map over the weight bytes viewed as u64 elements
  // [all rows, row_bytes / 8]: one copy request moves a 16-row x `stride`-byte box (the segment
  // plus up to 16 bytes of the next one, which give the padded row pitch), instead of 16 row copies
  // -- the copy engine's throughput per SM is bounded by requests in flight, not bytes.
  CUtensorMap tmap;
  int use_tmap;
  // weights
  const uint8_t* w;  // 16-byte aligned
  int K;             // reduction length
  int row_bytes;     // raw bytes per weight row
  int rows;          // rows per weight matrix (dense: N; MoE: rows of one expert)
  int tiles;         // ceil(rows / 16) per matrix
  // staging plan
  int kc;            // K elements per stage
  int nsplit;        // K / kc
  int seg_bytes;     // raw bytes of kc elements of one row
  int stride;        // shared-memory bytes per staged row
  int contiguous;    // 1: one bulk copy of the whole tile (nsplit == 1, stride == row_bytes)
  int stage_bytes;
  int stages;
  int off_stage, off_red, off_bar, off_grp;  // shared-memory layout
  // activations / outputs
  const bf16* x;     // dense: [R, K]; moe1: z [R, K]; moe2: h [P, K]
  int R;
  void* y;           // dense: bf16 [R, rows]; moe1: h bf16 [P, rows]; moe2: part f32 [P, rows]
  const float* gscale;  // dense NVFP4 only (device scalar), else nullptr
  float post;        // constant epilogue factor (2^16 for NVFP4, 1 otherwise)
  // MoE
  const int32_t* idx;  // [R, topk]
  int topk, P, E;
  int32_t* meta;       // moe1: written by CTA 0
  PeerOut po;          // dense, npeer > 0: row-split shard stored into every GPU of the group
  // split layouts (decode.cuh kFmt*S): the scale tensor, staged after the weights of each stage as
  // a [16 rows][sc_seg_bytes] slab at offset sc_off (same copy mode as the weights)
  CUtensorMap smap;    // 2-D map over the scale bytes [all rows, sc_row_bytes] (u8), box 16 x sc_seg_bytes
  const uint8_t* sc;
  int sc_row_bytes, sc_seg_bytes, sc_off;
};

__device__ __forceinline__ void named_bar_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}
__device__ __forceinline__ void named_bar_arrive(int id, int threads) {
  asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// Unique-expert grouping of idx (first-occurrence order, as src/bolt_ops.cu:1233-1261):
// s_uexp[u] = expert id of group u, s_pair[u*8 + row] = pair index (row*topk + k) or -1.
// Expert ids are taken relative to `offset` (the first expert this GPU holds under expert
// parallelism; 0 otherwise); pairs whose relative id is outside [0, E) are ignored.  Returns U (in
// shared memory).  s_idx must be 16-byte aligned.
__device__ __forceinline__ void moe_group(const int32_t* idx, int P, int E, int topk, int* s_idx, int offset = 0) {
  int* s_first = s_idx + kMaxPairs;
  int* s_rank = s_first + kMaxPairs;
  int* s_uexp = s_rank + kMaxPairs;
  int* s_pair = s_uexp + kMaxPairs;  // [kMaxPairs][8]
  int* s_U = s_pair + kMaxPairs * 8;
  const int tid = threadIdx.x, nth = blockDim.x;
  for (int i = tid; i < kMaxPairs * 8; i += nth) s_pair[i] = -1;
  if (tid < P) s_idx[tid] = idx[tid] - offset;
  __syncthreads();
  if (tid < P) {  // first pair with the same expert: 4 ids per 16-byte load (s_idx is 16-byte aligned)
    const int my = s_idx[tid];
    int q = -1;
    if (my >= 0 && my < E) {
      const int4* v4 = reinterpret_cast<const int4*>(s_idx);
      for (int j = 0; j <= tid; j += 4) {
        const int4 v = v4[j >> 2];  // in order: the scan stops at tid's own entry at the latest
        if (v.x == my) { q = j; break; }
        if (v.y == my) { q = j + 1; break; }
        if (v.z == my) { q = j + 2; break; }
        if (v.w == my) { q = j + 3; break; }
      }
    }
    s_first[tid] = q;
  }
  __syncthreads();
  if (tid < 32) {  // ranks of the first occurrences (their order = group order): ballots over the pairs
    int base = 0;
    for (int c = 0; c < P; c += 32) {
      const int i = c + tid;
      const bool head = i < P && s_first[i] == i;
      const unsigned m = __ballot_sync(0xffffffffu, head);
      if (head) {
        const int r = base + __popc(m & ((1u << tid) - 1u));
        s_rank[i] = r;
        s_uexp[r] = s_idx[i];
      }
      base += __popc(m);
    }
    if (tid == 0) *s_U = base;
  }
  __syncthreads();
  if (tid < P && s_first[tid] >= 0) s_pair[s_rank[s_first[tid]] * 8 + tid / topk] = tid;
  __syncthreads();
}

// One IQ2_XXS k-group (32-element sub-block) of a staged 16-row tile for lane (g, t) against one
// 8-column B fragment already in registers (xv = the lane's 8 activations k0 + 8t .. k0 + 8t + 7 of
// column g): rows g and g+8, grid entry t of each record.
__device__ __forceinline__ void iq2_group_mma_x(const uint8_t* smem, const uint8_t* st, uint32_t r0, uint32_t r1, int grp,
                                                int t, uint32_t lut_lane, const uint4 xv, float (&acc)[4]) {
  const uint32_t sbo = static_cast<uint32_t>(grp >> 3) * 66u;
  const uint32_t rec = sbo + 2u + static_cast<uint32_t>(grp & 7) * 8u;
  const uint2 q0 = ld_u64_a2(st, r0 + rec);
  const uint2 q1 = ld_u64_a2(st, r1 + rec);
  const float d0 = fp16_bits_to_f32(ld_u16(st, r0 + sbo));
  const float d1 = fp16_bits_to_f32(ld_u16(st, r1 + sbo));
  const uint32_t gi0 = (q0.x >> (8 * t)) & 0xFFu, gi1 = (q1.x >> (8 * t)) & 0xFFu;
  const uint4 m0 = *reinterpret_cast<const uint4*>(smem + lut_lane + (gi0 << 7));
  const uint4 m1 = *reinterpret_cast<const uint4*>(smem + lut_lane + (gi1 << 7));
  uint32_t A0[4], A1[4];
  iq2_apply_signs(m0, q0.y, 7u * t, A0);
  iq2_apply_signs(m1, q1.y, 7u * t, A1);
  const float db0 = iq2_db(d0, q0.y), db1 = iq2_db(d1, q1.y);
  const float z[4] = {0.f, 0.f, 0.f, 0.f};
  float D[4];
  mma_bf16_16816(D, A0[0], A1[0], A0[1], A1[1], xv.x, xv.y, z);
  mma_bf16_16816(D, A0[2], A1[2], A0[3], A1[3], xv.z, xv.w, D);
  acc[0] = fmaf(db0, D[0], acc[0]);
  acc[1] = fmaf(db0, D[1], acc[1]);
  acc[2] = fmaf(db1, D[2], acc[2]);
  acc[3] = fmaf(db1, D[3], acc[3]);
}

// One IQ2_XXS k-group (32-element sub-block) of a staged 16-row tile for lane (g, t): rows g and
// g+8 (byte offsets r0, r1 in the stage), grid entry t of each record, B fragments read from
// xr[nt] + k0 + 8t.  kCoherent: the activation rows were written earlier in the same kernel, so
// they are read through L2 (ld.global.cg) instead of the read-only path.
template <int NT, bool kCoherent>
__device__ __forceinline__ void iq2_group_mma(const uint8_t* smem, const uint8_t* st, uint32_t r0, uint32_t r1, int grp,
                                              int t, uint32_t lut_lane, const bf16* const (&xr)[NT], int k0,
                                              float (&acc)[NT][4]) {
  const uint32_t sbo = static_cast<uint32_t>(grp >> 3) * 66u;
  const uint32_t rec = sbo + 2u + static_cast<uint32_t>(grp & 7) * 8u;
  const uint2 q0 = ld_u64_a2(st, r0 + rec);
  const uint2 q1 = ld_u64_a2(st, r1 + rec);
  const float d0 = fp16_bits_to_f32(ld_u16(st, r0 + sbo));
  const float d1 = fp16_bits_to_f32(ld_u16(st, r1 + sbo));
  const uint32_t gi0 = (q0.x >> (8 * t)) & 0xFFu, gi1 = (q1.x >> (8 * t)) & 0xFFu;
  const uint4 m0 = *reinterpret_cast<const uint4*>(smem + lut_lane + (gi0 << 7));
  const uint4 m1 = *reinterpret_cast<const uint4*>(smem + lut_lane + (gi1 << 7));
  uint32_t A0[4], A1[4];
  iq2_apply_signs(m0, q0.y, 7u * t, A0);
  iq2_apply_signs(m1, q1.y, 7u * t, A1);
  const float db0 = iq2_db(d0, q0.y), db1 = iq2_db(d1, q1.y);
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    const uint4 xv = kCoherent ? __ldcg(reinterpret_cast<const uint4*>(xr[nt] + k0 + 8 * t)) : ldg128(xr[nt] + k0 + 8 * t);
    const float z[4] = {0.f, 0.f, 0.f, 0.f};
    float D[4];
    mma_bf16_16816(D, A0[0], A1[0], A0[1], A1[1], xv.x, xv.y, z);
    mma_bf16_16816(D, A0[2], A1[2], A0[3], A1[3], xv.z, xv.w, D);
    acc[nt][0] = fmaf(db0, D[0], acc[nt][0]);
    acc[nt][1] = fmaf(db0, D[1], acc[nt][1]);
    acc[nt][2] = fmaf(db1, D[2], acc[nt][2]);
    acc[nt][3] = fmaf(db1, D[3], acc[nt][3]);
  }
}

// One k-group of a split-layout stage for lane (g, t): rows g / g+8 at byte offsets r0 / r1 of the
// weight stage and s0 / s1 of the scale slab `sl`.  Weights enter the MMA exactly (decode.cuh);
// the per-group scale is applied to the fp32 MMA result (FP4S: folded into the exact bf16 weight).
template <int F, int NT, bool kCoherent>
__device__ __forceinline__ void split_group_mma(const uint8_t* smem, const uint8_t* st, const uint8_t* sl, uint32_t r0,
                                                uint32_t r1, uint32_t s0, uint32_t s1, int grp, int t,
                                                uint32_t lut_lane, const bf16* const (&xr)[NT], int k0,
                                                float (&acc)[NT][4]) {
  auto ldx128 = [&](const bf16* p) { return kCoherent ? __ldcg(reinterpret_cast<const uint4*>(p)) : ldg128(p); };
  auto ldx64 = [&](const bf16* p) { return kCoherent ? __ldcg(reinterpret_cast<const uint2*>(p)) : ldg64(p); };
  uint32_t A0[4], A1[4];
  float d0, d1;
  if constexpr (F == kFmtQ8S) {
    const uint32_t o = static_cast<uint32_t>(grp) * 32u + 4u * t;
    q8_to_bf16x4(*reinterpret_cast<const uint32_t*>(st + r0 + o) ^ 0x80808080u, A0[0], A0[1]);
    q8_to_bf16x4(*reinterpret_cast<const uint32_t*>(st + r0 + o + 16u) ^ 0x80808080u, A0[2], A0[3]);
    q8_to_bf16x4(*reinterpret_cast<const uint32_t*>(st + r1 + o) ^ 0x80808080u, A1[0], A1[1]);
    q8_to_bf16x4(*reinterpret_cast<const uint32_t*>(st + r1 + o + 16u) ^ 0x80808080u, A1[2], A1[3]);
  } else if constexpr (F == kFmtQ4S || F == kFmtIQ2C || F == kFmtFP4S) {
    const uint32_t o = static_cast<uint32_t>(grp) * 16u + 4u * t;
    const uint32_t v0 = *reinterpret_cast<const uint32_t*>(st + r0 + o);
    const uint32_t v1 = *reinterpret_cast<const uint32_t*>(st + r1 + o);
    if constexpr (F == kFmtQ4S) {
      q4s_words(v0, A0);
      q4s_words(v1, A1);
    } else if constexpr (F == kFmtIQ2C) {
      iq2c_words(v0, A0);
      iq2c_words(v1, A1);
    } else {
      fp4s_words(v0, A0);
      fp4s_words(v1, A1);
      const uint16_t* lut = reinterpret_cast<const uint16_t*>(smem);
      const uint32_t so = static_cast<uint32_t>(grp) * 2u + static_cast<uint32_t>(t >> 1);
      const uint32_t S0 = lut[sl[s0 + so]], S1 = lut[sl[s1 + so]];
      const uint32_t S0x2 = S0 | (S0 << 16), S1x2 = S1 | (S1 << 16);
#pragma unroll
      for (int p = 0; p < 4; ++p) {
        A0[p] = hmul2_bits(A0[p], S0x2);
        A1[p] = hmul2_bits(A1[p], S1x2);
      }
    }
  } else {  // kFmtIQ2N: 8-byte record = 4 grid indices + sign/scale word; d per 256 elements
    const uint32_t o = static_cast<uint32_t>(grp) * 8u;
    const uint2 q0 = *reinterpret_cast<const uint2*>(st + r0 + o);
    const uint2 q1 = *reinterpret_cast<const uint2*>(st + r1 + o);
    const uint32_t so = static_cast<uint32_t>(grp >> 3) * 2u;
    const uint32_t gi0 = (q0.x >> (8 * t)) & 0xFFu, gi1 = (q1.x >> (8 * t)) & 0xFFu;
    const uint4 m0 = *reinterpret_cast<const uint4*>(smem + lut_lane + (gi0 << 7));
    const uint4 m1 = *reinterpret_cast<const uint4*>(smem + lut_lane + (gi1 << 7));
    iq2_apply_signs(m0, q0.y, 7u * t, A0);
    iq2_apply_signs(m1, q1.y, 7u * t, A1);
    d0 = iq2_db(fp16_bits_to_f32(ld_u16(sl, s0 + so)), q0.y);
    d1 = iq2_db(fp16_bits_to_f32(ld_u16(sl, s1 + so)), q1.y);
  }
  if constexpr (F == kFmtQ8S || F == kFmtQ4S || F == kFmtIQ2C) {
    d0 = __uint_as_float(ld_u16(sl, s0 + static_cast<uint32_t>(grp) * 2u) << 16);  // bf16 scale
    d1 = __uint_as_float(ld_u16(sl, s1 + static_cast<uint32_t>(grp) * 2u) << 16);
  }
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    uint32_t b0, b1, b2, b3;
    if constexpr (F == kFmtQ8S) {
      const uint2 xl = ldx64(xr[nt] + k0 + 4 * t), xh = ldx64(xr[nt] + k0 + 16 + 4 * t);
      b0 = xl.x, b1 = xl.y, b2 = xh.x, b3 = xh.y;
    } else {
      const uint4 xv = ldx128(xr[nt] + k0 + 8 * t);
      b0 = xv.x, b1 = xv.y, b2 = xv.z, b3 = xv.w;
    }
    if constexpr (F == kFmtFP4S) {
      mma_bf16_16816(acc[nt], A0[0], A1[0], A0[1], A1[1], b0, b1, acc[nt]);
      mma_bf16_16816(acc[nt], A0[2], A1[2], A0[3], A1[3], b2, b3, acc[nt]);
    } else {
      const float z[4] = {0.f, 0.f, 0.f, 0.f};
      float D[4];
      mma_bf16_16816(D, A0[0], A1[0], A0[1], A1[1], b0, b1, z);
      mma_bf16_16816(D, A0[2], A1[2], A0[3], A1[3], b2, b3, D);
      acc[nt][0] = fmaf(d0, D[0], acc[nt][0]);
      acc[nt][1] = fmaf(d0, D[1], acc[nt][1]);
      acc[nt][2] = fmaf(d1, D[2], acc[nt][2]);
      acc[nt][3] = fmaf(d1, D[3], acc[nt][3]);
    }
  }
}

// Two CTAs fit on an SM (registers <= 60, shared memory <= half): the dense GEMV runs two per SM, and
// consecutive kernels on a stream can overlap under programmatic dependent launch.
template <int F, int NT, int KW, int MODE>
__global__ void __launch_bounds__((KW + 1) * 32, 2) engine_kernel(const __grid_constant__ EngineArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + a.off_bar);
  uint64_t* empty = full + a.stages;
  uint8_t* stages = smem + a.off_stage;
  float* red = reinterpret_cast<float*>(smem + a.off_red);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  // ---- prologue (independent of the previous kernel) ----
  if (threadIdx.x == 0) {
    for (int s = 0; s < a.stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], KW);
    }
    fence_mbar_init();
  }
  if constexpr (F == kFmtIQ2 || F == kFmtIQ2N) {
    fill_iq2_lut_bf16<(KW + 1) * 32>(smem, threadIdx.x);
  } else if constexpr (F == kFmtFP4) {
    uint16_t* sl = reinterpret_cast<uint16_t*>(smem);
    for (int i = threadIdx.x; i < 256; i += blockDim.x) sl[i] = static_cast<uint16_t>(fp4_scale_bf16_bits(i));
  } else if constexpr (F == kFmtFP4S) {
    uint16_t* sl = reinterpret_cast<uint16_t*>(smem);
    for (int i = threadIdx.x; i < 256; i += blockDim.x) sl[i] = static_cast<uint16_t>(e4m3fn_bf16_bits_x2p110(i));
  }

  int nitems;
  const int* s_uexp = nullptr;
  const int* s_pair = nullptr;
  __shared__ uint32_t s_call;  // row-split: this launch's call number (its tag)
  if constexpr (MODE == kModeDense) {
    nitems = a.tiles;
    if (a.po.npeer && threadIdx.x == 0) s_call = peer_call(a.po);  // before launch_dependents: see peer_call
    __syncthreads();
    pdl_launch_dependents();
  } else {
    // The expert ids come from the previous kernel (the router): wait first.
    pdl_wait();
    moe_group(a.idx, a.P, a.E, a.topk, reinterpret_cast<int*>(smem + a.off_grp));  // ends with __syncthreads
    const int* s_idx = reinterpret_cast<const int*>(smem + a.off_grp);
    s_uexp = s_idx + 3 * kMaxPairs;
    s_pair = s_uexp + kMaxPairs;
    const int U = s_pair[kMaxPairs * 8];
    nitems = U * a.tiles;
    if constexpr (MODE == kModeMoe1) {
      if (blockIdx.x == 0 && a.meta != nullptr) {
        for (int i = threadIdx.x; i < 1 + 9 * a.P; i += blockDim.x) {
          int v;
          if (i == 0) v = U;
          else if (i <= a.P) v = (i - 1 < U) ? s_uexp[i - 1] : -1;
          else v = s_pair[i - 1 - a.P];
          a.meta[i] = v;
        }
      }
    }
    pdl_launch_dependents();
  }

  auto tile_src = [&](int item, int& rows_valid) -> const uint8_t* {
    int tile = item, mat = 0;
    if constexpr (MODE != kModeDense) {
      tile = item % a.tiles;
      mat = s_uexp[item / a.tiles];
    }
    rows_valid = min(16, a.rows - tile * 16);
    return a.w + (static_cast<int64_t>(mat) * a.rows + static_cast<int64_t>(tile) * 16) * a.row_bytes;
  };

  if (warp == KW) {
    // ================= producer warp =================
    // lane 0 waits for a free stage and posts the expected byte count; in segmented mode the 16
    // per-row copies are then issued by lanes 0..15 in parallel.
    uint32_t it = 0;
    for (int item = blockIdx.x; item < nitems; item += gridDim.x) {
      int rv;
      const uint8_t* src = tile_src(item, rv);
      for (int sp = 0; sp < a.nsplit; ++sp, ++it) {
        const int s = static_cast<int>(it % a.stages);
        uint8_t* dst = stages + s * a.stage_bytes;
        uint8_t* sdst = dst + a.sc_off;
        const int64_t row0 = (src - a.w) / a.row_bytes;  // global row of the tile's first row
        const uint8_t* ssrc = is_split(F) ? a.sc + row0 * a.sc_row_bytes : nullptr;
        if (lane == 0) {
          if (it >= static_cast<uint32_t>(a.stages)) mbar_wait(&empty[s], ((it / a.stages) - 1) & 1, kSiteEmptyWait);
          if (a.contiguous) {
            const uint32_t bytes = static_cast<uint32_t>(rv * a.row_bytes);
            const uint32_t bulk = bytes & ~15u;
            for (uint32_t b = bulk; b < bytes; ++b) dst[b] = src[b];  // < 16 trailing bytes
            uint32_t sbulk = 0;
            if constexpr (is_split(F)) {
              const uint32_t sbytes = static_cast<uint32_t>(rv * a.sc_row_bytes);
              sbulk = sbytes & ~15u;
              for (uint32_t b = sbulk; b < sbytes; ++b) sdst[b] = ssrc[b];
            }
            fence_proxy_async_smem();
            mbar_arrive_expect_tx(&full[s], bulk + sbulk);
            if (bulk) bulk_g2s(dst, src, bulk, &full[s]);
            if (sbulk) bulk_g2s(sdst, ssrc, sbulk, &full[s]);
          } else if (a.use_tmap) {
            mbar_arrive_expect_tx(&full[s], static_cast<uint32_t>(16 * a.stride + (is_split(F) ? 16 * a.sc_seg_bytes : 0)));
            tma_load_2d(dst, &a.tmap, sp * (a.seg_bytes / 8), static_cast<int>(row0), &full[s]);
            if constexpr (is_split(F)) tma_load_2d(sdst, &a.smap, sp * a.sc_seg_bytes, static_cast<int>(row0), &full[s]);
          } else {
            mbar_arrive_expect_tx(&full[s], static_cast<uint32_t>(rv * (a.seg_bytes + (is_split(F) ? a.sc_seg_bytes : 0))));
          }
        }
        __syncwarp();
        if (!a.contiguous && !a.use_tmap && lane < rv) {
          bulk_g2s(dst + lane * a.stride, src + static_cast<int64_t>(sp) * a.seg_bytes + static_cast<int64_t>(lane) * a.row_bytes,
                   a.seg_bytes, &full[s]);
          if constexpr (is_split(F))
            bulk_g2s(sdst + lane * a.sc_seg_bytes,
                     ssrc + static_cast<int64_t>(sp) * a.sc_seg_bytes + static_cast<int64_t>(lane) * a.sc_row_bytes,
                     a.sc_seg_bytes, &full[s]);
        }
      }
    }
    // drain: the last uses of each stage must have landed before the CTA may exit
    if (lane == 0) {
      const uint32_t total = it;
      const uint32_t first = total > static_cast<uint32_t>(a.stages) ? total - a.stages : 0u;
      for (uint32_t j = first; j < total; ++j) mbar_wait(&full[j % a.stages], (j / a.stages) & 1, kSiteDrainWait);
    }
    return;
  }

  // ================= consumers =================
  if constexpr (MODE == kModeDense) pdl_wait();  // x was written by the previous kernel
  const int g = lane >> 2, t = lane & 3;
  const int gps = a.kc / 32;  // k-groups per stage
  const int g0 = (warp * gps) / KW, g1 = ((warp + 1) * gps) / KW;
  float post = a.post;
  if constexpr (MODE == kModeDense && (F == kFmtFP4 || F == kFmtFP4S)) post *= __ldg(a.gscale);
  const uint32_t lut_lane = static_cast<uint32_t>(lane & 7) * 16u;
  const uint16_t* fp4lut = reinterpret_cast<const uint16_t*>(smem);

  uint32_t it = 0;
  for (int item = blockIdx.x; item < nitems; item += gridDim.x) {
    int u = 0, tile = item;
    if constexpr (MODE != kModeDense) {
      u = item / a.tiles;
      tile = item % a.tiles;
    }
    // activation row for B-fragment column n = nt*8 + g
    const bf16* xr[NT];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const int col = nt * 8 + g;
      int xrow;
      if constexpr (MODE == kModeMoe2) {
        const int p = col < 8 ? s_pair[u * 8 + col] : -1;
        xrow = p < 0 ? 0 : p;
      } else {
        xrow = min(col, a.R - 1);
      }
      xr[nt] = a.x + static_cast<int64_t>(xrow) * a.K;
    }
    float acc[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;

    for (int sp = 0; sp < a.nsplit; ++sp, ++it) {
      const int s = static_cast<int>(it % a.stages);
      mbar_wait(&full[s], (it / a.stages) & 1, kSiteFullWait);
      const uint8_t* st = stages + s * a.stage_bytes;
      const uint32_t r0 = static_cast<uint32_t>(g * a.stride), r1 = static_cast<uint32_t>((g + 8) * a.stride);
      const int kbase = sp * a.kc;
      for (int grp = g0; grp < g1; ++grp) {
        const int k0 = kbase + grp * 32;
        if constexpr (F == kFmtQ8) {
          uint32_t A0[4], A1[4];
          float d0, d1;
          q8_decode_row(st, r0, grp, t, A0, d0);
          q8_decode_row(st, r1, grp, t, A1, d1);
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            const uint2 xl = ldg64(xr[nt] + k0 + 4 * t);
            const uint2 xh = ldg64(xr[nt] + k0 + 16 + 4 * t);
            const float z[4] = {0.f, 0.f, 0.f, 0.f};
            float D[4];
            mma_bf16_16816(D, A0[0], A1[0], A0[1], A1[1], xl.x, xl.y, z);
            mma_bf16_16816(D, A0[2], A1[2], A0[3], A1[3], xh.x, xh.y, D);
            acc[nt][0] = fmaf(d0, D[0], acc[nt][0]);
            acc[nt][1] = fmaf(d0, D[1], acc[nt][1]);
            acc[nt][2] = fmaf(d1, D[2], acc[nt][2]);
            acc[nt][3] = fmaf(d1, D[3], acc[nt][3]);
          }
        } else if constexpr (F == kFmtIQ2) {
          iq2_group_mma<NT, false>(smem, st, r0, r1, grp, t, lut_lane, xr, k0, acc);
        } else if constexpr (is_split(F)) {
          const uint32_t scs = static_cast<uint32_t>(a.contiguous ? a.sc_row_bytes : a.sc_seg_bytes);
          split_group_mma<F, NT, false>(smem, st, st + a.sc_off, r0, r1, g * scs, (g + 8) * scs, grp, t,
                                                    lut_lane, xr, k0, acc);
        } else {  // NVFP4: group = sub-blocks 2h, 2h+1 of block grp/2
          const uint32_t bo = static_cast<uint32_t>(grp >> 1) * 36u;
          const uint32_t h2 = static_cast<uint32_t>(grp & 1) * 2u;
          const uint32_t sc0 = ld_u16(st, r0 + bo + h2), sc1 = ld_u16(st, r1 + bo + h2);
#pragma unroll
          for (int s2 = 0; s2 < 2; ++s2) {
            const uint32_t nib = bo + 4u + (h2 + s2) * 8u + 2u * t;
            const uint32_t v0 = ld_u16(st, r0 + nib), v1 = ld_u16(st, r1 + nib);
            const uint32_t S0 = fp4lut[(sc0 >> (8 * s2)) & 0xFFu], S1 = fp4lut[(sc1 >> (8 * s2)) & 0xFFu];
            uint32_t l0, h0, l1, h1;
            fp4_patterns(v0, l0, h0);
            fp4_patterns(v1, l1, h1);
            const uint32_t S0x2 = S0 | (S0 << 16), S1x2 = S1 | (S1 << 16);
            l0 = hmul2_bits(l0, S0x2);
            h0 = hmul2_bits(h0, S0x2);
            l1 = hmul2_bits(l1, S1x2);
            h1 = hmul2_bits(h1, S1x2);
            const int ks = k0 + 16 * s2;
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
              const uint32_t b0 = ldg32(xr[nt] + ks + 2 * t);
              const uint32_t b1 = ldg32(xr[nt] + ks + 8 + 2 * t);
              mma_bf16_16816(acc[nt], l0, l1, h0, h1, b0, b1, acc[nt]);
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }

    // ---- cross-warp reduction of the 16 x (8*NT) tile ----
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      float* rw = red + (warp * NT + nt) * 128;
      rw[g * 8 + 2 * t] = acc[nt][0];
      rw[g * 8 + 2 * t + 1] = acc[nt][1];
      rw[(g + 8) * 8 + 2 * t] = acc[nt][2];
      rw[(g + 8) * 8 + 2 * t + 1] = acc[nt][3];
    }
    named_bar_sync(1, KW * 32);
    for (int i = threadIdx.x; i < NT * 128; i += KW * 32) {
      const int nt = i >> 7, rl = (i & 127) >> 3, col = nt * 8 + (i & 7);
      float v = 0.f;
#pragma unroll
      for (int w2 = 0; w2 < KW; ++w2) v += red[(w2 * NT + nt) * 128 + (i & 127)];
      const int row = tile * 16 + rl;
      if (row >= a.rows || col >= a.R) continue;
      if constexpr (MODE == kModeDense) {
        if (a.po.npeer) peer_store(a.po, s_call, col, row, __float2bfloat16(v * post));
        else reinterpret_cast<bf16*>(a.y)[static_cast<int64_t>(col) * a.rows + row] = __float2bfloat16(v * post);
      } else {
        const int p = s_pair[u * 8 + col];
        if (p < 0) continue;
        const float vb = round_bf16(v);
        if constexpr (MODE == kModeMoe1) {
          const float r = fmaxf(vb, 0.f);
          reinterpret_cast<bf16*>(a.y)[static_cast<int64_t>(p) * a.rows + row] = __float2bfloat16(r * r);
        } else {
          reinterpret_cast<float*>(a.y)[static_cast<int64_t>(p) * a.rows + row] = vb;
        }
      }
    }
    named_bar_sync(1, KW * 32);
  }
  if constexpr (MODE == kModeDense) {
    if (a.po.npeer) peer_gather(a.po, s_call, a.R, threadIdx.x, KW * 32);  // the whole y, from the staging buffer
  }
}

}  // namespace gguf_b200
