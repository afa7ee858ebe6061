// MoeVerify iq2=3 in one persistent launch: expert grouping, fc1 + relu^2 and fc2 (the weighted
// sum over the top-k experts stays a small follow-up kernel, launched with programmatic dependent
// launch so that it is resident before this one ends).
//
// Every CTA recomputes the unique-expert grouping of idx in shared memory, then its kMoeTeams teams
// of kMoeTeamWarps warps walk two work lists:
//   phase 1  items (u, tile1), tile1 < I/16 : h[pair, 16 rows] = bf16(relu(bf16(z . W1[e]^T))^2)
//   phase 2  items (u, tile2), tile2 < H/16 : part[pair, 16 rows] = bf16(h[pair] . W2[e]^T)
// A team owns one item at a time: its leader streams the item's 16 contiguous weight rows (one bulk
// copy) into the team's two-stage ring, each warp of the team decodes a quarter of the item's
// 32-element groups (up to 8 activation rows as MMA columns, engine.cuh's iq2_group_mma), and the
// team sums its four partial tiles through shared memory in warp order (deterministic) and stores.
// Items are dealt round-robin over all teams of the grid, so a decode-sized MoE (a few hundred
// items) runs in one or two rounds with no CTA-wide synchronisation per item.
//
// Phase order: a finished phase-1 item of expert u increments done[u] (release at GPU scope); a
// phase-2 item of expert u first waits (bounded, acquire) until done[u] == I/16, and reads h
// through L2.  Every team finishes its phase-1 items before its phase-2 items and the persistent
// grid holds one CTA per SM, so the waits always end.  The leader prefetches the team's next item
// while the team computes, which overlaps the W2 fetch with the tail of phase 1.
//
// done[] lives in the first bytes of the `out` tensor (zeroed by moe_zero_kernel, launched just
// before this kernel; `out` is only written by the finalize kernel that follows).
#pragma once

#include "engine.cuh"
#include "slice_iq2_i8.cuh"

namespace gguf_b200 {

struct MoeFusedArgs {
  const uint8_t* w1;  // [E, I, H/256*66]
  const uint8_t* w2;  // [E, H, I/256*66]
  const bf16* z;      // [R, H]
  const int32_t* idx; // [R, topk]
  bf16* h;            // [P, I]
  float* part;        // [P, H]
  int32_t* meta;      // [1 + 9P]
  int* done;          // [>= P] zeroed counters (in `out`)
  int R, topk, P, E, H, I;
  int rb1, rb2;       // row bytes of W1 / W2
  int T1, T2;         // 16-row tiles per expert: I/16, H/16
  int stage_bytes;    // one 16-row tile of either matrix (+ pad)
  int expert_offset;  // expert parallelism: global id of local expert 0 (idx holds global ids)
  int off_stage, off_red, off_bar, off_grp;
  int off_zf;         // moe_pairs_kernel: the z fragments of every activation row (kZFragBytes per row and slice)
};

// Publishes a finished fc1 tile: +1 on the expert's counter with release semantics at GPU scope
// (the caller's warp's, or after a barrier its CTA's, h stores are visible to whoever acquires the
// new count), without a separate full fence.
__device__ __forceinline__ void moe_publish(int* counter) {
  asm volatile("red.release.gpu.global.add.s32 [%0], 1;" ::"l"(counter) : "memory");
}

constexpr int kMoeDoneWaitSite = 4;
constexpr int kMoeTeams = 4, kMoeTeamWarps = 4, kMoeWarps = kMoeTeams * kMoeTeamWarps;
// The single-row kernel runs five teams per CTA (20 warps): 5 x 148 teams cover a decode step's
// phase-1 items (6 experts x I/16 = 672 at I = 1792) in one round, where four teams per CTA left
// the last expert's fc1 tiles for a second round that its fc2 items then waited for.
constexpr int kMoeR1Teams = 5, kMoeR1Warps = kMoeR1Teams * kMoeTeamWarps;

__global__ void __launch_bounds__(kMoeWarps * 32, 1) moe_fused_kernel(const MoeFusedArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int team = warp / kMoeTeamWarps, tw = warp % kMoeTeamWarps;
  const bool leader = tw == 0 && lane == 0;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + a.off_bar) + team * 4;  // [2] full, then [2] empty
  uint64_t* empty = full + 2;
  uint8_t* stage0 = smem + a.off_stage + team * 2 * a.stage_bytes;
  float* red = reinterpret_cast<float*>(smem + a.off_red) + team * 2 * kMoeTeamWarps * 128;  // [2][warps][128]
  int* s_grp = reinterpret_cast<int*>(smem + a.off_grp);

  if (leader) {
    for (int s = 0; s < 2; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kMoeTeamWarps);
    }
    fence_mbar_init();
  }
  fill_iq2_lut_bf16<kMoeWarps * 32>(smem, threadIdx.x);
  pdl_wait();  // idx (router) and z come from earlier kernels
  moe_group(a.idx, a.P, a.E, a.topk, s_grp, a.expert_offset);  // ends with __syncthreads
  const int* s_uexp = s_grp + 3 * kMaxPairs;
  const int* s_pair = s_uexp + kMaxPairs;
  const int U = s_pair[kMaxPairs * 8];
  if (blockIdx.x == 0)
    for (int i = threadIdx.x; i < 1 + 9 * a.P; i += blockDim.x) {
      int v;
      if (i == 0) v = U;
      else if (i <= a.P) v = (i - 1 < U) ? s_uexp[i - 1] + a.expert_offset : -1;
      else v = s_pair[i - 1 - a.P];
      a.meta[i] = v;
    }
  pdl_launch_dependents();

  const int n1 = U * a.T1, n2 = U * a.T2, nitems = n1 + n2;
  const int teams = kMoeTeams * static_cast<int>(gridDim.x);
  const int first = team * static_cast<int>(gridDim.x) + static_cast<int>(blockIdx.x);  // spread over SMs first
  // item q -> (phase, unique expert u, tile)
  auto item_of = [&](int q, int& phase, int& u, int& tile) {
    if (q < n1) {
      phase = 1;
      u = q / a.T1;
      tile = q % a.T1;
    } else {
      phase = 2;
      u = (q - n1) / a.T2;
      tile = (q - n1) % a.T2;
    }
  };
  // leader: stage (k & 1) <- the weights of this team's k-th item q
  auto fetch = [&](int q, uint32_t k) {
    int phase, u, tile;
    item_of(q, phase, u, tile);
    const int s = static_cast<int>(k & 1u);
    if (k >= 2u) mbar_wait(&empty[s], ((k >> 1) - 1u) & 1u, kSiteEmptyWait);
    const int e = s_uexp[u];
    const uint8_t* src = phase == 1 ? a.w1 + (static_cast<int64_t>(e) * a.I + tile * 16) * a.rb1
                                    : a.w2 + (static_cast<int64_t>(e) * a.H + tile * 16) * a.rb2;
    const uint32_t bytes = 16u * static_cast<uint32_t>(phase == 1 ? a.rb1 : a.rb2);
    mbar_arrive_expect_tx(&full[s], bytes);
    bulk_g2s(stage0 + s * a.stage_bytes, src, bytes, &full[s]);
  };
  if (leader) {
    if (first < nitems) fetch(first, 0u);
    if (first + teams < nitems) fetch(first + teams, 1u);
  }

  const int g = lane >> 2, t = lane & 3;
  const uint32_t lut_lane = static_cast<uint32_t>(lane & 7) * 16u;
  const int bar_id = 1 + team, bar_n = kMoeTeamWarps * 32;
  const int ti = tw * 32 + lane;  // thread index within the team
  uint32_t k = 0;
  for (int q = first; q < nitems; q += teams, ++k) {
    int phase, u, tile;
    item_of(q, phase, u, tile);
    const int K = phase == 1 ? a.H : a.I;
    const uint32_t stride = static_cast<uint32_t>(phase == 1 ? a.rb1 : a.rb2);
    if (phase == 2) {  // every phase-1 tile of expert u must be in h
      if (leader) {
        const uint64_t t0 = global_timer_ns();
        int v;
        for (;;) {
          asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(a.done + u) : "memory");
          if (v >= a.T1) break;
          if (global_timer_ns() - t0 > kWaitLimitNs) {
            record_device_error(kMoeDoneWaitSite);
            break;
          }
          __nanosleep(128);
        }
      }
      named_bar_sync(bar_id, bar_n);
    }
    // B column g = the activation row of pair (u, g) (columns without a pair read row 0; not stored)
    const bf16* xr[1];
    {
      const int p = s_pair[u * 8 + g];
      xr[0] = phase == 1 ? a.z + static_cast<int64_t>(p < 0 ? 0 : p / a.topk) * a.H
                         : a.h + static_cast<int64_t>(p < 0 ? 0 : p) * a.I;
    }
    const int s = static_cast<int>(k & 1u);
    mbar_wait(&full[s], (k >> 1) & 1u, kSiteFullWait);
    const uint8_t* st = stage0 + s * a.stage_bytes;
    const uint32_t r0 = static_cast<uint32_t>(g) * stride, r1 = static_cast<uint32_t>(g + 8) * stride;
    const int gps = K / 32;
    const int g0 = (tw * gps) / kMoeTeamWarps, g1 = ((tw + 1) * gps) / kMoeTeamWarps;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    // Activations in a 4-deep register ring: the loads of groups grp+4..grp+7 are in flight while
    // groups grp..grp+3 are decoded (h is read through L2: it was written by this launch).
    auto ldx = [&](int grp) -> uint4 {
      if (grp >= g1) return make_uint4(0u, 0u, 0u, 0u);
      const bf16* p = xr[0] + grp * 32 + 8 * t;
      return phase == 1 ? ldg128(p) : __ldcg(reinterpret_cast<const uint4*>(p));
    };
    uint4 x0 = ldx(g0), x1 = ldx(g0 + 1), x2 = ldx(g0 + 2), x3 = ldx(g0 + 3);
    for (int grp = g0; grp < g1; grp += 4) {
      const uint4 n0 = ldx(grp + 4), n1 = ldx(grp + 5), n2 = ldx(grp + 6), n3 = ldx(grp + 7);
      iq2_group_mma_x(smem, st, r0, r1, grp, t, lut_lane, x0, acc);
      if (grp + 1 < g1) iq2_group_mma_x(smem, st, r0, r1, grp + 1, t, lut_lane, x1, acc);
      if (grp + 2 < g1) iq2_group_mma_x(smem, st, r0, r1, grp + 2, t, lut_lane, x2, acc);
      if (grp + 3 < g1) iq2_group_mma_x(smem, st, r0, r1, grp + 3, t, lut_lane, x3, acc);
      x0 = n0;
      x1 = n1;
      x2 = n2;
      x3 = n3;
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
    // team reduction of the 16 x 8 tile; slot (k & 1) is rewritten two items later, after at least
    // one more team barrier
    float* rb = red + s * kMoeTeamWarps * 128;
    float* rw = rb + tw * 128;
    rw[g * 8 + 2 * t] = acc[0];
    rw[g * 8 + 2 * t + 1] = acc[1];
    rw[(g + 8) * 8 + 2 * t] = acc[2];
    rw[(g + 8) * 8 + 2 * t + 1] = acc[3];
    named_bar_sync(bar_id, bar_n);
    {
      const int rl = ti >> 3, col = ti & 7;  // 128 team threads <-> 16 rows x 8 columns
      const float v = (rb[ti] + rb[128 + ti]) + (rb[256 + ti] + rb[384 + ti]);
      const int p = s_pair[u * 8 + col];
      if (col < a.R && p >= 0) {
        const float vb = round_bf16(v);
        if (phase == 1) {
          const float r = fmaxf(vb, 0.f);
          a.h[static_cast<int64_t>(p) * a.I + tile * 16 + rl] = __float2bfloat16(r * r);
        } else {
          a.part[static_cast<int64_t>(p) * a.H + tile * 16 + rl] = vb;
        }
      }
    }
    if (leader && q + 2 * teams < nitems) fetch(q + 2 * teams, k + 2u);
    if (phase == 1) {  // publish: this tile of h is written (every team thread is past its store)
      named_bar_sync(bar_id, bar_n);
      if (leader) moe_publish(a.done + u);
    }
  }
}

// ---------------------------------------------------------------------------------------------
// The same MoE for one activation row (R = 1, the decode step) on the integer tensor cores: every
// unique expert has exactly one pair, so the single-row decode of slice_iq2_i8.cuh applies (exact
// u8 weights 64 + s*m, the row as two 8-bit limbs per 32-element group, block-diagonal MMA
// columns).  Phase 1 (K = 1024 = 4 slices): warp w of a team decodes slice w of its item with the
// fragments of z converted once per launch.  Phase 2 (K = I): warp w decodes slices w, w + 4, ...
// converting the pair's h slice (read through L2) right before each.  Work split, staging, phase
// order and outputs are those of moe_fused_kernel.  Tables (48 KB) sit at shared offset 0.
// ---------------------------------------------------------------------------------------------
// Phase-2 item q of a team: every phase-1 tile of its expert must be in h.  The team's leader warp
// polls the expert's counter in global memory (acquire, bounded) and then marks the item in the
// team's ready word (release, CTA scope); the other warps wait on that word in shared memory, so
// that one thread per team, not four, polls the counters the publishing warps update.  Items of a
// team increase, so `ready > q` also covers an item the leader has already gone past.
__device__ __forceinline__ void moe_wait_h(const int* done, int target, int* ready, int q, int tw, int lane) {
  if (lane == 0) {
    const uint64_t t0 = global_timer_ns();
    if (tw == 0) {
      int v;
      for (;;) {
        asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(done) : "memory");
        if (v >= target) break;
        if (global_timer_ns() - t0 > kWaitLimitNs) {
          record_device_error(kMoeDoneWaitSite);
          break;
        }
        __nanosleep(64);
      }
      asm volatile("st.release.cta.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(ready)), "r"(q + 1) : "memory");
    } else {
      int v;
      for (;;) {
        asm volatile("ld.acquire.cta.shared::cta.b32 %0, [%1];" : "=r"(v) : "r"(smem_u32(ready)) : "memory");
        if (v > q) break;
        if (global_timer_ns() - t0 > kWaitLimitNs) {
          record_device_error(kMoeDoneWaitSite);
          break;
        }
        __nanosleep(32);
      }
    }
  }
  __syncwarp();
}

__global__ void __launch_bounds__(kMoeR1Warps * 32, 1) moe_r1_i8_kernel(const MoeFusedArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int team = warp / kMoeTeamWarps, tw = warp % kMoeTeamWarps;
  const bool leader = tw == 0 && lane == 0;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + a.off_bar) + team * 4;  // [2] full, then [2] empty
  uint64_t* empty = full + 2;
  int* cnt = reinterpret_cast<int*>(smem + a.off_bar + kMoeR1Teams * 4 * 8) + team * 2;  // [2] arrivals per slot
  // the team's phase-2 ready word: 1 + the last item whose expert the leader saw complete in h
  int* ready = reinterpret_cast<int*>(smem + a.off_bar + kMoeR1Teams * 4 * 8) + 2 * kMoeR1Teams + team;
  uint8_t* stage0 = smem + a.off_stage + team * 2 * a.stage_bytes;
  float* red = reinterpret_cast<float*>(smem + a.off_red) + team * 2 * kMoeTeamWarps * 16;  // [2][warps][16]
  int* s_grp = reinterpret_cast<int*>(smem + a.off_grp);

  if (leader) {
    for (int s = 0; s < 2; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kMoeTeamWarps);
      cnt[s] = 0;
    }
    *ready = 0;
    fence_mbar_init();
  }
  i8_fill_tables<kMoeR1Warps * 32>(smem, threadIdx.x);
  pdl_wait();  // idx (router) and z come from earlier kernels
  const uint4 zv = ldg128(a.z + tw * 256 + 8 * lane);  // this warp's phase-1 slice of z, in flight during the grouping
  moe_group(a.idx, a.P, a.E, a.topk, s_grp, a.expert_offset);  // ends with __syncthreads
  const int* s_uexp = s_grp + 3 * kMaxPairs;
  const int* s_pair = s_uexp + kMaxPairs;
  const int U = s_pair[kMaxPairs * 8];
  if (blockIdx.x == 0)
    for (int i = threadIdx.x; i < 1 + 9 * a.P; i += blockDim.x) {
      int v;
      if (i == 0) v = U;
      else if (i <= a.P) v = (i - 1 < U) ? s_uexp[i - 1] + a.expert_offset : -1;
      else v = s_pair[i - 1 - a.P];
      a.meta[i] = v;
    }
  pdl_launch_dependents();

  const int n1 = U * a.T1, n2 = U * a.T2, nitems = n1 + n2;
  const int teams = kMoeR1Teams * static_cast<int>(gridDim.x);
  const int first = team * static_cast<int>(gridDim.x) + static_cast<int>(blockIdx.x);
  auto item_of = [&](int q, int& phase, int& u, int& tile) {
    if (q < n1) {
      phase = 1;
      u = q / a.T1;
      tile = q % a.T1;
    } else {
      phase = 2;
      u = (q - n1) / a.T2;
      tile = (q - n1) % a.T2;
    }
  };
  auto fetch = [&](int q, uint32_t k) {
    int phase, u, tile;
    item_of(q, phase, u, tile);
    const int s = static_cast<int>(k & 1u);
    if (k >= 2u) mbar_wait(&empty[s], ((k >> 1) - 1u) & 1u, kSiteEmptyWait);
    const int e = s_uexp[u];
    const uint8_t* src = phase == 1 ? a.w1 + (static_cast<int64_t>(e) * a.I + tile * 16) * a.rb1
                                    : a.w2 + (static_cast<int64_t>(e) * a.H + tile * 16) * a.rb2;
    const uint32_t bytes = 16u * static_cast<uint32_t>(phase == 1 ? a.rb1 : a.rb2);
    mbar_arrive_expect_tx(&full[s], bytes);
    bulk_g2s(stage0 + s * a.stage_bytes, src, bytes, &full[s]);
  };
  if (leader) {
    if (first < nitems) fetch(first, 0u);
    if (first + teams < nitems) fetch(first + teams, 1u);
  }

  const int g = lane >> 2, t = lane & 3;
  // z fragments of this warp's phase-1 slice (the single row's z, slice tw of H = 1024)
  I8XFrag zf;
  i8_x_frag<true>(zv, zf);
  const int slices2 = a.I / 256;
  // The warps of a team meet only through counters (as in moe_pairs_kernel): the last warp to
  // count itself into an item's slot sums it, stores the row, publishes and refills the stage.
  auto body = [&](int q, uint32_t k) {
    int phase, u, tile;
    item_of(q, phase, u, tile);
    const int p = s_pair[u * 8];  // the pair of row 0 (R = 1)
    if (phase == 2) moe_wait_h(a.done + u, a.T1, ready, q, tw, lane);  // every phase-1 tile of expert u is in h
    const int s = static_cast<int>(k & 1u);
    mbar_wait(&full[s], (k >> 1) & 1u, kSiteFullWait);
    const uint8_t* st = stage0 + s * a.stage_bytes;
    float acc0 = 0.f, acc1 = 0.f;
    if (phase == 1) {
      const uint32_t r0 = static_cast<uint32_t>(g * a.rb1), r1 = static_cast<uint32_t>((g + 8) * a.rb1);
      uint2 rc[4];
      uint32_t dbits;
      i8_records_any(st, r0, r1, static_cast<uint32_t>(tw) * 66u, rc, dbits);
      i8_slice(smem, rc, dbits, zf, acc0, acc1);
    } else {
      const uint32_t r0 = static_cast<uint32_t>(g * a.rb2), r1 = static_cast<uint32_t>((g + 8) * a.rb2);
      const bf16* hp = a.h + static_cast<int64_t>(p) * a.I;
      // every h slice of this warp in flight at once (read through L2: written by this launch)
      constexpr int kHPre = 2;
      uint4 hv[kHPre];
#pragma unroll
      for (int i = 0; i < kHPre; ++i) {
        const int sl = tw + i * kMoeTeamWarps;
        hv[i] = sl < slices2 ? __ldcg(reinterpret_cast<const uint4*>(hp + sl * 256 + 8 * lane)) : make_uint4(0u, 0u, 0u, 0u);
      }
      for (int sl = tw, i = 0; sl < slices2; sl += kMoeTeamWarps, ++i) {
        I8XFrag hf;
        uint4 xv = hv[0];
#pragma unroll
        for (int j = 1; j < kHPre; ++j)
          if (i == j) xv = hv[j];
        if (i >= kHPre) xv = __ldcg(reinterpret_cast<const uint4*>(hp + sl * 256 + 8 * lane));
        i8_x_frag<true>(xv, hf);
        uint2 rc[4];
        uint32_t dbits;
        i8_records_any(st, r0, r1, static_cast<uint32_t>(sl) * 66u, rc, dbits);
        float b0, b1;
        i8_slice(smem, rc, dbits, hf, b0, b1);
        acc0 += b0;
        acc1 += b1;
      }
    }
    acc0 += __shfl_xor_sync(0xffffffffu, acc0, 1);
    acc0 += __shfl_xor_sync(0xffffffffu, acc0, 2);
    acc1 += __shfl_xor_sync(0xffffffffu, acc1, 1);
    acc1 += __shfl_xor_sync(0xffffffffu, acc1, 2);
    // team reduction of the 16 rows.  Slot (k & 1) is rewritten two items later, after the stage
    // was refilled, which the last arriver of this item does after summing the slot.
    float* rb = red + s * kMoeTeamWarps * 16;
    if (t == 0) {
      rb[tw * 16 + g] = acc0;
      rb[tw * 16 + g + 8] = acc1;
    }
    __syncwarp();  // orders the lanes' slot writes and stage reads before lane 0's arrivals below
    int last = 0;
    if (lane == 0) {
      mbar_arrive(&empty[s]);
      last = atom_add_acq_rel_cta(&cnt[s], 1) == kMoeTeamWarps - 1;
    }
    if (__shfl_sync(0xffffffffu, last, 0)) {  // every warp's partials of this item are in the slot
      if (lane < 16 && p >= 0) {
        const float v = (rb[lane] + rb[16 + lane]) + (rb[32 + lane] + rb[48 + lane]);
        const float vb = round_bf16(v);
        if (phase == 1) {
          const float r = fmaxf(vb, 0.f);
          a.h[static_cast<int64_t>(p) * a.I + tile * 16 + lane] = __float2bfloat16(r * r);
        } else {
          a.part[static_cast<int64_t>(p) * a.H + tile * 16 + lane] = vb;
        }
      }
      __syncwarp();  // every lane's row stores (and slot reads) before lane 0's publish / refill
      if (lane == 0) {
        cnt[s] = 0;
        if (q + 2 * teams < nitems) {
          fence_proxy_async_smem();  // the warps' generic reads of the stage before the copy engine's writes
          fetch(q + 2 * teams, k + 2u);
        }
        if (phase == 1) moe_publish(a.done + u);  // this tile of h is written
      }
    }
  };
  uint32_t k = 0;
  for (int q = first; q < nitems; q += teams, ++k) body(q, k);
}

// ---------------------------------------------------------------------------------------------
// The same MoE for 2..8 activation rows (R > 1) on the integer tensor cores.  An expert's 16-row
// tile is decoded once (exact u8 weights 64 + s*m, the single-row decode of slice_iq2_i8.cuh) and
// the decoded A fragments are multiplied by every pair the expert has (the rows that selected it):
// per pair one set of block-diagonal B fragments (the pair's activation slice as two 8-bit limbs per
// 32-element group; column 2t carries group t, column 2t + 1 group t + 4, so each lane's C cells
// are the records it decoded) and one epilogue.  Phase 1 takes the B fragments of z from shared
// memory, where every CTA converts the R rows of z once per launch; phase 2 converts the pair's h
// slice (read through L2) right before its MMAs.  Work split, staging, phase order and outputs are
// those of moe_fused_kernel; the team sums its warps' partials per (pair, row) in warp order.
// ---------------------------------------------------------------------------------------------
constexpr int kZFragBytes = 8 * 64 + 8 * 8;  // per (row, slice): 8 groups x (8 high + 8 low limb words), xs[8], xoff[8]
constexpr int kZeroBytes = 64;                // zero limb words for lanes whose B half is empty
// moe_pairs_kernel: seven teams of two warps per CTA (more tiles in flight per SM and fewer warps per
// item reduction than four teams of four: C3 R = 8 58.7 against 63.4 µs)
constexpr int kMoePTW = 2;
constexpr int kMoePTeams = 7, kMoePWarps = kMoePTeams * kMoePTW;
static_assert(kMoePTW == 2 || kMoePTW == 4, "moe_pairs_kernel sums two or four warp partials");

// lane (g, t) of a permuted fragment (perm_x_frag): its non-zero B column carries group t (g = 2t,
// words bh0 / bl0) or group t + 4 (g = 2t + 1, words bh1 / bl1); every lane holds the xs / xoff of
// its groups t (xs0, xoff0) and t + 4 (xs1, xoff1)
__device__ __forceinline__ void zfrag_store(const I8XFrag& f, uint8_t* dst) {
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  uint32_t* w = reinterpret_cast<uint32_t*>(dst);
  if (g == 2 * t || g == 2 * t + 1) {
    const bool lo = g == 2 * t;
    uint32_t* gw = w + (lo ? t : t + 4) * 16;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      gw[j] = lo ? f.bh0[j] : f.bh1[j];
      gw[8 + j] = lo ? f.bl0[j] : f.bl1[j];
    }
  }
  if (g == 0) {
    float* xs = reinterpret_cast<float*>(w + 128);
    int* xo = reinterpret_cast<int*>(w + 136);
    xs[t] = f.xs0;
    xs[t + 4] = f.xs1;
    xo[t] = f.xoff0;
    xo[t + 4] = f.xoff1;
  }
}
// Each B half comes from its group's words or from the zero block (no selects).
__device__ __forceinline__ void zfrag_load(const uint8_t* src, const uint8_t* zero, I8XFrag& f) {
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const uint4* p0 = reinterpret_cast<const uint4*>(g == 2 * t ? src + t * 64 : zero);
  const uint4* p1 = reinterpret_cast<const uint4*>(g == 2 * t + 1 ? src + (t + 4) * 64 : zero);
  uint4 q[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    q[i] = p0[i];
    q[4 + i] = p1[i];
  }
  const uint32_t* v = reinterpret_cast<const uint32_t*>(q);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    f.bh0[j] = v[j];
    f.bl0[j] = v[8 + j];
    f.bh1[j] = v[16 + j];
    f.bl1[j] = v[24 + j];
  }
  const float* xs = reinterpret_cast<const float*>(src + 512);
  const int* xo = reinterpret_cast<const int*>(src + 544);
  f.xs0 = xs[t];
  f.xs1 = xs[t + 4];
  f.xoff0 = xo[t];
  f.xoff1 = xo[t + 4];
}

// The A fragments of one 16-row x 256-column slice (records rc of rows g, g + 8 x groups t, t + 4):
// A[e][r][h] = elements 8e + 4h .. 8e + 4h + 3 of record r as 64 + s * m bytes.
__device__ __forceinline__ void i8_decode(const uint8_t* smem, const uint2 (&rc)[4], uint32_t (&A)[4][4][2]) {
  const int lane = threadIdx.x & 31;
  const uint32_t lane_off = static_cast<uint32_t>(lane & 15) * 8u, lane_off128 = lane_off | 128u;
#pragma unroll
  for (int e = 0; e < 4; ++e) {
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const uint2 X = *reinterpret_cast<const uint2*>(smem + i8_mag_addr(rc[r].x, e, lane_off));
      const uint2 M = *reinterpret_cast<const uint2*>(smem + i8_sgn_addr(rc[r].y, e, lane_off128));
      A[e][r][0] = X.x - 2u * (X.x & M.x);
      A[e][r][1] = X.y - 2u * (X.y & M.y);
    }
  }
}
// 16 MMAs of decoded A against one pair's permuted fragments and the permuted-column epilogue: the
// lane's partial sums of weight rows g (acc0) and g + 8 (acc1) over its groups t, t + 4.
__device__ __forceinline__ void i8_pair_slice(const uint32_t (&A)[4][4][2], const uint2 (&rc)[4], uint32_t dbits,
                                              const I8XFrag& f, float& acc0, float& acc1) {
  int ch[4] = {0, 0, 0, 0};
  int cl[4] = {-f.xoff0, -f.xoff1, -f.xoff0, -f.xoff1};  // the weights' +64 offset, removed in the MMA
#pragma unroll
  for (int e = 0; e < 4; ++e) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int j = 2 * e + h;
      imma_u8s8(ch, A[e][0][h], A[e][2][h], A[e][1][h], A[e][3][h], f.bh0[j], f.bh1[j]);
      imma_u8u8(cl, A[e][0][h], A[e][2][h], A[e][1][h], A[e][3][h], f.bl0[j], f.bl1[j]);
    }
  }
  // cells [row g, group t], [g, t + 4], [g + 8, t], [g + 8, t + 4] = records 0..3; (2 s + 1) * cell
  // is exact in s32 (|cell| <= 32 * 43 * 32640, times 31 < 2^31); d * (0.5 + s) / 4 = d (2 s + 1) / 8
  const float v0 = static_cast<float>((ch[0] * 256 + cl[0]) * static_cast<int>((rc[0].y >> 27) | 1u));
  const float v1 = static_cast<float>((ch[1] * 256 + cl[1]) * static_cast<int>((rc[1].y >> 27) | 1u));
  const float v2 = static_cast<float>((ch[2] * 256 + cl[2]) * static_cast<int>((rc[2].y >> 27) | 1u));
  const float v3 = static_cast<float>((ch[3] * 256 + cl[3]) * static_cast<int>((rc[3].y >> 27) | 1u));
  const float d0 = fp16_bits_to_f32(dbits & 0xFFFFu) * 0.125f, d1 = fp16_bits_to_f32(dbits >> 16) * 0.125f;
  acc0 = fmaf(v0, f.xs0, v1 * f.xs1) * d0;
  acc1 = fmaf(v2, f.xs0, v3 * f.xs1) * d1;
}

__global__ void __launch_bounds__(kMoePWarps * 32, 1) moe_pairs_kernel(const MoeFusedArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int team = warp / kMoePTW, tw = warp % kMoePTW;
  const bool leader = tw == 0 && lane == 0;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + a.off_bar) + team * 4;  // [2] full, then [2] empty
  uint64_t* empty = full + 2;
  int* cnt = reinterpret_cast<int*>(smem + a.off_bar + kMoePTeams * 4 * 8) + team * 2;  // [2] arrivals per slot
  // the team's phase-2 ready word: 1 + the last item whose expert the leader saw complete in h
  int* ready = reinterpret_cast<int*>(smem + a.off_bar + kMoePTeams * 4 * 8) + 2 * kMoePTeams + team;
  uint8_t* stage0 = smem + a.off_stage + team * 2 * a.stage_bytes;
  float* red = reinterpret_cast<float*>(smem + a.off_red) + team * 2 * kMoePTW * 8 * 16;  // [2][warps][8 pairs][16]
  int* s_grp = reinterpret_cast<int*>(smem + a.off_grp);
  uint8_t* zf = smem + a.off_zf;  // [R][H / 256][kZFragBytes], then kZeroBytes of zeros, then the pair lists
  const uint8_t* zero = zf + a.R * (a.H / 256) * kZFragBytes;
  int* s_np = reinterpret_cast<int*>(zf + a.R * (a.H / 256) * kZFragBytes + kZeroBytes);  // [kMaxPairs]
  int* s_plist = s_np + kMaxPairs;  // [kMaxPairs][8]: pair id | activation row << 16

  if (leader) {
    for (int s = 0; s < 2; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kMoePTW);
      cnt[s] = 0;
    }
    *ready = 0;
    fence_mbar_init();
  }
  if (threadIdx.x < kZeroBytes / 4) reinterpret_cast<uint32_t*>(const_cast<uint8_t*>(zero))[threadIdx.x] = 0u;
  i8_fill_tables<kMoePWarps * 32>(smem, threadIdx.x);
  pdl_wait();  // idx (router) and z come from earlier kernels
  // z of this warp's (activation row, phase-1 slice) units (R * H / 256 <= 8 * 4), in flight during
  // the grouping
  const int slices1 = a.H / 256, slices2 = a.I / 256;
  constexpr int kZU = (8 * 4 + kMoePWarps - 1) / kMoePWarps;
  uint4 zv[kZU];
#pragma unroll
  for (int j = 0; j < kZU; ++j) {
    const int unit = warp + j * kMoePWarps;
    zv[j] = unit < a.R * slices1 ? ldg128(a.z + static_cast<int64_t>(unit / slices1) * a.H + (unit % slices1) * 256 + 8 * lane)
                                 : make_uint4(0u, 0u, 0u, 0u);
  }
  moe_group(a.idx, a.P, a.E, a.topk, s_grp, a.expert_offset);  // ends with __syncthreads
  const int* s_uexp = s_grp + 3 * kMaxPairs;
  const int* s_pair = s_uexp + kMaxPairs;
  const int U = s_pair[kMaxPairs * 8];
  if (blockIdx.x == 0)
    for (int i = threadIdx.x; i < 1 + 9 * a.P; i += blockDim.x) {
      int v;
      if (i == 0) v = U;
      else if (i <= a.P) v = (i - 1 < U) ? s_uexp[i - 1] + a.expert_offset : -1;
      else v = s_pair[i - 1 - a.P];
      a.meta[i] = v;
    }
  pdl_launch_dependents();
  // compact pair list of every unique expert (activation rows in increasing order)
  for (int u = threadIdx.x; u < U; u += blockDim.x) {
    int n = 0;
    for (int r = 0; r < a.R; ++r) {
      const int p = s_pair[u * 8 + r];
      if (p >= 0) s_plist[u * 8 + n++] = p | (r << 16);
    }
    s_np[u] = n;
  }

  const int n1 = U * a.T1, n2 = U * a.T2, nitems = n1 + n2;
  const int teams = kMoePTeams * static_cast<int>(gridDim.x);
  const int first = team * static_cast<int>(gridDim.x) + static_cast<int>(blockIdx.x);
  // item q -> (phase, unique expert u, tile); the quotients by T1 / T2 in fp32 (exact: q < 2^22)
  const float inv1 = 1.0f / static_cast<float>(a.T1), inv2 = 1.0f / static_cast<float>(a.T2);
  auto item_of = [&](int q, int& phase, int& u, int& tile) {
    const bool p1 = q < n1;
    const int qq = p1 ? q : q - n1, T = p1 ? a.T1 : a.T2;
    u = __float2int_rz((static_cast<float>(qq) + 0.5f) * (p1 ? inv1 : inv2));
    tile = qq - u * T;
    phase = p1 ? 1 : 2;
  };
  auto fetch = [&](int q, uint32_t k) {
    int phase, u, tile;
    item_of(q, phase, u, tile);
    const int s = static_cast<int>(k & 1u);
    if (k >= 2u) mbar_wait(&empty[s], ((k >> 1) - 1u) & 1u, kSiteEmptyWait);
    const int e = s_uexp[u];
    const uint8_t* src = phase == 1 ? a.w1 + (static_cast<int64_t>(e) * a.I + tile * 16) * a.rb1
                                    : a.w2 + (static_cast<int64_t>(e) * a.H + tile * 16) * a.rb2;
    const uint32_t bytes = 16u * static_cast<uint32_t>(phase == 1 ? a.rb1 : a.rb2);
    mbar_arrive_expect_tx(&full[s], bytes);
    bulk_g2s(stage0 + s * a.stage_bytes, src, bytes, &full[s]);
  };
  if (leader) {
    if (first < nitems) fetch(first, 0u);
    if (first + teams < nitems) fetch(first + teams, 1u);
  }

  // the z fragments of every (activation row, phase-1 slice): one conversion per CTA
#pragma unroll
  for (int j = 0; j < kZU; ++j) {
    const int unit = warp + j * kMoePWarps;
    if (unit < a.R * slices1) {
      I8XFrag f;
      perm_x_frag(zv[j], f);
      zfrag_store(f, zf + unit * kZFragBytes);
    }
  }
  __syncthreads();

  const int g = lane >> 2, t = lane & 3;
  // The four warps of a team meet only through counters: each warp adds its partial sums to the
  // item's reduction slot and counts itself in (acquire-release); the last one to arrive sums the
  // slot in warp order, stores the rows, publishes phase-1 tiles and refills the stage two items on.
  uint32_t k = 0;
  for (int q = first; q < nitems; q += teams, ++k) {
    int phase, u, tile;
    item_of(q, phase, u, tile);
    const int np = s_np[u];
    const int* pl = s_plist + u * 8;
    if (phase == 2) moe_wait_h(a.done + u, a.T1, ready, q, tw, lane);  // every phase-1 tile of expert u is in h
    const int s = static_cast<int>(k & 1u);
    mbar_wait(&full[s], (k >> 1) & 1u, kSiteFullWait);
    // this warp's partial row sums per pair.  Slot (k & 1) was summed by the last arriver of item
    // k - 2 before it refilled this stage, so it is free once the stage is full again.
    float* rbuf = red + s * kMoePTW * 8 * 16;
    float* mine = rbuf + tw * 8 * 16;
    for (int i = lane; i < np * 16; i += 32) mine[i] = 0.f;
    __syncwarp();
    const uint8_t* st = stage0 + s * a.stage_bytes;
    const uint32_t rb = static_cast<uint32_t>(phase == 1 ? a.rb1 : a.rb2);
    const uint32_t r0 = static_cast<uint32_t>(g) * rb, r1 = static_cast<uint32_t>(g + 8) * rb;
    // one pair's MMAs on decoded A, reduced over the quad and added to the warp's slot of the pair
    auto pair_step = [&](const uint32_t (&A)[4][4][2], const uint2 (&rc)[4], uint32_t dbits, const I8XFrag& f, int i) {
      float v0, v1;
      i8_pair_slice(A, rc, dbits, f, v0, v1);
      v0 += __shfl_xor_sync(0xffffffffu, v0, 1);
      v0 += __shfl_xor_sync(0xffffffffu, v0, 2);
      v1 += __shfl_xor_sync(0xffffffffu, v1, 1);
      v1 += __shfl_xor_sync(0xffffffffu, v1, 2);
      if (t == 0) {
        mine[i * 16 + g] += v0;
        mine[i * 16 + g + 8] += v1;
      }
    };
    if (phase == 1) {
      for (int sl = tw; sl < slices1; sl += kMoePTW) {
        uint2 rc[4];
        uint32_t dbits;
        i8_records_any(st, r0, r1, static_cast<uint32_t>(sl) * 66u, rc, dbits);
        uint32_t A[4][4][2];
        i8_decode(smem, rc, A);
        for (int i = 0; i < np; ++i) {  // every pair of the expert, same decoded A
          I8XFrag f;
          zfrag_load(zf + ((pl[i] >> 16) * slices1 + sl) * kZFragBytes, zero, f);
          pair_step(A, rc, dbits, f, i);
        }
      }
    } else {
      for (int sl = tw; sl < slices2; sl += kMoePTW) {
        // the first pair's h slice is in flight while the tile decodes (read through L2)
        uint4 hv = __ldcg(reinterpret_cast<const uint4*>(a.h + static_cast<int64_t>(pl[0] & 0xFFFF) * a.I + sl * 256 + 8 * lane));
        uint2 rc[4];
        uint32_t dbits;
        i8_records_any(st, r0, r1, static_cast<uint32_t>(sl) * 66u, rc, dbits);
        uint32_t A[4][4][2];
        i8_decode(smem, rc, A);
        for (int i = 0; i < np; ++i) {
          const uint4 cur = hv;
          if (i + 1 < np)  // the next pair's slice while this one computes
            hv = __ldcg(reinterpret_cast<const uint4*>(a.h + static_cast<int64_t>(pl[i + 1] & 0xFFFF) * a.I + sl * 256 + 8 * lane));
          I8XFrag f;
          perm_x_frag(cur, f);
          pair_step(A, rc, dbits, f, i);
        }
      }
    }
    __syncwarp();  // orders the lanes' slot writes and stage reads before lane 0's arrivals below
    int last = 0;
    if (lane == 0) {
      mbar_arrive(&empty[s]);
      last = atom_add_acq_rel_cta(&cnt[s], 1) == kMoePTW - 1;
    }
    if (__shfl_sync(0xffffffffu, last, 0)) {  // every warp's partials of this item are in the slot
      for (int ti = lane; ti < np * 16; ti += 32) {
        const int i = ti >> 4, rl = ti & 15;
        const int p = pl[i] & 0xFFFF;
        // fixed order: warps 0 + 1 (then 2 + 3 with four-warp teams)
        const float v = kMoePTW == 4 ? (rbuf[ti] + rbuf[128 + ti]) + (rbuf[256 + ti] + rbuf[384 + ti])
                                     : rbuf[ti] + rbuf[128 + ti];
        const float vb = round_bf16(v);
        if (phase == 1) {
          const float rr = fmaxf(vb, 0.f);
          a.h[static_cast<int64_t>(p) * a.I + tile * 16 + rl] = __float2bfloat16(rr * rr);
        } else {
          a.part[static_cast<int64_t>(p) * a.H + tile * 16 + rl] = vb;
        }
      }
      __syncwarp();  // every lane's row stores (and slot reads) before lane 0's publish / refill
      if (lane == 0) {
        cnt[s] = 0;
        if (q + 2 * teams < nitems) {
          fence_proxy_async_smem();  // the warps' generic reads of the stage before the copy engine's writes
          fetch(q + 2 * teams, k + 2u);
        }
        if (phase == 1) moe_publish(a.done + u);  // this tile of h is written
      }
    }
  }
}

}  // namespace gguf_b200
