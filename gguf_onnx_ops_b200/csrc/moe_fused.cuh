// MoeVerify iq2=3 in one persistent launch: expert grouping, fc1 + relu^2 and fc2 (the weighted
// sum over the top-k experts stays a small follow-up kernel).
//
// Every CTA recomputes the unique-expert grouping of idx in shared memory, then walks two work
// lists with the same producer / consumer ring as the GEMV engine:
//   phase 1  items (u, tile1), tile1 < I/16 : h[pair, 16 rows] = bf16(relu(bf16(z . W1[e]^T))^2)
//   phase 2  items (u, tile2), tile2 < H/16 : part[pair, 16 rows] = bf16(h[pair] . W2[e]^T)
// A finished phase-1 tile of expert u increments done[u] (release at GPU scope); a phase-2 item of
// expert u first waits (bounded, acquire) until done[u] == I/16, and reads h through L2.  Every
// CTA finishes all of its phase-1 items before any phase-2 item and the persistent grid holds one
// CTA per SM, so the waits always end.  The producer keeps streaming phase-2 weight tiles while
// the consumers wait, which overlaps the W2 fetch with the tail of phase 1.
//
// done[] lives in the first bytes of the `out` tensor (zeroed by the host with cudaMemsetAsync
// before the launch; `out` is only written by the finalize kernel that follows).
#pragma once

#include "engine.cuh"

namespace gguf_b200 {

struct MoeFusedArgs {
  const uint8_t* w1;  // [E, I, H/256*66]
  const uint8_t* w2;  // [E, H, I/256*66]
  const bf16* z;      // [R, H]
  const int32_t* idx; // [R, topk]
  bf16* h;            // [P, I]
  float* part;        // [P, H]
  int32_t* meta;      // [1 + 9P]
  int* done;          // [>= P] zeroed counters
  int R, topk, P, E, H, I;
  int rb1, rb2;       // row bytes of W1 / W2
  int T1, T2;         // 16-row tiles per expert: I/16, H/16
  int stage_bytes, stages;
  int off_stage, off_red, off_bar, off_grp;
};

constexpr int kMoeDoneWaitSite = 4;

template <int KW>
__global__ void __launch_bounds__((KW + 1) * 32, 1) moe_fused_kernel(const MoeFusedArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + a.off_bar);
  uint64_t* empty = full + a.stages;
  uint8_t* stages = smem + a.off_stage;
  float* red = reinterpret_cast<float*>(smem + a.off_red);
  int* s_grp = reinterpret_cast<int*>(smem + a.off_grp);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < a.stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], KW);
    }
    fence_mbar_init();
  }
  fill_iq2_lut_bf16<(KW + 1) * 32>(smem, threadIdx.x);
  pdl_wait();  // idx (router) and z come from earlier kernels
  moe_group(a.idx, a.P, a.E, a.topk, s_grp);  // ends with __syncthreads
  const int* s_uexp = s_grp + 3 * kMaxPairs;
  const int* s_pair = s_uexp + kMaxPairs;
  const int U = s_pair[kMaxPairs * 8];
  int* s_ready = s_grp + 4 * kMaxPairs + kMaxPairs * 8 + 4;  // per-CTA cache of "phase 1 of u done"
  if (blockIdx.x == 0)
    for (int i = threadIdx.x; i < 1 + 9 * a.P; i += blockDim.x) {
      int v;
      if (i == 0) v = U;
      else if (i <= a.P) v = (i - 1 < U) ? s_uexp[i - 1] : -1;
      else v = s_pair[i - 1 - a.P];
      a.meta[i] = v;
    }
  for (int i = threadIdx.x; i < kMaxPairs; i += blockDim.x) s_ready[i] = 0;
  __syncthreads();
  pdl_launch_dependents();

  const int n1 = U * a.T1, n2 = U * a.T2;
  // item q of this CTA's combined list: phase 1 items first, then phase 2
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

  if (warp == KW) {
    // ---------------- producer: one contiguous 16-row tile per stage ----------------
    if (lane == 0) {
      uint32_t it = 0;
      for (int q = blockIdx.x; q < n1 + n2; q += gridDim.x, ++it) {
        int phase, u, tile;
        item_of(q, phase, u, tile);
        const int s = static_cast<int>(it % a.stages);
        if (it >= static_cast<uint32_t>(a.stages)) mbar_wait(&empty[s], ((it / a.stages) - 1) & 1, kSiteEmptyWait);
        const int e = s_uexp[u];
        const uint8_t* src = phase == 1 ? a.w1 + (static_cast<int64_t>(e) * a.I + tile * 16) * a.rb1
                                        : a.w2 + (static_cast<int64_t>(e) * a.H + tile * 16) * a.rb2;
        const uint32_t bytes = 16u * static_cast<uint32_t>(phase == 1 ? a.rb1 : a.rb2);
        mbar_arrive_expect_tx(&full[s], bytes);
        bulk_g2s(stages + s * a.stage_bytes, src, bytes, &full[s]);
      }
      const uint32_t total = it;
      const uint32_t first = total > static_cast<uint32_t>(a.stages) ? total - a.stages : 0u;
      for (uint32_t j = first; j < total; ++j) mbar_wait(&full[j % a.stages], (j / a.stages) & 1, kSiteDrainWait);
    }
    return;
  }

  // ---------------- consumers ----------------
  const int g = lane >> 2, t = lane & 3;
  const uint32_t lut_lane = static_cast<uint32_t>(lane & 7) * 16u;
  uint32_t it = 0;
  for (int q = blockIdx.x; q < n1 + n2; q += gridDim.x, ++it) {
    int phase, u, tile;
    item_of(q, phase, u, tile);
    const int K = phase == 1 ? a.H : a.I;
    const uint32_t stride = static_cast<uint32_t>(phase == 1 ? a.rb1 : a.rb2);
    const bf16* xr[1];
    if (phase == 1) {
      xr[0] = a.z + static_cast<int64_t>(min(g, a.R - 1)) * a.H;
    } else {
      // All consumer threads read the cached flag before anyone may set it (barrier 2), so the
      // decision to take the barriers below is uniform.  Thread 0 then waits until every phase-1
      // tile of expert u has been published.
      const bool need = !s_ready[u];
      if (need) {
        named_bar_sync(2, KW * 32);
        if (threadIdx.x == 0) {
          const uint64_t t0 = global_timer_ns();
          int v;
          for (;;) {
            asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(a.done + u) : "memory");
            if (v >= a.T1) break;
            if (global_timer_ns() - t0 > kWaitLimitNs) {
              record_device_error(kMoeDoneWaitSite);
              break;
            }
            __nanosleep(256);
          }
          s_ready[u] = 1;
        }
        named_bar_sync(1, KW * 32);
      }
      const int p = s_pair[u * 8 + g];
      xr[0] = a.h + static_cast<int64_t>(p < 0 ? 0 : p) * a.I;
    }
    const int s = static_cast<int>(it % a.stages);
    mbar_wait(&full[s], (it / a.stages) & 1, kSiteFullWait);
    const uint8_t* st = stages + s * a.stage_bytes;
    const uint32_t r0 = static_cast<uint32_t>(g) * stride, r1 = static_cast<uint32_t>(g + 8) * stride;
    const int gps = K / 32;
    const int g0 = (warp * gps) / KW, g1 = ((warp + 1) * gps) / KW;
    float acc[1][4] = {{0.f, 0.f, 0.f, 0.f}};
    if (phase == 1) {
      for (int grp = g0; grp < g1; ++grp) iq2_group_mma<1, false>(smem, st, r0, r1, grp, t, lut_lane, xr, grp * 32, acc);
    } else {
      for (int grp = g0; grp < g1; ++grp) iq2_group_mma<1, true>(smem, st, r0, r1, grp, t, lut_lane, xr, grp * 32, acc);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
    // cross-warp reduction of the 16 x 8 tile
    float* rw = red + warp * 128;
    rw[g * 8 + 2 * t] = acc[0][0];
    rw[g * 8 + 2 * t + 1] = acc[0][1];
    rw[(g + 8) * 8 + 2 * t] = acc[0][2];
    rw[(g + 8) * 8 + 2 * t + 1] = acc[0][3];
    named_bar_sync(1, KW * 32);
    for (int i = threadIdx.x; i < 128; i += KW * 32) {
      const int rl = i >> 3, col = i & 7;
      float v = 0.f;
#pragma unroll
      for (int w2 = 0; w2 < KW; ++w2) v += red[w2 * 128 + i];
      const int p = s_pair[u * 8 + col];
      if (col >= a.R || p < 0) continue;
      const float vb = round_bf16(v);
      if (phase == 1) {
        const float r = fmaxf(vb, 0.f);
        a.h[static_cast<int64_t>(p) * a.I + tile * 16 + rl] = __float2bfloat16(r * r);
      } else {
        a.part[static_cast<int64_t>(p) * a.H + tile * 16 + rl] = vb;
      }
    }
    named_bar_sync(1, KW * 32);
    if (phase == 1 && threadIdx.x == 0) {  // publish: this tile of h is written
      __threadfence();
      atomicAdd(a.done + u, 1);
    }
  }
}

}  // namespace gguf_b200
