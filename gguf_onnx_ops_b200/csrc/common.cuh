// Common device helpers for the GGUF decode kernels (sm_100a): PTX wrappers for mbarriers, bulk
// async copies (TMA engine, this CTA only), programmatic dependent launch, mma.sync, bounded waits
// and the device-side error word.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace gguf_b200 {

using bf16 = __nv_bfloat16;

// Device-side error reporting: the first failing site wins; read back by gguf_device_status().
// (The library is a single translation unit; these are its only definitions.)
__device__ int g_dev_error = 0;
__device__ int g_dev_error_site = 0;

enum DeviceErrorSite : int {
  kSiteNone = 0,
  kSiteFullWait = 1,     // consumer waited too long for a weight stage
  kSiteEmptyWait = 2,    // producer waited too long for a free stage
  kSiteDrainWait = 3,    // producer waited too long for its last copies at exit
  kSitePeerWait = 5,     // a sharded op waited too long for a peer GPU's completion flag
  kSiteBadStateRow = 6,  // MambaVerify: the device-side state row was outside [0, state_rows) (row 0 used)
};

// A wait on an mbarrier that has not completed after this many nanoseconds is treated as a fault:
// the kernel records the site, stops waiting and finishes (results are then garbage, the status
// word says so).  Healthy waits last microseconds.
constexpr uint64_t kWaitLimitNs = 200ull * 1000ull * 1000ull;

__device__ __forceinline__ void record_device_error(int site) {
  if (atomicCAS(&g_dev_error, 0, 1) == 0) g_dev_error_site = site;
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------------------------------------
// mbarrier / bulk copy
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n"
      " .reg .pred p;\n"
      " mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n"
      "}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait for phase `parity` of `bar` to complete.  Returns false (and records `site`) on timeout.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int site) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (global_timer_ns() - t0 > kWaitLimitNs) {
      record_device_error(site);
      return false;
    }
  }
  return true;
}

// 1-D bulk copy global -> shared (this CTA), completion counted in bytes on `bar`.
// dst, src 16-byte aligned; bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// 2-D tiled tensor copy global -> shared (this CTA only): the box at element coordinates
// (x inner, y outer) of `map`; out-of-range elements are zero-filled and still counted in bytes.
// x * element size must be a multiple of 16 bytes; dst 128-byte aligned.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// ---------------------------------------------------------------------------------------------
// Programmatic dependent launch
// ---------------------------------------------------------------------------------------------
// Blocks until the preceding grid on the stream has completed and its writes are visible (no-op
// when the kernel was not launched as a programmatic dependent).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// Lets the next grid on the stream start launching (its CTAs run their prologue, then block in
// pdl_wait until this grid completes).
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---------------------------------------------------------------------------------------------
// Tensor core: D = A(16x16 bf16, row) * B(16x8 bf16, col) + C (f32)
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1, const float (&c)[4]) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%10,%11,%12,%13};\n"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(c[0]), "f"(c[1]), "f"(c[2]), "f"(c[3]));
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }
__device__ __forceinline__ float round_bf16(float v) { return __bfloat162float(__float2bfloat16(v)); }

// Read-only global loads (x rows are shared by all CTAs: keep them in L1/L2).
__device__ __forceinline__ uint4 ldg128(const void* p) { return __ldg(reinterpret_cast<const uint4*>(p)); }
__device__ __forceinline__ uint2 ldg64(const void* p) { return __ldg(reinterpret_cast<const uint2*>(p)); }
__device__ __forceinline__ uint32_t ldg32(const void* p) { return __ldg(reinterpret_cast<const uint32_t*>(p)); }

// ---------------------------------------------------------------------------------------------
// Sharded outputs over peer memory (row-split GEMV with its all-gather fused into the epilogue)
// ---------------------------------------------------------------------------------------------
constexpr int kMaxPeers = 8;

// Output of one shard of a row-split GEMV: every value is stored into the full-size y of every
// GPU of the group (peer pointers from CUDA IPC, NVLink stores), then an arrival count makes the
// launch complete only when every peer's shard has landed in this GPU's y.
struct PeerOut {
  bf16* y[kMaxPeers];          // y of GPU p: [R, ld] bf16 (this shard's rows start at row0)
  uint32_t* flags[kMaxPeers];  // arrival counters of GPU p: [kMaxPeers], slot q = CTAs of GPU q arrived (cumulative)
  uint32_t* state;             // this GPU: [0] = completed calls
  int npeer, rank, ld, row0;
  int vec;                     // 1: every y[p] 16-byte aligned, ld and row0 multiples of 8 (16-byte stores)
  int ctas;                    // CTAs every GPU of the group launches per call (the same on every GPU)
};

__device__ __forceinline__ void st_relaxed_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_relaxed_sys_add(uint32_t* p, uint32_t v) {
  asm volatile("red.relaxed.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// y[col, row] of this shard (row local to the shard) into every GPU's output.
__device__ __forceinline__ void peer_store(const PeerOut& po, int col, int row, bf16 v) {
  const int64_t off = static_cast<int64_t>(col) * po.ld + po.row0 + row;
#pragma unroll 1
  for (int p = 0; p < po.npeer; ++p) po.y[p][off] = v;
}

// The 16 y values of one activation row of a full 16-row tile (lane i of a 16-lane half-warp holds
// row i's value; both halves of the warp may hold different activation rows) into every GPU's y with
// 16-byte stores: a shuffle butterfly packs 8 consecutive values into lanes 0 and 8 of each half, which
// then store to each peer.  All 32 lanes call it (`v` of the lanes that hold no value is ignored when
// `ok` is false for that half); xr / row of the half's lane 0.
__device__ __forceinline__ void peer_store_tile16(const PeerOut& po, bf16 v, bool ok, int xr, int row) {
  const int lane = threadIdx.x & 31, li = lane & 15;
  uint32_t w = static_cast<uint32_t>(__bfloat16_as_ushort(v));
  w |= __shfl_down_sync(0xffffffffu, w, 1) << 16;  // even lanes: values i, i + 1
  const uint32_t w1 = __shfl_down_sync(0xffffffffu, w, 2);
  const uint32_t w2 = __shfl_down_sync(0xffffffffu, w, 4), w3 = __shfl_down_sync(0xffffffffu, w1, 4);
  // lanes 0 and 8 of each half: (w, w1, w2, w3) = values li .. li + 7
  const int src_xr = __shfl_sync(0xffffffffu, xr, lane & 16), src_row = __shfl_sync(0xffffffffu, row, lane & 16);
  const bool src_ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, lane & 16) != 0;
  if (src_ok && (li & 7) == 0) {
    const int64_t off = static_cast<int64_t>(src_xr) * po.ld + po.row0 + src_row + li;
    const uint4 q = make_uint4(w, w1, w2, w3);
#pragma unroll 1
    for (int p = 0; p < po.npeer; ++p) *reinterpret_cast<uint4*>(po.y[p] + off) = q;
  }
}

// Called by one thread per CTA after the CTA's last peer store (and a barrier over the threads that
// stored).  Every CTA makes its stores visible system-wide (one system-scope fence) and then counts
// itself as arrived at every GPU of the group (slot `rank` of each peer's arrival counters; the
// counters only grow, so nothing has to be reset between calls).  CTA 0 then waits, bounded, until
// every GPU's slot in its own counters holds calls * ctas: every CTA of every GPU, this call
// included, has arrived, so the whole y is present here when the launch ends.  Must run after
// griddepcontrol.wait (CTA 0 of the previous launch updates state[0] last).  A peer can be at most
// one call ahead (it cannot finish call e + 1 before this GPU's CTAs of call e + 1 arrive), so the
// counts compared below are at most one call's CTAs apart and the 32-bit difference is exact.
__device__ __forceinline__ void peer_complete(const PeerOut& po) {
  __threadfence_system();
  for (int p = 0; p < po.npeer; ++p) red_relaxed_sys_add(po.flags[p] + po.rank, 1u);
  if (blockIdx.x != 0) return;
  const uint32_t calls = *reinterpret_cast<volatile uint32_t*>(po.state) + 1u;
  const uint32_t target = calls * static_cast<uint32_t>(po.ctas);
  const uint32_t* mine = po.flags[po.rank];
  const uint64_t t0 = global_timer_ns();
  for (int p = 0; p < po.npeer; ++p) {
    while (static_cast<int32_t>(ld_acquire_sys(mine + p) - target) < 0) {
      if (global_timer_ns() - t0 > kWaitLimitNs) {
        record_device_error(kSitePeerWait);
        break;
      }
      __nanosleep(32);
    }
  }
  *reinterpret_cast<volatile uint32_t*>(po.state) = calls;
}

// Sum across GPUs of an f32 [R, H] partial (expert-parallel MoeVerify): every GPU stores its
// partial into slot `rank` of every GPU's reduction buffer [2 parities][world][r_max * H] (the
// parity of the call's epoch: a peer may run one call ahead), publishes its epoch, waits for every
// peer's, and sums the slots in rank order.
struct PeerReduce {
  float* slots[kMaxPeers];     // reduction buffer of GPU p
  uint32_t* flags[kMaxPeers];  // flag array of GPU p: [kMaxPeers]
  uint32_t* state;             // this GPU: [0] = completed epochs
  int npeer, rank;
  int slot_elems;              // r_max * H
};

// Thread 0 of the (single) reducing CTA, after the CTA's stores into the peers' slots: publish and
// wait (bounded).  Returns the epoch of this call.
__device__ __forceinline__ uint32_t peer_reduce_sync(const PeerReduce& pr, uint32_t epoch) {
  __threadfence_system();  // one system-scope fence orders the slot stores before every flag below
  for (int p = 0; p < pr.npeer; ++p) st_relaxed_sys(pr.flags[p] + pr.rank, epoch);
  const uint32_t* mine = pr.flags[pr.rank];
  const uint64_t t0 = global_timer_ns();
  for (int p = 0; p < pr.npeer; ++p) {
    while (static_cast<int32_t>(ld_acquire_sys(mine + p) - epoch) < 0) {
      if (global_timer_ns() - t0 > kWaitLimitNs) {
        record_device_error(kSitePeerWait);
        break;
      }
      __nanosleep(64);
    }
  }
  return epoch;
}

}  // namespace gguf_b200
