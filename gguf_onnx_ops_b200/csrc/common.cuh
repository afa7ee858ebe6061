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
  kSitePeerWait = 5,     // a sharded op waited too long for a peer GPU (its row-split words or EP partials)
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

// 2^n for -149 <= n <= 127, exactly (the IEEE single layout: exponent field n + 127 for normal numbers,
// one significand bit for subnormal ones); a few integer instructions where ldexpf is a library call.
__device__ __forceinline__ float pow2i(int n) {
  return __uint_as_float(n >= -126 ? static_cast<uint32_t>(n + 127) << 23 : 1u << (n + 149));
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

// Output of one shard of a row-split GEMV.  Every y value travels as one 32-bit word: the bf16
// bits in the low half and the call's tag (call number mod 2^16) in the high half, stored into the
// staging buffer of every GPU of the group (peer pointers from CUDA IPC, NVLink stores; one buffer
// per call parity, since a peer can be one call ahead).  A 32-bit store is seen whole or not at all,
// so a word whose tag is this call's is this call's value: no fence and no flag is needed.  After
// its tiles each CTA converts its slice of this GPU's staging buffer into y, waiting (bounded) for
// words that still carry an older tag; the launch therefore ends only when the whole y is present.
struct PeerOut {
  uint32_t* stage[2][kMaxPeers];  // staging buffer of GPU p for calls of parity c: [r_max, ld] words
  bf16* y;                        // this GPU's output: [R, ld] bf16
  unsigned long long* state;      // this GPU: CTAs of row-split launches started so far
  int npeer, rank, ld, row0;
  int vec;                        // 1: ld and row0 multiples of 8 and every buffer 16-byte aligned
  int ctas;                       // CTAs every GPU of the group launches per call (the same on every GPU)
};

// The call number of this launch (1, 2, ...) from this GPU's count of row-split CTAs started: every
// call of the group launches po.ctas CTAs and each CTA counts itself once.  Thread 0 calls it before
// the CTA's griddepcontrol.launch_dependents (and uses the result before the CTA's first barrier): a
// dependent launch starts only once every CTA of its predecessor has passed launch_dependents, so
// all of the previous call's counts precede this call's.
__device__ __forceinline__ uint32_t peer_call(const PeerOut& po) {
  const unsigned long long before = atomicAdd(po.state, 1ull);
  return static_cast<uint32_t>(before / static_cast<unsigned long long>(po.ctas)) + 1u;
}

__device__ __forceinline__ uint4 ld_relaxed_sys_v4(const uint32_t* p) {
  uint4 v;
  asm volatile("ld.relaxed.sys.global.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}
__device__ __forceinline__ uint32_t ld_relaxed_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_relaxed_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// y[col, row] of this shard (row local to the shard) into every GPU's staging buffer.
__device__ __forceinline__ void peer_store(const PeerOut& po, uint32_t call, int col, int row, bf16 v) {
  const int64_t off = static_cast<int64_t>(col) * po.ld + po.row0 + row;
  const uint32_t w = static_cast<uint32_t>(__bfloat16_as_ushort(v)) | (call << 16);
  uint32_t* const* st = po.stage[call & 1u];
#pragma unroll 1
  for (int p = 0; p < po.npeer; ++p) st[p][off] = w;
}

// The 16 y values of one activation row of a full 16-row tile (lane i of a 16-lane half-warp holds
// row i's value; both halves of the warp may hold different activation rows) into every GPU's
// staging buffer with 16-byte stores: lanes 0, 4, 8, 12 of each half gather four tagged words by
// shuffles and store them to each peer.  All 32 lanes call it (`ok` false: the half holds no
// activation row); xr / row of the half's lane 0.
__device__ __forceinline__ void peer_store_tile16(const PeerOut& po, uint32_t call, bf16 v, bool ok, int xr, int row) {
  const int lane = threadIdx.x & 31, li = lane & 15;
  const uint32_t w = static_cast<uint32_t>(__bfloat16_as_ushort(v)) | (call << 16);
  const uint32_t w1 = __shfl_down_sync(0xffffffffu, w, 1), w2 = __shfl_down_sync(0xffffffffu, w, 2);
  const uint32_t w3 = __shfl_down_sync(0xffffffffu, w, 3);
  const int src_xr = __shfl_sync(0xffffffffu, xr, lane & 16), src_row = __shfl_sync(0xffffffffu, row, lane & 16);
  const bool src_ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, lane & 16) != 0;
  if (src_ok && (li & 3) == 0) {
    const int64_t off = static_cast<int64_t>(src_xr) * po.ld + po.row0 + src_row + li;
    const uint4 q = make_uint4(w, w1, w2, w3);
    uint32_t* const* st = po.stage[call & 1u];
#pragma unroll 1
    for (int p = 0; p < po.npeer; ++p) *reinterpret_cast<uint4*>(st[p] + off) = q;
  }
}

// After the CTA's tiles (all of its stores issued): threads tid .. of nthr convert this CTA's slice of
// this GPU's staging buffer ([R, ld] words, the slices split evenly over the grid) into y, re-reading
// a word until it carries this call's tag (bounded: on timeout the site is recorded, the wait
// stops for the rest of the slice and y holds stale values).
__device__ __forceinline__ void peer_gather(const PeerOut& po, uint32_t call, int R, int tid, int nthr) {
  const uint32_t* src = po.stage[call & 1u][po.rank];
  const uint32_t tag = call & 0xFFFFu;
  const int64_t total = static_cast<int64_t>(R) * po.ld;
  const uint64_t t0 = global_timer_ns();
  bool late = false;
  if (po.vec) {  // four words -> four bf16 per step
    const int64_t n4 = total / 4;
    const int64_t lo = n4 * blockIdx.x / gridDim.x, hi = n4 * (blockIdx.x + 1) / gridDim.x;
    for (int64_t i = lo + tid; i < hi; i += nthr) {
      uint4 q = ld_relaxed_sys_v4(src + 4 * i);
      while (!late && ((q.x >> 16) != tag || (q.y >> 16) != tag || (q.z >> 16) != tag || (q.w >> 16) != tag)) {
        if (global_timer_ns() - t0 > kWaitLimitNs) {
          late = true;
          record_device_error(kSitePeerWait);
          break;
        }
        __nanosleep(32);
        q = ld_relaxed_sys_v4(src + 4 * i);
      }
      *reinterpret_cast<uint2*>(po.y + 4 * i) = make_uint2((q.x & 0xFFFFu) | (q.y << 16), (q.z & 0xFFFFu) | (q.w << 16));
    }
  } else {
    const int64_t lo = total * blockIdx.x / gridDim.x, hi = total * (blockIdx.x + 1) / gridDim.x;
    for (int64_t i = lo + tid; i < hi; i += nthr) {
      uint32_t q = ld_relaxed_sys(src + i);
      while (!late && (q >> 16) != tag) {
        if (global_timer_ns() - t0 > kWaitLimitNs) {
          late = true;
          record_device_error(kSitePeerWait);
          break;
        }
        __nanosleep(32);
        q = ld_relaxed_sys(src + i);
      }
      po.y[i] = __ushort_as_bfloat16(static_cast<unsigned short>(q & 0xFFFFu));
    }
  }
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
