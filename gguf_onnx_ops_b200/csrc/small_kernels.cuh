// Router (MoeRouteGGUF), MoE finalize and dequantise kernels.
#pragma once

#include "decode.cuh"

namespace gguf_b200 {

// ---------------------------------------------------------------------------------------------
// MoeRouteGGUF: one thread-block cluster of kRouteCtas CTAs per block of kRouteRows rows.
// CTA c of a cluster computes the sigmoid scores of experts [c*E/n, (c+1)*E/n) for the cluster's
// rows (gate row read once from HBM, rounded to bf16 in registers as src/bolt_ops.cu:441-448;
// fp32 dot products in a fixed order), writes them to `scores` and, through distributed shared
// memory, into CTA 0's shared copy; the cluster barrier (release/acquire at cluster scope) makes
// every CTA's copy visible to CTA 0, whose warp w selects the top-k of row (cluster row base + w)
// from shared memory: iterative arg-max of score + bias with ties to the lower expert index
// (src/bolt_ops.cu:459-510).
// ---------------------------------------------------------------------------------------------
constexpr int kRouteCtas = 8, kRouteRows = 8, kRouteWarps = 16;
static_assert(kRouteRows < kRouteWarps, "CTA 0's warps past the selecting ones write the scores output");
constexpr int kRouteMaxE = 512;  // experts the router takes (the op contract)
constexpr int kRoutePre = 4;  // 256-element chunks of a warp's first gate row fetched before the dependency wait

// Shared-memory address of the same variable in CTA 0 of the cluster, and a store to it.
__device__ __forceinline__ uint32_t map_shared_cta0(const void* p) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, 0;" : "=r"(r) : "r"(smem_u32(p)));
  return r;
}
__device__ __forceinline__ void st_shared_cluster_f32(uint32_t addr, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;\n" ::: "memory");
}

// float -> unsigned key with the same order
__device__ __forceinline__ uint32_t ordered_key(float f) {
  const uint32_t b = __float_as_uint(f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// Top-k of one row by one warp: lane l holds experts l, l + 32, ... (kPer of them).  Each pick is an
// arg-max of score + bias over the warp with ties to the lower expert index (src/bolt_ops.cu:459-510):
// one warp max of the ordered keys, then one warp min of the indices holding that key.
// sr: the row's scores in this CTA's shared memory; bv[i]: the bias of expert lane + 32 i.
template <int kPer>
__device__ __forceinline__ void route_select(const float* __restrict__ sr, const float (&bv)[kPer], int row, int E,
                                             int topk, float scale, int32_t* __restrict__ idx_out,
                                             float* __restrict__ w_out) {
  const int lane = threadIdx.x & 31;
  float sc[kPer];
  uint32_t key[kPer];
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int e = lane + 32 * i;
    sc[i] = e < E ? sr[e] : 0.f;
    const float v = e < E ? sc[i] + bv[i] : 0.f;
    key[i] = (e < E && v == v) ? ordered_key(v) : 0u;  // 0: below every real key (absent or NaN: never picked)
  }
  int my_idx = -1;
  float my_sc = 0.f, sum = 0.f;
  for (int j = 0; j < topk; ++j) {
    uint32_t bk = 0u;
    int bi = 0x7FFFFFFF;
#pragma unroll
    for (int i = 0; i < kPer; ++i)
      if (key[i] > bk) {  // ascending expert order within the lane: the first maximum wins
        bk = key[i];
        bi = lane + 32 * i;
      }
    const uint32_t wk = __reduce_max_sync(0xffffffffu, bk);
    const int wi = static_cast<int>(__reduce_min_sync(0xffffffffu, static_cast<uint32_t>(bk == wk ? bi : 0x7FFFFFFF)));
    float s = 0.f;
    if (wk != 0u) {
      const int owner = wi & 31, slot = wi >> 5;
      float mine = 0.f;
#pragma unroll
      for (int i = 0; i < kPer; ++i)
        if (i == slot) mine = sc[i];
      s = __shfl_sync(0xffffffffu, mine, owner);
      if (lane == owner) {
#pragma unroll
        for (int i = 0; i < kPer; ++i)
          if (i == slot) key[i] = 0u;
      }
    }
    if (lane == j) {
      my_idx = wk != 0u ? wi : -1;
      my_sc = s;
    }
    sum += s;
  }
  const float denom = sum + 1e-20f;
  if (lane < topk) {
    idx_out[static_cast<int64_t>(row) * topk + lane] = my_idx;
    w_out[static_cast<int64_t>(row) * topk + lane] = my_sc / denom * scale;
  }
}

// 8 consecutive gate weights of one lane: fp32 (MoeRouteGGUF, rounded to bf16 on use) or bf16
// (MoeRoute).  Both give the same bf16 values to the dot product, so the two ops agree exactly.
template <typename WT>
struct GateChunk;
template <>
struct GateChunk<float> {
  float4 a, b;
  __device__ __forceinline__ static GateChunk load(const float* row, int k) {
    return {__ldg(reinterpret_cast<const float4*>(row + k)), __ldg(reinterpret_cast<const float4*>(row + k + 4))};
  }
  __device__ __forceinline__ static GateChunk zero() {
    return {make_float4(0.f, 0.f, 0.f, 0.f), make_float4(0.f, 0.f, 0.f, 0.f)};
  }
  __device__ __forceinline__ void to8(float (&wb)[8]) const {
    wb[0] = round_bf16(a.x); wb[1] = round_bf16(a.y); wb[2] = round_bf16(a.z); wb[3] = round_bf16(a.w);
    wb[4] = round_bf16(b.x); wb[5] = round_bf16(b.y); wb[6] = round_bf16(b.z); wb[7] = round_bf16(b.w);
  }
};
template <>
struct GateChunk<bf16> {
  uint4 a;
  __device__ __forceinline__ static GateChunk load(const bf16* row, int k) { return {ldg128(row + k)}; }
  __device__ __forceinline__ static GateChunk zero() { return {make_uint4(0u, 0u, 0u, 0u)}; }
  __device__ __forceinline__ void to8(float (&wb)[8]) const {
    wb[0] = bf16_lo(a.x); wb[1] = bf16_hi(a.x); wb[2] = bf16_lo(a.y); wb[3] = bf16_hi(a.y);
    wb[4] = bf16_lo(a.z); wb[5] = bf16_hi(a.z); wb[6] = bf16_lo(a.w); wb[7] = bf16_hi(a.w);
  }
};

// kStaged: the cluster's x rows are copied once into shared memory (dynamic, kRouteRows x K bf16)
// right after the dependency wait, one load round trip for all rows, and every warp reads its
// chunks from there; otherwise each warp loads its rows' chunks through L1 row by row.
template <typename WT, bool kStaged>
__global__ void __cluster_dims__(kRouteCtas, 1, 1) __launch_bounds__(kRouteWarps * 32)
    route_kernel(const bf16* __restrict__ x, const WT* __restrict__ gw, const float* __restrict__ bias, int R, int K,
                 int E, int topk, float scale, int32_t* __restrict__ idx_out, float* __restrict__ w_out,
                 float* __restrict__ scores) {
  const int cluster = blockIdx.x / kRouteCtas, rank = blockIdx.x % kRouteCtas;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row0 = cluster * kRouteRows;
  const int nrows = min(kRouteRows, R - row0);
  const int e_lo = (rank * E) / kRouteCtas, e_hi = ((rank + 1) * E) / kRouteCtas;
  const int e_first = e_lo + warp;
  // scores of the cluster's rows, gathered in CTA 0's shared memory for the top-k (E <= kRouteMaxE)
  __shared__ float s_sc[kRouteRows][kRouteMaxE];
  // bias of the experts a top-k lane owns (lane + 32 i), fetched before the dependency wait
  constexpr int kPerMax = kRouteMaxE / 32;
  float bv[kPerMax];
#pragma unroll
  for (int i = 0; i < kPerMax; ++i) {
    const int e = lane + 32 * i;
    bv[i] = (rank == 0 && e < E) ? __ldg(bias + e) : 0.f;
  }
  // The gate weights do not depend on the previous kernel: this warp's first row (up to
  // kRoutePre * 256 elements) is in flight before the dependency wait.
  GateChunk<WT> pw[kRoutePre];
#pragma unroll
  for (int c = 0; c < kRoutePre; ++c) {
    const int k = c * 256 + lane * 8;
    pw[c] = (e_first < e_hi && k < K) ? GateChunk<WT>::load(gw + static_cast<int64_t>(e_first) * K, k)
                                      : GateChunk<WT>::zero();
  }
  pdl_wait();
  pdl_launch_dependents();
  extern __shared__ __align__(16) uint8_t route_xs[];
  const bf16* xr = x + static_cast<int64_t>(row0) * K;  // the cluster's first row (global, or staged)
  if constexpr (kStaged) {
    const uint4* src = reinterpret_cast<const uint4*>(xr);
    uint4* dst = reinterpret_cast<uint4*>(route_xs);
    for (int i = threadIdx.x; i < nrows * (K / 8); i += kRouteWarps * 32) dst[i] = ldg128(src + i);
    __syncthreads();
    xr = reinterpret_cast<const bf16*>(route_xs);
  }
  for (int e = e_first; e < e_hi; e += kRouteWarps) {
    const WT* wr = gw + static_cast<int64_t>(e) * K;
    float acc[kRouteRows];
#pragma unroll
    for (int r = 0; r < kRouteRows; ++r) acc[r] = 0.f;
    // one 8-element chunk at k (this lane's elements k..k+7), accumulated in increasing k
    auto chunk = [&](const GateChunk<WT> gc, int k) {
      float wb[8];
      gc.to8(wb);
#pragma unroll
      for (int r = 0; r < kRouteRows; ++r) {
        if (r < nrows) {
          const uint4 xv = kStaged ? *reinterpret_cast<const uint4*>(xr + static_cast<int64_t>(r) * K + k)
                                   : ldg128(xr + static_cast<int64_t>(r) * K + k);
          const uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            acc[r] = fmaf(bf16_lo(xw[i]), wb[2 * i], acc[r]);
            acc[r] = fmaf(bf16_hi(xw[i]), wb[2 * i + 1], acc[r]);
          }
        }
      }
    };
    int k0 = lane * 8;
    if (e == e_first) {
      // rows outer, chunks inner: acc[r] still accumulates in increasing k
      float wb[kRoutePre][8];
#pragma unroll
      for (int c = 0; c < kRoutePre; ++c) pw[c].to8(wb[c]);
#pragma unroll
      for (int r = 0; r < kRouteRows; ++r) {
        if (r >= nrows) break;
        uint4 xv[kRoutePre];
#pragma unroll
        for (int c = 0; c < kRoutePre; ++c)
          xv[c] = c * 256 + lane * 8 >= K ? make_uint4(0u, 0u, 0u, 0u)
                  : kStaged ? *reinterpret_cast<const uint4*>(xr + static_cast<int64_t>(r) * K + c * 256 + lane * 8)
                            : ldg128(xr + static_cast<int64_t>(r) * K + c * 256 + lane * 8);
#pragma unroll
        for (int c = 0; c < kRoutePre; ++c) {
          if (c * 256 + lane * 8 >= K) break;
          const uint32_t xw[4] = {xv[c].x, xv[c].y, xv[c].z, xv[c].w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            acc[r] = fmaf(bf16_lo(xw[i]), wb[c][2 * i], acc[r]);
            acc[r] = fmaf(bf16_hi(xw[i]), wb[c][2 * i + 1], acc[r]);
          }
        }
      }
      k0 += kRoutePre * 256;
    }
#pragma unroll 2
    for (int k = k0; k < K; k += 256) chunk(GateChunk<WT>::load(wr, k), k);
#pragma unroll
    for (int r = 0; r < kRouteRows; ++r) {
      float v = acc[r];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      if (lane == 0 && r < nrows) {
        const float sg = 1.0f / (1.0f + expf(-v));
        st_shared_cluster_f32(map_shared_cta0(&s_sc[r][e]), sg);  // CTA 0's copy for the top-k
      }
    }
  }
  cluster_sync_all();  // every CTA's remote score stores are visible in CTA 0 (release / acquire)
  if (rank != 0) return;
  // The scores output is written from CTA 0's copy by the warps that select nothing, after the
  // barrier, so that the barrier's release does not wait for global stores (C3 R = 4: 36.3 -> 34.8 µs).
  if (warp >= nrows) {
    for (int i = (warp - nrows) * 32 + lane; i < nrows * E; i += (kRouteWarps - nrows) * 32)
      scores[static_cast<int64_t>(row0 + i / E) * E + i % E] = s_sc[i / E][i % E];
    return;
  }
  const int row = row0 + warp;
  if (E <= 128) route_select<4>(s_sc[warp], reinterpret_cast<const float(&)[4]>(bv), row, E, topk, scale, idx_out, w_out);
  else if (E <= 256) route_select<8>(s_sc[warp], reinterpret_cast<const float(&)[8]>(bv), row, E, topk, scale, idx_out, w_out);
  else route_select<16>(s_sc[warp], bv, row, E, topk, scale, idx_out, w_out);
}

// ---------------------------------------------------------------------------------------------
// MoeVerify phase counters: n ints zeroed by one small kernel that takes part in the programmatic
// dependent launch chain (a memset node would end it: the fused MoE kernel could then not be
// resident, its tables filled, before the router finishes).  It waits for its predecessor (the
// counters live in `out`, which the previous call's finalize wrote) and lets its dependent launch at
// once; the dependent's own wait then covers these stores.
// ---------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(128) moe_zero_kernel(int* __restrict__ p, int n) {
  pdl_launch_dependents();
  pdl_wait();
  for (int i = threadIdx.x; i < n; i += blockDim.x) p[i] = 0;
}

// ---------------------------------------------------------------------------------------------
// MoeVerify finalize: out[t, n] = bf16(sum_j w[t, j] * part[t*topk + j, n]), f32, j ascending
// (src/bolt_ops.cu:627-662).  Pairs whose expert id is out of range contribute nothing.
// ---------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) moe_finalize_kernel(const float* __restrict__ part, const float* __restrict__ w,
                                                           const int32_t* __restrict__ idx, int topk, int H, int E,
                                                           bf16* __restrict__ out) {
  pdl_wait();
  pdl_launch_dependents();
  const int t = blockIdx.x;
  for (int v = threadIdx.x; v < H / 4; v += blockDim.x) {
    float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
    // the partial rows are loaded together with the expert ids (not after them): one round trip
    constexpr int kPre = 8;
    float4 pv[kPre];
#pragma unroll
    for (int k = 0; k < kPre; ++k)
      pv[k] = k < topk ? __ldcg(reinterpret_cast<const float4*>(part + static_cast<int64_t>(t * topk + k) * H) + v)
                       : make_float4(0.f, 0.f, 0.f, 0.f);
    for (int k = 0; k < topk; ++k) {
      const int p = t * topk + k;
      const int e = __ldg(idx + p);
      if (e < 0 || e >= E) continue;
      const float wk = __ldg(w + p);
      float4 q = pv[0];
#pragma unroll
      for (int j = 1; j < kPre; ++j)
        if (k == j) q = pv[j];
      if (k >= kPre) q = __ldcg(reinterpret_cast<const float4*>(part + static_cast<int64_t>(p) * H) + v);
      a0 += wk * q.x;
      a1 += wk * q.y;
      a2 += wk * q.z;
      a3 += wk * q.w;
    }
    uint2 o;
    o.x = pack_bf16x2(a0, a1);
    o.y = pack_bf16x2(a2, a3);
    reinterpret_cast<uint2*>(out + static_cast<int64_t>(t) * H)[v] = o;
  }
}

// ---------------------------------------------------------------------------------------------
// Dequantise: one thread per (row, k-group); emulates the four quad lanes of the engine with the
// same decoders, then applies the post-MMA scale in fp32 (bit-identical to gguf-py).
// ---------------------------------------------------------------------------------------------
template <int F>
__global__ void __launch_bounds__(256) dequant_kernel(const uint8_t* __restrict__ w, float* __restrict__ out,
                                                      int64_t rows, int K, int row_bytes) {
  const int G = K / 32;
  const int64_t gid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (gid >= rows * G) return;
  const int64_t row = gid / G;
  const int grp = static_cast<int>(gid % G);
  const uint8_t* base = w + row * row_bytes;  // row starts are 2-byte aligned: realign below
  const uint8_t* abase = reinterpret_cast<const uint8_t*>(reinterpret_cast<uintptr_t>(base) & ~uintptr_t(3));
  const uint32_t mis = static_cast<uint32_t>(reinterpret_cast<uintptr_t>(base) & 3);
  float* o = out + row * K + grp * 32;
  if constexpr (F == kFmtQ8) {
    for (int t = 0; t < 4; ++t) {
      uint32_t a[4];
      float d;
      q8_decode_row<true>(abase, mis, grp, t, a, d);
      o[4 * t + 0] = bf16_lo(a[0]) * d;
      o[4 * t + 1] = bf16_hi(a[0]) * d;
      o[4 * t + 2] = bf16_lo(a[1]) * d;
      o[4 * t + 3] = bf16_hi(a[1]) * d;
      o[16 + 4 * t + 0] = bf16_lo(a[2]) * d;
      o[16 + 4 * t + 1] = bf16_hi(a[2]) * d;
      o[16 + 4 * t + 2] = bf16_lo(a[3]) * d;
      o[16 + 4 * t + 3] = bf16_hi(a[3]) * d;
    }
  } else if constexpr (F == kFmtIQ2) {
    const uint32_t sbo = mis + static_cast<uint32_t>(grp >> 3) * 66u;
    const uint2 q = ld_u64_a2_exact(abase, sbo + 2u + static_cast<uint32_t>(grp & 7) * 8u);
    const float d = fp16_bits_to_f32(ld_u16(abase, sbo));
    const float db = iq2_db(d, q.y);
    for (int t = 0; t < 4; ++t) {
      const uint32_t gi = (q.x >> (8 * t)) & 0xFFu;
      const uint4 mag = __ldg(reinterpret_cast<const uint4*>(&g_iq2_mag_bf16[gi][0]));
      uint32_t a[4];
      iq2_apply_signs(mag, q.y, 7u * t, a);
      for (int p = 0; p < 4; ++p) {
        o[8 * t + 2 * p] = bf16_lo(a[p]) * db;
        o[8 * t + 2 * p + 1] = bf16_hi(a[p]) * db;
      }
    }
  } else {
    const uint32_t bo = mis + static_cast<uint32_t>(grp >> 1) * 36u;
    const uint32_t h2 = static_cast<uint32_t>(grp & 1) * 2u;
    const uint32_t sc = ld_u16(abase, bo + h2);
    for (int s2 = 0; s2 < 2; ++s2) {
      const uint32_t S = fp4_scale_bf16_bits((sc >> (8 * s2)) & 0xFFu);
      const uint32_t Sx2 = S | (S << 16);
      for (int t = 0; t < 4; ++t) {
        const uint32_t v = ld_u16(abase, bo + 4u + (h2 + s2) * 8u + 2u * t);
        uint32_t lo, hi;
        fp4_patterns(v, lo, hi);
        lo = hmul2_bits(lo, Sx2);
        hi = hmul2_bits(hi, Sx2);
        float* os = o + 16 * s2;
        // E2M1 code 0x8 is a negative zero; gguf-py's table maps it to +0.0 (the GEMV sums are
        // unaffected, the dequantised bits are canonicalised here)
        auto z = [](float f, uint32_t nib) { return (nib & 7u) ? f : 0.0f; };
        os[2 * t] = z(bf16_lo(lo) * 65536.0f, v);
        os[2 * t + 1] = z(bf16_hi(lo) * 65536.0f, v >> 8);
        os[8 + 2 * t] = z(bf16_lo(hi) * 65536.0f, v >> 4);
        os[8 + 2 * t + 1] = z(bf16_hi(hi) * 65536.0f, v >> 12);
      }
    }
  }
}

// ---------------------------------------------------------------------------------------------
// Expert-parallel MoeVerify finalize (one CTA): this GPU's weighted partial sum over its own pairs
// (pairs whose expert lies in [offset, offset + E_local)), summed across the group through peer
// memory in rank order, rounded once to bf16.
// ---------------------------------------------------------------------------------------------
constexpr int kEpThreads = 1024;

__global__ void __launch_bounds__(kEpThreads) moe_finalize_ep_kernel(const float* __restrict__ part, const float* __restrict__ w,
                                                                   const int32_t* __restrict__ idx, int topk, int H,
                                                                   int E_local, int offset, int R, bf16* __restrict__ out,
                                                                   const PeerReduce pr) {
  pdl_wait();
  pdl_launch_dependents();
  __shared__ uint32_t s_epoch;
  if (threadIdx.x == 0) s_epoch = *reinterpret_cast<volatile uint32_t*>(pr.state) + 1u;
  __syncthreads();
  const uint32_t epoch = s_epoch;
  const int64_t par = static_cast<int64_t>(epoch & 1u) * pr.npeer;
  const int n4 = R * (H / 4);
  for (int i = threadIdx.x; i < n4; i += kEpThreads) {
    const int t = i / (H / 4), v = i % (H / 4);
    float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int k = 0; k < topk; ++k) {
      const int p = t * topk + k;
      const int e = __ldg(idx + p) - offset;
      if (e < 0 || e >= E_local) continue;
      const float wk = __ldg(w + p);
      const float4 pv = __ldcg(reinterpret_cast<const float4*>(part + static_cast<int64_t>(p) * H) + v);
      a.x += wk * pv.x;
      a.y += wk * pv.y;
      a.z += wk * pv.z;
      a.w += wk * pv.w;
    }
    const int64_t off = (par + pr.rank) * pr.slot_elems + static_cast<int64_t>(t) * H;
    for (int q = 0; q < pr.npeer; ++q) reinterpret_cast<float4*>(pr.slots[q] + off)[v] = a;
  }
  __syncthreads();
  if (threadIdx.x == 0) peer_reduce_sync(pr, epoch);
  __syncthreads();
  const float* mine = pr.slots[pr.rank];
  for (int i = threadIdx.x; i < n4; i += kEpThreads) {
    const int t = i / (H / 4), v = i % (H / 4);
    float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int q = 0; q < pr.npeer; ++q) {
      const float4 b = __ldcg(reinterpret_cast<const float4*>(mine + (par + q) * pr.slot_elems + static_cast<int64_t>(t) * H) + v);
      a.x += b.x;
      a.y += b.y;
      a.z += b.z;
      a.w += b.w;
    }
    uint2 o;
    o.x = pack_bf16x2(a.x, a.y);
    o.y = pack_bf16x2(a.z, a.w);
    reinterpret_cast<uint2*>(out + static_cast<int64_t>(t) * H)[v] = o;
  }
  if (threadIdx.x == 0) *reinterpret_cast<volatile uint32_t*>(pr.state) = epoch;
}

// ---------------------------------------------------------------------------------------------
// Q8Embed (src/bolt_ops.cu:1645-1690): out[r, k] = bf16(fp32(d) * q[k]) of row ids[r] of a GGUF Q8_0
// table [vocab, nb * 34]; ids outside [0, vocab) read row 0.  A warp handles 4 blocks (128
// elements) of one token: lane -> block lane / 8, elements 4 (lane % 8) .. + 3; the 8-byte outputs
// of a warp are contiguous (512 bytes).
// ---------------------------------------------------------------------------------------------
constexpr int kEmbedWarps = 8;

__global__ void __launch_bounds__(kEmbedWarps * 32) q8_embed_kernel(const uint8_t* __restrict__ w,
                                                                    const int64_t* __restrict__ ids, int64_t vocab,
                                                                    int nb, int64_t R, bf16* __restrict__ out) {
  pdl_wait();
  pdl_launch_dependents();
  const int lane = threadIdx.x & 31;
  const int64_t quads = (static_cast<int64_t>(nb) + 3) / 4;  // 4-block groups per token
  const int64_t total = R * quads;
  for (int64_t wi = static_cast<int64_t>(blockIdx.x) * kEmbedWarps + (threadIdx.x >> 5); wi < total;
       wi += static_cast<int64_t>(gridDim.x) * kEmbedWarps) {
    const int64_t r = wi / quads;
    const int b = static_cast<int>(wi % quads) * 4 + (lane >> 3);
    if (b >= nb) continue;
    int64_t tok = __ldg(ids + r);
    if (tok < 0 || tok >= vocab) tok = 0;
    const uint8_t* blk = w + (tok * nb + b) * 34;
    const int j = lane & 7;
    const float d = fp16_bits_to_f32(__ldg(reinterpret_cast<const uint16_t*>(blk)));
    // q bytes 4j..4j+3 start 2-byte aligned: two 16-bit loads
    const uint32_t qlo = __ldg(reinterpret_cast<const uint16_t*>(blk + 2 + 4 * j));
    const uint32_t qhi = __ldg(reinterpret_cast<const uint16_t*>(blk + 4 + 4 * j));
    const uint32_t q = qlo | (qhi << 16);
    const float v0 = d * static_cast<float>(static_cast<int8_t>(q & 0xFFu));
    const float v1 = d * static_cast<float>(static_cast<int8_t>((q >> 8) & 0xFFu));
    const float v2 = d * static_cast<float>(static_cast<int8_t>((q >> 16) & 0xFFu));
    const float v3 = d * static_cast<float>(static_cast<int8_t>(q >> 24));
    uint2 o;
    o.x = pack_bf16x2(v0, v1);
    o.y = pack_bf16x2(v2, v3);
    *reinterpret_cast<uint2*>(out + (r * nb + b) * 32 + 4 * j) = o;
  }
}

// Vector form for rows whose block count is a multiple of 8 (row_bytes a multiple of 272 = 17 x 16 B)
// and 16-byte aligned tensors.  Unit = one token x 8 blocks: 272 bytes in (17 lanes x 16 B), 256
// elements out (32 lanes x 16 B).  A warp loads kEmbedU units before decoding any (bytes in flight per
// SM = warps x kEmbedU x 272), stages them in its own shared slice and writes 512 contiguous bytes per
// unit.  Lane l decodes block l / 4, elements 8 (l % 4) .. + 7.  Few units (decode) take kEmbedU = 1
// so that every unit has its own warp.
template <int kEmbedU>
__global__ void __launch_bounds__(kEmbedWarps * 32) q8_embed_vec_kernel(const uint8_t* __restrict__ w,
                                                                        const int64_t* __restrict__ ids,
                                                                        int64_t vocab, int nb, int64_t R,
                                                                        bf16* __restrict__ out) {
  __shared__ __align__(16) uint8_t stage[kEmbedWarps][kEmbedU][272];
  pdl_wait();
  pdl_launch_dependents();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int gpr = nb >> 3;  // 8-block groups per row
  const int64_t units = R * gpr;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kEmbedWarps * kEmbedU;
  const int64_t row_bytes = static_cast<int64_t>(nb) * 34;
  for (int64_t u0 = (static_cast<int64_t>(blockIdx.x) * kEmbedWarps + warp) * kEmbedU; u0 < units; u0 += stride) {
    int64_t r = u0 / gpr;
    int g = static_cast<int>(u0 - r * gpr);
    uint4 v[kEmbedU];
#pragma unroll
    for (int i = 0; i < kEmbedU; ++i) {
      v[i] = make_uint4(0u, 0u, 0u, 0u);
      if (u0 + i < units && lane < 17) {
        int64_t tok = __ldg(ids + r);
        if (tok < 0 || tok >= vocab) tok = 0;
        v[i] = __ldg(reinterpret_cast<const uint4*>(w + tok * row_bytes + g * 272) + lane);
      }
      if (++g == gpr) g = 0, ++r;
    }
#pragma unroll
    for (int i = 0; i < kEmbedU; ++i)
      if (lane < 17) *reinterpret_cast<uint4*>(&stage[warp][i][lane * 16]) = v[i];
    __syncwarp();
    const int b = lane >> 2, j = lane & 3;
#pragma unroll
    for (int i = 0; i < kEmbedU; ++i) {
      if (u0 + i >= units) break;
      const uint8_t* sb = &stage[warp][i][34 * b];
      const float d = fp16_bits_to_f32(*reinterpret_cast<const uint16_t*>(sb));
      const uint16_t* q16 = reinterpret_cast<const uint16_t*>(sb + 2 + 8 * j);
      const uint32_t qa = q16[0] | (static_cast<uint32_t>(q16[1]) << 16);
      const uint32_t qb = q16[2] | (static_cast<uint32_t>(q16[3]) << 16);
      uint4 o;
      o.x = pack_bf16x2(d * static_cast<float>(static_cast<int8_t>(qa & 0xFFu)),
                        d * static_cast<float>(static_cast<int8_t>((qa >> 8) & 0xFFu)));
      o.y = pack_bf16x2(d * static_cast<float>(static_cast<int8_t>((qa >> 16) & 0xFFu)),
                        d * static_cast<float>(static_cast<int8_t>(qa >> 24)));
      o.z = pack_bf16x2(d * static_cast<float>(static_cast<int8_t>(qb & 0xFFu)),
                        d * static_cast<float>(static_cast<int8_t>((qb >> 8) & 0xFFu)));
      o.w = pack_bf16x2(d * static_cast<float>(static_cast<int8_t>((qb >> 16) & 0xFFu)),
                        d * static_cast<float>(static_cast<int8_t>(qb >> 24)));
      *reinterpret_cast<uint4*>(out + (u0 + i) * 256 + lane * 8) = o;
    }
    __syncwarp();
  }
}

// ---------------------------------------------------------------------------------------------
// Relu2 (src/bolt_ops.cu:700-726): y = bf16(r * r), r = fmaxf(x, 0) in fp32 (NaN -> 0 through fmaxf).
// kVec: 8 elements per thread with 16-byte loads / stores (aligned tensors), tail elementwise.
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ float relu2_f(float v) {
  const float r = fmaxf(v, 0.f);
  return __fmul_rn(r, r);
}

template <bool kVec>
__global__ void __launch_bounds__(256) relu2_kernel(const bf16* __restrict__ x, bf16* __restrict__ y, int64_t n) {
  pdl_wait();
  pdl_launch_dependents();
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int64_t t0 = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if constexpr (kVec) {
    const int64_t n8 = n / 8;
    for (int64_t i = t0; i < n8; i += stride) {
      const uint4 v = ldg128(x + 8 * i);
      uint4 o;
      o.x = pack_bf16x2(relu2_f(bf16_lo(v.x)), relu2_f(bf16_hi(v.x)));
      o.y = pack_bf16x2(relu2_f(bf16_lo(v.y)), relu2_f(bf16_hi(v.y)));
      o.z = pack_bf16x2(relu2_f(bf16_lo(v.z)), relu2_f(bf16_hi(v.z)));
      o.w = pack_bf16x2(relu2_f(bf16_lo(v.w)), relu2_f(bf16_hi(v.w)));
      *reinterpret_cast<uint4*>(y + 8 * i) = o;
    }
    for (int64_t i = 8 * n8 + t0; i < n; i += stride) y[i] = __float2bfloat16(relu2_f(__bfloat162float(x[i])));
  } else {
    for (int64_t i = t0; i < n; i += stride) y[i] = __float2bfloat16(relu2_f(__bfloat162float(x[i])));
  }
}

}  // namespace gguf_b200
