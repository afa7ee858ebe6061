// RmsNorm / SkipRmsNorm (src/bolt_ops.cu:1692-1864):
//   v   = x                         (RmsNorm)
//   v   = bf16(x + skip)            (SkipRmsNorm; v is also the optional second output `sum`)
//   y   = bf16( (bf16(gamma) * v) * rsqrt(mean(v^2) + eps) )
// bf16 activations [R, H], fp32 gamma [H] rounded to bf16 (ORT SimplifiedLayerNorm's weight type).
//
// Canonical fp32 order of mean(v^2), shared by every kernel that normalises a row (the standalone
// op here and GEMV prologues): the row is cut into 8-element chunks; "virtual thread" t of 512 owns
// chunks t, t + 512, t + 1024, ... and accumulates acc = fma(v * (1/H), v, acc) over them in
// element order; the 512 partials are summed by a 32-lane butterfly inside each of 16 groups of 32
// consecutive t, then a 16-lane butterfly over the group sums.  A kernel with 512 threads maps
// thread t onto virtual thread t, so results are bit-identical wherever the row is normalised.
#pragma once

#include "common.cuh"

namespace gguf_b200 {

constexpr int kNormThreads = 512;

// Sum over the 512 threads of a CTA in the canonical butterfly order; every thread gets the total.
// red: 16 floats of shared memory; two barriers.
__device__ __forceinline__ float norm_block_sum(float acc, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  float v = red[threadIdx.x & 15];
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();  // red may be reused after this
  return v;
}

// Adds 8 bf16 values (one uint4) into the canonical accumulator.
__device__ __forceinline__ float norm_accumulate(float acc, uint4 v, float rld) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float a = bf16_lo(w[i]), b = bf16_hi(w[i]);
    acc = __fmaf_rn(__fmul_rn(a, rld), a, acc);
    acc = __fmaf_rn(__fmul_rn(b, rld), b, acc);
  }
  return acc;
}

// bf16(x + s) per element (round to nearest even), 8 at a time.
__device__ __forceinline__ uint4 bf16x8_add(uint4 a, uint4 b) {
  uint4 r;
  const uint32_t* pa = &a.x;
  const uint32_t* pb = &b.x;
  uint32_t* pr = &r.x;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __nv_bfloat162 s = __hadd2(*reinterpret_cast<const __nv_bfloat162*>(pa + i),
                               *reinterpret_cast<const __nv_bfloat162*>(pb + i));
    pr[i] = *reinterpret_cast<uint32_t*>(&s);
  }
  return r;
}

// 8 gamma values rounded to bf16 (kept as fp32).
struct Gamma8 {
  float g[8];
};
__device__ __forceinline__ Gamma8 load_gamma8(const float* gamma, int chunk) {
  const float4 a = __ldg(reinterpret_cast<const float4*>(gamma) + 2 * chunk);
  const float4 b = __ldg(reinterpret_cast<const float4*>(gamma) + 2 * chunk + 1);
  return Gamma8{{round_bf16(a.x), round_bf16(a.y), round_bf16(a.z), round_bf16(a.w), round_bf16(b.x),
                 round_bf16(b.y), round_bf16(b.z), round_bf16(b.w)}};
}

// y chunk = bf16((g * v) * rs).
__device__ __forceinline__ uint4 norm_scale8(uint4 v, const Gamma8& g, float rs) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  uint32_t o[4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
    o[i] = pack_bf16x2(__fmul_rn(__fmul_rn(g.g[2 * i], bf16_lo(w[i])), rs),
                       __fmul_rn(__fmul_rn(g.g[2 * i + 1], bf16_hi(w[i])), rs));
  return make_uint4(o[0], o[1], o[2], o[3]);
}

// One CTA of 512 threads per row (rows grid-strided).  kNC > 0: each thread keeps its kNC chunks in
// registers (H <= 4096 kNC); kNC == 0: any H, second pass re-reads v (from sum when it was written).
// gamma does not depend on the preceding kernel: with kNC > 0 it is loaded before pdl_wait.
template <bool kSkip, int kNC>
__global__ void __launch_bounds__(kNormThreads, 2) rms_norm_kernel(const bf16* __restrict__ x,
                                                                const bf16* __restrict__ skip,
                                                                const float* __restrict__ gamma, float eps, int H,
                                                                int64_t R, bf16* __restrict__ y,
                                                                bf16* __restrict__ sum) {
  __shared__ float red[16];
  const int t = threadIdx.x;
  const int nchunk = H >> 3;
  const float rld = 1.0f / static_cast<float>(H);
  constexpr int kRegs = kNC > 0 ? kNC : 1;
  Gamma8 g[kRegs];
  if constexpr (kNC > 0) {
#pragma unroll
    for (int c = 0; c < kNC; ++c)
      if (t + c * kNormThreads < nchunk) g[c] = load_gamma8(gamma, t + c * kNormThreads);
  }
  pdl_wait();
  pdl_launch_dependents();
  for (int64_t r = blockIdx.x; r < R; r += gridDim.x) {
    const bf16* xr = x + r * H;
    float acc = 0.f;
    if constexpr (kNC > 0) {
      uint4 v[kNC];
#pragma unroll
      for (int c = 0; c < kNC; ++c) {
        const int ch = t + c * kNormThreads;
        if (ch < nchunk) {
          v[c] = ldg128(xr + ch * 8);
          if constexpr (kSkip) {
            v[c] = bf16x8_add(v[c], ldg128(skip + r * H + ch * 8));
            if (sum) *reinterpret_cast<uint4*>(sum + r * H + ch * 8) = v[c];
          }
          acc = norm_accumulate(acc, v[c], rld);
        }
      }
      const float rs = rsqrtf(norm_block_sum(acc, red) + eps);
#pragma unroll
      for (int c = 0; c < kNC; ++c) {
        const int ch = t + c * kNormThreads;
        if (ch < nchunk) *reinterpret_cast<uint4*>(y + r * H + ch * 8) = norm_scale8(v[c], g[c], rs);
      }
    } else {
      for (int ch = t; ch < nchunk; ch += kNormThreads) {
        uint4 v = ldg128(xr + ch * 8);
        if constexpr (kSkip) {
          v = bf16x8_add(v, ldg128(skip + r * H + ch * 8));
          if (sum) *reinterpret_cast<uint4*>(sum + r * H + ch * 8) = v;
        }
        acc = norm_accumulate(acc, v, rld);
      }
      const float rs = rsqrtf(norm_block_sum(acc, red) + eps);
      for (int ch = t; ch < nchunk; ch += kNormThreads) {
        uint4 v;
        if (kSkip && sum) {
          v = *reinterpret_cast<const uint4*>(sum + r * H + ch * 8);  // written by this thread above
        } else {
          v = ldg128(xr + ch * 8);
          if constexpr (kSkip) v = bf16x8_add(v, ldg128(skip + r * H + ch * 8));
        }
        *reinterpret_cast<uint4*>(y + r * H + ch * 8) = norm_scale8(v, load_gamma8(gamma, ch), rs);
      }
    }
  }
}

}  // namespace gguf_b200
