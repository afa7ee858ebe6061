// MambaStep / MambaVerify (+ the GGUF variants with fp32 conv weights), src/bolt_ops.cu:68-378:
// one decode (or speculative-verify) step of a Mamba-2 mixer after its input projection.
//
//   proj row  = [gate (di) | xBC (cd = di + 2 ng ds) | dt (heads)]              bf16
//   conv      : act[r][c] = bf16(silu(b[c] + sum_j w[c][j] * in[r + j])), in = [3 state taps, xBC rows]
//   ssm       : dt = max(softplus(dt_raw + dt_bias), tmin); per (head, n, p):
//               s = s * exp(A dt) + (dt x[p]) B[n];  y[p] += C[n] s        (fp32 state [heads, ds, hd])
//   ypre      = y + D x;   out = bf16(v * rsqrt(mean_group(v^2) + eps) * norm_w),  v = ypre * silu(gate)
// Step: the state after the last row replaces the state; Verify: the step starts from row *state_row
// of [Rs, ...] state buffers and the state after token r is written to row r.
//
// B200 design: one CTA per head runs the conv of the channels it needs (its 64 x channels and its
// group's 128 B and 128 C channels, computed by every head of the group and stored by the group's
// first head), keeps the activations in shared memory and runs the state recurrence with the head's
// 32 KB of state in registers (thread (p, q) owns n in [32q, 32q + 32) of column p); a second kernel
// (programmatic dependent launch) applies the gated group norm.  fp32 order: explicit fma chains
// (conv: b + w0 i0 + w1 i1 + w2 i2 + w3 i3 left to right; state: fma(s, dA, dt x B)); the norm sums
// squares per thread, then a fixed butterfly.
#pragma once

#include "common.cuh"

namespace gguf_b200 {

constexpr int kMambaHD = 64, kMambaDS = 128, kMambaMaxRows = 16, kMambaThreads = 256;

struct MambaArgs {
  const bf16* proj;
  int R, proj_stride, di, cd, heads, hpg, ng;
  const bf16* conv_in;   // [Rs, cd, 3]
  const void* conv_w;    // [cd, 4] bf16 or fp32
  const void* conv_b;    // [cd]
  bf16* conv_out;        // [Rs, cd, 3] (step: [1, cd, 3])
  bf16* xbc;             // [R, cd]
  const float* ssm_in;   // [Rs, heads, ds, hd]
  const float* dt_bias;  // [heads]
  const float* a_neg;    // [heads]
  const float* d_skip;   // [heads]
  float tmin;
  float* ssm_out;
  float* ypre;           // [R, di]
  const int32_t* state_row;  // verify: device int32 (row of the input state), else null
  int state_rows;
};

__device__ __forceinline__ float silu_f(float v) { return v / (1.0f + expf(-v)); }

template <bool kF32W>
__device__ __forceinline__ void conv_weights(const MambaArgs& a, int c, float (&w)[4], float& b) {
  if constexpr (kF32W) {  // GGUF: fp32 weights rounded to bf16, as the bf16 op sees them
    const float4 v = __ldg(reinterpret_cast<const float4*>(a.conv_w) + c);
    w[0] = round_bf16(v.x), w[1] = round_bf16(v.y), w[2] = round_bf16(v.z), w[3] = round_bf16(v.w);
    b = round_bf16(__ldg(reinterpret_cast<const float*>(a.conv_b) + c));
  } else {
    const uint2 v = __ldg(reinterpret_cast<const uint2*>(a.conv_w) + c);
    w[0] = bf16_lo(v.x), w[1] = bf16_hi(v.x), w[2] = bf16_lo(v.y), w[3] = bf16_hi(v.y);
    b = __bfloat162float(reinterpret_cast<const bf16*>(a.conv_b)[c]);
  }
}

template <bool kF32W>
__global__ void __launch_bounds__(kMambaThreads) mamba_conv_ssm_kernel(const __grid_constant__ MambaArgs a) {
  __shared__ float sX[kMambaMaxRows][kMambaHD];
  __shared__ float sB[kMambaMaxRows][kMambaDS];
  __shared__ float sC[kMambaMaxRows][kMambaDS];
  __shared__ float sPart[kMambaMaxRows][4][kMambaHD];
  __shared__ float sDt[kMambaMaxRows];
  const int h = blockIdx.x, g = h / a.hpg, tid = threadIdx.x;
  const bool group_owner = (h % a.hpg) == 0;
  const bool verify = a.state_row != nullptr;
  const int R = a.R;
  pdl_wait();
  pdl_launch_dependents();
  int row = 0;
  if (verify) {
    row = *a.state_row;
    if (row < 0 || row >= a.state_rows) {
      if (tid == 0 && h == 0) record_device_error(kSiteBadStateRow);
      row = 0;
    }
  }
  const bf16* cin = a.conv_in + static_cast<int64_t>(row) * a.cd * 3;
  // The head's state does not depend on the conv: its loads are in flight during the conv phase.
  const int p = tid & (kMambaHD - 1), q = tid >> 6;
  const int64_t row_stride = static_cast<int64_t>(a.heads) * kMambaDS * kMambaHD;
  const int64_t head_off = (static_cast<int64_t>(h) * kMambaDS + q * 32) * kMambaHD + p;
  const float* sp = a.ssm_in + static_cast<int64_t>(row) * row_stride + head_off;
  float st[32];
#pragma unroll
  for (int n = 0; n < 32; ++n) st[n] = __ldcs(sp + n * kMambaHD);

  // ---- conv of this head's 64 x channels and its group's 128 B + 128 C channels ----
  for (int i = tid; i < kMambaHD + 2 * kMambaDS; i += kMambaThreads) {
    int c;
    bool store;
    if (i < kMambaHD) {
      c = h * kMambaHD + i;
      store = true;
    } else if (i < kMambaHD + kMambaDS) {
      c = a.di + g * kMambaDS + (i - kMambaHD);
      store = group_owner;
    } else {
      c = a.di + a.ng * kMambaDS + g * kMambaDS + (i - kMambaHD - kMambaDS);
      store = group_owner;
    }
    float w[4], b;
    conv_weights<kF32W>(a, c, w, b);
    float in[3 + kMambaMaxRows];
    in[0] = __bfloat162float(cin[c * 3 + 0]);
    in[1] = __bfloat162float(cin[c * 3 + 1]);
    in[2] = __bfloat162float(cin[c * 3 + 2]);
#pragma unroll
    for (int r = 0; r < kMambaMaxRows; ++r)
      if (r < R) in[3 + r] = __bfloat162float(a.proj[static_cast<int64_t>(r) * a.proj_stride + a.di + c]);
#pragma unroll
    for (int r = 0; r < kMambaMaxRows; ++r) {
      if (r >= R) break;
      float acc = __fmaf_rn(w[0], in[r], b);
      acc = __fmaf_rn(w[1], in[r + 1], acc);
      acc = __fmaf_rn(w[2], in[r + 2], acc);
      acc = __fmaf_rn(w[3], in[r + 3], acc);
      const bf16 act = __float2bfloat16(silu_f(acc));
      const float af = __bfloat162float(act);
      if (i < kMambaHD) sX[r][i] = af;
      else if (i < kMambaHD + kMambaDS) sB[r][i - kMambaHD] = af;
      else sC[r][i - kMambaHD - kMambaDS] = af;
      if (store) {
        a.xbc[static_cast<int64_t>(r) * a.cd + c] = act;
        // the 3 taps after token r: every row's in Verify, the last row's in Step (constant
        // indices into `in`, so it stays in registers)
        if (verify || r == R - 1) {
          bf16* o = a.conv_out + (static_cast<int64_t>(verify ? r : 0) * a.cd + c) * 3;
          o[0] = __float2bfloat16(in[r + 1]);
          o[1] = __float2bfloat16(in[r + 2]);
          o[2] = __float2bfloat16(in[r + 3]);
        }
      }
    }
  }
  if (tid < R) {
    const float raw = __bfloat162float(a.proj[static_cast<int64_t>(tid) * a.proj_stride + a.di + a.cd + h]) +
                      __ldg(a.dt_bias + h);
    const float dt = raw > 20.0f ? raw : log1pf(expf(raw));
    sDt[tid] = fmaxf(dt, a.tmin);
  }
  __syncthreads();

  // ---- state recurrence: thread (p, q) owns state[h][32q .. 32q + 31][p] ----
  const float A = __ldg(a.a_neg + h), D = __ldg(a.d_skip + h);
  for (int r = 0; r < R; ++r) {
    const float dt = sDt[r];
    const float dA = expf(A * dt);
    const float dtx = dt * sX[r][p];
    float acc = 0.f;
#pragma unroll
    for (int n = 0; n < 32; ++n) {
      st[n] = __fmaf_rn(st[n], dA, __fmul_rn(dtx, sB[r][q * 32 + n]));
      acc = __fmaf_rn(sC[r][q * 32 + n], st[n], acc);
    }
    sPart[r][q][p] = acc;
    if (verify) {
      float* o = a.ssm_out + r * row_stride + head_off;
#pragma unroll
      for (int n = 0; n < 32; ++n) o[n * kMambaHD] = st[n];
    }
  }
  if (!verify) {
    float* o = a.ssm_out + head_off;
#pragma unroll
    for (int n = 0; n < 32; ++n) o[n * kMambaHD] = st[n];
  }
  __syncthreads();
  for (int i = tid; i < R * kMambaHD; i += kMambaThreads) {
    const int r = i / kMambaHD, pp = i % kMambaHD;
    float sum = D * sX[r][pp];
#pragma unroll
    for (int qq = 0; qq < 4; ++qq) sum += sPart[r][qq][pp];
    a.ypre[static_cast<int64_t>(r) * a.di + h * kMambaHD + pp] = sum;
  }
}

// Gated group norm: grid (R, ng), 256 threads; v = ypre * silu(gate), y = bf16(v * rs * norm_w).
__global__ void __launch_bounds__(256) mamba_norm_kernel(const bf16* __restrict__ proj, int proj_stride, int di,
                                                         int group_size, float eps, const float* __restrict__ ypre,
                                                         const float* __restrict__ norm_w, bf16* __restrict__ y) {
  __shared__ float red[8];
  const int r = blockIdx.x, g = blockIdx.y, tid = threadIdx.x;
  const int64_t base = static_cast<int64_t>(r) * di + static_cast<int64_t>(g) * group_size;
  const bf16* gate = proj + static_cast<int64_t>(r) * proj_stride + static_cast<int64_t>(g) * group_size;
  pdl_wait();
  pdl_launch_dependents();
  float ss = 0.f;
  for (int i = tid; i < group_size; i += 256) {
    const float gt = __bfloat162float(gate[i]);
    const float v = ypre[base + i] * silu_f(gt);
    ss = __fmaf_rn(v, v, ss);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((tid & 31) == 0) red[tid >> 5] = ss;
  __syncthreads();
  float tot = red[tid & 7];
#pragma unroll
  for (int o = 4; o > 0; o >>= 1) tot += __shfl_xor_sync(0xffffffffu, tot, o);
  const float rs = rsqrtf(tot / static_cast<float>(group_size) + eps);
  for (int i = tid; i < group_size; i += 256) {
    const float gt = __bfloat162float(gate[i]);
    const float v = ypre[base + i] * silu_f(gt);
    y[base + i] = __float2bfloat16(v * rs * __ldg(norm_w + static_cast<int64_t>(g) * group_size + i));
  }
}

}  // namespace gguf_b200
