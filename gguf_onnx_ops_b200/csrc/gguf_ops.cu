// libgguf_onnx_ops: C ABI (include/gguf_ops.h) over the sm_100a GGUF decode kernels.
//
// Host responsibilities per call: validate the op contract (same constraints and messages as
// the reference ops in src/bolt_ops.cu), pick the staging plan of the engine, and enqueue the
// kernels on the caller's stream with cudaLaunchKernelEx (programmatic dependent launch
// attribute on by default).  No allocation, no synchronisation.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "../../include/gguf_ops.h"
#include "engine.cuh"
#include "slice_r1.cuh"
#include "slice_iq2_i8.cuh"
#include "slice_iq2_i8_rows.cuh"
#include "slice_q8_i8_rows.cuh"
#include "slice_fp4_rows.cuh"
#include "slice_fp4_i8.cuh"
#include "iq2_rowblock.cuh"
#include "moe_fused.cuh"
#include "small_kernels.cuh"
#include "rms_norm.cuh"
#include "mamba.cuh"

namespace gguf_b200 {

namespace {

thread_local std::string t_last_error;
std::atomic<int> g_pdl{1};
std::atomic<int> g_fast{1};  // specialised kernels (R = 1 paths); 0 forces the generic engine

int fail(int code, const std::string& msg) {
  t_last_error = msg;
  return code;
}
int cuda_fail(const char* op, cudaError_t e) { return fail(GGUF_ERR_CUDA, std::string(op) + ": " + cudaGetErrorString(e)); }

constexpr int kKW = 16;                     // consumer warps per CTA
constexpr int kThreads = (kKW + 1) * 32;    // + 1 producer warp
constexpr int kSmemBudget = 112 * 1024;     // <= half an SM: two kernels' CTAs can co-reside
constexpr int kSmemBudgetMax = 220 * 1024;  // fallback for very long rows
constexpr int kStageTarget = 20 * 1024;

struct DeviceInfo {
  int sms = 0;
};
DeviceInfo g_dev[64];

int current_sms(int* sms) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail("cudaGetDevice", e);
  if (dev < 0 || dev >= 64) return fail(GGUF_ERR_CUDA, "device ordinal out of range");
  if (g_dev[dev].sms == 0) {
    int n = 0;
    e = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return cuda_fail("cudaDeviceGetAttribute", e);
    g_dev[dev].sms = n;
  }
  *sms = g_dev[dev].sms;
  return GGUF_OK;
}

// Raises the dynamic shared-memory limit of `fn` once per device.
template <typename Fn>
int ensure_smem(Fn fn, size_t bytes, std::atomic<uint64_t>& done_mask) {
  int dev = 0;
  cudaGetDevice(&dev);
  const uint64_t bit = 1ull << (dev & 63);
  if (done_mask.load() & bit) return GGUF_OK;
  cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBudgetMax);
  if (e != cudaSuccess) return cuda_fail("cudaFuncSetAttribute", e);
  (void)bytes;
  done_mask.fetch_or(bit);
  return GGUF_OK;
}

// resident = true: a cooperative launch, for persistent kernels whose CTAs wait on one another (the
// runtime starts all CTAs together, or fails the launch if they cannot all be resident at once,
// instead of starting some while others stay queued behind kernels of other streams).
constexpr bool kMoeResident = true;
template <typename... KArgs, typename... Args>
cudaError_t launch_ex(bool resident, void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                      Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (g_pdl.load()) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  if (resident) {
    attr[na].id = cudaLaunchAttributeCooperative;
    attr[na].val.cooperative = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}
template <typename... KArgs, typename... Args>
cudaError_t launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args&&... args) {
  return launch_ex(false, kernel, grid, block, smem, s, std::forward<Args>(args)...);
}

// ---------------------------------------------------------------------------------------------
// Staging plan
// ---------------------------------------------------------------------------------------------
template <int F>
int make_plan(EngineArgs& a, int K, int row_bytes, int NT, bool moe, size_t* smem_out) {
  using Fi = FmtInfo<F>;
  a.K = K;
  a.row_bytes = row_bytes;
  const int lut = (F == kFmtIQ2 || F == kFmtIQ2N) ? 256 * 8 * 16 : ((F == kFmtFP4 || F == kFmtFP4S) ? 512 : 0);
  const int red = kKW * NT * 128 * 4;
  const int grp = moe ? (4 * kMaxPairs + kMaxPairs * 8 + 4) * 4 : 0;
  bool seg = (row_bytes % 16 == 0) && (K % Fi::kSeg == 0);
  int kc = K;
  if (seg) {
    // largest multiple of kSeg dividing K whose 16-row stage stays near kStageTarget
    kc = Fi::kSeg;
    for (int c = Fi::kSeg; c <= K; c += Fi::kSeg) {
      if (K % c) continue;
      if (16 * (c / Fi::kBlock * Fi::kBytes) <= kStageTarget || c == Fi::kSeg) kc = c;
    }
  }
  a.kc = kc;
  a.nsplit = K / kc;
  a.seg_bytes = kc / Fi::kBlock * Fi::kBytes;
  if (seg) {
    // padded row stride: 16-byte multiple with stride/4 == 4 (mod 8) words, so the 8 rows a warp
    // touches per load start in 8 different 4-bank groups.
    int st = (a.seg_bytes + 15) & ~15;
    if (st % 32 == 0) st += 16;
    a.stride = st;
    a.contiguous = 0;
  } else {
    a.stride = row_bytes;
    a.contiguous = 1;
  }
  a.stage_bytes = ((16 * a.stride + 16) + 127) & ~127;  // +16: unaligned-read overrun pad
  if constexpr (Fi::kScDiv > 0) {  // split layout: the stage's scale slab follows the weights
    a.sc_row_bytes = K / Fi::kScDiv;
    a.sc_seg_bytes = kc / Fi::kScDiv;
    a.sc_off = (16 * a.stride + 16 + 127) & ~127;  // TMA destination: 128-byte aligned
    const int slab = 16 * (a.contiguous ? a.sc_row_bytes : a.sc_seg_bytes) + 16;
    a.stage_bytes = ((a.sc_off + slab) + 127) & ~127;
  }
  const int fixed = lut + red + grp + 2 * 8 * 8 + 256;
  int budget = kSmemBudget;
  int stages = (budget - fixed) / a.stage_bytes;
  if (stages < 2) {
    budget = kSmemBudgetMax;
    stages = (budget - fixed) / a.stage_bytes;
  }
  if (stages < 1) return fail(GGUF_ERR_INVALID_ARGUMENT, "K too large for the shared-memory staging plan");
  a.stages = std::min(stages, 8);
  size_t off = (lut + 127) & ~127;
  a.off_stage = static_cast<int>(off);
  off += static_cast<size_t>(a.stages) * a.stage_bytes;
  a.off_red = static_cast<int>(off);
  off += red;
  off = (off + 15) & ~size_t(15);
  a.off_bar = static_cast<int>(off);
  off += 2 * a.stages * 8;
  a.off_grp = static_cast<int>(off);
  off += grp;
  *smem_out = off;
  return GGUF_OK;
}

bool aligned(const void* p, uintptr_t n) { return (reinterpret_cast<uintptr_t>(p) % n) == 0; }

// cuTensorMapEncodeTiled from the driver (no link-time dependency on libcuda).
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      p = nullptr;
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }();
  return fn;
}

// Segmented engine staging through a 2-D tensor map (see EngineArgs::tmap): rows_total rows of
// row_bytes (a multiple of 16) starting at a.w, boxes of 16 rows x a.stride bytes.  Leaves the
// per-row copies in place when the plan or the driver does not allow it.
void attach_tensor_map(EngineArgs& a, int64_t rows_total, bool split = false) {
  a.use_tmap = 0;
  if (a.contiguous || a.stride > 2048 || a.stride % 16 || a.row_bytes % 16 || a.seg_bytes % 16) return;
  auto enc = tensor_map_encoder();
  if (!enc) return;
  if (split) {  // the scale slab rides on a second map; without it both use per-row copies
    if (a.sc_row_bytes % 16 || a.sc_seg_bytes % 16 || a.sc_seg_bytes > 256) return;
    cuuint64_t sdims[2] = {static_cast<cuuint64_t>(a.sc_row_bytes), static_cast<cuuint64_t>(rows_total)};
    cuuint64_t sstride[1] = {static_cast<cuuint64_t>(a.sc_row_bytes)};
    cuuint32_t sbox[2] = {static_cast<cuuint32_t>(a.sc_seg_bytes), 16u};
    cuuint32_t ses[2] = {1u, 1u};
    if (enc(&a.smap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(a.sc), sdims, sstride, sbox, ses,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return;
  }
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(a.row_bytes / 8), static_cast<cuuint64_t>(rows_total)};
  cuuint64_t gstride[1] = {static_cast<cuuint64_t>(a.row_bytes)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(a.stride / 8), 16u};
  cuuint32_t estride[2] = {1u, 1u};
  const CUresult r = enc(&a.tmap, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<uint8_t*>(a.w), dims, gstride, box,
                         estride, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r == CUDA_SUCCESS) a.use_tmap = 1;
}

template <int F, int NT>
int run_dense(const void* x, const void* w, const float* gscale, void* y, int R, int N, int K, cudaStream_t s,
              const PeerOut* po = nullptr) {
  EngineArgs a = {};
  if (po) a.po = *po;
  size_t smem = 0;
  int rc = make_plan<F>(a, K, K / FmtInfo<F>::kBlock * FmtInfo<F>::kBytes, NT, false, &smem);
  if (rc) return rc;
  a.w = static_cast<const uint8_t*>(w);
  a.rows = N;
  a.tiles = (N + 15) / 16;
  attach_tensor_map(a, N);
  a.x = static_cast<const bf16*>(x);
  a.R = R;
  a.y = y;
  a.gscale = gscale;
  a.post = F == kFmtFP4 ? 65536.0f : 1.0f;
  int sms = 0;
  if ((rc = current_sms(&sms))) return rc;
  static std::atomic<uint64_t> done{0};
  auto kern = engine_kernel<F, NT, kKW, kModeDense>;
  if ((rc = ensure_smem(kern, smem, done))) return rc;
  // two CTAs per SM (engine_kernel launch bounds); row-split: the group's CTA count
  const int grid = a.po.npeer ? a.po.ctas : std::min(a.tiles, 2 * sms);
  cudaError_t e = launch(kern, dim3(grid), dim3(kThreads), smem, s, a);
  if (e != cudaSuccess) return cuda_fail("gemv launch", e);
  return GGUF_OK;
}

// Split (legacy) layouts on the engine: weights w [N, K/32 * kBytes], scales sc [N, K/kScDiv].
template <int F, int NT>
int run_dense_split(const void* x, const void* w, const void* sc, const float* gscale, void* y, int R, int N, int K,
                    cudaStream_t s) {
  EngineArgs a = {};
  size_t smem = 0;
  int rc = make_plan<F>(a, K, K / 32 * FmtInfo<F>::kBytes, NT, false, &smem);
  if (rc) return rc;
  a.w = static_cast<const uint8_t*>(w);
  a.sc = static_cast<const uint8_t*>(sc);
  a.rows = N;
  a.tiles = (N + 15) / 16;
  attach_tensor_map(a, N, true);
  a.x = static_cast<const bf16*>(x);
  a.R = R;
  a.y = y;
  a.gscale = gscale;
  a.post = F == kFmtFP4S ? 65536.0f : 1.0f;
  int sms = 0;
  if ((rc = current_sms(&sms))) return rc;
  static std::atomic<uint64_t> done{0};
  auto kern = engine_kernel<F, NT, kKW, kModeDense>;
  if ((rc = ensure_smem(kern, smem, done))) return rc;
  // two CTAs per SM (engine_kernel launch bounds); row-split: the group's CTA count
  const int grid = a.po.npeer ? a.po.ctas : std::min(a.tiles, 2 * sms);
  cudaError_t e = launch(kern, dim3(grid), dim3(kThreads), smem, s, a);
  if (e != cudaSuccess) return cuda_fail("legacy-layout gemv launch", e);
  return GGUF_OK;
}

// One activation row: slice kernel (slice_r1.cuh), K = 256 * kW * kSPW, rows 16-byte multiples.
template <int F, int kW, int kSPW>
int run_slice_r1(const void* x, const void* w, const float* gscale, void* y, int N, int K, cudaStream_t s,
                 const PeerOut* po = nullptr) {
  SliceArgs a = {};
  if (po) a.po = *po;
  a.w = static_cast<const uint8_t*>(w);
  a.x = static_cast<const bf16*>(x);
  a.gscale = gscale;
  a.y = static_cast<bf16*>(y);
  a.N = N;
  a.K = K;
  a.row_bytes = K / FmtInfo<F>::kBlock * FmtInfo<F>::kBytes;
  a.tiles = (N + 15) / 16;
  int st = (a.row_bytes + 15) & ~15;
  if (st % 32 == 0) st += 16;
  a.stride = st;
  a.stage_bytes = ((16 * st + 32) + 127) & ~127;  // +32: unaligned-window overrun pad
  const int lut = (SliceFmt<F>::kLut + 127) & ~127, red = 2 * kW * 16 * 4;
  a.stages = std::min(8, (kSmemBudgetMax - lut - red - 256) / a.stage_bytes);
  if (a.stages < 2) return -1;  // does not fit: the caller falls back to the engine
  a.off_stage = lut;
  a.off_red = lut + a.stages * a.stage_bytes;
  a.off_bar = a.off_red + red;
  const size_t smem = a.off_bar + 2 * a.stages * 8;
  int sms = 0, rc;
  if ((rc = current_sms(&sms))) return rc;
  static std::atomic<uint64_t> done{0};
  auto kern = slice_r1_kernel<F, kW, kSPW>;
  if ((rc = ensure_smem(kern, smem, done))) return rc;
  const int grid = a.po.npeer ? a.po.ctas : std::min(a.tiles, sms);  // row-split: the group's CTA count
  cudaError_t e = launch(kern, dim3(grid), dim3((kW + 1) * 32), smem, s, a);
  if (e != cudaSuccess) return cuda_fail("single-row GEMV launch", e);
  return GGUF_OK;
}

// IQ2_XXS R = 1 on the integer tensor cores (slice_iq2_i8.cuh); same staging plan as run_slice_r1.
// NVFP4 R = 1 on the integer tensor cores (slice_fp4_i8.cuh): K = 128 * kW * kSPW.
template <int kW, int kSPW>
int run_slice_fp4_i8(const void* x, const void* w, const float* gscale, void* y, int N, int K, cudaStream_t s) {
  SliceArgs a = {};
  a.w = static_cast<const uint8_t*>(w);
  a.x = static_cast<const bf16*>(x);
  a.gscale = gscale;
  a.y = static_cast<bf16*>(y);
  a.N = N;
  a.K = K;
  a.row_bytes = K / 64 * 36;  // K % 128 == 0: a multiple of 8 words
  a.tiles = (N + 15) / 16;
  a.stride = a.row_bytes + ((32 - a.row_bytes % 128) + 128) % 128;  // pitch = 32 mod 128 bytes
  a.stage_bytes = ((16 * a.stride) + 127) & ~127;
  const int red_per_stage = kW * 16 * 4 + 4;
  a.stages = std::min(8, (kSmemBudgetMax - 256) / (a.stage_bytes + red_per_stage + 16));
  if (a.stages < 2) return fail(GGUF_ERR_INVALID_ARGUMENT, "K too large for the single-row staging plan");
  a.off_stage = 0;
  a.off_red = a.stages * a.stage_bytes;
  a.off_bar = (a.off_red + a.stages * red_per_stage + 15) & ~15;
  const size_t smem = a.off_bar + 2 * a.stages * 8;
  int sms = 0, rc;
  if ((rc = current_sms(&sms))) return rc;
  static std::atomic<uint64_t> done{0};
  auto kern = slice_fp4_i8_kernel<kW, kSPW>;
  if ((rc = ensure_smem(kern, smem, done))) return rc;
  cudaError_t e = launch(kern, dim3(std::min(a.tiles, sms)), dim3(kW * 32), smem, s, a);
  if (e != cudaSuccess) return cuda_fail("single-row NVFP4 GEMV launch", e);
  return GGUF_OK;
}

// IQ2_XXS whole-tile staging (slice_iq2_i8.cuh, slice_iq2_i8_rows.cuh): rows land at pitch
// a.stride.  With the row bytes a multiple of 32, rows g and g+4 would share shared-memory banks in
// the eight-quad record loads; then the tile comes as one 2-D tensor box of 16 rows x (row bytes +
// 16) (the pad past the row end zero-filled), else as one bulk copy at pitch = row bytes.
void attach_slice_tmap(SliceArgs& a) {
  a.stride = a.row_bytes;
  a.use_tmap = 0;
  if (a.row_bytes % 32 != 0 || a.row_bytes / 8 + 2 > 256) return;
  auto enc = tensor_map_encoder();
  if (!enc) return;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(a.row_bytes / 8), static_cast<cuuint64_t>(a.N)};
  cuuint64_t gstride[1] = {static_cast<cuuint64_t>(a.row_bytes)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(a.row_bytes / 8 + 2), 16u};
  cuuint32_t estride[2] = {1u, 1u};
  if (enc(&a.tmap, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<uint8_t*>(a.w), dims, gstride, box, estride,
          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return;
  a.use_tmap = 1;
  a.stride = a.row_bytes + 16;
}

struct FusedNorm {  // optional (Skip)RmsNorm prologue of the single-row IQ2_XXS GEMV
  const float* gamma;
  const void* skip;
  void* x_norm_out;
  void* sum_out;
  float eps;
};

template <int kW>
int run_slice_iq2_i8(const void* x, const void* w, void* y, int N, int K, cudaStream_t s,
                     const FusedNorm* norm = nullptr) {
  SliceArgs a = {};
  if (norm) {
    a.gamma = norm->gamma;
    a.skip = static_cast<const bf16*>(norm->skip);
    a.x_norm_out = static_cast<bf16*>(norm->x_norm_out);
    a.sum_out = static_cast<bf16*>(norm->sum_out);
    a.eps = norm->eps;
  }
  a.w = static_cast<const uint8_t*>(w);
  a.x = static_cast<const bf16*>(x);
  a.y = static_cast<bf16*>(y);
  a.N = N;
  a.K = K;
  a.row_bytes = K / 256 * 66;
  a.tiles = (N + 15) / 16;
  attach_slice_tmap(a);  // whole-tile copies (rows at pitch a.stride)
  a.stage_bytes = ((16 * a.stride + 32) + 127) & ~127;  // +32: unaligned-window overrun pad
  const int red_per_stage = kW * 16 * 4 + 4;  // reduction slot + counter
  a.stages = std::min(8, (kSmemBudgetMax - kI8Lut - 256) / (a.stage_bytes + red_per_stage + 16));
  if (a.stages < 2) return fail(GGUF_ERR_INVALID_ARGUMENT, "K too large for the single-row staging plan");
  a.off_stage = kI8Lut;
  a.off_red = kI8Lut + a.stages * a.stage_bytes;
  a.off_bar = (a.off_red + a.stages * red_per_stage + 15) & ~15;
  const size_t smem = a.off_bar + 2 * a.stages * 8;
  int sms = 0, rc;
  if ((rc = current_sms(&sms))) return rc;
  static std::atomic<uint64_t> done{0};
  auto kern = slice_iq2_i8_kernel<kW>;
  if ((rc = ensure_smem(kern, smem, done))) return rc;
  cudaError_t e = launch(kern, dim3(std::min(a.tiles, sms)), dim3(kW * 32), smem, s, a);
  if (e != cudaSuccess) return cuda_fail("single-row GEMV launch", e);
  return GGUF_OK;
}

// IQ2_XXS 2 <= R <= 4 * kNR on the integer tensor cores (slice_iq2_i8_rows.cuh), the single-row
// kernel's staging plan with a reduction slot per activation row.
template <int kW, int kNR>
int run_slice_iq2_i8_rows(const void* x, const void* w, void* y, int R, int N, int K, cudaStream_t s) {
  SliceArgs a = {};
  a.w = static_cast<const uint8_t*>(w);
  a.x = static_cast<const bf16*>(x);
  a.y = static_cast<bf16*>(y);
  a.R = R;
  a.N = N;
  a.K = K;
  a.row_bytes = K / 256 * 66;
  a.tiles = (N + 15) / 16;
  attach_slice_tmap(a);
  a.stage_bytes = ((16 * a.stride + 32) + 127) & ~127;  // +32: unaligned-window overrun pad
  const int red_per_stage = kW * 4 * kNR * 16 * 4 + 4;  // reduction slot + counter
  a.stages = std::min(8, (kSmemBudgetMax - kI8Lut - 256) / (a.stage_bytes + red_per_stage + 16));
  if (a.stages < 2) return -1;  // does not fit: the caller falls back to the engine
  a.off_stage = kI8Lut;
  a.off_red = kI8Lut + a.stages * a.stage_bytes;
  a.off_bar = (a.off_red + a.stages * red_per_stage + 15) & ~15;
  const size_t smem = a.off_bar + 2 * a.stages * 8;
  int sms = 0, rc;
  if ((rc = current_sms(&sms))) return rc;
  static std::atomic<uint64_t> done{0};
  auto kern = slice_iq2_i8_rows_kernel<kW, kNR>;
  if ((rc = ensure_smem(kern, smem, done))) return rc;
  cudaError_t e = launch(kern, dim3(std::min(a.tiles, sms)), dim3(kW * 32), smem, s, a);
  if (e != cudaSuccess) return cuda_fail("few-row GEMV launch", e);
  return GGUF_OK;
}

// Dispatches 2 <= R <= 8 IQ2_XXS to the few-row integer kernel when K allows it (R > 4, a second MMA
// set on the same decoded tile: K = 4096 only, 17.5 against the engine's 18.2-18.5 µs at C1); -1
// otherwise.
int try_iq2_rows(const void* x, const void* w, void* y, int R, int N, int K, cudaStream_t s) {
  if (g_fast.load() != 1 || R < 2 || R > 8) return -1;
  if (R > 4) return K == 4096 ? run_slice_iq2_i8_rows<16, 2>(x, w, y, R, N, K, s) : -1;
  switch (K) {
    case 2048: return run_slice_iq2_i8_rows<8, 1>(x, w, y, R, N, K, s);
    case 4096: return run_slice_iq2_i8_rows<16, 1>(x, w, y, R, N, K, s);
    case 5120: return run_slice_iq2_i8_rows<20, 1>(x, w, y, R, N, K, s);
    default: return -1;
  }
}

// Q8_0 2 <= R <= 4 * kNR on the integer tensor cores (slice_q8_i8_rows.cuh): 16 whole rows per
// stage at pitch row bytes + 16, two or more stages.
template <int kW, int kNR, int kSPW = 1>
int run_slice_q8_i8_rows(const void* x, const void* w, void* y, int R, int N, int K, cudaStream_t s,
                         const PeerOut* po) {
  SliceArgs a = {};
  if (po) a.po = *po;
  a.w = static_cast<const uint8_t*>(w);
  a.x = static_cast<const bf16*>(x);
  a.y = static_cast<bf16*>(y);
  a.R = R;
  a.N = N;
  a.K = K;
  a.row_bytes = K / 32 * 34;  // K % 256 == 0: a multiple of 16
  a.tiles = (N + 15) / 16;
  a.stride = a.row_bytes + 16;
  a.stage_bytes = (16 * a.stride + 127) & ~127;
  const int red_per_stage = kW * 4 * kNR * 16 * 4 + 4;  // reduction slot + counter
  a.stages = std::min(4, (kSmemBudgetMax - 256) / (a.stage_bytes + red_per_stage + 16));
  if (a.stages < 2) return -1;  // does not fit: the caller falls back to the engine
  a.off_stage = 0;
  a.off_red = a.stages * a.stage_bytes;
  a.off_bar = (a.off_red + a.stages * red_per_stage + 15) & ~15;
  const size_t smem = a.off_bar + 2 * a.stages * 8;
  int sms = 0, rc;
  if ((rc = current_sms(&sms))) return rc;
  static std::atomic<uint64_t> done{0};
  auto kern = slice_q8_i8_rows_kernel<kW, kNR, kSPW>;
  if ((rc = ensure_smem(kern, smem, done))) return rc;
  const int grid = a.po.npeer ? a.po.ctas : std::min(a.tiles, sms);  // row-split: the group's CTA count
  cudaError_t e = launch(kern, dim3(grid), dim3(kW * 32), smem, s, a);
  if (e != cudaSuccess) return cuda_fail("few-row Q8_0 GEMV launch", e);
  return GGUF_OK;
}

// Dispatches 1 <= R <= 16 Q8_0 to the few-row integer kernel when K allows it (R > 8: K = 4096
// only); -1 otherwise.  One row uses four-row MMA columns with three empty rows: the quants need
// no decode, so the kernel is HBM-bound at large N even so (C4 R = 1: 91 µs, 0.96 of peak, where
// the bf16 slice kernel took 115 µs).  R > 8 runs 8 warps of two slices each: 256 threads leave
// each thread the 255 registers that four MMA sets for two slices need (16 warps capped at 128
// spilled), and the reduction slots stay small (C4 R = 16: 153 µs against 185 with 16 warps).
int try_q8_rows(const void* x, const void* w, void* y, int R, int N, int K, cudaStream_t s,
                const PeerOut* po = nullptr) {
  if (g_fast.load() != 1 || R < 1 || R > 16) return -1;
  if (R > 8) return K == 4096 ? run_slice_q8_i8_rows<8, 4, 2>(x, w, y, R, N, K, s, po) : -1;
  const bool two = R > 4;
  switch (K) {
    case 2048: return two ? run_slice_q8_i8_rows<8, 2>(x, w, y, R, N, K, s, po) : run_slice_q8_i8_rows<8, 1>(x, w, y, R, N, K, s, po);
    case 4096: return two ? run_slice_q8_i8_rows<8, 2, 2>(x, w, y, R, N, K, s, po) : run_slice_q8_i8_rows<16, 1>(x, w, y, R, N, K, s, po);
    case 5120: return two ? run_slice_q8_i8_rows<20, 2>(x, w, y, R, N, K, s, po) : run_slice_q8_i8_rows<20, 1>(x, w, y, R, N, K, s, po);
    default: return -1;
  }
}

// Q8Gemv gguf=0 (split layout: u8 q + 128 [N, K], bf16 scales [N, K/32]) through the few-row Q8
// kernel: 16 weight rows per stage at pitch K + 32 (conflict-free 8-byte quant loads), the tile's 16
// scale rows (contiguous in the scale tensor) after them, one bulk copy each.
template <int kW, int kNR, int kSPW = 1, int kLay = kLayQ8S>
int run_slice_q8s_rows(const void* x, const void* w, const void* scales, void* y, int R, int N, int K, cudaStream_t s) {
  SliceArgs a = {};
  a.w = static_cast<const uint8_t*>(w);
  a.sc = static_cast<const uint8_t*>(scales);
  a.x = static_cast<const bf16*>(x);
  a.y = static_cast<bf16*>(y);
  a.R = R;
  a.N = N;
  a.K = K;
  a.row_bytes = kLay == kLayQ4S ? K / 2 : K;
  a.sc_row_bytes = K / 16;  // K % 256 == 0: a multiple of 16
  a.tiles = (N + 15) / 16;
  a.stride = a.row_bytes + (kLay == kLayQ4S ? 16 : 32);  // row words = 4 (Q4: 32-bit loads) / 8 (8-byte loads) mod 32
  a.sc_off = 16 * a.stride;
  a.stage_bytes = (a.sc_off + 16 * a.sc_row_bytes + 127) & ~127;
  const int red_per_stage = kW * 4 * kNR * 16 * 4 + 4;  // reduction slot + counter
  a.stages = std::min(4, (kSmemBudgetMax - 256) / (a.stage_bytes + red_per_stage + 16));
  if (a.stages < 2) return -1;
  a.off_stage = 0;
  a.off_red = a.stages * a.stage_bytes;
  a.off_bar = (a.off_red + a.stages * red_per_stage + 15) & ~15;
  const size_t smem = a.off_bar + 2 * a.stages * 8;
  int sms = 0, rc;
  if ((rc = current_sms(&sms))) return rc;
  static std::atomic<uint64_t> done{0};
  auto kern = slice_q8_i8_rows_kernel<kW, kNR, kSPW, kLay>;
  if ((rc = ensure_smem(kern, smem, done))) return rc;
  cudaError_t e = launch(kern, dim3(std::min(a.tiles, sms)), dim3(kW * 32), smem, s, a);
  if (e != cudaSuccess) return cuda_fail("few-row Q8Gemv gguf=0 launch", e);
  return GGUF_OK;
}

// Q4Gemv iq2=0 (split nibbles n - 8, bf16 scales per 32) on the same kernel, R <= 4 (a second MMA
// set with the offset sums spills registers: R > 4 stays on the engine).
int try_q4s_rows(const void* x, const void* w, const void* scales, void* y, int R, int N, int K, cudaStream_t s) {
  if (g_fast.load() != 1 || R < 1 || R > 4) return -1;
  switch (K) {
    case 2048: return run_slice_q8s_rows<8, 1, 1, kLayQ4S>(x, w, scales, y, R, N, K, s);
    case 4096: return run_slice_q8s_rows<16, 1, 1, kLayQ4S>(x, w, scales, y, R, N, K, s);
    case 5120: return run_slice_q8s_rows<20, 1, 1, kLayQ4S>(x, w, scales, y, R, N, K, s);
    default: return -1;
  }
}

int try_q8s_rows(const void* x, const void* w, const void* scales, void* y, int R, int N, int K, cudaStream_t s) {
  if (g_fast.load() != 1 || R < 1 || R > 16) return -1;
  if (R > 8) return K == 4096 ? run_slice_q8s_rows<8, 4, 2>(x, w, scales, y, R, N, K, s) : -1;
  const bool two = R > 4;
  switch (K) {
    case 2048: return two ? run_slice_q8s_rows<8, 2>(x, w, scales, y, R, N, K, s) : run_slice_q8s_rows<8, 1>(x, w, scales, y, R, N, K, s);
    case 4096: return two ? run_slice_q8s_rows<8, 2, 2>(x, w, scales, y, R, N, K, s) : run_slice_q8s_rows<16, 1>(x, w, scales, y, R, N, K, s);
    case 5120: return two ? run_slice_q8s_rows<20, 2>(x, w, scales, y, R, N, K, s) : run_slice_q8s_rows<20, 1>(x, w, scales, y, R, N, K, s);
    default: return -1;
  }
}

// Tiles per SM from which the few-row NVFP4 kernel takes f16 operands (slice_fp4_rows.cuh, kF16).
constexpr int kFp4F16MinRounds = 4;

// NVFP4 2 <= R <= 8 kNB on the f16 / bf16 tensor cores with the activation rows as MMA columns
// (slice_fp4_rows.cuh): 16 whole rows per stage at pitch row bytes + 32; with kNB = 2 the second
// set of 8 rows is packed into 4 KB of shared memory per warp, ahead of the stages.
template <int kW, int kNB = 1>
int run_slice_fp4_rows(const void* x, const void* w, const float* gscale, void* y, int R, int N, int K, cudaStream_t s) {
  SliceArgs a = {};
  a.w = static_cast<const uint8_t*>(w);
  a.x = static_cast<const bf16*>(x);
  a.gscale = gscale;
  a.y = static_cast<bf16*>(y);
  a.R = R;
  a.N = N;
  a.K = K;
  a.row_bytes = K / 64 * 36;  // K % 256 == 0: a multiple of 16
  a.tiles = (N + 15) / 16;
  a.stride = a.row_bytes + 32;  // row words = 8 or 24 mod 32 for K = 2048, 4096, 5120
  a.stage_bytes = (16 * a.stride + 127) & ~127;
  const int lut = 512, red_per_stage = kW * 8 * kNB * 16 * 4 + 4, xs2 = kNB == 2 ? kW * 16 * 32 * 8 : 0;
  a.stages = std::min(4, (kSmemBudgetMax - lut - xs2 - 256) / (a.stage_bytes + red_per_stage + 16));
  if (a.stages < 2) return -1;
  a.off_x2 = lut;
  a.off_stage = lut + xs2;
  a.off_red = a.off_stage + a.stages * a.stage_bytes;
  a.off_bar = (a.off_red + a.stages * red_per_stage + 15) & ~15;
  const size_t smem = a.off_bar + 2 * a.stages * 8;
  int sms = 0, rc;
  if ((rc = current_sms(&sms))) return rc;
  static std::atomic<uint64_t> done{0}, done16{0};
  // f16 operands for one activation set when the launch is long enough to repay their x prologue
  const bool f16 = kNB == 1 && a.tiles >= kFp4F16MinRounds * sms;
  auto kern = f16 ? slice_fp4_rows_kernel<kW, false, kNB, kNB == 1> : slice_fp4_rows_kernel<kW, false, kNB, false>;
  if ((rc = ensure_smem(kern, smem, f16 ? done16 : done))) return rc;
  cudaError_t e = launch(kern, dim3(std::min(a.tiles, sms)), dim3(kW * 32), smem, s, a);
  if (e != cudaSuccess) return cuda_fail("few-row NVFP4 GEMV launch", e);
  return GGUF_OK;
}

template <int F>
int try_slice_r1(const void* x, const void* w, const float* gscale, void* y, int N, int K, cudaStream_t s);

// Nvfp4Gemv gguf=0 (split: nibbles [N, K/2], e4m3fn scales [N, K/16]) on the few-row NVFP4 kernel,
// 2 <= R <= 8: 16 weight rows at pitch K/2 + 32 (conflict-free 8-byte nibble loads), the tile's 16
// scale rows after them.
template <int kW>
int run_slice_fp4s_rows(const void* x, const void* w, const void* scales, const float* gscale, void* y, int R, int N,
                        int K, cudaStream_t s) {
  SliceArgs a = {};
  a.w = static_cast<const uint8_t*>(w);
  a.sc = static_cast<const uint8_t*>(scales);
  a.x = static_cast<const bf16*>(x);
  a.gscale = gscale;
  a.y = static_cast<bf16*>(y);
  a.R = R;
  a.N = N;
  a.K = K;
  a.row_bytes = K / 2;
  a.sc_row_bytes = K / 16;  // K % 256 == 0: a multiple of 16
  a.tiles = (N + 15) / 16;
  a.stride = a.row_bytes + 32;
  a.sc_off = 16 * a.stride;
  a.stage_bytes = (a.sc_off + 16 * a.sc_row_bytes + 127) & ~127;
  const int lut = 512, red_per_stage = kW * 8 * 16 * 4 + 4;
  a.stages = std::min(4, (kSmemBudgetMax - lut - 256) / (a.stage_bytes + red_per_stage + 16));
  if (a.stages < 2) return -1;
  a.off_stage = lut;
  a.off_red = lut + a.stages * a.stage_bytes;
  a.off_bar = (a.off_red + a.stages * red_per_stage + 15) & ~15;
  const size_t smem = a.off_bar + 2 * a.stages * 8;
  int sms = 0, rc;
  if ((rc = current_sms(&sms))) return rc;
  static std::atomic<uint64_t> done{0}, done16{0};
  const bool f16 = a.tiles >= kFp4F16MinRounds * sms;
  auto kern = f16 ? slice_fp4_rows_kernel<kW, true, 1, true> : slice_fp4_rows_kernel<kW, true, 1, false>;
  if ((rc = ensure_smem(kern, smem, f16 ? done16 : done))) return rc;
  cudaError_t e = launch(kern, dim3(std::min(a.tiles, sms)), dim3(kW * 32), smem, s, a);
  if (e != cudaSuccess) return cuda_fail("few-row Nvfp4Gemv gguf=0 launch", e);
  return GGUF_OK;
}

int try_fp4s_rows(const void* x, const void* w, const void* scales, const float* gscale, void* y, int R, int N, int K,
                  cudaStream_t s) {
  if (g_fast.load() != 1 || R < 2 || R > 8) return -1;
  switch (K) {
    case 2048: return run_slice_fp4s_rows<8>(x, w, scales, gscale, y, R, N, K, s);
    case 4096: return run_slice_fp4s_rows<16>(x, w, scales, gscale, y, R, N, K, s);
    case 5120: return run_slice_fp4s_rows<20>(x, w, scales, gscale, y, R, N, K, s);
    default: return -1;
  }
}

// Dispatches 2 <= R <= 16 NVFP4 to the few-row kernel when K allows it (R > 8: one launch with two
// activation sets, or, where that plan does not fit shared memory, two launches for rows 0..7 and
// 8..R-1, each streaming the weights once); -1 otherwise.
int try_fp4_rows(const void* x, const void* w, const float* gscale, void* y, int R, int N, int K, cudaStream_t s) {
  if (g_fast.load() != 1 || R < 2 || R > 16) return -1;
  if (K != 2048 && K != 4096 && K != 5120) return -1;
  if (R > 8) {
    // one launch, each decoded weight fragment feeding both activation sets
    const int r2 = K == 2048 ? run_slice_fp4_rows<8, 2>(x, w, gscale, y, R, N, K, s)
                             : (K == 4096 ? run_slice_fp4_rows<16, 2>(x, w, gscale, y, R, N, K, s)
                                          : run_slice_fp4_rows<20, 2>(x, w, gscale, y, R, N, K, s));
    if (r2 >= 0) return r2;
    const int rc = try_fp4_rows(x, w, gscale, y, 8, N, K, s);
    if (rc != GGUF_OK) return rc;
    const bf16* x8 = static_cast<const bf16*>(x) + static_cast<int64_t>(8) * K;
    bf16* y8 = static_cast<bf16*>(y) + static_cast<int64_t>(8) * N;
    return R - 8 == 1 ? try_slice_r1<kFmtFP4>(x8, w, gscale, y8, N, K, s) : try_fp4_rows(x8, w, gscale, y8, R - 8, N, K, s);
  }
  switch (K) {
    case 2048: return run_slice_fp4_rows<8>(x, w, gscale, y, R, N, K, s);
    case 4096: return run_slice_fp4_rows<16>(x, w, gscale, y, R, N, K, s);
    case 5120: return run_slice_fp4_rows<20>(x, w, gscale, y, R, N, K, s);
    default: return -1;
  }
}

// IQ2_XXS R = 1, 16-row blocks owned by warp pairs (iq2_rowblock.cuh).  Returns -1 when the shape
// does not fit its plan (K % 512, one stage of every pair in shared memory).
int run_iq2_rowblock(const void* x, const void* w, void* y, int N, int K, cudaStream_t s) {
  if (K % 512 != 0) return -1;
  RowBlockArgs a = {};
  a.w = static_cast<const uint8_t*>(w);
  a.x = static_cast<const bf16*>(x);
  a.y = static_cast<bf16*>(y);
  a.N = N;
  a.K = K;
  a.row_bytes = K / 256 * 66;
  a.blocks = (N + 15) / 16;
  a.stage_bytes = ((16 * a.row_bytes + 32) + 127) & ~127;  // +32: unaligned-window overrun pad
  const int slices = K / 256;
  const int xbytes = slices * 512 + slices * 8 * 8 + 64;
  a.off_x = kI8Lut;
  a.off_stage = (a.off_x + xbytes + 127) & ~127;
  a.off_red = a.off_stage + kRbPairs * a.stage_bytes;
  a.off_bar = a.off_red + kRbPairs * 16 * 4;
  const size_t smem = a.off_bar + kRbPairs * 8;
  if (smem > static_cast<size_t>(kSmemBudgetMax)) return -1;
  int sms = 0, rc;
  if ((rc = current_sms(&sms))) return rc;
  static std::atomic<uint64_t> done{0};
  auto kern = iq2_rowblock_kernel;
  if ((rc = ensure_smem(kern, smem, done))) return rc;
  cudaError_t e = launch(kern, dim3(sms), dim3(kRbWarps * 32), smem, s, a);
  if (e != cudaSuccess) return cuda_fail("single-row GEMV launch", e);
  return GGUF_OK;
}

// Dispatches R = 1 to the slice kernel when K and the row size allow it; returns -1 otherwise.
template <int F>
int try_slice_r1(const void* x, const void* w, const float* gscale, void* y, int N, int K, cudaStream_t s) {
  const int fast = g_fast.load();
  if (!fast || (K / FmtInfo<F>::kBlock * FmtInfo<F>::kBytes) % 16 != 0) return -1;
  if (F == kFmtIQ2 && fast == 3) return run_iq2_rowblock(x, w, y, N, K, s);
  if (F == kFmtIQ2 && fast == 1) {
    switch (K) {
      case 2048: return run_slice_iq2_i8<8>(x, w, y, N, K, s);
      case 4096: return run_slice_iq2_i8<16>(x, w, y, N, K, s);
      case 5120: return run_slice_iq2_i8<20>(x, w, y, N, K, s);
      default: return -1;
    }
  }
  if (F == kFmtFP4 && fast == 4) {  // integer-decode variant (cross-check / comparison)
    switch (K) {
      case 2048: return run_slice_fp4_i8<16, 1>(x, w, gscale, y, N, K, s);
      case 4096: return run_slice_fp4_i8<16, 2>(x, w, gscale, y, N, K, s);
      case 5120: return run_slice_fp4_i8<20, 2>(x, w, gscale, y, N, K, s);
      case 6144: return run_slice_fp4_i8<16, 3>(x, w, gscale, y, N, K, s);
      case 8192: return run_slice_fp4_i8<16, 4>(x, w, gscale, y, N, K, s);
      default: break;
    }
  }
  switch (K) {
    case 2048: return run_slice_r1<F, 8, 1>(x, w, gscale, y, N, K, s);
    case 4096: return run_slice_r1<F, 16, 1>(x, w, gscale, y, N, K, s);
    case 5120: return run_slice_r1<F, 20, 1>(x, w, gscale, y, N, K, s);
    case 6144: return F == kFmtFP4 ? run_slice_r1<F, 12, 2>(x, w, gscale, y, N, K, s) : -1;
    case 8192: return F == kFmtFP4 ? run_slice_r1<F, 16, 2>(x, w, gscale, y, N, K, s) : -1;
    default: return -1;
  }
}

// Row-split shard: Q8_0 through the few-row integer kernel (any R it takes; R = 1 at K = 2048 stays
// on the bf16 slice kernel as in gguf_q8_0_gemv), else the bf16 slice kernel for R = 1 (K in its
// instantiated set), else the engine.
template <int F>
int run_rowsplit(const void* x, const void* w, const float* gscale, int R, int rows, int K, cudaStream_t s,
                 const PeerOut& po) {
  if (F == kFmtQ8 && !(R == 1 && K == 2048)) {
    const int rc = try_q8_rows(x, w, nullptr, R, rows, K, s, &po);
    if (rc >= 0) return rc;
  }
  const bool slice_ok = R == 1 && (K / FmtInfo<F>::kBlock * FmtInfo<F>::kBytes) % 16 == 0;
  if (slice_ok) {
    switch (K) {
      case 2048: return run_slice_r1<F, 8, 1>(x, w, gscale, nullptr, rows, K, s, &po);
      case 4096: return run_slice_r1<F, 16, 1>(x, w, gscale, nullptr, rows, K, s, &po);
      case 5120: return run_slice_r1<F, 20, 1>(x, w, gscale, nullptr, rows, K, s, &po);
      default: break;
    }
  }
  return R <= 8 ? run_dense<F, 1>(x, w, gscale, nullptr, R, rows, K, s, &po)
                : run_dense<F, 2>(x, w, gscale, nullptr, R, rows, K, s, &po);
}

std::string dims(int64_t R, int64_t N, int64_t K) {
  char b[128];
  snprintf(b, sizeof(b), " (got R=%lld N=%lld K=%lld)", (long long)R, (long long)N, (long long)K);
  return b;
}

bool int_range(int64_t v) { return v > 0 && v < (1ll << 31); }

}  // namespace

// Error channel shared with the host-only translation units (gguf_file.cc).
int set_error(int code, const std::string& msg) { return fail(code, msg); }
void clear_error() { t_last_error.clear(); }

}  // namespace gguf_b200

using namespace gguf_b200;

extern "C" {

const char* gguf_version(void) { return "gguf_onnx_ops_b200 0.1 (sm_100a)"; }

const char* gguf_last_error(void) { return t_last_error.c_str(); }

void gguf_set_pdl(int enable) { g_pdl.store(enable ? 1 : 0); }

void gguf_set_fast_paths(int enable) { g_fast.store(enable < 0 ? 0 : (enable > 4 ? 1 : enable)); }

int gguf_q8_0_gemv(const void* x, const void* w, void* y, int64_t R, int64_t N, int64_t K, void* stream) {
  t_last_error.clear();
  if (!x || !w || !y) return fail(GGUF_ERR_INVALID_ARGUMENT, "Q8Gemv gguf=1: null tensor pointer");
  if (K <= 0 || K % 64 != 0 || R < 1 || R > 16 || !int_range(N) || !int_range(K))
    return fail(GGUF_ERR_INVALID_ARGUMENT, "Q8Gemv gguf=1: needs B [N, (K/32)*34], K % 64 == 0 and 1..16 rows" + dims(R, N, K));
  if (!aligned(w, 16) || !aligned(x, 16)) return fail(GGUF_ERR_INVALID_ARGUMENT, "Q8Gemv gguf=1: x and w must be 16-byte aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  {  // R = 1 at K = 2048: the bf16 slice kernel (more warps per SM than the 8 of the few-row kernel)
    const int rc = (R == 1 && K == 2048) ? try_slice_r1<kFmtQ8>(x, w, nullptr, y, (int)N, (int)K, s)
                                         : try_q8_rows(x, w, y, (int)R, (int)N, (int)K, s);
    if (rc >= 0) return rc;
  }
  if (R == 1) {
    const int rc = try_slice_r1<kFmtQ8>(x, w, nullptr, y, (int)N, (int)K, s);
    if (rc >= 0) return rc;
  }
  return R <= 8 ? run_dense<kFmtQ8, 1>(x, w, nullptr, y, (int)R, (int)N, (int)K, s)
                : run_dense<kFmtQ8, 2>(x, w, nullptr, y, (int)R, (int)N, (int)K, s);
}

int gguf_iq2_xxs_gemv(const void* x, const void* w, void* y, int64_t R, int64_t N, int64_t K, void* stream) {
  t_last_error.clear();
  if (!x || !w || !y) return fail(GGUF_ERR_INVALID_ARGUMENT, "Q4Gemv iq2=3: null tensor pointer");
  if (K <= 0 || K % 256 != 0 || R < 1 || R > 16 || !int_range(N) || !int_range(K))
    return fail(GGUF_ERR_INVALID_ARGUMENT, "Q4Gemv iq2=3: needs B [N, (K/256)*66], K % 256 == 0 and 1..16 rows" + dims(R, N, K));
  if (!aligned(w, 16) || !aligned(x, 16)) return fail(GGUF_ERR_INVALID_ARGUMENT, "Q4Gemv iq2=3: x and w must be 16-byte aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (R == 1) {
    const int rc = try_slice_r1<kFmtIQ2>(x, w, nullptr, y, (int)N, (int)K, s);
    if (rc >= 0) return rc;
  } else {
    const int rc = try_iq2_rows(x, w, y, (int)R, (int)N, (int)K, s);
    if (rc >= 0) return rc;
  }
  return R <= 8 ? run_dense<kFmtIQ2, 1>(x, w, nullptr, y, (int)R, (int)N, (int)K, s)
                : run_dense<kFmtIQ2, 2>(x, w, nullptr, y, (int)R, (int)N, (int)K, s);
}

int gguf_nvfp4_gemv(const void* x, const void* w, const float* gscale, void* y, int64_t R, int64_t N, int64_t K,
                    void* stream) {
  t_last_error.clear();
  if (!x || !w || !y || !gscale) return fail(GGUF_ERR_INVALID_ARGUMENT, "Nvfp4Gemv gguf=1: null tensor pointer");
  if (K <= 0 || K % 64 != 0 || R < 1 || R > 16 || !int_range(N) || !int_range(K))
    return fail(GGUF_ERR_INVALID_ARGUMENT, "Nvfp4Gemv gguf=1: needs w [N, (K/64)*36], K % 64 == 0 and 1..16 rows" + dims(R, N, K));
  if (!aligned(w, 16) || !aligned(x, 16) || !aligned(gscale, 4))
    return fail(GGUF_ERR_INVALID_ARGUMENT, "Nvfp4Gemv gguf=1: x and w must be 16-byte aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (R == 1) {
    const int rc = try_slice_r1<kFmtFP4>(x, w, gscale, y, (int)N, (int)K, s);
    if (rc >= 0) return rc;
  } else {
    const int rc = try_fp4_rows(x, w, gscale, y, (int)R, (int)N, (int)K, s);
    if (rc >= 0) return rc;
  }
  return R <= 8 ? run_dense<kFmtFP4, 1>(x, w, gscale, y, (int)R, (int)N, (int)K, s)
                : run_dense<kFmtFP4, 2>(x, w, gscale, y, (int)R, (int)N, (int)K, s);
}

extern "C++" {
namespace gguf_b200 {
namespace {
template <typename WT>
int run_route(const char* op, const void* x, const WT* gate_w, const float* bias, int32_t* idx, float* weights,
              float* scores, int64_t R, int64_t K, int64_t E, int64_t topk, float scale, void* stream) {
  t_last_error.clear();
  if (!x || !gate_w || !bias || !idx || !weights || !scores)
    return fail(GGUF_ERR_INVALID_ARGUMENT, std::string(op) + ": null tensor pointer");
  if (E < 1 || E > 512 || K <= 0 || K % 256 != 0 || topk < 1 || topk > 32 || topk > E || R < 1 || R > (1 << 24))
    return fail(GGUF_ERR_INVALID_ARGUMENT, "MoeRoute: unsupported shape (needs E <= 512, K % 256 == 0, 1 <= topk <= min(32, E))");
  if (!aligned(x, 16) || !aligned(gate_w, 16))
    return fail(GGUF_ERR_INVALID_ARGUMENT, std::string(op) + ": x and gate_w must be 16-byte aligned");
  const int clusters = static_cast<int>((R + kRouteRows - 1) / kRouteRows);
  // the cluster's x rows staged in shared memory when they fit in 64 KB (K <= 4096)
  const size_t xs = static_cast<size_t>(kRouteRows) * K * 2;
  const bool staged = xs <= 64 * 1024;
  cudaError_t e;
  if (staged) {
    static std::atomic<uint64_t> done{0};
    int dev = 0;
    cudaGetDevice(&dev);
    const uint64_t bit = 1ull << (dev & 63);
    if (!(done.load() & bit)) {
      e = cudaFuncSetAttribute(route_kernel<WT, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, 64 * 1024);
      if (e != cudaSuccess) return cuda_fail("cudaFuncSetAttribute", e);
      done.fetch_or(bit);
    }
  }
  e = launch(staged ? route_kernel<WT, true> : route_kernel<WT, false>, dim3(clusters * kRouteCtas),
             dim3(kRouteWarps * 32), staged ? xs : 0, static_cast<cudaStream_t>(stream), static_cast<const bf16*>(x), gate_w,
             bias, (int)R, (int)K, (int)E, (int)topk, scale, idx, weights, scores);
  if (e != cudaSuccess) return cuda_fail((std::string(op) + " launch").c_str(), e);
  return GGUF_OK;
}
}  // namespace
}  // namespace gguf_b200
}  // extern "C++"

int gguf_moe_route(const void* x, const float* gate_w, const float* bias, int32_t* idx, float* weights, float* scores,
                   int64_t R, int64_t K, int64_t E, int64_t topk, float scale, void* stream) {
  return run_route<float>("MoeRouteGGUF", x, gate_w, bias, idx, weights, scores, R, K, E, topk, scale, stream);
}

int gguf_moe_route_bf16(const void* x, const void* gate_w, const float* bias, int32_t* idx, float* weights,
                        float* scores, int64_t R, int64_t K, int64_t E, int64_t topk, float scale, void* stream) {
  return run_route<bf16>("MoeRoute", x, static_cast<const bf16*>(gate_w), bias, idx, weights, scores, R, K, E, topk,
                         scale, stream);
}

int gguf_relu2(const void* x, void* y, int64_t n, void* stream) {
  t_last_error.clear();
  if (n < 0) return fail(GGUF_ERR_INVALID_ARGUMENT, "Relu2: negative element count");
  if (n == 0) return GGUF_OK;
  if (!x || !y) return fail(GGUF_ERR_INVALID_ARGUMENT, "Relu2: null tensor pointer");
  if (!aligned(x, 2) || !aligned(y, 2)) return fail(GGUF_ERR_INVALID_ARGUMENT, "Relu2: tensors must be 2-byte aligned");
  int sms = 0, rc;
  if ((rc = current_sms(&sms))) return rc;
  const bool vec = aligned(x, 16) && aligned(y, 16);
  const int64_t items = vec ? (n + 7) / 8 : n;
  const int64_t ctas = std::min<int64_t>((items + 255) / 256, static_cast<int64_t>(sms) * 8);
  const cudaError_t e = launch(vec ? relu2_kernel<true> : relu2_kernel<false>, dim3(static_cast<unsigned>(ctas)),
                               dim3(256), 0, static_cast<cudaStream_t>(stream), static_cast<const bf16*>(x),
                               static_cast<bf16*>(y), n);
  if (e != cudaSuccess) return cuda_fail("Relu2 launch", e);
  return GGUF_OK;
}

namespace gguf_b200 {
namespace {
// MoeVerify iq2=3 as: zero the phase counters (first 4P bytes of out, moe_zero_kernel), one fused persistent kernel
// (grouping + fc1 + fc2, moe_fused.cuh), one finalize kernel.
int run_moe_fused(const void* z, const int32_t* idx, const float* weights, const void* fc1_w, const void* fc2_w, void* out,
                  void* h, float* part, int32_t* meta, int R, int E, int I, int topk, cudaStream_t s,
                  const PeerReduce* ep = nullptr, int expert_offset = 0) {
  constexpr int H = 1024;
  const int P = R * topk;
  MoeFusedArgs a = {};
  a.w1 = static_cast<const uint8_t*>(fc1_w);
  a.w2 = static_cast<const uint8_t*>(fc2_w);
  a.z = static_cast<const bf16*>(z);
  a.idx = idx;
  a.h = static_cast<bf16*>(h);
  a.part = part;
  a.meta = meta;
  a.done = static_cast<int*>(out);
  a.expert_offset = expert_offset;
  a.R = R;
  a.topk = topk;
  a.P = P;
  a.E = E;
  a.H = H;
  a.I = I;
  a.rb1 = H / 256 * 66;
  a.rb2 = I / 256 * 66;
  a.T1 = I / 16;
  a.T2 = H / 16;
  a.stage_bytes = ((16 * std::max(a.rb1, a.rb2) + 16) + 127) & ~127;
  const int lut = 256 * 8 * 16, red = kMoeTeams * 2 * kMoeTeamWarps * 128 * 4,
            grp = (5 * kMaxPairs + kMaxPairs * 8 + 8) * 4;
  a.off_stage = lut;
  a.off_red = lut + kMoeTeams * 2 * a.stage_bytes;
  a.off_bar = a.off_red + red;
  a.off_grp = (a.off_bar + kMoeTeams * 4 * 8 + 15) & ~15;
  const size_t smem = a.off_grp + grp;
  if (smem > static_cast<size_t>(kSmemBudgetMax))
    return fail(GGUF_ERR_INVALID_ARGUMENT, "MoeVerify: inter size too large for the staging plan");
  int sms = 0, rc;
  if ((rc = current_sms(&sms))) return rc;
  static std::atomic<uint64_t> done{0};
  cudaError_t e = launch(moe_zero_kernel, dim3(1), dim3(128), 0, s, static_cast<int*>(out), P);
  if (e != cudaSuccess) return cuda_fail("MoeVerify counters", e);
  if (R == 1 && g_fast.load() == 1) {
    // one row: the integer single-row decode; tables at offset 0 and a smaller reduction buffer
    MoeFusedArgs b = a;
    b.off_stage = kI8Lut;
    b.off_red = b.off_stage + kMoeR1Teams * 2 * a.stage_bytes;
    b.off_bar = b.off_red + kMoeR1Teams * 2 * kMoeTeamWarps * 16 * 4;
    b.off_grp = (b.off_bar + kMoeR1Teams * 4 * 8 + kMoeR1Teams * 3 * 4 + 15) & ~15;  // mbarriers, slot counters, ready words
    const size_t smem1 = b.off_grp + grp;
    if (smem1 > static_cast<size_t>(kSmemBudgetMax))
      return fail(GGUF_ERR_INVALID_ARGUMENT, "MoeVerify: inter size too large for the staging plan");
    static std::atomic<uint64_t> done1{0};
    if ((rc = ensure_smem(moe_r1_i8_kernel, smem1, done1))) return rc;
    e = launch_ex(kMoeResident, moe_r1_i8_kernel, dim3(sms), dim3(kMoeR1Warps * 32), smem1, s, b);
    if (e != cudaSuccess) return cuda_fail("MoeVerify fused launch", e);
  } else if (g_fast.load() == 1) {
    // 2..8 rows: the integer decode shared by every pair of an expert (moe_pairs_kernel)
    MoeFusedArgs b = a;
    b.off_stage = kI8Lut;
    b.off_red = b.off_stage + kMoePTeams * 2 * a.stage_bytes;
    b.off_bar = b.off_red + kMoePTeams * 2 * kMoePTW * 8 * 16 * 4;
    b.off_grp = (b.off_bar + kMoePTeams * 4 * 8 + kMoePTeams * 3 * 4 + 15) & ~15;  // mbarriers, slot counters, ready words
    b.off_zf = (b.off_grp + grp + 127) & ~127;
    const size_t smem2 = b.off_zf + static_cast<size_t>(R) * (H / 256) * kZFragBytes + kZeroBytes + kMaxPairs * 9 * 4;
    if (smem2 > static_cast<size_t>(kSmemBudgetMax)) {  // large I: the bf16-decode kernel's smaller tables
      auto kern = moe_fused_kernel;
      if ((rc = ensure_smem(kern, smem, done))) return rc;
      e = launch_ex(kMoeResident, kern, dim3(sms), dim3(kMoeWarps * 32), smem, s, a);
      if (e != cudaSuccess) return cuda_fail("MoeVerify fused launch", e);
      goto finalize;
    }
    static std::atomic<uint64_t> dp{0};
    auto kern = moe_pairs_kernel;
    if ((rc = ensure_smem(kern, smem2, dp))) return rc;
    // persistent: at most one CTA per SM, so that every CTA is resident while others wait on it
    e = launch_ex(kMoeResident, kern, dim3(sms), dim3(kMoePWarps * 32), smem2, s, b);
    if (e != cudaSuccess) return cuda_fail("MoeVerify fused launch", e);
  } else {
    auto kern = moe_fused_kernel;
    if ((rc = ensure_smem(kern, smem, done))) return rc;
    // persistent: at most one CTA per SM, so that every CTA is resident while others wait on it
    e = launch_ex(kMoeResident, kern, dim3(sms), dim3(kMoeWarps * 32), smem, s, a);
    if (e != cudaSuccess) return cuda_fail("MoeVerify fused launch", e);
  }
finalize:
  if (ep) {
    e = launch(moe_finalize_ep_kernel, dim3(1), dim3(kEpThreads), 0, s, static_cast<const float*>(part), weights, idx, topk,
               H, E, expert_offset, R, static_cast<bf16*>(out), *ep);
    if (e != cudaSuccess) return cuda_fail("MoeVerify expert-parallel finalize launch", e);
    return GGUF_OK;
  }
  e = launch(moe_finalize_kernel, dim3(static_cast<unsigned>(R)), dim3(256), 0, s, static_cast<const float*>(part), weights,
             idx, topk, H, E, static_cast<bf16*>(out));
  if (e != cudaSuccess) return cuda_fail("MoeVerify finalize launch", e);
  return GGUF_OK;
}
}  // namespace
}  // namespace gguf_b200

// Validation of MoeVerify iq2=3's caller-visible tensors and sizes (shared by the caller-scratch and
// the library-scratch entry points; runs before any device call).
static int moe_verify_check(const void* z, const int32_t* idx, const float* weights, const void* fc1_w,
                            const void* fc2_w, const void* out, int64_t R, int64_t E, int64_t I, int64_t topk) {
  if (!z || !idx || !weights || !fc1_w || !fc2_w || !out) return fail(GGUF_ERR_INVALID_ARGUMENT, "MoeVerify: null tensor pointer");
  if (R < 1 || R > 8 || topk < 1 || R * topk > 128)
    return fail(GGUF_ERR_INVALID_ARGUMENT, "MoeVerify: rows must be in [1,8] and rows*topk <= 128");
  if (I <= 0 || I % 256 != 0 || I > (1 << 20) || E < 1 || E > (1 << 20))
    return fail(GGUF_ERR_INVALID_ARGUMENT, "MoeVerify: inter size alignment mismatch (iq2=3 needs I % 256 == 0)");
  if (!aligned(fc1_w, 16) || !aligned(fc2_w, 16) || !aligned(z, 16))
    return fail(GGUF_ERR_INVALID_ARGUMENT, "MoeVerify: tensors must be 16-byte aligned");
  return GGUF_OK;
}

extern "C" int gguf_moe_verify_iq2_xxs(const void* z, const int32_t* idx, const float* weights, const void* fc1_w, const void* fc2_w,
                            void* out, void* h, float* part, int32_t* meta, int64_t R, int64_t E, int64_t I, int64_t topk,
                            void* stream) {
  t_last_error.clear();
  constexpr int H = 1024;
  if (!h || !part || !meta) return fail(GGUF_ERR_INVALID_ARGUMENT, "MoeVerify: null tensor pointer");
  if (int rc0 = moe_verify_check(z, idx, weights, fc1_w, fc2_w, out, R, E, I, topk)) return rc0;
  const int64_t P = R * topk;
  if (!aligned(h, 16) || !aligned(part, 16)) return fail(GGUF_ERR_INVALID_ARGUMENT, "MoeVerify: tensors must be 16-byte aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (g_fast.load())
    return run_moe_fused(z, idx, weights, fc1_w, fc2_w, out, h, part, meta, (int)R, (int)E, (int)I, (int)topk, s);
  int sms = 0, rc;
  if ((rc = current_sms(&sms))) return rc;
  // fc1: h = relu2(z . W1[e]^T), W1 [E, I, H/256*66]
  {
    EngineArgs a = {};
    size_t smem = 0;
    if ((rc = make_plan<kFmtIQ2>(a, H, H / 256 * 66, 1, true, &smem))) return rc;
    a.w = static_cast<const uint8_t*>(fc1_w);
    a.rows = static_cast<int>(I);
    a.tiles = static_cast<int>((I + 15) / 16);
    attach_tensor_map(a, E * I);
    a.x = static_cast<const bf16*>(z);
    a.R = static_cast<int>(R);
    a.y = h;
    a.post = 1.0f;
    a.idx = idx;
    a.topk = static_cast<int>(topk);
    a.P = static_cast<int>(P);
    a.E = static_cast<int>(E);
    a.meta = meta;
    static std::atomic<uint64_t> done{0};
    auto kern = engine_kernel<kFmtIQ2, 1, kKW, kModeMoe1>;
    if ((rc = ensure_smem(kern, smem, done))) return rc;
    const int grid = static_cast<int>(std::min<int64_t>(P * a.tiles, 2 * sms));
    cudaError_t e = launch(kern, dim3(grid), dim3(kThreads), smem, s, a);
    if (e != cudaSuccess) return cuda_fail("MoeVerify fc1 launch", e);
  }
  // fc2: part = h . W2[e]^T, W2 [E, H, I/256*66]
  {
    EngineArgs a = {};
    size_t smem = 0;
    if ((rc = make_plan<kFmtIQ2>(a, static_cast<int>(I), static_cast<int>(I / 256 * 66), 1, true, &smem))) return rc;
    a.w = static_cast<const uint8_t*>(fc2_w);
    a.rows = H;
    a.tiles = H / 16;
    attach_tensor_map(a, E * H);
    a.x = static_cast<const bf16*>(h);
    a.R = static_cast<int>(R);
    a.y = part;
    a.post = 1.0f;
    a.idx = idx;
    a.topk = static_cast<int>(topk);
    a.P = static_cast<int>(P);
    a.E = static_cast<int>(E);
    a.meta = meta;
    static std::atomic<uint64_t> done{0};
    auto kern = engine_kernel<kFmtIQ2, 1, kKW, kModeMoe2>;
    if ((rc = ensure_smem(kern, smem, done))) return rc;
    const int grid = static_cast<int>(std::min<int64_t>(P * a.tiles, 2 * sms));
    cudaError_t e = launch(kern, dim3(grid), dim3(kThreads), smem, s, a);
    if (e != cudaSuccess) return cuda_fail("MoeVerify fc2 launch", e);
  }
  cudaError_t e = launch(moe_finalize_kernel, dim3(static_cast<unsigned>(R)), dim3(256), 0, s, static_cast<const float*>(part),
                         weights, idx, static_cast<int>(topk), H, static_cast<int>(E), static_cast<bf16*>(out));
  if (e != cudaSuccess) return cuda_fail("MoeVerify finalize launch", e);
  return GGUF_OK;
}

// ---- MoeVerify / MoeDecode over the legacy split expert layouts ----
extern "C++" {
namespace gguf_b200 {
namespace {
// fc1 + fc2 on the engine's MoE modes with split-layout experts, for rows [0, R) (R <= 8,
// R * topk <= 128); meta may be null (MoeDecode).
template <int F>
int run_moe_split(const void* z, const int32_t* idx, const void* fc1_w, const void* fc1_s, const void* fc2_w,
                  const void* fc2_s, void* h, float* part, int32_t* meta, int R, int E, int I, int topk, cudaStream_t s) {
  constexpr int H = 1024;
  const int P = R * topk;
  int sms = 0, rc;
  if ((rc = current_sms(&sms))) return rc;
  {
    EngineArgs a = {};
    size_t smem = 0;
    if ((rc = make_plan<F>(a, H, H / 32 * FmtInfo<F>::kBytes, 1, true, &smem))) return rc;
    a.w = static_cast<const uint8_t*>(fc1_w);
    a.sc = static_cast<const uint8_t*>(fc1_s);
    a.rows = I;
    a.tiles = (I + 15) / 16;
    attach_tensor_map(a, static_cast<int64_t>(E) * I, true);
    a.x = static_cast<const bf16*>(z);
    a.R = R;
    a.y = h;
    a.post = 1.0f;
    a.idx = idx;
    a.topk = topk;
    a.P = P;
    a.E = E;
    a.meta = meta;
    static std::atomic<uint64_t> done{0};
    auto kern = engine_kernel<F, 1, kKW, kModeMoe1>;
    if ((rc = ensure_smem(kern, smem, done))) return rc;
    const int grid = static_cast<int>(std::min<int64_t>(static_cast<int64_t>(P) * a.tiles, 2 * sms));
    cudaError_t e = launch(kern, dim3(grid), dim3(kThreads), smem, s, a);
    if (e != cudaSuccess) return cuda_fail("MoE fc1 launch", e);
  }
  {
    EngineArgs a = {};
    size_t smem = 0;
    if ((rc = make_plan<F>(a, I, I / 32 * FmtInfo<F>::kBytes, 1, true, &smem))) return rc;
    a.w = static_cast<const uint8_t*>(fc2_w);
    a.sc = static_cast<const uint8_t*>(fc2_s);
    a.rows = H;
    a.tiles = H / 16;
    attach_tensor_map(a, static_cast<int64_t>(E) * H, true);
    a.x = static_cast<const bf16*>(h);
    a.R = R;
    a.y = part;
    a.post = 1.0f;
    a.idx = idx;
    a.topk = topk;
    a.P = P;
    a.E = E;
    a.meta = nullptr;
    static std::atomic<uint64_t> done{0};
    auto kern = engine_kernel<F, 1, kKW, kModeMoe2>;
    if ((rc = ensure_smem(kern, smem, done))) return rc;
    const int grid = static_cast<int>(std::min<int64_t>(static_cast<int64_t>(P) * a.tiles, 2 * sms));
    cudaError_t e = launch(kern, dim3(grid), dim3(kThreads), smem, s, a);
    if (e != cudaSuccess) return cuda_fail("MoE fc2 launch", e);
  }
  return GGUF_OK;
}
}  // namespace
}  // namespace gguf_b200
}  // extern "C++"

extern "C" int gguf_moe_legacy(int layout, const void* z, const int32_t* idx, const float* weights, const void* fc1_w,
                               const void* fc1_s, const void* fc2_w, const void* fc2_s, void* out, void* h, float* part,
                               int32_t* meta, int64_t R, int64_t E, int64_t I, int64_t topk, void* stream) {
  t_last_error.clear();
  constexpr int H = 1024;
  const char* op = meta ? "MoeVerify" : "MoeDecode";
  if (layout != GGUF_LAYOUT_Q4_SPLIT && layout != GGUF_LAYOUT_IQ2_CODES && layout != GGUF_LAYOUT_IQ2_NATIVE)
    return fail(GGUF_ERR_INVALID_ARGUMENT, std::string(op) + ": expert layout must be Q4_SPLIT, IQ2_CODES or IQ2_NATIVE");
  if (!z || !idx || !weights || !fc1_w || !fc1_s || !fc2_w || !fc2_s || !out || !h || !part)
    return fail(GGUF_ERR_INVALID_ARGUMENT, std::string(op) + ": null tensor pointer");
  if (topk < 1 || topk > 128 || R < 0 || R > (1 << 20) || E < 1 || E > (1 << 20))
    return fail(GGUF_ERR_INVALID_ARGUMENT, std::string(op) + ": unsupported rows / topk / experts");
  if (meta && (R < 1 || R > 8 || R * topk > 128))
    return fail(GGUF_ERR_INVALID_ARGUMENT, "MoeVerify: rows must be in [1,8] and rows*topk <= 128");
  const int64_t imul = layout == GGUF_LAYOUT_IQ2_NATIVE ? 256 : 32;
  if (I <= 0 || I % imul != 0 || I > (1 << 16))
    return fail(GGUF_ERR_INVALID_ARGUMENT, std::string(op) + ": bad inter size (I % " + std::to_string(imul) + " == 0)");
  if (!aligned(z, 16) || !aligned(fc1_w, 16) || !aligned(fc1_s, 16) || !aligned(fc2_w, 16) || !aligned(fc2_s, 16) ||
      !aligned(h, 16) || !aligned(part, 16))
    return fail(GGUF_ERR_INVALID_ARGUMENT, std::string(op) + ": tensors must be 16-byte aligned");
  if (R == 0) return GGUF_OK;
  auto* s = static_cast<cudaStream_t>(stream);
  // rows in chunks the grouped engine takes (<= 8 rows, <= 128 pairs); pair rows of h / part follow
  const int64_t chunk = std::max<int64_t>(1, std::min<int64_t>(8, 128 / topk));
  for (int64_t r0 = 0; r0 < R; r0 += chunk) {
    const int rc_rows = static_cast<int>(std::min(chunk, R - r0));
    const auto* zc = static_cast<const bf16*>(z) + r0 * H;
    const int32_t* ic = idx + r0 * topk;
    void* hc = static_cast<bf16*>(h) + r0 * topk * I;
    float* pc = part + r0 * topk * H;
    int rc;
    const int e = static_cast<int>(E), i = static_cast<int>(I), k = static_cast<int>(topk);
    if (layout == GGUF_LAYOUT_Q4_SPLIT)
      rc = run_moe_split<kFmtQ4S>(zc, ic, fc1_w, fc1_s, fc2_w, fc2_s, hc, pc, meta, rc_rows, e, i, k, s);
    else if (layout == GGUF_LAYOUT_IQ2_CODES)
      rc = run_moe_split<kFmtIQ2C>(zc, ic, fc1_w, fc1_s, fc2_w, fc2_s, hc, pc, meta, rc_rows, e, i, k, s);
    else
      rc = run_moe_split<kFmtIQ2N>(zc, ic, fc1_w, fc1_s, fc2_w, fc2_s, hc, pc, meta, rc_rows, e, i, k, s);
    if (rc) return rc;
  }
  for (int64_t r0 = 0; r0 < R; r0 += 65535) {  // finalize: one CTA per row
    const unsigned n = static_cast<unsigned>(std::min<int64_t>(65535, R - r0));
    cudaError_t e = launch(moe_finalize_kernel, dim3(n), dim3(256), 0, s, part + r0 * topk * H, weights + r0 * topk,
                           idx + r0 * topk, static_cast<int>(topk), H, static_cast<int>(E),
                           static_cast<bf16*>(out) + r0 * H);
    if (e != cudaSuccess) return cuda_fail("MoE finalize launch", e);
  }
  return GGUF_OK;
}

// ---- MoeVerify with library-owned scratch (no device allocation by the caller or the library) ----
// Some callers cannot allocate device memory around this op: a host binding without a CUDA
// allocator (a cgo / JNI / FFI caller that only holds the model's weight and activation buffers), a
// runtime whose allocator must not be entered on the decode path, or a graph that exposes only
// `out`.  For them, h, part and meta live in one file-scope device array of this library, sized for
// R * topk <= 128 pairs and I <= 4096.  The array is not zeroed and needs no zeroing: every call
// writes all of h, part and meta that it later reads; the only state that must start at zero (the
// per-expert completion counters kept in the first bytes of `out`) is cleared on the stream by each
// call.  The array is shared by all calls on a device, so calls whose executions overlap (on
// different streams, or from threads that do not order their streams) race on it.
constexpr int64_t kNoAllocMaxPairs = 128, kNoAllocMaxInter = 4096, kNoAllocH = 1024;
constexpr size_t kNoAllocHBytes = static_cast<size_t>(kNoAllocMaxPairs * kNoAllocMaxInter) * 2;  // bf16 h
constexpr size_t kNoAllocPartBytes = static_cast<size_t>(kNoAllocMaxPairs * kNoAllocH) * 4;      // f32 part
constexpr size_t kNoAllocMetaBytes = ((1 + 9 * kNoAllocMaxPairs) * 4 + 255) & ~size_t(255);     // i32 meta
static __device__ __align__(256) uint8_t g_moe_noalloc_scratch[kNoAllocHBytes + kNoAllocPartBytes + kNoAllocMetaBytes];

namespace {
// Address of the scratch array in the module instance of the current context.  Looked up on every
// call: the address belongs to a context (a driver-API context made current by the caller loads its
// own copy of the module, and cudaDeviceReset destroys the primary context's), so caching it per
// device ordinal could hand a kernel an address of another context.  After the first call in a
// context the lookup only reads the runtime's symbol table; the first call may load the module, so
// a caller that captures CUDA graphs makes one call on each device before it starts capturing.
int noalloc_scratch(void** ptr) {
  void* p = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&p, g_moe_noalloc_scratch);
  if (e != cudaSuccess) return cuda_fail("MoeVerify (no-alloc) scratch address", e);
  *ptr = p;
  return GGUF_OK;
}
}  // namespace

int gguf_moe_verify_iq2_xxs_noalloc(const void* z, const int32_t* idx, const float* weights, const void* fc1_w,
                                    const void* fc2_w, void* out, int64_t R, int64_t E, int64_t I, int64_t topk,
                                    void* stream) {
  t_last_error.clear();
  if (R < 1 || topk < 1 || R * topk > kNoAllocMaxPairs || I > kNoAllocMaxInter)
    return fail(GGUF_ERR_INVALID_ARGUMENT,
                "MoeVerify (no-alloc): needs rows*topk <= 128 and I <= 4096 (the size of the library-owned scratch)");
  // every argument check of the caller-scratch entry point runs before the scratch lookup, so an
  // invalid call fails with GGUF_ERR_INVALID_ARGUMENT and touches no device state
  if (const int rc = moe_verify_check(z, idx, weights, fc1_w, fc2_w, out, R, E, I, topk)) return rc;
  void* base = nullptr;
  if (const int rc = noalloc_scratch(&base)) return rc;
  uint8_t* b = static_cast<uint8_t*>(base);
  return gguf_moe_verify_iq2_xxs(z, idx, weights, fc1_w, fc2_w, out, b, reinterpret_cast<float*>(b + kNoAllocHBytes),
                                 reinterpret_cast<int32_t*>(b + kNoAllocHBytes + kNoAllocPartBytes), R, E, I, topk,
                                 stream);
}

int gguf_gemv_rowsplit(int type, const void* x, const void* w_shard, const float* gscale, const GgufPeerOut* out,
                       int64_t R, int64_t rows, int64_t K, void* stream) {
  t_last_error.clear();
  if (!x || !w_shard || !out) return fail(GGUF_ERR_INVALID_ARGUMENT, "rowsplit GEMV: null pointer");
  if (out->world < 1 || out->world > kMaxPeers || out->rank < 0 || out->rank >= out->world)
    return fail(GGUF_ERR_INVALID_ARGUMENT, "rowsplit GEMV: needs 1 <= world <= 8 and 0 <= rank < world");
  if (!out->state || !out->y || rows < 1 || out->row0 < 0 || out->row0 + rows > out->n_total || !int_range(out->n_total))
    return fail(GGUF_ERR_INVALID_ARGUMENT, "rowsplit GEMV: needs 0 <= row0, row0 + rows <= n_total, y and a state counter");
  for (int c = 0; c < 2; ++c)
    for (int p = 0; p < out->world; ++p)
      if (!out->stage[c][p] || !aligned(out->stage[c][p], 4))
        return fail(GGUF_ERR_INVALID_ARGUMENT, "rowsplit GEMV: null or misaligned staging buffer");
  if (R < 1 || R > 16 || R > out->r_max || K <= 0 || !int_range(K) || !aligned(w_shard, 16) || !aligned(x, 16) ||
      !aligned(out->y, 2) || !aligned(out->state, 8))
    return fail(GGUF_ERR_INVALID_ARGUMENT, "rowsplit GEMV: needs 1..16 rows (<= r_max) and 16-byte aligned x and w");
  PeerOut po = {};
  po.vec = out->n_total % 8 == 0 && out->row0 % 8 == 0 && aligned(out->y, 8);
  for (int c = 0; c < 2; ++c)
    for (int p = 0; p < out->world; ++p) {
      po.stage[c][p] = out->stage[c][p];
      po.vec = po.vec && aligned(out->stage[c][p], 16);
    }
  po.y = static_cast<bf16*>(out->y);
  po.state = out->state;
  po.npeer = out->world;
  po.rank = out->rank;
  po.ld = static_cast<int>(out->n_total);
  po.row0 = static_cast<int>(out->row0);
  po.ctas = out->ctas;
  if (po.ctas == 0 && current_sms(&po.ctas)) return GGUF_ERR_CUDA;
  if (po.ctas < 1 || po.ctas > (1 << 16))
    return fail(GGUF_ERR_INVALID_ARGUMENT, "rowsplit GEMV: ctas must be in [1, 65536] (0: this GPU's SM count)");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (type) {
    case GGUF_TYPE_Q8_0:
      if (K % 64) break;
      return run_rowsplit<kFmtQ8>(x, w_shard, nullptr, (int)R, (int)rows, (int)K, s, po);
    case GGUF_TYPE_IQ2_XXS:
      if (K % 256) break;
      return run_rowsplit<kFmtIQ2>(x, w_shard, nullptr, (int)R, (int)rows, (int)K, s, po);
    case GGUF_TYPE_NVFP4:
      if (K % 64 || !gscale) break;
      return run_rowsplit<kFmtFP4>(x, w_shard, gscale, (int)R, (int)rows, (int)K, s, po);
    default:
      return fail(GGUF_ERR_INVALID_ARGUMENT, "rowsplit GEMV: unknown GGUF type");
  }
  return fail(GGUF_ERR_INVALID_ARGUMENT, "rowsplit GEMV: K does not match the format's block size (or gscale missing)");
}

int gguf_moe_verify_iq2_xxs_ep(const void* z, const int32_t* idx, const float* weights, const void* fc1_w,
                               const void* fc2_w, void* out, void* h, float* part, int32_t* meta, const GgufPeerReduce* red,
                               int64_t R, int64_t E_local, int64_t expert_offset, int64_t I, int64_t topk, void* stream) {
  t_last_error.clear();
  if (!z || !idx || !weights || !fc1_w || !fc2_w || !out || !h || !part || !meta || !red)
    return fail(GGUF_ERR_INVALID_ARGUMENT, "MoeVerify (expert parallel): null tensor pointer");
  const int64_t P = R * topk;
  if (R < 1 || R > 8 || topk < 1 || P > 128)
    return fail(GGUF_ERR_INVALID_ARGUMENT, "MoeVerify (expert parallel): rows must be in [1,8] and rows*topk <= 128");
  if (I <= 0 || I % 256 != 0 || I > (1 << 20) || E_local < 1 || E_local > (1 << 20) || expert_offset < 0 ||
      expert_offset > (1 << 20))
    return fail(GGUF_ERR_INVALID_ARGUMENT, "MoeVerify (expert parallel): inter size alignment mismatch or bad expert range");
  if (red->world < 1 || red->world > kMaxPeers || red->rank < 0 || red->rank >= red->world || !red->state ||
      R > red->r_max || red->r_max > 8)
    return fail(GGUF_ERR_INVALID_ARGUMENT, "MoeVerify (expert parallel): needs 1 <= world <= 8, 0 <= rank < world, R <= r_max <= 8");
  for (int p = 0; p < red->world; ++p)
    if (!red->slots[p] || !red->flags[p]) return fail(GGUF_ERR_INVALID_ARGUMENT, "MoeVerify (expert parallel): null peer buffer");
  if (!aligned(fc1_w, 16) || !aligned(fc2_w, 16) || !aligned(z, 16) || !aligned(h, 16) || !aligned(part, 16))
    return fail(GGUF_ERR_INVALID_ARGUMENT, "MoeVerify (expert parallel): tensors must be 16-byte aligned");
  PeerReduce pr = {};
  for (int p = 0; p < red->world; ++p) {
    pr.slots[p] = red->slots[p];
    pr.flags[p] = red->flags[p];
  }
  pr.state = red->state;
  pr.npeer = red->world;
  pr.rank = red->rank;
  pr.slot_elems = static_cast<int>(red->r_max * 1024);
  return run_moe_fused(z, idx, weights, fc1_w, fc2_w, out, h, part, meta, (int)R, (int)E_local, (int)I, (int)topk,
                       static_cast<cudaStream_t>(stream), &pr, (int)expert_offset);
}

int gguf_ipc_get_handle(const void* dev_ptr, void* handle64, int64_t* offset) {
  t_last_error.clear();
  if (!dev_ptr || !handle64 || !offset) return fail(GGUF_ERR_INVALID_ARGUMENT, "ipc: null pointer");
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void*>(dev_ptr));
  if (e != cudaSuccess) return cuda_fail("cudaIpcGetMemHandle", e);
  static_assert(sizeof(h) == 64, "CUDA IPC handles are 64 bytes");
  std::memcpy(handle64, &h, sizeof(h));
  // the handle names the whole allocation; the peer opens its base, so report where dev_ptr lies
  static PFN_cuMemGetAddressRange_v3020 range = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      p = nullptr;
    return reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(p);
  }();
  if (!range) return fail(GGUF_ERR_CUDA, "ipc: cuMemGetAddressRange unavailable");
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(dev_ptr)) != CUDA_SUCCESS)
    return fail(GGUF_ERR_CUDA, "ipc: cuMemGetAddressRange failed");
  *offset = static_cast<int64_t>(reinterpret_cast<CUdeviceptr>(dev_ptr) - base);
  return GGUF_OK;
}

int gguf_ipc_open(const void* handle64, void** dev_ptr) {
  t_last_error.clear();
  if (!handle64 || !dev_ptr) return fail(GGUF_ERR_INVALID_ARGUMENT, "ipc: null pointer");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle64, sizeof(h));
  const cudaError_t e = cudaIpcOpenMemHandle(dev_ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return cuda_fail("cudaIpcOpenMemHandle", e);
  return GGUF_OK;
}

int gguf_ipc_close(void* dev_ptr) {
  t_last_error.clear();
  const cudaError_t e = cudaIpcCloseMemHandle(dev_ptr);
  if (e != cudaSuccess) return cuda_fail("cudaIpcCloseMemHandle", e);
  return GGUF_OK;
}

int gguf_q8_0_embed(const void* w, const int64_t* ids, void* out, int64_t vocab, int64_t row_bytes, int64_t R,
                    void* stream) {
  t_last_error.clear();
  if (vocab <= 0) return fail(GGUF_ERR_INVALID_ARGUMENT, "Q8Embed: invalid weight shape");
  if (row_bytes <= 0 || row_bytes % 34 != 0 || row_bytes / 34 > (1 << 24))
    return fail(GGUF_ERR_INVALID_ARGUMENT, "Q8Embed: row_bytes must be a positive multiple of 34");
  if (R < 0) return fail(GGUF_ERR_INVALID_ARGUMENT, "Q8Embed: negative number of ids");
  if (R == 0) return GGUF_OK;
  if (!w || !ids || !out) return fail(GGUF_ERR_INVALID_ARGUMENT, "Q8Embed: null tensor pointer");
  if (!aligned(w, 2) || !aligned(ids, 8) || !aligned(out, 8))
    return fail(GGUF_ERR_INVALID_ARGUMENT, "Q8Embed: w must be 2-byte, ids and out 8-byte aligned");
  const int nb = static_cast<int>(row_bytes / 34);
  int sms = 0, rc;
  if ((rc = current_sms(&sms))) return rc;
  // Decode-sized gathers (a few rows) keep the scalar kernel: its load -> store chain is the shortest.
  const int64_t units = R * (nb / 8);
  const bool vec = nb % 8 == 0 && aligned(w, 16) && aligned(out, 16) && units > 512;
  const int U = units > 4096 ? 4 : 1;
  const int64_t warps = vec ? (units + U - 1) / U : R * ((nb + 3) / 4);
  const int64_t ctas = std::min<int64_t>((warps + kEmbedWarps - 1) / kEmbedWarps, static_cast<int64_t>(sms) * 8);
  const auto kern = !vec ? q8_embed_kernel : U == 4 ? q8_embed_vec_kernel<4> : q8_embed_vec_kernel<1>;
  const cudaError_t e = launch(kern, dim3(static_cast<unsigned>(ctas)),
                               dim3(kEmbedWarps * 32), 0, static_cast<cudaStream_t>(stream),
                               static_cast<const uint8_t*>(w), ids, vocab, nb, R, static_cast<bf16*>(out));
  if (e != cudaSuccess) return cuda_fail("Q8Embed launch", e);
  return GGUF_OK;
}

int gguf_gemv_legacy(int layout, const void* x, const void* w, const void* scales, const float* gscale, void* y,
                     int64_t R, int64_t N, int64_t K, void* stream) {
  t_last_error.clear();
  static const char* const kNames[] = {"Q8Gemv gguf=0", "Q4Gemv iq2=0", "Q4Gemv iq2=1", "Q4Gemv iq2=2",
                                       "Nvfp4Gemv gguf=0"};
  if (layout < GGUF_LAYOUT_Q8_SPLIT || layout > GGUF_LAYOUT_NVFP4_SPLIT)
    return fail(GGUF_ERR_INVALID_ARGUMENT, "legacy GEMV: unknown layout " + std::to_string(layout));
  const std::string op = kNames[layout];
  if (!x || !w || !scales || !y || (layout == GGUF_LAYOUT_NVFP4_SPLIT && !gscale))
    return fail(GGUF_ERR_INVALID_ARGUMENT, op + ": null tensor pointer");
  const int64_t kmul = layout == GGUF_LAYOUT_IQ2_NATIVE ? 256 : 32;
  if (K <= 0 || K % kmul != 0 || K > (1 << 20))
    return fail(GGUF_ERR_INVALID_ARGUMENT, op + ": K mismatch (K % " + std::to_string(kmul) + " == 0 required)" +
                                               dims(R, N, K));
  if (R < 1 || R > 16) return fail(GGUF_ERR_INVALID_ARGUMENT, op + ": rows must be in [1,16]" + dims(R, N, K));
  if (!int_range(N)) return fail(GGUF_ERR_INVALID_ARGUMENT, op + ": bad N" + dims(R, N, K));
  if (!aligned(x, 16) || !aligned(w, 16) || !aligned(scales, 16))
    return fail(GGUF_ERR_INVALID_ARGUMENT, op + ": x, w and the scale tensor must be 16-byte aligned");
  auto* s = static_cast<cudaStream_t>(stream);
  const int r = static_cast<int>(R), n = static_cast<int>(N), k = static_cast<int>(K);
  switch (layout) {
    case GGUF_LAYOUT_Q8_SPLIT: {
      const int rc = try_q8s_rows(x, w, scales, y, r, n, k, s);
      if (rc >= 0) return rc;
    }
      return R <= 8 ? run_dense_split<kFmtQ8S, 1>(x, w, scales, gscale, y, r, n, k, s)
                    : run_dense_split<kFmtQ8S, 2>(x, w, scales, gscale, y, r, n, k, s);
    case GGUF_LAYOUT_Q4_SPLIT: {
      const int rc = try_q4s_rows(x, w, scales, y, r, n, k, s);
      if (rc >= 0) return rc;
    }
      return R <= 8 ? run_dense_split<kFmtQ4S, 1>(x, w, scales, gscale, y, r, n, k, s)
                    : run_dense_split<kFmtQ4S, 2>(x, w, scales, gscale, y, r, n, k, s);
    case GGUF_LAYOUT_IQ2_CODES:
      return R <= 8 ? run_dense_split<kFmtIQ2C, 1>(x, w, scales, gscale, y, r, n, k, s)
                    : run_dense_split<kFmtIQ2C, 2>(x, w, scales, gscale, y, r, n, k, s);
    case GGUF_LAYOUT_IQ2_NATIVE:
      return R <= 8 ? run_dense_split<kFmtIQ2N, 1>(x, w, scales, gscale, y, r, n, k, s)
                    : run_dense_split<kFmtIQ2N, 2>(x, w, scales, gscale, y, r, n, k, s);
    default: {
      const int rc = try_fp4s_rows(x, w, scales, gscale, y, r, n, k, s);
      if (rc >= 0) return rc;
    }
      return R <= 8 ? run_dense_split<kFmtFP4S, 1>(x, w, scales, gscale, y, r, n, k, s)
                    : run_dense_split<kFmtFP4S, 2>(x, w, scales, gscale, y, r, n, k, s);
  }
}

int gguf_mamba_step(const void* proj, const void* conv_state, const float* ssm_state, const void* conv_w,
                    const void* conv_b, int conv_w_f32, const float* dt_bias, const float* a_neg, const float* d_skip,
                    const float* norm_w, const int32_t* state_row, void* y, void* conv_state_out,
                    float* ssm_state_out, void* xbc_act, float* ypre, int64_t R, int64_t state_rows, int64_t heads,
                    int64_t head_dim, int64_t d_state, int64_t n_groups, float eps, float time_step_min,
                    void* stream) {
  t_last_error.clear();
  const std::string op = state_row ? "MambaVerify" : "MambaStep";
  if (head_dim != kMambaHD || d_state != kMambaDS)
    return fail(GGUF_ERR_INVALID_ARGUMENT, op + ": only head_dim=64, d_state=128 are implemented");
  if (heads < 1 || heads > 4096 || n_groups < 1 || heads % n_groups != 0)
    return fail(GGUF_ERR_INVALID_ARGUMENT, op + ": heads must be a positive multiple of n_groups");
  if (R < 1 || R > kMambaMaxRows) return fail(GGUF_ERR_INVALID_ARGUMENT, op + ": rows must be in [1,16]");
  if (state_row && state_rows < R) return fail(GGUF_ERR_INVALID_ARGUMENT, "MambaVerify: state buffer needs >= R rows");
  if (!proj || !conv_state || !ssm_state || !conv_w || !conv_b || !dt_bias || !a_neg || !d_skip || !norm_w || !y ||
      !conv_state_out || !ssm_state_out || !xbc_act || !ypre)
    return fail(GGUF_ERR_INVALID_ARGUMENT, op + ": null tensor pointer");
  if (!aligned(conv_w, conv_w_f32 ? 16 : 8) || !aligned(ssm_state, 4) || !aligned(proj, 2))
    return fail(GGUF_ERR_INVALID_ARGUMENT, op + ": conv weights must be aligned to one 4-tap row");
  MambaArgs a = {};
  a.proj = static_cast<const bf16*>(proj);
  a.R = static_cast<int>(R);
  a.di = static_cast<int>(heads * kMambaHD);
  a.cd = a.di + static_cast<int>(2 * n_groups * kMambaDS);
  a.proj_stride = a.di + a.cd + static_cast<int>(heads);
  a.heads = static_cast<int>(heads);
  a.hpg = static_cast<int>(heads / n_groups);
  a.ng = static_cast<int>(n_groups);
  a.conv_in = static_cast<const bf16*>(conv_state);
  a.conv_w = conv_w;
  a.conv_b = conv_b;
  a.conv_out = static_cast<bf16*>(conv_state_out);
  a.xbc = static_cast<bf16*>(xbc_act);
  a.ssm_in = ssm_state;
  a.dt_bias = dt_bias;
  a.a_neg = a_neg;
  a.d_skip = d_skip;
  a.tmin = time_step_min;
  a.ssm_out = ssm_state_out;
  a.ypre = ypre;
  a.state_row = state_row;
  a.state_rows = static_cast<int>(std::min<int64_t>(state_rows, 1 << 30));
  auto* s = static_cast<cudaStream_t>(stream);
  cudaError_t e = launch(conv_w_f32 ? mamba_conv_ssm_kernel<true> : mamba_conv_ssm_kernel<false>,
                         dim3(static_cast<unsigned>(heads)), dim3(kMambaThreads), 0, s, a);
  if (e != cudaSuccess) return cuda_fail((op + " launch").c_str(), e);
  e = launch(mamba_norm_kernel, dim3(static_cast<unsigned>(R), static_cast<unsigned>(n_groups)), dim3(256), 0, s,
             a.proj, a.proj_stride, a.di, static_cast<int>(a.di / n_groups), eps, static_cast<const float*>(ypre),
             norm_w, static_cast<bf16*>(y));
  if (e != cudaSuccess) return cuda_fail((op + " norm launch").c_str(), e);
  return GGUF_OK;
}

int gguf_rms_norm_iq2_xxs_gemv(const void* x, const void* skip, const float* gamma, float eps, const void* w,
                               void* y, void* x_norm_out, void* sum_out, int64_t N, int64_t K, void* stream) {
  t_last_error.clear();
  if (!x || !gamma || !w || !y) return fail(GGUF_ERR_INVALID_ARGUMENT, "RmsNorm+Q4Gemv: null tensor pointer");
  if (K != 4096) return fail(GGUF_ERR_INVALID_ARGUMENT, "RmsNorm+Q4Gemv: the fused single-row kernel needs K = 4096");
  if (!int_range(N)) return fail(GGUF_ERR_INVALID_ARGUMENT, "RmsNorm+Q4Gemv: bad N" + dims(1, N, K));
  if (!aligned(x, 16) || !aligned(w, 16) || !aligned(gamma, 16) || (skip && !aligned(skip, 16)) ||
      (x_norm_out && !aligned(x_norm_out, 16)) || (sum_out && !aligned(sum_out, 16)))
    return fail(GGUF_ERR_INVALID_ARGUMENT, "RmsNorm+Q4Gemv: tensors must be 16-byte aligned");
  const FusedNorm fn{gamma, skip, x_norm_out, skip ? sum_out : nullptr, eps};
  return run_slice_iq2_i8<16>(x, w, y, static_cast<int>(N), static_cast<int>(K), static_cast<cudaStream_t>(stream),
                              &fn);
}

int gguf_rms_norm(const void* x, const void* skip, const float* gamma, void* y, void* sum, int64_t R, int64_t H,
                  float eps, void* stream) {
  t_last_error.clear();
  const char* op = skip ? "SkipRmsNorm" : "RmsNorm";
  if (H <= 0 || H % 8 != 0 || H > (1 << 24))
    return fail(GGUF_ERR_INVALID_ARGUMENT, std::string(op) + ": hidden size H must be a positive multiple of 8");
  if (R < 0) return fail(GGUF_ERR_INVALID_ARGUMENT, std::string(op) + ": negative number of rows");
  if (R == 0) return GGUF_OK;
  if (!x || !gamma || !y) return fail(GGUF_ERR_INVALID_ARGUMENT, std::string(op) + ": null tensor pointer");
  if (!aligned(x, 16) || !aligned(gamma, 16) || !aligned(y, 16) || (skip && !aligned(skip, 16)) ||
      (sum && !aligned(sum, 16)))
    return fail(GGUF_ERR_INVALID_ARGUMENT, std::string(op) + ": tensors must be 16-byte aligned");
  if (!skip) sum = nullptr;
  int sms = 0, rc;
  if ((rc = current_sms(&sms))) return rc;
  const int nc = static_cast<int>((H / 8 + kNormThreads - 1) / kNormThreads);
  const dim3 grid(static_cast<unsigned>(std::min<int64_t>(R, static_cast<int64_t>(sms) * 4)));
  auto* s = static_cast<cudaStream_t>(stream);
  const auto* xb = static_cast<const bf16*>(x);
  const auto* sb = static_cast<const bf16*>(skip);
  auto* yb = static_cast<bf16*>(y);
  auto* ob = static_cast<bf16*>(sum);
  const int h = static_cast<int>(H);
  cudaError_t e;
  auto go = [&](auto kern) { return launch(kern, grid, dim3(kNormThreads), 0, s, xb, sb, gamma, eps, h, R, yb, ob); };
  if (skip) {
    e = nc == 1 ? go(rms_norm_kernel<true, 1>) : nc == 2 ? go(rms_norm_kernel<true, 2>)
      : nc <= 4 ? go(rms_norm_kernel<true, 4>) : go(rms_norm_kernel<true, 0>);
  } else {
    e = nc == 1 ? go(rms_norm_kernel<false, 1>) : nc == 2 ? go(rms_norm_kernel<false, 2>)
      : nc <= 4 ? go(rms_norm_kernel<false, 4>) : go(rms_norm_kernel<false, 0>);
  }
  if (e != cudaSuccess) return cuda_fail(skip ? "SkipRmsNorm launch" : "RmsNorm launch", e);
  return GGUF_OK;
}

int gguf_dequantize(int type, const void* w, float* out, int64_t rows, int64_t K, void* stream) {
  t_last_error.clear();
  if (!w || !out || rows < 0 || K <= 0) return fail(GGUF_ERR_INVALID_ARGUMENT, "dequantize: bad arguments");
  if (!aligned(w, 4)) return fail(GGUF_ERR_INVALID_ARGUMENT, "dequantize: w must be 4-byte aligned");
  if (rows == 0) return GGUF_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t groups = rows * (K / 32);
  const dim3 grid(static_cast<unsigned>((groups + 255) / 256));
  cudaError_t e;
  switch (type) {
    case GGUF_TYPE_Q8_0:
      if (K % 32) return fail(GGUF_ERR_INVALID_ARGUMENT, "dequantize Q8_0: K % 32 != 0");
      e = launch(dequant_kernel<kFmtQ8>, grid, dim3(256), 0, s, static_cast<const uint8_t*>(w), out, rows, (int)K, (int)(K / 32 * 34));
      break;
    case GGUF_TYPE_IQ2_XXS:
      if (K % 256) return fail(GGUF_ERR_INVALID_ARGUMENT, "dequantize IQ2_XXS: K % 256 != 0");
      e = launch(dequant_kernel<kFmtIQ2>, grid, dim3(256), 0, s, static_cast<const uint8_t*>(w), out, rows, (int)K, (int)(K / 256 * 66));
      break;
    case GGUF_TYPE_NVFP4:
      if (K % 64) return fail(GGUF_ERR_INVALID_ARGUMENT, "dequantize NVFP4: K % 64 != 0");
      e = launch(dequant_kernel<kFmtFP4>, grid, dim3(256), 0, s, static_cast<const uint8_t*>(w), out, rows, (int)K, (int)(K / 64 * 36));
      break;
    default:
      return fail(GGUF_ERR_NOT_IMPLEMENTED, "dequantize: unsupported GGUF type");
  }
  if (e != cudaSuccess) return cuda_fail("dequantize launch", e);
  return GGUF_OK;
}

int gguf_device_status(int* device_error_site) {
  t_last_error.clear();
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return cuda_fail("cudaDeviceSynchronize", e);
  int err = 0, site = 0, zero = 0;
  if ((e = cudaMemcpyFromSymbol(&err, g_dev_error, sizeof(int))) != cudaSuccess) return cuda_fail("status read", e);
  if ((e = cudaMemcpyFromSymbol(&site, g_dev_error_site, sizeof(int))) != cudaSuccess) return cuda_fail("status read", e);
  if ((e = cudaMemcpyToSymbol(g_dev_error, &zero, sizeof(int))) != cudaSuccess) return cuda_fail("status clear", e);
  if ((e = cudaMemcpyToSymbol(g_dev_error_site, &zero, sizeof(int))) != cudaSuccess) return cuda_fail("status clear", e);
  if (device_error_site) *device_error_site = site;
  return err ? GGUF_ERR_DEVICE : GGUF_OK;
}

}  // extern "C"
