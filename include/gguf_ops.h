/*
 * gguf_ops.h -- C ABI of libgguf_onnx_ops.so, the B200 (sm_100a) implementation of the decode-time
 * GGUF GEMV / MoE hot path of tianleiwu/gguf_onnx_ops.
 *
 * Every entry point takes raw device pointers, sizes and a CUDA stream (cudaStream_t passed as
 * void*), enqueues its kernels on that stream, never synchronises, never allocates device
 * memory and returns a status code (0 = success).  On failure, gguf_last_error() returns a
 * thread-local message naming the op and the violated constraint, in the style of the
 * reference's ORT error strings.  These are the functions that the ONNX Runtime custom-op shim
 * (RegisterCustomOps, gguf_onnx_ops_b200/csrc/ort_ops.cc) calls from each op's ComputeV2, with the
 * ORT tensors' data pointers and KernelContext_GetGPUComputeStream.
 *
 * Tensor conventions (identical to the reference ops):
 *   activations : bf16, row-major [R, K] (R = number of flattened leading rows)
 *   weights     : raw GGUF bytes, row-major [N, (K / block) * type_size], 16-byte aligned base
 *   outputs     : bf16 [R, N]
 */
#ifndef GGUF_OPS_H_
#define GGUF_OPS_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GGUF_OPS_API __attribute__((visibility("default")))

/* Status codes. */
enum {
  GGUF_OK = 0,
  GGUF_ERR_INVALID_ARGUMENT = 1, /* shape / attribute / alignment contract violated (ORT_INVALID_ARGUMENT / ORT_FAIL) */
  GGUF_ERR_CUDA = 2,             /* a CUDA launch or runtime call failed */
  GGUF_ERR_NOT_IMPLEMENTED = 3,  /* an attribute value outside the reference's set was requested */
  GGUF_ERR_DEVICE = 4,           /* a kernel reported a device-side error (bounded wait expired) */
  GGUF_ERR_IO = 5                /* a file could not be opened or mapped (gguf_file.h) */
};

/* GGUF tensor type ids (ggml numbering, docs/GGUF_ONNX_Custom_Ops.md:13-18). */
enum { GGUF_TYPE_Q8_0 = 8, GGUF_TYPE_IQ2_XXS = 16, GGUF_TYPE_NVFP4 = 40 };

/* Library version string. */
GGUF_OPS_API const char* gguf_version(void);

/* Message of the last failing call on this host thread ("" if none). */
GGUF_OPS_API const char* gguf_last_error(void);

/*
 * Q8Gemv, gguf=1:  y[R,N] = x[R,K] @ deq(W)^T,  W raw Q8_0 [N, (K/32)*34].
 * Replaces QGemvState<8>::ComputeV2 gguf=1 branch (src/bolt_ops.cu:1614-1616, :1629-1630).
 * Contract: K % 64 == 0, 1 <= R <= 16 (the reference accepts 1..8; 9..16 is a strict superset).
 */
GGUF_OPS_API int gguf_q8_0_gemv(const void* x, const void* w, void* y, int64_t R, int64_t N, int64_t K,
                                void* stream);

/*
 * Q4Gemv, iq2=3:  y[R,N] = x[R,K] @ deq(W)^T,  W raw IQ2_XXS [N, (K/256)*66].
 * Replaces QGemvState<4>::ComputeV2 iq2=3 branch (src/bolt_ops.cu:1608-1610, :1623-1624).
 * Contract: K % 256 == 0, 1 <= R <= 16.
 */
GGUF_OPS_API int gguf_iq2_xxs_gemv(const void* x, const void* w, void* y, int64_t R, int64_t N, int64_t K,
                                   void* stream);

/*
 * Nvfp4Gemv, gguf=1:  y[R,N] = gscale[0] * (x[R,K] @ deq(W)^T),  W raw NVFP4 [N, (K/64)*36],
 * gscale: device f32 [1].
 * Replaces Nvfp4GemvState::ComputeV2 gguf=1 branch (src/bolt_ops.cu:1424-1433).
 * Contract: K % 64 == 0, 1 <= R <= 16.  Scale bytes decode as gguf-py's unsigned E4M3 (bit 7
 * ignored, 0x00 and 0x7F -> 0).
 */
GGUF_OPS_API int gguf_nvfp4_gemv(const void* x, const void* w, const float* gscale, void* y, int64_t R, int64_t N,
                                 int64_t K, void* stream);

/*
 * Legacy (pre-GGUF, "split") weight layouts of the same ops, selected in the reference by attribute
 * values other than gguf=1 / iq2=3 (src/bolt_ops.cu:840-848, :1411-1469, :1593-1643):
 *
 *   layout                     op / attribute       w                         scales
 *   GGUF_LAYOUT_Q8_SPLIT       Q8Gemv gguf=0        u8 [N, K] = q + 128       bf16 [N, K/32]
 *   GGUF_LAYOUT_Q4_SPLIT       Q4Gemv iq2=0         u8 [N, K/2] nibbles n     bf16 [N, K/32]    (value (n - 8) * s)
 *   GGUF_LAYOUT_IQ2_CODES      Q4Gemv iq2=1         u8 [N, K/2] codes c       bf16 [N, K/32]    (value {8,25,43,0}[c&3] * (c&4 ? -1 : 1) * s)
 *   GGUF_LAYOUT_IQ2_NATIVE     Q4Gemv iq2=2         u8 [N, K/32, 8] records   fp16 bits [N, K/256] (IQ2_XXS blocks minus d)
 *   GGUF_LAYOUT_NVFP4_SPLIT    Nvfp4Gemv gguf=0     u8 [N, K/2] E2M1 nibbles  e4m3fn [N, K/16], times gscale[0]
 *
 * Nibble tensors hold element 2i in the low and 2i+1 in the high nibble of byte i.  x bf16 [R, K],
 * y bf16 [R, N]; 1 <= R <= 16; K % 32 == 0 (IQ2_NATIVE: K % 256 == 0); x, w and scales 16-byte
 * aligned.  Weights enter the tensor cores exactly; scales are applied in fp32 after the MMA.
 */
enum {
  GGUF_LAYOUT_Q8_SPLIT = 0,
  GGUF_LAYOUT_Q4_SPLIT = 1,
  GGUF_LAYOUT_IQ2_CODES = 2,
  GGUF_LAYOUT_IQ2_NATIVE = 3,
  GGUF_LAYOUT_NVFP4_SPLIT = 4
};
GGUF_OPS_API int gguf_gemv_legacy(int layout, const void* x, const void* w, const void* scales, const float* gscale,
                                  void* y, int64_t R, int64_t N, int64_t K, void* stream);

/*
 * MoeVerify iq2 = 0 / 1 / 2 and MoeDecode (src/bolt_ops.cu:664-699, :1327-1409): the relu^2 MoE of
 * gguf_moe_verify_iq2_xxs over experts in a legacy split layout (layout GGUF_LAYOUT_Q4_SPLIT for
 * iq2=0 and MoeDecode, GGUF_LAYOUT_IQ2_CODES for iq2=1, GGUF_LAYOUT_IQ2_NATIVE for iq2=2):
 *   fc1_w [E, I, 1024/32 * b] + fc1_s [E, I, 1024/g], fc2_w [E, 1024, I/32 * b] + fc2_s [E, 1024, I/g]
 *   (b = 16 bytes per 32 and g = 32 bf16 scales for Q4 / codes; b = 8 and g = 256 fp16 d for native).
 * h bf16 [R*topk, I], part f32 [R*topk, 1024], out bf16 [R, 1024]; meta i32 [1 + 9*R*topk] (the
 * grouping table, MoeVerify) or NULL (MoeDecode, any R: rows are processed in groups of <= 8).
 * I % 32 == 0 (native: % 256); MoeVerify: 1 <= R <= 8, R*topk <= 128.
 */
GGUF_OPS_API int gguf_moe_legacy(int layout, const void* z, const int32_t* idx, const float* weights, const void* fc1_w,
                                 const void* fc1_s, const void* fc2_w, const void* fc2_s, void* out, void* h,
                                 float* part, int32_t* meta, int64_t R, int64_t E, int64_t I, int64_t topk,
                                 void* stream);

/*
 * MambaStep / MambaVerify / MambaStepGGUF / MambaVerifyGGUF (src/bolt_ops.cu:68-378, :1886-1946):
 * one Mamba-2 mixer step after the input projection, for R <= 16 rows (tokens).
 *   proj bf16 [R, di + cd + heads] = [gate | xBC | dt], di = heads * 64, cd = di + 2 * n_groups * 128;
 *   conv_state bf16 [Rs, cd, 3]; ssm_state f32 [Rs, heads, 128, 64]; conv_w [cd, 4] and conv_b [cd]
 *   as bf16 (conv_w_f32 = 0) or fp32 rounded to bf16 on use (conv_w_f32 = 1, the GGUF ops);
 *   dt_bias, a_neg, d_skip f32 [heads]; norm_w f32 [di].
 * state_row == NULL (Step): the step starts from row 0 and the state after the last row is written
 * to conv_state_out [1, cd, 3] / ssm_state_out [1, heads, 128, 64].  state_row != NULL (Verify): a
 * device int32 selecting the input row of the [Rs >= R, ...] buffers; the state after token r goes
 * to row r of the outputs (a row outside [0, Rs) is read as row 0 and reported by
 * gguf_device_status).  Outputs: y bf16 [R, di], xbc_act bf16 [R, cd], ypre f32 [R, di].  Outputs
 * must not alias the state inputs.  head_dim must be 64 and d_state 128 (the reference's limit).
 */
GGUF_OPS_API int gguf_mamba_step(const void* proj, const void* conv_state, const float* ssm_state, const void* conv_w,
                                 const void* conv_b, int conv_w_f32, const float* dt_bias, const float* a_neg,
                                 const float* d_skip, const float* norm_w, const int32_t* state_row, void* y,
                                 void* conv_state_out, float* ssm_state_out, void* xbc_act, float* ypre, int64_t R,
                                 int64_t state_rows, int64_t heads, int64_t head_dim, int64_t d_state,
                                 int64_t n_groups, float eps, float time_step_min, void* stream);

/*
 * Q8Embed:  out[..., k] = bf16(fp32(d) * q[k]) of the rows input_ids[...] of a GGUF Q8_0 embedding
 * table w [vocab, row_bytes] (row_bytes = (K/32)*34); ids outside [0, vocab) read row 0.
 * ids: int64 [R] (any shape, flattened); out: bf16 [R, K].  R = 0 is a no-op.
 * Replaces Q8EmbedState::ComputeV2 (src/bolt_ops.cu:1662-1688).
 */
GGUF_OPS_API int gguf_q8_0_embed(const void* w, const int64_t* ids, void* out, int64_t vocab, int64_t row_bytes,
                                 int64_t R, void* stream);

/*
 * RmsNorm / SkipRmsNorm:  v = x, or v = bf16(x + skip) when skip != NULL (then also stored to sum
 * when sum != NULL);  y = bf16(bf16(gamma) * v * rsqrt(mean(v^2) + eps)).
 * x, skip, y, sum: bf16 [R, H]; gamma: fp32 [H]; H a positive multiple of 8; 16-byte aligned
 * tensors.  R = 0 is a no-op.  Replaces RmsNormState<HAS_SKIP>::ComputeV2 (src/bolt_ops.cu:1817-1863)
 * and its kernels (:1695-1815); the mean of squares is summed in a fixed fp32 order of 512 partial
 * sums that the fused GEMV prologues reproduce.
 */
GGUF_OPS_API int gguf_rms_norm(const void* x, const void* skip, const float* gamma, void* y, void* sum, int64_t R,
                               int64_t H, float eps, void* stream);

/*
 * (Skip)RmsNorm fused into the single-row IQ2_XXS GEMV (no counterpart in the reference, which runs
 * the two ops as separate kernels): y = Q4Gemv_iq2=3(RmsNorm(x [+ skip], gamma, eps), w), one launch.
 * Every CTA normalises the row in its prologue with the standalone op's arithmetic, so y, and the
 * optional x_norm_out (the normalised row) and sum_out (bf16(x + skip)), are bit-identical to
 * gguf_rms_norm followed by gguf_iq2_xxs_gemv.  x, skip, x_norm_out, sum_out bf16 [1, K]; gamma fp32
 * [K]; w raw IQ2_XXS [N, K/256*66]; K = 4096; skip, x_norm_out and sum_out may be NULL.
 */
GGUF_OPS_API int gguf_rms_norm_iq2_xxs_gemv(const void* x, const void* skip, const float* gamma, float eps,
                                            const void* w, void* y, void* x_norm_out, void* sum_out, int64_t N,
                                            int64_t K, void* stream);

/*
 * MoeRouteGGUF:  scores[R,E] = sigmoid(x[R,K] @ bf16(gate_w)^T);  idx[R,topk] = top-k of scores + bias
 * (descending, ties to the lower expert index);  weights = s_sel / (sum s_sel + 1e-20) * scale.
 * x bf16 [R,K]; gate_w f32 [E,K]; bias f32 [E] -> idx i32 [R,topk], weights f32 [R,topk], scores f32 [R,E].
 * Replaces MoeRouteStateT<float>::ComputeV2 (src/bolt_ops.cu:512-546).
 * Contract: E <= 512, K % 256 == 0, 1 <= topk <= 32, topk <= E, R >= 1.
 */
GGUF_OPS_API int gguf_moe_route(const void* x, const float* gate_w, const float* bias, int32_t* idx, float* weights,
                                float* scores, int64_t R, int64_t K, int64_t E, int64_t topk, float scale,
                                void* stream);

/*
 * MoeRoute: MoeRouteGGUF with bf16 gate weights [E, K] (src/bolt_ops.cu:513-547, :1947-1956); the
 * same kernel, so for gate weights that are bf16 values both ops return identical outputs.
 */
GGUF_OPS_API int gguf_moe_route_bf16(const void* x, const void* gate_w, const float* bias, int32_t* idx,
                                     float* weights, float* scores, int64_t R, int64_t K, int64_t E, int64_t topk,
                                     float scale, void* stream);

/*
 * Relu2: y = bf16(max(x, 0)^2) elementwise over n bf16 values (src/bolt_ops.cu:700-726, :1997-2003).
 */
GGUF_OPS_API int gguf_relu2(const void* x, void* y, int64_t n, void* stream);

/*
 * MoeVerify, iq2=3 (expert-grouped relu^2 MoE over raw IQ2_XXS expert tensors):
 *   for each pair p = (t, j), e = idx[t,j]:  h[p] = bf16(relu(bf16(z[t] . W1[e]^T))^2)
 *                                            part[p] = bf16(h[p] . W2[e]^T)   (stored as f32)
 *   out[t] = bf16(sum_j weights[t,j] * part[t*topk + j])   (f32 sum, j ascending)
 * z bf16 [R,1024]; idx i32 [R,topk]; weights f32 [R,topk]; fc1_w u8 [E, I, 4*66]; fc2_w u8 [E, 1024, (I/256)*66]
 * -> out bf16 [R,1024]; h bf16 [R*topk, I]; part f32 [R*topk, 1024]; meta i32 [1 + 9*R*topk]
 * (meta[0] = number of unique experts U, meta[1..U] their ids, meta[1+P+u*8+t] = pair of row t for expert u or -1).
 * Replaces MoeVerifyState::ComputeV2 iq2=3 (src/bolt_ops.cu:1327-1409).
 * Contract: 1 <= R <= 8, R*topk <= 128, I % 256 == 0, every idx in [0, E).
 */
GGUF_OPS_API int gguf_moe_verify_iq2_xxs(const void* z, const int32_t* idx, const float* weights, const void* fc1_w,
                                         const void* fc2_w, void* out, void* h, float* part, int32_t* meta, int64_t R,
                                         int64_t E, int64_t I, int64_t topk, void* stream);

/*
 * MoeVerify, iq2=3, for callers that cannot allocate device memory (no counterpart in the
 * reference): the same computation and `out` as gguf_moe_verify_iq2_xxs, with h, part and meta held
 * in a device array owned by this library instead of caller tensors.  For a host binding without a
 * CUDA allocator, or a decode loop that must not enter an allocator.
 * Limits: rows*topk <= 128 and I <= 4096 (larger sizes return GGUF_ERR_INVALID_ARGUMENT); the other
 * contract terms of gguf_moe_verify_iq2_xxs apply.
 * Every call looks the array's address up in the current context (cudaGetSymbolAddress; a driver-API
 * context made current by the caller has its own copy of the array).  The first call in a context
 * may load the library's device code there, so make it before any stream capture.  Argument errors
 * are reported before that lookup.  The array is shared by every call on a device: calls
 * whose executions may overlap (different streams, unordered threads) race on it and must be ordered
 * by the caller.  Nothing in the array needs to start at zero; the per-call counters are cleared on
 * the stream by each call.
 */
GGUF_OPS_API int gguf_moe_verify_iq2_xxs_noalloc(const void* z, const int32_t* idx, const float* weights,
                                                 const void* fc1_w, const void* fc2_w, void* out, int64_t R, int64_t E,
                                                 int64_t I, int64_t topk, void* stream);

/*
 * Row-split (tensor-parallel) GEMV with the all-gather fused into the kernel (no counterpart in the
 * reference, which runs on one GPU; meant for LM-head-sized Q8Gemv calls).  GPU `rank` of
 * `world` holds rows [row0, row0 + rows) of W (w_shard, raw GGUF rows) and computes those outputs
 * for all R activation rows.  Every value is stored into the staging buffer of every GPU of the
 * group (peer pointers opened with gguf_ipc_open, NVLink stores) as one 32-bit word: the bf16 bits
 * in the low half, the call number mod 2^16 in the high half.  Each GPU converts its own staging
 * buffer into y, waiting (bounded, timeouts reported through gguf_device_status) for words that do
 * not carry the current call's number yet; the launch ends only when the whole y [R, n_total] is
 * on this GPU.  No fence or flag is exchanged: a 32-bit store arrives whole.  All GPUs of the group
 * must issue the same sequence of calls; a GPU can run one call ahead of another, so there are two
 * staging buffers, one per call parity.
 */
typedef struct {
  uint32_t* stage[2][8];     /* staging buffer of GPU p for calls of parity c: uint32 [r_max, n_total],
                                zero-initialised; stage[c][rank] = this GPU's own */
  void* y;                   /* this GPU's output: bf16 [R, n_total] (rewritten by every call) */
  unsigned long long* state; /* this GPU: uint64 [1], zero-initialised, shared by all calls */
  int world, rank;
  int64_t n_total, row0;
  int32_t ctas;              /* CTAs each GPU launches per call: the same value on every GPU of the group;
                                0 = this GPU's SM count (only when every GPU of the group has the same) */
  int32_t r_max;             /* activation rows the staging buffers hold (R <= r_max) */
} GgufPeerOut;

/* type = GGUF_TYPE_*; gscale for NVFP4 only.  Contract as the single-GPU GEMV of that type, plus
 * 1 <= world <= 8, 0 <= rank < world, row0 + rows <= n_total. */
GGUF_OPS_API int gguf_gemv_rowsplit(int type, const void* x, const void* w_shard, const float* gscale,
                                    const GgufPeerOut* out, int64_t R, int64_t rows, int64_t K, void* stream);

/*
 * Expert-parallel MoeVerify iq2=3 (no counterpart in the reference, which runs on one GPU): GPU
 * `rank` holds experts [expert_offset, expert_offset + E_local) (fc1_w / fc2_w are
 * those experts' tensors) and processes the pairs routed to them; idx holds global expert ids (the
 * router is replicated).  The f32 [R, 1024] partial outputs are summed across the group through peer
 * memory (every GPU stores its partial into its slot of every GPU's buffer, epoch flags, bounded
 * waits), in rank order, and rounded once to bf16 into out.  h / part / meta hold this GPU's pairs
 * only (meta with global expert ids).  All GPUs must issue the same sequence of calls.
 */
typedef struct {
  float* slots[8];      /* reduction buffer of GPU p: f32 [2][world][r_max * 1024] */
  uint32_t* flags[8];   /* flag array of GPU p: uint32 [8], zero-initialised */
  uint32_t* state;      /* this GPU: uint32 [1], zero-initialised */
  int world, rank;
  int64_t r_max;
} GgufPeerReduce;

GGUF_OPS_API int gguf_moe_verify_iq2_xxs_ep(const void* z, const int32_t* idx, const float* weights, const void* fc1_w,
                                            const void* fc2_w, void* out, void* h, float* part, int32_t* meta,
                                            const GgufPeerReduce* red, int64_t R, int64_t E_local,
                                            int64_t expert_offset, int64_t I, int64_t topk, void* stream);

/* CUDA IPC plumbing for the peer pointers: the 64-byte handle of the device allocation holding
 * dev_ptr and dev_ptr's offset in it; open a peer's handle in this process (returns the allocation
 * base: add the peer's offset; peer access is enabled lazily); close an opened handle. */
GGUF_OPS_API int gguf_ipc_get_handle(const void* dev_ptr, void* handle64, int64_t* offset);
GGUF_OPS_API int gguf_ipc_open(const void* handle64, void** dev_ptr);
GGUF_OPS_API int gguf_ipc_close(void* dev_ptr);

/*
 * Dequantise raw GGUF rows to f32 with the same device decoders the GEMVs use (debug / parity
 * entry point; no counterpart op in the reference).  type = GGUF_TYPE_*; w [rows, row_bytes(K)];
 * out f32 [rows, K].  Results are bit-identical to gguf-py 0.19.0 dequantize.
 */
GGUF_OPS_API int gguf_dequantize(int type, const void* w, float* out, int64_t rows, int64_t K, void* stream);

/*
 * Device-side status: returns the first error code recorded by a kernel on the current device
 * since the last call (0 if none) and clears it.  Synchronises the device; for tests and
 * diagnostics, not for the hot path.
 */
GGUF_OPS_API int gguf_device_status(int* device_error_site);

/* Tuning: enable (1) / disable (0) programmatic dependent launch for subsequent calls (default 1). */
GGUF_OPS_API void gguf_set_pdl(int enable);

/* Tuning / testing: enable (1, default) or disable (0) the shape-specialised kernels (the single-row
 * kernels and the fused MoeVerify); disabled, every call uses the generic engine.  2 and 3 = as 1,
 * but single-row IQ2_XXS uses the bf16 tensor-core slice kernel (2) or the integer row-block kernel
 * (3) instead of the integer slice kernel; 4 = as 1, but single-row NVFP4 uses the integer-decode
 * slice kernel instead of the bf16 one (cross-checks of the decoders). */
GGUF_OPS_API void gguf_set_fast_paths(int enable);

#ifdef __cplusplus
}
#endif

#endif /* GGUF_OPS_H_ */
