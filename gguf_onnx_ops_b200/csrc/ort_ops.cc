// ONNX Runtime custom-op shim: exports RegisterCustomOps and maps the reference's op names onto the
// C ABI of include/gguf_ops.h.  Compiled into libgguf_onnx_ops.so only when ONNX Runtime headers are
// available (gguf_onnx_ops_b200/build.py, ORT_INCLUDE_DIR), as the reference's CMakeLists.txt:4-7 requires.
//
// Contract kept from the reference (src/bolt_ops.cu:2065-2115, :1865-2061):
//   * the same 15 op names are registered in both the "bolt" and the "gguf" domains, for the CUDA EP;
//   * each op keeps its input / output count, element types and optional inputs;
//   * shape errors come back as ORT_FAIL with the reference's message, attribute values that select
//     the legacy (non-GGUF) layouts and the ops outside the GGUF decode path come back as
//     ORT_NOT_IMPLEMENTED.
// The shim is table-driven: one op class reads its name, types and compute function from a
// descriptor, and each compute function is a thin adapter over one C-ABI entry point.
#define ORT_API_MANUAL_INIT
#include <onnxruntime_cxx_api.h>

#include <cstdint>
#include <mutex>
#include <stdexcept>
#include <string>
#include <vector>

#include "gguf_ops.h"

namespace {

constexpr auto kBF = ONNX_TENSOR_ELEMENT_DATA_TYPE_BFLOAT16;
constexpr auto kF32 = ONNX_TENSOR_ELEMENT_DATA_TYPE_FLOAT;
constexpr auto kU8 = ONNX_TENSOR_ELEMENT_DATA_TYPE_UINT8;
constexpr auto kI32 = ONNX_TENSOR_ELEMENT_DATA_TYPE_INT32;
constexpr auto kI64 = ONNX_TENSOR_ELEMENT_DATA_TYPE_INT64;

struct NotImplemented : std::runtime_error {
  using std::runtime_error::runtime_error;
};

// Attributes of one node, read once at kernel creation.
struct Attrs {
  int64_t gguf = 0, iq2 = 0, topk = 0;
  float scale = 1.0f, epsilon = 1e-5f;
  int64_t heads = 0, head_dim = 0, d_state = 0, n_groups = 0;  // Mamba*
  float time_step_min = 0.0f;
};

int64_t opt_int(const OrtKernelInfo* info, const char* name, int64_t dflt) {
  int64_t v = dflt;
  OrtStatus* st = Ort::GetApi().KernelInfoGetAttribute_int64(info, name, &v);
  if (st != nullptr) {
    Ort::GetApi().ReleaseStatus(st);
    return dflt;
  }
  return v;
}
// A required attribute (the reference reads it with KernelInfo::GetAttribute, which throws when the
// node lacks it, and CreateKernelV2 turns that into ORT_INVALID_ARGUMENT: src/bolt_ops.cu:1873).
bool has_int(const OrtKernelInfo* info, const char* name) {
  int64_t v = 0;
  OrtStatus* st = Ort::GetApi().KernelInfoGetAttribute_int64(info, name, &v);
  if (st == nullptr) return true;
  Ort::GetApi().ReleaseStatus(st);
  return false;
}
bool has_float(const OrtKernelInfo* info, const char* name) {
  float v = 0.f;
  OrtStatus* st = Ort::GetApi().KernelInfoGetAttribute_float(info, name, &v);
  if (st == nullptr) return true;
  Ort::GetApi().ReleaseStatus(st);
  return false;
}
float opt_float(const OrtKernelInfo* info, const char* name, float dflt) {
  float v = dflt;
  OrtStatus* st = Ort::GetApi().KernelInfoGetAttribute_float(info, name, &v);
  if (st != nullptr) {
    Ort::GetApi().ReleaseStatus(st);
    return dflt;
  }
  return v;
}

using ComputeFn = void (*)(Ort::KernelContext&, const Attrs&);

struct OpDesc {
  const char* name;
  std::vector<ONNXTensorElementDataType> in, out;
  std::vector<int> optional_in;  // indices of optional inputs
  ComputeFn compute;             // nullptr: op outside the GGUF decode path
  std::vector<int> optional_out = {};  // indices of optional outputs
  std::vector<const char*> req_int = {};    // attributes whose absence fails kernel creation
  std::vector<const char*> req_float = {};
};

// ---- helpers over the C++ API ----
int64_t count(const Ort::ConstValue& v) { return v.GetTensorTypeAndShapeInfo().GetElementCount(); }
std::vector<int64_t> shape(const Ort::ConstValue& v) { return v.GetTensorTypeAndShapeInfo().GetShape(); }
bool present(Ort::KernelContext& c, size_t i) {
  if (i >= c.GetInputCount()) return false;
  return static_cast<const OrtValue*>(c.GetInput(i)) != nullptr;
}
void* stream(Ort::KernelContext& c) { return c.GetGPUComputeStream(); }
void check(int rc) {
  if (rc == GGUF_OK) return;
  if (rc == GGUF_ERR_NOT_IMPLEMENTED) throw NotImplemented(gguf_last_error());
  throw std::runtime_error(gguf_last_error());
}

// ---- compute adapters ----
void gemv_shapes(Ort::KernelContext& c, int64_t& R, int64_t& N, int64_t& K, std::vector<int64_t>& yshape) {
  auto x = c.GetInput(0);
  auto w = c.GetInput(1);
  yshape = shape(x);
  if (yshape.empty()) throw std::invalid_argument("x must have rank >= 1");
  K = yshape.back();
  R = K > 0 ? count(x) / K : 0;
  auto ws = shape(w);
  N = ws.empty() ? 0 : ws[0];
  yshape.back() = N;
}

// Legacy split layouts: weights in input 1, scales in input 2 (src/bolt_ops.cu:1593-1643, :1411-1469).
void gemv_legacy(Ort::KernelContext& c, int layout, const char* op, int64_t kmul) {
  int64_t R, N, K;
  std::vector<int64_t> ys;
  gemv_shapes(c, R, N, K, ys);
  if (!present(c, 2)) throw std::invalid_argument(std::string(op) + ": the scale input is required");
  if (K % kmul != 0) throw std::invalid_argument("QGemv: K mismatch");
  auto y = c.GetOutput(0, ys);
  const float* g = layout == GGUF_LAYOUT_NVFP4_SPLIT ? c.GetInput(3).GetTensorData<float>() : nullptr;
  check(gguf_gemv_legacy(layout, c.GetInput(0).GetTensorRawData(), c.GetInput(1).GetTensorRawData(),
                         c.GetInput(2).GetTensorRawData(), g, y.GetTensorMutableRawData(), R, N, K, stream(c)));
}

void q8_gemv(Ort::KernelContext& c, const Attrs& a) {
  if (a.gguf != 1) return gemv_legacy(c, GGUF_LAYOUT_Q8_SPLIT, "Q8Gemv", 32);
  int64_t R, N, K;
  std::vector<int64_t> ys;
  gemv_shapes(c, R, N, K, ys);
  if (K % 64 != 0 || count(c.GetInput(1)) != N * (K / 32) * 34 || R < 1 || R > 16)
    throw std::invalid_argument("Q8Gemv gguf=1: needs B [N, (K/32)*34] and 1..16 rows");
  auto y = c.GetOutput(0, ys);
  check(gguf_q8_0_gemv(c.GetInput(0).GetTensorRawData(), c.GetInput(1).GetTensorRawData(), y.GetTensorMutableRawData(),
                       R, N, K, stream(c)));
}

void q4_gemv(Ort::KernelContext& c, const Attrs& a) {
  if (a.iq2 == 0) return gemv_legacy(c, GGUF_LAYOUT_Q4_SPLIT, "Q4Gemv", 32);
  if (a.iq2 == 1) return gemv_legacy(c, GGUF_LAYOUT_IQ2_CODES, "Q4Gemv iq2=1", 32);
  if (a.iq2 == 2) return gemv_legacy(c, GGUF_LAYOUT_IQ2_NATIVE, "Q4Gemv iq2=2", 256);
  if (a.iq2 != 3) throw NotImplemented("Q4Gemv: unknown iq2 value");
  int64_t R, N, K;
  std::vector<int64_t> ys;
  gemv_shapes(c, R, N, K, ys);
  if (K % 256 != 0 || count(c.GetInput(1)) != N * (K / 256) * 66 || R < 1 || R > 16)
    throw std::invalid_argument("Q4Gemv iq2=3: needs B [N, (K/256)*66] and 1..16 rows");
  auto y = c.GetOutput(0, ys);
  check(gguf_iq2_xxs_gemv(c.GetInput(0).GetTensorRawData(), c.GetInput(1).GetTensorRawData(),
                          y.GetTensorMutableRawData(), R, N, K, stream(c)));
}

void fp4_gemv(Ort::KernelContext& c, const Attrs& a) {
  if (a.gguf != 1) return gemv_legacy(c, GGUF_LAYOUT_NVFP4_SPLIT, "Nvfp4Gemv", 32);
  int64_t R, N, K;
  std::vector<int64_t> ys;
  gemv_shapes(c, R, N, K, ys);
  if (K % 64 != 0 || count(c.GetInput(1)) != N * (K / 64) * 36 || R < 1 || R > 16)
    throw std::invalid_argument("Nvfp4Gemv gguf=1: needs w [N, (K/64)*36] and 1..16 rows");
  auto y = c.GetOutput(0, ys);
  check(gguf_nvfp4_gemv(c.GetInput(0).GetTensorRawData(), c.GetInput(1).GetTensorRawData(),
                        c.GetInput(3).GetTensorData<float>(), y.GetTensorMutableRawData(), R, N, K, stream(c)));
}

void route_gguf(Ort::KernelContext& c, const Attrs& a) {
  auto x = c.GetInput(0);
  auto gw = c.GetInput(1);
  auto xs = shape(x), gs = shape(gw);
  if (xs.size() != 2 || gs.size() != 2) throw std::invalid_argument("MoeRoute: unsupported shape");
  const int64_t R = xs[0], K = xs[1], E = gs[0];
  if (E > 512 || K % 256 != 0 || a.topk > 32 || gs[1] != K || count(c.GetInput(2)) != E)
    throw std::invalid_argument("MoeRoute: unsupported shape");
  auto idx = c.GetOutput(0, {R, a.topk});
  auto wt = c.GetOutput(1, {R, a.topk});
  auto sc = c.GetOutput(2, {R, E});
  check(gguf_moe_route(x.GetTensorRawData(), gw.GetTensorData<float>(), c.GetInput(2).GetTensorData<float>(),
                       idx.GetTensorMutableData<int32_t>(), wt.GetTensorMutableData<float>(),
                       sc.GetTensorMutableData<float>(), R, K, E, a.topk, a.scale, stream(c)));
}

void route_bf16(Ort::KernelContext& c, const Attrs& a) {
  auto x = c.GetInput(0);
  auto gw = c.GetInput(1);
  auto xs = shape(x), gs = shape(gw);
  if (xs.size() != 2 || gs.size() != 2) throw std::invalid_argument("MoeRoute: unsupported shape");
  const int64_t R = xs[0], K = xs[1], E = gs[0];
  if (E > 512 || K % 256 != 0 || a.topk > 32 || gs[1] != K || count(c.GetInput(2)) != E)
    throw std::invalid_argument("MoeRoute: unsupported shape");
  auto idx = c.GetOutput(0, {R, a.topk});
  auto wt = c.GetOutput(1, {R, a.topk});
  auto sc = c.GetOutput(2, {R, E});
  check(gguf_moe_route_bf16(x.GetTensorRawData(), gw.GetTensorRawData(), c.GetInput(2).GetTensorData<float>(),
                            idx.GetTensorMutableData<int32_t>(), wt.GetTensorMutableData<float>(),
                            sc.GetTensorMutableData<float>(), R, K, E, a.topk, a.scale, stream(c)));
}

void relu2(Ort::KernelContext& c, const Attrs&) {
  auto x = c.GetInput(0);
  auto y = c.GetOutput(0, shape(x));
  check(gguf_relu2(x.GetTensorRawData(), y.GetTensorMutableRawData(), count(x), stream(c)));
}

// MoeVerify iq2 = 0 / 1 / 2 and MoeDecode: experts in a split layout, scales in inputs 4 and 6.
void moe_legacy(Ort::KernelContext& c, int layout, int64_t topk, bool verify) {
  auto z = c.GetInput(0);
  auto zs = shape(z);
  const char* op = verify ? "MoeVerify" : "MoeDecode";
  if (zs.size() != 2 || zs[1] != 1024) throw std::invalid_argument(std::string(op) + ": latent size must be 1024");
  const int64_t R = zs[0], P = R * topk;
  if (verify && (R < 1 || R > 8 || P > 128))
    throw std::invalid_argument("MoeVerify: rows must be in [1,8] and rows*topk <= 128");
  auto w1s = shape(c.GetInput(3));
  if (w1s.size() < 2) throw std::invalid_argument(std::string(op) + ": fc1_w must be [E, I, ...]");
  const int64_t E = w1s[0], I = w1s[1];
  if (!present(c, 4) || !present(c, 6)) throw std::invalid_argument(std::string(op) + ": expert scales are required");
  auto out = c.GetOutput(0, {R, 1024});
  auto h = c.GetOutput(1, {P, I});
  auto part = c.GetOutput(2, {P, 1024});
  int32_t* meta = nullptr;
  if (verify) meta = c.GetOutput(3, {1 + 9 * P}).GetTensorMutableData<int32_t>();
  check(gguf_moe_legacy(layout, z.GetTensorRawData(), c.GetInput(1).GetTensorData<int32_t>(),
                        c.GetInput(2).GetTensorData<float>(), c.GetInput(3).GetTensorRawData(),
                        c.GetInput(4).GetTensorRawData(), c.GetInput(5).GetTensorRawData(),
                        c.GetInput(6).GetTensorRawData(), out.GetTensorMutableRawData(), h.GetTensorMutableRawData(),
                        part.GetTensorMutableData<float>(), meta, R, E, I, topk, stream(c)));
}

void moe_decode(Ort::KernelContext& c, const Attrs& a) { moe_legacy(c, GGUF_LAYOUT_Q4_SPLIT, a.topk, false); }

void moe_verify(Ort::KernelContext& c, const Attrs& a) {
  if (a.iq2 == 0) return moe_legacy(c, GGUF_LAYOUT_Q4_SPLIT, a.topk, true);
  if (a.iq2 == 1) return moe_legacy(c, GGUF_LAYOUT_IQ2_CODES, a.topk, true);
  if (a.iq2 == 2) return moe_legacy(c, GGUF_LAYOUT_IQ2_NATIVE, a.topk, true);
  if (a.iq2 != 3) throw NotImplemented("MoeVerify: unknown iq2 value");
  auto z = c.GetInput(0);
  auto zs = shape(z);
  if (zs.size() != 2) throw std::invalid_argument("MoeVerify: z must be [R, 1024]");
  const int64_t R = zs[0], P = R * a.topk;
  if (R < 1 || R > 8 || P > 128) throw std::invalid_argument("MoeVerify: rows must be in [1,8] and rows*topk <= 128");
  if (zs[1] != 1024) throw std::invalid_argument("MoeVerify: latent size must be 1024");
  auto w1s = shape(c.GetInput(3));
  if (w1s.size() < 2) throw std::invalid_argument("MoeVerify: fc1_w must be [E, I, ...]");
  const int64_t E = w1s[0], I = w1s[1];
  if (I % 256 != 0 || count(c.GetInput(3)) != E * I * 4 * 66 || count(c.GetInput(5)) != E * 1024 * (I / 256) * 66)
    throw std::invalid_argument("MoeVerify: inter size alignment mismatch");
  auto out = c.GetOutput(0, {R, 1024});
  auto h = c.GetOutput(1, {P, I});
  auto part = c.GetOutput(2, {P, 1024});
  auto meta = c.GetOutput(3, {1 + 9 * P});
  check(gguf_moe_verify_iq2_xxs(z.GetTensorRawData(), c.GetInput(1).GetTensorData<int32_t>(),
                                c.GetInput(2).GetTensorData<float>(), c.GetInput(3).GetTensorRawData(),
                                c.GetInput(5).GetTensorRawData(), out.GetTensorMutableRawData(),
                                h.GetTensorMutableRawData(), part.GetTensorMutableData<float>(),
                                meta.GetTensorMutableData<int32_t>(), R, E, I, a.topk, stream(c)));
}

void q8_embed(Ort::KernelContext& c, const Attrs&) {
  auto w = c.GetInput(0);
  auto ids = c.GetInput(1);
  const auto ws = shape(w);
  const int64_t vocab = ws.empty() ? 0 : ws[0];
  if (vocab <= 0 || count(w) % vocab != 0) throw std::invalid_argument("Q8Embed: invalid weight shape");
  const int64_t row_bytes = count(w) / vocab;
  if (row_bytes <= 0 || row_bytes % 34 != 0)
    throw std::invalid_argument("Q8Embed: row_bytes must be a positive multiple of 34");
  auto os = shape(ids);
  os.push_back(row_bytes / 34 * 32);
  auto out = c.GetOutput(0, os);
  check(gguf_q8_0_embed(w.GetTensorRawData(), ids.GetTensorData<int64_t>(), out.GetTensorMutableRawData(), vocab,
                        row_bytes, count(ids), stream(c)));
}

template <bool kSkip>
void rms_norm(Ort::KernelContext& c, const Attrs& a) {
  auto x = c.GetInput(0);
  auto xs = shape(x);
  if (xs.empty()) throw std::invalid_argument("RmsNorm: input must be at least 1D");
  const int64_t H = xs.back();
  if (H <= 0 || H % 8 != 0) throw std::invalid_argument("RmsNorm: hidden size H must be a positive multiple of 8");
  if (kSkip && count(c.GetInput(1)) != count(x)) throw std::invalid_argument("SkipRmsNorm: skip shape mismatch");
  auto gamma = c.GetInput(kSkip ? 2 : 1);
  if (count(gamma) != H) throw std::invalid_argument("RmsNorm: gamma size mismatch");
  auto y = c.GetOutput(0, xs);
  void* sum = nullptr;
  if (kSkip && c.GetOutputCount() > 1) {
    auto so = c.GetOutput(1, xs);
    if (so) sum = so.GetTensorMutableRawData();
  }
  check(gguf_rms_norm(x.GetTensorRawData(), kSkip ? c.GetInput(1).GetTensorRawData() : nullptr,
                      gamma.GetTensorData<float>(), y.GetTensorMutableRawData(), sum, count(x) / H, H, a.epsilon,
                      stream(c)));
}

// Mamba*: 9 inputs (+ state_row for Verify), 5 outputs shaped as the reference (src/bolt_ops.cu:319-370).
template <bool kVerify, bool kF32W>
void mamba(Ort::KernelContext& c, const Attrs& a) {
  auto proj = c.GetInput(0);
  auto ps = shape(proj);
  if (ps.size() != 2) throw std::invalid_argument("MambaStep: proj must be [R, width]");
  const int64_t R = ps[0], di = a.heads * a.head_dim, cd = di + 2 * a.n_groups * a.d_state;
  if (R < 1 || R > 16) throw std::invalid_argument("MambaStep: rows must be in [1,16]");
  if (ps[1] != di + cd + a.heads) throw std::invalid_argument("MambaStep: bad proj width");
  const auto cs = shape(c.GetInput(1)), ss = shape(c.GetInput(2));
  if (cs.empty()) throw std::invalid_argument("MambaStep: bad conv state");
  auto y = c.GetOutput(0, {R, di});
  auto conv_out = c.GetOutput(1, cs);
  auto ssm_out = c.GetOutput(2, ss);
  auto xbc = c.GetOutput(3, {R, cd});
  auto ypre = c.GetOutput(4, {R, di});
  check(gguf_mamba_step(proj.GetTensorRawData(), c.GetInput(1).GetTensorRawData(), c.GetInput(2).GetTensorData<float>(),
                        c.GetInput(3).GetTensorRawData(), c.GetInput(4).GetTensorRawData(), kF32W ? 1 : 0,
                        c.GetInput(5).GetTensorData<float>(), c.GetInput(6).GetTensorData<float>(),
                        c.GetInput(7).GetTensorData<float>(), c.GetInput(8).GetTensorData<float>(),
                        kVerify ? c.GetInput(9).GetTensorData<int32_t>() : nullptr, y.GetTensorMutableRawData(),
                        conv_out.GetTensorMutableRawData(), ssm_out.GetTensorMutableData<float>(),
                        xbc.GetTensorMutableRawData(), ypre.GetTensorMutableData<float>(), R, cs[0], a.heads,
                        a.head_dim, a.d_state, a.n_groups, a.epsilon, a.time_step_min, stream(c)));
}

// Required attributes of the Mamba ops (src/bolt_ops.cu:311-316).
const std::vector<const char*> kMambaInt = {"heads", "head_dim", "d_state", "n_groups"};
const std::vector<const char*> kMambaFloat = {"epsilon", "time_step_min"};

// Names, signatures, optional inputs and required attributes of the reference's 15 ops
// (src/bolt_ops.cu:1886-2061; attributes read with GetAttribute at :311-316, :519-520, :669, :1333;
// gguf / iq2 / RmsNorm's epsilon are optional there, :1319-1326, :1819-1823).
const std::vector<OpDesc>& op_table() {
  static const std::vector<OpDesc> t = {
      {"MambaStep", {kBF, kBF, kF32, kBF, kBF, kF32, kF32, kF32, kF32}, {kBF, kBF, kF32, kBF, kF32}, {}, mamba<false, false>,
       {}, kMambaInt, kMambaFloat},
      {"MambaStepGGUF", {kBF, kBF, kF32, kF32, kF32, kF32, kF32, kF32, kF32}, {kBF, kBF, kF32, kBF, kF32}, {},
       mamba<false, true>, {}, kMambaInt, kMambaFloat},
      {"MambaVerify", {kBF, kBF, kF32, kBF, kBF, kF32, kF32, kF32, kF32, kI32}, {kBF, kBF, kF32, kBF, kF32}, {},
       mamba<true, false>, {}, kMambaInt, kMambaFloat},
      {"MambaVerifyGGUF", {kBF, kBF, kF32, kF32, kF32, kF32, kF32, kF32, kF32, kI32}, {kBF, kBF, kF32, kBF, kF32}, {},
       mamba<true, true>, {}, kMambaInt, kMambaFloat},
      {"MoeRoute", {kBF, kBF, kF32}, {kI32, kF32, kF32}, {}, route_bf16, {}, {"topk"}, {"scale"}},
      {"MoeRouteGGUF", {kBF, kF32, kF32}, {kI32, kF32, kF32}, {}, route_gguf, {}, {"topk"}, {"scale"}},
      {"MoeDecode", {kBF, kI32, kF32, kU8, kBF, kU8, kBF}, {kBF, kBF, kF32}, {}, moe_decode, {}, {"topk"}},
      {"MoeVerify", {kBF, kI32, kF32, kU8, kBF, kU8, kBF}, {kBF, kBF, kF32, kI32}, {4, 6}, moe_verify, {}, {"topk"}},
      {"Relu2", {kBF}, {kBF}, {}, relu2},
      {"Nvfp4Gemv", {kBF, kU8, kU8, kF32}, {kBF}, {2}, fp4_gemv},
      {"Q8Gemv", {kBF, kU8, kBF}, {kBF}, {2}, q8_gemv},
      {"Q4Gemv", {kBF, kU8, kBF}, {kBF}, {2}, q4_gemv},
      {"Q8Embed", {kU8, kI64}, {kBF}, {}, q8_embed},
      {"RmsNorm", {kBF, kF32}, {kBF}, {}, rms_norm<false>},
      {"SkipRmsNorm", {kBF, kBF, kF32}, {kBF, kBF}, {}, rms_norm<true>, {1}},
  };
  return t;
}

struct GgufKernel {
  const OpDesc* d;
  Attrs a;
  OrtStatus* ComputeV2(OrtKernelContext* raw) noexcept {
    const OrtApi& api = Ort::GetApi();
    try {
      if (d->compute == nullptr)
        throw NotImplemented(std::string(d->name) + ": not part of the GGUF decode path implemented by this library");
      Ort::KernelContext c(raw);
      d->compute(c, a);
      return nullptr;
    } catch (const NotImplemented& e) {
      return api.CreateStatus(ORT_NOT_IMPLEMENTED, e.what());
    } catch (const std::exception& e) {
      return api.CreateStatus(ORT_FAIL, e.what());
    }
  }
};

struct GgufOp : Ort::CustomOpBase<GgufOp, GgufKernel, true> {
  explicit GgufOp(const OpDesc* desc) : d(desc) {}
  const OpDesc* d;
  const char* GetName() const { return d->name; }
  const char* GetExecutionProviderType() const { return "CUDAExecutionProvider"; }
  size_t GetInputTypeCount() const { return d->in.size(); }
  ONNXTensorElementDataType GetInputType(size_t i) const { return d->in[i]; }
  size_t GetOutputTypeCount() const { return d->out.size(); }
  ONNXTensorElementDataType GetOutputType(size_t i) const { return d->out[i]; }
  OrtCustomOpInputOutputCharacteristic GetInputCharacteristic(size_t i) const {
    for (int o : d->optional_in)
      if (static_cast<size_t>(o) == i) return INPUT_OUTPUT_OPTIONAL;
    return INPUT_OUTPUT_REQUIRED;
  }
  OrtCustomOpInputOutputCharacteristic GetOutputCharacteristic(size_t i) const {
    for (int o : d->optional_out)
      if (static_cast<size_t>(o) == i) return INPUT_OUTPUT_OPTIONAL;
    return INPUT_OUTPUT_REQUIRED;
  }
  OrtStatus* CreateKernelV2(const OrtApi& api, const OrtKernelInfo* info, void** kernel) const noexcept {
    try {
      for (const char* n : d->req_int)
        if (!has_int(info, n)) throw std::invalid_argument(std::string(d->name) + ": missing required attribute '" + n + "'");
      for (const char* n : d->req_float)
        if (!has_float(info, n)) throw std::invalid_argument(std::string(d->name) + ": missing required attribute '" + n + "'");
      if (std::string(d->name).rfind("Mamba", 0) == 0 &&
          (opt_int(info, "head_dim", 0) != 64 || opt_int(info, "d_state", 0) != 128))
        throw std::invalid_argument("MambaStep: only head_dim=64, d_state=128 are implemented");
      auto* k = new GgufKernel{d, {}};
      k->a.gguf = opt_int(info, "gguf", 0);
      k->a.iq2 = opt_int(info, "iq2", 0);
      k->a.topk = opt_int(info, "topk", 0);
      k->a.scale = opt_float(info, "scale", 1.0f);
      k->a.epsilon = opt_float(info, "epsilon", 1e-5f);
      k->a.heads = opt_int(info, "heads", 0);
      k->a.head_dim = opt_int(info, "head_dim", 0);
      k->a.d_state = opt_int(info, "d_state", 0);
      k->a.n_groups = opt_int(info, "n_groups", 0);
      k->a.time_step_min = opt_float(info, "time_step_min", 0.0f);
      *kernel = k;
      return nullptr;
    } catch (const std::exception& e) {
      return api.CreateStatus(ORT_INVALID_ARGUMENT, e.what());
    }
  }
};

}  // namespace

extern "C" __attribute__((visibility("default"))) OrtStatus* ORT_API_CALL RegisterCustomOps(OrtSessionOptions* options,
                                                                                          const OrtApiBase* api_base) {
  // API version 22 first (the version the reference library is built against), then the headers'
  // own version (src/bolt_ops.cu:2066-2068)
  const OrtApi* api = api_base->GetApi(22);
  if (api == nullptr) api = api_base->GetApi(ORT_API_VERSION);
  if (api == nullptr) return api_base->GetApi(1)->CreateStatus(ORT_FAIL, "Unsupported ORT API");
  Ort::InitApi(api);
  try {
    static std::vector<GgufOp> ops;
    static Ort::CustomOpDomain bolt("bolt");
    static Ort::CustomOpDomain gguf("gguf");
    static std::once_flag once;
    std::call_once(once, [] {
      const auto& t = op_table();
      ops.reserve(t.size());
      for (const auto& d : t) ops.emplace_back(&d);
      for (auto& op : ops) {
        bolt.Add(&op);
        gguf.Add(&op);
      }
    });
    Ort::UnownedSessionOptions so(options);
    so.Add(bolt);
    so.Add(gguf);
    return nullptr;
  } catch (const std::exception& e) {
    return api->CreateStatus(ORT_FAIL, e.what());
  }
}
