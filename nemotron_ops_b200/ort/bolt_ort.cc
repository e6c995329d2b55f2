// ONNX Runtime adapter of libbolt_b200.so: exports RegisterCustomOps, which registers the custom-op
// domain "bolt" with the reference's op set -- MambaStep, MambaVerify, MoeRoute, MoeDecode,
// MoeVerify, Relu2, Nvfp4Gemv, Q8Gemv, Q4Gemv -- with the same input / output element types,
// attributes and execution provider as the reference's registration (src/bolt_ops.cu:1469-1625),
// so a model exported for the reference loads this library unchanged (SessionOptions
// .register_custom_ops_library).  Each kernel reads its ORT tensors, allocates its outputs with
// KernelContext::GetOutput in the shapes the reference allocates, and calls the matching bolt_*
// entry point of include/bolt_b200.h on the EP's compute stream.  Nothing here computes.
//
// Status mapping as in the reference: a kernel constructor that throws (missing attribute,
// unsupported head_dim / d_state) -> ORT_INVALID_ARGUMENT from CreateKernelV2; a failing compute
// (shape check, launch error) -> ORT_FAIL with the bolt_last_error() text.
//
// Build: compiled only when ONNX Runtime's headers are available (ORT_INCLUDE_DIR, as the
// reference's CMakeLists.txt), linked against libbolt_b200.so (python -m nemotron_ops_b200.build).
#include <cstdint>
#include <mutex>
#include <stdexcept>
#include <string>
#include <vector>

#include "bolt_b200.h"
#include "onnxruntime_cxx_api.h"

namespace {

using Dims = std::vector<int64_t>;

Dims dims_of(const Ort::ConstValue& v) { return v.GetTensorTypeAndShapeInfo().GetShape(); }

int64_t dim(const Dims& d, size_t i) {
  if (i >= d.size()) throw std::invalid_argument("bolt: input has too few dimensions");
  return d[i];
}

void* compute_stream(const OrtApi& api, OrtKernelContext* ctx) {
  void* s = nullptr;
  Ort::ThrowOnError(api.KernelContext_GetGPUComputeStream(ctx, &s));
  return s;
}

void check(int rc) {
  if (rc != BOLT_OK) throw std::runtime_error(bolt_last_error());
}

// custom-op attributes are not declared, so an optional one is probed (absent -> default)
int64_t optional_int(const OrtKernelInfo* info, const char* name, int64_t def) {
  try {
    return Ort::ConstKernelInfo(info).GetAttribute<int64_t>(name);
  } catch (...) {
    return def;
  }
}

const void* in(Ort::KernelContext& c, size_t i) { return c.GetInput(i).GetTensorRawData(); }

// Every kernel: ComputeV2 runs Body under the reference's error mapping.
struct KernelBase {
  const OrtApi& api;
  explicit KernelBase(const OrtApi& a) : api(a) {}
  template <typename F>
  OrtStatus* guarded(F&& body) noexcept {
    try {
      body();
      return nullptr;
    } catch (const std::exception& e) {
      return api.CreateStatus(ORT_FAIL, e.what());
    } catch (...) {
      return api.CreateStatus(ORT_FAIL, "bolt: unknown error");
    }
  }
};

// ---- GEMVs: y takes x's shape with the last dimension replaced by N ---------------------------
struct Nvfp4GemvKernel : KernelBase {
  Nvfp4GemvKernel(const OrtApi& a, const OrtKernelInfo*) : KernelBase(a) {}
  OrtStatus* ComputeV2(OrtKernelContext* raw) noexcept {
    return guarded([&] {
      Ort::KernelContext c(raw);
      const Dims xd = dims_of(c.GetInput(0)), wd = dims_of(c.GetInput(1));
      Dims yd = xd;
      if (yd.empty()) throw std::invalid_argument("Nvfp4Gemv: x needs at least one dimension");
      yd.back() = dim(wd, 0);
      auto y = c.GetOutput(0, yd);
      check(bolt_nvfp4_gemv(in(c, 0), xd.data(), static_cast<int>(xd.size()), in(c, 1), wd.data(),
                            static_cast<int>(wd.size()), in(c, 2), in(c, 3), y.GetTensorMutableRawData(),
                            compute_stream(api, raw)));
    });
  }
};

template <int BITS>
struct QGemvKernel : KernelBase {
  int64_t iq2;
  QGemvKernel(const OrtApi& a, const OrtKernelInfo* info)
      : KernelBase(a), iq2(BITS == 4 ? optional_int(info, "iq2", 0) : 0) {}
  OrtStatus* ComputeV2(OrtKernelContext* raw) noexcept {
    return guarded([&] {
      Ort::KernelContext c(raw);
      const Dims xd = dims_of(c.GetInput(0)), bd = dims_of(c.GetInput(1));
      Dims yd = xd;
      if (yd.empty()) throw std::invalid_argument("QGemv: x needs at least one dimension");
      yd.back() = dim(bd, 0);
      auto y = c.GetOutput(0, yd);
      void* s = compute_stream(api, raw);
      if (BITS == 8)
        check(bolt_q8_gemv(in(c, 0), xd.data(), static_cast<int>(xd.size()), in(c, 1), bd.data(),
                           static_cast<int>(bd.size()), in(c, 2), y.GetTensorMutableRawData(), s));
      else
        check(bolt_q4_gemv(in(c, 0), xd.data(), static_cast<int>(xd.size()), in(c, 1), bd.data(),
                           static_cast<int>(bd.size()), in(c, 2), iq2, y.GetTensorMutableRawData(), s));
    });
  }
};

// ---- MoE -----------------------------------------------------------------------------------
struct MoeRouteKernel : KernelBase {
  int64_t topk;
  float scale;
  MoeRouteKernel(const OrtApi& a, const OrtKernelInfo* info) : KernelBase(a) {
    Ort::ConstKernelInfo k(info);
    topk = k.GetAttribute<int64_t>("topk");
    scale = k.GetAttribute<float>("scale");
  }
  OrtStatus* ComputeV2(OrtKernelContext* raw) noexcept {
    return guarded([&] {
      Ort::KernelContext c(raw);
      const Dims xd = dims_of(c.GetInput(0)), gd = dims_of(c.GetInput(1));
      const int64_t R = dim(xd, 0), E = dim(gd, 0);
      auto idx = c.GetOutput(0, Dims{R, topk});
      auto w = c.GetOutput(1, Dims{R, topk});
      auto scores = c.GetOutput(2, Dims{R, E});
      check(bolt_moe_route(in(c, 0), xd.data(), static_cast<int>(xd.size()), in(c, 1), gd.data(),
                           static_cast<int>(gd.size()), in(c, 2), topk, scale, idx.GetTensorMutableRawData(),
                           w.GetTensorMutableRawData(), scores.GetTensorMutableRawData(), compute_stream(api, raw)));
    });
  }
};

// MoeDecode (verify = false) and MoeVerify (verify = true): out [R, 1024], h [R*topk, I],
// part [R*topk, 1024] (+ meta [1 + P + 8P] for MoeVerify)
template <bool VERIFY>
struct MoeKernel : KernelBase {
  int64_t topk, iq2;
  MoeKernel(const OrtApi& a, const OrtKernelInfo* info) : KernelBase(a) {
    topk = Ort::ConstKernelInfo(info).GetAttribute<int64_t>("topk");
    iq2 = VERIFY ? optional_int(info, "iq2", 0) : 0;
  }
  OrtStatus* ComputeV2(OrtKernelContext* raw) noexcept {
    return guarded([&] {
      Ort::KernelContext c(raw);
      const Dims zd = dims_of(c.GetInput(0)), w1d = dims_of(c.GetInput(3));
      const int64_t R = dim(zd, 0), I = dim(w1d, 1), P = R * topk;
      auto out = c.GetOutput(0, Dims{R, 1024});
      auto h = c.GetOutput(1, Dims{P, I});
      auto part = c.GetOutput(2, Dims{P, 1024});
      void* s = compute_stream(api, raw);
      if (VERIFY) {
        auto meta = c.GetOutput(3, Dims{1 + P + 8 * P});
        check(bolt_moe_verify(in(c, 0), zd.data(), static_cast<int>(zd.size()), in(c, 1), in(c, 2), in(c, 3),
                              w1d.data(), static_cast<int>(w1d.size()), in(c, 4), in(c, 5), in(c, 6), topk, iq2,
                              out.GetTensorMutableRawData(), h.GetTensorMutableRawData(),
                              part.GetTensorMutableRawData(), meta.GetTensorMutableRawData(), s));
      } else {
        check(bolt_moe_decode(in(c, 0), zd.data(), static_cast<int>(zd.size()), in(c, 1), in(c, 2), in(c, 3),
                              w1d.data(), static_cast<int>(w1d.size()), in(c, 4), in(c, 5), in(c, 6), topk,
                              out.GetTensorMutableRawData(), h.GetTensorMutableRawData(),
                              part.GetTensorMutableRawData(), s));
      }
    });
  }
};

// ---- Relu2: y takes x's shape ----------------------------------------------------------------
struct Relu2Kernel : KernelBase {
  Relu2Kernel(const OrtApi& a, const OrtKernelInfo*) : KernelBase(a) {}
  OrtStatus* ComputeV2(OrtKernelContext* raw) noexcept {
    return guarded([&] {
      Ort::KernelContext c(raw);
      const Dims xd = dims_of(c.GetInput(0));
      auto y = c.GetOutput(0, xd);
      check(bolt_relu2(in(c, 0), xd.data(), static_cast<int>(xd.size()), y.GetTensorMutableRawData(),
                       compute_stream(api, raw)));
    });
  }
};

// ---- MambaStep / MambaVerify ----------------------------------------------------------------
template <bool VERIFY>
struct MambaKernel : KernelBase {
  int64_t heads, hd, ds, ng;
  float eps, tmin;
  MambaKernel(const OrtApi& a, const OrtKernelInfo* info) : KernelBase(a) {
    Ort::ConstKernelInfo k(info);
    heads = k.GetAttribute<int64_t>("heads");
    hd = k.GetAttribute<int64_t>("head_dim");
    ds = k.GetAttribute<int64_t>("d_state");
    ng = k.GetAttribute<int64_t>("n_groups");
    eps = k.GetAttribute<float>("epsilon");
    tmin = k.GetAttribute<float>("time_step_min");
    if (hd != 64 || ds != 128) throw std::invalid_argument("MambaStep: only head_dim=64, d_state=128 are implemented");
  }
  OrtStatus* ComputeV2(OrtKernelContext* raw) noexcept {
    return guarded([&] {
      Ort::KernelContext c(raw);
      const Dims pd = dims_of(c.GetInput(0)), cd = dims_of(c.GetInput(1)), sd = dims_of(c.GetInput(2));
      const int64_t R = dim(pd, 0), di = heads * hd, conv_dim = di + 2 * ng * ds;
      auto y = c.GetOutput(0, Dims{R, di});
      auto conv_out = c.GetOutput(1, cd);
      auto ssm_out = c.GetOutput(2, sd);
      auto xbc = c.GetOutput(3, Dims{R, conv_dim});
      auto ypre = c.GetOutput(4, Dims{R, di});
      void* s = compute_stream(api, raw);
      if (VERIFY)
        check(bolt_mamba_verify(in(c, 0), pd.data(), static_cast<int>(pd.size()), in(c, 1), cd.data(),
                                static_cast<int>(cd.size()), in(c, 2), sd.data(), static_cast<int>(sd.size()),
                                in(c, 3), in(c, 4), in(c, 5), in(c, 6), in(c, 7), in(c, 8), in(c, 9), heads, hd, ds,
                                ng, eps, tmin, y.GetTensorMutableRawData(), conv_out.GetTensorMutableRawData(),
                                ssm_out.GetTensorMutableRawData(), xbc.GetTensorMutableRawData(),
                                ypre.GetTensorMutableRawData(), s));
      else
        check(bolt_mamba_step(in(c, 0), pd.data(), static_cast<int>(pd.size()), in(c, 1), cd.data(),
                              static_cast<int>(cd.size()), in(c, 2), sd.data(), static_cast<int>(sd.size()),
                              in(c, 3), in(c, 4), in(c, 5), in(c, 6), in(c, 7), in(c, 8), heads, hd, ds, ng, eps,
                              tmin, y.GetTensorMutableRawData(), conv_out.GetTensorMutableRawData(),
                              ssm_out.GetTensorMutableRawData(), xbc.GetTensorMutableRawData(),
                              ypre.GetTensorMutableRawData(), s));
    });
  }
};

// ---- registration ----------------------------------------------------------------------------
constexpr auto kBf = ONNX_TENSOR_ELEMENT_DATA_TYPE_BFLOAT16;
constexpr auto kF32 = ONNX_TENSOR_ELEMENT_DATA_TYPE_FLOAT;
constexpr auto kU8 = ONNX_TENSOR_ELEMENT_DATA_TYPE_UINT8;
constexpr auto kI32 = ONNX_TENSOR_ELEMENT_DATA_TYPE_INT32;

// One op: its name, element types and kernel type; the kernel is created per node.
template <typename Kernel, const char* Name, size_t NIn, size_t NOut>
struct BoltOpDef : Ort::CustomOpBase<BoltOpDef<Kernel, Name, NIn, NOut>, Kernel, true> {
  ONNXTensorElementDataType in_types[NIn];
  ONNXTensorElementDataType out_types[NOut];
  BoltOpDef(std::initializer_list<ONNXTensorElementDataType> ins, std::initializer_list<ONNXTensorElementDataType> outs) {
    size_t i = 0;
    for (auto t : ins) in_types[i++] = t;
    i = 0;
    for (auto t : outs) out_types[i++] = t;
  }
  const char* GetName() const { return Name; }
  const char* GetExecutionProviderType() const { return "CUDAExecutionProvider"; }
  size_t GetInputTypeCount() const { return NIn; }
  ONNXTensorElementDataType GetInputType(size_t i) const { return in_types[i]; }
  size_t GetOutputTypeCount() const { return NOut; }
  ONNXTensorElementDataType GetOutputType(size_t i) const { return out_types[i]; }
  OrtCustomOpInputOutputCharacteristic GetInputCharacteristic(size_t) const { return INPUT_OUTPUT_REQUIRED; }
  OrtCustomOpInputOutputCharacteristic GetOutputCharacteristic(size_t) const { return INPUT_OUTPUT_REQUIRED; }
  OrtStatus* CreateKernelV2(const OrtApi& api, const OrtKernelInfo* info, void** kernel) const noexcept {
    try {
      *kernel = new Kernel(api, info);
      return nullptr;
    } catch (const std::exception& e) {
      return api.CreateStatus(ORT_INVALID_ARGUMENT, e.what());
    }
  }
};

constexpr char kMambaStep[] = "MambaStep", kMambaVerify[] = "MambaVerify", kMoeRoute[] = "MoeRoute",
               kMoeDecode[] = "MoeDecode", kMoeVerify[] = "MoeVerify", kRelu2[] = "Relu2",
               kNvfp4Gemv[] = "Nvfp4Gemv", kQ8Gemv[] = "Q8Gemv", kQ4Gemv[] = "Q4Gemv";

}  // namespace

extern "C" __attribute__((visibility("default"))) OrtStatus* ORT_API_CALL
RegisterCustomOps(OrtSessionOptions* options, const OrtApiBase* api_base) {
  const OrtApi* api = api_base->GetApi(ORT_API_VERSION);
  if (api == nullptr) return api_base->GetApi(1)->CreateStatus(ORT_FAIL, "bolt: unsupported ONNX Runtime API version");
  Ort::InitApi(api);
  try {
    // inputs / outputs in the reference's order (src/bolt_ops.cu:1489-1589)
    static BoltOpDef<MambaKernel<false>, kMambaStep, 9, 5> mamba({kBf, kBf, kF32, kBf, kBf, kF32, kF32, kF32, kF32},
                                                                 {kBf, kBf, kF32, kBf, kF32});
    static BoltOpDef<MambaKernel<true>, kMambaVerify, 10, 5> mamba_verify(
        {kBf, kBf, kF32, kBf, kBf, kF32, kF32, kF32, kF32, kI32}, {kBf, kBf, kF32, kBf, kF32});
    static BoltOpDef<MoeRouteKernel, kMoeRoute, 3, 3> route({kBf, kBf, kF32}, {kI32, kF32, kF32});
    static BoltOpDef<MoeKernel<false>, kMoeDecode, 7, 3> decode({kBf, kI32, kF32, kU8, kBf, kU8, kBf}, {kBf, kBf, kF32});
    static BoltOpDef<MoeKernel<true>, kMoeVerify, 7, 4> verify({kBf, kI32, kF32, kU8, kBf, kU8, kBf},
                                                               {kBf, kBf, kF32, kI32});
    static BoltOpDef<Relu2Kernel, kRelu2, 1, 1> relu2({kBf}, {kBf});
    static BoltOpDef<Nvfp4GemvKernel, kNvfp4Gemv, 4, 1> nvfp4({kBf, kU8, kU8, kF32}, {kBf});
    static BoltOpDef<QGemvKernel<8>, kQ8Gemv, 3, 1> q8({kBf, kU8, kBf}, {kBf});
    static BoltOpDef<QGemvKernel<4>, kQ4Gemv, 3, 1> q4({kBf, kU8, kBf}, {kBf});
    static Ort::CustomOpDomain domain("bolt");
    static std::once_flag once;
    std::call_once(once, [&] {
      for (const OrtCustomOp* op : std::initializer_list<const OrtCustomOp*>{&mamba, &mamba_verify, &route, &decode,
                                                                              &verify, &relu2, &nvfp4, &q8, &q4})
        domain.Add(op);
    });
    Ort::UnownedSessionOptions(options).Add(domain);
    return nullptr;
  } catch (const std::exception& e) {
    return api->CreateStatus(ORT_FAIL, e.what());
  }
}
