// Minimal stand-in for the ONNX Runtime custom-op API (C table + C++ wrappers) -- TEST
// INFRASTRUCTURE, not part of the product.
//
// There is no onnxruntime in this environment.  This header restates, from their call sites,
// only the ORT entities that two translation units use:
//   * the reference's src/bolt_ops.cu (tianleiwu/nemotron_ops): Ort::KernelContext / ConstValue /
//     UnownedValue / ConstKernelInfo / CustomOpBase<Op, State, true> / CustomOpDomain /
//     UnownedSessionOptions / InitApi / ThrowOnError and OrtApi::{CreateStatus,
//     KernelContext_GetGPUComputeStream} (src/bolt_ops.cu:29-61, :1469-1625);
//   * this repository's ORT adapter, nemotron_ops_b200/ort/bolt_ort.cc, which uses the same subset.
// Both compile against it unchanged, and ort_host.cc (the "session" side) implements the OrtApi
// table, so the tests can load either library, call RegisterCustomOps and run its kernels on
// device buffers.  The names and the C++ surface follow ONNX Runtime's; the binary layout of the
// tables is this header's own (libraries built against it load only into ort_host.cc).
#pragma once

#include <cstddef>
#include <cstdint>
#include <stdexcept>
#include <string>
#include <vector>

#define ORT_API_VERSION 22
#define ORT_API_CALL

typedef enum OrtErrorCode { ORT_OK = 0, ORT_FAIL = 1, ORT_INVALID_ARGUMENT = 2 } OrtErrorCode;

// ONNX element type codes (TensorProto.DataType)
typedef enum ONNXTensorElementDataType {
  ONNX_TENSOR_ELEMENT_DATA_TYPE_UNDEFINED = 0,
  ONNX_TENSOR_ELEMENT_DATA_TYPE_FLOAT = 1,
  ONNX_TENSOR_ELEMENT_DATA_TYPE_UINT8 = 2,
  ONNX_TENSOR_ELEMENT_DATA_TYPE_INT32 = 6,
  ONNX_TENSOR_ELEMENT_DATA_TYPE_FLOAT16 = 10,
  ONNX_TENSOR_ELEMENT_DATA_TYPE_BFLOAT16 = 16,
} ONNXTensorElementDataType;

typedef enum OrtCustomOpInputOutputCharacteristic {
  INPUT_OUTPUT_REQUIRED = 0,
  INPUT_OUTPUT_OPTIONAL = 1,
  INPUT_OUTPUT_VARIADIC = 2,
} OrtCustomOpInputOutputCharacteristic;

// opaque objects owned by the session side (ort_host.cc)
struct OrtStatus;
struct OrtKernelContext;
struct OrtKernelInfo;
struct OrtSessionOptions;
struct OrtCustomOpDomain;
struct OrtValue;
struct OrtCustomOp;

struct OrtApi {
  OrtStatus* (*CreateStatus)(OrtErrorCode code, const char* msg);
  OrtErrorCode (*GetErrorCode)(const OrtStatus* status);
  const char* (*GetErrorMessage)(const OrtStatus* status);
  void (*ReleaseStatus)(OrtStatus* status);
  OrtStatus* (*KernelContext_GetInput)(const OrtKernelContext* context, size_t index, const OrtValue** out);
  OrtStatus* (*KernelContext_GetOutput)(OrtKernelContext* context, size_t index, const int64_t* dims,
                                        size_t dim_count, OrtValue** out);
  OrtStatus* (*KernelContext_GetGPUComputeStream)(const OrtKernelContext* context, void** out);
  OrtStatus* (*GetTensorMutableData)(OrtValue* value, void** out);
  OrtStatus* (*GetTensorShape)(const OrtValue* value, const int64_t** dims, size_t* dim_count);
  OrtStatus* (*KernelInfoGetAttribute_int64)(const OrtKernelInfo* info, const char* name, int64_t* out);
  OrtStatus* (*KernelInfoGetAttribute_float)(const OrtKernelInfo* info, const char* name, float* out);
  OrtStatus* (*CreateCustomOpDomain)(const char* domain, OrtCustomOpDomain** out);
  OrtStatus* (*CustomOpDomain_Add)(OrtCustomOpDomain* domain, const OrtCustomOp* op);
  OrtStatus* (*AddCustomOpDomain)(OrtSessionOptions* options, OrtCustomOpDomain* domain);
};

struct OrtApiBase {
  const OrtApi* (*GetApi)(uint32_t version);
  const char* (*GetVersionString)();
};

// A custom op as the session sees it: a table of callbacks (filled by Ort::CustomOpBase).
struct OrtCustomOp {
  uint32_t version;
  const char* (*GetName)(const OrtCustomOp* op);
  const char* (*GetExecutionProviderType)(const OrtCustomOp* op);
  size_t (*GetInputTypeCount)(const OrtCustomOp* op);
  ONNXTensorElementDataType (*GetInputType)(const OrtCustomOp* op, size_t index);
  size_t (*GetOutputTypeCount)(const OrtCustomOp* op);
  ONNXTensorElementDataType (*GetOutputType)(const OrtCustomOp* op, size_t index);
  OrtCustomOpInputOutputCharacteristic (*GetInputCharacteristic)(const OrtCustomOp* op, size_t index);
  OrtCustomOpInputOutputCharacteristic (*GetOutputCharacteristic)(const OrtCustomOp* op, size_t index);
  OrtStatus* (*CreateKernelV2)(const OrtCustomOp* op, const OrtApi* api, const OrtKernelInfo* info, void** kernel);
  OrtStatus* (*KernelComputeV2)(void* kernel, OrtKernelContext* context);
  void (*KernelDestroy)(void* kernel);
};

namespace Ort {

inline const OrtApi*& global_api() {
  static const OrtApi* api = nullptr;
  return api;
}
inline void InitApi(const OrtApi* api) { global_api() = api; }
inline const OrtApi& GetApi() { return *global_api(); }

struct Exception : std::runtime_error {
  Exception(const std::string& msg, OrtErrorCode code) : std::runtime_error(msg), code_(code) {}
  OrtErrorCode GetOrtErrorCode() const { return code_; }
  OrtErrorCode code_;
};

inline void ThrowOnError(OrtStatus* status) {
  if (status == nullptr) return;
  const std::string msg = GetApi().GetErrorMessage(status);
  const OrtErrorCode code = GetApi().GetErrorCode(status);
  GetApi().ReleaseStatus(status);
  throw Exception(msg, code);
}

struct TensorTypeAndShapeInfo {
  std::vector<int64_t> shape;
  std::vector<int64_t> GetShape() const { return shape; }
  size_t GetElementCount() const {
    size_t n = 1;
    for (int64_t d : shape) n *= static_cast<size_t>(d);
    return n;
  }
};

inline TensorTypeAndShapeInfo shape_of(const OrtValue* v) {
  const int64_t* dims = nullptr;
  size_t n = 0;
  ThrowOnError(GetApi().GetTensorShape(v, &dims, &n));
  return TensorTypeAndShapeInfo{std::vector<int64_t>(dims, dims + n)};
}

struct ConstValue {
  const OrtValue* p_;
  explicit ConstValue(const OrtValue* p) : p_(p) {}
  const void* GetTensorRawData() const {
    void* d = nullptr;
    ThrowOnError(GetApi().GetTensorMutableData(const_cast<OrtValue*>(p_), &d));
    return d;
  }
  TensorTypeAndShapeInfo GetTensorTypeAndShapeInfo() const { return shape_of(p_); }
};

struct UnownedValue {
  OrtValue* p_;
  explicit UnownedValue(OrtValue* p) : p_(p) {}
  void* GetTensorMutableRawData() {
    void* d = nullptr;
    ThrowOnError(GetApi().GetTensorMutableData(p_, &d));
    return d;
  }
  TensorTypeAndShapeInfo GetTensorTypeAndShapeInfo() const { return shape_of(p_); }
};

struct KernelContext {
  OrtKernelContext* ctx_;
  explicit KernelContext(OrtKernelContext* ctx) : ctx_(ctx) {}
  ConstValue GetInput(size_t index) const {
    const OrtValue* v = nullptr;
    ThrowOnError(GetApi().KernelContext_GetInput(ctx_, index, &v));
    return ConstValue(v);
  }
  UnownedValue GetOutput(size_t index, const int64_t* dims, size_t dim_count) const {
    OrtValue* v = nullptr;
    ThrowOnError(GetApi().KernelContext_GetOutput(ctx_, index, dims, dim_count, &v));
    return UnownedValue(v);
  }
  UnownedValue GetOutput(size_t index, const std::vector<int64_t>& dims) const {
    return GetOutput(index, dims.data(), dims.size());
  }
  void* GetGPUComputeStream() const {
    void* s = nullptr;
    ThrowOnError(GetApi().KernelContext_GetGPUComputeStream(ctx_, &s));
    return s;
  }
};

struct ConstKernelInfo {
  const OrtKernelInfo* info_;
  explicit ConstKernelInfo(const OrtKernelInfo* info) : info_(info) {}
  template <typename T>
  T GetAttribute(const char* name) const;
};
template <>
inline int64_t ConstKernelInfo::GetAttribute<int64_t>(const char* name) const {
  int64_t v = 0;
  ThrowOnError(GetApi().KernelInfoGetAttribute_int64(info_, name, &v));
  return v;
}
template <>
inline float ConstKernelInfo::GetAttribute<float>(const char* name) const {
  float v = 0.f;
  ThrowOnError(GetApi().KernelInfoGetAttribute_float(info_, name, &v));
  return v;
}

// CRTP base that fills the OrtCustomOp table from TOp's methods; with WithStatus the kernel is
// created by TOp::CreateKernelV2 and run by TKernel::ComputeV2, both returning OrtStatus*.
template <typename TOp, typename TKernel, bool WithStatus = false>
struct CustomOpBase : OrtCustomOp {
  static_assert(WithStatus, "only the status-returning (V2) kernel interface is provided");
  CustomOpBase() {
    OrtCustomOp::version = ORT_API_VERSION;
    OrtCustomOp::GetName = [](const OrtCustomOp* op) { return static_cast<const TOp*>(op)->GetName(); };
    OrtCustomOp::GetExecutionProviderType = [](const OrtCustomOp* op) {
      return static_cast<const TOp*>(op)->GetExecutionProviderType();
    };
    OrtCustomOp::GetInputTypeCount = [](const OrtCustomOp* op) { return static_cast<const TOp*>(op)->GetInputTypeCount(); };
    OrtCustomOp::GetInputType = [](const OrtCustomOp* op, size_t i) { return static_cast<const TOp*>(op)->GetInputType(i); };
    OrtCustomOp::GetOutputTypeCount = [](const OrtCustomOp* op) {
      return static_cast<const TOp*>(op)->GetOutputTypeCount();
    };
    OrtCustomOp::GetOutputType = [](const OrtCustomOp* op, size_t i) { return static_cast<const TOp*>(op)->GetOutputType(i); };
    OrtCustomOp::GetInputCharacteristic = [](const OrtCustomOp* op, size_t i) {
      return static_cast<const TOp*>(op)->GetInputCharacteristic(i);
    };
    OrtCustomOp::GetOutputCharacteristic = [](const OrtCustomOp* op, size_t i) {
      return static_cast<const TOp*>(op)->GetOutputCharacteristic(i);
    };
    OrtCustomOp::CreateKernelV2 = [](const OrtCustomOp* op, const OrtApi* api, const OrtKernelInfo* info,
                                     void** kernel) -> OrtStatus* {
      return static_cast<const TOp*>(op)->CreateKernelV2(*api, info, kernel);
    };
    OrtCustomOp::KernelComputeV2 = [](void* kernel, OrtKernelContext* ctx) -> OrtStatus* {
      return static_cast<TKernel*>(kernel)->ComputeV2(ctx);
    };
    OrtCustomOp::KernelDestroy = [](void* kernel) { delete static_cast<TKernel*>(kernel); };
  }
  const char* GetExecutionProviderType() const { return nullptr; }
  OrtCustomOpInputOutputCharacteristic GetInputCharacteristic(size_t) const { return INPUT_OUTPUT_REQUIRED; }
  OrtCustomOpInputOutputCharacteristic GetOutputCharacteristic(size_t) const { return INPUT_OUTPUT_REQUIRED; }
};

struct CustomOpDomain {
  OrtCustomOpDomain* p_ = nullptr;
  explicit CustomOpDomain(const char* name) { ThrowOnError(GetApi().CreateCustomOpDomain(name, &p_)); }
  void Add(const OrtCustomOp* op) { ThrowOnError(GetApi().CustomOpDomain_Add(p_, op)); }
  operator OrtCustomOpDomain*() const { return p_; }
};

struct UnownedSessionOptions {
  OrtSessionOptions* p_;
  explicit UnownedSessionOptions(OrtSessionOptions* p) : p_(p) {}
  UnownedSessionOptions& Add(OrtCustomOpDomain* domain) {
    ThrowOnError(GetApi().AddCustomOpDomain(p_, domain));
    return *this;
  }
};

}  // namespace Ort
