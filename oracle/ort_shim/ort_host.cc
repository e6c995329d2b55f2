// Session side of the ONNX Runtime stand-in (onnxruntime_cxx_api.h) -- TEST INFRASTRUCTURE.
//
// Loads a custom-op library (the reference's libbolt_ops built against the stand-in header, or
// this repository's ORT adapter), calls its RegisterCustomOps like an InferenceSession does, and
// runs one op at a time on caller-provided device buffers:
//   * attributes are given per kernel (int64 or float), missing ones make GetAttribute throw;
//   * inputs are (device pointer, shape); outputs are preallocated buffers with a byte
//     capacity -- GetOutput(i, dims) returns buffer i when dims fit in it and records the shape,
//     so a run allocates nothing and can be captured into a CUDA graph;
//   * the compute stream is the caller's.
// Plain C entry points (ort_shim_*) for ctypes; no CUDA calls here.
#include <dlfcn.h>

#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "onnxruntime_cxx_api.h"

struct OrtStatus {
  OrtErrorCode code;
  std::string msg;
};
struct OrtValue {
  void* data = nullptr;
  std::vector<int64_t> shape;
  int64_t capacity = -1;  // bytes (outputs)
  int elem_bytes = 1;
  bool bound = false;  // output: GetOutput was called
};
struct OrtKernelContext {
  std::vector<OrtValue> inputs, outputs;
  void* stream = nullptr;
};
struct OrtKernelInfo {
  std::map<std::string, int64_t> ints;
  std::map<std::string, float> floats;
};
struct OrtCustomOpDomain {
  std::string name;
  std::vector<const OrtCustomOp*> ops;
};
struct OrtSessionOptions {
  std::vector<OrtCustomOpDomain*> domains;
};

namespace {

thread_local std::string g_error;

OrtStatus* make_status(OrtErrorCode code, const std::string& msg) { return new OrtStatus{code, msg}; }

int elem_bytes(int type) {
  switch (type) {
    case ONNX_TENSOR_ELEMENT_DATA_TYPE_FLOAT:
    case ONNX_TENSOR_ELEMENT_DATA_TYPE_INT32: return 4;
    case ONNX_TENSOR_ELEMENT_DATA_TYPE_FLOAT16:
    case ONNX_TENSOR_ELEMENT_DATA_TYPE_BFLOAT16: return 2;
    default: return 1;
  }
}

const OrtApi g_api = {
    [](OrtErrorCode code, const char* msg) { return make_status(code, msg ? msg : ""); },
    [](const OrtStatus* s) { return s ? s->code : ORT_OK; },
    [](const OrtStatus* s) { return s ? s->msg.c_str() : ""; },
    [](OrtStatus* s) { delete s; },
    [](const OrtKernelContext* c, size_t i, const OrtValue** out) -> OrtStatus* {
      if (i >= c->inputs.size()) return make_status(ORT_FAIL, "input index out of range");
      *out = &c->inputs[i];
      return nullptr;
    },
    [](OrtKernelContext* c, size_t i, const int64_t* dims, size_t n, OrtValue** out) -> OrtStatus* {
      if (i >= c->outputs.size()) return make_status(ORT_FAIL, "output index out of range");
      OrtValue& v = c->outputs[i];
      int64_t count = 1;
      for (size_t d = 0; d < n; ++d) {
        if (dims[d] < 0) return make_status(ORT_FAIL, "negative output dimension");
        count *= dims[d];
      }
      if (count * v.elem_bytes > v.capacity)
        return make_status(ORT_FAIL, "output " + std::to_string(i) + " needs " + std::to_string(count * v.elem_bytes) +
                                         " bytes, the buffer has " + std::to_string(v.capacity));
      v.shape.assign(dims, dims + n);
      v.bound = true;
      *out = &v;
      return nullptr;
    },
    [](const OrtKernelContext* c, void** out) -> OrtStatus* {
      *out = c->stream;
      return nullptr;
    },
    [](OrtValue* v, void** out) -> OrtStatus* {
      *out = v->data;
      return nullptr;
    },
    [](const OrtValue* v, const int64_t** dims, size_t* n) -> OrtStatus* {
      *dims = v->shape.data();
      *n = v->shape.size();
      return nullptr;
    },
    [](const OrtKernelInfo* k, const char* name, int64_t* out) -> OrtStatus* {
      auto it = k->ints.find(name);
      if (it == k->ints.end()) return make_status(ORT_FAIL, std::string("no int attribute ") + name);
      *out = it->second;
      return nullptr;
    },
    [](const OrtKernelInfo* k, const char* name, float* out) -> OrtStatus* {
      auto it = k->floats.find(name);
      if (it == k->floats.end()) return make_status(ORT_FAIL, std::string("no float attribute ") + name);
      *out = it->second;
      return nullptr;
    },
    [](const char* name, OrtCustomOpDomain** out) -> OrtStatus* {
      *out = new OrtCustomOpDomain{name, {}};
      return nullptr;
    },
    [](OrtCustomOpDomain* d, const OrtCustomOp* op) -> OrtStatus* {
      d->ops.push_back(op);
      return nullptr;
    },
    [](OrtSessionOptions* s, OrtCustomOpDomain* d) -> OrtStatus* {
      s->domains.push_back(d);
      return nullptr;
    },
};

const OrtApi* get_api(uint32_t version) { return version <= ORT_API_VERSION ? &g_api : nullptr; }
const char* version_string() { return "bolt-test-shim"; }
const OrtApiBase g_api_base = {get_api, version_string};

struct Library {
  void* handle = nullptr;
  OrtSessionOptions options;
};
std::mutex g_mu;
std::vector<std::unique_ptr<Library>> g_libs;

const OrtCustomOp* find_op(int lib, const char* domain, const char* name) {
  std::lock_guard<std::mutex> lock(g_mu);
  if (lib < 0 || lib >= static_cast<int>(g_libs.size())) return nullptr;
  for (OrtCustomOpDomain* d : g_libs[lib]->options.domains) {
    if (domain && d->name != domain) continue;
    for (const OrtCustomOp* op : d->ops)
      if (std::strcmp(op->GetName(op), name) == 0) return op;
  }
  return nullptr;
}

struct Kernel {
  const OrtCustomOp* op;
  void* state;
};

int fail(int code, const std::string& msg) {
  g_error = msg;
  return code;
}

int from_status(OrtStatus* s) {
  if (!s) return ORT_OK;
  const int code = s->code;
  g_error = s->msg;
  delete s;
  return code;
}

}  // namespace

extern "C" {

__attribute__((visibility("default"))) const char* ort_shim_last_error() { return g_error.c_str(); }

// Loads `path` and registers its ops; returns a library id >= 0, or -1 (message in last_error).
__attribute__((visibility("default"))) int ort_shim_load(const char* path) {
  void* h = dlopen(path, RTLD_NOW | RTLD_LOCAL);
  if (!h) return fail(-1, std::string("dlopen: ") + dlerror());
  using Reg = OrtStatus* (*)(OrtSessionOptions*, const OrtApiBase*);
  auto reg = reinterpret_cast<Reg>(dlsym(h, "RegisterCustomOps"));
  if (!reg) return fail(-1, "RegisterCustomOps is not exported");
  auto lib = std::make_unique<Library>();
  lib->handle = h;
  const int rc = from_status(reg(&lib->options, &g_api_base));
  if (rc != ORT_OK) return -1;
  std::lock_guard<std::mutex> lock(g_mu);
  g_libs.push_back(std::move(lib));
  return static_cast<int>(g_libs.size()) - 1;
}

// Registered ops as "domain:name" strings joined by ';' into buf (returns the number of ops).
__attribute__((visibility("default"))) int ort_shim_list_ops(int lib, char* buf, int len) {
  std::lock_guard<std::mutex> lock(g_mu);
  if (lib < 0 || lib >= static_cast<int>(g_libs.size())) return fail(-1, "bad library id");
  std::string s;
  int n = 0;
  for (OrtCustomOpDomain* d : g_libs[lib]->options.domains)
    for (const OrtCustomOp* op : d->ops) {
      s += (n ? ";" : "") + d->name + ":" + op->GetName(op);
      ++n;
    }
  std::strncpy(buf, s.c_str(), static_cast<size_t>(len) - 1);
  buf[len - 1] = '\0';
  return n;
}

// Signature of an op: input / output element types and characteristics, the EP type.
__attribute__((visibility("default"))) int ort_shim_op_signature(int lib, const char* domain, const char* name,
                                                                  int* n_in, int* in_types, int* in_chars, int* n_out,
                                                                  int* out_types, int* out_chars, char* ep, int ep_len) {
  const OrtCustomOp* op = find_op(lib, domain, name);
  if (!op) return fail(ORT_FAIL, std::string("no op ") + name);
  *n_in = static_cast<int>(op->GetInputTypeCount(op));
  *n_out = static_cast<int>(op->GetOutputTypeCount(op));
  if (*n_in > 16 || *n_out > 16) return fail(ORT_FAIL, "too many inputs or outputs");
  for (int i = 0; i < *n_in; ++i) {
    in_types[i] = op->GetInputType(op, i);
    in_chars[i] = op->GetInputCharacteristic(op, i);
  }
  for (int i = 0; i < *n_out; ++i) {
    out_types[i] = op->GetOutputType(op, i);
    out_chars[i] = op->GetOutputCharacteristic(op, i);
  }
  const char* e = op->GetExecutionProviderType(op);
  std::strncpy(ep, e ? e : "", static_cast<size_t>(ep_len) - 1);
  ep[ep_len - 1] = '\0';
  return ORT_OK;
}

// Creates a kernel of op `name` with the given attributes (kinds: 0 = int64, 1 = float).
// Returns the kernel, or null with *code / last_error set.
__attribute__((visibility("default"))) void* ort_shim_create_kernel(int lib, const char* domain, const char* name,
                                                                     int n_attr, const char* const* attr_names,
                                                                     const int* kinds, const int64_t* ivals,
                                                                     const float* fvals, int* code) {
  const OrtCustomOp* op = find_op(lib, domain, name);
  if (!op) {
    *code = fail(ORT_FAIL, std::string("no op ") + name);
    return nullptr;
  }
  OrtKernelInfo info;
  for (int i = 0; i < n_attr; ++i) {
    if (kinds[i] == 0) info.ints[attr_names[i]] = ivals[i];
    else info.floats[attr_names[i]] = fvals[i];
  }
  void* state = nullptr;
  *code = from_status(op->CreateKernelV2(op, &g_api, &info, &state));
  if (*code != ORT_OK) return nullptr;
  return new Kernel{op, state};
}

__attribute__((visibility("default"))) void ort_shim_destroy_kernel(void* kernel) {
  Kernel* k = static_cast<Kernel*>(kernel);
  if (!k) return;
  k->op->KernelDestroy(k->state);
  delete k;
}

// Runs a kernel once.  in_shapes / out_shapes: n x 8 int64 (rank <= 8).  Output i is bound to
// out_ptrs[i] (capacity out_caps[i] bytes, element type out_types[i]); its shape is written back
// to out_shapes / out_ranks.  Returns the op's status code (0 = ok).
__attribute__((visibility("default"))) int ort_shim_compute(void* kernel, void* stream, int n_in,
                                                             void* const* in_ptrs, const int64_t* in_shapes,
                                                             const int* in_ranks, int n_out, void* const* out_ptrs,
                                                             const int64_t* out_caps, const int* out_types,
                                                             int64_t* out_shapes, int* out_ranks) {
  Kernel* k = static_cast<Kernel*>(kernel);
  if (!k) return fail(ORT_FAIL, "null kernel");
  OrtKernelContext ctx;
  ctx.stream = stream;
  ctx.inputs.resize(n_in);
  for (int i = 0; i < n_in; ++i) {
    if (in_ranks[i] < 0 || in_ranks[i] > 8) return fail(ORT_FAIL, "input rank out of range");
    ctx.inputs[i].data = in_ptrs[i];
    ctx.inputs[i].shape.assign(in_shapes + 8 * i, in_shapes + 8 * i + in_ranks[i]);
  }
  ctx.outputs.resize(n_out);
  for (int i = 0; i < n_out; ++i) {
    ctx.outputs[i].data = out_ptrs[i];
    ctx.outputs[i].capacity = out_caps[i];
    ctx.outputs[i].elem_bytes = elem_bytes(out_types[i]);
  }
  const int rc = from_status(k->op->KernelComputeV2(k->state, &ctx));
  for (int i = 0; i < n_out; ++i) {
    const OrtValue& v = ctx.outputs[i];
    out_ranks[i] = v.bound ? static_cast<int>(v.shape.size()) : -1;
    for (size_t d = 0; d < v.shape.size() && d < 8; ++d) out_shapes[8 * i + d] = v.shape[d];
  }
  return rc;
}

}  // extern "C"
