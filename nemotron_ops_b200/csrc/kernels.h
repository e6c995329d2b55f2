// Host-side launch interface of the bolt B200 kernels (internal to libbolt_b200.so).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>

namespace bolt {

using bf16 = __nv_bfloat16;

// How a kernel is launched.  `pdl` adds the programmatic-stream-serialization attribute so a
// kernel may start while the previous kernel of the stream drains; kernels still wait
// (griddepcontrol.wait) before touching activations or outputs.  `early_weights` lets them
// stream weights before that wait, which is only valid when the preceding kernel does not
// write the weights (true for inference graphs, where weights are initializers).
struct LaunchCfg {
  cudaStream_t stream = nullptr;
  int sms = 148;
  bool pdl = false;
  bool early_weights = false;
  // staged bytes per CTA; 0 = the kernel family's default (the tensor-core GEMV keeps two CTAs
  // per SM so a PDL successor can stream while this call computes; the others use one)
  size_t smem_budget = 0;
};

template <typename... KArgs, typename... Args>
cudaError_t launch_kernel(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, const LaunchCfg& cfg,
                          Args&&... args) {
  cudaLaunchConfig_t lc = {};
  lc.gridDim = grid;
  lc.blockDim = block;
  lc.dynamicSmemBytes = smem;
  lc.stream = cfg.stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  lc.attrs = attr;
  lc.numAttrs = cfg.pdl ? 1 : 0;
  return cudaLaunchKernelEx(&lc, kernel, std::forward<Args>(args)...);
}

// ---- GEMV ------------------------------------------------------------------------------
// Exact fp32-weight path (Q8 bits=8 / Q4 bits=4).
cudaError_t launch_gemv_exact(int bits, const bf16* x, int R, const uint8_t* w, const bf16* sc, int64_t N, int K,
                              bf16* y, const LaunchCfg& cfg);

// Tensor-core path.  fmt: weight format (see Fmt in gemv_mma.cu).
enum WeightFmt : int { kFmtQ8 = 0, kFmtQ4 = 1, kFmtFp4 = 2, kFmtIq2Lut = 3, kFmtIq2N = 4 };
cudaError_t launch_gemv_mma(int fmt, const bf16* x, int R, const uint8_t* w, const void* sc, const float* gscale,
                            int64_t N, int K, bf16* y, const LaunchCfg& cfg);

// R = 1 streaming GEMV (fmt kFmtFp4, kFmtQ4 or kFmtIq2N, 16-byte aligned tensors): cudaErrorNotSupported,
// with nothing launched, for shapes it does not take (gemv_r1.cu).
cudaError_t launch_gemv_r1(int fmt, const bf16* x, const uint8_t* w, const void* sc, const float* gscale, int64_t N,
                           int K, bf16* y, const LaunchCfg& cfg);

// Debug: dequantise rows [0, N) with the exact contract of `fmt` (fp32 out) -- used by the
// bit-exactness tests of the weight decode.
cudaError_t launch_dequant(int fmt, int exact, const uint8_t* w, const void* sc, int64_t N, int K, float* out,
                           const LaunchCfg& cfg);

// ---- Relu2 -----------------------------------------------------------------------------
// y = bf16(max(x, 0)^2) over n bf16 values.
cudaError_t launch_relu2(const bf16* x, bf16* y, int64_t n, const LaunchCfg& cfg);

// ---- NVLink peer reduction of the expert-sharded MoE --------------------------------------
// bufs: device array of every rank's peer-visible buffer: two halves of `world` slots of `stride`
// fp32 partials (slot q holds rank q's partial), then kPeerReduceCtas * world uint32 flag words
// (zero at start); epoch: this rank's kPeerReduceCtas uint32 call counters (zero at start).
constexpr int kPeerReduceCtas = 16;
struct PeerReduce {
  float* const* bufs;
  uint32_t* epoch;
  int64_t stride;
  int rank, world;
};

// ---- Mamba ---------------------------------------------------------------------------
// One MambaStep (sel == null: state row 0 in and out) or MambaVerify (start from row *sel,
// the state after token r to row r) over R tokens; see mamba.cu.
struct MambaParams {
  const bf16* proj;      // [R, stride], stride = di + cd + heads
  const bf16* conv_in;   // [rows, cd, 3]
  const bf16* conv_w;    // [cd, 1, 4]
  const bf16* conv_b;    // [cd]
  const float* ssm_in;   // [rows, heads, ds, hd]
  const float* dt_bias;  // [heads]
  const float* a_neg;    // [heads]
  const float* d_skip;   // [heads]
  const float* norm_w;   // [di]
  const int* sel;        // device pointer to the start row (MambaVerify) or null (MambaStep)
  bf16* y;               // [R, di]
  bf16* conv_out;        // like conv_in
  float* ssm_out;        // like ssm_in
  bf16* xbc;             // [R, cd]
  float* ypre;           // [R, di]
  int R, rows, stride, di, cd, heads, hd, ds, ng, hpg;
  float eps, tmin;
};
cudaError_t launch_mamba(const MambaParams& p, const LaunchCfg& cfg);

// ---- MoE -------------------------------------------------------------------------------
cudaError_t launch_moe_route(const bf16* x, const bf16* gate_w, const float* bias, int R, int K, int E, int topk,
                             float scale, int* idx, float* w, float* scores, const LaunchCfg& cfg);

// MoeDecode over the pairs whose expert is in [e_begin, e_end) (I % 256 == 0); out and/or
// out_partial (fp32, the shard's share) may be null.
cudaError_t launch_moe_decode(const bf16* z, const int* idx, const float* w, const uint8_t* fc1_w, const bf16* fc1_s,
                              const uint8_t* fc2_w, const bf16* fc2_s, int R, int E, int I, int topk, int e_begin,
                              int e_end, bf16* out, bf16* h, float* part, float* out_partial, const LaunchCfg& cfg);
// MoeDecode on the register-streaming kernels (moe_stream.cu; P <= 128, R <= 16, I % 32 == 0,
// I <= 8192, P * (I / 32) * 68 + 512 * ceil(1024 / sms) bytes of shared memory <= 200 KB,
// 16-byte aligned z, weights and h): cudaErrorNotSupported, with nothing launched, for shapes
// they do not take.
cudaError_t launch_moe_decode_stream(const bf16* z, const int* idx, const float* w, const uint8_t* fc1_w,
                                     const bf16* fc1_s, const uint8_t* fc2_w, const bf16* fc2_s, int R, int E, int I,
                                     int topk, int e_begin, int e_end, bf16* out, bf16* h, float* part,
                                     float* out_partial, const LaunchCfg& cfg);
// MoeDecode for any I % 32 == 0 (SIMT), all experts.
cudaError_t launch_moe_decode_simt(const bf16* z, const int* idx, const float* w, const uint8_t* fc1_w,
                                   const bf16* fc1_s, const uint8_t* fc2_w, const bf16* fc2_s, int R, int E, int I,
                                   int topk, bf16* out, bf16* h, float* part, const LaunchCfg& cfg);

// MoeDecode / MoeVerify finalize (moe.cu).  round_part: part holds fp32 fc2 sums, rounded to bf16
// (and written back) here; 0: part already holds the rounded per-pair outputs.
cudaError_t launch_moe_finalize(float* part, int round_part, const float* w, const int* idx, int R, int topk,
                                int e_begin, int e_end, bf16* out, float* out_partial, const LaunchCfg& cfg);
// the same, fused with the sum over the ranks' partials through peer memory (moe.cu)
cudaError_t launch_moe_finalize_allreduce(float* part, int round_part, const float* w, const int* idx, int R,
                                          int topk, int e_begin, int e_end, const PeerReduce& pr, bf16* out,
                                          const LaunchCfg& cfg);
// MoeVerify (fmt kFmtQ4, kFmtIq2Lut or kFmtIq2N) on the register-streaming tensor-core kernels
// (moe_vstream.cu; R <= 8, R * topk <= 128, I % 256 == 0, 16-byte aligned z, weights and h):
// cudaErrorNotSupported, with nothing launched, for shapes they do not take.
cudaError_t launch_moe_verify_stream(int fmt, const bf16* z, const int* idx, const float* w, const uint8_t* fc1_w,
                                     const bf16* fc1_s, const uint8_t* fc2_w, const bf16* fc2_s, int R, int E, int I,
                                     int topk, int e_begin, int e_end, bf16* out, bf16* h, float* part, int* meta,
                                     float* out_partial, const LaunchCfg& cfg, const PeerReduce* pr);
cudaError_t launch_moe_verify(int fmt, const bf16* z, const int* idx, const float* w, const uint8_t* fc1_w,
                              const bf16* fc1_s, const uint8_t* fc2_w, const bf16* fc2_s, int R, int E, int I,
                              int topk, int e_begin, int e_end, bf16* out, bf16* h, float* part, int* meta,
                              float* out_partial, const LaunchCfg& cfg, const PeerReduce* pr = nullptr);

}  // namespace bolt
