// C ABI of libbolt_b200.so (declared in include/bolt_b200.h).
//
// Each bolt_* function is the host body of one reference op (the *State::ComputeV2 functions
// of src/bolt_ops.cu): the same shape checks with the same messages, the same dispatch by
// row count / K / iq2 mode, then the B200 kernels.  Exceptions never cross the ABI: every
// failure becomes a status code plus a thread-local message.
#include <cuda_runtime.h>

#include <atomic>
#include <initializer_list>
#include <cstdlib>
#include <mutex>
#include <stdexcept>
#include <string>

#include "../../include/bolt_b200.h"
#include "common.cuh"
#include "kernels.h"

namespace bolt {

__device__ unsigned g_status = 0;

namespace {

thread_local std::string g_last_error;

struct Options {
  std::atomic<int> pdl{1};  // on by default: every kernel still waits before reading upstream data
  std::atomic<int> early{0};
  std::atomic<int64_t> budget{0};
  Options() {
    if (const char* v = std::getenv("BOLT_PDL")) pdl = std::atoi(v) != 0;
    if (const char* v = std::getenv("BOLT_EARLY_WEIGHTS")) early = std::atoi(v) != 0;
    if (const char* v = std::getenv("BOLT_SMEM_BUDGET")) budget = std::atoll(v);
  }
};

Options& options() {
  static Options o;
  return o;
}

int sm_count() {
  static std::mutex mu;
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  std::lock_guard<std::mutex> lock(mu);
  if (cache[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cache[dev] = n;
  }
  return cache[dev];
}

LaunchCfg make_cfg(void* stream) {
  LaunchCfg c;
  c.stream = static_cast<cudaStream_t>(stream);
  c.sms = sm_count();
  c.pdl = options().pdl.load() != 0;
  c.early_weights = c.pdl && options().early.load() != 0;
  const int64_t b = options().budget.load();
  if (b > 0) c.smem_budget = static_cast<size_t>(b);
  return c;
}

struct Shape {
  const int64_t* d;
  int rank;
  int64_t dim(int i) const {
    if (i < 0 || i >= rank) throw std::invalid_argument("tensor rank too small");
    return d[i];
  }
  int64_t count() const {
    int64_t n = 1;
    for (int i = 0; i < rank; ++i) n *= d[i];
    return n;
  }
  int64_t last() const { return dim(rank - 1); }
};

void check_launch(cudaError_t e) {
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) throw std::runtime_error(cudaGetErrorString(e));
}

template <typename F>
int guarded(F&& f) {
  try {
    f();
    g_last_error.clear();
    return BOLT_OK;
  } catch (const std::exception& e) {
    g_last_error = e.what();
    return BOLT_FAIL;
  }
}

void require(bool ok, const char* msg) {
  if (!ok) throw std::invalid_argument(msg);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// The vectorised activation loads and the bulk copies of weight rows need 16-byte aligned
// tensors (ORT and torch allocations always are).
void require_aligned(std::initializer_list<const void*> ps, const char* op) {
  for (const void* p : ps)
    if (!aligned16(p)) throw std::invalid_argument(std::string(op) + ": tensors must be 16-byte aligned");
}

__global__ void f32_to_bf16_kernel(const float* __restrict__ in, bf16* __restrict__ out, int64_t n) {
  pdl_trigger();
  pdl_wait();
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < n) out[i] = __float2bfloat16(in[i]);
}

int moe_verify_impl(const void* z, const int64_t* z_shape, int z_rank, const void* idx, const void* w,
                    const void* fc1_w, const int64_t* fc1_w_shape, int fc1_w_rank, const void* fc1_s,
                    const void* fc2_w, const void* fc2_s, int64_t topk, int64_t iq2, int64_t e_begin, int64_t e_end,
                    bool sharded, void* out, void* h, void* part, void* meta, void* out_partial, void* stream,
                    const PeerReduce* pr = nullptr) {
  return guarded([&] {
    const Shape zs{z_shape, z_rank}, w1s{fc1_w_shape, fc1_w_rank};
    const int64_t R = zs.dim(0);
    const int64_t P = R * topk;
    // src/bolt_ops.cu:1193-1196
    require(R >= 1 && R <= 8 && P <= 128 && topk >= 1, "MoeVerify: rows must be in [1,8] and rows*topk <= 128");
    require(zs.dim(1) == 1024, "MoeVerify: latent size must be 1024");
    const int64_t I = w1s.dim(1);
    require(I % 64 == 0, "MoeVerify: inter size must be a multiple of 64");
    require(iq2 != 2 || I % 256 == 0, "MoeVerify iq2=2: inter size must be a multiple of 256");
    require(I <= 8192, "MoeVerify: inter size must be <= 8192");
    const int64_t E = w1s.dim(0);
    if (!sharded) {
      e_begin = 0;
      e_end = E;
    }
    require(e_begin >= 0 && e_begin <= e_end && e_end <= E, "MoeVerify: expert range outside [0, E]");
    const int fmt = iq2 == 2 ? kFmtIq2N : (iq2 ? kFmtIq2Lut : kFmtQ4);
    require_aligned({z, fc1_w, fc2_w}, "MoeVerify");
    check_launch(launch_moe_verify(fmt, static_cast<const bf16*>(z), static_cast<const int*>(idx),
                                   static_cast<const float*>(w), static_cast<const uint8_t*>(fc1_w),
                                   static_cast<const bf16*>(fc1_s), static_cast<const uint8_t*>(fc2_w),
                                   static_cast<const bf16*>(fc2_s), static_cast<int>(R), static_cast<int>(E),
                                   static_cast<int>(I), static_cast<int>(topk), static_cast<int>(e_begin),
                                   static_cast<int>(e_end), static_cast<bf16*>(out), static_cast<bf16*>(h),
                                   static_cast<float*>(part), static_cast<int*>(meta), static_cast<float*>(out_partial),
                                   make_cfg(stream), pr));
  });
}

}  // namespace
}  // namespace bolt

using namespace bolt;

extern "C" {

const char* bolt_last_error(void) { return g_last_error.c_str(); }

int bolt_abi_version(void) { return 100; }

int bolt_set_launch_options(int pdl, int early_weights, int64_t smem_budget) {
  options().pdl = pdl != 0;
  options().early = early_weights != 0;
  options().budget = smem_budget > 0 ? smem_budget : 0;
  return BOLT_OK;
}

int bolt_get_device_status(unsigned* status) {
  return guarded([&] {
    unsigned v = 0, zero = 0;
    check_launch(cudaDeviceSynchronize());
    check_launch(cudaMemcpyFromSymbol(&v, g_status, sizeof(v)));
    check_launch(cudaMemcpyToSymbol(g_status, &zero, sizeof(zero)));
    if (status) *status = v;
  });
}

int bolt_nvfp4_gemv(const void* x, const int64_t* x_shape, int x_rank, const void* w, const int64_t* w_shape,
                    int w_rank, const void* w_scale, const void* g, void* y, void* stream) {
  return guarded([&] {
    const Shape xs{x_shape, x_rank}, ws{w_shape, w_rank};
    const int64_t K = xs.last();
    const int64_t R = K > 0 ? xs.count() / K : 0;
    const int64_t N = ws.dim(0);
    // src/bolt_ops.cu:1271, :1298
    require(ws.dim(1) * 2 == K && K % 1024 == 0 && K > 0, "Nvfp4Gemv: K mismatch (K % 1024 required)");
    require(R >= 1 && R <= 8, "Nvfp4Gemv: rows must be in [1,8]");
    require_aligned({x, w}, "Nvfp4Gemv");
    require(K <= 8192, "Nvfp4Gemv: K must be <= 8192");
    check_launch(launch_gemv_mma(kFmtFp4, static_cast<const bf16*>(x), static_cast<int>(R),
                                 static_cast<const uint8_t*>(w), w_scale, static_cast<const float*>(g), N,
                                 static_cast<int>(K), static_cast<bf16*>(y), make_cfg(stream)));
  });
}

static int qgemv(int bits, const void* x, const int64_t* x_shape, int x_rank, const void* B, const int64_t* B_shape,
                 int B_rank, const void* scales, int64_t iq2, void* y, void* stream) {
  return guarded([&] {
    const Shape xs{x_shape, x_rank}, bs{B_shape, B_rank};
    const int64_t K = xs.last();
    const int64_t R = K > 0 ? xs.count() / K : 0;
    const int64_t N = bs.dim(0);
    if (bits == 8) iq2 = 0;  // Q8Gemv has no iq2 attribute (src/bolt_ops.cu:1433)
    // src/bolt_ops.cu:1443-1451
    if (iq2 == 2) {
      require(K % 256 == 0 && B_rank >= 3 && bs.dim(1) * 32 == K && bs.dim(2) == 8 && R >= 1 && R <= 8,
              "Q4Gemv iq2=2: needs B [N, K/32, 8] and 1..8 rows");
    } else {
      require(K % 32 == 0 && K > 0 && bs.dim(1) * 32 == K, "QGemv: K mismatch");
    }
    require(!(iq2 && iq2 != 2) || (R >= 2 && R <= 8 && K % 128 == 0), "Q4Gemv iq2: needs 2..8 rows and K % 128 == 0");
    require(R >= 1 && R <= 8, "QGemv: rows must be in [1,8]");
    if (iq2 || (R >= 2 && K % 64 == 0)) {
      require_aligned({x, B}, bits == 8 ? "Q8Gemv" : "Q4Gemv");
      require(K <= 8192, "QGemv: K must be <= 8192 for 2..8 rows and for iq2 modes");
    }
    const LaunchCfg cfg = make_cfg(stream);
    const bf16* xb = static_cast<const bf16*>(x);
    const uint8_t* wb = static_cast<const uint8_t*>(B);
    bf16* yb = static_cast<bf16*>(y);
    cudaError_t e;
    if (iq2 == 2) {
      e = launch_gemv_mma(kFmtIq2N, xb, static_cast<int>(R), wb, scales, nullptr, N, static_cast<int>(K), yb, cfg);
    } else if (iq2) {
      e = launch_gemv_mma(kFmtIq2Lut, xb, static_cast<int>(R), wb, scales, nullptr, N, static_cast<int>(K), yb, cfg);
    } else if ((R >= 2 || (bits == 4 && K % 256 == 0)) && K % 64 == 0 && K <= 8192 && aligned16(x) &&
               aligned16(B) && aligned16(scales)) {
      // 2..8 rows: tensor-core contract; Q4 at R = 1: exact contract in block-column mode
      e = launch_gemv_mma(bits == 8 ? kFmtQ8 : kFmtQ4, xb, static_cast<int>(R), wb, scales, nullptr, N,
                          static_cast<int>(K), yb, cfg);
    } else {
      e = launch_gemv_exact(bits, xb, static_cast<int>(R), wb, static_cast<const bf16*>(scales), N,
                            static_cast<int>(K), yb, cfg);
    }
    check_launch(e);
  });
}

int bolt_q8_gemv(const void* x, const int64_t* x_shape, int x_rank, const void* B, const int64_t* B_shape, int B_rank,
                 const void* scales, void* y, void* stream) {
  return qgemv(8, x, x_shape, x_rank, B, B_shape, B_rank, scales, 0, y, stream);
}

int bolt_q4_gemv(const void* x, const int64_t* x_shape, int x_rank, const void* B, const int64_t* B_shape, int B_rank,
                 const void* scales, int64_t iq2, void* y, void* stream) {
  return qgemv(4, x, x_shape, x_rank, B, B_shape, B_rank, scales, iq2, y, stream);
}

int bolt_moe_route(const void* x, const int64_t* x_shape, int x_rank, const void* gate_w, const int64_t* gw_shape,
                   int gw_rank, const void* bias, int64_t topk, float scale, void* idx, void* w, void* scores,
                   void* stream) {
  return guarded([&] {
    const Shape xs{x_shape, x_rank}, gs{gw_shape, gw_rank};
    const int64_t R = xs.dim(0), K = xs.dim(1), E = gs.dim(0);
    // src/bolt_ops.cu:458
    require(E <= 512 && K % 256 == 0 && topk <= 32 && topk >= 1 && E >= 1 && K > 0, "MoeRoute: unsupported shape");
    if (R == 0) return;
    require_aligned({x, gate_w}, "MoeRoute");
    check_launch(launch_moe_route(static_cast<const bf16*>(x), static_cast<const bf16*>(gate_w),
                                  static_cast<const float*>(bias), static_cast<int>(R), static_cast<int>(K),
                                  static_cast<int>(E), static_cast<int>(topk), scale, static_cast<int*>(idx),
                                  static_cast<float*>(w), static_cast<float*>(scores), make_cfg(stream)));
  });
}

namespace {
int moe_decode_impl(const void* z, const int64_t* z_shape, int z_rank, const void* idx, const void* w,
                    const void* fc1_w, const int64_t* fc1_w_shape, int fc1_w_rank, const void* fc1_s, const void* fc2_w,
                    const void* fc2_s, int64_t topk, int64_t e_begin, int64_t e_end, bool sharded, void* out, void* h,
                    void* part, void* out_partial, void* stream) {
  return guarded([&] {
    const Shape zs{z_shape, z_rank}, w1s{fc1_w_shape, fc1_w_rank};
    const int64_t R = zs.dim(0);
    // src/bolt_ops.cu:601-603
    require(zs.dim(1) == 1024, "MoeDecode: latent size must be 1024");
    const int64_t I = w1s.dim(1);
    require(I % 32 == 0 && I % 8 == 0 && I > 0, "MoeDecode: bad inter size");
    require(topk >= 1 && R * topk <= 128, "MoeDecode: rows*topk must be in [1,128]");
    require(I <= 8192, "MoeDecode: inter size must be <= 8192");
    if (R == 0) return;
    const int64_t E = w1s.dim(0);
    if (!sharded) {
      e_begin = 0;
      e_end = E;
    }
    require(e_begin >= 0 && e_begin <= e_end && e_end <= E, "MoeDecode: expert range outside [0, E]");
    require(!sharded || I % 256 == 0, "MoeDecode shard: inter size must be a multiple of 256");
    require_aligned({z, fc1_w, fc2_w}, "MoeDecode");
    const LaunchCfg cfg = make_cfg(stream);
    if (I % 256 == 0 && aligned16(fc1_s) && aligned16(fc2_s)) {
      check_launch(launch_moe_decode(static_cast<const bf16*>(z), static_cast<const int*>(idx),
                                     static_cast<const float*>(w), static_cast<const uint8_t*>(fc1_w),
                                     static_cast<const bf16*>(fc1_s), static_cast<const uint8_t*>(fc2_w),
                                     static_cast<const bf16*>(fc2_s), static_cast<int>(R), static_cast<int>(E),
                                     static_cast<int>(I), static_cast<int>(topk), static_cast<int>(e_begin),
                                     static_cast<int>(e_end), static_cast<bf16*>(out), static_cast<bf16*>(h),
                                     static_cast<float*>(part), static_cast<float*>(out_partial), cfg));
    } else {
      check_launch(launch_moe_decode_simt(static_cast<const bf16*>(z), static_cast<const int*>(idx),
                                          static_cast<const float*>(w), static_cast<const uint8_t*>(fc1_w),
                                          static_cast<const bf16*>(fc1_s), static_cast<const uint8_t*>(fc2_w),
                                          static_cast<const bf16*>(fc2_s), static_cast<int>(R), static_cast<int>(E),
                                          static_cast<int>(I), static_cast<int>(topk), static_cast<bf16*>(out),
                                          static_cast<bf16*>(h), static_cast<float*>(part), cfg));
    }
  });
}
}  // namespace

int bolt_moe_decode(const void* z, const int64_t* z_shape, int z_rank, const void* idx, const void* w,
                    const void* fc1_w, const int64_t* fc1_w_shape, int fc1_w_rank, const void* fc1_s, const void* fc2_w,
                    const void* fc2_s, int64_t topk, void* out, void* h, void* part, void* stream) {
  return moe_decode_impl(z, z_shape, z_rank, idx, w, fc1_w, fc1_w_shape, fc1_w_rank, fc1_s, fc2_w, fc2_s, topk, 0, 0,
                         false, out, h, part, nullptr, stream);
}

int bolt_moe_decode_shard(const void* z, const int64_t* z_shape, int z_rank, const void* idx, const void* w,
                          const void* fc1_w, const int64_t* fc1_w_shape, int fc1_w_rank, const void* fc1_s,
                          const void* fc2_w, const void* fc2_s, int64_t topk, int64_t e_begin, int64_t e_end, void* out,
                          void* h, void* part, void* out_partial, void* stream) {
  return moe_decode_impl(z, z_shape, z_rank, idx, w, fc1_w, fc1_w_shape, fc1_w_rank, fc1_s, fc2_w, fc2_s, topk,
                         e_begin, e_end, true, out, h, part, out_partial, stream);
}

int bolt_moe_verify(const void* z, const int64_t* z_shape, int z_rank, const void* idx, const void* w,
                    const void* fc1_w, const int64_t* fc1_w_shape, int fc1_w_rank, const void* fc1_s, const void* fc2_w,
                    const void* fc2_s, int64_t topk, int64_t iq2, void* out, void* h, void* part, void* meta,
                    void* stream) {
  return moe_verify_impl(z, z_shape, z_rank, idx, w, fc1_w, fc1_w_shape, fc1_w_rank, fc1_s, fc2_w, fc2_s, topk, iq2, 0,
                         0, false, out, h, part, meta, nullptr, stream);
}

int bolt_moe_verify_shard(const void* z, const int64_t* z_shape, int z_rank, const void* idx, const void* w,
                          const void* fc1_w, const int64_t* fc1_w_shape, int fc1_w_rank, const void* fc1_s,
                          const void* fc2_w, const void* fc2_s, int64_t topk, int64_t iq2, int64_t e_begin,
                          int64_t e_end, void* out, void* h, void* part, void* meta, void* out_partial, void* stream) {
  return moe_verify_impl(z, z_shape, z_rank, idx, w, fc1_w, fc1_w_shape, fc1_w_rank, fc1_s, fc2_w, fc2_s, topk, iq2,
                         e_begin, e_end, true, out, h, part, meta, out_partial, stream);
}

int bolt_moe_verify_shard_allreduce(const void* z, const int64_t* z_shape, int z_rank, const void* idx, const void* w,
                                    const void* fc1_w, const int64_t* fc1_w_shape, int fc1_w_rank, const void* fc1_s,
                                    const void* fc2_w, const void* fc2_s, int64_t topk, int64_t iq2, int64_t e_begin,
                                    int64_t e_end, void* h, void* part, void* meta, const void* peer_bufs,
                                    void* counters, int64_t half_floats, int64_t rank, int64_t world, void* out,
                                    void* stream) {
  PeerReduce pr{};
  const int rc = guarded([&] {
    require(world >= 1 && world <= 64 && rank >= 0 && rank < world, "MoeVerify allreduce: rank outside [0, world)");
    require(peer_bufs != nullptr && counters != nullptr && out != nullptr,
            "MoeVerify allreduce: null peer buffers, counters or output");
    require(z_rank >= 1 && z_shape != nullptr && half_floats >= z_shape[0] * 1024,
            "MoeVerify allreduce: peer buffer halves must hold R * 1024 floats");
    pr.bufs = static_cast<float* const*>(peer_bufs);
    pr.epoch = static_cast<uint32_t*>(counters);
    pr.stride = half_floats;
    pr.rank = static_cast<int>(rank);
    pr.world = static_cast<int>(world);
  });
  if (rc != BOLT_OK) return rc;
  return moe_verify_impl(z, z_shape, z_rank, idx, w, fc1_w, fc1_w_shape, fc1_w_rank, fc1_s, fc2_w, fc2_s, topk, iq2,
                         e_begin, e_end, true, out, h, part, meta, nullptr, stream, &pr);
}

namespace {
int mamba_impl(const void* proj, const int64_t* proj_shape, int proj_rank, const void* conv_state,
               const int64_t* conv_shape, int conv_rank, const void* ssm_state, const int64_t* ssm_shape, int ssm_rank,
               const void* conv_w, const void* conv_b, const void* dt_bias, const void* a_neg, const void* d_skip,
               const void* norm_w, const void* sel, int64_t heads, int64_t head_dim, int64_t d_state,
               int64_t n_groups, float epsilon, float time_step_min, void* y, void* conv_out, void* ssm_out,
               void* xbc_act, void* ypre, void* stream) {
  return guarded([&] {
    const bool verify = sel != nullptr;
    // src/bolt_ops.cu:311 (attributes), :316-322 (rows, proj width), :325 (verify rows)
    if (head_dim != 64 || d_state != 128)
      throw std::invalid_argument("MambaStep: only head_dim=64, d_state=128 are implemented");
    const Shape ps{proj_shape, proj_rank}, cs{conv_shape, conv_rank}, ss{ssm_shape, ssm_rank};
    const int64_t R = ps.dim(0);
    require(R >= 1 && R <= 16, "MambaStep: rows must be in [1,16]");
    require(heads >= 1 && n_groups >= 1 && heads % n_groups == 0, "MambaStep: heads must be a multiple of n_groups");
    const int64_t di = heads * head_dim, cd = di + 2 * n_groups * d_state, stride = di + cd + heads;
    require(ps.dim(1) == stride, "MambaStep: bad proj width");
    if (verify) require(cs.dim(0) >= R, "MambaVerify: state buffer needs >= R rows");
    // shapes the reference takes on trust
    require(conv_rank == 3 && cs.dim(0) >= 1 && cs.dim(1) == cd && cs.dim(2) == 3,
            "MambaStep: conv state must be [rows, conv_dim, 3]");
    require(ssm_rank == 4 && ss.dim(0) == cs.dim(0) && ss.dim(1) == heads && ss.dim(2) == d_state &&
                ss.dim(3) == head_dim,
            "MambaStep: ssm state must be [rows, heads, d_state, head_dim] with the conv state's rows");
    MambaParams p{};
    p.proj = static_cast<const bf16*>(proj);
    p.conv_in = static_cast<const bf16*>(conv_state);
    p.conv_w = static_cast<const bf16*>(conv_w);
    p.conv_b = static_cast<const bf16*>(conv_b);
    p.ssm_in = static_cast<const float*>(ssm_state);
    p.dt_bias = static_cast<const float*>(dt_bias);
    p.a_neg = static_cast<const float*>(a_neg);
    p.d_skip = static_cast<const float*>(d_skip);
    p.norm_w = static_cast<const float*>(norm_w);
    p.sel = static_cast<const int*>(sel);
    p.y = static_cast<bf16*>(y);
    p.conv_out = static_cast<bf16*>(conv_out);
    p.ssm_out = static_cast<float*>(ssm_out);
    p.xbc = static_cast<bf16*>(xbc_act);
    p.ypre = static_cast<float*>(ypre);
    p.R = static_cast<int>(R);
    p.rows = static_cast<int>(cs.dim(0));
    p.stride = static_cast<int>(stride);
    p.di = static_cast<int>(di);
    p.cd = static_cast<int>(cd);
    p.heads = static_cast<int>(heads);
    p.hd = static_cast<int>(head_dim);
    p.ds = static_cast<int>(d_state);
    p.ng = static_cast<int>(n_groups);
    p.hpg = static_cast<int>(heads / n_groups);
    p.eps = epsilon;
    p.tmin = time_step_min;
    check_launch(launch_mamba(p, make_cfg(stream)));
  });
}
}  // namespace

int bolt_mamba_step(const void* proj, const int64_t* proj_shape, int proj_rank, const void* conv_state,
                    const int64_t* conv_shape, int conv_rank, const void* ssm_state, const int64_t* ssm_shape,
                    int ssm_rank, const void* conv_w, const void* conv_b, const void* dt_bias, const void* a_neg,
                    const void* d_skip, const void* norm_w, int64_t heads, int64_t head_dim, int64_t d_state,
                    int64_t n_groups, float epsilon, float time_step_min, void* y, void* conv_state_out,
                    void* ssm_state_out, void* xbc_act, void* ypre, void* stream) {
  return mamba_impl(proj, proj_shape, proj_rank, conv_state, conv_shape, conv_rank, ssm_state, ssm_shape, ssm_rank,
                    conv_w, conv_b, dt_bias, a_neg, d_skip, norm_w, nullptr, heads, head_dim, d_state, n_groups,
                    epsilon, time_step_min, y, conv_state_out, ssm_state_out, xbc_act, ypre, stream);
}

int bolt_mamba_verify(const void* proj, const int64_t* proj_shape, int proj_rank, const void* conv_state,
                      const int64_t* conv_shape, int conv_rank, const void* ssm_state, const int64_t* ssm_shape,
                      int ssm_rank, const void* conv_w, const void* conv_b, const void* dt_bias, const void* a_neg,
                      const void* d_skip, const void* norm_w, const void* sel, int64_t heads, int64_t head_dim,
                      int64_t d_state, int64_t n_groups, float epsilon, float time_step_min, void* y,
                      void* conv_state_out, void* ssm_state_out, void* xbc_act, void* ypre, void* stream) {
  if (sel == nullptr) {
    g_last_error = "MambaVerify: sel must not be null";
    return BOLT_FAIL;
  }
  return mamba_impl(proj, proj_shape, proj_rank, conv_state, conv_shape, conv_rank, ssm_state, ssm_shape, ssm_rank,
                    conv_w, conv_b, dt_bias, a_neg, d_skip, norm_w, sel, heads, head_dim, d_state, n_groups, epsilon,
                    time_step_min, y, conv_state_out, ssm_state_out, xbc_act, ypre, stream);
}

int bolt_relu2(const void* x, const int64_t* x_shape, int x_rank, void* y, void* stream) {
  return guarded([&] {
    const Shape xs{x_shape, x_rank};
    require(x_rank >= 0 && (x_rank == 0 || x_shape != nullptr), "Relu2: bad shape");
    for (int i = 0; i < x_rank; ++i) require(x_shape[i] >= 0, "Relu2: negative dimension");
    const int64_t n = xs.count();
    if (n == 0) return;
    require(x != nullptr && y != nullptr, "Relu2: null buffer");
    check_launch(launch_relu2(static_cast<const bf16*>(x), static_cast<bf16*>(y), n, make_cfg(stream)));
  });
}

int bolt_f32_to_bf16(const void* in, void* out, int64_t n, void* stream) {
  return guarded([&] {
    require(n >= 0, "bolt_f32_to_bf16: negative size");
    if (n == 0) return;
    check_launch(launch_kernel(f32_to_bf16_kernel, dim3(static_cast<unsigned>((n + 255) / 256)), dim3(256), 0,
                               make_cfg(stream), static_cast<const float*>(in), static_cast<bf16*>(out), n));
  });
}

int bolt_memcpy_async(void* dst, const void* src, int64_t bytes, void* stream) {
  return guarded([&] {
    require(bytes >= 0, "bolt_memcpy_async: negative size");
    if (bytes == 0) return;
    require(dst != nullptr && src != nullptr, "bolt_memcpy_async: null buffer");
    check_launch(cudaMemcpyAsync(dst, src, static_cast<size_t>(bytes), cudaMemcpyDefault,
                                 static_cast<cudaStream_t>(stream)));
  });
}

int bolt_dequant(int fmt, int exact, const void* w, const void* scales, int64_t N, int64_t K, void* out, void* stream) {
  return guarded([&] {
    require(fmt >= 0 && fmt <= 4, "bolt_dequant: unknown format");
    require(!exact || fmt == kFmtQ8 || fmt == kFmtQ4, "bolt_dequant: exact contract exists for Q8 / Q4 only");
    const int64_t kmod = fmt == kFmtIq2N ? 256 : fmt == kFmtFp4 ? 64 : 64;
    require(N >= 0 && K > 0 && K % kmod == 0, "bolt_dequant: K must be a multiple of 64 (256 for IQ2_XXS)");
    if (N == 0) return;
    check_launch(launch_dequant(fmt, exact, static_cast<const uint8_t*>(w), scales, N, static_cast<int>(K),
                                static_cast<float*>(out), make_cfg(stream)));
  });
}

}  // extern "C"

// ---------------------------------------------------------------------------------------
// MoeVerify without caller-provided scratch (no counterpart in the reference)
// ---------------------------------------------------------------------------------------
namespace {
// Scratch of bolt_moe_verify_noalloc: meta, part and h of one call live here instead of in
// caller buffers.  One buffer per device, shared by every call on that device.
constexpr size_t kNoAllocScratchBytes = size_t(3) << 19;  // 1.5 MiB
constexpr size_t kNoAllocMetaBytes = 8192;                 // meta of up to 128 pairs (4,612 bytes)
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_ptr[kMaxDevices] = {};

size_t round256(size_t n) { return (n + 255) & ~size_t(255); }

// Device address of the scratch buffer of the current device (looked up once per device).
void* noalloc_scratch() {
  int dev = 0;
  const cudaError_t e0 = cudaGetDevice(&dev);
  if (e0 != cudaSuccess) throw std::runtime_error(std::string("MoeVerify (no-alloc): ") + cudaGetErrorString(e0));
  if (dev < 0 || dev >= kMaxDevices) throw std::runtime_error("MoeVerify (no-alloc): device ordinal out of range");
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess)
      throw std::runtime_error(std::string("MoeVerify (no-alloc): cudaGetSymbolAddress failed: ") +
                               cudaGetErrorString(e));
    g_noalloc_ptr[dev] = p;
  }
  return g_noalloc_ptr[dev];
}
}  // namespace

extern "C" {

int bolt_moe_verify_noalloc(const void* z, const int64_t* z_shape, int z_rank, const void* idx, const void* w,
                            const void* fc1_w, const int64_t* fc1_w_shape, int fc1_w_rank, const void* fc1_s,
                            const void* fc2_w, const void* fc2_s, int64_t topk, int64_t iq2, void* out, void* stream) {
  void* h = nullptr;
  void* part = nullptr;
  void* meta = nullptr;
  const int rc = guarded([&] {
    const Shape zs{z_shape, z_rank}, w1s{fc1_w_shape, fc1_w_rank};
    const int64_t R = zs.dim(0), I = w1s.dim(1);
    const int64_t P = R * topk;
    require(R >= 1 && R <= 8 && topk >= 1 && P <= 128 && I > 0, "MoeVerify: rows must be in [1,8] and rows*topk <= 128");
    const size_t part_bytes = round256(static_cast<size_t>(P) * 1024 * sizeof(float));
    const size_t h_bytes = round256(static_cast<size_t>(P) * static_cast<size_t>(I) * 2);
    const size_t need = kNoAllocMetaBytes + part_bytes + h_bytes;
    if (need > kNoAllocScratchBytes)
      throw std::invalid_argument("MoeVerify (no-alloc): rows*topk*(4096 + 2*I) needs " + std::to_string(need) +
                                  " bytes of scratch, more than the " + std::to_string(kNoAllocScratchBytes) +
                                  "-byte static buffer; use bolt_moe_verify with caller buffers");
    uint8_t* base = static_cast<uint8_t*>(noalloc_scratch());
    meta = base;
    part = base + kNoAllocMetaBytes;
    h = base + kNoAllocMetaBytes + part_bytes;
  });
  if (rc != BOLT_OK) return rc;
  return bolt_moe_verify(z, z_shape, z_rank, idx, w, fc1_w, fc1_w_shape, fc1_w_rank, fc1_s, fc2_w, fc2_s, topk, iq2,
                         out, h, part, meta, stream);
}

}  // extern "C"
