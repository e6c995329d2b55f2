// MambaStep / MambaVerify: one Mamba-2 decode step over R tokens (reference: MambaStepState,
// src/bolt_ops.cu:299-357, kernels :63-297).  proj row = [gate (di) | xBC (cd = di + 2 ng ds) |
// dt (heads)], di = heads * head_dim.  Per token r, in order:
//   xBC_act[r] = bf16(silu(conv_b + sum_k conv_w[k] * window_r[k]))  (depthwise 4-tap causal conv
//                over the 3 stored inputs and the tokens so far)
//   dt = max(softplus(dt_raw + dt_bias), time_step_min), dA = exp(A * dt)
//   state[h, n, p] = state * dA + dt * x[h, p] * B[g, n];  ypre = sum_n C[g, n] state + D x
//   y = bf16(rmsnorm_group(ypre * silu(gate)) * norm_w)
// MambaStep reads and writes state row 0 (the state after the last token); MambaVerify starts
// from row *sel of [rows, ...] state buffers and writes the state after token r to row r.
//
// B200 design: the fp32 SSM state (heads x 128 x 64, 4 MB at 128 heads) dominates the traffic;
// it is read once and written once (per token in verify mode), 128-byte coalesced: a CTA owns
// half a head (32 p) and 4 warps split d_state, each lane holding 32 state values of one p in
// registers through all R tokens.  The conv (one thread per channel) and the gated RMSNorm (one
// CTA per token and group) are separate small kernels; all three use programmatic dependent
// launch waits like the rest of the library.
#include "common.cuh"
#include "kernels.h"

namespace bolt {

namespace {

constexpr int kMambaMaxRows = 16;  // src/bolt_ops.cu:32
constexpr int kHD = 64, kDS = 128;
constexpr int kPT = 32;            // p per SSM CTA
constexpr int kQP = 4;             // d_state parts (warps) per SSM CTA
constexpr int kNH = kDS / kQP;     // state values per thread

__device__ __forceinline__ float silu(float v) { return v / (1.0f + expf(-v)); }

// the state row this call starts from; false (and a status bit) when `sel` is out of range
// (read at L2: the SSM kernel reads it before its dependency wait, see there)
__device__ __forceinline__ bool start_row(const MambaParams& p, int64_t& row) {
  row = 0;
  if (p.sel == nullptr) return true;
  row = __ldcg(p.sel);
  if (row < 0 || row >= p.rows) {
    if (threadIdx.x == 0 && blockIdx.x == 0 && blockIdx.y == 0) set_status(kStatusBadRow);
    return false;
  }
  return true;
}

__global__ void __launch_bounds__(128) mamba_conv_kernel(const MambaParams p) {
  pdl_wait();
  pdl_trigger();
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  int64_t row;
  if (!start_row(p, row) || c >= p.cd) return;
  const int R = p.R;
  float inp[3 + kMambaMaxRows];
  const bf16* ci = p.conv_in + (row * p.cd + c) * 3;
  inp[0] = __bfloat162float(ci[0]);
  inp[1] = __bfloat162float(ci[1]);
  inp[2] = __bfloat162float(ci[2]);
  const bf16* wp = p.conv_w + static_cast<int64_t>(c) * 4;
  const float w0 = __bfloat162float(wp[0]), w1 = __bfloat162float(wp[1]), w2 = __bfloat162float(wp[2]),
              w3 = __bfloat162float(wp[3]);
  const float bias = __bfloat162float(p.conv_b[c]);
#pragma unroll
  for (int r = 0; r < kMambaMaxRows; ++r)
    if (r < R) inp[3 + r] = __bfloat162float(p.proj[static_cast<int64_t>(r) * p.stride + p.di + c]);
#pragma unroll
  for (int r = 0; r < kMambaMaxRows; ++r) {
    if (r < R) {
      const float acc = bias + w0 * inp[r] + w1 * inp[r + 1] + w2 * inp[r + 2] + w3 * inp[r + 3];
      p.xbc[static_cast<int64_t>(r) * p.cd + c] = __float2bfloat16(silu(acc));
      if (p.sel != nullptr) {  // verify: the conv state after token r goes to row r
        bf16* o = p.conv_out + (static_cast<int64_t>(r) * p.cd + c) * 3;
        o[0] = __float2bfloat16(inp[r + 1]);
        o[1] = __float2bfloat16(inp[r + 2]);
        o[2] = __float2bfloat16(inp[r + 3]);
      }
    }
  }
  if (p.sel == nullptr) {
    bf16* o = p.conv_out + static_cast<int64_t>(c) * 3;
    o[0] = __float2bfloat16(inp[R]);
    o[1] = __float2bfloat16(inp[R + 1]);
    o[2] = __float2bfloat16(inp[R + 2]);
  }
}

// grid (heads, kHD / kPT), block kQP * 32: warp q holds state[h, q * kNH + n, p_base + lane]
__global__ void __launch_bounds__(kQP * 32) mamba_ssm_kernel(const MambaParams p) {
  __shared__ float sB[kMambaMaxRows][kDS], sC[kMambaMaxRows][kDS];
  __shared__ float sDt[kMambaMaxRows], sDA[kMambaMaxRows];
  __shared__ float sPart[kMambaMaxRows][kQP][kPT];
  pdl_trigger();
  // The state and sel are inputs of the op, not outputs of the conv kernel before this one, and
  // that kernel triggers this launch only after its own dependency wait (the previous op has
  // completed by then), so they are read (at L2) before this kernel's wait: the 4 MB state
  // stream overlaps the conv kernel.
  int64_t row;
  if (!start_row(p, row)) return;
  const int h = blockIdx.x, g = h / p.hpg;
  const int tid = threadIdx.x, lane = tid & 31, q = tid >> 5;
  const int pb = blockIdx.y * kPT, pi = pb + lane;
  const int R = p.R;
  const int64_t hstate = static_cast<int64_t>(kDS) * kHD;
  const int64_t row_stride = static_cast<int64_t>(p.heads) * hstate;
  // this thread's state values first: their HBM latency overlaps the set-up below
  float st[kNH];
  const float* sp = p.ssm_in + row * row_stride + h * hstate + static_cast<int64_t>(q * kNH) * kHD + pi;
#pragma unroll
  for (int n = 0; n < kNH; ++n) st[n] = __ldcg(sp + static_cast<int64_t>(n) * kHD);
  pdl_wait();  // xbc_act (the conv kernel's output)
  const int b_off = p.di + g * kDS, c_off = p.di + p.ng * kDS + g * kDS;
  for (int i = tid; i < R * kDS; i += blockDim.x) {
    const int r = i / kDS, n = i % kDS;
    const bf16* xr = p.xbc + static_cast<int64_t>(r) * p.cd;
    sB[r][n] = __bfloat162float(xr[b_off + n]);
    sC[r][n] = __bfloat162float(xr[c_off + n]);
  }
  const float A = p.a_neg[h], D = p.d_skip[h];
  if (tid < R) {
    const float raw = __bfloat162float(p.proj[static_cast<int64_t>(tid) * p.stride + p.di + p.cd + h]) + p.dt_bias[h];
    const float sp_ = raw > 20.0f ? raw : log1pf(expf(raw));  // softplus
    const float dt = fmaxf(sp_, p.tmin);
    sDt[tid] = dt;
    sDA[tid] = expf(A * dt);
  }
  __syncthreads();
  for (int r = 0; r < R; ++r) {
    const float dt = sDt[r], dA = sDA[r];
    const float x = __bfloat162float(p.xbc[static_cast<int64_t>(r) * p.cd + h * kHD + pi]);
    const float dtx = dt * x;
    float acc = 0.f;
#pragma unroll
    for (int n = 0; n < kNH; ++n) {
      st[n] = st[n] * dA + dtx * sB[r][q * kNH + n];
      acc += sC[r][q * kNH + n] * st[n];
    }
    sPart[r][q][lane] = acc;
    if (p.sel != nullptr) {  // verify: the state after token r goes to row r
      float* o = p.ssm_out + r * row_stride + h * hstate + static_cast<int64_t>(q * kNH) * kHD + pi;
#pragma unroll
      for (int n = 0; n < kNH; ++n) o[static_cast<int64_t>(n) * kHD] = st[n];
    }
  }
  if (p.sel == nullptr) {
    float* o = p.ssm_out + h * hstate + static_cast<int64_t>(q * kNH) * kHD + pi;
#pragma unroll
    for (int n = 0; n < kNH; ++n) o[static_cast<int64_t>(n) * kHD] = st[n];
  }
  __syncthreads();
  for (int i = tid; i < R * kPT; i += blockDim.x) {
    const int r = i / kPT, pp = i % kPT;
    const float x = __bfloat162float(p.xbc[static_cast<int64_t>(r) * p.cd + h * kHD + pb + pp]);
    float sum = D * x;
#pragma unroll
    for (int qq = 0; qq < kQP; ++qq) sum += sPart[r][qq][pp];
    p.ypre[static_cast<int64_t>(r) * p.di + h * kHD + pb + pp] = sum;
  }
}

// grid (R, ng), block 256: y = bf16(v * rsqrt(mean(v^2) + eps) * norm_w), v = ypre * silu(gate)
__global__ void __launch_bounds__(256) mamba_norm_kernel(const MambaParams p) {
  __shared__ float red[8];
  pdl_wait();
  pdl_trigger();
  int64_t row;
  if (!start_row(p, row)) return;
  const int r = blockIdx.x, g = blockIdx.y, tid = threadIdx.x;
  const int gs = p.di / p.ng;
  const int64_t base = static_cast<int64_t>(r) * p.di + static_cast<int64_t>(g) * gs;
  const bf16* gate = p.proj + static_cast<int64_t>(r) * p.stride + static_cast<int64_t>(g) * gs;
  float ss = 0.f;
  for (int i = tid; i < gs; i += blockDim.x) {
    const float v = p.ypre[base + i] * silu(__bfloat162float(gate[i]));
    ss += v * v;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((tid & 31) == 0) red[tid >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int w = 0; w < 8; ++w) tot += red[w];
  const float rs = rsqrtf(tot / gs + p.eps);
  for (int i = tid; i < gs; i += blockDim.x) {
    const float v = p.ypre[base + i] * silu(__bfloat162float(gate[i]));
    p.y[base + i] = __float2bfloat16(v * rs * p.norm_w[static_cast<int64_t>(g) * gs + i]);
  }
}

}  // namespace

cudaError_t launch_mamba(const MambaParams& p, const LaunchCfg& cfg) {
  if (p.R < 1 || p.R > kMambaMaxRows || p.hd != kHD || p.ds != kDS || p.heads % p.ng || p.di % p.ng)
    return cudaErrorInvalidValue;
  cudaError_t e = launch_kernel(mamba_conv_kernel, dim3(static_cast<unsigned>((p.cd + 127) / 128)), dim3(128), 0, cfg, p);
  if (e != cudaSuccess) return e;
  LaunchCfg c2 = cfg;
  c2.pdl = true;  // same op: each kernel waits for its predecessor with griddepcontrol.wait
  e = launch_kernel(mamba_ssm_kernel, dim3(static_cast<unsigned>(p.heads), kHD / kPT), dim3(kQP * 32), 0, c2, p);
  if (e != cudaSuccess) return e;
  return launch_kernel(mamba_norm_kernel, dim3(static_cast<unsigned>(p.R), static_cast<unsigned>(p.ng)), dim3(256), 0,
                       c2, p);
}

}  // namespace bolt
