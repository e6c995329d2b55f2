// Relu2: y = bf16(max(x, 0)^2), the square taken in fp32 (reference: Relu2Kernel,
// src/bolt_ops.cu:624-629; op :630-646).  max follows fmaxf, so a NaN input gives 0, as there.
//
// B200 design: a pure HBM stream (2 bytes in, 2 out per element).  Each thread moves 16-byte
// vectors (8 values) with streaming loads and stores, two vectors in flight per loop step, over a
// grid of 8 CTAs of 256 threads per SM (grid-stride); the rest of a size that is not a multiple of
// 8, or buffers that are not 16-byte aligned, go element by element.
#include "common.cuh"
#include "kernels.h"

namespace bolt {

namespace {

__device__ __forceinline__ float relu2_f32(float v) {
  const float r = fmaxf(v, 0.f);
  return r * r;
}

// two packed bf16 -> two packed bf16 results
__device__ __forceinline__ uint32_t relu2_pair(uint32_t w) {
  const float lo = relu2_f32(__uint_as_float(w << 16));
  const float hi = relu2_f32(__uint_as_float(w & 0xFFFF0000u));
  const __nv_bfloat162 o = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&o);
}

__device__ __forceinline__ uint4 relu2_vec(uint4 v) {
  return make_uint4(relu2_pair(v.x), relu2_pair(v.y), relu2_pair(v.z), relu2_pair(v.w));
}

__global__ void __launch_bounds__(256) relu2_kernel(const bf16* __restrict__ x, bf16* __restrict__ y, int64_t n,
                                                    int vec) {
  pdl_wait();
  pdl_trigger();
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int64_t i0 = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  int64_t done = 0;
  if (vec) {
    const uint4* xv = reinterpret_cast<const uint4*>(x);
    uint4* yv = reinterpret_cast<uint4*>(y);
    const int64_t nv = n >> 3;
    int64_t j = i0;
    for (; j + stride < nv; j += 2 * stride) {
      const uint4 a = __ldcs(xv + j), b = __ldcs(xv + j + stride);
      __stcs(yv + j, relu2_vec(a));
      __stcs(yv + j + stride, relu2_vec(b));
    }
    if (j < nv) __stcs(yv + j, relu2_vec(__ldcs(xv + j)));
    done = nv << 3;
  }
  for (int64_t j = done + i0; j < n; j += stride) y[j] = __float2bfloat16(relu2_f32(__bfloat162float(x[j])));
}

}  // namespace

cudaError_t launch_relu2(const bf16* x, bf16* y, int64_t n, const LaunchCfg& cfg) {
  if (n <= 0) return cudaSuccess;
  const bool vec = ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y)) & 15) == 0;
  const int64_t units = vec ? std::max<int64_t>(n >> 3, 1) : n;
  const int64_t blocks = std::min<int64_t>((units + 255) / 256, static_cast<int64_t>(cfg.sms) * 8);
  return launch_kernel(relu2_kernel, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, cfg, x, y, n, vec ? 1 : 0);
}

}  // namespace bolt
