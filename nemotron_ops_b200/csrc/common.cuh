// Shared device helpers for the bolt B200 kernels (sm_100a only).
//
// * mbarrier + cp.async.bulk (1-D TMA) staging of weight rows into shared memory;
// * bounded waits: every spin on an mbarrier gives up after kWaitLimitNs of %globaltimer,
//   records a code in the device status word and lets the kernel return;
// * programmatic dependent launch (PDL) hooks;
// * bf16 / fp16 bit helpers.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <atomic>
#include <stdint.h>

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "nemotron_ops_b200 kernels are written for sm_100a (B200) only"
#endif

namespace bolt {

using bf16 = __nv_bfloat16;

// ---------------------------------------------------------------------------------------
// device status word: bit flags OR-ed by kernels that had to give up (never set on success)
// ---------------------------------------------------------------------------------------
enum StatusBits : unsigned {
  kStatusFullWait = 1u << 0,    // consumer timed out waiting for staged data
  kStatusEmptyWait = 1u << 1,   // producer timed out waiting for a free stage
  kStatusDrainWait = 1u << 2,   // exit drain of in-flight copies timed out
  kStatusBadExpert = 1u << 3,   // an expert id outside [0, E) was skipped
  kStatusGridWait = 1u << 4,    // a cross-CTA wait timed out
  kStatusSmemAlign = 1u << 5,   // the shared-memory carve-out was not aligned as required
  kStatusBadRow = 1u << 6,      // a MambaVerify state row (sel) outside the state buffer: nothing written
};

extern __device__ unsigned g_status;

__device__ __forceinline__ void set_status(unsigned bits) { atomicOr(&g_status, bits); }

constexpr unsigned long long kWaitLimitNs = 2000000000ull;  // 2 s: far above any legal wait

__device__ __forceinline__ unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------------------------------
// mbarrier / bulk copy
// ---------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint32_t bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n"
      " mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2, 1000000;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Waits for the phase of `parity` to complete.  Gives up after kWaitLimitNs, sets `code` in
// the status word and returns false; the caller then stops consuming and returns.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, unsigned code) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (globaltimer() - t0 > kWaitLimitNs) {
      set_status(code);
      return false;
    }
  }
}

// 1-D bulk copy global -> shared (TMA engine); completion is signalled on `bar` as tx bytes.
// dst, src and bytes must be multiples of 16.
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}

// Asks the bulk-copy engine to pull [p, p + bytes) into L2 (no destination, no completion).
// p and bytes must be multiples of 16.
__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// L2 prefetch of the 16-byte aligned body of [p, p + len), in pieces of at most 1 MB.
__device__ __forceinline__ void prefetch_span_l2(const void* p, uint64_t len) {
  uintptr_t a = (reinterpret_cast<uintptr_t>(p) + 15) & ~uintptr_t(15);
  const uintptr_t e = (reinterpret_cast<uintptr_t>(p) + len) & ~uintptr_t(15);
  while (a < e) {
    const uint32_t n = static_cast<uint32_t>(e - a < (1u << 20) ? e - a : (1u << 20));
    prefetch_l2(reinterpret_cast<const void*>(a), n);
    a += n;
  }
}

// Stages the byte range [src, src + len) of a tensor whose valid bytes end at `end` into
// shared memory so that byte src[i] lands at dst + (src & 15) + i.  The 16-byte aligned body
// goes through the bulk-copy engine (its byte count is added to `tx`); the part beyond the
// last 16-byte boundary of the tensor is copied with plain loads by the calling thread, which
// must be the thread that later arrives on the barrier (the arrive's release orders it).
// Returns the offset (src & 15) at which the first byte lands.
__device__ __forceinline__ uint32_t stage_span(uint8_t* dst, const uint8_t* src, uint32_t len, const uint8_t* end,
                                               uint32_t bar, uint32_t& tx) {
  const uintptr_t s = reinterpret_cast<uintptr_t>(src);
  const uintptr_t a0 = s & ~uintptr_t(15);
  const uintptr_t e = s + len;
  const uintptr_t lim = reinterpret_cast<uintptr_t>(end) & ~uintptr_t(15);
  uintptr_t a1 = (e + 15) & ~uintptr_t(15);
  if (a1 > lim) a1 = lim > a0 ? lim : a0;
  if (a1 > a0) {
    bulk_g2s(smem_u32(dst), reinterpret_cast<const void*>(a0), static_cast<uint32_t>(a1 - a0), bar);
    tx += static_cast<uint32_t>(a1 - a0);
  }
  for (uintptr_t p = a1 > s ? a1 : s; p < e; ++p) dst[p - a0] = *reinterpret_cast<const uint8_t*>(p);
  return static_cast<uint32_t>(s - a0);
}

// ---------------------------------------------------------------------------------------
// programmatic dependent launch
// ---------------------------------------------------------------------------------------
// Waits until the preceding grid in the stream (if launched as a PDL primary) has completed
// and its memory is visible.  A no-op when the kernel was launched without the attribute.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// Lets the next grid in the stream (launched with the PDL attribute) start its prologue.
// A kernel's dynamic shared-memory limit is raised once per device and size: the attribute call
// costs host time on every launch otherwise.  One SmemOptIn per kernel (a static beside its
// launcher; static storage starts at zero).  A kernel with large static shared memory needs the
// opt-in even for a small dynamic size, which the zero start gives.
struct SmemOptIn {
  static constexpr int kMaxDevices = 64;
  std::atomic<size_t> bytes[kMaxDevices];
};

template <typename Kern>
inline cudaError_t allow_smem(Kern kern, size_t bytes, SmemOptIn& s) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= SmemOptIn::kMaxDevices)
    return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes));
  std::atomic<size_t>& cur = s.bytes[dev];
  if (bytes <= cur.load(std::memory_order_relaxed)) return cudaSuccess;
  const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes));
  if (e == cudaSuccess) {
    size_t c = cur.load();
    while (c < bytes && !cur.compare_exchange_weak(c, bytes)) {
    }
  }
  return e;
}

__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;"); }

// Named barrier `id` (1..15) over the first `threads` threads of the block (a multiple of 32);
// barrier 0 is __syncthreads.
__device__ __forceinline__ void named_bar_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// 16-byte shared-memory load
__device__ __forceinline__ uint4 lds128(const void* p) { return *reinterpret_cast<const uint4*>(p); }

// ---------------------------------------------------------------------------------------
// arithmetic helpers
// ---------------------------------------------------------------------------------------
__device__ __forceinline__ float bf16_bits_to_f32(uint32_t bits16) { return __uint_as_float(bits16 << 16); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// packed fp32x2 fused multiply-add (sm_100): d = a * b + c on both lanes
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
  unsigned long long ra = *reinterpret_cast<unsigned long long*>(&a);
  unsigned long long rb = *reinterpret_cast<unsigned long long*>(&b);
  unsigned long long rc = *reinterpret_cast<unsigned long long*>(&c);
  unsigned long long rd;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(rd) : "l"(ra), "l"(rb), "l"(rc));
  return *reinterpret_cast<float2*>(&rd);
}

__device__ __forceinline__ float2 fadd2(float2 a, float2 b) {
  unsigned long long ra = *reinterpret_cast<unsigned long long*>(&a);
  unsigned long long rb = *reinterpret_cast<unsigned long long*>(&b);
  unsigned long long rd;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(rd) : "l"(ra), "l"(rb));
  return *reinterpret_cast<float2*>(&rd);
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}

}  // namespace bolt
