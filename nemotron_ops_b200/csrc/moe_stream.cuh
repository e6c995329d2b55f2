// Shared pieces of the expert-layer streaming kernels (moe_stream.cu, moe_vstream.cu): launch
// shape, parameters, weight-stream loads, warp reductions and the per-CTA grouping of the live
// (token, expert) pairs by expert.
#pragma once

#include <atomic>

#include "mma_decode.cuh"

namespace bolt {
namespace {


constexpr int kMsWarps = 16;
constexpr int kMsThreads = kMsWarps * 32;
constexpr int kMsMaxP = 128;             // pairs per call
constexpr int kBadPair = -2;

struct MsParams {
  const bf16* z;       // [R, 1024]
  const int* idx;      // [P]
  const float* w;      // [P]
  const uint8_t* w1;   // [E, I, 512]
  const bf16* s1;      // [E, I, 32]
  const uint8_t* w2;   // [E, 1024, I/2]
  const bf16* s2;      // [E, 1024, I/32]
  bf16* h;             // [P, I]
  float* part;         // [P, 1024]
  bf16* out;           // [R, 1024] or null
  float* out_partial;  // [R, 1024] or null
  int* meta;           // MoeVerify: [1 + P + 8 P] expert list (reference layout) or null
  int R, P, topk, E, I, e_begin, e_end;
  int nrow;            // fc2: output rows per CTA
};

// live pairs grouped by expert
struct Groups {
  int es[kMsMaxP];         // expert of pair q if live, kBadPair if outside [0, E), else -1
  int fs[kMsMaxP];         // first pair with the same expert (live pairs), else a large value
  int plist[kMsMaxP];      // live pairs: groups in first-occurrence order, pairs ascending
  int gstart[kMsMaxP + 1]; // group g's pairs are plist[gstart[g] .. gstart[g + 1])
  int gexp[kMsMaxP];       // expert of group g
  int ptok[kMsMaxP];       // token of plist[a]
  int pgrp[kMsMaxP];       // group of plist[a]
  int U, nl;
};

// weight streams: read once, keep out of L1
__device__ __forceinline__ uint4 ld_stream(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}
__device__ __forceinline__ uint32_t ld_u16(const void* p) {
  unsigned short v;
  asm volatile("ld.global.nc.L1::no_allocate.u16 %0, [%1];" : "=h"(v) : "l"(p));
  return v;
}

// Butterfly reduction of N = 8 (or 4) per-lane values over the warp: lane l ends with the warp
// total of value (l >> 2) & 7 (N = 8) or (l >> 3) & 3 (N = 4).  The additions follow the same tree
// as a per-value xor-16, 8, 4, 2, 1 warp sum, in fewer shuffles.
__device__ __forceinline__ float warp_sum8_t(const float (&v)[8]) {
  const int lane = threadIdx.x & 31;
  const bool b4 = lane & 16, b3 = lane & 8, b2 = lane & 4;
  float w[4], u[2];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float send = b4 ? v[i] : v[i + 4], keep = b4 ? v[i + 4] : v[i];
    w[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
  }
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const float send = b3 ? w[i] : w[i + 2], keep = b3 ? w[i + 2] : w[i];
    u[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
  }
  const float send = b2 ? u[0] : u[1], keep = b2 ? u[1] : u[0];
  float s = keep + __shfl_xor_sync(0xffffffffu, send, 4);
  s += __shfl_xor_sync(0xffffffffu, s, 2);
  s += __shfl_xor_sync(0xffffffffu, s, 1);
  return s;
}
__device__ __forceinline__ float warp_sum4_t(const float (&v)[4]) {
  const int lane = threadIdx.x & 31;
  const bool b4 = lane & 16, b3 = lane & 8;
  float w[2];
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const float send = b4 ? v[i] : v[i + 2], keep = b4 ? v[i + 2] : v[i];
    w[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
  }
  const float send = b3 ? w[0] : w[1], keep = b3 ? w[1] : w[0];
  float s = keep + __shfl_xor_sync(0xffffffffu, send, 8);
  s += __shfl_xor_sync(0xffffffffu, s, 4);
  s += __shfl_xor_sync(0xffffffffu, s, 2);
  s += __shfl_xor_sync(0xffffffffu, s, 1);
  return s;
}

__device__ __forceinline__ float warp_sum2_t(const float (&v)[2]) {
  const bool b4 = threadIdx.x & 16;
  const float send = b4 ? v[0] : v[1], keep = b4 ? v[1] : v[0];
  float s = keep + __shfl_xor_sync(0xffffffffu, send, 16);
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  return s;
}

// Groups the live pairs by expert (threads 0 .. kMsMaxP - 1 do the work; every thread of the
// block calls it).  report: set the status bit for expert ids outside [0, E).
__device__ void build_groups(const MsParams& p, Groups& g, bool report) {
  const int tid = threadIdx.x;
  int e = -1;
  bool live = false;
  if (tid < kMsMaxP) {
    if (tid < p.P) {
      const int ei = __ldcg(p.idx + tid);
      if (report && (ei < 0 || ei >= p.E)) set_status(kStatusBadExpert);
      live = ei >= 0 && ei < p.E && ei >= p.e_begin && ei < p.e_end;
      e = live ? ei : (ei < 0 || ei >= p.E) ? kBadPair : -1;
    }
    g.es[tid] = e;
  }
  __syncthreads();
  int f = 1 << 30, rank = 0;
  if (live) {
    f = tid;
    for (int q = 0; q < tid; ++q)
      if (g.es[q] == e) {
        if (f == tid) f = q;
        ++rank;
      }
  }
  if (tid < kMsMaxP) g.fs[tid] = f;
  const bool first = live && f == tid;
  const int U = __syncthreads_count(first);
  if (live) {
    int before = 0, slot = 0;
    for (int q = 0; q < p.P; ++q) {
      const int fq = g.fs[q];
      before += fq < f;
      slot += (fq == q) & (q < f);
    }
    g.plist[before + rank] = tid;
    g.ptok[before + rank] = tid / p.topk;
    g.pgrp[before + rank] = slot;
    if (first) {
      g.gexp[slot] = e;
      g.gstart[slot] = before;
    }
  }
  const int nl = __syncthreads_count(live);
  if (tid == 0) {
    g.U = U;
    g.nl = nl;
    g.gstart[U] = nl;
  }
  __syncthreads();
}

}  // namespace
}  // namespace bolt
