// MoeRoute kernels and the small kernels around the MoE expert GEMMs (reference
// src/bolt_ops.cu:359-472, :552-587, :1084-1112); the expert GEMMs are in moe_tc.cu.
//
// MoeRoute: the fp32 router logits are one streaming dot per expert spread over all SMs (each
// gate row is read once and applied to every activation row); the selection sorts packed
// (score + bias, expert) keys per warp and merges the sorted runs in a tree (one CTA per row).
//
// MoeVerify grouping: one CTA writes the reference's `meta` layout (unique experts in
// first-occurrence order and each expert's (token -> pair) map), restricted to a shard's expert
// range.  Finalize: out = bf16(sum_k w * part), k ascending, over the pairs of the expert range,
// optionally also as an fp32 partial for the sharded op.
#include "mma_decode.cuh"

namespace bolt {

namespace {

// =======================================================================================
// MoeRoute
// =======================================================================================
// Logits: two gate rows per CTA, four warps (128 lanes) per row.  K is walked in passes of 4096
// (512 16-byte vectors per row); in a pass lane t of a row loads vectors t, t+128, t+256, t+384,
// all issued before the first use, so one pass of the whole grid puts the full 2.5 MB gate of
// E = 304, K = 4096 in flight at once.  The pass's activation rows (at most 8 x 4096 bf16 = 64 KB)
// are staged in shared memory once per CTA instead of being re-read from L2 by every warp.  The
// row's four warp sums are added in warp order, so results do not depend on scheduling.  Before its
// dependency wait a CTA only pulls its gate rows into L2 (coherent with an upstream writer).
constexpr int kRouteExperts = 2;                            // gate rows per CTA
constexpr int kRouteRowLanes = 128;                         // lanes per gate row
constexpr int kRouteVec = 4;                                // 16-byte gate vectors per lane and pass
constexpr int kRoutePassVec = kRouteRowLanes * kRouteVec;   // 512 vectors = 4096 k per pass
constexpr int kRouteThreads = kRouteExperts * kRouteRowLanes;

__device__ __forceinline__ void dot_bf16x8(const uint4& a, const uint4& b, float& acc) {
  const uint32_t aa[4] = {a.x, a.y, a.z, a.w}, bb[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    acc = fmaf(__uint_as_float(aa[q] << 16), __uint_as_float(bb[q] << 16), acc);
    acc = fmaf(__uint_as_float(aa[q] & 0xFFFF0000u), __uint_as_float(bb[q] & 0xFFFF0000u), acc);
  }
}

template <int RB>  // activation rows per block of rows (1 for R = 1, else 8)
__global__ void __launch_bounds__(kRouteThreads, 2)
    router_logits_kernel(const bf16* __restrict__ x, const bf16* __restrict__ gw, int R, int K, int E, int early,
                         float* __restrict__ scores) {
  extern __shared__ __align__(16) uint4 xs[];  // [RB][kRoutePassVec]
  __shared__ float red[kRouteThreads / 32][RB];
  pdl_trigger();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int e = blockIdx.x * kRouteExperts + (warp >> 2);
  const int t = (warp & 3) * 32 + lane;
  const int V = K >> 3;  // 16-byte vectors per row (K % 256 == 0)
  const uint4* wr = reinterpret_cast<const uint4*>(gw) + static_cast<int64_t>(e < E ? e : E - 1) * V;
  const uint4* xv = reinterpret_cast<const uint4*>(x);
  if (!early && threadIdx.x == 0) {  // pull the CTA's gate rows into L2 while the previous kernel runs
    const int e0 = blockIdx.x * kRouteExperts, ne = min(kRouteExperts, E - e0);
    if (ne > 0) prefetch_span_l2(gw + static_cast<int64_t>(e0) * K, static_cast<uint64_t>(ne) * K * 2);
  }
  bool waited = false;
  for (int r0 = 0; r0 < R; r0 += RB) {
    const int rows = min(RB, R - r0);
    float acc[RB];
#pragma unroll
    for (int r = 0; r < RB; ++r) acc[r] = 0.f;
    for (int base = 0; base < V; base += kRoutePassVec) {
      const int pv = min(kRoutePassVec, V - base);
      if (!early && !waited) {  // the gate may be written upstream: wait before reading it
        pdl_wait();
        waited = true;
      }
      uint4 wv[kRouteVec];
#pragma unroll
      for (int j = 0; j < kRouteVec; ++j) {
        const int v = t + j * kRouteRowLanes;
        wv[j] = v < pv ? __ldg(wr + base + v) : make_uint4(0u, 0u, 0u, 0u);
      }
      if (!waited) {
        pdl_wait();
        waited = true;
      }
      // every activation load of the pass is issued before the first shared-memory store
      constexpr int XJ = kRoutePassVec / kRouteThreads;
      uint4 xr[RB][XJ];
#pragma unroll
      for (int r = 0; r < RB; ++r) {
#pragma unroll
        for (int j = 0; j < XJ; ++j) {
          const int v = threadIdx.x + j * kRouteThreads;
          xr[r][j] = (r < rows && v < pv) ? __ldg(xv + static_cast<int64_t>(r0 + r) * V + base + v)
                                          : make_uint4(0u, 0u, 0u, 0u);
        }
      }
      __syncthreads();  // the previous pass has finished reading xs
#pragma unroll
      for (int r = 0; r < RB; ++r) {
#pragma unroll
        for (int j = 0; j < XJ; ++j) xs[r * kRoutePassVec + threadIdx.x + j * kRouteThreads] = xr[r][j];
      }
      __syncthreads();
#pragma unroll
      for (int r = 0; r < RB; ++r) {
        if (r < rows) {
#pragma unroll
          for (int j = 0; j < kRouteVec; ++j) {
            const int v = t + j * kRouteRowLanes;
            if (v < pv) dot_bf16x8(wv[j], xs[r * kRoutePassVec + v], acc[r]);
          }
        }
      }
    }
#pragma unroll
    for (int r = 0; r < RB; ++r) {
      const float a = warp_sum(acc[r]);
      if (lane == 0) red[warp][r] = a;
    }
    __syncthreads();
    if (threadIdx.x < kRouteExperts * RB) {
      const int eo = threadIdx.x / RB, r = threadIdx.x % RB;
      const int ee = blockIdx.x * kRouteExperts + eo;
      if (ee < E && r < rows) {
        const float* q = &red[eo * 4][r];
        const float a = ((q[0] + q[RB]) + q[2 * RB]) + q[3 * RB];
        scores[static_cast<int64_t>(r0 + r) * E + ee] = 1.0f / (1.0f + expf(-a));
      }
    }
  }
}

// Selection (one CTA per activation row, one warp per 32 experts, E <= 512).  Every expert
// becomes one 64-bit key: the high word is the bias-corrected score as an order-preserving
// unsigned integer (0 for NaN and -inf, which are never chosen), the low word is ~expert id, so a
// larger key is the better choice and equal scores prefer the lower id.  A warp sorts its 32 keys
// with a bitonic network over shuffles; the sorted runs then meet in a binary tree of merges that
// each keep the best 32 of 64 keys (the larger of a run and the partner run reversed is a bitonic
// sequence holding them; five half-cleaner steps sort it).  The first topk keys of the final run
// are the choices in selection order.
__device__ __forceinline__ unsigned long long route_key(float v, int e) {
  if (!(v > -INFINITY)) return 0ull;  // NaN and -inf are never chosen
  const uint32_t b = __float_as_uint(v == 0.f ? 0.f : v);  // -0 and +0 compare equal
  const uint32_t o = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return (static_cast<unsigned long long>(o) << 32) | static_cast<uint32_t>(~e);
}

__device__ __forceinline__ unsigned long long shfl_key(unsigned long long k, int m) {
  return __shfl_xor_sync(0xffffffffu, k, m);
}

// 32 keys over the lanes of a warp -> descending (lane 0 holds the largest)
__device__ __forceinline__ unsigned long long warp_sort_desc(unsigned long long k, int lane) {
#pragma unroll
  for (int blk = 2; blk <= 32; blk <<= 1) {
#pragma unroll
    for (int m = blk >> 1; m > 0; m >>= 1) {
      const unsigned long long o = shfl_key(k, m);
      // inside a descending block the lower lane of a pair keeps the larger key
      const bool desc = (lane & blk) == 0, lower = (lane & m) == 0;
      k = (desc == lower) ? (o > k ? o : k) : (o < k ? o : k);
    }
  }
  return k;
}

// k: a descending run over the lanes; p: lane's key of a descending partner run taken in reverse
// order.  Returns the best 32 of both runs, descending.
__device__ __forceinline__ unsigned long long warp_merge_best(unsigned long long k, unsigned long long p, int lane) {
  k = p > k ? p : k;  // bitonic, holds the 32 largest keys of the union
#pragma unroll
  for (int m = 16; m > 0; m >>= 1) {
    const unsigned long long o = shfl_key(k, m);
    k = ((lane & m) == 0) ? (o > k ? o : k) : (o < k ? o : k);
  }
  return k;
}

__global__ void __launch_bounds__(512) router_select_kernel(const float* __restrict__ scores,
                                                            const float* __restrict__ bias, int E, int topk,
                                                            float scale, int* __restrict__ idx,
                                                            float* __restrict__ wout) {
  __shared__ unsigned long long runs[16][32];
  __shared__ float srow[512];
  pdl_trigger();
  pdl_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  const int64_t r = blockIdx.x;
  const int e = threadIdx.x;
  float s = 0.f;
  unsigned long long key = 0ull;
  if (e < E) {
    s = scores[r * E + e];
    key = route_key(s + bias[e], e);
  }
  srow[e] = s;
  key = warp_sort_desc(key, lane);
  for (int span = 1; span < nw; span <<= 1) {
    runs[warp][lane] = key;
    __syncthreads();
    if ((warp & (2 * span - 1)) == 0 && warp + span < nw) key = warp_merge_best(key, runs[warp + span][31 - lane], lane);
    __syncthreads();
  }
  if (nw == 1) __syncwarp();  // srow written by this warp only
  if (warp != 0) return;
  const bool chosen = lane < topk && (key >> 32) != 0ull;
  const int ce = chosen ? static_cast<int>(~static_cast<uint32_t>(key)) : -1;
  const float cs = chosen ? srow[ce] : 0.f;
  // the weights' denominator adds the chosen scores in selection order, as the op defines it
  float total = 0.f;
  for (int j = 0; j < topk; ++j) total += __shfl_sync(0xffffffffu, cs, j);
  if (lane < topk) {
    idx[r * topk + lane] = ce;
    wout[r * topk + lane] = cs / (total + 1e-20f) * scale;
  }
}

// =======================================================================================
// MoeDecode, SIMT fallback for inter sizes that are not a multiple of 256: segmented
// exact-weight streaming GEMV (int4, zero point 8, bf16 block-32 scales)
// =======================================================================================
constexpr int kMaxPairs = 128;
constexpr int kSegWarps = 8;
constexpr int kSegThreads = kSegWarps * 32;
constexpr int kSegRows = 8;  // rows per stage

struct SegParams {
  const bf16* x;         // fc1: z [R, K]; fc2: h [P, K]
  const int* idx;        // [P] expert ids
  const float* w;        // [P] routing weights (fc2 finalize)
  const uint8_t* wq;     // [E, Nseg, K/2]
  const bf16* sc;        // [E, Nseg, K/32]
  bf16* h_out;           // fc1 output [P, Nseg]
  float* part_out;       // fc2 output [P, Nseg]
  bf16* out;             // fc2 finalize output [R, Nseg]
  int P, topk, E, Nseg, K;
  int nstage;
  uint32_t stage_bytes;
  int early_weights;
};

// stage s of a CTA: segment p = s / spp, rows [a + (s % spp) * 8, ...) of that segment
struct SegRange {
  int a, b, spp;
};

__device__ __forceinline__ SegRange seg_range(const SegParams& p) {
  SegRange r;
  r.a = static_cast<int>(static_cast<int64_t>(blockIdx.x) * p.Nseg / gridDim.x);
  r.b = static_cast<int>(static_cast<int64_t>(blockIdx.x + 1) * p.Nseg / gridDim.x);
  r.spp = (r.b - r.a + kSegRows - 1) / kSegRows;
  return r;
}

// Reads at L2 (the coherence point): kernels that start early under programmatic dependent
// launch read values produced before their primary's wait this way, never from L1.
__device__ __forceinline__ int ld_cg(const int* p) {
  int v;
  asm volatile("ld.global.cg.s32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}

__device__ __forceinline__ int load_expert(const int* idx, int pp) { return ld_cg(idx + pp); }

__device__ __forceinline__ void seg_issue(const SegParams& p, uint8_t* smem, uint64_t* full_bar, const SegRange& rg,
                                          int s, int e) {
  const int slot_i = s % p.nstage;
  const int pp = s / rg.spp;
  const int row = rg.a + (s % rg.spp) * kSegRows;
  const int rows = min(kSegRows, rg.b - row);
  uint8_t* slot = smem + static_cast<size_t>(slot_i) * p.stage_bytes;
  const uint32_t fb = smem_u32(&full_bar[slot_i]);
  uint32_t tx = 0;
  if (e >= 0 && e < p.E && rows > 0) {
    const int64_t rb = p.K / 2;
    const int nb = p.K / 32;
    const int64_t grow = static_cast<int64_t>(e) * p.Nseg + row;
    bulk_g2s(smem_u32(slot), p.wq + grow * rb, static_cast<uint32_t>(rows * rb), fb);
    tx += static_cast<uint32_t>(rows * rb);
    const uint8_t* scb = reinterpret_cast<const uint8_t*>(p.sc);
    stage_span(slot + kSegRows * rb, scb + grow * nb * 2, rows * nb * 2, scb + static_cast<int64_t>(p.E) * p.Nseg * nb * 2,
               fb, tx);
  }
  mbar_arrive_expect_tx(fb, tx);
}

// FC: 1 = fc1 (relu2 -> h), 2 = fc2 (part, then this CTA's rows of out)
template <int FC, int TPR, int SPT>
__global__ void __launch_bounds__(kSegThreads, 1) moe_seg_kernel(const SegParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  constexpr int RP = kSegThreads / TPR;
  constexpr int NP = kSegRows / RP;
  __shared__ uint64_t full_bar[16];
  __shared__ float red[2][kSegWarps][kSegRows];
  __shared__ int experts[kMaxPairs];
  __shared__ float part_s[FC == 2 ? kMaxPairs * kSegRows * 2 : 1];
  __shared__ volatile int abort_flag;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const SegRange rg = seg_range(p);
  const int nst = rg.spp * p.P;
  const int NS = p.nstage;
  const int K = p.K;
  const int nb = K >> 5;
  const int64_t rb = K / 2;

  if (tid == 0) {
    for (int s = 0; s < NS; ++s) mbar_init(smem_u32(&full_bar[s]), 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  if (FC == 1) {
    // the routing ids are this op's inputs: wait for the producer of those before reading
    pdl_wait();
    pdl_trigger();
  } else {
    pdl_trigger();
    if (!p.early_weights) pdl_wait();
  }
  for (int i = tid; i < p.P; i += kSegThreads) experts[i] = load_expert(p.idx, i);
  __syncthreads();
  if (tid == 0)
    for (int s = 0; s < min(NS, nst); ++s) seg_issue(p, smem, full_bar, rg, s, experts[s / rg.spp]);
  pdl_wait();

  const int grp = tid / TPR, pt = tid % TPR;
  const int nslots = K >> 4;
  float2 xv[SPT][8];
  float xoff[SPT];
  int xsrc = -1;  // activation row currently held in registers

  for (int s = 0; s < nst; ++s) {
    const int slot_i = s % NS;
    const uint32_t ph = (s / NS) & 1;
    const int pp = s / rg.spp;
    const int row0 = rg.a + (s % rg.spp) * kSegRows;
    const int rows = min(kSegRows, rg.b - row0);
    const int e = experts[pp];
    const bool live = e >= 0 && e < p.E;
    if (!abort_flag && !mbar_wait(smem_u32(&full_bar[slot_i]), ph, kStatusFullWait)) abort_flag = 1;
    const int src = (FC == 1) ? pp / p.topk : pp;
    if (live && src != xsrc) {
      xsrc = src;
#pragma unroll
      for (int j = 0; j < SPT; ++j) {
        const int slot = pt + j * TPR;
        float xf[16];
        if (slot < nslots) {
          const uint4* xp = reinterpret_cast<const uint4*>(p.x + static_cast<int64_t>(src) * K + slot * 16);
          const uint4 a = xp[0], b = xp[1];
          const uint32_t u[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            xf[2 * i] = __uint_as_float(u[i] << 16);
            xf[2 * i + 1] = __uint_as_float(u[i] & 0xFFFF0000u);
          }
        } else {
#pragma unroll
          for (int i = 0; i < 16; ++i) xf[i] = 0.f;
        }
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          xv[j][4 * q + 0] = make_float2(xf[8 * q + 0], xf[8 * q + 2]);
          xv[j][4 * q + 1] = make_float2(xf[8 * q + 4], xf[8 * q + 6]);
          xv[j][4 * q + 2] = make_float2(xf[8 * q + 1], xf[8 * q + 3]);
          xv[j][4 * q + 3] = make_float2(xf[8 * q + 5], xf[8 * q + 7]);
        }
        float sum = 0.f;
#pragma unroll
        for (int i = 0; i < 16; ++i) sum += xf[i];
        xoff[j] = -136.f * sum;
      }
    }
    const uint8_t* slot_w = smem + static_cast<size_t>(slot_i) * p.stage_bytes;
    const int64_t grow = static_cast<int64_t>(live ? e : 0) * p.Nseg + row0;
    const uint8_t* slot_sc = slot_w + kSegRows * rb + (reinterpret_cast<uintptr_t>(p.sc + grow * nb) & 15);

    float part[NP];
#pragma unroll
    for (int u = 0; u < NP; ++u) {
      const int rl = u * RP + grp;
      float acc = 0.f;
      if (live && rl < rows) {
        const uint8_t* wrow = slot_w + rl * rb;
        const bf16* srow = reinterpret_cast<const bf16*>(slot_sc) + rl * nb;
#pragma unroll
        for (int j = 0; j < SPT; ++j) {
          const int slot = pt + j * TPR;
          if (slot < nslots) {
            const float scv = __bfloat162float(srow[slot >> 1]);
            const uint2 wv = *reinterpret_cast<const uint2*>(wrow + slot * 8);
            const uint32_t M = 0x3F000000u;
            const uint32_t wd[2] = {wv.x, wv.y};
            float2 a = make_float2(0.f, 0.f), b = make_float2(0.f, 0.f);
#pragma unroll
            for (int q = 0; q < 2; ++q) {
              const uint32_t lo = wd[q] & 0x0F0F0F0Fu, hi = (wd[q] >> 4) & 0x0F0F0F0Fu;
              a = ffma2(make_float2(__uint_as_float(prmt(lo, M, 0x7044)), __uint_as_float(prmt(lo, M, 0x7144))),
                        xv[j][4 * q + 0], a);
              b = ffma2(make_float2(__uint_as_float(prmt(lo, M, 0x7244)), __uint_as_float(prmt(lo, M, 0x7344))),
                        xv[j][4 * q + 1], b);
              a = ffma2(make_float2(__uint_as_float(prmt(hi, M, 0x7044)), __uint_as_float(prmt(hi, M, 0x7144))),
                        xv[j][4 * q + 2], a);
              b = ffma2(make_float2(__uint_as_float(prmt(hi, M, 0x7244)), __uint_as_float(prmt(hi, M, 0x7344))),
                        xv[j][4 * q + 3], b);
            }
            const float S = (a.x + a.y) + (b.x + b.y);
            acc = fmaf(fmaf(256.f, S, xoff[j]), scv, acc);
          }
        }
      }
      part[u] = acc;
    }
    // reduce-scatter over lanes, then across the warps of each row group
    {
      int o = 16;
#pragma unroll
      for (int n = NP; n > 1; n >>= 1, o >>= 1) {
        const bool upper = (lane & o) != 0;
#pragma unroll
        for (int i = 0; i < n / 2; ++i) {
          const float send = upper ? part[i] : part[i + n / 2];
          const float keep = upper ? part[i + n / 2] : part[i];
          part[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
        }
      }
#pragma unroll
      for (; o >= 1; o >>= 1) part[0] += __shfl_xor_sync(0xffffffffu, part[0], o);
    }
    constexpr int kLanesPerRow = 32 / NP;
    constexpr int kLog2NP = NP == 8 ? 3 : NP == 4 ? 2 : NP == 2 ? 1 : 0;
    const int buf = s & 1;
    if ((lane & (kLanesPerRow - 1)) == 0) red[buf][warp][((lane >> (5 - kLog2NP)) & (NP - 1)) * RP + grp] = part[0];
    asm volatile("bar.sync 1;" ::: "memory");
    if (tid == 0 && s + NS < nst && !abort_flag) seg_issue(p, smem, full_bar, rg, s + NS, experts[(s + NS) / rg.spp]);
    if (tid < rows) {
      const int rl = tid;
      const int gg = rl % RP;
      constexpr int WPG = TPR / 32;
      float tsum = 0.f;
#pragma unroll
      for (int w = 0; w < WPG; ++w) tsum += red[buf][gg * WPG + w][rl];
      const int64_t o = static_cast<int64_t>(pp) * p.Nseg + row0 + rl;
      const float bfv = __bfloat162float(__float2bfloat16(tsum));
      if (FC == 1) {
        const float r = live ? fmaxf(bfv, 0.f) : 0.f;
        p.h_out[o] = __float2bfloat16(r * r);
      } else {
        const float v = live ? bfv : 0.f;
        p.part_out[o] = v;
        part_s[pp * kSegRows * 2 + (s % rg.spp) * kSegRows + rl] = v;
      }
    }
  }
  if constexpr (FC == 2) {
    // out[t, n] = bf16(sum_k w[t, k] * part[t * topk + k, n]) for this CTA's rows, k ascending
    __syncthreads();
    const int R = p.P / p.topk;
    const int nrow = rg.b - rg.a;
    for (int i = tid; i < R * nrow; i += kSegThreads) {
      const int t = i / nrow, rl = i % nrow;
      float a = 0.f;
      for (int k = 0; k < p.topk; ++k) {
        const int pp = t * p.topk + k;
        a = fmaf(p.w[pp], part_s[pp * kSegRows * 2 + rl], a);
      }
      p.out[static_cast<int64_t>(t) * p.Nseg + rg.a + rl] = __float2bfloat16(a);
    }
  }
  if (tid == 0 && abort_flag)
    for (int s = max(0, nst - NS); s < nst; ++s) mbar_wait(smem_u32(&full_bar[s % NS]), (s / NS) & 1, kStatusDrainWait);
}

// =======================================================================================
// MoeVerify grouping and the finalize
// =======================================================================================
// meta: [0] = U, [1 .. P] = unique expert ids in first-occurrence order (unused slots -1),
// [1 + P + u * 8 + row] = pair index of `row` for unique expert u, or -1.
// Experts outside [e_begin, e_end) (the shard's range; the whole [0, E) unsharded) are left
// out of the list.
__global__ void __launch_bounds__(128) moe_group_kernel(const int* __restrict__ idx, int P, int topk, int e_begin,
                                                        int e_end, int* __restrict__ meta) {
  __shared__ int sid[kMaxPairs];
  __shared__ int srank[kMaxPairs];
  __shared__ int wtot[4];
  pdl_wait();
  pdl_trigger();
  const int p = threadIdx.x, lane = p & 31, warp = p >> 5;
  for (int i = p; i < 8 * P + P; i += blockDim.x) meta[1 + i] = -1;
  const int e = p < P ? idx[p] : -1;
  if (p < P) sid[p] = e;
  __syncthreads();
  const bool local = p < P && e >= e_begin && e < e_end;
  int first = -1;
  if (local) {
    for (int j = 0; j <= p; ++j)
      if (sid[j] == e) { first = j; break; }
  }
  const bool lead = local && first == p;
  const unsigned bal = __ballot_sync(0xffffffffu, lead);
  if (lane == 0) wtot[warp] = __popc(bal);
  __syncthreads();
  int off = 0;
  for (int w = 0; w < warp; ++w) off += wtot[w];
  if (lead) srank[p] = off + __popc(bal & ((1u << lane) - 1u));
  __syncthreads();  // the -1 fill above is complete before the writes below (same threads' order
                    // is not enough: another thread may own the slot)
  if (lead) meta[1 + srank[p]] = e;
  if (local) meta[1 + P + srank[first] * 8 + p / topk] = p;
  if (p == 0) meta[0] = wtot[0] + wtot[1] + wtot[2] + wtot[3];
}

// sum over token t's local pairs of w * part[., n] (k ascending).  round_part: part holds fp32
// sums; each pair's fc2 output is bf16(part), written back so part holds the per-pair outputs.
__device__ __forceinline__ float local_partial(float* __restrict__ part, int round_part, const float* __restrict__ w,
                                               const int* __restrict__ idx, int t, int n, int topk, int Nout,
                                               int e_begin, int e_end) {
  // batches of 8 pairs: their ids, then their values, load together (two round trips per batch
  // instead of two per pair); the sum stays in k order
  constexpr int kB = 8;
  float a = 0.f;
  for (int k0 = 0; k0 < topk; k0 += kB) {
    bool use[kB];
    float v[kB], wk[kB];
#pragma unroll
    for (int j = 0; j < kB; ++j) {
      const int k = k0 + j;
      const int e = k < topk ? idx[t * topk + k] : -1;
      use[j] = k < topk && e >= e_begin && e < e_end;
    }
#pragma unroll
    for (int j = 0; j < kB; ++j) {
      const int pp = t * topk + k0 + j;
      v[j] = use[j] ? part[static_cast<int64_t>(pp) * Nout + n] : 0.f;
      wk[j] = use[j] ? w[pp] : 0.f;
    }
#pragma unroll
    for (int j = 0; j < kB; ++j) {
      if (!use[j]) continue;
      if (round_part) {
        v[j] = __bfloat162float(__float2bfloat16(v[j]));
        part[static_cast<int64_t>(t * topk + k0 + j) * Nout + n] = v[j];
      }
      a = fmaf(wk[j], v[j], a);
    }
  }
  return a;
}

// out[t] = the local partial of token t (bf16 and / or fp32).
__global__ void __launch_bounds__(256) moe_finalize_kernel(float* __restrict__ part, int round_part,
                                                           const float* __restrict__ w,
                                                           const int* __restrict__ idx, int R, int topk, int Nout,
                                                           int e_begin, int e_end, bf16* __restrict__ out,
                                                           float* __restrict__ out_f32) {
  pdl_wait();
  pdl_trigger();
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= static_cast<int64_t>(R) * Nout) return;
  const int t = static_cast<int>(i / Nout), n = static_cast<int>(i % Nout);
  const float a = local_partial(part, round_part, w, idx, t, n, topk, Nout, e_begin, e_end);
  if (out) out[i] = __float2bfloat16(a);
  if (out_f32) out_f32[i] = a;
}

// Expert-sharded finalize fused with the all-reduce over NVLink peer memory (no NCCL): CTA c owns
// a slice of the R x Nout outputs on every rank.  It computes this rank's partials of its slice and
// pushes them into slot `rank` of every rank's peer-visible buffer (half e & 1 of it, e = the CTA's
// call count; posted stores, no remote loads), publishes e to its flag word on every peer
// (system-scope release after a system fence), waits for every peer's e in its own flag words
// (acquire; bounded, status bit on timeout), then sums the slice of all slots in rank order -- the
// same order on every rank, so all ranks get identical bits -- from local memory and writes bf16.
// A rank writes half h at call e only after every rank's flags for call e - 1 arrived, and a rank
// sums half h of call e - 2 before it raises its flags for call e - 1, so alternating halves keeps
// every write off data still being read.  The call counters advance in device memory, so a
// replayed CUDA graph stays in step.
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// rank q's flag words: after its two halves of world slots of partials
__device__ __forceinline__ uint32_t* peer_flags(const PeerReduce& pr, int q) {
  return reinterpret_cast<uint32_t*>(pr.bufs[q] + 2 * pr.world * pr.stride);
}

__global__ void __launch_bounds__(256) moe_finalize_allreduce_kernel(float* __restrict__ part, int round_part,
                                                                     const float* __restrict__ w,
                                                                     const int* __restrict__ idx, int R, int topk,
                                                                     int Nout, int e_begin, int e_end, PeerReduce pr,
                                                                     bf16* __restrict__ out) {
  __shared__ uint32_t s_e;
  __shared__ int s_ok;
  pdl_wait();
  pdl_trigger();
  const int c = blockIdx.x, tid = threadIdx.x;
  const int64_t n = static_cast<int64_t>(R) * Nout;
  const int64_t i0 = static_cast<int64_t>(c) * n / gridDim.x, i1 = static_cast<int64_t>(c + 1) * n / gridDim.x;
  if (tid == 0) {
    s_e = __ldcg(pr.epoch + c) + 1u;
    s_ok = 1;
  }
  __syncthreads();
  const uint32_t e = s_e;
  const int64_t half = static_cast<int64_t>(e & 1u) * pr.world * pr.stride;
  const int64_t slot = half + static_cast<int64_t>(pr.rank) * pr.stride;
  for (int64_t i = i0 + tid; i < i1; i += blockDim.x) {
    const int t = static_cast<int>(i / Nout), col = static_cast<int>(i % Nout);
    const float v = local_partial(part, round_part, w, idx, t, col, topk, Nout, e_begin, e_end);
    for (int q = 0; q < pr.world; ++q) pr.bufs[q][slot + i] = v;  // this rank's slot on every rank
  }
  __syncthreads();
  if (tid == 0) {
    __threadfence_system();  // the CTA's pushed partials are visible to the peers before its flags
    for (int q = 0; q < pr.world; ++q)
      if (q != pr.rank) st_release_sys(peer_flags(pr, q) + c * pr.world + pr.rank, e);
    const unsigned long long t0 = globaltimer();
    for (int q = 0; q < pr.world && s_ok; ++q) {
      if (q == pr.rank) continue;
      const uint32_t* f = peer_flags(pr, pr.rank) + c * pr.world + q;
      while (static_cast<int>(ld_acquire_sys(f) - e) < 0) {
        if (globaltimer() - t0 > kWaitLimitNs) {
          set_status(kStatusGridWait);
          s_ok = 0;
          break;
        }
      }
    }
    pr.epoch[c] = e;
  }
  __syncthreads();
  if (!s_ok) return;
  const float* mine = pr.bufs[pr.rank] + half;
  for (int64_t i = i0 + tid; i < i1; i += blockDim.x) {
    float s = 0.f;
    for (int q = 0; q < pr.world; ++q) s += __ldcg(mine + static_cast<int64_t>(q) * pr.stride + i);
    out[i] = __float2bfloat16(s);
  }
}

template <int FC, int TPR, int SPT>
cudaError_t launch_seg(const SegParams& p, int grid, const LaunchCfg& cfg) {
  auto kern = moe_seg_kernel<FC, TPR, SPT>;
  const size_t smem = static_cast<size_t>(p.nstage) * p.stage_bytes;
  static SmemOptIn opt;
  cudaError_t e = allow_smem(kern, smem, opt);
  if (e != cudaSuccess) return e;
  return launch_kernel(kern, dim3(grid), dim3(kSegThreads), smem, cfg, p);
}

// threads per row: the candidate with the best lane utilisation (nslots / (TPR * SPT))
template <int FC>
cudaError_t dispatch_seg(SegParams& p, int grid, const LaunchCfg& cfg) {
  const int nslots = p.K >> 4;
  int best = 0;
  double best_u = -1.0;
  const int cand[4] = {256, 128, 64, 32};
  for (int c : cand) {
    const int spt = (nslots + c - 1) / c;
    if (spt > 5) continue;
    const double u = static_cast<double>(nslots) / (c * spt);
    if (u > best_u + 1e-9) { best_u = u; best = c; }
  }
  const int spt = (nslots + best - 1) / best;
  switch (best * 10 + spt) {
    case 2561: return launch_seg<FC, 256, 1>(p, grid, cfg);
    case 2562: return launch_seg<FC, 256, 2>(p, grid, cfg);
    case 2563: return launch_seg<FC, 256, 3>(p, grid, cfg);
    case 2564: return launch_seg<FC, 256, 4>(p, grid, cfg);
    case 2565: return launch_seg<FC, 256, 5>(p, grid, cfg);
    case 1281: return launch_seg<FC, 128, 1>(p, grid, cfg);
    case 1282: return launch_seg<FC, 128, 2>(p, grid, cfg);
    case 641: return launch_seg<FC, 64, 1>(p, grid, cfg);
    case 642: return launch_seg<FC, 64, 2>(p, grid, cfg);
    case 643: return launch_seg<FC, 64, 3>(p, grid, cfg);
    case 321: return launch_seg<FC, 32, 1>(p, grid, cfg);
    case 322: return launch_seg<FC, 32, 2>(p, grid, cfg);
    case 323: return launch_seg<FC, 32, 3>(p, grid, cfg);
    case 324: return launch_seg<FC, 32, 4>(p, grid, cfg);
    case 325: return launch_seg<FC, 32, 5>(p, grid, cfg);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

cudaError_t launch_moe_route(const bf16* x, const bf16* gate_w, const float* bias, int R, int K, int E, int topk,
                             float scale, int* idx, float* w, float* scores, const LaunchCfg& cfg) {
  const unsigned blocks = static_cast<unsigned>((E + kRouteExperts - 1) / kRouteExperts);
  const int early = cfg.early_weights ? 1 : 0;
  cudaError_t e;
  if (R <= 1) {
    e = launch_kernel(router_logits_kernel<1>, dim3(blocks), dim3(kRouteThreads), kRoutePassVec * sizeof(uint4), cfg,
                      x, gate_w, R, K, E, early, scores);
  } else {
    constexpr size_t smem = 8 * kRoutePassVec * sizeof(uint4);
    static SmemOptIn opt;
    e = allow_smem(router_logits_kernel<8>, smem, opt);
    if (e == cudaSuccess)
      e = launch_kernel(router_logits_kernel<8>, dim3(blocks), dim3(kRouteThreads), smem, cfg, x, gate_w, R, K, E,
                        early, scores);
  }
  if (e != cudaSuccess) return e;
  LaunchCfg c2 = cfg;
  c2.pdl = true;  // same op: the selection waits for the logits with griddepcontrol.wait
  const unsigned threads = static_cast<unsigned>(32 * ((E + 31) / 32));
  return launch_kernel(router_select_kernel, dim3(R), dim3(threads), 0, c2, scores, bias, E, topk, scale, idx, w);
}

cudaError_t launch_moe_decode_simt(const bf16* z, const int* idx, const float* w, const uint8_t* fc1_w, const bf16* fc1_s,
                              const uint8_t* fc2_w, const bf16* fc2_s, int R, int E, int I, int topk, bf16* out,
                              bf16* h, float* part, const LaunchCfg& cfg) {
  const int P = R * topk;
  const int grid1 = std::min(cfg.sms, std::max(1, I / kSegRows));
  SegParams p1{z, idx, w, fc1_w, fc1_s, h, nullptr, nullptr, P, topk, E, I, 1024, 0, 0, cfg.early_weights ? 1 : 0};
  p1.stage_bytes = (kSegRows * 512 + kSegRows * 64 + 32 + 127) & ~127u;
  const int want1 = P * ((I / grid1 + kSegRows) / kSegRows + 1);
  p1.nstage = std::max(2, std::min({want1, static_cast<int>((cfg.smem_budget ? cfg.smem_budget : 200 * 1024) / p1.stage_bytes), 16}));
  cudaError_t e = dispatch_seg<1>(p1, grid1, cfg);
  if (e != cudaSuccess) return e;
  LaunchCfg c2 = cfg;
  c2.pdl = true;
  c2.early_weights = true;  // fc1 triggers only after its own wait: every input of this op is ready
  const int grid2 = std::max(64, std::min(cfg.sms, 1024));  // <= 16 rows of every pair per CTA
  SegParams p2{h, idx, w, fc2_w, fc2_s, nullptr, part, out, P, topk, E, 1024, I, 0, 0, 1};
  p2.stage_bytes = static_cast<uint32_t>((kSegRows * (I / 2) + kSegRows * (I / 16) + 32 + 127) & ~127);
  p2.nstage = std::max(2, std::min({P * 2, static_cast<int>((c2.smem_budget ? c2.smem_budget : 200 * 1024) / p2.stage_bytes), 16}));
  return dispatch_seg<2>(p2, grid2, c2);
}

cudaError_t launch_moe_group(const int* idx, int P, int topk, int e_begin, int e_end, int* meta, const LaunchCfg& cfg) {
  return launch_kernel(moe_group_kernel, dim3(1), dim3(128), 0, cfg, idx, P, topk, e_begin, e_end, meta);
}

cudaError_t launch_moe_finalize(float* part, int round_part, const float* w, const int* idx, int R, int topk,
                                int e_begin, int e_end, bf16* out, float* out_partial, const LaunchCfg& cfg) {
  const int64_t n = static_cast<int64_t>(R) * 1024;
  return launch_kernel(moe_finalize_kernel, dim3(static_cast<unsigned>((n + 255) / 256)), dim3(256), 0, cfg, part,
                       round_part, w, idx, R, topk, 1024, e_begin, e_end, out, out_partial);
}


cudaError_t launch_moe_finalize_allreduce(float* part, int round_part, const float* w, const int* idx, int R,
                                          int topk, int e_begin, int e_end, const PeerReduce& pr, bf16* out,
                                          const LaunchCfg& cfg) {
  if (pr.world < 1 || pr.rank < 0 || pr.rank >= pr.world || pr.stride < static_cast<int64_t>(R) * 1024)
    return cudaErrorInvalidValue;
  return launch_kernel(moe_finalize_allreduce_kernel, dim3(kPeerReduceCtas), dim3(256), 0, cfg, part, round_part, w,
                       idx, R, topk, 1024, e_begin, e_end, pr, out);
}

}  // namespace bolt
