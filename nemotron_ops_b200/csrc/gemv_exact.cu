// Exact-weight SIMT GEMV for Q8Gemv / Q4Gemv (block-32, bf16 scales, zero point 128 / 8).
//
// Contract (reference src/bolt_ops.cu:1315-1392, :480-494): every weight is the exact fp32
// product (q - zp) * s, products with bf16 x are accumulated in fp32, y = bf16(sum).  This is
// the path the reference takes for R = 1 and for any R when K % 64 != 0.
//
// B200 design (not a translation of QGemvKernel):
//  * persistent grid, one CTA per SM, each CTA owns a contiguous range of weight rows, so its
//    weight bytes are one contiguous span of HBM;
//  * 16-row stages (weights + the matching scale span) are streamed with cp.async.bulk into an
//    smem ring guarded by mbarriers; the whole per-CTA working set of the benchmark shapes is
//    in flight from the first microsecond;
//  * 16 warps compute: each thread owns 16-wide k slots of every row, keeps its x
//    slice in fp32 registers for the life of the CTA and dequantises with one prmt per weight
//    into a float whose mantissa carries the code (Q4: 0.5 + n/256; Q8: 2^23 + b), feeding
//    packed fma.rn.f32x2;
//  * rows are reduced with a butterfly (reduce-scatter) over lanes; the cross-warp sum of a ring
//    slot is done by the last warp to finish it, which also refills the slot -- there is no
//    CTA-wide barrier in the main loop, so no warp waits for another.
#include "common.cuh"
#include "kernels.h"

namespace bolt {

namespace {

constexpr int kWarps = 16;
constexpr int kThreads = kWarps * 32;
constexpr int kRowsPerStage = 16;

struct ExactParams {
  const bf16* x;
  const uint8_t* w;
  const bf16* sc;
  bf16* y;
  int64_t N;
  int K;
  int nstage;
  uint32_t stage_bytes;  // bytes of one ring slot (weights + scale span), multiple of 128
  int early_weights;     // stream weights before griddepcontrol.wait (weights are constants)
};

// Reduce-scatter of NP per-row partials across the 32 lanes of a warp.  Afterwards every lane
// holds the warp total of row (lane >> (5 - log2 NP)) & (NP - 1).
template <int NP>
__device__ __forceinline__ float warp_reduce_rows(float (&v)[NP], int lane) {
  int o = 16;
#pragma unroll
  for (int n = NP; n > 1; n >>= 1, o >>= 1) {
    const bool upper = (lane & o) != 0;
#pragma unroll
    for (int i = 0; i < n / 2; ++i) {
      const float send = upper ? v[i] : v[i + n / 2];
      const float keep = upper ? v[i + n / 2] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
    }
  }
#pragma unroll
  for (; o >= 1; o >>= 1) v[0] += __shfl_xor_sync(0xffffffffu, v[0], o);
  return v[0];
}

template <int NP>
struct Log2 {
  static constexpr int v = NP == 16 ? 4 : NP == 8 ? 3 : NP == 4 ? 2 : NP == 2 ? 1 : 0;
};

// Issues the bulk copies of stage `i` (16 rows + their scale span) into ring slot i % NS.
// Called by all lanes of one warp: lane 1 issues the weight copy, lane 0 the scale span and
// the byte count (issuing a bulk copy costs a thread ~100 ns, so the two run side by side).
template <int BITS>
__device__ __forceinline__ void exact_issue_stage(const ExactParams& p, uint8_t* smem, uint64_t* full_bar, int i,
                                                  int64_t r0, int nrows, int lane) {
  const int nb = p.K >> 5;
  const uint32_t row_bytes = static_cast<uint32_t>(p.K) * BITS / 8;
  const int s = i % p.nstage;
  const int64_t row = r0 + static_cast<int64_t>(i) * kRowsPerStage;
  const int rows = min(kRowsPerStage, nrows - i * kRowsPerStage);
  uint8_t* slot = smem + static_cast<size_t>(s) * p.stage_bytes;
  const uint32_t fb = smem_u32(&full_bar[s]);
  const uint8_t* sc_bytes = reinterpret_cast<const uint8_t*>(p.sc);
  uint32_t tx = rows * row_bytes;
  if (lane == 1) bulk_g2s(smem_u32(slot), p.w + row * row_bytes, rows * row_bytes, fb);
  if (lane == 0) {
    stage_span(slot + kRowsPerStage * row_bytes, sc_bytes + row * nb * 2, rows * nb * 2, sc_bytes + p.N * nb * 2, fb, tx);
    mbar_arrive_expect_tx(fb, tx);
  }
  __syncwarp();
}

// Returns true in every lane of the warp that is the last of kWarps to finish ring slot `s`;
// that warp then sees every other warp's partials (release / acquire through the counter).
__device__ __forceinline__ bool last_warp_of_slot(int* cnt, int lane) {
  __threadfence_block();
  __syncwarp();
  int last = 0;
  if (lane == 0) last = atomicAdd(cnt, 1) == kWarps - 1;
  last = __shfl_sync(0xffffffffu, last, 0);
  if (last) __threadfence_block();
  return last != 0;
}

// BITS: 4 or 8.  TPR: threads per row (256, 128 or 64).  SPT: 16-k slots per thread.
// No CTA-wide barrier after the prologue: each warp writes the per-row partials of a ring slot
// into red[slot], and the last warp to finish the slot sums them, writes those rows of y and
// refills the slot with the stage NS ahead.
template <int BITS, int TPR, int SPT>
__global__ void __launch_bounds__(kThreads, 1) gemv_exact_kernel(const ExactParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  constexpr int RP = kThreads / TPR;         // rows processed side by side
  constexpr int NP = kRowsPerStage / RP;     // rows a thread touches per stage
  constexpr int WPG = TPR / 32;              // warps per row group
  constexpr int SLOT_BYTES = BITS * 2;       // 16 weights
  __shared__ uint64_t full_bar[16];
  __shared__ int done_cnt[16];
  __shared__ float red[16][kWarps][kRowsPerStage];
  __shared__ volatile int abort_flag;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int K = p.K;
  const int nb = K >> 5;                       // scale blocks per row
  const uint32_t row_bytes = static_cast<uint32_t>(K) * BITS / 8;
  const int64_t r0 = static_cast<int64_t>(blockIdx.x) * p.N / gridDim.x;
  const int64_t r1 = static_cast<int64_t>(blockIdx.x + 1) * p.N / gridDim.x;
  const int nrows = static_cast<int>(r1 - r0);
  const int ntiles = (nrows + kRowsPerStage - 1) / kRowsPerStage;
  const int NS = p.nstage;

  if (tid == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(smem_u32(&full_bar[s]), 1);
      done_cnt[s] = 0;
    }
    abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  if (warp == 0) {
    if (p.early_weights) {
      if (lane == 0) {
        prefetch_span_l2(p.w + r0 * row_bytes, static_cast<uint64_t>(nrows) * row_bytes);
        prefetch_span_l2(p.sc + r0 * nb, static_cast<uint64_t>(nrows) * nb * 2);
      }
    } else {
      pdl_wait();
    }
    for (int i = 0; i < min(NS, ntiles); ++i) exact_issue_stage<BITS>(p, smem, full_bar, i, r0, nrows, lane);
  }
  pdl_wait();

  const int rg = tid / TPR;         // row group
  const int pt = tid % TPR;         // position inside the row group
  const int nslots = K >> 4;

  // x slice: xv[j][0..7] float2 pairs arranged to match the dequant order below
  float2 xv[SPT][8];
  float xoff[SPT];  // Q4: -136 * sum(x) of the slot; Q8: unused
#pragma unroll
  for (int j = 0; j < SPT; ++j) {
    const int slot = pt + j * TPR;
    float xf[16];
    if (slot < nslots) {
      const uint4* xp = reinterpret_cast<const uint4*>(p.x + slot * 16);
      const uint4 a = __ldg(xp), b = __ldg(xp + 1);
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
    if constexpr (BITS == 4) {
      // word q (bytes 4q..4q+3 of the slot): low nibbles = k 8q + {0,2,4,6}, high = 8q + {1,3,5,7}
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        xv[j][4 * q + 0] = make_float2(xf[8 * q + 0], xf[8 * q + 2]);
        xv[j][4 * q + 1] = make_float2(xf[8 * q + 4], xf[8 * q + 6]);
        xv[j][4 * q + 2] = make_float2(xf[8 * q + 1], xf[8 * q + 3]);
        xv[j][4 * q + 3] = make_float2(xf[8 * q + 5], xf[8 * q + 7]);
      }
      float s = 0.f;
#pragma unroll
      for (int i = 0; i < 16; ++i) s += xf[i];
      xoff[j] = -136.f * s;
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) xv[j][i] = make_float2(xf[2 * i], xf[2 * i + 1]);
      xoff[j] = 0.f;
    }
  }

  pdl_trigger();  // the next call's CTAs start once the activations are loaded, not during our first loads
  for (int i = 0; i < ntiles; ++i) {
    const int s = i % NS;
    const uint32_t ph = (i / NS) & 1;
    if (!abort_flag && !mbar_wait(smem_u32(&full_bar[s]), ph, kStatusFullWait)) abort_flag = 1;
    const uint8_t* slot_w = smem + static_cast<size_t>(s) * p.stage_bytes;
    const int64_t row0 = r0 + static_cast<int64_t>(i) * kRowsPerStage;
    const uint8_t* slot_sc = slot_w + kRowsPerStage * row_bytes +
                             (reinterpret_cast<uintptr_t>(p.sc + row0 * nb) & 15);
    const int rows = min(kRowsPerStage, nrows - i * kRowsPerStage);

    float part[NP];
#pragma unroll
    for (int u = 0; u < NP; ++u) {
      const int rl = u * RP + rg;  // row inside the stage
      float acc = 0.f;
      if (rl < rows) {
        const uint8_t* wrow = slot_w + rl * row_bytes;
        const bf16* srow = reinterpret_cast<const bf16*>(slot_sc) + rl * nb;
#pragma unroll
        for (int j = 0; j < SPT; ++j) {
          const int slot = pt + j * TPR;
          if (slot < nslots) {
            const float sc = __bfloat162float(srow[slot >> 1]);
            float2 a = make_float2(0.f, 0.f), b = make_float2(0.f, 0.f);
            if constexpr (BITS == 4) {
              const uint2 wv = *reinterpret_cast<const uint2*>(wrow + slot * SLOT_BYTES);
              const uint32_t M = 0x3F000000u;  // float 0x3F nn 00 00 = 0.5 + n / 256
              const uint32_t wd[2] = {wv.x, wv.y};
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
              acc = fmaf(fmaf(256.f, S, xoff[j]), sc, acc);  // sum (n - 8) x = 256 S - 136 sum x
            } else {
              const uint4 wv = *reinterpret_cast<const uint4*>(wrow + slot * SLOT_BYTES);
              const uint32_t M = 0x4B000000u;  // float 0x4B 00 00 bb = 2^23 + b
              const float2 zp = make_float2(-8388736.f, -8388736.f);
              const uint32_t wd[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                const float2 f01 = fadd2(make_float2(__uint_as_float(prmt(wd[q], M, 0x7440)),
                                                     __uint_as_float(prmt(wd[q], M, 0x7441))), zp);
                const float2 f23 = fadd2(make_float2(__uint_as_float(prmt(wd[q], M, 0x7442)),
                                                     __uint_as_float(prmt(wd[q], M, 0x7443))), zp);
                a = ffma2(f01, xv[j][2 * q], a);
                b = ffma2(f23, xv[j][2 * q + 1], b);
              }
              const float S = (a.x + a.y) + (b.x + b.y);
              acc = fmaf(S, sc, acc);
            }
          }
        }
      }
      part[u] = acc;
    }

    // rows of this stage: warp-level reduce-scatter into red[s]; the last warp sums the warps
    const float v = warp_reduce_rows<NP>(part, lane);
    constexpr int kLanesPerRow = 32 / NP;
    if ((lane & (kLanesPerRow - 1)) == 0) {
      const int li = (lane >> (5 - Log2<NP>::v)) & (NP - 1);
      red[s][warp][li * RP + rg] = v;
    }
    if (last_warp_of_slot(&done_cnt[s], lane)) {
      if (lane < rows) {
        const int grp = lane % RP;
        float t = 0.f;
#pragma unroll
        for (int w = 0; w < WPG; ++w) t += red[s][grp * WPG + w][lane];
        p.y[row0 + lane] = __float2bfloat16(t);
      }
      __syncwarp();
      if (lane == 0) done_cnt[s] = 0;
      if (i + NS < ntiles && !abort_flag) exact_issue_stage<BITS>(p, smem, full_bar, i + NS, r0, nrows, lane);
    }
  }
  if (tid == 0 && abort_flag)  // copies may still be landing: wait for them before exiting
    for (int i = max(0, ntiles - NS); i < ntiles; ++i)
      mbar_wait(smem_u32(&full_bar[i % NS]), (i / NS) & 1, kStatusDrainWait);
}

// Generic exact kernel for shapes the streaming kernel does not take (R > 1 with K % 64 != 0,
// K > 16384, or unaligned pointers): one warp per (row), every x row reused from L1.
template <int BITS>
__global__ void __launch_bounds__(256) gemv_exact_generic_kernel(const bf16* __restrict__ x, const uint8_t* __restrict__ w,
                                                                 const bf16* __restrict__ sc, bf16* __restrict__ y,
                                                                 int R, int64_t N, int K) {
  pdl_trigger();
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int64_t n = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (n >= N) return;
  const int nb = K >> 5;
  float acc[8];
#pragma unroll
  for (int r = 0; r < 8; ++r) acc[r] = 0.f;
  for (int b = lane; b < nb; b += 32) {
    const float s = __bfloat162float(sc[n * nb + b]);
    float wf[32];
    const uint8_t* wb = w + (n * nb + b) * (BITS * 4);
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      int q;
      if constexpr (BITS == 8) q = static_cast<int>(wb[i]) - 128;
      else q = static_cast<int>((wb[i >> 1] >> (4 * (i & 1))) & 15) - 8;
      wf[i] = static_cast<float>(q) * s;
    }
    for (int r = 0; r < R; ++r) {
      const bf16* xr = x + static_cast<int64_t>(r) * K + b * 32;
      float d = 0.f;
#pragma unroll
      for (int i = 0; i < 32; ++i) d = fmaf(wf[i], __bfloat162float(xr[i]), d);
      acc[r] += d;
    }
  }
  for (int r = 0; r < R; ++r) {
    const float v = warp_sum(acc[r]);
    if (lane == 0) y[static_cast<int64_t>(r) * N + n] = __float2bfloat16(v);
  }
}

template <int BITS, int TPR, int SPT>
cudaError_t launch_stream(const ExactParams& p, int grid, const LaunchCfg& cfg) {
  auto kern = gemv_exact_kernel<BITS, TPR, SPT>;
  const size_t smem = static_cast<size_t>(p.nstage) * p.stage_bytes;
  static SmemOptIn opt;
  cudaError_t e = allow_smem(kern, smem, opt);
  if (e != cudaSuccess) return e;
  return launch_kernel(kern, dim3(grid), dim3(kThreads), smem, cfg, p);
}

template <int BITS>
cudaError_t dispatch_stream(ExactParams& p, int grid, const LaunchCfg& cfg) {
  const int nslots = p.K >> 4;
  if (nslots >= 256) {
    const int spt = (nslots + 255) / 256;
    switch (spt) {
      case 1: return launch_stream<BITS, 256, 1>(p, grid, cfg);
      case 2: return launch_stream<BITS, 256, 2>(p, grid, cfg);
      case 3: return launch_stream<BITS, 256, 3>(p, grid, cfg);
      default: return launch_stream<BITS, 256, 4>(p, grid, cfg);
    }
  }
  // every 16-k slot needs a thread: TPR * SPT >= nslots
  if (nslots >= 128) return nslots > 128 ? launch_stream<BITS, 128, 2>(p, grid, cfg) : launch_stream<BITS, 128, 1>(p, grid, cfg);
  return nslots > 64 ? launch_stream<BITS, 64, 2>(p, grid, cfg) : launch_stream<BITS, 64, 1>(p, grid, cfg);
}

}  // namespace

bool gemv_exact_stream_ok(int R, int64_t N, int K, const void* x, const void* w, const void* sc) {
  const auto al = [](const void* q, uintptr_t a) { return (reinterpret_cast<uintptr_t>(q) & (a - 1)) == 0; };
  return R == 1 && N > 0 && K >= 1024 && K <= 16384 && K % 32 == 0 && al(x, 16) && al(w, 16) && al(sc, 2);
}

cudaError_t launch_gemv_exact(int bits, const bf16* x, int R, const uint8_t* w, const bf16* sc, int64_t N, int K,
                              bf16* y, const LaunchCfg& cfg) {
  if (bits == 8 && R == 1) {  // the staged R = 1 kernel (gemv_r1.cu) where it applies
    const cudaError_t e = launch_gemv_r1(kFmtQ8, x, w, sc, nullptr, N, K, y, cfg);
    if (e != cudaErrorNotSupported) return e;
  }
  const uint32_t budget = cfg.smem_budget ? cfg.smem_budget : 200 * 1024;
  const uint32_t stage_bytes =
      (kRowsPerStage * (static_cast<uint32_t>(K) * bits / 8) + kRowsPerStage * (K / 32) * 2 + 32 + 127) & ~127u;
  // the ring needs two stages in shared memory (Q8 with K > 6016 takes the generic kernel)
  if (gemv_exact_stream_ok(R, N, K, x, w, sc) && 2 * stage_bytes <= budget) {
    ExactParams p{x, w, sc, y, N, K, 0, 0, cfg.early_weights ? 1 : 0};
    p.stage_bytes = stage_bytes;
    const int grid = static_cast<int>(std::min<int64_t>(cfg.sms, (N + 7) / 8));
    const int64_t rows_per_cta = (N + grid - 1) / grid;
    const int want = static_cast<int>((rows_per_cta + kRowsPerStage - 1) / kRowsPerStage);
    const int fit = static_cast<int>(budget / p.stage_bytes);
    p.nstage = std::max(2, std::min({want, fit, 16}));
    return bits == 8 ? dispatch_stream<8>(p, grid, cfg) : dispatch_stream<4>(p, grid, cfg);
  }
  const int64_t grid = (N + 7) / 8;
  if (bits == 8)
    return launch_kernel(gemv_exact_generic_kernel<8>, dim3(static_cast<unsigned>(grid)), dim3(256), 0, cfg, x, w, sc, y, R, N, K);
  return launch_kernel(gemv_exact_generic_kernel<4>, dim3(static_cast<unsigned>(grid)), dim3(256), 0, cfg, x, w, sc, y, R, N, K);
}

}  // namespace bolt
