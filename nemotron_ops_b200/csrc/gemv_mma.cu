// Tensor-core skinny GEMV: y[R, N] = x[R, K] @ W^T for R <= 8 (mma.sync m16n8k16, fp32 acc).
//
// Used for Q8Gemv / Q4Gemv at 2 <= R <= 8 (K % 64 == 0), for every R with iq2 = 1 / 2, for
// Nvfp4Gemv at every R, and for Q4Gemv at R = 1 (reference dispatch: src/bolt_ops.cu:1259-1306,
// :1429-1468).  Weight contracts: the reference's tensor-core one (bf16-rounded weights,
// DequantRow :860-919) for 2 <= R <= 8 and the iq2 modes; the exact one ((q - zp) * s, fp32
// accumulation, :1315-1392) for Q4 at R = 1 and for NVFP4 (whose weights are exact either way).
//
// B200 design
//  * persistent CTAs own contiguous weight-row ranges; 16-row tiles (optionally split into K
//    segments) are streamed by one cp.async.bulk.tensor request per stage through a 128-byte
//    swizzled tensor map, so the 8 rows a warp reads hit 8 different bank groups; a second
//    request stages the scales;
//  * 16 warps split K and keep their activation fragments in registers for the whole CTA;
//  * R = 1 exact-weight GEMVs run in block-column mode: the activation row is placed in MMA
//    column (scale block & 7), so each column of the accumulator is one scale block's raw dot
//    product and the block scale is applied once in fp32 -- the weights enter the tensor core
//    undecoded (Q4 as bf16 128 + n, NVFP4 as fp16 e2m1);
//  * the last warp to finish a ring slot refills it; per-warp tile partials are summed once per
//    tmax tiles; with early weights, the CTA's whole byte range is prefetched into L2 before
//    griddepcontrol.wait, so a call streams HBM while its predecessor drains.
#include <cstring>

#include "mma_decode.cuh"

namespace bolt {

namespace {

constexpr int kTileRows = 16;
constexpr int kWarps = 16;

struct MmaParams {
  const bf16* x;
  const uint8_t* w;
  const uint8_t* sc;
  const float* gscale;
  bf16* y;
  int64_t N;
  int K;
  int R;
  int nstage;
  int kseg;                // K segments per tile: stage = (tile, segment), 16 / kseg warps per segment
  int tmax;                // tiles whose partials are buffered before one CTA-wide reduction
  int pieces;              // weight pieces per stage
  int spieces;             // 128-byte scale pieces per stage (0: scales as a plain span)
  int wsw;                 // weight pieces: 1 = 128 bytes, swizzled; 0 = 16 bytes
  uint32_t w_bytes;        // weight bytes of one stage (16 rows)
  uint32_t stage_bytes;    // ring slot bytes (weights + scales), multiple of 1024
  int early_weights;
};

__device__ __forceinline__ bool last_warp_of_slot(int* cnt, int lane, int nwarps) {
  __threadfence_block();
  __syncwarp();
  int last = 0;
  if (lane == 0) last = atomicAdd(cnt, 1) == nwarps - 1;
  last = __shfl_sync(0xffffffffu, last, 0);
  if (last) __threadfence_block();
  return last != 0;
}

// Issues stage `i` = (tile i / kseg, segment i % kseg) into ring slot i % NS: one tensor request
// for the weights (lane 0) and one for the scales (lane 1; a plain span when the scale rows are
// not 128-byte multiples).  Rows past the matrix end are zero-filled by the tensor unit.
__device__ __forceinline__ void mma_issue_stage(const CUtensorMap* tmw, const CUtensorMap* tms, const MmaParams& p,
                                                uint8_t* smem, uint64_t* full_bar, int i, int64_t r0, int nrows,
                                                int64_t sc_row_bytes, int lane) {
  const int s = i % p.nstage;
  const int tile = i / p.kseg, q = i % p.kseg;
  const int64_t row0 = r0 + static_cast<int64_t>(tile) * kTileRows;
  uint8_t* slot = smem + static_cast<size_t>(s) * p.stage_bytes;
  const uint32_t fb = smem_u32(&full_bar[s]);
  uint32_t tx = p.w_bytes;
  if (lane == 0) tma_load_3d(smem_u32(slot), tmw, 0, static_cast<int>(row0), q * p.pieces, fb);  // q > 0 only when wsw
  if (p.spieces) {
    tx += static_cast<uint32_t>(p.spieces) * kTileRows * 128;
    if (lane == 1) tma_load_3d(smem_u32(slot + p.w_bytes), tms, 0, static_cast<int>(row0), q * p.spieces, fb);
  } else if (lane == 0) {
    const int rows = min(kTileRows, nrows - tile * kTileRows);
    stage_span(slot + p.w_bytes, p.sc + row0 * sc_row_bytes, static_cast<uint32_t>(rows * sc_row_bytes),
               p.sc + p.N * sc_row_bytes, fb, tx);
  }
  __syncwarp();
  if (lane == 0) mbar_arrive_expect_tx(fb, tx);
}

template <int FMT>
__device__ __forceinline__ int bc_block(int c, int t) {
  return FMT == kFmtQ4 ? 2 * c + (t >> 1) : 4 * c + t;
}

// BC: block-column mode (R = 1, FMT = Q4 or NVFP4).  CPW: max 64-k chunks per warp.
template <int FMT, bool BC, int CPW>
__global__ void __launch_bounds__(kWarps * 32, 1)
    gemv_mma_kernel(const __grid_constant__ CUtensorMap tmw, const __grid_constant__ CUtensorMap tms,
                    const MmaParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  constexpr int OUTS = BC ? 16 : 128;  // partial outputs per warp and tile
  __shared__ uint64_t full_bar[8];
  __shared__ int done_cnt[8];
  __shared__ __align__(16) uint32_t grid_s[(FMT == kFmtIq2N) ? 1024 : 4];
  __shared__ volatile int abort_flag;
  // the 128-byte swizzle needs 1024-byte aligned stage buffers
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* red = reinterpret_cast<float*>(smem + static_cast<size_t>(p.nstage) * p.stage_bytes);  // [tmax][16][OUTS]

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  const int K = p.K;
  const int KS = p.kseg;
  const int64_t row_bytes = fmt_row_bytes(FMT, K);
  const int64_t sc_row_bytes = fmt_scale_row_bytes(FMT, K);
  const int64_t r0 = static_cast<int64_t>(blockIdx.x) * p.N / gridDim.x;
  const int64_t r1 = static_cast<int64_t>(blockIdx.x + 1) * p.N / gridDim.x;
  const int nrows = static_cast<int>(r1 - r0);
  const int ntiles = (nrows + kTileRows - 1) / kTileRows;
  const int nstages = ntiles * KS;
  const int NS = p.nstage;
  const bool sc_swz = p.spieces != 0;
  const int sc_rb = sc_swz ? 0 : static_cast<int>(sc_row_bytes);
  const int wsw = p.wsw;

  // prologue: descriptors first, then the weight stream and the activations side by side
  if (tid == 0) {
    prefetch_tensor_map(&tmw);
    if (p.spieces) prefetch_tensor_map(&tms);
    for (int s = 0; s < NS; ++s) {
      mbar_init(smem_u32(&full_bar[s]), 1);
      done_cnt[s] = 0;
    }
    abort_flag = 0;
    fence_barrier_init();
  }
  pdl_trigger();
  if (warp == 0) {
    __syncwarp();
    if (p.early_weights) {
      if (lane == 0) {
        prefetch_span_l2(p.w + r0 * row_bytes, static_cast<uint64_t>(nrows) * row_bytes);
        prefetch_span_l2(p.sc + r0 * sc_row_bytes, static_cast<uint64_t>(nrows) * sc_row_bytes);
      }
    } else {
      pdl_wait();
    }
    for (int i = 0; i < min(NS, nstages); ++i) mma_issue_stage(&tmw, &tms, p, smem, full_bar, i, r0, nrows, sc_row_bytes, lane);
  }
  pdl_wait();

  // warp -> K segment q and its chunk range [cb, ce) (absolute chunk indices)
  const int wps = kWarps / KS;
  const int q = warp / wps, wq = warp % wps;
  const int nch = (K >> 6) / KS;
  const int cb = q * nch + static_cast<int>(static_cast<int64_t>(wq) * nch / wps);
  const int ce = q * nch + static_cast<int>(static_cast<int64_t>(wq + 1) * nch / wps);
  const int cseg0 = q * nch;  // first chunk of the warp's segment (stage-relative offsets)

  // activation fragments: raw bf16 pairs land in bfr first (loads in flight across the barrier),
  // then are rearranged in place
  uint32_t bfr[CPW][8];
#pragma unroll
  for (int j = 0; j < CPW; ++j) {
    const int c = cb + j;
    const int xr = BC ? 0 : g;
    uint4 a = make_uint4(0u, 0u, 0u, 0u), b = a;
    if (c < ce && (BC || g < p.R)) {
      const uint4* xp = reinterpret_cast<const uint4*>(p.x + static_cast<int64_t>(xr) * K + 64 * c + 16 * t);
      a = __ldg(xp);
      b = __ldg(xp + 1);
    }
    bfr[j][0] = a.x; bfr[j][1] = a.y; bfr[j][2] = a.z; bfr[j][3] = a.w;
    bfr[j][4] = b.x; bfr[j][5] = b.y; bfr[j][6] = b.z; bfr[j][7] = b.w;
  }
  if constexpr (FMT == kFmtIq2N) {
    for (int i = tid; i < 1024; i += blockDim.x) grid_s[i] = kIq2xxsGridBf16x2[i];
  }
  __syncthreads();  // barrier initialisation and the codebook are visible to every warp
#pragma unroll
  for (int j = 0; j < CPW; ++j) {
    uint32_t x16[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) x16[i] = bfr[j][i];
    make_b_frags<FMT>(x16, bfr[j]);
    if constexpr (BC) {
      if (g != (bc_block<FMT>(cb + j, t) & 7)) {
#pragma unroll
        for (int i = 0; i < 8; ++i) bfr[j][i] = 0u;
      }
    }
  }
  // block-column groups: GC chunks = 8 scale blocks; per group the blocks held in columns 2t,
  // 2t+1 and (Q4) the x sums that remove the +128 magic offset
  constexpr int GC = FMT == kFmtQ4 ? 4 : 2;
  constexpr int BPC = FMT == kFmtQ4 ? 2 : 4;  // scale blocks per chunk
  constexpr int NG = BC ? (CPW + GC - 1) / GC : 1;
  int gblk[NG][2];
  float gxs[NG][2];
#pragma unroll
  for (int j = 0; j < NG; ++j) {
    const int b0 = (cb + j * GC) * BPC;
    const int bend = min(ce, cb + (j + 1) * GC) * BPC;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int n = 2 * t + h;
      const int b = b0 + ((n - b0) & 7);
      gblk[j][h] = (BC && b < bend) ? b : -1;
      float xs = 0.f;
      if (BC && FMT == kFmtQ4 && b < bend) {
        const uint4* xp = reinterpret_cast<const uint4*>(p.x + 32 * b);
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          const uint4 u = __ldg(xp + v);
          const uint32_t w4[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) xs += __uint_as_float(w4[e] << 16) + __uint_as_float(w4[e] & 0xFFFF0000u);
        }
      }
      gxs[j][h] = -136.f * xs;
    }
  }
  const float gs = (FMT == kFmtFp4) ? p.gscale[0] * 64.f : 1.f;
  const int tmax = p.tmax;
  // per-lane smem offsets (row g; row g + 8 adds wrow8 / srow8) of every chunk of the warp
  const uint32_t wrow8 = wsw ? 1024u : 128u;
  const uint32_t srow8 = sc_swz ? 1024u : 8u * static_cast<uint32_t>(sc_rb);
  uint32_t woff[CPW], soff[BC ? 1 : CPW];
#pragma unroll
  for (int j = 0; j < CPW; ++j) {
    const int cl = cb + j - cseg0;
    woff[j] = tile_off(wsw, g, chunk_byte<FMT>(cl, t));
    if constexpr (!BC) {
      const int sb = chunk_scale_byte<FMT>(cl, t);
      soff[j] = sc_swz ? swz_off(g, sb) : static_cast<uint32_t>(g * sc_rb + sb);
    }
  }
  uint32_t goff[NG][2];  // BC: scale offsets of the two columns' blocks (row g)
#pragma unroll
  for (int j = 0; j < NG; ++j)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int bl = gblk[j][h] >= 0 ? gblk[j][h] - cseg0 * BPC : 0;
      const int sb = FMT == kFmtQ4 ? 2 * bl : bl;
      goff[j][h] = sc_swz ? swz_off(g, sb) : static_cast<uint32_t>(g * sc_rb + sb);
    }

  for (int i = 0; i < ntiles; ++i) {
    const int st = i * KS + q;  // this warp's stage of tile i
    const int s = st % NS;
    const uint32_t ph = (st / NS) & 1;
    if (!abort_flag && !mbar_wait(smem_u32(&full_bar[s]), ph, kStatusFullWait)) abort_flag = 1;
    const uint8_t* wt = smem + static_cast<size_t>(s) * p.stage_bytes;
    const uint8_t* stl = wt + p.w_bytes;
    if (!sc_swz) stl += reinterpret_cast<uintptr_t>(p.sc + (r0 + static_cast<int64_t>(i) * kTileRows) * sc_row_bytes) & 15;
    float* rt = red + (static_cast<size_t>(i % tmax) * kWarps + warp) * OUTS;

    if constexpr (BC) {
      float tot0 = 0.f, tot1 = 0.f;  // rows g, g + 8 (this lane's two columns)
#pragma unroll
      for (int jg = 0; jg < NG; ++jg) {
        float d[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
        for (int jj = 0; jj < GC; ++jj) {
          const int j = jg * GC + jj;
          if (j < CPW && cb + j < ce) {
            RawRow ra, rb;
            ra.w = load_w_at<FMT>(wt + woff[j]);
            rb.w = load_w_at<FMT>(wt + woff[j] + wrow8);
            uint32_t da[8], db[8];
            decode_row_raw<FMT>(ra, da);
            decode_row_raw<FMT>(rb, db);
#pragma unroll
            for (int s2 = 0; s2 < 4; ++s2)
              mma16816<FmtTraits<FMT>::kF16>(d[jj & 1], da[2 * s2], db[2 * s2], da[2 * s2 + 1], db[2 * s2 + 1],
                                            bfr[j][2 * s2], bfr[j][2 * s2 + 1]);
          }
        }
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          if (gblk[jg][h] >= 0) {
            float s_g, s_g8;
            if constexpr (FMT == kFmtQ4) {
              s_g = bf16_bits_to_f32(load_s_at<FMT>(stl + goff[jg][h]));
              s_g8 = bf16_bits_to_f32(load_s_at<FMT>(stl + goff[jg][h] + srow8));
            } else {
              uint32_t sh;
              const uint32_t two = load_s_at<FMT>(stl + goff[jg][h]) | (load_s_at<FMT>(stl + goff[jg][h] + srow8) << 8);
              asm("{\n .reg .b16 t16;\n cvt.u16.u32 t16, %1;\n cvt.rn.f16x2.e4m3x2 %0, t16;\n}\n" : "=r"(sh) : "r"(two));
              s_g = __low2float(bits_h2(sh));
              s_g8 = __high2float(bits_h2(sh));
            }
            tot0 = fmaf(d[0][h] + d[1][h] + gxs[jg][h], s_g, tot0);
            tot1 = fmaf(d[0][2 + h] + d[1][2 + h] + gxs[jg][h], s_g8, tot1);
          }
        }
      }
      tot0 += __shfl_xor_sync(0xffffffffu, tot0, 1);
      tot0 += __shfl_xor_sync(0xffffffffu, tot0, 2);
      tot1 += __shfl_xor_sync(0xffffffffu, tot1, 1);
      tot1 += __shfl_xor_sync(0xffffffffu, tot1, 2);
      if (t == 0) {
        rt[g] = tot0;
        rt[g + 8] = tot1;
      }
    } else {
      float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
      for (int j = 0; j < CPW; ++j) {
        if (cb + j < ce) {
          RawRow ra, rb;
          ra.w = load_w_at<FMT>(wt + woff[j]);
          rb.w = load_w_at<FMT>(wt + woff[j] + wrow8);
          ra.s = load_s_at<FMT>(stl + soff[j]);
          rb.s = load_s_at<FMT>(stl + soff[j] + srow8);
          uint32_t da[8], db[8];
          decode_row<FMT>(ra, t, grid_s, da);
          decode_row<FMT>(rb, t, grid_s, db);
#pragma unroll
          for (int s2 = 0; s2 < 4; ++s2)
            mma16816<FmtTraits<FMT>::kF16>(acc[j & 1], da[2 * s2], db[2 * s2], da[2 * s2 + 1], db[2 * s2 + 1],
                                          bfr[j][2 * s2], bfr[j][2 * s2 + 1]);
        }
      }
      *reinterpret_cast<float2*>(&rt[g * 8 + 2 * t]) = make_float2(acc[0][0] + acc[1][0], acc[0][1] + acc[1][1]);
      *reinterpret_cast<float2*>(&rt[(g + 8) * 8 + 2 * t]) = make_float2(acc[0][2] + acc[1][2], acc[0][3] + acc[1][3]);
    }
    if (last_warp_of_slot(&done_cnt[s], lane, wps)) {
      if (lane == 0) done_cnt[s] = 0;
      if (st + NS < nstages && !abort_flag)
        mma_issue_stage(&tmw, &tms, p, smem, full_bar, st + NS, r0, nrows, sc_row_bytes, lane);
    }
    if ((i % tmax) == tmax - 1 || i == ntiles - 1) {
      __syncthreads();
      const int i0 = i - (i % tmax);
      const int nout = BC ? kTileRows : kTileRows * p.R;
      for (int o = tid; o < (i - i0 + 1) * nout; o += blockDim.x) {
        const int ti = i0 + o / nout, oo = o % nout;
        const int col = BC ? 0 : oo >> 4, rl = oo & 15;
        if (rl < min(kTileRows, nrows - ti * kTileRows)) {
          const float* rb = red + static_cast<size_t>(ti % tmax) * kWarps * OUTS;
          float v = 0.f;
#pragma unroll
          for (int w = 0; w < kWarps; ++w) v += rb[w * OUTS + (BC ? rl : rl * 8 + col)];
          p.y[static_cast<int64_t>(col) * p.N + r0 + static_cast<int64_t>(ti) * kTileRows + rl] = __float2bfloat16(v * gs);
        }
      }
      __syncthreads();
    }
  }
  if (tid == 0 && abort_flag)  // copies may still be landing: wait for them before exiting
    for (int i = max(0, nstages - NS); i < nstages; ++i)
      mbar_wait(smem_u32(&full_bar[i % NS]), (i / NS) & 1, kStatusDrainWait);
}

template <int FMT, bool BC, int CPW>
cudaError_t launch_mma(const CUtensorMap& tmw, const CUtensorMap& tms, const MmaParams& p, int grid,
                       const LaunchCfg& cfg) {
  auto kern = gemv_mma_kernel<FMT, BC, CPW>;
  const size_t smem = 1024 + static_cast<size_t>(p.nstage) * p.stage_bytes +
                      static_cast<size_t>(p.tmax) * kWarps * (BC ? 16 : 128) * sizeof(float);
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  return launch_kernel(kern, dim3(grid), dim3(kWarps * 32), smem, cfg, tmw, tms, p);
}

template <int FMT, bool BC>
cudaError_t dispatch_mma(const CUtensorMap& tmw, const CUtensorMap& tms, const MmaParams& p, int grid,
                         const LaunchCfg& cfg) {
  const int cpw = ((p.K >> 6) + kWarps - 1) / kWarps;
  if (cpw <= 1) return launch_mma<FMT, BC, 1>(tmw, tms, p, grid, cfg);
  if (cpw <= 2) return launch_mma<FMT, BC, 2>(tmw, tms, p, grid, cfg);
  if (cpw <= 4) return launch_mma<FMT, BC, 4>(tmw, tms, p, grid, cfg);
  if (cpw <= 6) return launch_mma<FMT, BC, 6>(tmw, tms, p, grid, cfg);
  return launch_mma<FMT, BC, 8>(tmw, tms, p, grid, cfg);  // K <= 8192
}

// ------------------------------------------------------------------------------------------
// debug: decode weights with the kernel's own decoders (contract checks)
// ------------------------------------------------------------------------------------------
template <int FMT>
__global__ void dequant_mma_kernel(const uint8_t* __restrict__ w, const uint8_t* __restrict__ sc, int64_t N, int K,
                                   float* __restrict__ out) {
  __shared__ __align__(16) uint32_t grid_s[1024];
  for (int i = threadIdx.x; i < 1024; i += blockDim.x) grid_s[i] = kIq2xxsGridBf16x2[i];
  __syncthreads();
  const int groups = K / 16;
  const int64_t gid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (gid >= N * groups) return;
  const int64_t n = gid / groups;
  const int grp = static_cast<int>(gid % groups);
  const int c = grp >> 2, t = grp & 3;
  const RawRow r = load_raw<FMT>(w + n * fmt_row_bytes(FMT, K), sc + n * fmt_scale_row_bytes(FMT, K), c, t);
  uint32_t d[8];
  decode_row<FMT>(r, t, grid_s, d);
  float v[16];
#pragma unroll
  for (int s = 0; s < 4; ++s) {
    float a0, a1, b0, b1;
    if constexpr (FmtTraits<FMT>::kF16) {
      a0 = __low2float(bits_h2(d[2 * s])); a1 = __high2float(bits_h2(d[2 * s]));
      b0 = __low2float(bits_h2(d[2 * s + 1])); b1 = __high2float(bits_h2(d[2 * s + 1]));
    } else {
      a0 = __low2float(bits_bf2(d[2 * s])); a1 = __high2float(bits_bf2(d[2 * s]));
      b0 = __low2float(bits_bf2(d[2 * s + 1])); b1 = __high2float(bits_bf2(d[2 * s + 1]));
    }
    if constexpr (FmtTraits<FMT>::kXLayout == kXPerm) {
      v[s] = a0; v[s + 4] = a1; v[8 + s] = b0; v[12 + s] = b1;
    } else {
      v[4 * s] = a0; v[4 * s + 1] = a1; v[4 * s + 2] = b0; v[4 * s + 3] = b1;
    }
  }
  float* o = out + n * K + 16 * grp;
#pragma unroll
  for (int i = 0; i < 16; ++i) o[i] = v[i];
}

template <int BITS>
__global__ void dequant_exact_kernel(const uint8_t* __restrict__ w, const bf16* __restrict__ sc, int64_t N, int K,
                                     float* __restrict__ out) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= N * K) return;
  const int64_t n = i / K;
  const int k = static_cast<int>(i % K);
  const float s = __bfloat162float(sc[n * (K / 32) + k / 32]);
  int q;
  if constexpr (BITS == 8) q = static_cast<int>(w[n * K + k]) - 128;
  else q = static_cast<int>((w[n * (K / 2) + k / 2] >> (4 * (k & 1))) & 15) - 8;
  out[i] = static_cast<float>(q) * s;
}


}  // namespace

cudaError_t launch_gemv_mma(int fmt, const bf16* x, int R, const uint8_t* w, const void* sc, const float* gscale,
                            int64_t N, int K, bf16* y, const LaunchCfg& cfg) {
  MmaParams p{x, w, static_cast<const uint8_t*>(sc), gscale, y, N, K, R, 0, 1, 4, 0, 0, 0, 0, 0, cfg.early_weights ? 1 : 0};
  const bool bc = R == 1 && (fmt == kFmtQ4 || fmt == kFmtFp4);
  const int64_t rb = fmt_row_bytes(fmt, K);
  const int64_t srb = fmt_scale_row_bytes(fmt, K);
  p.wsw = rb % 128 == 0 ? 1 : 0;
  const int pb = p.wsw ? 128 : 16;
  const int pieces = static_cast<int>(rb / pb);
  if (!p.wsw && pieces > 256) return cudaErrorInvalidValue;
  const int nch = K >> 6;
  // K segments: the smallest split whose stage stays near 40 KB; a segment holds whole 128-byte
  // pieces of weights and scales and a whole number of chunks per warp group
  int ks = 1;
  for (int cand : {2, 4}) {
    if (!p.wsw || kTileRows * (rb / ks + srb / ks) <= 40 * 1024) break;
    if (pieces % cand || srb % (128 * cand) || nch % cand || (nch / cand) % (kWarps / cand)) break;
    ks = cand;
  }
  p.kseg = ks;
  p.pieces = pieces / ks;
  p.spieces = (srb % (128 * ks) == 0 && (reinterpret_cast<uintptr_t>(sc) & 15) == 0) ? static_cast<int>(srb / 128 / ks) : 0;
  if (ks > 1 && !p.spieces) return cudaErrorInvalidValue;
  CUtensorMap tmw, tms;
  if (!row_tile_map(&tmw, w, N, rb, p.pieces, pb)) return cudaErrorInvalidValue;
  if (p.spieces && !row_tile_map(&tms, sc, N, srb, p.spieces, 128)) p.spieces = 0;
  if (!p.spieces) std::memset(&tms, 0, sizeof(tms));
  p.w_bytes = static_cast<uint32_t>(p.pieces) * kTileRows * pb;
  const uint32_t sc_bytes = p.spieces ? static_cast<uint32_t>(p.spieces) * kTileRows * 128
                                      : static_cast<uint32_t>(kTileRows * srb + 32);
  p.stage_bytes = (p.w_bytes + sc_bytes + 1023) & ~1023u;
  p.tmax = bc ? 8 : 4;
  const int grid = static_cast<int>(std::min<int64_t>(cfg.sms, (N + 7) / 8));
  const int64_t rows_per_cta = (N + grid - 1) / grid;
  const int want = static_cast<int>((rows_per_cta + kTileRows - 1) / kTileRows) * ks;
  const size_t red_bytes = static_cast<size_t>(p.tmax) * kWarps * (bc ? 16 : 128) * sizeof(float) + 1024;
  const size_t budget = cfg.smem_budget > red_bytes ? cfg.smem_budget - red_bytes : 0;
  const int fit = static_cast<int>(budget / p.stage_bytes);
  p.nstage = std::max(std::min(2, want), std::min({want, fit, 8}));
  if (bc) return fmt == kFmtQ4 ? dispatch_mma<kFmtQ4, true>(tmw, tms, p, grid, cfg)
                               : dispatch_mma<kFmtFp4, true>(tmw, tms, p, grid, cfg);
  switch (fmt) {
    case kFmtQ8: return dispatch_mma<kFmtQ8, false>(tmw, tms, p, grid, cfg);
    case kFmtQ4: return dispatch_mma<kFmtQ4, false>(tmw, tms, p, grid, cfg);
    case kFmtFp4: return dispatch_mma<kFmtFp4, false>(tmw, tms, p, grid, cfg);
    case kFmtIq2Lut: return dispatch_mma<kFmtIq2Lut, false>(tmw, tms, p, grid, cfg);
    default: return dispatch_mma<kFmtIq2N, false>(tmw, tms, p, grid, cfg);
  }
}

cudaError_t launch_dequant(int fmt, int exact, const uint8_t* w, const void* sc, int64_t N, int K, float* out,
                           const LaunchCfg& cfg) {
  const uint8_t* s8 = static_cast<const uint8_t*>(sc);
  if (exact) {
    const int64_t n = N * K;
    const unsigned blocks = static_cast<unsigned>((n + 255) / 256);
    if (fmt == kFmtQ8)
      return launch_kernel(dequant_exact_kernel<8>, dim3(blocks), dim3(256), 0, cfg, w, static_cast<const bf16*>(sc), N, K, out);
    return launch_kernel(dequant_exact_kernel<4>, dim3(blocks), dim3(256), 0, cfg, w, static_cast<const bf16*>(sc), N, K, out);
  }
  const unsigned blocks = static_cast<unsigned>((N * (K / 16) + 127) / 128);
  switch (fmt) {
    case kFmtQ8: return launch_kernel(dequant_mma_kernel<kFmtQ8>, dim3(blocks), dim3(128), 0, cfg, w, s8, N, K, out);
    case kFmtQ4: return launch_kernel(dequant_mma_kernel<kFmtQ4>, dim3(blocks), dim3(128), 0, cfg, w, s8, N, K, out);
    case kFmtFp4: return launch_kernel(dequant_mma_kernel<kFmtFp4>, dim3(blocks), dim3(128), 0, cfg, w, s8, N, K, out);
    case kFmtIq2Lut: return launch_kernel(dequant_mma_kernel<kFmtIq2Lut>, dim3(blocks), dim3(128), 0, cfg, w, s8, N, K, out);
    default: return launch_kernel(dequant_mma_kernel<kFmtIq2N>, dim3(blocks), dim3(128), 0, cfg, w, s8, N, K, out);
  }
}

}  // namespace bolt
