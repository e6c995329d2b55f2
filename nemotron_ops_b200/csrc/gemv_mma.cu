// Tensor-core skinny GEMV: y[R, N] = x[R, K] @ W^T for R <= 8 (mma.sync m16n8k16, fp32 acc).
//
// Used for Q8Gemv / Q4Gemv at 2 <= R <= 8 (K % 64 == 0), for every R with iq2 = 1 / 2, for
// Nvfp4Gemv at every R, and for Q4Gemv at R = 1 when K % 256 == 0 (reference dispatch:
// src/bolt_ops.cu:1259-1306, :1429-1468).  Weight contracts: the reference's tensor-core one
// (bf16-rounded weights, DequantRow :860-919) for 2 <= R <= 8 and the iq2 modes; the exact one
// ((q - zp) * s, fp32 accumulation, :1315-1392) for Q4 at R = 1 and for NVFP4 (whose weights are
// exact either way).
//
// B200 design
//  * one CTA per SM = 8 MMA warps + 1 producer warp.  A tile is 16*MT weight rows; the producer
//    streams it as K segments ("stages", ~16 KB) through a ring of shared-memory slots, one
//    cp.async.bulk.tensor request per stage through a 128-byte swizzled tensor map (a tensor
//    request costs ~0.2 us to issue whatever its size, so requests are few and large), plus one
//    request for the whole tile's scales riding on its first stage; a slot is refilled once all
//    8 MMA warps released it (empty mbarrier);
//  * the activations arrive by one bulk copy per row and are converted in place into MMA
//    B-fragment order, so a lane fetches a chunk's B operand with two 16-byte loads;
//  * every per-lane shared-memory offset is fixed per warp (stages of a tile have the same
//    layout), MT m16 tiles share every B fragment, and MMA row g of a tile is weight row pi(g),
//    chosen so the lanes of one shared-memory phase hit distinct banks under the swizzle;
//  * R = 1 exact-weight GEMVs run in block-column mode: the activation row is placed in MMA
//    column (scale block & 7), so each accumulator column is one scale block's raw dot product
//    and the block scale is applied once in fp32 -- the weights enter the tensor core undecoded
//    (Q4 as bf16 128 + n, NVFP4 as fp16 e2m1);
//  * programmatic dependent launch: the weights are constants, so with early weights the first
//    ring stages and an L2 prefetch of the CTA's whole range are issued before
//    griddepcontrol.wait, and a call streams HBM while its predecessor finishes.  The kernel
//    stays within half an SM (<= 96 registers, ~100 KB shared memory) so the next call's CTA
//    fits beside it.
#include <cstring>

#include "mma_decode.cuh"

namespace bolt {

namespace {

constexpr int kCWarps = 8;                    // MMA (consumer) warps
constexpr int kThreads = (kCWarps + 1) * 32;  // + the producer warp
constexpr int kMaxSlots = 8;

struct GemvParams {
  const bf16* x;
  const uint8_t* w;
  const uint8_t* sc;
  const float* gscale;
  bf16* y;
  int64_t N;
  int K;
  int R;
  int kseg;            // K segments per tile: stage = (tile, segment)
  int nslot;           // ring slots
  int pieces;          // weight pieces per stage
  int wsw;             // weight pieces: 1 = 128 bytes, swizzled; 0 = 16 bytes
  int smode;           // tile scales: 1 = 16-byte pieces through a tensor map, 0 = plain span
  int spieces;         // 16-byte scale pieces per row (smode 1)
  int nsbuf;           // scale buffers (2: the next tile's scales load during this tile)
  uint32_t w_bytes;    // weight bytes of one stage = ring slot size (multiple of 1024)
  uint32_t sc_bytes;   // one scale buffer (multiple of 128)
  uint32_t sc_off;     // smem offsets from the 1024-aligned base: scale buffers,
  uint32_t xs_off;     // B fragments of x (row r at xs_off + r * xs_row),
  uint32_t xs_row;
  uint32_t aux_off;    // 32 zero bytes, then (Q4 block-column) the fp32 sums of x per 32-k block,
  uint32_t red_off;    // cross-warp partial sums
  int early_weights;
};

// MMA row g of a tile <-> weight row pi(g) (and pi(g) + 8): one shared-memory phase of 8-byte
// loads covers 4 consecutive g, of 16-byte loads 2, and those rows must fall on different
// 16-byte bank groups after the XOR swizzle.
template <int FMT>
__host__ __device__ __forceinline__ int row_perm(int g) {
  if constexpr (FMT == kFmtQ8) return ((g & 1) << 2) | (g >> 1);
  else return ((g & 3) << 1) | (g >> 2);
}

// Tile-local offset of scale byte b of tile row r (see GemvParams::smode; sc_rb = scale bytes
// of a row).  Linear in b along a row for b multiple of 16 apart, and in r.
template <int ROWS>
__device__ __forceinline__ uint32_t sc_off(int smode, int r, int b, int sc_rb) {
  return smode ? p16_off(r, b, ROWS) : static_cast<uint32_t>(r * sc_rb + b);
}

// Issues stage st = (tile st / kseg, segment st % kseg) into ring slot st % nslot; the first
// stage of a tile also brings the tile's scales.  Rows past the matrix end are zero-filled.
template <int ROWS>
__device__ __forceinline__ void issue_stage(const CUtensorMap* tmw, const CUtensorMap* tms, const GemvParams& p,
                                            uint8_t* smem, uint64_t* full_bar, int st, int64_t r0, int nrows,
                                            int64_t sc_row_bytes) {
  const int s = st % p.nslot;
  const int tile = st / p.kseg, q = st % p.kseg;
  const int64_t row0 = r0 + static_cast<int64_t>(tile) * ROWS;
  const uint32_t fb = smem_u32(&full_bar[s]);
  uint32_t tx = p.w_bytes;
  if (q == 0) {
    uint8_t* sdst = smem + p.sc_off + static_cast<size_t>(tile % p.nsbuf) * p.sc_bytes;
    if (p.smode) {
      tx += static_cast<uint32_t>(p.spieces) * ROWS * 16u;
      tma_load_3d(smem_u32(sdst), tms, 0, static_cast<int>(row0), 0, fb);
    } else {
      const int rows = min(ROWS, nrows - tile * ROWS);
      stage_span(sdst, p.sc + row0 * sc_row_bytes, static_cast<uint32_t>(rows * sc_row_bytes),
                 p.sc + p.N * sc_row_bytes, fb, tx);
    }
  }
  tma_load_3d(smem_u32(smem + static_cast<size_t>(s) * p.w_bytes), tmw, 0, static_cast<int>(row0), q * p.pieces, fb);
  mbar_arrive_expect_tx(fb, tx);
}

// BC: block-column mode (R = 1, FMT = Q4 or NVFP4).  MT: m16 tiles per row tile.  CPW: max
// chunks (64 k) per warp and stage.  FIX: the common layout (128-byte swizzled weight pieces,
// 16-byte scale pieces) fixed at compile time.
template <int FMT, bool BC, int MT, int CPW, bool FIX>
__global__ void __launch_bounds__(kThreads, 2)
    gemv_tc_kernel(const __grid_constant__ CUtensorMap tmw, const __grid_constant__ CUtensorMap tms,
                   const GemvParams p) {
  constexpr int ROWS = 16 * MT;
  constexpr int GC = BC ? (FMT == kFmtQ4 ? 4 : 2) : 1;  // chunks per group (BC: 8 scale blocks)
  constexpr int BPC = FMT == kFmtQ4 ? 2 : 4;             // BC: scale blocks per chunk
  constexpr int NG = CPW / GC;                            // max groups per warp and stage
  extern __shared__ __align__(16) uint8_t smem_raw[];  // only 16-byte alignment is guaranteed
  __shared__ uint64_t full_bar[kMaxSlots], empty_bar[kMaxSlots], x_bar;
  __shared__ __align__(16) uint32_t grid_s[(FMT == kFmtIq2N) ? 1024 : 4];
  __shared__ volatile int abort_flag;
  // the 128-byte swizzle needs 1024-byte aligned stage buffers (offset from the shared array
  // itself, so every derived pointer stays a shared-memory pointer)
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int K = p.K, KS = p.kseg, NS = p.nslot;
  const int64_t row_bytes = fmt_row_bytes(FMT, K);
  const int64_t sc_row_bytes = fmt_scale_row_bytes(FMT, K);
  const int64_t r0 = static_cast<int64_t>(blockIdx.x) * p.N / gridDim.x;
  const int64_t r1 = static_cast<int64_t>(blockIdx.x + 1) * p.N / gridDim.x;
  const int nrows = static_cast<int>(r1 - r0);
  const int ntiles = (nrows + ROWS - 1) / ROWS;
  const int nstages = ntiles * KS;
  uint8_t* xs = smem + p.xs_off;
  // the host sized the carve-out with 1024 bytes of slack for this alignment; check it anyway
  if ((smem_u32(smem) & 1023u) != 0u || smem - smem_raw > 1023) {
    if (tid == 0) set_status(kStatusSmemAlign);
    return;
  }

  if (tid == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(smem_u32(&full_bar[s]), 1);
      mbar_init(smem_u32(&empty_bar[s]), kCWarps);
    }
    mbar_init(smem_u32(&x_bar), 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  if constexpr (FMT == kFmtIq2N) {
    load_iq2_grid<false>(grid_s, tid, kThreads);
  }
  __syncthreads();

  // ------------------------------------------------------------------ producer warp
  if (warp == kCWarps) {
    int first = 0;
    if (lane == 0) {
      prefetch_tensor_map(&tmw);
      if (p.smode) prefetch_tensor_map(&tms);
      // up-front stages: as many as the ring holds, from the tiles whose scale buffers are free
      first = min(min(NS, nstages), p.nsbuf * KS);
      // weights are constants: with early weights the ring fills, and the rest of the range is
      // pulled into L2, while the previous kernel runs
      const bool rest = nstages > first;
      if (p.early_weights) {
        for (int st = 0; st < first; ++st) issue_stage<ROWS>(&tmw, &tms, p, smem, full_bar, st, r0, nrows, sc_row_bytes);
        if (rest) {
          prefetch_span_l2(p.w + r0 * row_bytes, static_cast<uint64_t>(nrows) * row_bytes);
          prefetch_span_l2(p.sc + r0 * sc_row_bytes, static_cast<uint64_t>(nrows) * sc_row_bytes);
        }
      }
      pdl_wait();
      // the activation rows, ahead of any weight copy issued from here on
      const uint32_t xb = smem_u32(&x_bar);
      mbar_arrive_expect_tx(xb, static_cast<uint32_t>(p.R) * static_cast<uint32_t>(K) * 2u);
      for (int r = 0; r < p.R; ++r)
        bulk_g2s(smem_u32(xs + static_cast<size_t>(r) * p.xs_row), p.x + static_cast<int64_t>(r) * K,
                 static_cast<uint32_t>(K) * 2u, xb);
      if (!p.early_weights) {
        for (int st = 0; st < first; ++st) issue_stage<ROWS>(&tmw, &tms, p, smem, full_bar, st, r0, nrows, sc_row_bytes);
        if (rest) {  // the rest of the range: pulled into L2 now, staged from there later
          prefetch_span_l2(p.w + r0 * row_bytes, static_cast<uint64_t>(nrows) * row_bytes);
          prefetch_span_l2(p.sc + r0 * sc_row_bytes, static_cast<uint64_t>(nrows) * sc_row_bytes);
        }
      }
    }
    // the next call's CTAs are released once the activations have landed (every warp of the CTA
    // triggers at that point), so their prologues do not compete with this call's first copies
    __syncwarp();
    mbar_wait(smem_u32(&x_bar), 0, kStatusFullWait);
    pdl_trigger();
    if (lane == 0) {
      const uint32_t xb = smem_u32(&x_bar);
      int issued = first;
      for (int st = first; st < nstages; ++st) {
        const int s = st % NS;
        bool okw = mbar_wait(smem_u32(&empty_bar[s]), ((st / NS) - 1) & 1, kStatusEmptyWait);
        const int tile = st / KS;
        if (okw && st % KS == 0 && tile >= p.nsbuf) {
          // the scale buffer of tile - nsbuf must be released too (its last stage consumed);
          // stages up to st - NS are known to be consumed already
          const int last = (tile - p.nsbuf + 1) * KS - 1;
          if (last > st - NS) okw = mbar_wait(smem_u32(&empty_bar[last % NS]), (last / NS) & 1, kStatusEmptyWait);
        }
        if (!okw) abort_flag = 1;
        if (abort_flag) break;
        issue_stage<ROWS>(&tmw, &tms, p, smem, full_bar, st, r0, nrows, sc_row_bytes);
        ++issued;
      }
      // no copy may still be landing when the CTA exits
      mbar_wait(xb, 0, kStatusDrainWait);
      for (int st = max(0, issued - NS); st < issued; ++st)
        mbar_wait(smem_u32(&full_bar[st % NS]), (st / NS) & 1, kStatusDrainWait);
    }
    return;
  }

  // ------------------------------------------------------------------ MMA warps
  const int g = lane >> 2, t = lane & 3;
  const int pg = row_perm<FMT>(g);
  const int nch = K >> 6;
  const int nchs = nch / KS;  // chunks per K segment
  int cb, ce;                 // this warp's chunks [cb, ce) of every segment
  {
    const int ng = nchs / GC;
    cb = GC * (warp * ng / kCWarps);
    ce = GC * ((warp + 1) * ng / kCWarps);
  }
  const uint8_t* zero = smem + p.aux_off;
  float* xsum = reinterpret_cast<float*>(smem + p.aux_off + 32);
  float* red = reinterpret_cast<float*>(smem + p.red_off);

  pdl_wait();  // (gscale and y belong to the dependency chain as well)
  const float gsv = (FMT == kFmtFp4) ? __ldcg(p.gscale) : 1.f;  // in flight during the x copy
  if (tid < 8) reinterpret_cast<uint32_t*>(smem + p.aux_off)[tid] = 0u;
  bool ok = mbar_wait(smem_u32(&x_bar), 0, kStatusFullWait);
  if (!ok) abort_flag = 1;
  if constexpr (x_needs_conversion<FMT>()) {
    // activations -> B fragments, in place, 16-byte pieces (8 k): each thread loads a batch of
    // pieces, then converts and stores them, so the shared-memory latencies overlap
    const int np = K >> 3;  // pieces per row
    constexpr int kB = 4;
    for (int r = 0; r < p.R; ++r) {
      uint8_t* xr = xs + static_cast<size_t>(r) * p.xs_row;
      for (int base = 0; base < np; base += kB * kCWarps * 32) {
        uint4 v[kB];
#pragma unroll
        for (int k = 0; k < kB; ++k) {
          const int pi = base + k * kCWarps * 32 + tid;
          v[k] = pi < np ? lds128(xr + pi * 16) : make_uint4(0u, 0u, 0u, 0u);
        }
#pragma unroll
        for (int k = 0; k < kB; ++k) {
          const int pi = base + k * kCWarps * 32 + tid;
          if (pi < np) *reinterpret_cast<uint4*>(xr + pi * 16) = x_piece_to_frag<FMT>(v[k]);
          if constexpr (BC && FMT == kFmtQ4) {
            // fp32 sum of the 32 k of a scale block: 4 consecutive pieces on 4 consecutive lanes
            const uint32_t w4[4] = {v[k].x, v[k].y, v[k].z, v[k].w};
            float sum = 0.f;
#pragma unroll
            for (int e = 0; e < 4; ++e) sum += __uint_as_float(w4[e] << 16) + __uint_as_float(w4[e] & 0xFFFF0000u);
            sum += __shfl_xor_sync(0xffffffffu, sum, 1);
            sum += __shfl_xor_sync(0xffffffffu, sum, 2);
            if (pi < np && (pi & 3) == 0) xsum[pi >> 2] = sum;
          }
        }
      }
    }
  }
  named_bar_sync(1, kCWarps * 32);
  pdl_trigger();  // the activations are converted (see the producer warp)

  // ---- per-warp constant offsets (every stage of a tile has the same layout)
  const int wsw = FIX ? 1 : p.wsw;
  const int smode = FIX ? 1 : p.smode;
  const int sc_rb = static_cast<int>(sc_row_bytes);
  const uint32_t wrow8 = wsw ? 1024u : 128u;  // +8 rows in a weight stage
  const uint32_t srow8 = smode ? 128u : 8u * static_cast<uint32_t>(sc_rb);  // +8 rows in a scale tile
  const uint32_t sc_seg = smode ? static_cast<uint32_t>(sc_row_bytes / KS / 16) * ROWS * 16
                                : static_cast<uint32_t>(sc_row_bytes / KS);  // tile-local shift per segment
  uint32_t woff[CPW];  // weights of row pg, chunk cb + j (stage-local)
  int xoff[CPW];       // B fragment of chunk cb + j relative to the segment's first chunk; -1: zero
  uint32_t soff[NG];   // scale bytes (row pg, tile-local for segment 0) of group / chunk jg
#pragma unroll
  for (int j = 0; j < CPW; ++j) {
    const int c = cb + j;
    woff[j] = tile_off(wsw, pg, chunk_byte<FMT>(c, t), ROWS);
    if constexpr (BC) {
      const int blk = BPC * c + (FMT == kFmtQ4 ? (t >> 1) : t);  // stage-invariant mod 8
      xoff[j] = (g == (blk & 7)) ? (4 * c + t) * 32 : -1;
    } else {
      xoff[j] = (g < p.R) ? static_cast<int>(g * p.xs_row) + (4 * c + t) * 32 : -1;
    }
  }
#pragma unroll
  for (int jg = 0; jg < NG; ++jg) {
    int sb;
    if constexpr (BC) sb = (FMT == kFmtQ4 ? 2 : 1) * (BPC * (cb + jg * GC) + 2 * t);
    else sb = chunk_scale_byte<FMT>(cb + jg, t);
    soff[jg] = sc_off<ROWS>(smode, pg, sb, sc_rb);
  }

  int s = 0;          // ring slot and phase of the next stage
  uint32_t ph = 0;
  for (int i = 0; i < ntiles; ++i) {
    const uint8_t* sct = smem + p.sc_off + ((p.nsbuf == 2 && (i & 1)) ? p.sc_bytes : 0u);
    if (!smode)  // plain span: the first byte landed at the source's offset within 16 bytes
      sct += reinterpret_cast<uintptr_t>(p.sc + (r0 + static_cast<int64_t>(i) * ROWS) * sc_row_bytes) & 15;
    float acc[MT][4];  // BC: [m][0] row pg, [m][1] row pg + 8 (this lane's two columns, scaled)
#pragma unroll
    for (int m = 0; m < MT; ++m) acc[m][0] = acc[m][1] = acc[m][2] = acc[m][3] = 0.f;
    for (int q = 0; q < KS; ++q) {
      if (ok && abort_flag) ok = false;
      if (ok && !mbar_wait(smem_u32(&full_bar[s]), ph, kStatusFullWait)) {
        ok = false;
        abort_flag = 1;
      }
      if (ok) {
        const uint8_t* wt = smem + static_cast<size_t>(s) * p.w_bytes;
        const uint8_t* sq = sct + q * sc_seg;
        const uint8_t* xq = xs + static_cast<size_t>(q * nchs) * 128;
        if constexpr (BC) {
#pragma unroll
          for (int jg = 0; jg < NG; ++jg) {
            if (cb + jg * GC < ce) {
              // the group's raw weights and activations first, then decode + MMA
              uint2 wr[GC][MT][2];
              uint4 xv[GC][2];
#pragma unroll
              for (int jj = 0; jj < GC; ++jj) {
                const int j = jg * GC + jj;
                const uint8_t* xp = xoff[j] >= 0 ? xq + xoff[j] : zero;
                xv[jj][0] = lds128(xp);
                xv[jj][1] = lds128(xp + 16);
#pragma unroll
                for (int m = 0; m < MT; ++m) {
                  wr[jj][m][0] = *reinterpret_cast<const uint2*>(wt + woff[j] + m * 2 * wrow8);
                  wr[jj][m][1] = *reinterpret_cast<const uint2*>(wt + woff[j] + m * 2 * wrow8 + wrow8);
                }
              }
              float d[GC][MT][4];  // one accumulator chain per (chunk, tile): the MMA latency overlaps
#pragma unroll
              for (int jj = 0; jj < GC; ++jj)
#pragma unroll
                for (int m = 0; m < MT; ++m) d[jj][m][0] = d[jj][m][1] = d[jj][m][2] = d[jj][m][3] = 0.f;
#pragma unroll
              for (int jj = 0; jj < GC; ++jj) {
                uint32_t bf[8];
                frag_from_pieces<FMT>(xv[jj][0], xv[jj][1], bf);
#pragma unroll
                for (int m = 0; m < MT; ++m) {
                  RawRow ra, rb;
                  ra.w = make_uint4(wr[jj][m][0].x, wr[jj][m][0].y, 0u, 0u);
                  rb.w = make_uint4(wr[jj][m][1].x, wr[jj][m][1].y, 0u, 0u);
                  uint32_t da[8], db[8];
                  decode_row_raw<FMT>(ra, da);
                  decode_row_raw<FMT>(rb, db);
#pragma unroll
                  for (int s2 = 0; s2 < 4; ++s2)
                    mma16816<FmtTraits<FMT>::kF16>(d[jj][m], da[2 * s2], db[2 * s2], da[2 * s2 + 1], db[2 * s2 + 1],
                                                  bf[2 * s2], bf[2 * s2 + 1]);
                }
              }
              // group epilogue: this lane's columns 2t, 2t+1 hold blocks bl0 + 2t, bl0 + 2t + 1
#pragma unroll
              for (int m = 0; m < MT; ++m) {
                float e0 = d[0][m][0], e1 = d[0][m][1], e2 = d[0][m][2], e3 = d[0][m][3];
#pragma unroll
                for (int jj = 1; jj < GC; ++jj) {
                  e0 += d[jj][m][0];
                  e1 += d[jj][m][1];
                  e2 += d[jj][m][2];
                  e3 += d[jj][m][3];
                }
                if constexpr (FMT == kFmtQ4) {  // remove the +128 magic: -136 * (block sum of x)
                  const float2 xsm = *reinterpret_cast<const float2*>(xsum + BPC * (q * nchs + cb + jg * GC) + 2 * t);
                  e0 = fmaf(-136.f, xsm.x, e0);
                  e1 = fmaf(-136.f, xsm.y, e1);
                  e2 = fmaf(-136.f, xsm.x, e2);
                  e3 = fmaf(-136.f, xsm.y, e3);
                }
                const uint8_t* sp = sq + soff[jg] + m * 2 * srow8;
                float sa0, sa1, sb0, sb1;  // rows pg, pg + 8; blocks h = 0, 1
                if constexpr (FMT == kFmtQ4) {
                  const uint32_t ua = *reinterpret_cast<const uint32_t*>(sp);
                  const uint32_t ub = *reinterpret_cast<const uint32_t*>(sp + srow8);
                  sa0 = __uint_as_float(ua << 16);
                  sa1 = __uint_as_float(ua & 0xFFFF0000u);
                  sb0 = __uint_as_float(ub << 16);
                  sb1 = __uint_as_float(ub & 0xFFFF0000u);
                } else {
                  const uint32_t ua = *reinterpret_cast<const uint16_t*>(sp);
                  const uint32_t ub = *reinterpret_cast<const uint16_t*>(sp + srow8);
                  uint32_t ha, hb;
                  asm("{\n .reg .b16 t16;\n cvt.u16.u32 t16, %1;\n cvt.rn.f16x2.e4m3x2 %0, t16;\n}\n" : "=r"(ha) : "r"(ua));
                  asm("{\n .reg .b16 t16;\n cvt.u16.u32 t16, %1;\n cvt.rn.f16x2.e4m3x2 %0, t16;\n}\n" : "=r"(hb) : "r"(ub));
                  sa0 = __low2float(bits_h2(ha));
                  sa1 = __high2float(bits_h2(ha));
                  sb0 = __low2float(bits_h2(hb));
                  sb1 = __high2float(bits_h2(hb));
                }
                acc[m][0] = fmaf(e0, sa0, acc[m][0]);
                acc[m][0] = fmaf(e1, sa1, acc[m][0]);
                acc[m][1] = fmaf(e2, sb0, acc[m][1]);
                acc[m][1] = fmaf(e3, sb1, acc[m][1]);
              }
            }
          }
        } else {
          float acc2[MT][4];  // odd chunks: a second accumulator chain per tile
#pragma unroll
          for (int m = 0; m < MT; ++m) acc2[m][0] = acc2[m][1] = acc2[m][2] = acc2[m][3] = 0.f;
#pragma unroll
          for (int j = 0; j < CPW; ++j) {
            if (cb + j < ce) {
              const uint8_t* xp = xoff[j] >= 0 ? xq + xoff[j] : zero;
              uint32_t bf[8];
              frag_from_pieces<FMT>(lds128(xp), lds128(xp + 16), bf);
#pragma unroll
              for (int m = 0; m < MT; ++m) {
                RawRow ra, rb;
                ra.w = load_w_at<FMT>(wt + woff[j] + m * 2 * wrow8);
                rb.w = load_w_at<FMT>(wt + woff[j] + m * 2 * wrow8 + wrow8);
                ra.s = load_s_at<FMT>(sq + soff[j] + m * 2 * srow8);
                rb.s = load_s_at<FMT>(sq + soff[j] + m * 2 * srow8 + srow8);
                uint32_t da[8], db[8];
                decode_row<FMT>(ra, t, grid_s, da);
                decode_row<FMT>(rb, t, grid_s, db);
#pragma unroll
                for (int s2 = 0; s2 < 4; ++s2)
                  mma16816<FmtTraits<FMT>::kF16>((j & 1) ? acc2[m] : acc[m], da[2 * s2], db[2 * s2], da[2 * s2 + 1],
                                                db[2 * s2 + 1], bf[2 * s2], bf[2 * s2 + 1]);
              }
            }
          }
#pragma unroll
          for (int m = 0; m < MT; ++m)
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[m][e] += acc2[m][e];
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&empty_bar[s]));
      if (++s == NS) s = 0, ph ^= 1u;
    }

    // ---- tile epilogue: sum the 8 warps' partials, write y
    if constexpr (BC) {
#pragma unroll
      for (int m = 0; m < MT; ++m) {
        float a = acc[m][0], b = acc[m][1];
        a += __shfl_xor_sync(0xffffffffu, a, 1);
        a += __shfl_xor_sync(0xffffffffu, a, 2);
        b += __shfl_xor_sync(0xffffffffu, b, 1);
        b += __shfl_xor_sync(0xffffffffu, b, 2);
        if (t == 0) {
          red[warp * ROWS + 16 * m + pg] = a;
          red[warp * ROWS + 16 * m + 8 + pg] = b;
        }
      }
    } else {
#pragma unroll
      for (int m = 0; m < MT; ++m) {
        *reinterpret_cast<float2*>(&red[(warp * ROWS + 16 * m + pg) * 8 + 2 * t]) = make_float2(acc[m][0], acc[m][1]);
        *reinterpret_cast<float2*>(&red[(warp * ROWS + 16 * m + 8 + pg) * 8 + 2 * t]) = make_float2(acc[m][2], acc[m][3]);
      }
    }
    named_bar_sync(1, kCWarps * 32);
    const int nout = BC ? ROWS : ROWS * p.R;
    const int vrows = min(ROWS, nrows - i * ROWS);
    for (int o = tid; o < nout; o += kCWarps * 32) {
      const int col = BC ? 0 : o / ROWS, rl = o % ROWS;
      if (rl < vrows && !abort_flag) {
        float v = 0.f;
#pragma unroll
        for (int w = 0; w < kCWarps; ++w) v += BC ? red[w * ROWS + rl] : red[(w * ROWS + rl) * 8 + col];
        p.y[static_cast<int64_t>(col) * p.N + r0 + static_cast<int64_t>(i) * ROWS + rl] =
            __float2bfloat16(FMT == kFmtFp4 ? v * (gsv * 64.f) : v);
      }
    }
    named_bar_sync(1, kCWarps * 32);
  }
}

template <int FMT, bool BC, int MT, int CPW, bool FIX>
cudaError_t launch_tc(const CUtensorMap& tmw, const CUtensorMap& tms, const GemvParams& p, int grid, size_t smem,
                      const LaunchCfg& cfg) {
  auto kern = gemv_tc_kernel<FMT, BC, MT, CPW, FIX>;
  static SmemOptIn opt;
  cudaError_t e = allow_smem(kern, smem, opt);
  if (e != cudaSuccess) return e;
  return launch_kernel(kern, dim3(grid), dim3(kThreads), smem, cfg, tmw, tms, p);
}

template <int FMT, bool BC, int MT, bool FIX>
cudaError_t dispatch_cpw(int cpw, const CUtensorMap& tmw, const CUtensorMap& tms, const GemvParams& p, int grid,
                         size_t smem, const LaunchCfg& cfg) {
  // block-column mode: whole groups of 8 scale blocks per warp (2 NVFP4 / 4 Q4 chunks)
  if constexpr (!BC) {
    if (cpw <= 1) return launch_tc<FMT, BC, MT, 1, FIX>(tmw, tms, p, grid, smem, cfg);
  }
  if constexpr (!BC || FMT == kFmtFp4) {
    if (cpw <= 2) return launch_tc<FMT, BC, MT, 2, FIX>(tmw, tms, p, grid, smem, cfg);
  }
  if (cpw <= 4) return launch_tc<FMT, BC, MT, 4, FIX>(tmw, tms, p, grid, smem, cfg);
  return launch_tc<FMT, BC, MT, 8, FIX>(tmw, tms, p, grid, smem, cfg);
}

template <int FMT, bool BC>
cudaError_t dispatch_mt(int mt, int cpw, const CUtensorMap& tmw, const CUtensorMap& tms, const GemvParams& p,
                        int grid, size_t smem, const LaunchCfg& cfg) {
  const bool fix = p.wsw == 1 && p.smode == 1;
  if constexpr (BC) {  // block-column shapes always have the common layout (checked by the caller)
    if (mt == 1) return dispatch_cpw<FMT, BC, 1, true>(cpw, tmw, tms, p, grid, smem, cfg);
    return dispatch_cpw<FMT, BC, 2, true>(cpw, tmw, tms, p, grid, smem, cfg);
  } else {
    if (mt == 1) return fix ? dispatch_cpw<FMT, BC, 1, true>(cpw, tmw, tms, p, grid, smem, cfg)
                            : dispatch_cpw<FMT, BC, 1, false>(cpw, tmw, tms, p, grid, smem, cfg);
    return fix ? dispatch_cpw<FMT, BC, 2, true>(cpw, tmw, tms, p, grid, smem, cfg)
               : dispatch_cpw<FMT, BC, 2, false>(cpw, tmw, tms, p, grid, smem, cfg);
  }
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

// Shape checks (K % 64 == 0, R * K <= 65536, NVFP4 K % 1024, iq2 K % 128 / 256, 16-byte aligned
// tensors) are the caller's; the Q4 block-column mode additionally needs K % 256 == 0.
cudaError_t launch_gemv_mma(int fmt, const bf16* x, int R, const uint8_t* w, const void* sc, const float* gscale,
                            int64_t N, int K, bf16* y, const LaunchCfg& cfg) {
  const bool bc = R == 1 && (fmt == kFmtQ4 || fmt == kFmtFp4);
  if (bc && fmt == kFmtQ4 && K % 256) return cudaErrorInvalidValue;
  if (R == 1 && fmt == kFmtIq2N) {  // the register-streaming IQ2_XXS kernel (gemv_r1.cu)
    const cudaError_t e = launch_gemv_r1(fmt, x, w, sc, gscale, N, K, y, cfg);
    if (e != cudaErrorNotSupported) return e;
  }
  if (bc) {  // the register-streaming block-column kernel when it takes the shape (gemv_r1.cu)
    const cudaError_t e = launch_gemv_r1(fmt, x, w, sc, gscale, N, K, y, cfg);
    if (e != cudaErrorNotSupported) return e;
  }
  GemvParams p{};
  p.x = x;
  p.w = w;
  p.sc = static_cast<const uint8_t*>(sc);
  p.gscale = gscale;
  p.y = y;
  p.N = N;
  p.K = K;
  p.R = R;
  p.early_weights = cfg.early_weights ? 1 : 0;
  const int64_t rb = fmt_row_bytes(fmt, K);
  const int64_t srb = fmt_scale_row_bytes(fmt, K);
  p.wsw = rb % 128 == 0 ? 1 : 0;
  const int pb = p.wsw ? 128 : 16;
  const int pieces = static_cast<int>(rb / pb);
  const int nch = K >> 6;
  const int gc = bc ? (fmt == kFmtQ4 ? 4 : 2) : 1;
  // R = 1 without PDL: two CTAs per SM (measured 7-11% faster: more warps hide the decode and
  // stream latency).  With PDL the second slot is left to the next call's CTAs, which stream
  // their weights while this call computes; R > 1 keeps one CTA per SM (larger row tiles).
  const int ctas = (R == 1 && !cfg.pdl) ? 2 * cfg.sms : cfg.sms;
  const int grid = static_cast<int>(std::min<int64_t>(ctas, (N + 7) / 8));
  const int64_t rows_per_cta = (N + grid - 1) / grid;
  const int mt = rows_per_cta <= 16 ? 1 : 2;
  const int rows = 16 * mt;
  const int ntiles_max = static_cast<int>((rows_per_cta + rows - 1) / rows);
  // scales of a tile: one tensor request of 16-byte pieces (or a plain span)
  p.smode = (srb % 16 == 0 && srb / 16 <= 256 && (reinterpret_cast<uintptr_t>(sc) & 15) == 0) ? 1 : 0;
  p.spieces = p.smode ? static_cast<int>(srb / 16) : 0;
  p.sc_bytes = static_cast<uint32_t>(((p.smode ? srb * rows : srb * rows + 32) + 127) & ~int64_t(127));
  p.nsbuf = ntiles_max > 1 ? 2 : 1;
  // K segments: the smallest split whose weight stage stays within ~16 KB; a segment holds
  // whole weight pieces, whole scale groups and whole block groups, and gives each MMA warp at
  // most 8 chunks
  const size_t target = 16 * 1024;
  int ks = 0;
  for (int cand = 1; cand <= 64; ++cand) {
    if (pieces % cand || nch % cand || (nch / cand) % gc) continue;
    // a segment's scales are a fixed shift of the first one's inside the tile's scale buffer
    if (srb % cand || (p.smode && (srb / cand) % 16) || (fmt == kFmtIq2N && (nch / cand) % 4)) continue;
    const int ng = nch / cand / gc;
    if (gc * ((ng + kCWarps - 1) / kCWarps) > 8) continue;
    // every MMA warp gets work in every stage once the row is long enough for that
    if (ng < kCWarps && ks && nch / gc >= kCWarps) break;
    ks = cand;  // the smallest split within the target, else the largest valid one
    if (static_cast<size_t>(rows) * static_cast<size_t>(rb / cand) <= target) break;
  }
  if (!ks) return cudaErrorInvalidValue;
  p.kseg = ks;
  p.pieces = pieces / ks;
  CUtensorMap tmw, tms;
  if (!row_tile_map(&tmw, w, N, rb, p.pieces, pb, rows)) return cudaErrorInvalidValue;
  if (p.smode && !row_tile_map(&tms, sc, N, srb, p.spieces, 16, rows)) {  // plain span instead
    p.smode = 0;
    p.spieces = 0;
    p.sc_bytes = static_cast<uint32_t>((srb * rows + 32 + 127) & ~int64_t(127));
  }
  if (!p.smode) std::memset(&tms, 0, sizeof(tms));
  p.w_bytes = (static_cast<uint32_t>(p.pieces) * rows * pb + 1023) & ~1023u;
  const int nchs = nch / ks;
  const int cpw = gc * ((nchs / gc + kCWarps - 1) / kCWarps);
  // shared memory: ring | scale buffers | x fragments | zero page + block sums | partials
  p.xs_row = static_cast<uint32_t>(nch) * 128u + (R > 1 ? 16u : 0u);  // +16: rows on distinct banks
  const size_t sc_total = static_cast<size_t>(p.nsbuf) * p.sc_bytes;
  const size_t xs_bytes = (static_cast<size_t>(R) * p.xs_row + 127) & ~size_t(127);
  const size_t aux_bytes = (32 + (bc && fmt == kFmtQ4 ? static_cast<size_t>(K / 32) * 4 : 0) + 127) & ~size_t(127);
  const size_t red_bytes = static_cast<size_t>(kCWarps) * rows * (bc ? 1 : 8) * sizeof(float);
  const size_t fixed = 1024 + sc_total + xs_bytes + aux_bytes + red_bytes;
  const int want = ntiles_max * ks;
  // two CTAs fit on an SM (this call's and the next one's) when the budget allows; large
  // activation blocks fall back to one CTA per SM
  size_t budget = cfg.smem_budget ? cfg.smem_budget : 104 * 1024;
  if (fixed + 2 * static_cast<size_t>(p.w_bytes) > budget) budget = 220 * 1024;
  if (fixed + p.w_bytes > budget) return cudaErrorInvalidValue;
  p.nslot = static_cast<int>(std::min<size_t>({(budget - fixed) / p.w_bytes, static_cast<size_t>(kMaxSlots),
                                               static_cast<size_t>(want)}));
  p.nslot = std::max(p.nslot, 1);
  p.sc_off = static_cast<uint32_t>(static_cast<size_t>(p.nslot) * p.w_bytes);
  p.xs_off = static_cast<uint32_t>(p.sc_off + sc_total);
  p.aux_off = static_cast<uint32_t>(p.xs_off + xs_bytes);
  p.red_off = static_cast<uint32_t>(p.aux_off + aux_bytes);
  const size_t smem = 1024 + p.red_off + red_bytes;
  if (bc && !(p.wsw == 1 && p.smode == 1)) return cudaErrorInvalidValue;
  if (bc) return fmt == kFmtQ4 ? dispatch_mt<kFmtQ4, true>(mt, cpw, tmw, tms, p, grid, smem, cfg)
                               : dispatch_mt<kFmtFp4, true>(mt, cpw, tmw, tms, p, grid, smem, cfg);
  switch (fmt) {
    case kFmtQ8: return dispatch_mt<kFmtQ8, false>(mt, cpw, tmw, tms, p, grid, smem, cfg);
    case kFmtQ4: return dispatch_mt<kFmtQ4, false>(mt, cpw, tmw, tms, p, grid, smem, cfg);
    case kFmtFp4: return dispatch_mt<kFmtFp4, false>(mt, cpw, tmw, tms, p, grid, smem, cfg);
    case kFmtIq2Lut: return dispatch_mt<kFmtIq2Lut, false>(mt, cpw, tmw, tms, p, grid, smem, cfg);
    default: return dispatch_mt<kFmtIq2N, false>(mt, cpw, tmw, tms, p, grid, smem, cfg);
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
