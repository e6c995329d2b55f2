// Expert GEMMs of MoeVerify and MoeDecode on tensor cores (reference: MoeMmaKernel
// src/bolt_ops.cu:1115-1167 for MoeVerify; MoeFc1Kernel / MoeFc2Kernel :497-550 for MoeDecode).
//
// Both ops are grouped skinny GEMMs over the experts the routing selected:
//  * MoeVerify (tensor-core weight contract): a group is one unique expert u of meta; its MMA
//    columns are the token rows (column j = token j, R <= 8); fc1 uses x = z, fc2 uses the h rows
//    of the pairs meta lists for u;
//  * MoeDecode (exact fp32 weight contract): a group is one (token, expert) pair; fc1 x = z of the
//    token, fc2 x = h of the pair; R = 1 per group, so the block-column mode of the streaming
//    GEMV applies (block scales in fp32, weights undecoded).
// fc1 writes h = bf16(relu(bf16(acc))^2), fc2 writes part = float(bf16(acc)) (reference
// :519-520, :549, :1159-1164); the weighted sum over k is a separate finalize kernel.
//
// B200 design: the work is a flat list of (group, 32-row tile) items over the experts' rows,
// split evenly over one CTA per SM; one tensor map covers the rows of all experts, so a tile of
// any expert is one cp.async.bulk.tensor request (128-byte swizzle); 8 MMA warps + 1 producer
// warp, K segments as ring stages, the tile's scales ride on its first stage, and a group's
// activation rows are bulk-copied into one of two shared buffers and converted in place into
// B-fragment order (the other buffer still serves the previous group).  fc2 learns its experts
// from meta before it waits for fc1, so its weights stream while fc1 finishes.
#include <algorithm>
#include <cstring>

#include "mma_decode.cuh"

namespace bolt {

namespace {

// MMA warps per CTA (CW, 8 or 16) + 1 producer warp; one CTA per SM
constexpr int kSlots = 8;

struct MoeTcParams {
  const bf16* x;        // fc1: z [R, K]; fc2: h [P, K]
  const int* list;      // verify: meta ([0] = U, experts, then the 8 columns' pairs per expert)
  const int* idx;       // [P] expert ids
  const uint8_t* w;     // expert rows [E * rows_pg, row_bytes]
  const uint8_t* sc;    // [E * rows_pg, sc_row_bytes]
  bf16* h_out;          // fc1 output [P, rows_pg]
  float* part_out;      // fc2 output [P, rows_pg]
  int verify;
  int fmt;
  int P, R, topk, K, rows_pg, E, e_begin, e_end;
  int rows;             // rows per tile: 16 * MT
  int x_once;           // the activation rows are the same for every group: staged once
  int nxb;              // activation buffers (2: the next group's rows land during this group)
  int kseg, nslot, nsbuf, pieces, wsw, smode, spieces;
  uint32_t w_bytes, sc_bytes, xs_row, xs_buf, sc_off, xs_off, aux_off, red_off;
};

__device__ __forceinline__ int ldcg_i(const int* p) {
  int v;
  asm volatile("ld.global.cg.s32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}

// Groups: MoeVerify reads them from meta; MoeDecode's groups are the pairs whose expert is in
// [e_begin, e_end) (every CTA compacts them from idx into shared memory, `lps`).
__device__ __forceinline__ int group_expert(const MoeTcParams& p, const int* lps, int g) {
  return p.verify ? ldcg_i(p.list + 1 + g) : ldcg_i(p.idx + lps[g]);
}
// pair index feeding MMA column j of group g, or -1
__device__ __forceinline__ int column_pair(const MoeTcParams& p, const int* lps, int g, int j) {
  if (p.verify) return ldcg_i(p.list + 1 + p.P + 8 * g + j);
  return j == 0 ? lps[g] : -1;
}
// activation row of column j of group g (fc1: token row of z; fc2: pair row of h), or -1
template <int FC>
__device__ __forceinline__ int column_xrow(const MoeTcParams& p, const int* lps, int g, int j) {
  if (FC == 1 && p.verify) return j < p.R ? j : -1;  // column j = token j
  const int pr = column_pair(p, lps, g, j);
  if (pr < 0) return -1;
  return FC == 1 ? pr / p.topk : pr;
}

__device__ __forceinline__ uint32_t sc_tile_off(int smode, int r, int b, int sc_rb, int rows) {
  return smode ? p16_off(r, b, rows) : static_cast<uint32_t>(r * sc_rb + b);
}

// the CTA's tiles [t0, t1) of the flat (group, tile) list
__device__ __forceinline__ void cta_tiles(int ngroups, int tpg, int& t0, int& t1) {
  const int64_t T = static_cast<int64_t>(ngroups) * tpg;
  t0 = static_cast<int>(static_cast<int64_t>(blockIdx.x) * T / gridDim.x);
  t1 = static_cast<int>(static_cast<int64_t>(blockIdx.x + 1) * T / gridDim.x);
}

template <int FC>
__device__ __forceinline__ void issue_x(const MoeTcParams& p, const int* lps, uint8_t* xs, uint64_t* x_bar, int g,
                                        int buf) {
  const int ncol = p.verify ? 8 : 1;
  uint32_t tx = 0;
  for (int j = 0; j < ncol; ++j)
    if (column_xrow<FC>(p, lps, g, j) >= 0) tx += static_cast<uint32_t>(p.K) * 2u;
  const uint32_t xb = smem_u32(&x_bar[buf]);
  mbar_arrive_expect_tx(xb, tx);
  for (int j = 0; j < ncol; ++j) {
    const int xr = column_xrow<FC>(p, lps, g, j);
    if (xr >= 0)
      bulk_g2s(smem_u32(xs + static_cast<size_t>(buf) * p.xs_buf + static_cast<size_t>(j) * p.xs_row),
               p.x + static_cast<int64_t>(xr) * p.K, static_cast<uint32_t>(p.K) * 2u, xb);
  }
}

__device__ __forceinline__ void issue_stage(const CUtensorMap* tmw, const CUtensorMap* tms, const MoeTcParams& p,
                                            uint8_t* smem, uint64_t* full_bar, int st, int t0, int tpg, int expert) {
  const int s = st % p.nslot;
  const int ti = st / p.kseg, q = st % p.kseg;
  const int t = t0 + ti;
  const int prow = expert * p.rows_pg + (t % tpg) * p.rows;  // first physical row of the tile
  const uint32_t fb = smem_u32(&full_bar[s]);
  uint32_t tx = p.w_bytes;
  if (q == 0) {
    uint8_t* sdst = smem + p.sc_off + static_cast<size_t>(ti % p.nsbuf) * p.sc_bytes;
    if (p.smode) {
      tx += static_cast<uint32_t>(p.spieces) * p.rows * 16u;
      tma_load_3d(smem_u32(sdst), tms, 0, prow, 0, fb);
    } else {  // scale rows of a non-16-byte multiple: the tile's rows are one contiguous span
      const int64_t srb = fmt_scale_row_bytes(p.fmt, p.K);
      stage_span(sdst, p.sc + static_cast<int64_t>(prow) * srb, static_cast<uint32_t>(p.rows * srb),
                 p.sc + static_cast<int64_t>(p.e_end) * p.rows_pg * srb, fb, tx);
    }
  }
  tma_load_3d(smem_u32(smem + static_cast<size_t>(s) * p.w_bytes), tmw, 0, prow, q * p.pieces, fb);
  mbar_arrive_expect_tx(fb, tx);
}

template <int FMT, bool BC, int CPW, bool FIX, int FC, int WM, int CW, int MT>
__global__ void __launch_bounds__((CW + 1) * 32, 1)
    moe_tc_kernel(const __grid_constant__ CUtensorMap tmw, const __grid_constant__ CUtensorMap tms,
                  const MoeTcParams p) {
  constexpr int ROWS = 16 * MT;
  constexpr int GC = BC ? 4 : 1;  // block-column mode exists for Q4 (exact contract) only
  constexpr int BPC = 2;
  constexpr int NG = CPW / GC;
  constexpr int KW = CW / WM;     // warps along K
  constexpr int kThr = (CW + 1) * 32;
  static_assert(!BC || FMT == kFmtQ4, "MoE block-column mode is the int4 exact contract");
  extern __shared__ __align__(16) uint8_t smem_raw[];
  __shared__ uint64_t full_bar[kSlots], empty_bar[kSlots], x_bar[2];
  __shared__ __align__(16) uint32_t grid_s[(FMT == kFmtIq2N) ? 1024 : 4];
  __shared__ int cols_s[2][8];
  __shared__ int lps[128];  // MoeDecode: the local pairs (group g = pair lps[g])
  __shared__ int nlp;
  __shared__ volatile int abort_flag;
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int K = p.K, KS = p.kseg, NS = p.nslot;
  const int tpg = p.rows_pg / ROWS;
  uint8_t* xs = smem + p.xs_off;
  if ((smem_u32(smem) & 1023u) != 0u || smem - smem_raw > 1023) {
    if (tid == 0) set_status(kStatusSmemAlign);
    return;
  }
  if (tid == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(smem_u32(&full_bar[s]), 1);
      mbar_init(smem_u32(&empty_bar[s]), CW);
    }
    mbar_init(smem_u32(&x_bar[0]), 1);
    mbar_init(smem_u32(&x_bar[1]), 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  if constexpr (FMT == kFmtIq2N) {
    for (int i = tid; i < 1024; i += kThr) grid_s[i] = kIq2xxsGridBf16x2[i];
  }
  __syncthreads();
  if constexpr (FC == 1) {
    // the group list is the previous kernel's output; fc2 may only start (and read the list
    // early) once this grid has passed its own wait
    pdl_wait();
    pdl_trigger();
  } else {
    pdl_trigger();
  }
  if (!p.verify) {
    // local pairs, in pair order; pairs whose id is outside [0, E) get zero h (fc1) / part (fc2)
    // rows from CTA 0 (the reference reads out of bounds for them)
    if (warp == 0) {
      int base = 0;
      for (int q0 = 0; q0 < p.P; q0 += 32) {
        const int q = q0 + lane;
        const int e = q < p.P ? ldcg_i(p.idx + q) : -1;
        const bool live = q < p.P && e >= p.e_begin && e < p.e_end && e >= 0 && e < p.E;
        const unsigned bal = __ballot_sync(0xffffffffu, live);
        if (live) lps[base + __popc(bal & ((1u << lane) - 1u))] = q;
        base += __popc(bal);
        if (blockIdx.x == 0 && FC == 1 && q < p.P && (e < 0 || e >= p.E)) set_status(kStatusBadExpert);
      }
      if (lane == 0) nlp = base;
    }
    if (blockIdx.x == 0) {
      for (int q = 0; q < p.P; ++q) {
        const int e = ldcg_i(p.idx + q);
        if (e >= 0 && e < p.E) continue;
        for (int i = tid; i < p.rows_pg; i += kThr) {
          if (FC == 1) p.h_out[static_cast<int64_t>(q) * p.rows_pg + i] = __float2bfloat16(0.f);
          else p.part_out[static_cast<int64_t>(q) * p.rows_pg + i] = 0.f;
        }
      }
    }
    __syncthreads();
  }
  int t0, t1;
  const int ngroups = p.verify ? ldcg_i(p.list) : nlp;
  cta_tiles(ngroups, tpg, t0, t1);
  const int ntl = t1 - t0;
  const int nstages = ntl * KS;
  const int g0 = t0 / tpg;

  // ------------------------------------------------------------------ producer warp
  if (warp == CW) {
    if (lane == 0 && ntl > 0) {
      prefetch_tensor_map(&tmw);
      if (p.smode) prefetch_tensor_map(&tms);
      // weights are constants and the expert list is ready: the first stages go out now
      const int first = min(min(NS, nstages), p.nsbuf * KS);  // a scale buffer per tile in flight
      int cur_e = -1, cur_g = -1;
      for (int st = 0; st < first; ++st) {
        const int g = (t0 + st / KS) / tpg;
        if (g != cur_g) cur_g = g, cur_e = group_expert(p, lps, g);
        issue_stage(&tmw, &tms, p, smem, full_bar, st, t0, tpg, cur_e);
      }
      pdl_wait();  // activations (z, or h of fc1) are ready
      issue_x<FC>(p, lps, xs, x_bar, g0, 0);
      int xk = 0;  // ordinal (within the CTA) of the last group whose activations were issued
      if (!p.x_once && p.nxb == 2 && cur_g > g0) {  // the up-front stages reached into the next group
        issue_x<FC>(p, lps, xs, x_bar, g0 + 1, 1);
        xk = 1;
      }
      int issued = first;
      for (int st = first; st < nstages; ++st) {
        const int s = st % NS;
        const int ti = st / KS;
        bool okw = mbar_wait(smem_u32(&empty_bar[s]), ((st / NS) - 1) & 1, kStatusEmptyWait);
        if (okw && st % KS == 0 && ti >= p.nsbuf) {  // scale buffer of tile ti - nsbuf released
          const int last = (ti - p.nsbuf + 1) * KS - 1;
          if (last > st - NS) okw = mbar_wait(smem_u32(&empty_bar[last % NS]), (last / NS) & 1, kStatusEmptyWait);
        }
        const int g = (t0 + ti) / tpg;
        // activations of every group up to this stage's: group kn goes to buffer kn % nxb once
        // group kn - nxb (all of whose stages are issued) has released its last stage
        while (okw && !p.x_once && xk < g - g0) {
          const int kn = xk + 1;
          if (kn >= p.nxb) {
            const int last = ((g0 + kn - p.nxb + 1) * tpg - t0) * KS - 1;
            if (last > st - NS) okw = mbar_wait(smem_u32(&empty_bar[last % NS]), (last / NS) & 1, kStatusEmptyWait);
          }
          if (okw) {
            issue_x<FC>(p, lps, xs, x_bar, g0 + kn, kn % p.nxb);
            xk = kn;
          }
        }
        if (!okw) abort_flag = 1;
        if (abort_flag) break;
        if (g != cur_g) cur_g = g, cur_e = group_expert(p, lps, g);
        issue_stage(&tmw, &tms, p, smem, full_bar, st, t0, tpg, cur_e);
        ++issued;
      }
      // no copy may still be landing when the CTA exits
      for (int b = 0; b <= min(xk, p.x_once ? 0 : p.nxb - 1); ++b) {
        const int k = xk - b;
        mbar_wait(smem_u32(&x_bar[k % p.nxb]), (k / p.nxb) & 1, kStatusDrainWait);
      }
      for (int st = max(0, issued - NS); st < issued; ++st)
        mbar_wait(smem_u32(&full_bar[st % NS]), (st / NS) & 1, kStatusDrainWait);
    }
    return;
  }

  // ------------------------------------------------------------------ MMA warps
  const int g = lane >> 2, t = lane & 3;
  const int pg = ((g & 3) << 1) | (g >> 2);  // MMA row g <-> tile row pg (bank spread, see GEMV)
  const int wm = warp / KW, wk = warp % KW;
  const int nch = K >> 6;
  const int nchs = nch / KS;
  int cb, ce;
  {
    const int ng = nchs / GC;
    cb = GC * (wk * ng / KW);
    ce = GC * ((wk + 1) * ng / KW);
  }
  const uint8_t* zero = smem + p.aux_off;
  float* xsum = reinterpret_cast<float*>(smem + p.aux_off + 32);  // [2][K / 32] (BC)
  float* red = reinterpret_cast<float*>(smem + p.red_off);
  if (tid < 8) reinterpret_cast<uint32_t*>(smem + p.aux_off)[tid] = 0u;

  const int wsw = FIX ? 1 : p.wsw;
  const int smode = FIX ? 1 : p.smode;
  const int sc_rb = static_cast<int>(fmt_scale_row_bytes(FMT, K));
  const uint32_t wrow8 = wsw ? 1024u : 128u;
  const uint32_t srow8 = smode ? 128u : 8u * static_cast<uint32_t>(sc_rb);
  const uint32_t sc_seg = smode ? static_cast<uint32_t>(sc_rb / KS / 16) * ROWS * 16 : static_cast<uint32_t>(sc_rb / KS);
  uint32_t woff[CPW];
  int xoff[CPW];
  uint32_t soff[NG];
#pragma unroll
  for (int j = 0; j < CPW; ++j) {
    const int c = cb + j;
    woff[j] = tile_off(wsw, pg, chunk_byte<FMT>(c, t), ROWS);
    if constexpr (BC) {
      const int blk = BPC * c + (t >> 1);
      xoff[j] = (g == (blk & 7)) ? (4 * c + t) * 32 : -1;
    } else {
      xoff[j] = static_cast<int>(g * p.xs_row) + (4 * c + t) * 32;
    }
  }
#pragma unroll
  for (int jg = 0; jg < NG; ++jg) {
    int sb;
    if constexpr (BC) sb = 2 * (BPC * (cb + jg * GC) + 2 * t);
    else sb = chunk_scale_byte<FMT>(cb + jg, t);
    soff[jg] = sc_tile_off(smode, pg, sb, sc_rb, ROWS);
  }

  bool ok = true;
  int s = 0;
  uint32_t ph = 0;
  int xbuf = 0;
  const int ncol = p.verify ? 8 : 1;
  // running tile bookkeeping (no divisions in the loop): group gg, tile tig within it, scale
  // buffer sbuf, and the 16-byte misalignment of the group's plain-span scale rows
  int gg = g0, tig = t0 - g0 * tpg, sbuf = 0;
  uint32_t sc_mis = 0;
  for (int ti = 0; ti < ntl; ++ti) {
    const int kg = gg - g0;
    if (ti == 0 || tig == 0) {  // a new group: its activations, in fragment order
      if (ti == 0 || !p.x_once) {
        xbuf = p.x_once ? 0 : kg % p.nxb;
        if (ok && !mbar_wait(smem_u32(&x_bar[xbuf]), (kg / p.nxb) & 1, kStatusFullWait)) {
          ok = false;
          abort_flag = 1;
        }
        uint8_t* xb = xs + static_cast<size_t>(xbuf) * p.xs_buf;
        if (ok && x_needs_conversion<FMT>()) {
          const int np = K >> 3;
          for (int j = 0; j < ncol; ++j) {
            if (column_xrow<FC>(p, lps, gg, j) < 0) continue;
            uint8_t* xr = xb + static_cast<size_t>(j) * p.xs_row;
            for (int base = 0; base < np; base += 4 * CW * 32) {
              uint4 v[4];
#pragma unroll
              for (int k = 0; k < 4; ++k) {
                const int pi = base + k * CW * 32 + tid;
                v[k] = pi < np ? lds128(xr + pi * 16) : make_uint4(0u, 0u, 0u, 0u);
              }
#pragma unroll
              for (int k = 0; k < 4; ++k) {
                const int pi = base + k * CW * 32 + tid;
                if (pi < np) *reinterpret_cast<uint4*>(xr + pi * 16) = x_piece_to_frag<FMT>(v[k]);
                if constexpr (BC) {
                  const uint32_t w4[4] = {v[k].x, v[k].y, v[k].z, v[k].w};
                  float sum = 0.f;
#pragma unroll
                  for (int e = 0; e < 4; ++e) sum += __uint_as_float(w4[e] << 16) + __uint_as_float(w4[e] & 0xFFFF0000u);
                  sum += __shfl_xor_sync(0xffffffffu, sum, 1);
                  sum += __shfl_xor_sync(0xffffffffu, sum, 2);
                  if (pi < np && (pi & 3) == 0) xsum[xbuf * (K >> 5) + (pi >> 2)] = sum;
                }
              }
            }
          }
        }
      }
      if (tid < 8) cols_s[kg & 1][tid] = tid < ncol ? column_pair(p, lps, gg, tid) : -1;
      // plain-span scales land at the source's offset within 16 bytes; ROWS * sc_rb is a
      // multiple of 16 (even scale rows), so the offset is the same for every tile of the group
      if (!smode)
        sc_mis = static_cast<uint32_t>(
            reinterpret_cast<uintptr_t>(p.sc + static_cast<int64_t>(group_expert(p, lps, gg)) * p.rows_pg * sc_rb) & 15);
      named_bar_sync(1, CW * 32);
    }
    const uint8_t* sct = smem + p.sc_off + static_cast<size_t>(sbuf) * p.sc_bytes + sc_mis;
    const uint8_t* xq0 = xs + static_cast<size_t>(xbuf) * p.xs_buf;
    const float* xsm0 = xsum + xbuf * (K >> 5);
    float acc[MT][4];
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
        const uint8_t* xq = xq0 + static_cast<size_t>(q * nchs) * 128;
        if constexpr (BC) {
#pragma unroll
          for (int jg = 0; jg < NG; ++jg) {
            if (cb + jg * GC < ce) {
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
                  if (WM == 1 || m == wm) {
                    wr[jj][m][0] = *reinterpret_cast<const uint2*>(wt + woff[j] + m * 2 * wrow8);
                    wr[jj][m][1] = *reinterpret_cast<const uint2*>(wt + woff[j] + m * 2 * wrow8 + wrow8);
                  }
                }
              }
              float d[GC][MT][4];
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
                  if (WM == 1 || m == wm) {
                    RawRow ra, rb;
                    ra.w = make_uint4(wr[jj][m][0].x, wr[jj][m][0].y, 0u, 0u);
                    rb.w = make_uint4(wr[jj][m][1].x, wr[jj][m][1].y, 0u, 0u);
                    uint32_t da[8], db[8];
                    decode_row_raw<FMT>(ra, da);
                    decode_row_raw<FMT>(rb, db);
#pragma unroll
                    for (int s2 = 0; s2 < 4; ++s2)
                      mma16816<false>(d[jj][m], da[2 * s2], db[2 * s2], da[2 * s2 + 1], db[2 * s2 + 1], bf[2 * s2],
                                      bf[2 * s2 + 1]);
                  }
                }
              }
              // this lane's columns 2t, 2t+1 hold scale blocks bl0 + 2t, bl0 + 2t + 1
              const int bl0 = BPC * (cb + jg * GC);
              const float2 xsv = *reinterpret_cast<const float2*>(xsm0 + BPC * q * nchs + bl0 + 2 * t);
#pragma unroll
              for (int m = 0; m < MT; ++m) {
                if (WM == 1 || m == wm) {
                  float e0 = d[0][m][0], e1 = d[0][m][1], e2 = d[0][m][2], e3 = d[0][m][3];
#pragma unroll
                  for (int jj = 1; jj < GC; ++jj) {
                    e0 += d[jj][m][0];
                    e1 += d[jj][m][1];
                    e2 += d[jj][m][2];
                    e3 += d[jj][m][3];
                  }
                  e0 = fmaf(-136.f, xsv.x, e0);
                  e1 = fmaf(-136.f, xsv.y, e1);
                  e2 = fmaf(-136.f, xsv.x, e2);
                  e3 = fmaf(-136.f, xsv.y, e3);
                  const uint8_t* sp = sq + soff[jg] + m * 2 * srow8;
                  const uint32_t ua = *reinterpret_cast<const uint32_t*>(sp);
                  const uint32_t ub = *reinterpret_cast<const uint32_t*>(sp + srow8);
                  acc[m][0] = fmaf(e0, __uint_as_float(ua << 16), acc[m][0]);
                  acc[m][0] = fmaf(e1, __uint_as_float(ua & 0xFFFF0000u), acc[m][0]);
                  acc[m][1] = fmaf(e2, __uint_as_float(ub << 16), acc[m][1]);
                  acc[m][1] = fmaf(e3, __uint_as_float(ub & 0xFFFF0000u), acc[m][1]);
                }
              }
            }
          }
        } else {
          // independent accumulator chains per m tile: chunk parity x k-step parity (MT <= 2),
          // chunk parity (MT = 4)
          constexpr int NX = MT <= 2 ? 3 : 1;
          float accx[NX][MT][4];
#pragma unroll
          for (int c = 0; c < NX; ++c)
#pragma unroll
            for (int m = 0; m < MT; ++m) accx[c][m][0] = accx[c][m][1] = accx[c][m][2] = accx[c][m][3] = 0.f;
#pragma unroll
          for (int j = 0; j < CPW; ++j) {
            if (cb + j < ce) {
              const uint8_t* xp = g < ncol ? xq + xoff[j] : zero;
              uint32_t bf[8];
              frag_from_pieces<FMT>(lds128(xp), lds128(xp + 16), bf);
#pragma unroll
              for (int m = 0; m < MT; ++m) {
                if (WM == 1 || m == wm) {
                  RawRow ra, rb;
                  ra.w = load_w_at<FMT>(wt + woff[j] + m * 2 * wrow8);
                  rb.w = load_w_at<FMT>(wt + woff[j] + m * 2 * wrow8 + wrow8);
                  ra.s = load_s_at<FMT>(sq + soff[j] + m * 2 * srow8);
                  rb.s = load_s_at<FMT>(sq + soff[j] + m * 2 * srow8 + srow8);
                  uint32_t da[8], db[8];
                  decode_row<FMT>(ra, t, grid_s, da);
                  decode_row<FMT>(rb, t, grid_s, db);
#pragma unroll
                  for (int s2 = 0; s2 < 4; ++s2) {
                    float(&dst)[4] = NX == 1 ? ((j & 1) ? accx[0][m] : acc[m])
                                             : ((j & 1) ? ((s2 & 1) ? accx[NX - 1][m] : accx[NX > 1 ? 1 : 0][m])
                                                        : ((s2 & 1) ? accx[0][m] : acc[m]));
                    mma16816<false>(dst, da[2 * s2], db[2 * s2], da[2 * s2 + 1], db[2 * s2 + 1], bf[2 * s2],
                                    bf[2 * s2 + 1]);
                  }
                }
              }
            }
          }
#pragma unroll
          for (int m = 0; m < MT; ++m)
#pragma unroll
            for (int c = 0; c < NX; ++c)
#pragma unroll
              for (int e = 0; e < 4; ++e) acc[m][e] += accx[c][m][e];
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&empty_bar[s]));
      if (++s == NS) s = 0, ph ^= 1u;
    }

    // ---- tile epilogue: sum the warps' partials, write h (fc1) or part (fc2) of the pairs.
    // The partials go to one of two buffers (tile parity), so one barrier per tile suffices: a
    // warp writes this buffer again two tiles later, after every warp has passed the barrier of
    // the tile in between, i.e. after every warp has finished reading it.
    float* redb = red + (ti & 1) * (CW * ROWS * (BC ? 1 : 8));
    if constexpr (BC) {
#pragma unroll
      for (int m = 0; m < MT; ++m) {
        float a = acc[m][0], b = acc[m][1];
        a += __shfl_xor_sync(0xffffffffu, a, 1);
        a += __shfl_xor_sync(0xffffffffu, a, 2);
        b += __shfl_xor_sync(0xffffffffu, b, 1);
        b += __shfl_xor_sync(0xffffffffu, b, 2);
        if (t == 0) {
          redb[warp * ROWS + 16 * m + pg] = a;
          redb[warp * ROWS + 16 * m + 8 + pg] = b;
        }
      }
    } else {
      // [warp][row][8 columns], the column index XOR-swizzled by row bits 2..3 (pairs stay
      // adjacent) so the column-major reads below spread over the banks
#pragma unroll
      for (int m = 0; m < MT; ++m) {
        const int ra = 16 * m + pg, rb = 16 * m + 8 + pg;
        *reinterpret_cast<float2*>(&redb[(warp * ROWS + ra) * 8 + ((2 * t) ^ (((ra >> 2) & 3) << 1))]) =
            make_float2(acc[m][0], acc[m][1]);
        *reinterpret_cast<float2*>(&redb[(warp * ROWS + rb) * 8 + ((2 * t) ^ (((rb >> 2) & 3) << 1))]) =
            make_float2(acc[m][2], acc[m][3]);
      }
    }
    named_bar_sync(1, CW * 32);
    const int row0 = tig * ROWS;
    for (int o = tid; o < ROWS * ncol; o += CW * 32) {
      const int col = o / ROWS, rl = o % ROWS;
      const int pr = cols_s[kg & 1][col];
      if (pr >= 0 && !abort_flag) {
        float v = 0.f;
        const int cs = col ^ (((rl >> 2) & 3) << 1);
#pragma unroll
        for (int w = 0; w < CW; ++w) v += BC ? redb[w * ROWS + rl] : redb[(w * ROWS + rl) * 8 + cs];
        const float bv = __bfloat162float(__float2bfloat16(v));
        const int64_t oi = static_cast<int64_t>(pr) * p.rows_pg + row0 + rl;
        if constexpr (FC == 1) {
          const float r = fmaxf(bv, 0.f);
          p.h_out[oi] = __float2bfloat16(r * r);  // r * r is exact in fp32
        } else {
          p.part_out[oi] = bv;
        }
      }
    }
    if (++tig == tpg) tig = 0, ++gg;
    if (++sbuf == p.nsbuf) sbuf = 0;
  }
}

template <int FMT, bool BC, int CPW, bool FIX, int FC, int WM, int CW, int MT>
cudaError_t launch_one(const CUtensorMap& tmw, const CUtensorMap& tms, const MoeTcParams& p, size_t smem,
                       const LaunchCfg& cfg) {
  auto kern = moe_tc_kernel<FMT, BC, CPW, FIX, FC, WM, CW, MT>;
  static SmemOptIn opt;
  cudaError_t e = allow_smem(kern, smem, opt);
  if (e != cudaSuccess) return e;
  return launch_kernel(kern, dim3(cfg.sms), dim3((CW + 1) * 32), smem, cfg, tmw, tms, p);
}

template <int FMT, bool BC, int FC, int WM, int CW, int MT>
cudaError_t dispatch_fix(int cpw, bool fix, const CUtensorMap& tmw, const CUtensorMap& tms, const MoeTcParams& p,
                         size_t smem, const LaunchCfg& cfg) {
  if constexpr (BC) {
    if (!fix) return cudaErrorInvalidValue;
    if (cpw <= 4) return launch_one<FMT, BC, 4, true, FC, WM, CW, MT>(tmw, tms, p, smem, cfg);
    return launch_one<FMT, BC, 8, true, FC, WM, CW, MT>(tmw, tms, p, smem, cfg);
  } else {
    static_assert(WM == 1, "grouped MMA path splits K only");
    if (cpw <= 2) return fix ? launch_one<FMT, BC, 2, true, FC, 1, CW, MT>(tmw, tms, p, smem, cfg)
                             : launch_one<FMT, BC, 2, false, FC, 1, CW, MT>(tmw, tms, p, smem, cfg);
    if (cpw <= 4) return fix ? launch_one<FMT, BC, 4, true, FC, 1, CW, MT>(tmw, tms, p, smem, cfg)
                             : launch_one<FMT, BC, 4, false, FC, 1, CW, MT>(tmw, tms, p, smem, cfg);
    return fix ? launch_one<FMT, BC, 8, true, FC, 1, CW, MT>(tmw, tms, p, smem, cfg)
               : launch_one<FMT, BC, 8, false, FC, 1, CW, MT>(tmw, tms, p, smem, cfg);
  }
}

// dense (tensor-core contract) dispatch over the format and the tile height
template <int FC>
cudaError_t dispatch_dense(int fmt, int mt, int cpw, bool fix, const CUtensorMap& tmw, const CUtensorMap& tms,
                           const MoeTcParams& p, size_t smem, const LaunchCfg& cfg) {
  switch (fmt) {
    case kFmtQ4:
      return mt == 4 ? dispatch_fix<kFmtQ4, false, FC, 1, 8, 4>(cpw, fix, tmw, tms, p, smem, cfg)
                     : dispatch_fix<kFmtQ4, false, FC, 1, 8, 2>(cpw, fix, tmw, tms, p, smem, cfg);
    case kFmtIq2Lut:
      return mt == 4 ? dispatch_fix<kFmtIq2Lut, false, FC, 1, 8, 4>(cpw, fix, tmw, tms, p, smem, cfg)
                     : dispatch_fix<kFmtIq2Lut, false, FC, 1, 8, 2>(cpw, fix, tmw, tms, p, smem, cfg);
    default:
      return mt == 4 ? dispatch_fix<kFmtIq2N, false, FC, 1, 8, 4>(cpw, fix, tmw, tms, p, smem, cfg)
                     : dispatch_fix<kFmtIq2N, false, FC, 1, 8, 2>(cpw, fix, tmw, tms, p, smem, cfg);
  }
}

// Plans and launches one grouped GEMM (fc1 or fc2) over the expert rows.
cudaError_t launch_grouped(int fmt, bool bc, int fc, bool verify, const bf16* x, const int* list, const int* idx,
                           const uint8_t* w, const void* sc, bf16* h_out, float* part_out, int P, int R, int topk,
                           int E, int e_begin, int e_end, int K, int rows_pg, const LaunchCfg& cfg) {
  MoeTcParams p{};
  p.x = x;
  p.list = list;
  p.idx = idx;
  p.w = w;
  p.sc = static_cast<const uint8_t*>(sc);
  p.h_out = h_out;
  p.part_out = part_out;
  p.verify = verify ? 1 : 0;
  p.fmt = fmt;
  p.P = P;
  p.R = R;
  p.topk = topk;
  p.K = K;
  p.rows_pg = rows_pg;
  p.E = E;
  p.e_begin = e_begin;
  p.e_end = e_end;
  p.x_once = (fc == 1 && (verify || R == 1)) ? 1 : 0;
  // tile height: 64 rows where every CTA still gets >= 8 tiles at the largest group count
  // (halves the per-tile reduction and gives each warp four m tiles per B fragment), else 32
  const int max_groups = verify ? std::min(P, e_end - e_begin) : P;
  const int mt =
      (!bc && rows_pg % 64 == 0 && static_cast<int64_t>(max_groups) * (rows_pg / 64) >= 8LL * cfg.sms) ? 4 : 2;
  const int rows = 16 * mt;
  p.rows = rows;
  if (rows_pg % rows) return cudaErrorInvalidValue;
  const int64_t rb = fmt_row_bytes(fmt, K);
  const int64_t srb = fmt_scale_row_bytes(fmt, K);
  p.wsw = rb % 128 == 0 ? 1 : 0;
  const int pb = p.wsw ? 128 : 16;
  const int pieces = static_cast<int>(rb / pb);
  const int nch = K >> 6;
  const int gc = bc ? 4 : 1;
  p.smode = (srb % 16 == 0 && srb / 16 <= 256 && (reinterpret_cast<uintptr_t>(sc) & 15) == 0) ? 1 : 0;
  p.spieces = p.smode ? static_cast<int>(srb / 16) : 0;
  p.sc_bytes = static_cast<uint32_t>((srb * rows + (p.smode ? 0 : 32) + 127) & ~int64_t(127));
  const int ncol = verify ? 8 : 1;
  p.xs_row = static_cast<uint32_t>(nch) * 128u + (ncol > 1 ? 16u : 0u);
  p.xs_buf = (static_cast<uint32_t>(ncol) * p.xs_row + 127u) & ~127u;
  const size_t aux_bytes = (32 + (bc ? 2 * static_cast<size_t>(K / 32) * 4 : 0) + 127) & ~size_t(127);
  const int cw = 8;  // MMA warps (16 measured no faster: the decode is issue-bound)
  const size_t red_bytes = 2 * static_cast<size_t>(cw) * rows * (bc ? 1 : 8) * sizeof(float);
  const size_t budget = cfg.smem_budget ? cfg.smem_budget : 220 * 1024;
  // K segments: every MMA warp busy, stages within ~32 KB, at least two stages in the budget;
  // two activation buffers where they fit, else one (the next group's rows wait for this group)
  // scale buffers: one per tile that the ring of ns stages can hold, plus the one being read
  auto nsbuf_for = [](int ns, int kseg) { return std::min(kSlots, (ns + kseg - 1) / kseg + 1); };
  int ks = 0, wm = 1;
  size_t fixed = 0;
  for (int nxb = 2; nxb >= 1 && !ks; --nxb) {
    p.nxb = p.x_once ? 1 : nxb;
    fixed = 1024 + static_cast<size_t>(p.nxb) * p.xs_buf + aux_bytes + red_bytes;
    for (int cand = 1; cand <= 64; ++cand) {
      if (pieces % cand || nch % cand || (nch / cand) % gc || srb % cand) continue;
      if (p.smode && (srb / cand) % 16) continue;
      if (fmt == kFmtIq2N && (nch / cand) % 4) continue;
      const int ng = nch / cand / gc;
      const int kw = (bc && ng < cw) ? cw / 2 : cw;
      if (ng < kw && ks) break;
      if (gc * ((ng + kw - 1) / kw) > 8) continue;
      const size_t wb = (static_cast<size_t>(pieces / cand) * rows * pb + 1023) & ~size_t(1023);
      if (fixed + 2 * wb + static_cast<size_t>(nsbuf_for(2, cand)) * p.sc_bytes > budget) continue;
      ks = cand;
      wm = cw / kw;
      if (wb <= static_cast<size_t>(rows) * 1024) break;
    }
    if (p.x_once) break;
  }
  if (!ks) return cudaErrorInvalidValue;
  p.kseg = ks;
  p.pieces = pieces / ks;
  CUtensorMap tmw, tms;
  if (!row_tile_map(&tmw, w, static_cast<int64_t>(E) * rows_pg, rb, p.pieces, pb, rows)) return cudaErrorInvalidValue;
  if (p.smode && !row_tile_map(&tms, sc, static_cast<int64_t>(E) * rows_pg, srb, p.spieces, 16, rows))
    return cudaErrorInvalidValue;
  if (!p.smode) std::memset(&tms, 0, sizeof(tms));
  p.w_bytes = (static_cast<uint32_t>(p.pieces) * rows * pb + 1023) & ~1023u;
  const int nchs = nch / ks;
  const int kw = cw / wm;
  const int cpw = gc * ((nchs / gc + kw - 1) / kw);
  const size_t xs_bytes = static_cast<size_t>(p.nxb) * p.xs_buf;
  for (p.nslot = kSlots; p.nslot > 2; --p.nslot)
    if (fixed + static_cast<size_t>(p.nslot) * p.w_bytes + static_cast<size_t>(nsbuf_for(p.nslot, ks)) * p.sc_bytes <=
        budget)
      break;
  p.nsbuf = nsbuf_for(p.nslot, ks);
  p.sc_off = static_cast<uint32_t>(static_cast<size_t>(p.nslot) * p.w_bytes);
  p.xs_off = p.sc_off + static_cast<uint32_t>(p.nsbuf) * p.sc_bytes;
  p.aux_off = static_cast<uint32_t>(p.xs_off + xs_bytes);
  p.red_off = static_cast<uint32_t>(p.aux_off + aux_bytes);
  const size_t smem = 1024 + p.red_off + red_bytes;
  const bool fix = p.wsw == 1 && p.smode == 1;
  if (bc) {  // block-column mode (32-row tiles)
    if (fmt != kFmtQ4 || mt != 2) return cudaErrorInvalidValue;
    if (fc == 1) return wm == 2 ? dispatch_fix<kFmtQ4, true, 1, 2, 8, 2>(cpw, fix, tmw, tms, p, smem, cfg)
                                : dispatch_fix<kFmtQ4, true, 1, 1, 8, 2>(cpw, fix, tmw, tms, p, smem, cfg);
    return wm == 2 ? dispatch_fix<kFmtQ4, true, 2, 2, 8, 2>(cpw, fix, tmw, tms, p, smem, cfg)
                   : dispatch_fix<kFmtQ4, true, 2, 1, 8, 2>(cpw, fix, tmw, tms, p, smem, cfg);
  }
  return fc == 1 ? dispatch_dense<1>(fmt, mt, cpw, fix, tmw, tms, p, smem, cfg)
                 : dispatch_dense<2>(fmt, mt, cpw, fix, tmw, tms, p, smem, cfg);
}

}  // namespace

// group kernel (moe.cu): meta of the unique experts in [e_begin, e_end)
cudaError_t launch_moe_group(const int* idx, int P, int topk, int e_begin, int e_end, int* meta, const LaunchCfg& cfg);
// tcgen05 expert layer (moe_umma.cu): whether it takes a layer, and the launch.  Its CTAs build the
// expert list from idx themselves; fc1 zeroes part_out when given one (fc2 with split relies on
// that to split tiles) and writes meta when given meta_out.
bool moe_layer_umma_ok(int fmt, const void* sc, int P, int K, int rows_pg);
cudaError_t launch_moe_layer_umma(int fmt, int fc, const bf16* x, const int* idx, int topk, int e_begin, int* meta_out,
                                  const uint8_t* w, const void* sc, bf16* h_out, float* part_out, int P, int R, int E,
                                  int e_end, int K, int rows_pg, const LaunchCfg& cfg, int split);

cudaError_t launch_moe_verify(int fmt, const bf16* z, const int* idx, const float* w, const uint8_t* fc1_w,
                              const bf16* fc1_s, const uint8_t* fc2_w, const bf16* fc2_s, int R, int E, int I,
                              int topk, int e_begin, int e_end, bf16* out, bf16* h, float* part, int* meta,
                              float* out_partial, const LaunchCfg& cfg, const PeerReduce* pr) {
  const int P = R * topk;
  {  // register-streaming tensor-core kernels (moe_vstream.cu) where they take the shape
    const cudaError_t e = launch_moe_verify_stream(fmt, z, idx, w, fc1_w, fc1_s, fc2_w, fc2_s, R, E, I, topk, e_begin,
                                                   e_end, out, h, part, meta, out_partial, cfg, pr);
    if (e != cudaErrorNotSupported) return e;
  }
  // tcgen05 layers where they apply (int4 / native IQ2_XXS, 128-row tiles), else mma.sync.  The
  // tcgen05 layers build the expert list from idx in every CTA; the grouping kernel (which writes
  // meta, read by the mma.sync layers) runs only when a layer falls back, else fc1 writes meta.
  const bool u1 = moe_layer_umma_ok(fmt, fc1_s, P, 1024, I), u2 = moe_layer_umma_ok(fmt, fc2_s, P, I, 1024);
  const bool group = !(u1 && u2);
  LaunchCfg c2 = cfg;
  c2.pdl = true;  // same op: each kernel waits for its predecessor with griddepcontrol.wait
  cudaError_t e = cudaSuccess;
  if (group) {
    e = launch_moe_group(idx, P, topk, e_begin, e_end, meta, cfg);
    if (e != cudaSuccess) return e;
  }
  // the tcgen05 fc1 also zeroes part (16-byte aligned), which lets the tcgen05 fc2 split tiles
  const bool part16 = (reinterpret_cast<uintptr_t>(part) & 15) == 0;
  if (u1)
    e = launch_moe_layer_umma(fmt, 1, z, idx, topk, e_begin, group ? nullptr : meta, fc1_w, fc1_s, h,
                              part16 ? part : nullptr, P, R, E, e_end, 1024, I, group ? c2 : cfg, 0);
  else
    e = launch_grouped(fmt, false, 1, true, z, meta, idx, fc1_w, fc1_s, h, nullptr, P, R, topk, E, e_begin, e_end,
                       1024, I, c2);
  if (e != cudaSuccess) return e;
  const bool zeroed = u1 && part16;
  if (u2)
    e = launch_moe_layer_umma(fmt, 2, h, idx, topk, e_begin, nullptr, fc2_w, fc2_s, nullptr, part, P, R, E, e_end, I,
                              1024, c2, zeroed ? 1 : 0);
  else
    e = launch_grouped(fmt, false, 2, true, h, meta, idx, fc2_w, fc2_s, nullptr, part, P, R, topk, E, e_begin, e_end,
                       I, 1024, c2);
  if (e != cudaSuccess) return e;
  if (pr != nullptr) return launch_moe_finalize_allreduce(part, 1, w, idx, R, topk, e_begin, e_end, *pr, out, c2);
  return launch_moe_finalize(part, 1, w, idx, R, topk, e_begin, e_end, out, out_partial, c2);
}

cudaError_t launch_moe_decode(const bf16* z, const int* idx, const float* w, const uint8_t* fc1_w, const bf16* fc1_s,
                              const uint8_t* fc2_w, const bf16* fc2_s, int R, int E, int I, int topk, int e_begin,
                              int e_end, bf16* out, bf16* h, float* part, float* out_partial, const LaunchCfg& cfg) {
  const int P = R * topk;
  {  // bulk-copy streaming kernels (moe_stream.cu) where they take the shape
    const cudaError_t e = launch_moe_decode_stream(z, idx, w, fc1_w, fc1_s, fc2_w, fc2_s, R, E, I, topk, e_begin, e_end,
                                               out, h, part, out_partial, cfg);
    if (e != cudaErrorNotSupported) return e;
  }
  cudaError_t e = launch_grouped(kFmtQ4, true, 1, false, z, nullptr, idx, fc1_w, fc1_s, h, nullptr, P, R, topk, E,
                                 e_begin, e_end, 1024, I, cfg);
  if (e != cudaSuccess) return e;
  LaunchCfg c2 = cfg;
  c2.pdl = true;  // same op: fc2 waits for fc1 with griddepcontrol.wait
  e = launch_grouped(kFmtQ4, true, 2, false, h, nullptr, idx, fc2_w, fc2_s, nullptr, part, P, R, topk, E, e_begin,
                     e_end, I, 1024, c2);
  if (e != cudaSuccess) return e;
  return launch_moe_finalize(part, 0, w, idx, R, topk, e_begin, e_end, out, out_partial, c2);
}

}  // namespace bolt
