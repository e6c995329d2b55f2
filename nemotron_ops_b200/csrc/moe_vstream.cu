// MoeVerify (int4 and both iq2 formats) on register-streaming tensor-core kernels (the reference op is
// MoeVerify's ComputeV2, src/bolt_ops.cu:1178-1257, with MoeGroupKernel :1083-1112 and the grouped
// expert GEMMs).  Weight contract of the tensor-core path: W = bf16((q - 8) * bf16(s)), bf16
// activations, fp32 sums,
//   fc1  h[p, j]    = bf16(relu(bf16(z[t] . W1[e, j]))^2)
//   fc2  part[p, n] = float(bf16(h[p] . W2[e, n]))
// then moe_finalize_kernel forms out[t, n] = bf16(sum over t's pairs, k ascending, of w * part).
//
// B200 design.  One CTA of 16 warps per SM; every CTA groups the live pairs by expert.  A layer
// is a list of 16-row tiles over the experts in use (expert-major), split evenly over the CTAs;
// a tile's K is cut into sub-units of 3 chunks of 128 k, and warp w takes every 16th sub-unit of
// its CTA.  The MMA is m16n8k16 with the tile's weight rows as M and the tokens as N (column t =
// token t: the B operand of fc1 is z for every expert, that of fc2 the h rows of the expert's
// pairs, zero for tokens that do not use the expert).  Lane (g, c) owns block 4 j + c (32 k) of
// rows g and g + 8 for chunk j: one 16-byte load per row and chunk straight from the checkpoint
// layout, all loads of the next sub-unit issued before the current one is decoded.  The decode is
// the reference rounding in bf16x2 arithmetic (bf16(128 + q) - 136, times bf16(s); see
// mma_decode.cuh).  The activations are staged in shared memory once, already in B-fragment order.
// Each sub-unit's 16 x 8 fp32 sums go to shared memory; after the CTA's last sub-unit they are
// added per tile in a fixed order (deterministic) and the epilogue writes h or part.
#include "moe_stream.cuh"

namespace bolt {

namespace {

constexpr int kVsKG = 3;       // chunks of 128 k per sub-unit
constexpr int kVsTok = 8;      // MMA columns: tokens (MoeVerify takes R <= 8)
constexpr int kVsMaxSpan = 3;  // fc2: groups a CTA's tiles may touch (staged h rows)

// uint4 offset of the B fragments (quad q of half h of chunk j, lane c) inside a staged source row;
// a row is nch * 16 + 4 uint4 long, so rows that lanes read together start 64 bytes apart mod 128
__device__ __forceinline__ int bx_index(int j, int h, int q, int c) { return ((j * 2 + h) * 2 + q) * 4 + c; }

// one 32-k block (four 16-byte pieces of 8 k, row-major bf16) -> the B fragments of its two
// 16-k halves for lane c = blk & 3 of chunk j = blk >> 2
template <int FMT>
__device__ __forceinline__ void stage_block(uint4* row, int blk, const uint4 (&v)[4]) {
  const int j = blk >> 2, c = blk & 3;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const uint32_t x16[8] = {v[2 * h].x, v[2 * h].y, v[2 * h].z, v[2 * h].w,
                             v[2 * h + 1].x, v[2 * h + 1].y, v[2 * h + 1].z, v[2 * h + 1].w};
    uint32_t b[8];
    make_b_frags<FMT>(x16, b);
    row[bx_index(j, h, 0, c)] = make_uint4(b[0], b[1], b[2], b[3]);
    row[bx_index(j, h, 1, c)] = make_uint4(b[4], b[5], b[6], b[7]);
  }
}

// 16 int4 weights (8 bytes: k 0..15 of the lane's half block) -> 8 A registers in PERM pair order
// (out[2 s] = k (s, s + 4), out[2 s + 1] = k (8 + s, 12 + s)), each bf16((q - 8) * bf16(s)): the
// arithmetic of decode_row<kFmtQ4> with the scale pair given
__device__ __forceinline__ void decode_q4_mma(uint32_t wx, uint32_t wy, __nv_bfloat162 s2, uint32_t (&out)[8]) {
  const __nv_bfloat162 zp = bits_bf2(0x43084308u);  // 136, 136
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t a = ((wx >> (4 * i)) & 0x000F000Fu) | 0x43004300u;  // 128 + n, exact
    const uint32_t b = ((wy >> (4 * i)) & 0x000F000Fu) | 0x43004300u;
    out[2 * i] = bf2_bits(__hmul2(__hsub2(bits_bf2(a), zp), s2));
    out[2 * i + 1] = bf2_bits(__hmul2(__hsub2(bits_bf2(b), zp), s2));
  }
}

__device__ __forceinline__ uint2 ld_stream8(const void* p) {
  uint2 v;
  asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
  return v;
}

// FMT: kFmtQ4 (int4), kFmtIq2Lut (iq2 = 1: 4-bit LUT codes, bf16 block-32 scales) or kFmtIq2N
// (iq2 = 2: 8-byte IQ2_XXS records per 32 k, an fp16 scale per 256 k)
template <int FC, int FMT>
__global__ void __launch_bounds__(kMsThreads, 1) moe_vstream_kernel(const MsParams p) {
  constexpr bool kIq2n = FMT == kFmtIq2N;
  __shared__ __align__(16) uint32_t grid_s[kIq2n ? 8192 : 4];  // IQ2_XXS codebook, 8 bank-group copies
  extern __shared__ __align__(16) uint8_t dsm[];
  __shared__ Groups g;
  __shared__ int tok_pair[kVsMaxSpan][kVsTok];  // fc2: pair of (group slot, token), -1: none
  __shared__ int gtp[kMsMaxP][kVsTok];          // first pair of (group, token), -1: none
  __shared__ int gdup[kMsMaxP];                 // the group has a token with two pairs
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, gq = lane >> 2, c = lane & 3;
  const int I = p.I;
  const int K = FC == 1 ? 1024 : I, NR = FC == 1 ? I : 1024, nch = K / 128;
  const int spt = (nch + kVsKG - 1) / kVsKG, TE = NR / 16;
  const int64_t wrow = kIq2n ? K / 4 : K / 2, srow = kIq2n ? K / 256 : K / 32;
  const uint8_t* W = FC == 1 ? p.w1 : p.w2;
  const uint16_t* S = reinterpret_cast<const uint16_t*>(FC == 1 ? p.s1 : p.s2);
  const int rstride = nch * 16 + 4;  // uint4 per staged source row

  if constexpr (kIq2n)
    load_iq2_grid<true>(grid_s, tid, kMsThreads);
  uint4 zv[4];
  const bool zjob = FC == 1 && tid < p.R * 32;
  if constexpr (FC == 1) {
    pdl_wait();  // z, idx and w come from the previous kernels of the stream
    pdl_trigger();
    if (zjob) {  // token tid / 32, block tid % 32, loaded while the groups form
      const uint4* zr = reinterpret_cast<const uint4*>(p.z + static_cast<int64_t>(tid >> 5) * 1024 + 32 * (tid & 31));
#pragma unroll
      for (int j = 0; j < 4; ++j) zv[j] = __ldcg(zr + j);
    }
  } else {
    pdl_trigger();  // idx is an op input: this grid starts after every fc1 CTA passed its wait
  }
  build_groups(p, g, FC == 1 && blockIdx.x == 0);
  const int T = g.U * TE;
  const int t0 = static_cast<int>(static_cast<int64_t>(blockIdx.x) * T / gridDim.x);
  const int t1 = static_cast<int>(static_cast<int64_t>(blockIdx.x + 1) * T / gridDim.x);
  const int nsu = (t1 - t0) * spt;
  const int gA = t0 / TE;

  // ---- sub-unit coordinates (group, 16-row tile in the expert, K segment), advanced by 16
  //      sub-units without divisions; the first sub-unit's loads go out before anything waits
  struct Su {
    int gi, rt, kg;
  };
  const int dtl = kMsWarps / spt, dkg = kMsWarps % spt;
  auto advance = [&](Su& u) {
    int d = dtl;
    u.kg += dkg;
    if (u.kg >= spt) {
      u.kg -= spt;
      ++d;
    }
    u.rt += d;
    while (u.rt >= TE) {
      u.rt -= TE;
      ++u.gi;
    }
  };
  Su ua;  // sub-unit `warp`
  {
    const int tile = t0 + warp / spt;
    ua = Su{tile / TE, tile % TE, warp % spt};
  }
  uint4 wq[2][kVsKG][2];
  uint32_t sq[2][kVsKG][2];
  // one base address per row and sub-unit; the chunks of the sub-unit are immediate offsets
  auto issue = [&](const Su& u, uint4 (&w)[kVsKG][2], uint32_t (&s)[kVsKG][2]) {
    const int nj = min(kVsKG, nch - u.kg * kVsKG);
    const int64_t row = static_cast<int64_t>(g.gexp[u.gi]) * NR + u.rt * 16 + gq;
    const int blk0 = 4 * kVsKG * u.kg + c;
    const uint8_t* w0 = W + row * wrow + (kIq2n ? 8 : 16) * blk0;
    const uint8_t* w1 = w0 + 8 * wrow;
    const uint16_t* s0 = S + row * srow + (kIq2n ? 0 : blk0);
    const uint16_t* s1 = s0 + 8 * srow;
#pragma unroll
    for (int jj = 0; jj < kVsKG; ++jj)
      if (jj < nj) {
        if constexpr (kIq2n) {  // one 8-byte record per row; the scale of its 256-k superblock
          const uint2 a = ld_stream8(w0 + 32 * jj), b = ld_stream8(w1 + 32 * jj);
          w[jj][0] = make_uint4(a.x, a.y, 0u, 0u);
          w[jj][1] = make_uint4(b.x, b.y, 0u, 0u);
          const int sb = (kVsKG * u.kg + jj) >> 1;
          s[jj][0] = ld_u16(s0 + sb);
          s[jj][1] = ld_u16(s1 + sb);
        } else {
          w[jj][0] = ld_stream(w0 + 64 * jj);
          w[jj][1] = ld_stream(w1 + 64 * jj);
          s[jj][0] = ld_u16(s0 + 4 * jj);
          s[jj][1] = ld_u16(s1 + 4 * jj);
        }
      }
  };
  if (warp < nsu) issue(ua, wq[0], sq[0]);
  // epilogue map, first pair of (group, token): cleared here, filled after the next barrier
  for (int i = tid; i < g.U * kVsTok; i += kMsThreads) gtp[i / kVsTok][i % kVsTok] = -1;
  if (tid < g.U) gdup[tid] = 0;

  // ---- bookkeeping of CTA 0: zero rows of pairs with an expert id outside [0, E); fc1 writes meta
  if (blockIdx.x == 0) {
    for (int q = 0; q < p.P; ++q)
      if (g.es[q] == kBadPair) {
        if constexpr (FC == 1)
          for (int i = tid; i < I; i += kMsThreads) p.h[static_cast<int64_t>(q) * I + i] = __float2bfloat16(0.f);
        else
          for (int i = tid; i < 1024; i += kMsThreads) p.part[static_cast<int64_t>(q) * 1024 + i] = 0.f;
      }
    if (FC == 1 && p.meta != nullptr) {
      // [0] U, [1 .. U] experts in first-occurrence order, then -1; [1 + P + u * 8 + token] = pair
      for (int i = tid; i < 9 * p.P; i += kMsThreads) p.meta[1 + i] = -1;
      __syncthreads();
      if (tid == 0) p.meta[0] = g.U;
      if (tid < g.U) p.meta[1 + tid] = g.gexp[tid];
      if (tid < g.nl) {
        int gi = 0;
        while (g.gstart[gi + 1] <= tid) ++gi;
        p.meta[1 + p.P + gi * 8 + g.ptok[tid]] = g.plist[tid];
      }
    }
  }

  // ---- activations in B-fragment order
  uint4* bx = reinterpret_cast<uint4*>(dsm);
  int span = 0;
  if constexpr (FC == 1) {
    if (zjob) stage_block<FMT>(bx + (tid >> 5) * rstride, tid & 31, zv);
  } else {
    span = nsu > 0 ? (t1 - 1) / TE - gA + 1 : 0;
    if (tid < kVsMaxSpan * kVsTok) tok_pair[tid / kVsTok][tid % kVsTok] = -1;
    __syncthreads();
    if (tid < g.nl) {
      int gi = 0;
      while (g.gstart[gi + 1] <= tid) ++gi;
      if (gi >= gA && gi - gA < span) tok_pair[gi - gA][g.ptok[tid]] = g.plist[tid];
    }
    pdl_wait();  // h is fc1's output
    __syncthreads();
    const int nblk = I / 32;
    for (int job = tid; job < span * kVsTok * nblk; job += kMsThreads) {
      const int sl = job / (kVsTok * nblk), rem = job - sl * kVsTok * nblk, t = rem / nblk, blk = rem - t * nblk;
      const int q = tok_pair[sl][t];
      uint4 v[4];
      if (q >= 0) {
        const uint4* src = reinterpret_cast<const uint4*>(p.h + static_cast<int64_t>(q) * I + 32 * blk);
#pragma unroll
        for (int i = 0; i < 4; ++i) v[i] = __ldcg(src + i);
      } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) v[i] = make_uint4(0u, 0u, 0u, 0u);
      }
      stage_block<FMT>(bx + (sl * kVsTok + t) * rstride, blk, v);
    }
  }
  // a zero row after the staged rows (B of tokens without a pair of the expert), then the sums
  // two zero rows after the staged rows (B of tokens without a pair of the expert): token g reads
  // the one whose 64-byte bank half matches its own staged row's, so the lanes stay conflict-free
  const int nbrows = FC == 1 ? p.R : span * kVsTok;
  const int z0 = nbrows + (nbrows & 1);  // even row index
  for (int i = tid; i < 2 * rstride; i += kMsThreads) bx[z0 * rstride + i] = make_uint4(0u, 0u, 0u, 0u);
  const uint4* bzero = bx + (z0 + (gq & 1)) * rstride;
  float* psum = reinterpret_cast<float*>(dsm + static_cast<size_t>(z0 + 2) * rstride * 16);
  __syncthreads();
  if (tid < g.nl) {  // a group's pairs ascend, so a token's pairs are adjacent
    const int gi = g.pgrp[tid];
    if (tid == g.gstart[gi] || g.ptok[tid - 1] != g.ptok[tid]) gtp[gi][g.ptok[tid]] = g.plist[tid];
    else gdup[gi] = 1;
  }

  // ---- sub-units: decode + MMA, sums to shared memory
  auto compute = [&](int su, const Su& u, const uint4 (&w)[kVsKG][2], const uint32_t (&s)[kVsKG][2]) {
    const int nj = min(kVsKG, nch - u.kg * kVsKG);
    // this lane's B row (a zero row for a token without a pair of this expert), at the sub-unit's first chunk
    const uint4* brow;
    if constexpr (FC == 1) {
      brow = gq < p.R ? bx + gq * rstride : bzero;
    } else {
      const int sl = u.gi - gA;
      brow = tok_pair[sl][gq] >= 0 ? bx + (sl * kVsTok + gq) * rstride : bzero;
    }
    brow += bx_index(kVsKG * u.kg, 0, 0, c);
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int jj = 0; jj < kVsKG; ++jj) {
      if (jj < nj) {
        const __nv_bfloat162 s0 = bits_bf2(prmt(s[jj][0], s[jj][0], 0x1010u));
        const __nv_bfloat162 s1 = bits_bf2(prmt(s[jj][1], s[jj][1], 0x1010u));
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          uint32_t a0[8], a1[8];
          if constexpr (FMT == kFmtQ4) {
            decode_q4_mma(h ? w[jj][0].z : w[jj][0].x, h ? w[jj][0].w : w[jj][0].y, s0, a0);
            decode_q4_mma(h ? w[jj][1].z : w[jj][1].x, h ? w[jj][1].w : w[jj][1].y, s1, a1);
          } else if constexpr (kIq2n) {  // half h of the record: its groups 2 h and 2 h + 1
            decode_row<kFmtIq2N, true>(RawRow{w[jj][0], s[jj][0]}, h, grid_s, a0);
            decode_row<kFmtIq2N, true>(RawRow{w[jj][1], s[jj][1]}, h, grid_s, a1);
          } else {
            decode_row<FMT>(RawRow{make_uint4(h ? w[jj][0].z : w[jj][0].x, h ? w[jj][0].w : w[jj][0].y, 0u, 0u),
                                   s[jj][0]}, 0, nullptr, a0);
            decode_row<FMT>(RawRow{make_uint4(h ? w[jj][1].z : w[jj][1].x, h ? w[jj][1].w : w[jj][1].y, 0u, 0u),
                                   s[jj][1]}, 0, nullptr, a1);
          }
          const uint4 lo = brow[bx_index(jj, h, 0, 0)], hi = brow[bx_index(jj, h, 1, 0)];
          const uint32_t b[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
#pragma unroll
          for (int m = 0; m < 4; ++m) mma16816<false>(acc, a0[2 * m], a1[2 * m], a0[2 * m + 1], a1[2 * m + 1], b[2 * m], b[2 * m + 1]);
        }
      }
    }
    *reinterpret_cast<float4*>(psum + su * 128 + lane * 4) = make_float4(acc[0], acc[1], acc[2], acc[3]);
  };
  Su ub = ua;
  advance(ub);
  for (int su = warp; su < nsu; su += 2 * kMsWarps) {
    if (su + kMsWarps < nsu) issue(ub, wq[1], sq[1]);
    compute(su, ua, wq[0], sq[0]);
    if (su + kMsWarps >= nsu) break;
    advance(ua);
    advance(ua);
    if (su + 2 * kMsWarps < nsu) issue(ua, wq[0], sq[0]);
    compute(su + kMsWarps, ub, wq[1], sq[1]);
    advance(ub);
    advance(ub);
  }
  __syncthreads();

  // ---- epilogue: per tile, the sub-units' sums in K order, then h (fc1) or part (fc2)
  {
    const int pos = tid & 127, ln = pos >> 2, e = pos & 3;
    const int t = 2 * (ln & 3) + (e & 1);          // token (MMA column)
    const int rin = (ln >> 2) + (e >= 2 ? 8 : 0);  // row inside the tile
    constexpr int kStep = kMsThreads / 128;
    int tl = tid >> 7;
    int gi = (t0 + tl) / TE, rt = (t0 + tl) % TE;
    for (; tl < t1 - t0; tl += kStep) {
      if (t < p.R) {
        float v = 0.f;
        for (int kg = 0; kg < spt; ++kg) v += psum[(tl * spt + kg) * 128 + pos];
        const float b = __bfloat162float(__float2bfloat16(v));
        const int row = rt * 16 + rin;
        auto put = [&](int q) {
          if constexpr (FC == 1) {
            const float rl = fmaxf(b, 0.f);
            p.h[static_cast<int64_t>(q) * I + row] = __float2bfloat16(rl * rl);
          } else {
            p.part[static_cast<int64_t>(q) * 1024 + row] = b;
          }
        };
        const int q = gtp[gi][t];
        if (q >= 0) put(q);
        if (gdup[gi])  // a token that names this expert twice: its other pairs get the same row
          for (int a = g.gstart[gi]; a < g.gstart[gi + 1]; ++a)
            if (g.ptok[a] == t && g.plist[a] != q) put(g.plist[a]);
      }
      rt += kStep;
      while (rt >= TE) {
        rt -= TE;
        ++gi;
      }
    }
  }
}

SmemOptIn g_vs_smem[3][2];

template <int FMT>
cudaError_t launch_layers(const MsParams& p, size_t smem1, size_t smem2, const LaunchCfg& c1, const LaunchCfg& c2) {
  SmemOptIn* cur = g_vs_smem[FMT == kFmtQ4 ? 0 : FMT == kFmtIq2N ? 1 : 2];
  cudaError_t e = allow_smem(moe_vstream_kernel<1, FMT>, smem1, cur[0]);
  if (e != cudaSuccess) return e;
  e = allow_smem(moe_vstream_kernel<2, FMT>, smem2, cur[1]);
  if (e != cudaSuccess) return e;
  e = launch_kernel(moe_vstream_kernel<1, FMT>, dim3(c1.sms), dim3(kMsThreads), smem1, c1, p);
  if (e != cudaSuccess) return e;
  return launch_kernel(moe_vstream_kernel<2, FMT>, dim3(c1.sms), dim3(kMsThreads), smem2, c2, p);
}
constexpr size_t kVsSmemCap = 200 * 1024;

}  // namespace

cudaError_t launch_moe_verify_stream(int fmt, const bf16* z, const int* idx, const float* w, const uint8_t* fc1_w,
                                     const bf16* fc1_s, const uint8_t* fc2_w, const bf16* fc2_s, int R, int E, int I,
                                     int topk, int e_begin, int e_end, bf16* out, bf16* h, float* part, int* meta,
                                     float* out_partial, const LaunchCfg& cfg, const PeerReduce* pr) {
  const int P = R * topk;
  if (fmt != kFmtQ4 && fmt != kFmtIq2Lut && fmt != kFmtIq2N) return cudaErrorNotSupported;
  if (R < 1 || R > kVsTok || P > kMsMaxP || I < 256 || I % 256) return cudaErrorNotSupported;
  const auto al = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
  if (!al(z) || !al(fc1_w) || !al(fc2_w) || !al(h) || (reinterpret_cast<uintptr_t>(fc1_s) & 1) ||
      (reinterpret_cast<uintptr_t>(fc2_s) & 1))
    return cudaErrorNotSupported;
  const int G = cfg.sms;
  // fc2: a CTA's (at most tiles2) tiles touch at most span2 groups of 64 tiles
  const int64_t tiles2 = (static_cast<int64_t>(P) * 64 + G - 1) / G;
  const int span2 = static_cast<int>((tiles2 + 63) / 64 + 1);
  // shared memory: staged activation rows (+ two zero rows and a parity pad) and the sub-unit
  // sums of the CTA's tiles
  const auto smem_for = [&](int fc) {
    const int K = fc == 1 ? 1024 : I, NR = fc == 1 ? I : 1024, nch = K / 128;
    const int spt = (nch + kVsKG - 1) / kVsKG;
    const int64_t tiles = (static_cast<int64_t>(P) * (NR / 16) + G - 1) / G;  // at most U <= P experts
    const int rows = (fc == 1 ? R : span2 * kVsTok) + 3;
    return static_cast<size_t>(rows) * (nch * 16 + 4) * 16 + static_cast<size_t>(tiles) * spt * 512;
  };
  const size_t smem1 = smem_for(1), smem2 = smem_for(2);
  if (smem1 > kVsSmemCap || smem2 > kVsSmemCap || span2 > kVsMaxSpan) return cudaErrorNotSupported;
  MsParams p{z, idx, w, fc1_w, fc1_s, fc2_w, fc2_s, h, part, out, out_partial, meta, R, P, topk, E, I, e_begin, e_end,
             0};
  LaunchCfg c2 = cfg;
  c2.pdl = true;  // same op: each kernel waits for its predecessor with griddepcontrol.wait
  cudaError_t e = fmt == kFmtQ4      ? launch_layers<kFmtQ4>(p, smem1, smem2, cfg, c2)
                  : fmt == kFmtIq2N  ? launch_layers<kFmtIq2N>(p, smem1, smem2, cfg, c2)
                                     : launch_layers<kFmtIq2Lut>(p, smem1, smem2, cfg, c2);
  if (e != cudaSuccess) return e;
  if (pr != nullptr) return launch_moe_finalize_allreduce(part, 0, w, idx, R, topk, e_begin, e_end, *pr, out, c2);
  return launch_moe_finalize(part, 0, w, idx, R, topk, e_begin, e_end, out, out_partial, c2);
}

}  // namespace bolt
