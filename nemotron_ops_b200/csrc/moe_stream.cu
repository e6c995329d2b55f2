// MoeDecode on two weight-streaming kernels (the reference op is MoeDecodeState,
// src/bolt_ops.cu:589-619; kernels MoeFc1Kernel / MoeFc2Kernel / MoeFinalizeKernel :497-587).
// Exact fp32 weight contract: every (token, expert) pair is a GEMV over its expert's int4 rows,
//   fc1  h[p, j]    = bf16(relu(bf16(z[t] . W1[e, j]))^2)        W = (q - 8) * s, fp32
//   fc2  part[p, n] = float(bf16(h[p] . W2[e, n]))
//   out[t, n]       = bf16(sum over t's pairs, k ascending, of w[t, k] * part[p, n])
// with the last line done by the fc2 kernel itself (two launches per op).
//
// B200 design.  One CTA of 16 warps per SM.  Every CTA first groups the live pairs by expert
// (groups in order of first occurrence, pairs ascending), so an expert's rows are read once
// whatever the number of its pairs.  The weights are small per CTA (tens of KB in rows of
// 512-1152 bytes), so they stream through registers: every warp issues the loads of all its rows
// (16 bytes = one 32-k scale block per lane, 512 contiguous bytes per load instruction) before it
// uses any, which puts the CTA's whole share in flight in one round trip.  (Bulk copies were
// measured slower here: the copy engine takes ~0.2 us to accept each request, and a CTA needs
// one per expert slab.)  A lane decodes bf16(128 + q) pairs (a shift and a LOP3 per two
// weights), multiplies them by the activations with mixed-precision fma.rn.f32.bf16 (exact
// products, fp32 sums) and removes 136 * (the block's sum of x) afterwards; the decoded block is
// reused for every pair of the expert.
//   fc1: the CTA's units are a contiguous range of (group, row j); warp w takes every 16th row.
//        The tokens' activations sit in shared memory in PERM order.
//   fc2: the CTA owns output rows [n0, n0 + nrow) of every group; warp w takes every 16th
//        (group, row) unit.  The weights do not depend on fc1 and are loaded before the
//        dependency wait; then the h rows of all live pairs are staged in shared memory (PERM
//        order, block sums), and at the end the CTA forms out[t, n] for its rows.
// Pairs whose expert is outside [0, E) get zero h / part rows and set a status bit; pairs outside
// the shard's expert range [e_begin, e_end) are left untouched and do not enter the sum.
#include "moe_stream.cuh"

namespace bolt {

namespace {
constexpr int kFc1Batch = 8;             // fc1 rows in flight per warp

// a += lo(q) * lo(x), b += hi(q) * hi(x) for bf16 pairs: exact products, fp32 sums
__device__ __forceinline__ void fma2_bf16_f32(uint32_t q, uint32_t x, float& a, float& b) {
  asm("{\n .reg .b16 ql, qh, xl, xh;\n mov.b32 {ql, qh}, %2;\n mov.b32 {xl, xh}, %3;\n"
      " fma.rn.f32.bf16 %0, ql, xl, %0;\n fma.rn.f32.bf16 %1, qh, xh, %1;\n}\n"
      : "+f"(a), "+f"(b)
      : "r"(q), "r"(x));
}

// the 16 bf16(128 + q) pairs of one 16-byte block (word i, nibbles s and s + 4 -> pair 4 i + s)
__device__ __forceinline__ void decode128(const uint4& wq, uint32_t (&d)[16]) {
  const uint32_t wv[4] = {wq.x, wq.y, wq.z, wq.w};
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int s = 0; s < 4; ++s) d[4 * i + s] = ((wv[i] >> (4 * s)) & 0x000F000Fu) | 0x43004300u;
}

// sum over the block of (128 + q) * x; x as four 16-byte PERM pieces (pair order of decode128)
__device__ __forceinline__ float dot128(const uint32_t (&d)[16], const uint4 (&x)[4]) {
  float a0 = 0.f, b0 = 0.f, a1 = 0.f, b1 = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    fma2_bf16_f32(d[4 * i + 0], x[i].x, a0, b0);
    fma2_bf16_f32(d[4 * i + 1], x[i].y, a1, b1);
    fma2_bf16_f32(d[4 * i + 2], x[i].z, a0, b0);
    fma2_bf16_f32(d[4 * i + 3], x[i].w, a1, b1);
  }
  return (a0 + b0) + (a1 + b1);
}

// 32 bf16 activations (four 16-byte pieces of 8 k) -> PERM pieces, and their fp32 sum
__device__ __forceinline__ float perm_block(const uint4 (&v)[4], uint4 (&o)[4]) {
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    o[i] = x_piece_to_frag<kFmtQ4>(v[i]);
    const uint32_t w4[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
#pragma unroll
    for (int e = 0; e < 4; ++e) sum += __uint_as_float(w4[e] << 16) + __uint_as_float(w4[e] & 0xFFFF0000u);
  }
  return sum;
}

// ------------------------------------------------------------------------------------------
// fc1: h[p, j] = bf16(relu(bf16(z[t] . W1[e, j]))^2) for the live pairs (K = 1024)
// ------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(kMsThreads, 1) moe_stream_fc1_kernel(const MsParams p) {
  extern __shared__ __align__(16) uint8_t dsm[];
  __shared__ Groups g;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // z, idx and w come from the previous kernels of the stream
  pdl_wait();
  pdl_trigger();
  // the lane's 32 activations of one token (R * 32 jobs), loaded while the groups form
  const bool zjob = tid < p.R * 32;
  uint4 zv[4];
  if (zjob) {
    const uint4* zr = reinterpret_cast<const uint4*>(p.z + static_cast<int64_t>(tid >> 5) * 1024 + 32 * (tid & 31));
#pragma unroll
    for (int j = 0; j < 4; ++j) zv[j] = __ldcg(zr + j);
  }
  build_groups(p, g, blockIdx.x == 0);
  const int I = p.I;
  // units (group, row j) in a flat index < U * I <= 128 * 4096; the CTA owns [u0, u1)
  const int total = g.U * I;
  const int u0 = static_cast<int>(static_cast<int64_t>(blockIdx.x) * total / gridDim.x);
  const int u1 = static_cast<int>(static_cast<int64_t>(blockIdx.x + 1) * total / gridDim.x);
  uint4 wq[kFc1Batch];
  uint32_t sq[kFc1Batch];
  int gr[kFc1Batch], jr[kFc1Batch];  // (group, row) of each row of the batch; gr < 0: none
  // rows ub, ub + 16, ... of the CTA's range: every load of the batch before any use
  int ub = u0 + warp;
  int gcur = ub / I, jcur = ub - (ub / I) * I;  // position of row ub, advanced by 16 per row
  auto issue = [&]() {
#pragma unroll
    for (int r = 0; r < kFc1Batch; ++r) {
      const bool ok = ub + r * kMsWarps < u1;
      gr[r] = ok ? gcur : -1;
      jr[r] = jcur;
      if (ok) {
        const int64_t row = static_cast<int64_t>(g.gexp[gcur]) * I + jcur;
        wq[r] = ld_stream(p.w1 + row * 512 + 16 * lane);
        sq[r] = ld_u16(p.s1 + row * 32 + lane);
      }
      jcur += kMsWarps;
      if (jcur >= I) {
        jcur -= I;
        ++gcur;
      }
    }
  };
  issue();
  {  // fc2's weights of these experts into L2 (fc2 loads them from there): this CTA's share, one
     // 128-byte line per thread and step
    const uint32_t per_w = 1024u * (I / 2), per = per_w + 1024u * (I / 16);  // bytes per expert
    const uint32_t tot = static_cast<uint32_t>(g.U) * per;
    const uint32_t b0 = static_cast<uint32_t>(static_cast<uint64_t>(blockIdx.x) * tot / gridDim.x) & ~127u;
    const uint32_t b1 = static_cast<uint32_t>(static_cast<uint64_t>(blockIdx.x + 1) * tot / gridDim.x);
    for (uint32_t o = b0 + 128u * tid; o < b1; o += 128u * kMsThreads) {
      const uint32_t gi = o / per, off = o - gi * per;
      const int64_t e = g.gexp[gi];
      const uint8_t* a = off < per_w ? p.w2 + e * per_w + off
                                     : reinterpret_cast<const uint8_t*>(p.s2) + e * (1024 * (I / 16)) + (off - per_w);
      asm volatile("prefetch.global.L2 [%0];" ::"l"(a));
    }
  }
  if (blockIdx.x == 0)  // pairs whose expert id is outside [0, E): zero h rows
    for (int q = 0; q < p.P; ++q)
      if (g.es[q] == kBadPair)
        for (int i = tid; i < I; i += kMsThreads) p.h[static_cast<int64_t>(q) * I + i] = __float2bfloat16(0.f);
  // the tokens' activations in PERM pieces [t][piece][lane] and the lanes' block sums [t][lane]
  uint4* xz = reinterpret_cast<uint4*>(dsm);
  float* xsz = reinterpret_cast<float*>(dsm + static_cast<size_t>(p.R) * 2048);
  if (zjob) {
    const int t = tid >> 5, l = tid & 31;
    uint4 o[4];
    xsz[tid] = perm_block(zv, o);
#pragma unroll
    for (int j = 0; j < 4; ++j) xz[(t * 4 + j) * 32 + l] = o[j];
  }
  __syncthreads();
  while (ub < u1) {
    // pair slot k of every row's group: the 8 rows' dots with their k-th pair's token, one
    // butterfly reduction, and lane 4 r writes row r
    int kmax = 0;
#pragma unroll
    for (int r = 0; r < kFc1Batch; ++r)
      if (gr[r] >= 0) kmax = max(kmax, g.gstart[gr[r] + 1] - g.gstart[gr[r]]);
    const int myr = (lane >> 2) & 7;
    int myg = -1, myj = 0;
#pragma unroll
    for (int r = 0; r < kFc1Batch; ++r)
      if (r == myr) {
        myg = gr[r];
        myj = jr[r];
      }
    for (int k = 0; k < kmax; ++k) {
      float vals[kFc1Batch];
      int tprev = -1;
      uint4 x[4];
      float xsv = 0.f;
#pragma unroll
      for (int r = 0; r < kFc1Batch; ++r) {
        vals[r] = 0.f;
        if (gr[r] < 0) continue;
        const int a = g.gstart[gr[r]] + k;
        if (a >= g.gstart[gr[r] + 1]) continue;
        const int t = g.ptok[a];
        if (t != tprev) {  // warp-uniform
#pragma unroll
          for (int i = 0; i < 4; ++i) x[i] = xz[(t * 4 + i) * 32 + lane];
          xsv = xsz[t * 32 + lane];
          tprev = t;
        }
        uint32_t d[16];
        decode128(wq[r], d);
        vals[r] = fmaf(-136.f, xsv, dot128(d, x)) * bf16_bits_to_f32(sq[r]);
      }
      const float v = warp_sum8_t(vals);
      if ((lane & 3) == 0 && myg >= 0 && g.gstart[myg] + k < g.gstart[myg + 1]) {
        const int q = g.plist[g.gstart[myg] + k];
        const float rl = fmaxf(__bfloat162float(__float2bfloat16(v)), 0.f);
        p.h[static_cast<int64_t>(q) * I + myj] = __float2bfloat16(rl * rl);
      }
    }
    ub += kFc1Batch * kMsWarps;
    if (ub < u1) issue();
  }
}

// ------------------------------------------------------------------------------------------
// fc2 + finalize: part[p, n] for the live pairs and this CTA's rows n, then out[t, n]
// ------------------------------------------------------------------------------------------
// A warp task is rn <= RT rows of one group.  A row's nchunk = 32 F + L 16-byte chunks: lane l
// takes chunks l + 32 f (f < F) of every row of the task, so one activation chunk serves all the
// task's rows, plus at most one of the rn * L <= 32 remaining chunks; the task's row sums then
// meet in one butterfly reduction.  Every load of the task is issued before the first use.
template <int F>
struct Fc2Shape {
  static constexpr int RT = F <= 2 ? 4 : (F <= 4 ? 2 : 1);  // rows per task: RT * F <= 8 chunks in registers
};

template <int RT>
__device__ __forceinline__ float warp_sum_rows(const float (&v)[RT]) {
  if constexpr (RT == 4) return warp_sum4_t(v);
  else if constexpr (RT == 2) return warp_sum2_t(v);
  else return warp_sum(v[0]);
}

template <int F>
__global__ void __launch_bounds__(kMsThreads, 1) moe_stream_fc2_kernel(const MsParams p) {
  constexpr int RT = Fc2Shape<F>::RT;
  extern __shared__ __align__(16) uint8_t dsm[];
  __shared__ Groups g;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  __shared__ float ws[kMsMaxP];
  pdl_trigger();
  // idx and w are op inputs: this grid starts only after every fc1 CTA passed its dependency wait
  if (tid < p.P) ws[tid] = __ldcg(p.w + tid);
  build_groups(p, g, false);
  const int I = p.I, nchunk = I / 32, L = nchunk - 32 * F;
  const int64_t wrow = I / 2;
  const int n0 = blockIdx.x * p.nrow, nr = min(p.nrow, 1024 - n0);
  const int rt = L > 0 ? min(RT, 32 / L) : RT;  // rows per task: the remaining chunks fit the lanes
  const int tpe = (nr + rt - 1) / rt;            // tasks per group
  const int ntask = g.U * tpe;
  uint4 wq[RT][F > 0 ? F : 1], wl = make_uint4(0u, 0u, 0u, 0u);
  uint32_t sq[RT][F > 0 ? F : 1], sl = 0u;
  int gi = 0, r0 = 0, rn = 0;  // the current task: group, first row, rows
  const int lr = L > 0 ? lane / L : 0, lc = 32 * F + (L > 0 ? lane % L : 0);  // this lane's remaining chunk
  auto issue = [&](int task) {
    gi = task / tpe;
    r0 = (task - gi * tpe) * rt;
    rn = min(rt, nr - r0);
    const int64_t row0 = static_cast<int64_t>(g.gexp[gi]) * 1024 + n0 + r0;
#pragma unroll
    for (int r = 0; r < RT; ++r)
      if (r < rn)
#pragma unroll
        for (int f = 0; f < F; ++f) {
          wq[r][f] = ld_stream(p.w2 + (row0 + r) * wrow + 16 * (lane + 32 * f));
          sq[r][f] = ld_u16(p.s2 + (row0 + r) * nchunk + lane + 32 * f);
        }
    if (lane < rn * L) {
      wl = ld_stream(p.w2 + (row0 + lr) * wrow + 16 * lc);
      sl = ld_u16(p.s2 + (row0 + lr) * nchunk + lc);
    }
  };
  int task = warp;
  if (task < ntask) issue(task);  // weights are op inputs, complete before fc1 passed its wait
  pdl_wait();  // h is fc1's output
  if (blockIdx.x == 0)  // pairs whose expert id is outside [0, E): zero part rows
    for (int q = 0; q < p.P; ++q)
      if (g.es[q] == kBadPair)
        for (int i = tid; i < 1024; i += kMsThreads) p.part[static_cast<int64_t>(q) * 1024 + i] = 0.f;
  // h rows of the live pairs (plist order) in PERM pieces [a][piece][chunk], block sums [a][chunk]
  uint4* xh = reinterpret_cast<uint4*>(dsm);
  float* xs = reinterpret_cast<float*>(dsm + static_cast<size_t>(g.nl) * nchunk * 64);
  float* pv = reinterpret_cast<float*>(dsm + static_cast<size_t>(g.nl) * nchunk * 68);  // [nrow][kMsMaxP]
  for (int job = tid; job < g.nl * nchunk; job += kMsThreads) {
    const int a = job / nchunk, c = job - a * nchunk;
    const uint4* src = reinterpret_cast<const uint4*>(p.h + static_cast<int64_t>(g.plist[a]) * I + 32 * c);
    uint4 v[4], o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) v[j] = __ldcg(src + j);
    xs[job] = perm_block(v, o);
#pragma unroll
    for (int j = 0; j < 4; ++j) xh[(a * 4 + j) * nchunk + c] = o[j];
  }
  __syncthreads();
  const int myr = RT == 1 ? 0 : (lane >> (RT == 4 ? 3 : 4)) & (RT - 1);  // row whose sum this lane ends with
  for (; task < ntask; task += kMsWarps) {
    for (int a = g.gstart[gi]; a < g.gstart[gi + 1]; ++a) {  // every pair of this expert
      float vals[RT];
#pragma unroll
      for (int r = 0; r < RT; ++r) vals[r] = 0.f;
#pragma unroll
      for (int f = 0; f < F; ++f) {
        const int c = lane + 32 * f;
        uint4 x[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) x[j] = xh[(a * 4 + j) * nchunk + c];
        const float xsv = xs[a * nchunk + c];
#pragma unroll
        for (int r = 0; r < RT; ++r)
          if (r < rn) {
            uint32_t d[16];
            decode128(wq[r][f], d);
            vals[r] = fmaf(fmaf(-136.f, xsv, dot128(d, x)), bf16_bits_to_f32(sq[r][f]), vals[r]);
          }
      }
      if (lane < rn * L) {
        uint4 x[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) x[j] = xh[(a * 4 + j) * nchunk + lc];
        uint32_t d[16];
        decode128(wl, d);
        const float v = fmaf(-136.f, xs[a * nchunk + lc], dot128(d, x)) * bf16_bits_to_f32(sl);
#pragma unroll
        for (int r = 0; r < RT; ++r)
          if (r == lr) vals[r] += v;
      }
      const float v = warp_sum_rows<RT>(vals);
      if ((lane & (32 / RT - 1)) == 0 && myr < rn) {
        const float b = __bfloat162float(__float2bfloat16(v));
        const int q = g.plist[a];
        p.part[static_cast<int64_t>(q) * 1024 + n0 + r0 + myr] = b;
        pv[(r0 + myr) * kMsMaxP + q] = b;
      }
    }
    if (task + kMsWarps < ntask) issue(task + kMsWarps);
  }
  __syncthreads();
  // out[t, n] = bf16(sum over t's live pairs, k ascending, of w * part)
  for (int o = tid; o < p.R * nr; o += kMsThreads) {
    const int t = o / nr, r = o % nr;
    float acc = 0.f;
    for (int kk = 0; kk < p.topk; ++kk) {
      const int q = t * p.topk + kk;
      if (g.es[q] >= 0) acc = fmaf(ws[q], pv[r * kMsMaxP + q], acc);
    }
    if (p.out) p.out[static_cast<int64_t>(t) * 1024 + n0 + r] = __float2bfloat16(acc);
    if (p.out_partial) p.out_partial[static_cast<int64_t>(t) * 1024 + n0 + r] = acc;
  }
}

SmemOptIn g_fc1_smem;
SmemOptIn g_fc2_smem[9];

template <int F>
cudaError_t launch_fc2(const MsParams& p, size_t smem, const LaunchCfg& cfg) {
  auto kern = moe_stream_fc2_kernel<F>;
  const cudaError_t e = allow_smem(kern, smem, g_fc2_smem[F]);
  if (e != cudaSuccess) return e;
  return launch_kernel(kern, dim3((1024 + p.nrow - 1) / p.nrow), dim3(kMsThreads), smem, cfg, p);
}

constexpr size_t kSmemCap = 200 * 1024;  // dynamic bytes (static arrays and the driver's share stay below 227 KB)

}  // namespace

cudaError_t launch_moe_decode_stream(const bf16* z, const int* idx, const float* w, const uint8_t* fc1_w,
                                     const bf16* fc1_s, const uint8_t* fc2_w, const bf16* fc2_s, int R, int E, int I,
                                     int topk, int e_begin, int e_end, bf16* out, bf16* h, float* part,
                                     float* out_partial, const LaunchCfg& cfg) {
  const int P = R * topk;
  if (P < 1 || P > kMsMaxP || R > 16 || I < 32 || I % 32 || I > 8192) return cudaErrorNotSupported;
  // fc2 stages the h rows of every live pair: P rows of (I / 32) * 68 bytes
  const int nrow = (1024 + cfg.sms - 1) / cfg.sms;
  const size_t smem2 = static_cast<size_t>(P) * (I / 32) * 68 + static_cast<size_t>(nrow) * kMsMaxP * 4;
  if (smem2 > kSmemCap) return cudaErrorNotSupported;
  const auto al = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
  if (!al(z) || !al(fc1_w) || !al(fc2_w) || !al(h) || (reinterpret_cast<uintptr_t>(fc1_s) & 1) ||
      (reinterpret_cast<uintptr_t>(fc2_s) & 1))
    return cudaErrorNotSupported;
  MsParams p{z, idx, w, fc1_w, fc1_s, fc2_w, fc2_s, h, part, out, out_partial, nullptr, R, P, topk, E, I, e_begin, e_end,
             nrow};
  const size_t smem1 = static_cast<size_t>(R) * 2176;
  cudaError_t e = allow_smem(moe_stream_fc1_kernel, smem1, g_fc1_smem);
  if (e != cudaSuccess) return e;
  e = launch_kernel(moe_stream_fc1_kernel, dim3(cfg.sms), dim3(kMsThreads), smem1, cfg, p);
  if (e != cudaSuccess) return e;
  LaunchCfg c2 = cfg;
  c2.pdl = true;  // same op: fc2 loads its weights, then waits for fc1 before it reads h
  switch ((I / 32) / 32) {
    case 0: return launch_fc2<0>(p, smem2, c2);
    case 1: return launch_fc2<1>(p, smem2, c2);
    case 2: return launch_fc2<2>(p, smem2, c2);
    case 3: return launch_fc2<3>(p, smem2, c2);
    case 4: return launch_fc2<4>(p, smem2, c2);
    case 5: return launch_fc2<5>(p, smem2, c2);
    case 6: return launch_fc2<6>(p, smem2, c2);
    case 7: return launch_fc2<7>(p, smem2, c2);
    default: return launch_fc2<8>(p, smem2, c2);
  }
}

}  // namespace bolt
