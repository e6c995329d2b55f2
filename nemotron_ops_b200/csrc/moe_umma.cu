// MoeVerify expert GEMMs on the 5th-generation tensor cores (tcgen05.mma, accumulators and the
// weight operand in tensor memory).  Reference: MoeMmaKernel src/bolt_ops.cu:1115-1167 (mma
// weight contract: weights rounded to bf16 once, fp32 accumulation).
//
// Work: the flat list of (unique expert, 128-row tile) items over the selected experts' rows,
// split evenly over one CTA per SM (as in moe_tc.cu).  Per tile the CTA computes
// D[128 rows, 16 cols] = A[128 rows, K] * B[16 cols, K]^T with
//   * A: the expert's weight rows, decoded to bf16 by 16 decode warps straight into tensor
//     memory (tcgen05.st): thread (warp w, lane l) owns row 32 * (w & 3) + l -- the tensor
//     memory lane it may address; warps 0-7 decode the even 256-element K steps and warps 8-15
//     the odd ones, each warp half of a step; its 16-byte shared-memory reads of a 128- or
//     64-byte-swizzled stage are bank-conflict-free;
//   * B: the group's 8 activation rows (fc1: z; fc2: the h rows of the expert's pairs) in
//     shared memory, K-major core matrices (8 rows x 16 bytes) without swizzle; the descriptor's
//     8-row-group stride is 0, so columns 8..15 repeat columns 0..7 (N = 16 is the smallest
//     N for M = 128);
//   * D: fp32 in tensor memory, double-buffered so the epilogue of one tile (tcgen05.ld; fc1:
//     bf16 rounding, relu^2; fc2: fp32 partial sums) overlaps the MMAs of the next.
// fc2 has 8 tiles per expert, few against 148 CTAs (40 experts: two or three tiles a CTA), so
// its (tile, K segment) stages are divided evenly instead of its tiles: a tile may be split
// between two CTAs at a stage boundary.  fc1 zeroes part_out; fc2 stores the fp32 sums of whole
// tiles and adds (red.global.add) those of split ones -- with two addends on a zero the result
// is a + b whichever lands first, so it stays deterministic.  The finalize kernel rounds the
// per-pair outputs to bf16 (the contract's rounding of the fc2 output).
// One elected thread issues the MMAs (16 per 256-element K step) as soon as the decode warps
// have filled an A slot (three slots of 128 columns rotate); tcgen05.commit releases A slots,
// completes D buffers and frees activation buffers through mbarriers.  The K reduction happens in
// the accumulator: no cross-warp reduction, no per-tile CTA barrier.
//
// Decoded A values follow the mma contract: int4 bf16((n - 8) * s), native IQ2_XXS
// +-bf16(mag * bf16(d * (0.5 + s4) * 0.25)).  Within each group of 8 K elements the int4 decoder
// emits the order (0, 4, 1, 5, 2, 6, 3, 7) (one mask per pair); the activation rows are permuted
// the same way when they are laid out as core matrices, so the products pair up unchanged.
#include <algorithm>
#include <cstring>

#include "mma_decode.cuh"

namespace bolt {

namespace {

constexpr int kDecW = 16;                   // decode warps: 4 per tensor-memory lane quarter
constexpr int kParts = kDecW / 4;           // accumulator columns are drained in kParts parts
// The decode warps form two groups of 8 that take alternate K steps (each warp decodes half a
// step for its 32 rows), so one group's waits (stage, A slot, tensor-memory stores) overlap the
// other group's arithmetic instead of idling the SM.
constexpr int kGroups = 2;
constexpr int kGroupW = kDecW / kGroups;    // warps per group: 2 per lane quarter
constexpr int kDParts = kGroupW / 4;        // K parts of a K step within a group
constexpr int kProdW = kDecW;               // TMA producer warp
constexpr int kMmaW = kDecW + 1;            // MMA-issuing warp (also owns the tensor memory)
constexpr int kUThreads = (kDecW + 2) * 32;
constexpr int kTileRows = 128;              // UMMA M
constexpr int kKStep = 256;                 // K elements per A slot / per weight piece
constexpr int kASlots = 3;
constexpr int kUSlots = 8;
constexpr int kMaxXPieces = 3072 / (kDecW * 32);  // activation pieces per decode thread (K <= 3072)
constexpr uint32_t kTmemCols = 512;
__device__ __forceinline__ uint32_t d_col(int b) { return static_cast<uint32_t>(b) * 32u; }
__device__ __forceinline__ uint32_t a_col(int a) { return 128u + static_cast<uint32_t>(a) * 128u; }

// tcgen05.mma kind::f16 instruction descriptor: fp32 D, bf16 A and B, both K-major, M = 128, N = 16
constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) | ((16u >> 3) << 17) | ((128u >> 4) << 24);

struct UmmaParams {
  const bf16* x;        // fc1: z [R, K]; fc2: h [P, K]
  const int* idx;       // expert id of each (token, k) pair [P]; pair p is token p / topk
  int topk, e_begin;    // pairs whose expert is outside [e_begin, e_end) are not computed
  int* meta_out;        // fc1: CTA 0 writes the op's meta output here (null: written elsewhere)
  const uint8_t* w;     // expert rows [E * rows_pg, row_bytes]
  const uint8_t* sc;    // [E * rows_pg, sc_row_bytes]
  bf16* h_out;          // fc1 output [P, rows_pg]
  float* part_out;      // fc2: fp32 output [P, rows_pg]; fc1: fc2's output [P, zero_cols] (or null)
  int zero_cols;        // fc1: zeroes the part_out rows of the listed pairs, zero_cols floats each
  int split;            // fc2: part_out starts zeroed, so a tile may be split between two CTAs
  int P, R, K, rows_pg, e_end;
  int x_once;           // fc1: the activation rows are the same for every group
  int nxb;              // activation buffers (2 where they fit)
  int kseg;             // stages per tile
  int sp;               // weight pieces (= K steps) per stage
  int nslot, nsbuf;     // weight stage slots, per-tile scale buffers
  int pb;               // weight piece bytes (128 int4, 64 IQ2_XXS)
  int sc_rb;            // scale row bytes; a tile's scale rows are one contiguous span
  uint32_t w_bytes, w_stride, sc_bytes, xs_bytes, sc_off, xs_off;
};

__device__ __forceinline__ int ldcg_i(const int* p) {
  int v;
  asm volatile("ld.global.cg.s32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}
// The call's groups -- one per selected expert, in first-occurrence order over the pairs, each
// with the pair of every token row (or -1) -- built by every CTA in shared memory from idx (the
// layout of the op's meta output: src/bolt_ops.cu:1084-1112).
constexpr int kMaxPairs = 128;
struct GroupList {
  int n;                              // groups (unique local experts)
  int exp[kMaxPairs];                 // expert of group g
  signed char pair[kMaxPairs * 8];    // pair of (group g, token row j), -1 for none
  int idx[kMaxPairs];                 // (build scratch) the pairs' expert ids
  int rank[kMaxPairs];                // (build scratch) group of a first-occurrence pair
  int wtot[kMaxPairs / 32];           // (build scratch) first occurrences per warp
};

// All threads of the CTA; ends with a CTA barrier.  idx is read at L2 (fc2 reads it before its
// dependency wait: fc1 triggers fc2 only after its own wait, so idx is final by then).
__device__ void build_group_list(const UmmaParams& p, GroupList& gl) {
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  for (int i = t; i < 8 * p.P; i += blockDim.x) gl.pair[i] = -1;
  const int e = t < p.P ? __ldcg(p.idx + t) : -1;
  if (t < p.P) gl.idx[t] = e;
  __syncthreads();
  const bool local = t < p.P && e >= p.e_begin && e < p.e_end;
  int first = -1;
  if (local)
    for (int j = 0; j <= t; ++j)
      if (gl.idx[j] == e) {
        first = j;
        break;
      }
  const bool lead = local && first == t;
  const unsigned bal = __ballot_sync(0xffffffffu, lead);
  if (warp < kMaxPairs / 32 && lane == 0) gl.wtot[warp] = __popc(bal);
  __syncthreads();
  if (lead) {
    int off = 0;
    for (int w = 0; w < warp; ++w) off += gl.wtot[w];
    const int g = off + __popc(bal & ((1u << lane) - 1u));
    gl.rank[t] = g;
    gl.exp[g] = e;
  }
  if (t == 0) {
    int u = 0;
    for (int w = 0; w < kMaxPairs / 32; ++w) u += gl.wtot[w];
    gl.n = u;
  }
  __syncthreads();
  if (local) gl.pair[gl.rank[first] * 8 + t / p.topk] = static_cast<signed char>(t);
  __syncthreads();
}

__device__ __forceinline__ int group_expert(const GroupList& gl, int g) { return gl.exp[g]; }
__device__ __forceinline__ int column_pair(const GroupList& gl, int g, int j) { return gl.pair[8 * g + j]; }
template <int FC>
__device__ __forceinline__ int column_xrow(const UmmaParams& p, const GroupList& gl, int g, int j) {
  if (FC == 1) return j < p.R ? j : -1;
  return column_pair(gl, g, j);
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
// MMA and commit are issued by the whole (converged) MMA warp with warp-uniform operands and one
// elected lane: the operands then live in uniform registers, which keeps the issue cost near
// 20 ns per MMA (a single lane of a diverged warp computing descriptors took 37-75 ns, measured)
__device__ __forceinline__ void tc_commit(uint32_t bar) {
  asm volatile(
      "{\n .reg .pred e;\n elect.sync _|e, 0xffffffff;\n"
      " @e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n}\n" ::"r"(bar)
      : "memory");
}
// The 16 MMAs of one 256-element K step under a single election: MMA s reads A columns a + 8 s
// (16 bf16 per lane) and B core matrices 2 s, 2 s + 1 (descriptor start + 16 in 16-byte units);
// the first accumulates into D only when `accumulate` is set, the others always do.  The warp
// issuing them shares its scheduler with decode warps, so each MMA costs three instructions.
#define BOLT_MMA_NEXT                        \
  " add.u32 a, a, 8;\n add.u64 b, b, 16;\n" \
  " @e tcgen05.mma.cta_group::1.kind::f16 [%0], [a], b, %3, t;\n"
__device__ __forceinline__ void tc_mma_kstep(uint32_t d, uint32_t a, uint64_t bdesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p, t, e;\n .reg .b32 a;\n .reg .b64 b;\n"
      " setp.ne.b32 p, %4, 0;\n setp.ne.b32 t, %3, 0;\n mov.b32 a, %1;\n mov.b64 b, %2;\n"
      " elect.sync _|e, 0xffffffff;\n"
      " @e tcgen05.mma.cta_group::1.kind::f16 [%0], [a], b, %3, p;\n"
      BOLT_MMA_NEXT BOLT_MMA_NEXT BOLT_MMA_NEXT BOLT_MMA_NEXT BOLT_MMA_NEXT BOLT_MMA_NEXT BOLT_MMA_NEXT
      BOLT_MMA_NEXT BOLT_MMA_NEXT BOLT_MMA_NEXT BOLT_MMA_NEXT BOLT_MMA_NEXT BOLT_MMA_NEXT BOLT_MMA_NEXT
      BOLT_MMA_NEXT "}\n" ::"r"(d),
      "r"(a), "l"(bdesc), "r"(kIdesc), "r"(accumulate)
      : "memory");
}
#undef BOLT_MMA_NEXT
__device__ __forceinline__ void tc_st16(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}
template <int N>
__device__ __forceinline__ void tc_ld(uint32_t taddr, uint32_t (&v)[N]) {
  static_assert(N == 2 || N == 4, "tc_ld: 2 or 4 columns");
  if constexpr (N == 4)
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3])
                 : "r"(taddr)
                 : "memory");
  else
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x2.b32 {%0, %1}, [%2];" : "=r"(v[0]), "=r"(v[1]) : "r"(taddr) : "memory");
}
// shared-memory matrix descriptor: K-major, no swizzle, 8x16-byte core matrices, adjacent K core
// matrices 128 bytes apart, 8-row groups 0 bytes apart (rows 8..15 repeat rows 0..7)
__device__ __forceinline__ uint64_t b_desc(uint32_t saddr) {
  return static_cast<uint64_t>((saddr >> 4) & 0x3FFFu) | (static_cast<uint64_t>(128u >> 4) << 16) |
         (static_cast<uint64_t>(1) << 46);
}

// int4 (zero point 8), mma contract: 32 elements of one row (16 bytes) with one bf16 scale ->
// 16 bf16x2 in the order (0,4)(1,5)(2,6)(3,7) per 8 elements
__device__ __forceinline__ void decode_q4_32(const uint4 v, uint32_t s16, uint32_t (&o)[16]) {
  const __nv_bfloat162 s2 = bits_bf2(s16 | (s16 << 16));
  const __nv_bfloat162 zp = bits_bf2(0x43084308u);  // 136, 136
  const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int s = 0; s < 4; ++s) {
      const uint32_t a = ((w4[i] >> (4 * s)) & 0x000F000Fu) | 0x43004300u;  // 128 + n, exact
      o[4 * i + s] = bf2_bits(__hmul2(__hsub2(bits_bf2(a), zp), s2));
    }
}

// native IQ2_XXS, one 8-byte record (32 elements: 4 grid indices, 4 x 7 sign bits + 4-bit scale)
__device__ __forceinline__ void decode_iq2n_32(uint32_t idx4, uint32_t sg, float d, const uint32_t* grid,
                                               uint32_t (&o)[16]) {
  const float db = d * (0.5f + static_cast<float>(sg >> 28)) * 0.25f;
  const __nv_bfloat162 s2 = __bfloat162bfloat162(__float2bfloat16_rn(db));
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    const uint32_t ix = (idx4 >> (8 * g)) & 0xFFu;
    uint32_t pat = (sg >> (7 * g)) & 127u;
    pat |= (__popc(pat) & 1u) << 7;
    const uint4 ge = *reinterpret_cast<const uint4*>(grid + 4 * ix);
    const uint32_t gw[4] = {ge.x, ge.y, ge.z, ge.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) o[4 * g + j] = bf2_bits(__hmul2(bits_bf2(gw[j] ^ iq2_sign_mask(pat, j)), s2));
  }
}

template <int FMT>
__device__ __forceinline__ uint4 x_piece_order(uint4 v) {
  if constexpr (FMT == kFmtQ4) {  // (0,1)(2,3)(4,5)(6,7) -> (0,4)(1,5)(2,6)(3,7)
    return make_uint4(prmt(v.x, v.z, 0x5410), prmt(v.x, v.z, 0x7632), prmt(v.y, v.w, 0x5410),
                      prmt(v.y, v.w, 0x7632));
  } else {
    return v;
  }
}

template <int FC>
__device__ __forceinline__ void issue_x(const UmmaParams& p, const GroupList& gl, uint8_t* xs, uint64_t* x_bar, int g,
                                        int buf) {
  uint32_t tx = 0;
  for (int j = 0; j < 8; ++j)
    if (column_xrow<FC>(p, gl, g, j) >= 0) tx += static_cast<uint32_t>(p.K) * 2u;
  const uint32_t xb = smem_u32(&x_bar[buf]);
  mbar_arrive_expect_tx(xb, tx);
  for (int j = 0; j < 8; ++j) {
    const int xr = column_xrow<FC>(p, gl, g, j);
    if (xr >= 0)
      bulk_g2s(smem_u32(xs + static_cast<size_t>(buf) * p.xs_bytes + static_cast<size_t>(j) * p.K * 2),
               p.x + static_cast<int64_t>(xr) * p.K, static_cast<uint32_t>(p.K) * 2u, xb);
  }
}

// one weight stage (slot s, K segment q of the tile whose first physical row is prow; the tile's
// scales go to scale buffer sb with the first segment this CTA reads of it, `scales`)
__device__ __forceinline__ void issue_stage(const CUtensorMap* tmw, const UmmaParams& p, uint8_t* smem,
                                            uint64_t* full_bar, int s, int q, bool scales, int sb, int prow) {
  const uint32_t fb = smem_u32(&full_bar[s]);
  uint32_t tx = p.w_bytes;
  if (scales) {  // the tile's scales (one contiguous span, one bulk copy) ride on its first stage
    uint8_t* sdst = smem + p.sc_off + static_cast<size_t>(sb) * p.sc_bytes;
    const int64_t srb = p.sc_rb;
    stage_span(sdst, p.sc + static_cast<int64_t>(prow) * srb, static_cast<uint32_t>(kTileRows * srb),
               p.sc + static_cast<int64_t>(p.e_end) * p.rows_pg * srb, fb, tx);
  }
  tma_load_3d(smem_u32(smem + static_cast<size_t>(s) * p.w_stride), tmw, 0, prow, q * p.sp, fb);
  mbar_arrive_expect_tx(fb, tx);
}

template <int FMT, int FC>
__global__ void __launch_bounds__(kUThreads, 1)
    moe_umma_kernel(const __grid_constant__ CUtensorMap tmw, const UmmaParams p) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  __shared__ uint64_t full_bar[kUSlots], empty_bar[kUSlots];
  __shared__ uint64_t x_bar[2], xr_bar[2], xf_bar[2];
  __shared__ uint64_t af_bar[kASlots], ae_bar[kASlots], df_bar[2], de_bar[2], done_bar;
  __shared__ __align__(16) uint32_t grid_s[(FMT == kFmtIq2N) ? 1024 : 4];
  __shared__ int cols_s[3][8];
  __shared__ GroupList gl;
  __shared__ uint32_t tmem_base;
  __shared__ volatile int abort_flag;
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int KS = p.kseg, NS = p.nslot;
  const int tpg = p.rows_pg / kTileRows;
  uint8_t* xs = smem + p.xs_off;
  if ((smem_u32(smem) & 1023u) != 0u || smem - smem_raw > 1023) {
    if (tid == 0) set_status(kStatusSmemAlign);
    return;
  }
  if (tid == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(smem_u32(&full_bar[s]), 1);
      mbar_init(smem_u32(&empty_bar[s]), kDecW);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_u32(&x_bar[b]), 1);
      mbar_init(smem_u32(&xr_bar[b]), kDecW);
      mbar_init(smem_u32(&xf_bar[b]), 1);
      mbar_init(smem_u32(&df_bar[b]), 1);
      mbar_init(smem_u32(&de_bar[b]), kDecW);
    }
    for (int a = 0; a < kASlots; ++a) {
      mbar_init(smem_u32(&af_bar[a]), kGroupW);
      mbar_init(smem_u32(&ae_bar[a]), 1);
    }
    mbar_init(smem_u32(&done_bar), 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  if constexpr (FMT == kFmtIq2N) {
    for (int i = tid; i < 1024; i += kUThreads) grid_s[i] = kIq2xxsGridBf16x2[i];
  }
  if (warp == kMmaW) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tb = tmem_base;
  if constexpr (FC == 1) {
    pdl_wait();  // idx is the previous kernel's output
    pdl_trigger();
  } else {
    pdl_trigger();
  }
  build_group_list(p, gl);
  const int ngroups = gl.n;
  if constexpr (FC == 1) {
    // fc2's output rows of the listed pairs start at zero (this CTA's share of the 8 slots per
    // group; other rows stay untouched; fc2 adds into them only after this grid completes)
    if (p.part_out != nullptr) {
      const int nslots = 8 * ngroups;
      const int c4 = p.zero_cols >> 2;
      for (int j = static_cast<int>(static_cast<int64_t>(blockIdx.x) * nslots / gridDim.x),
               j1 = static_cast<int>(static_cast<int64_t>(blockIdx.x + 1) * nslots / gridDim.x);
           j < j1; ++j) {
        const int pp = gl.pair[j];
        if (pp < 0) continue;
        float4* row = reinterpret_cast<float4*>(p.part_out + static_cast<int64_t>(pp) * p.zero_cols);
        for (int i = tid; i < c4; i += kUThreads) row[i] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
    // the op's meta output: [0] = groups, [1 + g] = expert (-1 past the groups), then the pairs
    if (p.meta_out != nullptr && blockIdx.x == 0) {
      for (int i = tid; i < 1 + 9 * p.P; i += kUThreads) {
        int v;
        if (i == 0) v = ngroups;
        else if (i <= p.P) v = i - 1 < ngroups ? gl.exp[i - 1] : -1;
        else v = gl.pair[i - 1 - p.P];
        p.meta_out[i] = v;
      }
    }
  }
  const int64_t T = static_cast<int64_t>(ngroups) * tpg;
  // This CTA's work: tiles [t0, t0 + ntl), K segments [seg_lo(ti), seg_hi(ti)) of tile ti.  fc2
  // divides the flat list of (tile, K segment) stages evenly when there are at least as many tiles
  // as CTAs, so every CTA takes at least one tile's worth and a tile is shared by at most two
  // consecutive CTAs; fc1 (and fc2 with fewer tiles than CTAs) divides whole tiles.
  int t0, ntl, q_first = 0, q_end = KS, nstages;
  if (FC == 2 && p.split && T >= gridDim.x) {
    const int64_t W = T * KS;
    const int64_t f0 = static_cast<int64_t>(blockIdx.x) * W / gridDim.x;
    const int64_t f1 = static_cast<int64_t>(blockIdx.x + 1) * W / gridDim.x;
    t0 = static_cast<int>(f0 / KS);
    q_first = static_cast<int>(f0 % KS);
    ntl = static_cast<int>((f1 - 1) / KS) - t0 + 1;
    q_end = static_cast<int>((f1 - 1) % KS) + 1;
    nstages = static_cast<int>(f1 - f0);
  } else {
    t0 = static_cast<int>(static_cast<int64_t>(blockIdx.x) * T / gridDim.x);
    ntl = static_cast<int>(static_cast<int64_t>(blockIdx.x + 1) * T / gridDim.x) - t0;
    nstages = ntl * KS;
  }
  const int g0 = ntl > 0 ? t0 / tpg : 0;
  auto seg_lo = [&](int ti) { return ti == 0 ? q_first : 0; };
  auto seg_hi = [&](int ti) { return ti == ntl - 1 ? q_end : KS; };

  if (warp == kProdW) {
    // ------------------------------------------------------------------ TMA producer
    // The producer shares its scheduler with decode warps that keep it busy, so its loop keeps
    // running counters instead of dividing (each of its instructions waits for an issue slot).
    if (lane == 0 && ntl > 0) {
      prefetch_tensor_map(&tmw);
      // a scale buffer per tile in flight
      const int first = min(min(NS, nstages), p.nsbuf * KS - q_first);
      // stage cursor: slot s (use `round`), K segment q of tile ti (tile tig of group g), scale buffer sb
      int s = 0, round = 0, q = q_first, ti = 0, tig = t0 - g0 * tpg, g = g0, sb = 0;
      int cur_e = group_expert(gl, g0);
      int prow = cur_e * p.rows_pg + tig * kTileRows;
      auto advance = [&]() {
        if (++s == NS) s = 0, ++round;
        if (++q == KS) {
          q = 0;
          ++ti;
          if (++sb == p.nsbuf) sb = 0;
          if (++tig == tpg) {
            tig = 0;
            ++g;
            if (ti < ntl) cur_e = group_expert(gl, g);
          }
          prow = cur_e * p.rows_pg + tig * kTileRows;
        }
      };
      int st = 0;
      for (; st < first; ++st) {
        issue_stage(&tmw, p, smem, full_bar, s, q, q == seg_lo(ti), sb, prow);
        advance();
      }
      pdl_wait();  // activations (z, or h of fc1) are ready
      issue_x<FC>(p, gl, xs, x_bar, g0, 0);
      int xk = 0;  // ordinal of the last group whose activations were issued
      bool okw = true;
      int issued = first;
      // activations of every group up to gmax: group kn goes to buffer kn % nxb once the MMAs of
      // group kn - nxb have completed
      auto issue_x_upto = [&](int gmax) {
        while (okw && !p.x_once && xk < gmax - g0) {
          const int kn = xk + 1;
          if (kn >= p.nxb && !abort_flag)
            okw = mbar_wait(smem_u32(&xf_bar[kn % p.nxb]), ((kn / p.nxb) - 1) & 1, kStatusEmptyWait);
          if (okw && !abort_flag) {
            issue_x<FC>(p, gl, xs, x_bar, g0 + kn, kn % p.nxb);
            xk = kn;
          }
          if (abort_flag) okw = false;
        }
      };
      for (; st < nstages; ++st) {
        issue_x_upto(g);
        if (okw) okw = mbar_wait(smem_u32(&empty_bar[s]), (round - 1) & 1, kStatusEmptyWait);
        if (okw && q == 0 && ti >= p.nsbuf) {  // scale buffer of tile ti - nsbuf released
          const int last = (ti - p.nsbuf + 1) * KS - q_first - 1;  // its last stage
          if (last > st - NS) okw = mbar_wait(smem_u32(&empty_bar[last % NS]), (last / NS) & 1, kStatusEmptyWait);
        }
        if (!okw) abort_flag = 1;
        if (abort_flag) break;
        issue_stage(&tmw, p, smem, full_bar, s, q, q == seg_lo(ti), sb, prow);
        ++issued;
        advance();
      }
      issue_x_upto(g0 + (t0 + ntl - 1 - g0 * tpg) / tpg);  // groups whose stages all went out up front
      // no copy may still be landing when the CTA exits
      for (int b = 0; b <= min(xk, p.x_once ? 0 : p.nxb - 1); ++b) {
        const int k = xk - b;
        mbar_wait(smem_u32(&x_bar[k % p.nxb]), (k / p.nxb) & 1, kStatusDrainWait);
      }
      for (int st = max(0, issued - NS); st < issued; ++st)
        mbar_wait(smem_u32(&full_bar[st % NS]), (st / NS) & 1, kStatusDrainWait);
    }
  } else if (warp == kMmaW) {
    // ------------------------------------------------------------------ MMA issuer (whole warp)
    if (ntl > 0) {
      int ka = 0, gg = g0, tig = t0 - g0 * tpg;
      bool ok = true;
      for (int ti = 0; ti < ntl && ok; ++ti) {
        const int kg = gg - g0;
        const int xb = p.x_once ? 0 : kg % p.nxb;
        const int b = ti & 1;
        if (ti == 0 || (tig == 0 && !p.x_once))
          ok = mbar_wait(smem_u32(&xr_bar[xb]), (p.x_once ? 0 : kg / p.nxb) & 1, kStatusFullWait);
        if (ok && ti >= 2) ok = mbar_wait(smem_u32(&de_bar[b]), ((ti - 2) >> 1) & 1, kStatusFullWait);
        ok = __all_sync(0xffffffffu, ok);
        const uint64_t xdesc = b_desc(smem_u32(xs + static_cast<size_t>(xb) * p.xs_bytes));
        const int ks_lo = seg_lo(ti) * p.sp, ks_hi = seg_hi(ti) * p.sp;
        for (int ks = ks_lo; ks < ks_hi && ok; ++ks) {
          const int a = ka % kASlots;
          ok = !abort_flag && mbar_wait(smem_u32(&af_bar[a]), (ka / kASlots) & 1, kStatusFullWait);
          ok = __all_sync(0xffffffffu, ok);
          if (!ok) break;
          tc_fence_after();
          // K step ks starts at core matrix 32 * ks (128 bytes each, 8 in the descriptor's units)
          const uint64_t kdesc = xdesc + static_cast<uint64_t>(32 * ks) * 8u;
          const uint32_t dd = tb + d_col(b), aa = tb + a_col(a);
          static_assert(kKStep == 16 * 16, "tc_mma_kstep issues 16 MMAs of K = 16");
          tc_mma_kstep(dd, aa, kdesc, ks != ks_lo ? 1u : 0u);
          tc_commit(smem_u32(&ae_bar[a]));
          ++ka;
        }
        if (!ok) break;
        tc_commit(smem_u32(&df_bar[b]));
        if (!p.x_once && (tig == tpg - 1 || ti == ntl - 1)) tc_commit(smem_u32(&xf_bar[xb]));
        if (++tig == tpg) tig = 0, ++gg;
      }
      if (!ok) abort_flag = 1;
      // every MMA issued by this warp has completed before the tensor memory is released
      tc_commit(smem_u32(&done_bar));
      mbar_wait(smem_u32(&done_bar), 0, kStatusDrainWait);
    }
  } else {
    // ------------------------------------------------------------------ decode warps
    const int q4 = warp & 3, hh = warp >> 2;  // lane quarter, accumulator part
    const int grp = warp / kGroupW, hd = (warp >> 2) % kDParts;  // K-step group, K part within a step
    const int r = 32 * q4 + lane;             // tile row = tensor memory lane
    const uint32_t lane_off = static_cast<uint32_t>(32 * q4) << 16;
    const int sc_rb = static_cast<int>(fmt_scale_row_bytes(FMT, p.K));
    bool ok = true;
    int s = 0;
    uint32_t ph = 0;
    int ka = 0, gg = g0, tig = t0 - g0 * tpg, sbuf = 0;
    uint32_t sc_mis = 0;
    // tile whose epilogue is pending: its row, column slot and whether its sums cover all of K
    int pend_ti = -1, pend_row0 = 0, pend_cols = 0;
    bool pend_whole = true;

    auto epilogue = [&](int tj, int row0, int cslot, bool whole) {
      const int b = tj & 1;
      constexpr int kCols = 8 / kParts;  // token columns drained by this warp
      uint32_t v[kCols];
#pragma unroll
      for (int c = 0; c < kCols; ++c) v[c] = 0u;
      bool good = ok && !abort_flag;
      if (good) good = mbar_wait(smem_u32(&df_bar[b]), (tj >> 1) & 1, kStatusFullWait);
      good = __all_sync(0xffffffffu, good);
      if (!good) {
        ok = false;
        abort_flag = 1;
      } else {
        tc_fence_after();
        tc_ld<kCols>(tb + lane_off + d_col(b) + kCols * hh, v);
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&de_bar[b]));
      if (good) {
#pragma unroll
        for (int c = 0; c < kCols; ++c) {
          const int pr = cols_s[cslot][kCols * hh + c];
          if (pr < 0) continue;
          const int64_t oi = static_cast<int64_t>(pr) * p.rows_pg + row0 + r;
          if constexpr (FC == 1) {
            const float rr = fmaxf(__bfloat162float(__float2bfloat16(__uint_as_float(v[c]))), 0.f);
            p.h_out[oi] = __float2bfloat16(rr * rr);  // rr * rr is exact in fp32
          } else {
            // fp32 sums (the finalize kernel rounds them); a split tile's two K ranges add up
            if (whole) p.part_out[oi] = __uint_as_float(v[c]);
            else atomicAdd(p.part_out + oi, __uint_as_float(v[c]));
          }
        }
      }
    };

    for (int ti = 0; ti < ntl; ++ti) {
      const int kg = gg - g0;
      if (ti == 0 || tig == 0) {  // a new group: activations as core matrices, column pairs
        if (ti == 0 || !p.x_once) {
          const int xb = p.x_once ? 0 : kg % p.nxb;
          if (ok && !abort_flag &&
              !mbar_wait(smem_u32(&x_bar[xb]), (p.x_once ? 0 : kg / p.nxb) & 1, kStatusFullWait)) {
            ok = false;
            abort_flag = 1;
          }
          ok = __all_sync(0xffffffffu, ok);
          // rows are row-major (K * 2 bytes each); core matrix kb holds 16 bytes of each row
          uint8_t* xbuf = xs + static_cast<size_t>(xb) * p.xs_bytes;
          const int kp = p.K >> 3;  // 16-byte pieces per row
          uint4 v[kMaxXPieces];
#pragma unroll
          for (int i = 0; i < kMaxXPieces; ++i) {
            const int pi = tid + i * kDecW * 32;
            v[i] = (ok && pi < 8 * kp) ? x_piece_order<FMT>(lds128(xbuf + static_cast<size_t>(pi) * 16))
                                       : make_uint4(0u, 0u, 0u, 0u);
          }
          named_bar_sync(1, kDecW * 32);
#pragma unroll
          for (int i = 0; i < kMaxXPieces; ++i) {
            const int pi = tid + i * kDecW * 32;
            if (ok && pi < 8 * kp) {
              const int j = pi / kp, kb = pi - j * kp;
              *reinterpret_cast<uint4*>(xbuf + static_cast<size_t>(kb) * 128 + j * 16) = v[i];
            }
          }
          // generic-proxy writes -> visible to the tensor core's reads
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          __syncwarp();
          if (lane == 0) mbar_arrive(smem_u32(&xr_bar[xb]));
        }
        if (tid < 8) cols_s[kg % 3][tid] = column_pair(gl, gg, tid);
        if constexpr (FMT == kFmtIq2N)
          sc_mis = static_cast<uint32_t>(
              reinterpret_cast<uintptr_t>(p.sc + static_cast<int64_t>(group_expert(gl, gg)) * p.rows_pg * sc_rb) & 15);
        named_bar_sync(1, kDecW * 32);
      }
      const uint8_t* sct = smem + p.sc_off + static_cast<size_t>(sbuf) * p.sc_bytes + sc_mis;
      for (int q = seg_lo(ti); q < seg_hi(ti); ++q) {
        if (ok && abort_flag) ok = false;
        if (ok && !mbar_wait(smem_u32(&full_bar[s]), ph, kStatusFullWait)) {
          ok = false;
          abort_flag = 1;
        }
        ok = __all_sync(0xffffffffu, ok);  // the tensor-memory stores below are warp-collective
        const uint8_t* wst = smem + static_cast<size_t>(s) * p.w_stride;
        for (int kk = 0; kk < p.sp; ++kk) {
          const int ks = q * p.sp + kk;
          const int a = ka % kASlots;
          const bool mine = ka % kGroups == grp;  // this warp's group decodes K step ks
          // this thread's share of K step ks (weights, scales) goes to registers first; after the
          // stage's last step the slot returns to the producer, so decoding does not hold it
          constexpr int kU = FMT == kFmtQ4 ? 8 / kDParts : 4 / kDParts;  // 16-byte units
          uint4 wv[kU];
          uint32_t s4[kU];
          float d = 0.f;
          if (ok && mine) {
            if constexpr (FMT == kFmtQ4) {  // unit = 32 elements, one bf16 scale block each
              const uint8_t* wp = wst + static_cast<size_t>(kk) * kTileRows * 128 + r * 128;
              // (the host keeps int4 scale spans 16-byte aligned)
              const uint8_t* spt = sct + r * sc_rb + ks * 16 + hd * (2 * kU);
              if constexpr (kU == 4) {
                const uint2 sv = *reinterpret_cast<const uint2*>(spt);
                s4[0] = sv.x & 0xFFFFu, s4[1] = sv.x >> 16, s4[2] = sv.y & 0xFFFFu, s4[3] = sv.y >> 16;
              } else {
                const uint32_t sv = *reinterpret_cast<const uint32_t*>(spt);
                s4[0] = sv & 0xFFFFu, s4[1] = sv >> 16;
              }
#pragma unroll
              for (int i = 0; i < kU; ++i) wv[i] = lds128(wp + (((kU * hd + i) ^ (r & 7)) << 4));
            } else {  // unit = two 32-element records
              const uint8_t* wp = wst + static_cast<size_t>(kk) * kTileRows * 64 + r * 64;
              d = __half2float(__ushort_as_half(*reinterpret_cast<const uint16_t*>(sct + r * sc_rb + ks * 2)));
#pragma unroll
              for (int i = 0; i < kU; ++i) wv[i] = lds128(wp + (((kU * hd + i) ^ ((r >> 1) & 3)) << 4));
            }
          }
          if (kk == p.sp - 1) {  // the arrive releases (orders) the loads above
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&empty_bar[s]));
          }
          if (!mine) {
            ++ka;
            continue;
          }
          if (ok && abort_flag) ok = false;
          if (ok && ka >= kASlots && !mbar_wait(smem_u32(&ae_bar[a]), ((ka / kASlots) - 1) & 1, kStatusFullWait)) {
            ok = false;
            abort_flag = 1;
          }
          ok = __all_sync(0xffffffffu, ok);
          if (ok) {
            // this thread's part: K elements [hd, hd + 1) * 256 / kDParts of the step = columns
            // [hd, hd + 1) * 128 / kDParts of the A slot
            const uint32_t tcol = tb + lane_off + a_col(a) + (128u / kDParts) * hd;
            if constexpr (FMT == kFmtQ4) {
#pragma unroll
              for (int i = 0; i < kU; ++i) {
                uint32_t o[16];
                decode_q4_32(wv[i], s4[i], o);
                tc_st16(tcol + 16u * i, o);
              }
            } else {
#pragma unroll
              for (int i = 0; i < kU; ++i) {
                uint32_t o[16];
                decode_iq2n_32(wv[i].x, wv[i].y, d, grid_s, o);
                tc_st16(tcol + 32u * i, o);
                decode_iq2n_32(wv[i].z, wv[i].w, d, grid_s, o);
                tc_st16(tcol + 32u * i + 16u, o);
              }
            }
            asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(smem_u32(&af_bar[a]));
          ++ka;
        }
        if (++s == NS) s = 0, ph ^= 1u;
      }
      // the previous tile's accumulators are complete by now: drain them
      if (pend_ti >= 0) epilogue(pend_ti, pend_row0, pend_cols, pend_whole);
      pend_ti = ti;
      pend_row0 = tig * kTileRows;
      pend_cols = kg % 3;
      pend_whole = seg_lo(ti) == 0 && seg_hi(ti) == KS;
      if (++tig == tpg) tig = 0, ++gg;
      if (++sbuf == p.nsbuf) sbuf = 0;
    }
    if (pend_ti >= 0) epilogue(pend_ti, pend_row0, pend_cols, pend_whole);
  }
  // release the tensor memory once every MMA and every tensor-memory access has finished
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == kMmaW) {
    __syncwarp();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tb), "r"(kTmemCols));
  }
}

template <int FMT, int FC>
cudaError_t launch_umma(const CUtensorMap& tmw, const UmmaParams& p, size_t smem,
                        const LaunchCfg& cfg) {
  auto kern = moe_umma_kernel<FMT, FC>;
  static SmemOptIn opt;
  cudaError_t e = allow_smem(kern, smem, opt);
  if (e != cudaSuccess) return e;
  return launch_kernel(kern, dim3(cfg.sms), dim3(kUThreads), smem, cfg, tmw, p);
}

// Static shared memory of a kernel instance (the dynamic carve-out gets the rest of the 227 KB).
template <int FMT, int FC>
size_t umma_static_smem() {
  static const size_t bytes = [] {
    cudaFuncAttributes a{};
    return cudaFuncGetAttributes(&a, moe_umma_kernel<FMT, FC>) == cudaSuccess ? a.sharedSizeBytes : size_t(16384);
  }();
  return bytes;
}

}  // namespace

bool moe_layer_umma_ok(int fmt, const void* sc, int P, int K, int rows_pg) {
  if (fmt != kFmtQ4 && fmt != kFmtIq2N) return false;
  // the activation rows (8 x K / 8 pieces of 16 bytes) are permuted through registers
  if (rows_pg % kTileRows || K % kKStep || K > kMaxXPieces * kDecW * 32 || P > kMaxPairs || P < 1) return false;
  // int4 scales are read as 8-byte words: the span of every tile must start 16-byte aligned
  const int64_t srb = fmt_scale_row_bytes(fmt, K);
  return !(fmt == kFmtQ4 && (srb % 16 || (reinterpret_cast<uintptr_t>(sc) & 15)));
}

// One MoeVerify expert layer (fc1: K = 1024, rows_pg = I; fc2: K = I, rows_pg = 1024) on the
// tcgen05 path, over the pairs of idx whose expert is in [e_begin, e_end).  fc1 with part_out set
// zeroes the listed pairs' rows of part_out [P, 1024] (fc2's output), and with meta_out set
// writes the op's meta output; fc2 with split (those rows zeroed) divides its stages evenly,
// splitting tiles between CTAs.  cudaErrorNotSupported when moe_layer_umma_ok says no.
cudaError_t launch_moe_layer_umma(int fmt, int fc, const bf16* x, const int* idx, int topk, int e_begin, int* meta_out,
                                  const uint8_t* w, const void* sc, bf16* h_out, float* part_out, int P, int R, int E,
                                  int e_end, int K, int rows_pg, const LaunchCfg& cfg, int split) {
  if (!moe_layer_umma_ok(fmt, sc, P, K, rows_pg)) return cudaErrorNotSupported;
  UmmaParams p{};
  p.x = x;
  p.idx = idx;
  p.topk = topk;
  p.e_begin = e_begin;
  p.meta_out = fc == 1 ? meta_out : nullptr;
  p.w = w;
  p.sc = static_cast<const uint8_t*>(sc);
  p.h_out = h_out;
  p.part_out = part_out;
  // fc1 zeroes the listed pairs' rows of fc2's output [P, 1024] (16-byte aligned) so that fc2
  // may split tiles
  p.zero_cols = 1024;
  if (fc == 1 && part_out != nullptr && (reinterpret_cast<uintptr_t>(part_out) & 15)) return cudaErrorInvalidValue;
  p.split = fc == 2 ? split : 0;
  p.P = P;
  p.R = R;
  p.K = K;
  p.rows_pg = rows_pg;
  p.e_end = e_end;
  p.x_once = fc == 1 ? 1 : 0;
  const int64_t rb = fmt_row_bytes(fmt, K);
  const int64_t srb = fmt_scale_row_bytes(fmt, K);
  p.pb = fmt == kFmtQ4 ? 128 : 64;  // one 256-element K step per piece
  const int pieces = static_cast<int>(rb / p.pb);
  p.sc_rb = static_cast<int>(srb);
  // pieces per stage: the largest divisor of the row's pieces with a stage of <= 48 KB (each
  // tensor copy costs a fixed ~0.2-0.7 us to issue, more while the decode warps keep the SM busy)
  p.sp = 1;
  for (int c = 2; c <= pieces; ++c)
    if (pieces % c == 0 && static_cast<size_t>(c) * kTileRows * p.pb <= 48 * 1024) p.sp = c;
  p.kseg = pieces / p.sp;
  p.w_bytes = static_cast<uint32_t>(p.sp) * kTileRows * p.pb;
  p.w_stride = (p.w_bytes + 1023u) & ~1023u;
  p.sc_bytes = static_cast<uint32_t>((srb * kTileRows + 32 + 127) & ~int64_t(127));
  p.xs_bytes = (static_cast<uint32_t>(8 * K * 2) + 1023u) & ~1023u;
  const size_t static_smem = fmt == kFmtQ4 ? (fc == 1 ? umma_static_smem<kFmtQ4, 1>() : umma_static_smem<kFmtQ4, 2>())
                                           : (fc == 1 ? umma_static_smem<kFmtIq2N, 1>() : umma_static_smem<kFmtIq2N, 2>());
  const size_t smem_cap = 227 * 1024 - static_smem;  // dynamic bytes a CTA may have
  const size_t budget = std::min(cfg.smem_budget ? cfg.smem_budget : 220 * 1024, smem_cap - 1024);
  auto nsbuf_for = [](int ns, int kseg) { return std::min(4, (ns + kseg - 1) / kseg + 1); };
  // one or two activation buffers: whichever leaves more weight bytes in flight (ties: two, so
  // the next group's rows land while this group computes)
  int best_nxb = 0, best_ns = 0;
  for (int nxb = p.x_once ? 1 : 2; nxb >= 1; --nxb) {
    const size_t fixed = 1024 + static_cast<size_t>(nxb) * p.xs_bytes;
    for (int ns = kUSlots; ns >= 2; --ns) {
      if (fixed + static_cast<size_t>(ns) * p.w_stride + static_cast<size_t>(nsbuf_for(ns, p.kseg)) * p.sc_bytes <=
          budget) {
        if (ns > best_ns) best_nxb = nxb, best_ns = ns;
        break;
      }
    }
  }
  if (!best_ns) return cudaErrorNotSupported;
  p.nxb = best_nxb;
  p.nslot = best_ns;
  p.nsbuf = nsbuf_for(p.nslot, p.kseg);
  p.sc_off = static_cast<uint32_t>(p.nslot) * p.w_stride;
  p.xs_off = p.sc_off + static_cast<uint32_t>(p.nsbuf) * p.sc_bytes;
  p.xs_off = (p.xs_off + 1023u) & ~1023u;
  // at least 116 KB, so that one CTA holds the SM (the kernel allocates all 512 TMEM columns)
  const size_t smem = std::max<size_t>(1024 + p.xs_off + static_cast<size_t>(p.nxb) * p.xs_bytes, 116 * 1024);
  if (smem > smem_cap) return cudaErrorNotSupported;
  CUtensorMap tmw;
  if (!row_tile_map(&tmw, w, static_cast<int64_t>(E) * rows_pg, rb, p.sp, p.pb, kTileRows)) return cudaErrorNotSupported;
  if (fmt == kFmtQ4) return fc == 1 ? launch_umma<kFmtQ4, 1>(tmw, p, smem, cfg) : launch_umma<kFmtQ4, 2>(tmw, p, smem, cfg);
  return fc == 1 ? launch_umma<kFmtIq2N, 1>(tmw, p, smem, cfg) : launch_umma<kFmtIq2N, 2>(tmw, p, smem, cfg);
}

}  // namespace bolt
