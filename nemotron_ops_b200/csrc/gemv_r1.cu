// Nvfp4Gemv at R = 1: a streaming SIMT GEMV (the reference's R = 1 kernel is Nvfp4GemvKernel,
// src/bolt_ops.cu:663-736).  Arithmetic: each e2m1 weight times fp16(x * 2^-6) is formed exactly
// and summed in fp32 (mixed-precision fma.rn.f32.f16) over its 16-weight scale block, the block
// sum is multiplied by its e4m3 scale and accumulated in fp32; y = bf16(sum * g * 2^6).  (The
// reference sums the block in fp16; fp32 keeps outputs that cancel within the elementwise bound.)
//
// B200 design
//  * 16 warps per CTA, at most 64 registers per thread and ~90 KB of shared memory at K = 8192,
//    so two CTAs share an SM: with programmatic dependent launch the next call's CTA is resident
//    while this call computes.  A CTA owns N / grid consecutive rows and a warp the rows w,
//    w + 16, ... of it, one at a time;
//  * a warp stages its row into shared memory with cp.async, 512 contiguous bytes per copy
//    instruction (16 bytes per lane, 1024 k: whole 128-byte lines), plus the row's e4m3 scales,
//    computes it from there and issues the next row's copies before its reduction;
//  * a lane decodes its 32 e2m1 per row and chunk with one cvt.rn.f16x2.e2m1x2 per byte and runs
//    two fp32 chains per scale block; the activations sit in shared memory as fp16 * 2^-6, laid
//    out so that a warp's 16-byte reads are contiguous (conflict-free);
//  * programmatic dependent launch: weights and scales are read after griddepcontrol.wait (an
//    earlier kernel may write them); before it the CTA only pulls its rows into L2, which stays
//    coherent with such writes.  With early weights the first row's copies go before the wait.
//    After the wait the activations' loads go out first (every CTA reads the same lines, which
//    return last when queued behind the weight copies), and the dependents are released only
//    once the activations are staged: 6.64 -> 5.61 us per call at N = 4096, K = 8192.
// The file also holds the Q4Gemv int4 and IQ2_XXS R = 1 kernels on the same layout and schedule (below).
#include "mma_decode.cuh"

namespace bolt {

namespace {

constexpr int kR1Warps = 16;
constexpr int kR1Threads = kR1Warps * 32;
constexpr int kR1MaxChunks = 8;  // 1024-k chunks per row (K <= 8192)

struct R1Params {
  const bf16* x;
  const uint8_t* w;
  const uint8_t* sc;
  const float* gscale;
  bf16* y;
  int64_t N;
  int K;
  int early_weights;
};

__device__ __forceinline__ uint4 ldg_stream(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// a += lo(w) * lo(x), b += hi(w) * hi(x): fp16 products (exact here) added in fp32
__device__ __forceinline__ void fma2_f16_f32(uint32_t w, uint32_t x, float& a, float& b) {
  asm("{\n .reg .f16 wl, wh, xl, xh;\n mov.b32 {wl, wh}, %2;\n mov.b32 {xl, xh}, %3;\n"
      " fma.rn.f32.f16 %0, wl, xl, %0;\n fma.rn.f32.f16 %1, wh, xh, %1;\n}\n"
      : "+f"(a), "+f"(b)
      : "r"(w), "r"(x));
}

// sum of 16 e2m1 weights (8 bytes) times 16 fp16 activations (8 pairs), in fp32
__device__ __forceinline__ float block_dot(uint32_t w0, uint32_t w1, const uint32_t* xp) {
  uint32_t d[8];
  RawRow r;
  r.w = make_uint4(w0, w1, 0u, 0u);
  decode_row_raw<kFmtFp4>(r, d);
  float a = 0.f, b = 0.f;
#pragma unroll
  for (int j = 0; j < 8; ++j) fma2_f16_f32(d[j], xp[j], a, b);
  return a + b;
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

template <int KC>
__global__ void __launch_bounds__(kR1Threads, 2) gemv_nvfp4_r1_kernel(const R1Params p) {
  // [x as fp16 * 2^-6: K * 2 bytes][rows: warp][chunk][lane] 16 B][scales: warp][512 B]
  extern __shared__ __align__(16) uint8_t smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int K = p.K;
  const int64_t rb = K / 2, srb = K / 16;
  const int64_t r0 = static_cast<int64_t>(blockIdx.x) * p.N / gridDim.x;
  const int64_t r1 = static_cast<int64_t>(blockIdx.x + 1) * p.N / gridDim.x;
  uint8_t* rowb = smem + static_cast<size_t>(K) * 2 + static_cast<size_t>(warp) * KC * 512;
  uint8_t* ssl = smem + static_cast<size_t>(K) * 2 + static_cast<size_t>(kR1Warps) * KC * 512 + warp * 512;
  auto stage_row = [&](int64_t r) {  // row r's KC chunks and its scales -> this warp's buffers
    const uint8_t* wr = p.w + r * rb + 16 * lane;
#pragma unroll
    for (int i = 0; i < KC; ++i) cp_async16(rowb + i * 512 + 16 * lane, wr + 512 * i);
    if (16 * lane < srb) cp_async16(ssl + 16 * lane, p.sc + r * srb + 16 * lane);
    cp_async_commit();
  };
  int64_t r = r0 + warp;
  if (p.early_weights) {
    if (r < r1) stage_row(r);
  } else if (tid == 0) {  // the CTA's rows are contiguous: pull them into L2 during the previous kernel
    prefetch_span_l2(p.w + r0 * rb, static_cast<uint64_t>(r1 - r0) * rb);
    prefetch_span_l2(p.sc + r0 * srb, static_cast<uint64_t>(r1 - r0) * srb);
  }
  pdl_wait();
  // The activations' loads go out first (every CTA reads the same lines, so they are the slowest
  // to return when queued behind the weights), then the warp's first row.
  constexpr int XP = (KC * 128 + kR1Threads - 1) / kR1Threads;  // 16-byte pieces per thread
  uint4 xv[XP];
#pragma unroll
  for (int j = 0; j < XP; ++j) {
    const int q = tid + j * kR1Threads;
    if (q < K / 8) xv[j] = __ldcg(reinterpret_cast<const uint4*>(p.x) + q);
  }
  const float gsv = __ldcg(p.gscale) * 64.f;
  if (!p.early_weights && r < r1) stage_row(r);
  // activations -> fp16 * 2^-6; input piece q (8 k) goes to chunk q / 128, lane (q % 128) / 4, part q % 4
#pragma unroll
  for (int j = 0; j < XP; ++j) {
    const int q = tid + j * kR1Threads;
    if (q < K / 8) {
      const int i = q >> 7, l = (q & 127) >> 2, part = q & 3;
      *reinterpret_cast<uint4*>(smem + ((i * 4 + part) * 32 + l) * 16) = x_piece_to_frag<kFmtFp4>(xv[j]);
    }
  }
  __syncthreads();
  // The next call's CTAs may start only now: started at this kernel's entry, their prologues
  // delayed this CTA's activation loads, and the whole call, by ~1 us (measured).
  pdl_trigger();

  for (; r < r1; r += kR1Warps) {
    cp_async_wait_all();
    __syncwarp();  // the row's scales were copied by other lanes
    float acc = 0.f;
#pragma unroll
    for (int i = 0; i < KC; ++i) {
      uint32_t xf[16];
#pragma unroll
      for (int part = 0; part < 4; ++part) {
        const uint4 v = lds128(smem + ((i * 4 + part) * 32 + lane) * 16);
        xf[4 * part] = v.x;
        xf[4 * part + 1] = v.y;
        xf[4 * part + 2] = v.z;
        xf[4 * part + 3] = v.w;
      }
      const uint4 wq = lds128(rowb + i * 512 + 16 * lane);
      const float b0 = block_dot(wq.x, wq.y, xf);      // block 64 i + 2 lane
      const float b1 = block_dot(wq.z, wq.w, xf + 8);  // and the next one
      const uint32_t s8 = *reinterpret_cast<const uint16_t*>(ssl + 64 * i + 2 * lane);
      uint32_t s2;
      asm("{\n .reg .b16 t16;\n cvt.u16.u32 t16, %1;\n cvt.rn.f16x2.e4m3x2 %0, t16;\n}\n" : "=r"(s2) : "r"(s8));
      const float2 sc = __half22float2(bits_h2(s2));
      acc = fmaf(b0, sc.x, acc);
      acc = fmaf(b1, sc.y, acc);
    }
    __syncwarp();  // every lane is done with the buffers
    if (r + kR1Warps < r1) stage_row(r + kR1Warps);  // the warp's next row streams while it reduces
    const float a = warp_sum(acc);
    if (lane == 0) p.y[r] = __float2bfloat16(a * gsv);
  }
  cp_async_wait_all();  // nothing in flight into shared memory at exit
}

template <int KC>
cudaError_t launch_r1(const R1Params& p, int grid, const LaunchCfg& cfg) {
  const size_t smem = static_cast<size_t>(p.K) * 2 + static_cast<size_t>(kR1Warps) * (KC * 512 + 512);
  auto kern = gemv_nvfp4_r1_kernel<KC>;
  static SmemOptIn opt;
  cudaError_t e = allow_smem(kern, smem, opt);
  if (e != cudaSuccess) return e;
  return launch_kernel(kern, dim3(grid), dim3(kR1Threads), smem, cfg, p);
}


// ------------------------------------------------------------------------------------------
// Q4Gemv (int4, zero point 8) at R = 1, exact contract (the reference's R = 1 kernel is
// QGemvKernel, src/bolt_ops.cu:1315-1392): y = bf16(sum over blocks of s * sum (q - 8) x), fp32.
// Same layout: lane l takes 16 bytes (one 32-k block) per 1024-k chunk of each row; a lane
// decodes bf16(128 + q) pairs (a shift and a LOP3 per two weights), multiplies them by x with
// mixed-precision fma.rn.f32.bf16 (exact products, fp32 sums) and removes 136 * (the block's sum
// of x).  gemv_q4_r1_kernel stages a warp's rows through shared memory like the NVFP4 kernel
// (the C ABI hands it 16-byte aligned tensors only).
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t ldg_u16(const void* p) {
  unsigned short v;
  asm volatile("ld.global.nc.L1::no_allocate.u16 %0, [%1];" : "=h"(v) : "l"(p));
  return v;
}

// a += lo(q) * lo(x), b += hi(q) * hi(x) for bf16 pairs: exact products, fp32 sums
__device__ __forceinline__ void fma2_bf16_f32r(uint32_t q, uint32_t x, float& a, float& b) {
  asm("{\n .reg .b16 ql, qh, xl, xh;\n mov.b32 {ql, qh}, %2;\n mov.b32 {xl, xh}, %3;\n"
      " fma.rn.f32.bf16 %0, ql, xl, %0;\n fma.rn.f32.bf16 %1, qh, xh, %1;\n}\n"
      : "+f"(a), "+f"(b)
      : "r"(q), "r"(x));
}

// sum over one 16-byte int4 block of (128 + q) * x, x as four PERM pieces (x_piece_to_frag order)
__device__ __forceinline__ float q4_block_dot(const uint4& wq, const uint4 (&x)[4]) {
  const uint32_t wv[4] = {wq.x, wq.y, wq.z, wq.w};
  const uint32_t xv[16] = {x[0].x, x[0].y, x[0].z, x[0].w, x[1].x, x[1].y, x[1].z, x[1].w,
                           x[2].x, x[2].y, x[2].z, x[2].w, x[3].x, x[3].y, x[3].z, x[3].w};
  float a0 = 0.f, b0 = 0.f, a1 = 0.f, b1 = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int s = 0; s < 4; ++s) {
      const uint32_t d = ((wv[i] >> (4 * s)) & 0x000F000Fu) | 0x43004300u;  // bf16(128 + q), exact
      if (s & 1) fma2_bf16_f32r(d, xv[4 * i + s], a1, b1);
      else fma2_bf16_f32r(d, xv[4 * i + s], a0, b0);
    }
  return (a0 + b0) + (a1 + b1);
}

// lane l ends with the warp total of v[l >> (5 - log2 RB)] (same tree as a per-value warp sum)
template <int RB>
__device__ __forceinline__ float warp_sum_t(const float (&v)[RB]) {
  const int lane = threadIdx.x & 31;
  if constexpr (RB == 4) {
    float w[2];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const bool up = lane & 16;
      const float send = up ? v[i] : v[i + 2], keep = up ? v[i + 2] : v[i];
      w[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
    }
    const bool up = lane & 8;
    const float send = up ? w[0] : w[1], keep = up ? w[1] : w[0];
    float s = keep + __shfl_xor_sync(0xffffffffu, send, 8);
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    return s;
  } else {
    const bool up = lane & 16;
    const float send = up ? v[0] : v[1], keep = up ? v[1] : v[0];
    float s = keep + __shfl_xor_sync(0xffffffffu, send, 16);
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    return s;
  }
}

// Q4Gemv int4 at R = 1 with the rows staged through shared memory (the NVFP4 kernel's layout and
// schedule: rows copied per warp by cp.async, at most 64 registers, two CTAs per SM, the
// dependents released once the activations are staged).  A warp keeps a ring of D row slots
// (D = 2 while two CTAs still fit an SM): the next row streams in while it computes the current
// one (6.09 -> 5.95 us at K = 4096, N = 8192).  16-byte aligned scales.
template <int KC, int D>
__global__ void __launch_bounds__(kR1Threads, 2) gemv_q4_r1_kernel(const R1Params p) {
  // [x: PERM pieces [chunk][piece][lane], K * 2 bytes][block sums of x: K / 8 bytes]
  // [per warp: the row's KC chunks [chunk][lane] 16 B, then its K / 16 bytes of bf16 scales]
  extern __shared__ __align__(16) uint8_t smem[];
  constexpr int SLOT = KC * 576;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int K = p.K;
  const int64_t rb = K / 2, srb = K / 16;  // bytes per weight row, scale bytes per row
  const int64_t r0 = static_cast<int64_t>(blockIdx.x) * p.N / gridDim.x;
  const int64_t r1 = static_cast<int64_t>(blockIdx.x + 1) * p.N / gridDim.x;
  uint4* xs = reinterpret_cast<uint4*>(smem);
  float* xsum = reinterpret_cast<float*>(smem + static_cast<size_t>(K) * 2);
  uint8_t* ring = smem + static_cast<size_t>(K) * 2 + static_cast<size_t>(K) / 8 + static_cast<size_t>(warp) * D * SLOT;
  auto stage_row = [&](int64_t r, int sl) {
    uint8_t* rowb = ring + sl * SLOT;
    if (r < r1) {
    const uint8_t* wr = p.w + r * rb + 16 * lane;
#pragma unroll
    for (int i = 0; i < KC; ++i) cp_async16(rowb + i * 512 + 16 * lane, wr + 512 * i);
    if (lane < KC * 4) cp_async16(rowb + KC * 512 + 16 * lane, p.sc + r * srb + 16 * lane);
    }
    cp_async_commit();
  };
  int64_t r = r0 + warp;
  if (p.early_weights) {
#pragma unroll
    for (int d = 0; d < D; ++d) stage_row(r + d * kR1Warps, d);
  } else if (tid == 0) {  // the CTA's rows are contiguous: pull them into L2 during the previous kernel
    prefetch_span_l2(p.w + r0 * rb, static_cast<uint64_t>(r1 - r0) * rb);
    prefetch_span_l2(p.sc + r0 * srb, static_cast<uint64_t>(r1 - r0) * srb);
  }
  pdl_wait();
  constexpr int XP = (KC * 128 + kR1Threads - 1) / kR1Threads;  // 16-byte activation pieces per thread
  uint4 xv[XP];
#pragma unroll
  for (int j = 0; j < XP; ++j) {
    const int q = tid + j * kR1Threads;
    if (q < K / 8) xv[j] = __ldcg(reinterpret_cast<const uint4*>(p.x) + q);
  }
  if (!p.early_weights) {
#pragma unroll
    for (int d = 0; d < D; ++d) stage_row(r + d * kR1Warps, d);
  }
  // piece q = 4 b + part of scale block b (32 k) = 32 i + l -> PERM pieces [i][part][l], block sums
#pragma unroll
  for (int j = 0; j < XP; ++j) {
    const int q = tid + j * kR1Threads;
    if (q < K / 8) {  // K / 8 is a multiple of 128: whole warps take this branch
      const int b = q >> 2, part = q & 3, i = b >> 5, l = b & 31;
      xs[(i * 4 + part) * 32 + l] = x_piece_to_frag<kFmtQ4>(xv[j]);
      const uint32_t w4[4] = {xv[j].x, xv[j].y, xv[j].z, xv[j].w};
      float sum = 0.f;
#pragma unroll
      for (int e = 0; e < 4; ++e) sum += __uint_as_float(w4[e] << 16) + __uint_as_float(w4[e] & 0xFFFF0000u);
      sum += __shfl_xor_sync(0xffffffffu, sum, 1);  // the block's four pieces sit in four adjacent lanes
      sum += __shfl_xor_sync(0xffffffffu, sum, 2);
      if (part == 0) xsum[b] = sum;
    }
  }
  __syncthreads();
  pdl_trigger();  // the next call's CTAs start now, not during this call's activation loads

  int sl = 0;
  for (; r < r1; r += kR1Warps) {
    if constexpr (D == 2) asm volatile("cp.async.wait_group 1;" ::: "memory");  // the older row has landed
    else cp_async_wait_all();
    __syncwarp();  // the row's scales were copied by other lanes
    const uint8_t* rowb = ring + sl * SLOT;
    float acc = 0.f;
#pragma unroll
    for (int i = 0; i < KC; ++i) {
      uint4 x[4];
#pragma unroll
      for (int part = 0; part < 4; ++part) x[part] = xs[(i * 4 + part) * 32 + lane];
      const float xb = xsum[i * 32 + lane];
      const uint4 wq = lds128(rowb + i * 512 + 16 * lane);
      const uint32_t sb = *reinterpret_cast<const uint16_t*>(rowb + KC * 512 + 64 * i + 2 * lane);
      acc = fmaf(fmaf(-136.f, xb, q4_block_dot(wq, x)), bf16_bits_to_f32(sb), acc);
    }
    __syncwarp();  // every lane is done with the buffers
    stage_row(r + D * kR1Warps, sl);  // into the slot just read: streams while the ring's other rows are used
    sl = (sl + 1 == D) ? 0 : sl + 1;
    const float a = warp_sum(acc);
    if (lane == 0) p.y[r] = __float2bfloat16(a);
  }
  cp_async_wait_all();  // nothing in flight into shared memory at exit
}

template <int KC>
cudaError_t launch_q4_r1(const R1Params& p, int grid, const LaunchCfg& cfg) {
  constexpr int D = KC <= 4 ? 2 : 1;  // a second row slot per warp while two CTAs still fit an SM
  const size_t smem = static_cast<size_t>(p.K) * 2 + static_cast<size_t>(p.K) / 8 + static_cast<size_t>(kR1Warps) * KC * 576 * D;
  auto kern = gemv_q4_r1_kernel<KC, D>;
  static SmemOptIn opt;
  cudaError_t e = allow_smem(kern, smem, opt);
  if (e != cudaSuccess) return e;
  return launch_kernel(kern, dim3(grid), dim3(kR1Threads), smem, cfg, p);
}


// ------------------------------------------------------------------------------------------
// Q4Gemv iq2 = 2 (native IQ2_XXS records) at R = 1.  Weight contract of the reference's iq2 path:
// w = +-bf16(mag * bf16(d * (0.5 + s4) * 0.25)) (the decode of mma_decode.cuh), products with x
// exact and summed in fp32.  A row is K / 4 bytes (an 8-byte record per 32 k); lane l reads 16
// bytes (two records, 64 k) per 2048-k chunk and the fp16 scale of their 256-k superblock (x in
// shared memory as [chunk][8-k piece][lane], so a warp's 16-byte reads are contiguous); the
// codebook sits in shared memory in 8 bank-group copies (conflict-free lookups).
// gemv_iq2n_r1_kernel (the default) stages a warp's rows through shared memory like the NVFP4
// kernel; gemv_iq2n_r1_reg_kernel, for scales that are not 16-byte aligned, streams RB rows per
// warp through registers and reduces their sums in one butterfly.
// ------------------------------------------------------------------------------------------
// One IQ2_XXS record (32 k: four grid indices in idx4; four 7-bit sign patterns and the 4-bit
// sub-scale in sg) -> 16 bf16 pairs in k order, each +-bf16(mag * bf16(d * (0.5 + s4) * 0.25)):
// the arithmetic of decode_row<kFmtIq2N>, with the block scale formed once per record.
// grid: the codebook in 8 bank-group copies, entry e of copy c at uint4 index 8 e + c; lane l reads
// copy l % 8, so the 8 lanes of a shared-memory phase never share a bank group.
__device__ __forceinline__ void iq2n_record(uint32_t idx4, uint32_t sg, uint32_t dbits, const uint4* grid,
                                            uint32_t (&out)[16]) {
  const int copy = threadIdx.x & 7;
  const float d = __half2float(__ushort_as_half(static_cast<unsigned short>(dbits)));
  const float db = d * (0.5f + static_cast<float>(sg >> 28)) * 0.25f;
  const __nv_bfloat162 s2 = __bfloat162bfloat162(__float2bfloat16_rn(db));
#pragma unroll
  for (int gi = 0; gi < 4; ++gi) {
    const uint4 gv = grid[8 * ((idx4 >> (8 * gi)) & 0xFFu) + copy];
    uint32_t pat = (sg >> (7 * gi)) & 127u;
    pat |= (__popc(pat) & 1u) << 7;
    const uint32_t gw[4] = {gv.x, gv.y, gv.z, gv.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) out[4 * gi + j] = bf2_bits(__hmul2(bits_bf2(gw[j] ^ iq2_sign_mask(pat, j)), s2));
  }
}

template <int KC, int RB>
__global__ void __launch_bounds__(kR1Threads, 1) gemv_iq2n_r1_reg_kernel(const R1Params p) {
  extern __shared__ __align__(16) uint8_t smem[];  // x: [chunk][piece 0..7][lane] 16-byte pieces
  __shared__ uint4 grid_s[256 * 8];  // 8 bank-group copies of the codebook (32 KB)
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int K = p.K;
  const int64_t rb = K / 4, srb = K / 256;  // bytes per weight row, scales per row
  const int64_t r0 = static_cast<int64_t>(blockIdx.x) * p.N / gridDim.x;
  const int64_t r1 = static_cast<int64_t>(blockIdx.x + 1) * p.N / gridDim.x;
  const uint16_t* sc = reinterpret_cast<const uint16_t*>(p.sc);
  pdl_trigger();
  for (int i = tid; i < 256 * 8; i += kR1Threads)
    grid_s[i] = reinterpret_cast<const uint4*>(kIq2xxsGridBf16x2)[i >> 3];

  uint4 wv[RB][KC];
  uint32_t sv[RB][KC];
  auto load_rows = [&](int64_t ra) {
#pragma unroll
    for (int q = 0; q < RB; ++q) {
      const int64_t r = ra + 16 * q;
      if (r < r1) {
        const uint8_t* wr = p.w + r * rb + 16 * lane;
        const uint16_t* sr = sc + r * srb + (lane >> 2);
#pragma unroll
        for (int i = 0; i < KC; ++i) {
          wv[q][i] = ldg_stream(wr + 512 * i);
          sv[q][i] = ldg_u16(sr + 8 * i);
        }
      }
    }
  };
  int64_t ra = r0 + warp;
  if (p.early_weights) {
    load_rows(ra);
  } else if (tid == 0) {  // the CTA's rows are contiguous: pull them into L2 during the previous kernel
    prefetch_span_l2(p.w + r0 * rb, static_cast<uint64_t>(r1 - r0) * rb);
  }
  pdl_wait();
  if (!p.early_weights) load_rows(ra);

  uint4* xs = reinterpret_cast<uint4*>(smem);
  for (int q = tid; q < K / 8; q += kR1Threads) {  // 8-k piece q -> chunk q / 256, lane (q / 8) % 32, piece q % 8
    const int i = q >> 8, l = (q >> 3) & 31, piece = q & 7;
    xs[(i * 8 + piece) * 32 + l] = __ldcg(reinterpret_cast<const uint4*>(p.x) + q);
  }
  __syncthreads();

  constexpr int kLanesPerRow = 32 / RB;
  for (; ra < r1; ra += 16 * RB) {
    float acc[RB];
#pragma unroll
    for (int q = 0; q < RB; ++q) acc[q] = 0.f;
#pragma unroll
    for (int i = 0; i < KC; ++i) {
      uint32_t x[32];  // the lane's 64 k as bf16 pairs
#pragma unroll
      for (int piece = 0; piece < 8; ++piece) {
        const uint4 v = xs[(i * 8 + piece) * 32 + lane];
        x[4 * piece] = v.x;
        x[4 * piece + 1] = v.y;
        x[4 * piece + 2] = v.z;
        x[4 * piece + 3] = v.w;
      }
#pragma unroll
      for (int q = 0; q < RB; ++q) {
        float a = 0.f, b = 0.f;
#pragma unroll
        for (int rec = 0; rec < 2; ++rec) {
          uint32_t d[16];
          iq2n_record(rec ? wv[q][i].z : wv[q][i].x, rec ? wv[q][i].w : wv[q][i].y, sv[q][i], grid_s, d);
#pragma unroll
          for (int j = 0; j < 16; ++j) fma2_bf16_f32r(d[j], x[16 * rec + j], a, b);
        }
        acc[q] += a + b;
      }
    }
    if (ra + 16 * RB < r1) load_rows(ra + 16 * RB);  // the warp's next rows, while it reduces
    const float v = warp_sum_t<RB>(acc);
    const int q = lane / kLanesPerRow;
    if (lane % kLanesPerRow == 0 && ra + 16 * q < r1) p.y[ra + 16 * q] = __float2bfloat16(v);
  }
}

// IQ2_XXS at R = 1 with the rows staged through shared memory (the NVFP4 kernel's schedule, with
// the Q4 kernel's ring of D row slots per warp: 7.13 -> 6.76 us at K = 4096, N = 8192 for D = 2;
// two CTAs per SM, the dependents released once the activations are staged).  Same arithmetic as
// the register kernel above.  Needs 16-byte aligned scales (the register kernel takes the rest).
// KC = K / 2048.
template <int KC, int D>
__global__ void __launch_bounds__(kR1Threads, 2) gemv_iq2n_r1_kernel(const R1Params p) {
  // [x: [chunk][piece 0..7][lane] 16-byte pieces, K * 2 bytes][per warp: the row's KC chunks
  // [chunk][lane] 16 B, then its K / 128 bytes of fp16 superblock scales]
  extern __shared__ __align__(16) uint8_t smem[];
  __shared__ uint4 grid_s[256 * 8];  // 8 bank-group copies of the codebook (32 KB)
  constexpr int SLOT = KC * 528;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int K = p.K;
  const int64_t rb = K / 4, srb = K / 128;  // bytes per weight row, scale bytes per row
  const int64_t r0 = static_cast<int64_t>(blockIdx.x) * p.N / gridDim.x;
  const int64_t r1 = static_cast<int64_t>(blockIdx.x + 1) * p.N / gridDim.x;
  for (int i = tid; i < 256 * 8; i += kR1Threads)
    grid_s[i] = reinterpret_cast<const uint4*>(kIq2xxsGridBf16x2)[i >> 3];
  uint4* xs = reinterpret_cast<uint4*>(smem);
  uint8_t* ring = smem + static_cast<size_t>(K) * 2 + static_cast<size_t>(warp) * D * SLOT;
  auto stage_row = [&](int64_t r, int sl) {
    uint8_t* rowb = ring + sl * SLOT;
    if (r < r1) {
    const uint8_t* wr = p.w + r * rb + 16 * lane;
#pragma unroll
    for (int i = 0; i < KC; ++i) cp_async16(rowb + i * 512 + 16 * lane, wr + 512 * i);
    if (lane < KC) cp_async16(rowb + KC * 512 + 16 * lane, p.sc + r * srb + 16 * lane);
    }
    cp_async_commit();
  };
  int64_t r = r0 + warp;
  if (p.early_weights) {
#pragma unroll
    for (int d = 0; d < D; ++d) stage_row(r + d * kR1Warps, d);
  } else if (tid == 0) {  // the CTA's rows are contiguous: pull them into L2 during the previous kernel
    prefetch_span_l2(p.w + r0 * rb, static_cast<uint64_t>(r1 - r0) * rb);
    prefetch_span_l2(p.sc + r0 * srb, static_cast<uint64_t>(r1 - r0) * srb);
  }
  pdl_wait();
  constexpr int XP = (KC * 256 + kR1Threads - 1) / kR1Threads;  // 16-byte activation pieces per thread
  uint4 xv[XP];
#pragma unroll
  for (int j = 0; j < XP; ++j) {
    const int q = tid + j * kR1Threads;
    if (q < K / 8) xv[j] = __ldcg(reinterpret_cast<const uint4*>(p.x) + q);
  }
  if (!p.early_weights) {
#pragma unroll
    for (int d = 0; d < D; ++d) stage_row(r + d * kR1Warps, d);
  }
#pragma unroll
  for (int j = 0; j < XP; ++j) {  // 8-k piece q -> chunk q / 256, lane (q / 8) % 32, piece q % 8
    const int q = tid + j * kR1Threads;
    if (q < K / 8) xs[((q >> 8) * 8 + (q & 7)) * 32 + ((q >> 3) & 31)] = xv[j];
  }
  __syncthreads();
  pdl_trigger();  // the next call's CTAs start now, not during this call's activation loads

  int sl = 0;
  for (; r < r1; r += kR1Warps) {
    if constexpr (D == 2) asm volatile("cp.async.wait_group 1;" ::: "memory");  // the older row has landed
    else cp_async_wait_all();
    __syncwarp();  // the row's scales were copied by other lanes
    const uint8_t* rowb = ring + sl * SLOT;
    float acc = 0.f;
#pragma unroll
    for (int i = 0; i < KC; ++i) {
      const uint4 wq = lds128(rowb + i * 512 + 16 * lane);
      const uint32_t sb = *reinterpret_cast<const uint16_t*>(rowb + KC * 512 + 16 * i + 2 * (lane >> 2));
      float a = 0.f, b = 0.f;
#pragma unroll
      for (int rec = 0; rec < 2; ++rec) {
        uint32_t d[16];
        iq2n_record(rec ? wq.z : wq.x, rec ? wq.w : wq.y, sb, grid_s, d);
#pragma unroll
        for (int pc = 0; pc < 4; ++pc) {
          const uint4 xq = xs[(i * 8 + 4 * rec + pc) * 32 + lane];
          fma2_bf16_f32r(d[4 * pc], xq.x, a, b);
          fma2_bf16_f32r(d[4 * pc + 1], xq.y, a, b);
          fma2_bf16_f32r(d[4 * pc + 2], xq.z, a, b);
          fma2_bf16_f32r(d[4 * pc + 3], xq.w, a, b);
        }
      }
      acc += a + b;
    }
    __syncwarp();  // every lane is done with the buffers
    stage_row(r + D * kR1Warps, sl);  // into the slot just read: streams while the ring's other rows are used
    sl = (sl + 1 == D) ? 0 : sl + 1;
    const float v = warp_sum(acc);
    if (lane == 0) p.y[r] = __float2bfloat16(v);
  }
  cp_async_wait_all();  // nothing in flight into shared memory at exit
}

template <int KC>
cudaError_t launch_iq2n_r1(const R1Params& p, int grid, const LaunchCfg& cfg) {
  constexpr int D = KC <= 2 ? 2 : 1;  // a second row slot per warp while two CTAs still fit an SM
  const size_t smem = static_cast<size_t>(p.K) * 2 + static_cast<size_t>(kR1Warps) * KC * 528 * D;
  auto kern = gemv_iq2n_r1_kernel<KC, D>;
  static SmemOptIn opt;
  cudaError_t e = allow_smem(kern, smem, opt);
  if (e != cudaSuccess) return e;
  return launch_kernel(kern, dim3(grid), dim3(kR1Threads), smem, cfg, p);
}

template <int KC>
cudaError_t launch_iq2n_r1_reg(const R1Params& p, int grid, const LaunchCfg& cfg) {
  const size_t smem = static_cast<size_t>(p.K) * 2;
  constexpr int RB = KC <= 1 ? 4 : 2;  // rows per warp batch without spilling
  auto kern = gemv_iq2n_r1_reg_kernel<KC, RB>;
  static SmemOptIn opt;
  cudaError_t e = allow_smem(kern, smem, opt);
  if (e != cudaSuccess) return e;
  return launch_kernel(kern, dim3(grid), dim3(kR1Threads), smem, cfg, p);
}

// ------------------------------------------------------------------------------------------
// Q8Gemv at R = 1, exact contract (every weight the exact fp32 (b - 128) * s, fp32 sums; the
// reference's R = 1 kernel is QGemvKernel, src/bolt_ops.cu:1315-1392), on the NVFP4 kernel's
// layout and schedule: a warp stages one row at a time through shared memory by cp.async (16
// bytes = 16 k per lane and 512-k chunk, plus the row's bf16 scales), two CTAs per SM, the
// dependents released once the activations are staged.  x sits in shared memory as fp32,
// [chunk][part 0..3][lane] 16 bytes, the 16 k of lane l in k order.  A lane turns four weight
// bytes into floats with one prmt each (bits 0x4B0000bb = 2^23 + b) and one packed add of
// -(2^23 + 128) per pair -- exact -- then runs packed fma.rn.f32x2 with x, and scales its 16-k
// sum once (a 32-k scale block spans two lanes).  KC = K / 512, K <= 4096.
// ------------------------------------------------------------------------------------------
template <int KC>
__global__ void __launch_bounds__(kR1Threads, 2) gemv_q8_r1_kernel(const R1Params p) {
  extern __shared__ __align__(16) uint8_t smem[];
  constexpr int SLOT = KC * 544;  // 512 weight bytes + 32 scale bytes per chunk
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int K = p.K;
  const int64_t rb = K, srb = K / 16;  // bytes per weight row, scale bytes per row
  const int64_t r0 = static_cast<int64_t>(blockIdx.x) * p.N / gridDim.x;
  const int64_t r1 = static_cast<int64_t>(blockIdx.x + 1) * p.N / gridDim.x;
  uint8_t* rowb = smem + static_cast<size_t>(K) * 4 + static_cast<size_t>(warp) * SLOT;
  auto stage_row = [&](int64_t r) {
    const uint8_t* wr = p.w + r * rb + 16 * lane;
#pragma unroll
    for (int i = 0; i < KC; ++i) cp_async16(rowb + i * 512 + 16 * lane, wr + 512 * i);
    if (lane < KC * 2) cp_async16(rowb + KC * 512 + 16 * lane, p.sc + r * srb + 16 * lane);
    cp_async_commit();
  };
  int64_t r = r0 + warp;
  if (p.early_weights) {
    if (r < r1) stage_row(r);
  } else if (tid == 0) {  // the CTA's rows are contiguous: pull them into L2 during the previous kernel
    prefetch_span_l2(p.w + r0 * rb, static_cast<uint64_t>(r1 - r0) * rb);
    prefetch_span_l2(p.sc + r0 * srb, static_cast<uint64_t>(r1 - r0) * srb);
  }
  pdl_wait();
  constexpr int XP = (KC * 64 + kR1Threads - 1) / kR1Threads;  // 16-byte activation pieces per thread
  uint4 xv[XP];
#pragma unroll
  for (int j = 0; j < XP; ++j) {
    const int q = tid + j * kR1Threads;
    if (q < K / 8) xv[j] = __ldcg(reinterpret_cast<const uint4*>(p.x) + q);
  }
  if (!p.early_weights && r < r1) stage_row(r);
  // piece q (8 k) -> chunk q / 64, lane (q % 64) / 2, parts 2 (q % 2) and 2 (q % 2) + 1
#pragma unroll
  for (int j = 0; j < XP; ++j) {
    const int q = tid + j * kR1Threads;
    if (q < K / 8) {
      const int i = q >> 6, l = (q & 63) >> 1, h = q & 1;
      const uint32_t u[4] = {xv[j].x, xv[j].y, xv[j].z, xv[j].w};
      float f[8];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        f[2 * e] = __uint_as_float(u[e] << 16);
        f[2 * e + 1] = __uint_as_float(u[e] & 0xFFFF0000u);
      }
      *reinterpret_cast<float4*>(smem + ((i * 4 + 2 * h) * 32 + l) * 16) = make_float4(f[0], f[1], f[2], f[3]);
      *reinterpret_cast<float4*>(smem + ((i * 4 + 2 * h + 1) * 32 + l) * 16) = make_float4(f[4], f[5], f[6], f[7]);
    }
  }
  __syncthreads();
  pdl_trigger();  // the next call's CTAs start now, not during this call's activation loads

  const uint32_t M = 0x4B000000u;
  const float2 zp = make_float2(-8388736.f, -8388736.f);  // -(2^23 + 128)
  for (; r < r1; r += kR1Warps) {
    cp_async_wait_all();
    __syncwarp();  // the row's scales were copied by other lanes
    float acc = 0.f;
#pragma unroll
    for (int i = 0; i < KC; ++i) {
      const uint4 wq = lds128(rowb + i * 512 + 16 * lane);
      const uint32_t wd[4] = {wq.x, wq.y, wq.z, wq.w};
      float2 a = make_float2(0.f, 0.f), b = make_float2(0.f, 0.f);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float4 xq = *reinterpret_cast<const float4*>(smem + ((i * 4 + q) * 32 + lane) * 16);
        const float2 f01 = fadd2(make_float2(__uint_as_float(prmt(wd[q], M, 0x7440)),
                                             __uint_as_float(prmt(wd[q], M, 0x7441))), zp);
        const float2 f23 = fadd2(make_float2(__uint_as_float(prmt(wd[q], M, 0x7442)),
                                             __uint_as_float(prmt(wd[q], M, 0x7443))), zp);
        a = ffma2(f01, make_float2(xq.x, xq.y), a);
        b = ffma2(f23, make_float2(xq.z, xq.w), b);
      }
      const uint32_t sb = *reinterpret_cast<const uint16_t*>(rowb + KC * 512 + 32 * i + 2 * (lane >> 1));
      acc = fmaf((a.x + a.y) + (b.x + b.y), bf16_bits_to_f32(sb), acc);
    }
    __syncwarp();  // every lane is done with the buffers
    if (r + kR1Warps < r1) stage_row(r + kR1Warps);  // the warp's next row streams while it reduces
    const float v = warp_sum(acc);
    if (lane == 0) p.y[r] = __float2bfloat16(v);
  }
  cp_async_wait_all();  // nothing in flight into shared memory at exit
}

template <int KC>
cudaError_t launch_q8_r1(const R1Params& p, int grid, const LaunchCfg& cfg) {
  const size_t smem = static_cast<size_t>(p.K) * 4 + static_cast<size_t>(kR1Warps) * KC * 544;
  auto kern = gemv_q8_r1_kernel<KC>;
  static SmemOptIn opt;
  cudaError_t e = allow_smem(kern, smem, opt);
  if (e != cudaSuccess) return e;
  return launch_kernel(kern, dim3(grid), dim3(kR1Threads), smem, cfg, p);
}

}  // namespace

cudaError_t launch_gemv_r1(int fmt, const bf16* x, const uint8_t* w, const void* sc, const float* gscale, int64_t N,
                           int K, bf16* y, const LaunchCfg& cfg) {
  if (fmt == kFmtIq2N) {
    if (N < 1 || K < 2048 || K % 2048 || K / 2048 > 4 || (reinterpret_cast<uintptr_t>(w) & 15) ||
        (reinterpret_cast<uintptr_t>(sc) & 1) || (reinterpret_cast<uintptr_t>(x) & 15))
      return cudaErrorNotSupported;
    const R1Params q{x, w, static_cast<const uint8_t*>(sc), gscale, y, N, K, cfg.early_weights ? 1 : 0};
    const int grid = static_cast<int>(std::min<int64_t>(cfg.sms, (N + 15) / 16));
    if (!(reinterpret_cast<uintptr_t>(sc) & 15)) {
      switch (K / 2048) {
        case 1: return launch_iq2n_r1<1>(q, grid, cfg);
        case 2: return launch_iq2n_r1<2>(q, grid, cfg);
        case 3: return launch_iq2n_r1<3>(q, grid, cfg);
        default: return launch_iq2n_r1<4>(q, grid, cfg);
      }
    }
    switch (K / 2048) {
      case 1: return launch_iq2n_r1_reg<1>(q, grid, cfg);
      case 2: return launch_iq2n_r1_reg<2>(q, grid, cfg);
      case 3: return launch_iq2n_r1_reg<3>(q, grid, cfg);
      default: return launch_iq2n_r1_reg<4>(q, grid, cfg);
    }
  }
  if (fmt == kFmtQ8) {
    if (N < 1 || K < 512 || K % 512 || K > 4096 || (reinterpret_cast<uintptr_t>(w) & 15) ||
        (reinterpret_cast<uintptr_t>(sc) & 15) || (reinterpret_cast<uintptr_t>(x) & 15))
      return cudaErrorNotSupported;
    const R1Params q{x, w, static_cast<const uint8_t*>(sc), gscale, y, N, K, cfg.early_weights ? 1 : 0};
    const int grid = static_cast<int>(std::min<int64_t>(cfg.sms, (N + 15) / 16));
    switch (K / 512) {
      case 1: return launch_q8_r1<1>(q, grid, cfg);
      case 2: return launch_q8_r1<2>(q, grid, cfg);
      case 3: return launch_q8_r1<3>(q, grid, cfg);
      case 4: return launch_q8_r1<4>(q, grid, cfg);
      case 5: return launch_q8_r1<5>(q, grid, cfg);
      case 6: return launch_q8_r1<6>(q, grid, cfg);
      case 7: return launch_q8_r1<7>(q, grid, cfg);
      default: return launch_q8_r1<8>(q, grid, cfg);
    }
  }
  if ((fmt != kFmtFp4 && fmt != kFmtQ4) || N < 1 || K < 1024 || K % 1024 || K / 1024 > kR1MaxChunks)
    return cudaErrorNotSupported;
  if ((reinterpret_cast<uintptr_t>(w) & 15) || (reinterpret_cast<uintptr_t>(sc) & 15) ||
      (reinterpret_cast<uintptr_t>(x) & 15))
    return cudaErrorNotSupported;
  R1Params p{x, w, static_cast<const uint8_t*>(sc), gscale, y, N, K, cfg.early_weights ? 1 : 0};
  const int grid = static_cast<int>(std::min<int64_t>(cfg.sms, (N + 15) / 16));
  if (fmt == kFmtQ4) {
    switch (K / 1024) {
      case 1: return launch_q4_r1<1>(p, grid, cfg);
      case 2: return launch_q4_r1<2>(p, grid, cfg);
      case 3: return launch_q4_r1<3>(p, grid, cfg);
      case 4: return launch_q4_r1<4>(p, grid, cfg);
      case 5: return launch_q4_r1<5>(p, grid, cfg);
      case 6: return launch_q4_r1<6>(p, grid, cfg);
      case 7: return launch_q4_r1<7>(p, grid, cfg);
      default: return launch_q4_r1<8>(p, grid, cfg);
    }
  }
  switch (K / 1024) {
    case 1: return launch_r1<1>(p, grid, cfg);
    case 2: return launch_r1<2>(p, grid, cfg);
    case 3: return launch_r1<3>(p, grid, cfg);
    case 4: return launch_r1<4>(p, grid, cfg);
    case 5: return launch_r1<5>(p, grid, cfg);
    case 6: return launch_r1<6>(p, grid, cfg);
    case 7: return launch_r1<7>(p, grid, cfg);
    default: return launch_r1<8>(p, grid, cfg);
  }
}

}  // namespace bolt
