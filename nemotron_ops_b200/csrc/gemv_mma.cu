// Tensor-core skinny GEMV: y[R, N] = x[R, K] @ W^T for R <= 8 (mma.sync m16n8k16, fp32 acc).
//
// Used for Q8Gemv / Q4Gemv at 2 <= R <= 8 (K % 64 == 0), for every R with iq2 = 1 / 2, and for
// Nvfp4Gemv at every R (reference dispatch: src/bolt_ops.cu:1259-1306, :1429-1468).  The
// weight contract is the reference's tensor-core one (bf16-rounded weights, DequantRow
// :860-919) -- see mma_decode.cuh.
//
// B200 design: persistent CTAs own contiguous weight-row ranges; 16-row tiles are streamed
// with per-row cp.async.bulk copies into padded smem rows (the padding makes the per-thread
// fragment reads bank-conflict free) plus the tile's scale span, several tiles in flight; KW
// warps split K, keep their activation fragments in registers for the whole CTA (the
// activations are shared by all tiles), decode weights in registers and issue mma.sync; per
// tile the K partials are combined through a double-buffered smem pass.
#include "mma_decode.cuh"

namespace bolt {

namespace {

constexpr int kTileRows = 16;

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
  uint32_t stage_bytes;
  uint32_t row_stride;  // padded smem bytes per row
  int early_weights;
};

template <int KW>
__device__ __forceinline__ void bar_consumers() {
  asm volatile("bar.sync 1, %0;" ::"n"(KW * 32) : "memory");
}

// Issues the bulk copies of tile `i` (16 rows + scale span) into ring slot i % NS.
template <int FMT>
__device__ __forceinline__ void mma_issue_tile(const MmaParams& p, uint8_t* smem, uint64_t* full_bar, int i, int64_t r0,
                                               int nrows, int64_t row_bytes, int64_t sc_row_bytes) {
  const int s = i % p.nstage;
  const int64_t row0 = r0 + static_cast<int64_t>(i) * kTileRows;
  const int rows = min(kTileRows, nrows - i * kTileRows);
  uint8_t* slot = smem + static_cast<size_t>(s) * p.stage_bytes;
  const uint32_t fb = smem_u32(&full_bar[s]);
  uint32_t tx = static_cast<uint32_t>(rows * row_bytes);
  for (int r = 0; r < rows; ++r)
    bulk_g2s(smem_u32(slot + r * p.row_stride), p.w + (row0 + r) * row_bytes, static_cast<uint32_t>(row_bytes), fb);
  stage_span(slot + kTileRows * p.row_stride, p.sc + row0 * sc_row_bytes, static_cast<uint32_t>(rows * sc_row_bytes),
             p.sc + p.N * sc_row_bytes, fb, tx);
  mbar_arrive_expect_tx(fb, tx);
}

// CPW: max 64-k chunks per warp held as register fragments.  Thread 0 doubles as the copy
// issuer: it fills the ring up front and refills a slot right after the per-tile barrier,
// which proves that every warp has finished reading it.
template <int FMT, int KW, int CPW>
__global__ void __launch_bounds__(KW * 32, 1) gemv_mma_kernel(const MmaParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ uint64_t full_bar[16];
  __shared__ float red[2][KW][128];
  __shared__ __align__(16) uint32_t grid_s[(FMT == kFmtIq2N) ? 1024 : 4];
  __shared__ volatile int abort_flag;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  const int K = p.K;
  const int64_t row_bytes = fmt_row_bytes(FMT, K);
  const int64_t sc_row_bytes = fmt_scale_row_bytes(FMT, K);
  const int64_t r0 = static_cast<int64_t>(blockIdx.x) * p.N / gridDim.x;
  const int64_t r1 = static_cast<int64_t>(blockIdx.x + 1) * p.N / gridDim.x;
  const int nrows = static_cast<int>(r1 - r0);
  const int ntiles = (nrows + kTileRows - 1) / kTileRows;
  const int NS = p.nstage;
  const uint32_t stride = p.row_stride;

  if (tid == 0) {
    for (int s = 0; s < NS; ++s) mbar_init(smem_u32(&full_bar[s]), 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  if constexpr (FMT == kFmtIq2N) {
    for (int i = tid; i < 1024; i += blockDim.x) grid_s[i] = kIq2xxsGridBf16x2[i];
  }
  __syncthreads();
  pdl_trigger();
  if (tid == 0) {
    if (!p.early_weights) pdl_wait();
    for (int i = 0; i < min(NS, ntiles); ++i) mma_issue_tile<FMT>(p, smem, full_bar, i, r0, nrows, row_bytes, sc_row_bytes);
  }
  pdl_wait();

  const int nchunks = K >> 6;
  const int cb = static_cast<int>(static_cast<int64_t>(warp) * nchunks / KW);
  const int ce = static_cast<int>(static_cast<int64_t>(warp + 1) * nchunks / KW);
  uint32_t bfr[CPW][8];
#pragma unroll
  for (int j = 0; j < CPW; ++j) {
    uint32_t x16[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    const int c = cb + j;
    if (c < ce && g < p.R) {
      const uint4* xp = reinterpret_cast<const uint4*>(p.x + static_cast<int64_t>(g) * K + 64 * c + 16 * t);
      const uint4 a = __ldg(xp), b = __ldg(xp + 1);
      x16[0] = a.x; x16[1] = a.y; x16[2] = a.z; x16[3] = a.w;
      x16[4] = b.x; x16[5] = b.y; x16[6] = b.z; x16[7] = b.w;
    }
    make_b_frags<FMT>(x16, bfr[j]);
  }
  const float gs = (FMT == kFmtFp4) ? p.gscale[0] * 64.f : 1.f;

  for (int i = 0; i < ntiles; ++i) {
    const int s = i % NS;
    const uint32_t ph = (i / NS) & 1;
    if (!abort_flag && !mbar_wait(smem_u32(&full_bar[s]), ph, kStatusFullWait)) abort_flag = 1;
    const uint8_t* slot = smem + static_cast<size_t>(s) * p.stage_bytes;
    const int64_t row0 = r0 + static_cast<int64_t>(i) * kTileRows;
    const uint8_t* sc_base = slot + kTileRows * stride + (reinterpret_cast<uintptr_t>(p.sc + row0 * sc_row_bytes) & 15);
    const uint8_t* row_g = slot + g * stride;
    const uint8_t* row_g8 = slot + (g + 8) * stride;
    const uint8_t* sc_g = sc_base + g * sc_row_bytes;
    const uint8_t* sc_g8 = sc_base + (g + 8) * sc_row_bytes;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int j = 0; j < CPW; ++j)
      if (cb + j < ce) mma_chunk<FMT>(row_g, row_g8, sc_g, sc_g8, cb + j, t, grid_s, bfr[j], acc);

    const int buf = i & 1;
    *reinterpret_cast<float2*>(&red[buf][warp][g * 8 + 2 * t]) = make_float2(acc[0], acc[1]);
    *reinterpret_cast<float2*>(&red[buf][warp][(g + 8) * 8 + 2 * t]) = make_float2(acc[2], acc[3]);
    bar_consumers<KW>();
    if (tid == 0 && i + NS < ntiles && !abort_flag)
      mma_issue_tile<FMT>(p, smem, full_bar, i + NS, r0, nrows, row_bytes, sc_row_bytes);
    const int rows = min(kTileRows, nrows - i * kTileRows);
    if (tid < kTileRows * p.R) {
      const int col = tid >> 4, rl = tid & 15;
      if (rl < rows) {
        float v = 0.f;
#pragma unroll
        for (int w = 0; w < KW; ++w) v += red[buf][w][rl * 8 + col];
        p.y[static_cast<int64_t>(col) * p.N + row0 + rl] = __float2bfloat16(v * gs);
      }
    }
  }
  if (tid == 0 && abort_flag)  // copies may still be landing: wait for them before exiting
    for (int i = max(0, ntiles - NS); i < ntiles; ++i)
      mbar_wait(smem_u32(&full_bar[i % NS]), (i / NS) & 1, kStatusDrainWait);
}

template <int FMT, int KW, int CPW>
cudaError_t launch_mma(const MmaParams& p, int grid, const LaunchCfg& cfg) {
  auto kern = gemv_mma_kernel<FMT, KW, CPW>;
  const size_t smem = static_cast<size_t>(p.nstage) * p.stage_bytes;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  return launch_kernel(kern, dim3(grid), dim3(KW * 32), smem, cfg, p);
}

template <int FMT>
cudaError_t dispatch_mma(const MmaParams& p, int grid, const LaunchCfg& cfg) {
  const int nchunks = p.K >> 6;
  if (nchunks <= 8 * 2) return launch_mma<FMT, 8, 2>(p, grid, cfg);
  if (nchunks <= 8 * 4) return launch_mma<FMT, 8, 4>(p, grid, cfg);
  if (nchunks <= 8 * 8) return launch_mma<FMT, 8, 8>(p, grid, cfg);
  return launch_mma<FMT, 16, 8>(p, grid, cfg);  // K <= 8192
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
  MmaParams p{x, w, static_cast<const uint8_t*>(sc), gscale, y, N, K, R, 0, 0, 0, cfg.early_weights ? 1 : 0};
  const int64_t rb = fmt_row_bytes(fmt, K);
  int bpc = 32;
  if (fmt == kFmtQ8) bpc = 64;
  if (fmt == kFmtIq2N) bpc = 16;
  const uint32_t pad = static_cast<uint32_t>((bpc - rb % 128 + 128) % 128);
  p.row_stride = static_cast<uint32_t>(rb) + pad;
  const uint32_t sc_bytes = static_cast<uint32_t>(kTileRows * fmt_scale_row_bytes(fmt, K) + 32);
  p.stage_bytes = (kTileRows * p.row_stride + sc_bytes + 127) & ~127u;
  const int grid = static_cast<int>(std::min<int64_t>(cfg.sms, (N + kTileRows - 1) / kTileRows));
  const int64_t rows_per_cta = (N + grid - 1) / grid;
  const int want = static_cast<int>((rows_per_cta + kTileRows - 1) / kTileRows);
  const int fit = static_cast<int>(cfg.smem_budget / p.stage_bytes);
  p.nstage = std::max(1, std::min({want, fit, 16}));
  switch (fmt) {
    case kFmtQ8: return dispatch_mma<kFmtQ8>(p, grid, cfg);
    case kFmtQ4: return dispatch_mma<kFmtQ4>(p, grid, cfg);
    case kFmtFp4: return dispatch_mma<kFmtFp4>(p, grid, cfg);
    case kFmtIq2Lut: return dispatch_mma<kFmtIq2Lut>(p, grid, cfg);
    default: return dispatch_mma<kFmtIq2N>(p, grid, cfg);
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
