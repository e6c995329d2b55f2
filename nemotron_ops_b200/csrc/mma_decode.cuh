// Weight decoders and fragment helpers of the tensor-core (mma.sync m16n8k16) path.
//
// Fragment ownership: for a 64-k chunk of a 16-row tile, thread (g = lane/4, t = lane%4)
// owns the 16 consecutive k [16t, 16t + 16) of weight rows g and g + 8.  An m16n8k16 MMA
// consumes, per thread and row, two k-pairs: A slots (2t, 2t+1) and (2t+8, 2t+9).  Any k
// permutation shared by A and B is valid, so each decoder picks the pairing that is cheapest
// for its format and the activation fragments (B) are permuted to match once per CTA:
//   * PERM layout (Q4, Q8): MMA s takes k (s, s+4) and (8+s, 12+s) of the thread's 16 -- the
//     two nibbles s and s+4 of a 32-bit word fall into the two bf16 halves with one mask;
//   * ADJ layout (NVFP4, IQ2 LUT, native IQ2_XXS): MMA s takes k (4s, 4s+1), (4s+2, 4s+3).
// Decoders write 8 registers: out[2s] = pair for slots (2t, 2t+1) of MMA s, out[2s+1] = pair
// for slots (2t+8, 2t+9).
//
// Weight contracts (reference src/bolt_ops.cu:860-919; oracle/bolt_oracle.py):
//   Q8   bf16((b - 128) * s)          Q4  bf16((n - 8) * bf16(s))
//   IQ2 LUT bf16(v[code] * bf16(s)),  v = {8, 25, 43, 0, -8, -25, -43, 0}
//   IQ2N +-bf16(mag * bf16(d * (0.5 + s4) * 0.25)), sign j = bit j of the ggml sign pattern
//   NVFP4 e2m1 * e4m3 (exact, computed in fp16; the global scale is applied in the epilogue)
#pragma once

#include "common.cuh"
#include "iq2xxs_grid.h"
#include "kernels.h"
#include "tensor_map.h"

namespace bolt {

enum XLayout { kXPerm = 0, kXAdj = 1 };

template <int FMT>
struct FmtTraits;

template <>
struct FmtTraits<kFmtQ4> {
  static constexpr int kRowBytesPerChunk = 32;  // bytes of one row per 64-k chunk
  static constexpr int kXLayout = kXPerm;
  static constexpr bool kF16 = false;
};
template <>
struct FmtTraits<kFmtQ8> {
  static constexpr int kRowBytesPerChunk = 64;
  static constexpr int kXLayout = kXPerm;
  static constexpr bool kF16 = false;
};
template <>
struct FmtTraits<kFmtIq2Lut> {
  static constexpr int kRowBytesPerChunk = 32;
  static constexpr int kXLayout = kXAdj;
  static constexpr bool kF16 = false;
};
template <>
struct FmtTraits<kFmtIq2N> {
  static constexpr int kRowBytesPerChunk = 16;
  static constexpr int kXLayout = kXAdj;
  static constexpr bool kF16 = false;
};
template <>
struct FmtTraits<kFmtFp4> {
  static constexpr int kRowBytesPerChunk = 32;
  static constexpr int kXLayout = kXAdj;
  static constexpr bool kF16 = true;
};

// bytes of one weight row / one scale row
__host__ __device__ inline int64_t fmt_row_bytes(int fmt, int K) {
  switch (fmt) {
    case kFmtQ8: return K;
    case kFmtIq2N: return K / 4;
    default: return K / 2;
  }
}
__host__ __device__ inline int64_t fmt_scale_row_bytes(int fmt, int K) {
  switch (fmt) {
    case kFmtFp4: return K / 16;     // e4m3 per 16
    case kFmtIq2N: return K / 128;   // fp16 per 256
    default: return K / 16;          // bf16 per 32
  }
}

__device__ __forceinline__ uint32_t bf2_bits(__nv_bfloat162 v) { return *reinterpret_cast<uint32_t*>(&v); }
__device__ __forceinline__ __nv_bfloat162 bits_bf2(uint32_t v) { return *reinterpret_cast<__nv_bfloat162*>(&v); }
__device__ __forceinline__ uint32_t h2_bits(__half2 v) { return *reinterpret_cast<uint32_t*>(&v); }
__device__ __forceinline__ __half2 bits_h2(uint32_t v) { return *reinterpret_cast<__half2*>(&v); }

// ---------------------------------------------------------------------------------------
// raw per-thread data of one row for one chunk, read from the staged row / scale bytes
// ---------------------------------------------------------------------------------------
struct RawRow {
  uint4 w;     // weight bytes (Q4/FP4/LUT use .x .y; Q8 all four; IQ2N .x .y = one record)
  uint32_t s;  // raw scale bits (bf16 bits, e4m3 byte, or fp16 bits)
};

template <int FMT>
__device__ __forceinline__ RawRow load_raw(const uint8_t* row, const uint8_t* sc_row, int c, int t) {
  RawRow r;
  if constexpr (FMT == kFmtQ8) {
    r.w = *reinterpret_cast<const uint4*>(row + 64 * c + 16 * t);
    r.s = reinterpret_cast<const uint16_t*>(sc_row)[2 * c + (t >> 1)];
  } else if constexpr (FMT == kFmtIq2N) {
    const uint2 v = *reinterpret_cast<const uint2*>(row + 8 * (2 * c + (t >> 1)));
    r.w = make_uint4(v.x, v.y, 0u, 0u);
    r.s = reinterpret_cast<const uint16_t*>(sc_row)[c >> 2];
  } else {
    const uint2 v = *reinterpret_cast<const uint2*>(row + 32 * c + 8 * t);
    r.w = make_uint4(v.x, v.y, 0u, 0u);
    if constexpr (FMT == kFmtFp4) r.s = sc_row[4 * c + t];
    else r.s = reinterpret_cast<const uint16_t*>(sc_row)[2 * c + (t >> 1)];
  }
  return r;
}

// Byte offset (row-relative layout) of this thread's weights for stage-local chunk c: the
// kernels precompute tile offsets from it once per CTA.
template <int FMT>
__host__ __device__ __forceinline__ int chunk_byte(int c, int t) {
  if (FMT == kFmtQ8) return 64 * c + 16 * t;
  if (FMT == kFmtIq2N) return 8 * (2 * c + (t >> 1));
  return 32 * c + 8 * t;
}
// Byte offset of this thread's scale for stage-local chunk c inside the row's scales.
template <int FMT>
__host__ __device__ __forceinline__ int chunk_scale_byte(int c, int t) {
  if (FMT == kFmtFp4) return 4 * c + t;
  if (FMT == kFmtIq2N) return 2 * (c >> 2);
  return 2 * (2 * c + (t >> 1));
}

template <int FMT>
__device__ __forceinline__ uint4 load_w_at(const uint8_t* p) {
  if constexpr (FMT == kFmtQ8) {
    return *reinterpret_cast<const uint4*>(p);
  } else {
    const uint2 v = *reinterpret_cast<const uint2*>(p);
    return make_uint4(v.x, v.y, 0u, 0u);
  }
}
template <int FMT>
__device__ __forceinline__ uint32_t load_s_at(const uint8_t* p) {
  if constexpr (FMT == kFmtFp4) return static_cast<uint32_t>(*p);
  else return static_cast<uint32_t>(*reinterpret_cast<const uint16_t*>(p));
}

// IQ2 LUT byte planes: bf16 of {8, 25, 43, 0} (codes 0..3) and their negatives (codes 4..7)
constexpr uint32_t kLutHiPos = 0x00424141u, kLutHiNeg = 0x00C2C1C1u;
constexpr uint32_t kLutLoPos = 0x002CC800u, kLutLoNeg = 0x002CC800u;

__device__ __forceinline__ uint32_t iq2_sign_mask(uint32_t pattern, int pair) {
  // bit 2*pair of the 8-bit pattern -> bit 15, bit 2*pair+1 -> bit 31 (the two partial
  // products occupy disjoint bit ranges, so no carry reaches bits 15 or 31)
  return (pattern * ((1u << (15 - 2 * pair)) + (1u << (30 - 2 * pair)))) & 0x80008000u;
}

// The IQ2_XXS codebook in shared memory: plain (256 entries of 16 bytes) or in 8 bank-group copies
// (entry e of copy c at 16-byte index 8 e + c; lane l reads copy l % 8, so the 8 lanes of a
// shared-memory phase never share a bank group -- 32 KB).
template <bool BANKED>
__device__ __forceinline__ void load_iq2_grid(uint32_t* grid, int tid, int nthreads) {
  const uint4* src = reinterpret_cast<const uint4*>(kIq2xxsGridBf16x2);
  uint4* dst = reinterpret_cast<uint4*>(grid);
  for (int i = tid; i < (BANKED ? 2048 : 256); i += nthreads) dst[i] = src[BANKED ? i >> 3 : i];
}
template <bool BANKED>
__device__ __forceinline__ uint4 iq2_grid_entry(const uint32_t* grid, uint32_t e) {
  const uint4* g = reinterpret_cast<const uint4*>(grid);
  return BANKED ? g[8 * e + (threadIdx.x & 7)] : g[e];
}

// Decodes one row's 16 weights of the chunk into 8 MMA A registers (see the file comment).
// `grid` points at the IQ2_XXS codebook in shared memory (BANKED: the 8-copy layout above).
template <int FMT, bool BANKED = false>
__device__ __forceinline__ void decode_row(const RawRow& r, int t, const uint32_t* grid, uint32_t (&out)[8]) {
  if constexpr (FMT == kFmtQ4) {
    const __nv_bfloat162 s2 = bits_bf2(r.s | (r.s << 16));
    const __nv_bfloat162 zp = bits_bf2(0x43084308u);  // 136, 136
#pragma unroll
    for (int s = 0; s < 4; ++s) {
      const uint32_t a = ((r.w.x >> (4 * s)) & 0x000F000Fu) | 0x43004300u;  // 128 + n, exact
      const uint32_t b = ((r.w.y >> (4 * s)) & 0x000F000Fu) | 0x43004300u;
      out[2 * s] = bf2_bits(__hmul2(__hsub2(bits_bf2(a), zp), s2));
      out[2 * s + 1] = bf2_bits(__hmul2(__hsub2(bits_bf2(b), zp), s2));
    }
  } else if constexpr (FMT == kFmtQ8) {
    const float sc = bf16_bits_to_f32(r.s);
    const uint32_t M = 0x4B000000u;
#pragma unroll
    for (int s = 0; s < 4; ++s) {
      const uint32_t sel = 0x7440u | s;
      const float a0 = (__uint_as_float(prmt(r.w.x, M, sel)) - 8388736.f) * sc;
      const float a1 = (__uint_as_float(prmt(r.w.y, M, sel)) - 8388736.f) * sc;
      const float b0 = (__uint_as_float(prmt(r.w.z, M, sel)) - 8388736.f) * sc;
      const float b1 = (__uint_as_float(prmt(r.w.w, M, sel)) - 8388736.f) * sc;
      out[2 * s] = bf2_bits(__floats2bfloat162_rn(a0, a1));
      out[2 * s + 1] = bf2_bits(__floats2bfloat162_rn(b0, b1));
    }
  } else if constexpr (FMT == kFmtIq2Lut) {
    const __nv_bfloat162 s2 = bits_bf2(r.s | (r.s << 16));
#pragma unroll
    for (int s = 0; s < 4; ++s) {
      const uint32_t w = (s < 2) ? r.w.x : r.w.y;
      const uint32_t sel = (s & 1) ? (w >> 16) : w;
      const uint32_t H = prmt(kLutHiPos, kLutHiNeg, sel);
      const uint32_t L = prmt(kLutLoPos, kLutLoNeg, sel);
      out[2 * s] = bf2_bits(__hmul2(bits_bf2(prmt(L, H, 0x5140)), s2));
      out[2 * s + 1] = bf2_bits(__hmul2(bits_bf2(prmt(L, H, 0x7362)), s2));
    }
  } else if constexpr (FMT == kFmtIq2N) {
    const int h = t & 1;
    const uint32_t sg = r.w.y;
    const float d = __half2float(__ushort_as_half(static_cast<unsigned short>(r.s)));
    const float db = d * (0.5f + static_cast<float>(sg >> 28)) * 0.25f;
    const __nv_bfloat162 s2 = __bfloat162bfloat162(__float2bfloat16_rn(db));
    const uint32_t ia = (r.w.x >> (16 * h)) & 0xFFu, ib = (r.w.x >> (16 * h + 8)) & 0xFFu;
    uint32_t pa = (sg >> (14 * h)) & 127u, pb = (sg >> (14 * h + 7)) & 127u;
    pa |= (__popc(pa) & 1u) << 7;
    pb |= (__popc(pb) & 1u) << 7;
    const uint4 ga = iq2_grid_entry<BANKED>(grid, ia);
    const uint4 gb = iq2_grid_entry<BANKED>(grid, ib);
    const uint32_t gw[8] = {ga.x, ga.y, ga.z, ga.w, gb.x, gb.y, gb.z, gb.w};
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint32_t pat = j < 4 ? pa : pb;
      out[j] = bf2_bits(__hmul2(bits_bf2(gw[j] ^ iq2_sign_mask(pat, j & 3)), s2));
    }
  } else {  // kFmtFp4: e2m1 pairs -> fp16x2 (hardware convert), times the e4m3 block scale
    uint32_t sh;
    asm("{\n .reg .b16 t16;\n cvt.u16.u32 t16, %1;\n cvt.rn.f16x2.e4m3x2 %0, t16;\n}\n" : "=r"(sh) : "r"(r.s));
    const __half2 s2 = __low2half2(bits_h2(sh));
    uint32_t p[8];
    asm("{\n .reg .b8 b0, b1, b2, b3, b4, b5, b6, b7;\n"
        " mov.b32 {b0, b1, b2, b3}, %8;\n mov.b32 {b4, b5, b6, b7}, %9;\n"
        " cvt.rn.f16x2.e2m1x2 %0, b0;\n cvt.rn.f16x2.e2m1x2 %1, b1;\n"
        " cvt.rn.f16x2.e2m1x2 %2, b2;\n cvt.rn.f16x2.e2m1x2 %3, b3;\n"
        " cvt.rn.f16x2.e2m1x2 %4, b4;\n cvt.rn.f16x2.e2m1x2 %5, b5;\n"
        " cvt.rn.f16x2.e2m1x2 %6, b6;\n cvt.rn.f16x2.e2m1x2 %7, b7;\n}\n"
        : "=r"(p[0]), "=r"(p[1]), "=r"(p[2]), "=r"(p[3]), "=r"(p[4]), "=r"(p[5]), "=r"(p[6]), "=r"(p[7])
        : "r"(r.w.x), "r"(r.w.y));
#pragma unroll
    for (int j = 0; j < 8; ++j) out[j] = h2_bits(__hmul2(bits_h2(p[j]), s2));
  }
}

// Raw (unscaled) decode for the block-column mode of R = 1 exact-weight GEMVs: the block
// scales are applied to the MMA results instead.
//   Q4:    bf16 (128 + n), PERM pairs -- the constant 136 is removed with the block sums of x
//   NVFP4: fp16 e2m1 values (exact), ADJ pairs
template <int FMT>
__device__ __forceinline__ void decode_row_raw(const RawRow& r, uint32_t (&out)[8]) {
  if constexpr (FMT == kFmtQ4) {
#pragma unroll
    for (int s = 0; s < 4; ++s) {
      out[2 * s] = ((r.w.x >> (4 * s)) & 0x000F000Fu) | 0x43004300u;
      out[2 * s + 1] = ((r.w.y >> (4 * s)) & 0x000F000Fu) | 0x43004300u;
    }
  } else {
    static_assert(FMT == kFmtFp4, "block-column mode exists for Q4 and NVFP4");
    asm("{\n .reg .b8 b0, b1, b2, b3, b4, b5, b6, b7;\n"
        " mov.b32 {b0, b1, b2, b3}, %8;\n mov.b32 {b4, b5, b6, b7}, %9;\n"
        " cvt.rn.f16x2.e2m1x2 %0, b0;\n cvt.rn.f16x2.e2m1x2 %1, b1;\n"
        " cvt.rn.f16x2.e2m1x2 %2, b2;\n cvt.rn.f16x2.e2m1x2 %3, b3;\n"
        " cvt.rn.f16x2.e2m1x2 %4, b4;\n cvt.rn.f16x2.e2m1x2 %5, b5;\n"
        " cvt.rn.f16x2.e2m1x2 %6, b6;\n cvt.rn.f16x2.e2m1x2 %7, b7;\n}\n"
        : "=r"(out[0]), "=r"(out[1]), "=r"(out[2]), "=r"(out[3]), "=r"(out[4]), "=r"(out[5]), "=r"(out[6]),
          "=r"(out[7])
        : "r"(r.w.x), "r"(r.w.y));
  }
}

// ---------------------------------------------------------------------------------------
// activation (B) fragments
// ---------------------------------------------------------------------------------------
// x16: the 16 consecutive bf16 of one activation row owned by this lane (as 8 pair words).
// Writes the 8 B registers of one chunk: b[2s], b[2s+1] for MMA s.
template <int FMT>
__device__ __forceinline__ void make_b_frags(const uint32_t (&x16)[8], uint32_t (&b)[8]) {
  if constexpr (FmtTraits<FMT>::kXLayout == kXPerm) {
    // word i holds k (2i, 2i+1).  MMA s: (s, s+4) and (8+s, 12+s).
#pragma unroll
    for (int s = 0; s < 4; ++s) {
      const int wa = s >> 1, wb = 2 + (s >> 1);  // words holding k s and s+4 / 8+s and 12+s
      const uint32_t sel = (s & 1) ? 0x7632u : 0x5410u;
      b[2 * s] = prmt(x16[wa], x16[wb], sel);
      b[2 * s + 1] = prmt(x16[4 + wa], x16[4 + wb], sel);
    }
  } else if constexpr (FmtTraits<FMT>::kF16) {
    // fp16 of x * 2^-6 (keeps |x| up to 4e6 finite; undone in the epilogue), adjacent pairs
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float lo = __uint_as_float(x16[i] << 16) * 0.015625f;
      const float hi = __uint_as_float(x16[i] & 0xFFFF0000u) * 0.015625f;
      b[i] = h2_bits(__floats2half2_rn(lo, hi));
    }
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) b[i] = x16[i];
  }
}

// Shared-memory B-fragment layout of the streaming kernels: an activation row is kept as
// 16-byte pieces (8 consecutive k); a lane's chunk operand is two pieces.  Converting a piece in
// place needs no other piece, so the conversion pass reads and writes conflict-free.
//   PERM (Q4, Q8): piece 0 of a lane's 16 k becomes (b0, b2, b4, b6), piece 1 (b1, b3, b5, b7);
//   fp16 (NVFP4): each bf16 pair becomes fp16 of x * 2^-6, in place;
//   ADJ bf16 (IQ2 LUT, native IQ2_XXS): the raw bf16 pairs are the operand.
template <int FMT>
__device__ __forceinline__ uint4 x_piece_to_frag(uint4 v) {
  if constexpr (FmtTraits<FMT>::kXLayout == kXPerm) {
    return make_uint4(prmt(v.x, v.z, 0x5410u), prmt(v.x, v.z, 0x7632u), prmt(v.y, v.w, 0x5410u),
                      prmt(v.y, v.w, 0x7632u));
  } else if constexpr (FmtTraits<FMT>::kF16) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
    uint32_t o[4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
      o[i] = h2_bits(__floats2half2_rn(__uint_as_float(w[i] << 16) * 0.015625f,
                                       __uint_as_float(w[i] & 0xFFFF0000u) * 0.015625f));
    return make_uint4(o[0], o[1], o[2], o[3]);
  } else {
    return v;
  }
}
template <int FMT>
__host__ __device__ constexpr bool x_needs_conversion() {
  return FmtTraits<FMT>::kXLayout == kXPerm || FmtTraits<FMT>::kF16;
}
// The 8 B registers of one chunk from its two converted pieces.
template <int FMT>
__device__ __forceinline__ void frag_from_pieces(uint4 p0, uint4 p1, uint32_t (&b)[8]) {
  if constexpr (FmtTraits<FMT>::kXLayout == kXPerm) {
    b[0] = p0.x; b[1] = p1.x; b[2] = p0.y; b[3] = p1.y;
    b[4] = p0.z; b[5] = p1.z; b[6] = p0.w; b[7] = p1.w;
  } else {
    b[0] = p0.x; b[1] = p0.y; b[2] = p0.z; b[3] = p0.w;
    b[4] = p1.x; b[5] = p1.y; b[6] = p1.z; b[7] = p1.w;
  }
}

template <bool F16>
__device__ __forceinline__ void mma16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  if constexpr (F16) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
                 : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
                 : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  } else {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
                 : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
                 : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  }
}

// One chunk of one 16-row tile: decode rows g and g+8, four MMAs.
template <int FMT>
__device__ __forceinline__ void mma_chunk(const uint8_t* row_g, const uint8_t* row_g8, const uint8_t* sc_g,
                                          const uint8_t* sc_g8, int c, int t, const uint32_t* grid,
                                          const uint32_t (&b)[8], float (&acc)[4]) {
  const RawRow ra = load_raw<FMT>(row_g, sc_g, c, t);
  const RawRow rb = load_raw<FMT>(row_g8, sc_g8, c, t);
  uint32_t da[8], db[8];
  decode_row<FMT>(ra, t, grid, da);
  decode_row<FMT>(rb, t, grid, db);
#pragma unroll
  for (int s = 0; s < 4; ++s)
    mma16816<FmtTraits<FMT>::kF16>(acc, da[2 * s], db[2 * s], da[2 * s + 1], db[2 * s + 1], b[2 * s], b[2 * s + 1]);
}

}  // namespace bolt
