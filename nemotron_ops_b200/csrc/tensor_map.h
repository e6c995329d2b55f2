// Tensor-map (TMA descriptor) helpers for streaming row tiles of weights with a 128-byte swizzle.
//
// A weight matrix of `rows` rows of `row_bytes` bytes (row_bytes % 128 == 0) is described as the
// 3-D tensor (128-byte piece, row, piece index) with strides (1, row_bytes, 128).  A box of
// (128, BR rows, S pieces) lands in shared memory as [piece][row][128 B]; with the 128-byte
// swizzle, the 16-byte chunks of smem line L are permuted by XOR with (L & 7), and line
// L = piece * BR + row (BR a multiple of 8), so eight consecutive rows of one piece sit in eight
// different bank groups.  One request moves a whole (BR x S*128)-byte stage.
#pragma once

#include <cuda.h>
#include <stdint.h>

#include "common.cuh"

namespace bolt {

// Rows whose size is not a multiple of 128 bytes use 16-byte pieces without swizzle instead:
// [piece][row][16 B] interleaves the rows at 16-byte granularity, which is just as free of bank
// conflicts for 8- and 16-byte lane loads.
//
// 64-byte pieces use the 64-byte swizzle: [piece][row][64 B] with the 16-byte chunks of each
// row permuted by XOR with ((row >> 1) & 3), which spreads eight consecutive rows over the banks.
//
// Encodes (or returns the cached) map of `base` viewed as above with a box of
// (piece_bytes, box_rows, pieces); piece_bytes is 128 or 64 (swizzled) or 16 (plain), box_rows
// up to 256 (swz_off below assumes a multiple of 8; swz_line_off takes any count).
// Returns false when the view cannot be encoded.
bool row_tile_map(CUtensorMap* out, const void* base, int64_t rows, int64_t row_bytes, int pieces, int piece_bytes,
                  int box_rows);

// smem byte offset of byte `b` of row `r` in a tile of `br` rows written by a row_tile_map box
__device__ __forceinline__ uint32_t swz_off(int r, int b, int br) {
  return static_cast<uint32_t>((((b >> 7) * br + r) << 7) | ((((b >> 4) & 7) ^ (r & 7)) << 4) | (b & 15));
}
// as swz_off for a box of any row count: the swizzle phase is the smem line index
__device__ __forceinline__ uint32_t swz_line_off(int r, int b, int br) {
  const int line = (b >> 7) * br + r;
  return static_cast<uint32_t>((line << 7) | ((((b >> 4) & 7) ^ (line & 7)) << 4) | (b & 15));
}
__device__ __forceinline__ uint32_t p16_off(int r, int b, int br) {
  return static_cast<uint32_t>((((b >> 4) * br + r) << 4) | (b & 15));
}
// sw: 1 = 128-byte swizzled pieces, 0 = 16-byte pieces
__device__ __forceinline__ uint32_t tile_off(int sw, int r, int b, int br) {
  return sw ? swz_off(r, b, br) : p16_off(r, b, br);
}

// Pulls a tensor map into the descriptor cache ahead of its first use.
__device__ __forceinline__ void prefetch_tensor_map(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, int c0, int c1, int c2,
                                            uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
      "[%5];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(bar)
      : "memory");
}

}  // namespace bolt
