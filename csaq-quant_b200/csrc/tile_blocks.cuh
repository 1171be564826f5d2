// Geometry of the GEMV block layout of a tier (csaq_repack_tiles): one block
// per (unit, 128-column chunk), unit-major; a unit is 2 tiles of 16 rows for
// 2- and 4-bit tiers and 1 tile otherwise. Inside a block, tile mt starts at
// mt * tile_block_bytes: its codes (code_bytes), then the 16 rows' fp32 scales
// (64 B) and uint8 zero points (16 B) of the chunk's group.
#pragma once

namespace csaq {

constexpr int kTileRows = 16;

__host__ __device__ __forceinline__ constexpr int unit_tiles(int bits) { return (bits == 2 || bits == 4) ? 2 : 1; }
__host__ __device__ __forceinline__ constexpr int code_bytes(int bits) {  // one tile x one chunk
  return bits == 2 ? 512 : bits == 4 ? 1024 : bits == 8 ? 2048 : 4096;
}
__host__ __device__ __forceinline__ constexpr int tile_block_bytes(int bits) {
  return bits == 16 ? 4096 : (code_bytes(bits) + 80 + 15) / 16 * 16;
}
__host__ __device__ __forceinline__ constexpr int chunk_bytes(int bits) {  // one unit x one chunk
  return unit_tiles(bits) * tile_block_bytes(bits);
}

}  // namespace csaq
