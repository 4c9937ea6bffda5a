// tsrc_layout.cuh -- the device weight layout shared by upload, download, synthesis and matvec.
//
// Each row of a shard is cut into tiles of 16 blocks (Q8_0: 16 x 32 weights) or 16 superblocks
// (Q4_K: 16 x 256 weights); the last tile of a row may hold fewer (nv) blocks. Inside a tile the
// quants are stored chunk-major: 16-byte chunk j of block b sits at tile + 16 nv j + 16 (b mod 16).
// So one warp reads the same chunk of 16 blocks of two rows as two fully used 256-byte segments,
// lane b then owns block b of its row entirely (no cross-lane sums), and rows stay compact (a row
// holds exactly its ggml quant bytes, so tile ranges and whole rows are contiguous byte ranges
// that bulk copies can move).
//   Q8_0: 32 quant bytes (2 chunks) per block; meta = fp16 d per block, row padded to 16 bytes
//   Q4_K: 128 quant bytes (8 chunks) per superblock; meta = its 16 bytes {d, dmin, scales[12]}
// The reference keeps its own FPGA beat layout (jwkim04/tesseract-npu sw/sim/tsr_ref.c:255-333);
// both are pure byte permutations of the ggml rows.
#pragma once

#include <stddef.h>
#include <stdint.h>

namespace tsrc {

struct Layout {
    uint32_t fmt, K;
    __host__ __device__ uint32_t blocks() const { return fmt == 0 ? K / 32u : K / 256u; }
    __host__ __device__ uint32_t tiles() const { return (blocks() + 15u) / 16u; }
    __host__ __device__ uint32_t chunks() const { return fmt == 0 ? 2u : 8u; }        // 16-B chunks per block
    __host__ __device__ uint32_t block_qs_bytes() const { return 16u * chunks(); }
    __host__ __device__ uint32_t tile_blocks(uint32_t t) const {                      // nv of tile t
        const uint32_t r = blocks() - 16u * t;
        return r < 16u ? r : 16u;
    }
    __host__ __device__ size_t meta_entry_bytes() const { return fmt == 0 ? 2u : 16u; }
    __host__ __device__ size_t qs_row_bytes() const { return (size_t)blocks() * block_qs_bytes(); }
    __host__ __device__ size_t meta_row_bytes() const { return ((size_t)blocks() * meta_entry_bytes() + 15u) & ~(size_t)15u; }
    // byte offsets (within the shard) of chunk j of block b of row r, and of its meta entry
    __host__ __device__ size_t qs_off(uint32_t r, uint32_t b, uint32_t j) const {
        const uint32_t t = b >> 4;
        return (size_t)r * qs_row_bytes() + (size_t)t * 16u * block_qs_bytes() + 16u * tile_blocks(t) * j + 16u * (b & 15u);
    }
    __host__ __device__ size_t meta_off(uint32_t r, uint32_t b) const {
        return (size_t)r * meta_row_bytes() + (size_t)b * meta_entry_bytes();
    }
};

}  // namespace tsrc
