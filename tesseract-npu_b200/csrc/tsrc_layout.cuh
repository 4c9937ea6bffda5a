// tsrc_layout.cuh -- the device weight layout shared by upload, download, synthesis and matvec.
//
// Each row of a shard is cut into tiles of 16 blocks (Q8_0: 16 x 32 weights) or 16 superblocks
// (Q4_K: 16 x 256 weights); the last tile of a row is zero-padded. Inside a tile the quants are
// stored chunk-major: 16-byte chunk j of block b sits at tile + 256 j + 16 b. One warp reads the
// same chunk of 16 blocks of two rows with one 128-bit load per lane, i.e. two fully used
// 256-byte segments, and lane b then owns block b of its row entirely (no cross-lane sums).
//   Q8_0: qs tile 2 x 256 B (32 quants per block), meta tile 16 fp16 d (32 B)
//   Q4_K: qs tile 8 x 256 B (128 quant bytes per superblock), meta tile 16 x 16 B
//         {d, dmin, scales[12]} (the ggml superblock's first 16 bytes, unchanged)
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
    __host__ __device__ uint32_t chunks() const { return fmt == 0 ? 2u : 8u; }     // 16-B chunks per block
    __host__ __device__ size_t qs_tile_bytes() const { return (size_t)chunks() * 256u; }
    __host__ __device__ size_t meta_entry_bytes() const { return fmt == 0 ? 2u : 16u; }
    __host__ __device__ size_t qs_row_bytes() const { return qs_tile_bytes() * tiles(); }
    __host__ __device__ size_t meta_row_bytes() const { return meta_entry_bytes() * 16u * tiles(); }
    // byte offsets (within the shard) of chunk j of block b of row r, and of its meta entry
    __host__ __device__ size_t qs_off(uint32_t r, uint32_t b, uint32_t j) const {
        return (size_t)r * qs_row_bytes() + (size_t)(b >> 4) * qs_tile_bytes() + 256u * j + 16u * (b & 15u);
    }
    __host__ __device__ size_t meta_off(uint32_t r, uint32_t b) const {
        return (size_t)r * meta_row_bytes() + (size_t)b * meta_entry_bytes();
    }
};

}  // namespace tsrc
