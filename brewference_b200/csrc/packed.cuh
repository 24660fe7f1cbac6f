// packed.cuh — "fragment-packed tiles": the decode kernel's HBM layout of a
// quantized weight matrix.
//
// GGUF rows store a 32-element block as fp16 scale + quants (Q8_0: 2 + 32
// bytes, Q4_0: 2 + 16), so inside a row the quants sit at 2-byte offsets and
// one MMA fragment of 16 rows x 32 elements is spread over 16 rows of the
// matrix.  The decode kernel instead reads the weights in the order the
// int8 tensor-core MMA (m16n8k32) consumes them.  For every tile of 16 rows
// and every block column kb, one "block-tile" holds
//     Q8_0 (544 bytes): [32 lanes][16 bytes]  lane (g, t) = row g quants 4t..4t+3,
//                                              row g+8 4t..4t+3, row g 16+4t..,
//                                              row g+8 16+4t..   (the A fragment)
//                       [8][2] fp16 scales     word g = (d of row g, d of row g+8)
//     Q4_0 (288 bytes): [32 lanes][8 bytes]   lane (g, t) = row g nibble bytes 4t..4t+3,
//                                              row g+8 nibble bytes 4t..4t+3
//                       [8][2] fp16 scales
// (the Q4_0 low nibbles of bytes 4t..4t+3 are elements 4t..4t+3 and the high
// nibbles elements 16+4t.., exactly the a0/a2 halves of the fragment).  The
// block-tiles of one tile are contiguous over kb ([tile][kb][bytes]), so a
// stage of the pipeline is one bulk copy per tile.  Same bytes as the GGUF
// rows (16 * 34 = 544, 16 * 18 = 288): the packing moves bytes, it changes
// no value.
#pragma once

#include "brew_common.cuh"

namespace brew {

__host__ __device__ constexpr int pk_block_bytes(int type) { return type == BREW_TYPE_Q8_0 ? 544 : 288; }
__host__ __device__ constexpr int pk_scale_off(int type) { return type == BREW_TYPE_Q8_0 ? 512 : 256; }

// Row sources of a packed family.
//   PK_ROWS: tile rows are the concatenation of up to three matrices
//            (rows[0] rows of src[0], then src[1], then src[2]); rows past
//            the end are zero (scale 0).
//   PK_GLU:  tile i = rows 8i..8i+7 of src[0] (gate) then the same rows of
//            src[1] (up); rows[0] = rows of each.
enum { PK_ROWS = 0, PK_GLU = 1 };

struct PackSpec {
    const uint8_t* src[3];
    int rows[3];          // rows of each source per layer
    int mode, type, K, layers;
};

// Tiles of one layer of a packed family.
inline int pk_tiles(const PackSpec& s) {
    if (s.mode == PK_GLU) return s.rows[0] / 8;
    return (s.rows[0] + s.rows[1] + s.rows[2] + 15) / 16;
}
inline size_t pk_layer_bytes(const PackSpec& s) {
    return (size_t)pk_tiles(s) * (s.K / 32) * pk_block_bytes(s.type);
}

// Writes the packed copy of all layers of a family to dst
// (layers * pk_layer_bytes bytes).
int pack_tiles_launch(uint8_t* dst, const PackSpec& spec, cudaStream_t stream);

}  // namespace brew
