// packed.cu — builds fragment-packed tiles from GGUF rows (layout in packed.cuh).
#include "packed.cuh"

namespace brew {
namespace {

// GGUF row of packed row r (0..15) of tile `tile` of layer l, or null (zero row).
__device__ const uint8_t* pk_src_row(const PackSpec& s, int l, int tile, int r, int row_bytes) {
    if (s.mode == PK_GLU) {
        const int i = tile * 8 + (r & 7);
        const uint8_t* base = s.src[r >> 3];
        return base + ((int64_t)l * s.rows[0] + i) * row_bytes;
    }
    int row = tile * 16 + r;
    for (int k = 0; k < 3; ++k) {
        if (row < s.rows[k]) return s.src[k] + ((int64_t)l * s.rows[k] + row) * row_bytes;
        row -= s.rows[k];
    }
    return nullptr;
}

// One warp per (layer, tile, kb): lane (g, t) writes its fragment bytes, lanes
// t == 0 the scale word of rows g and g + 8.
__global__ void pack_tiles_kernel(uint8_t* dst, const PackSpec s, int tiles) {
    const int lane = threadIdx.x & 31;
    const int64_t wid = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int KB = s.K / 32;
    const int64_t total = (int64_t)s.layers * tiles * KB;
    if (wid >= total) return;
    const int kb = (int)(wid % KB);
    const int tile = (int)((wid / KB) % tiles);
    const int l = (int)(wid / ((int64_t)KB * tiles));
    const bool q8 = s.type == BREW_TYPE_Q8_0;
    const int bb = q8 ? 34 : 18;
    const int row_bytes = KB * bb;
    const int g = lane >> 2, t = lane & 3;
    const uint8_t* r0 = pk_src_row(s, l, tile, g, row_bytes);
    const uint8_t* r1 = pk_src_row(s, l, tile, g + 8, row_bytes);
    uint8_t* out = dst + ((((int64_t)l * tiles + tile) * KB) + kb) * pk_block_bytes(s.type);
    auto byte_at = [&](const uint8_t* row, int off) -> uint8_t { return row ? row[(int64_t)kb * bb + off] : 0; };
    if (q8) {
        uint8_t* o = out + lane * 16;
        for (int i = 0; i < 4; ++i) {
            o[i] = byte_at(r0, 2 + 4 * t + i);
            o[4 + i] = byte_at(r1, 2 + 4 * t + i);
            o[8 + i] = byte_at(r0, 2 + 16 + 4 * t + i);
            o[12 + i] = byte_at(r1, 2 + 16 + 4 * t + i);
        }
    } else {
        uint8_t* o = out + lane * 8;
        for (int i = 0; i < 4; ++i) {
            o[i] = byte_at(r0, 2 + 4 * t + i);
            o[4 + i] = byte_at(r1, 2 + 4 * t + i);
        }
    }
    if (t == 0) {
        uint8_t* o = out + pk_scale_off(s.type) + g * 4;
        o[0] = byte_at(r0, 0);
        o[1] = byte_at(r0, 1);
        o[2] = byte_at(r1, 0);
        o[3] = byte_at(r1, 1);
    }
}

}  // namespace

int pack_tiles_launch(uint8_t* dst, const PackSpec& spec, cudaStream_t stream) {
    BREW_CHECK(spec.type == BREW_TYPE_Q8_0 || spec.type == BREW_TYPE_Q4_0, BREW_ERR_UNSUPPORTED,
               "packed tiles: Q8_0 or Q4_0 only");
    BREW_CHECK(spec.K % 32 == 0 && spec.layers >= 1, BREW_ERR_INVALID_ARG, "packed tiles: bad shape");
    BREW_CHECK(spec.mode != PK_GLU || spec.rows[0] % 8 == 0, BREW_ERR_INVALID_ARG, "packed tiles: GLU rows % 8");
    const int tiles = pk_tiles(spec);
    const int64_t warps = (int64_t)spec.layers * tiles * (spec.K / 32);
    const int64_t blocks = (warps * 32 + 255) / 256;
    pack_tiles_kernel<<<(unsigned)blocks, 256, 0, stream>>>(dst, spec, tiles);
    BREW_CUDA(cudaGetLastError());
    return BREW_OK;
}

}  // namespace brew
