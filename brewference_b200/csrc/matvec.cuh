// matvec.cuh — quantized matvec over unchanged GGUF blocks (host interface).
#pragma once

#include <cuda.h>

#include "brew_common.cuh"

namespace brew {

constexpr int MV_TILE_ROWS = 16;        // rows per tile (one m16 MMA row block)
constexpr int MV_CONSUMER_WARPS = 8;
constexpr int MV_THREADS = (MV_CONSUMER_WARPS + 1) * 32;
constexpr int MV_MAX_BOXES = 8;         // TMA boxes (16 rows x kcb blocks) per stage
constexpr int MV_MAX_BATCH = 16;        // per launch; larger batches loop on the host
constexpr int MV_ARGMAX_MAX_BATCH = 16;

enum MvEpi { MV_EPI_STORE = 0, MV_EPI_GLU_SILU = 1, MV_EPI_GLU_GELU = 2 };
enum MvPost { MV_POST_NONE = 0, MV_POST_PREP = 1, MV_POST_ARGMAX = 2 };

// How a stage reaches shared memory:
//   TMA     cp.async.bulk.tensor.2d boxes of 16 rows x kcb blocks through a
//           tensor map (row pitch a multiple of 16 bytes); rows past the
//           matrix read as zeros
//   CONTIG  a tile of whole rows is contiguous: one bulk copy per region
//   ROW     one bulk copy per row (any pitch)
enum MvMode { MV_MODE_ROW = 0, MV_MODE_CONTIG = 1, MV_MODE_TMA = 2 };

// One weight matrix feeding the launch.  Tiles never straddle segments.
struct MvSeg {
    const uint8_t* w;     // packed rows of this matrix (already at its layer)
    float* y;             // output [batch][ldy]
    const float* bias;    // [rows] added to the output, or null
    const float* resid;   // [batch][ldy] residual: y = resid + v, or null
    int rows;             // output rows (GLU: output indices)
    int tile0;            // first tile of this segment
};

struct alignas(64) MvParams {
    CUtensorMap tmap[3];       // MV_MODE_TMA: one map per segment (GLU: gate, up)
    MvSeg seg[3];
    int nseg;
    int type;
    int K, KB;                 // columns, blocks per row
    int64_t row_bytes;
    int batch, ldy;
    int epi;
    int total_tiles;
    int mode, kcb, nb_cap;     // staging mode; blocks per TMA box / ROW chunk; boxes per tile cap
    int nstages, stage_bytes, stage_w;
    int region_stride, slot_pitch;
    const uint8_t* prep;       // prep records of x, [KB][rec_bytes]
    int rec_bytes;
    // GLU: emit prep records of the output for the next matvec
    uint8_t* next_prep;
    int* group_counters;       // [rows/32], zero, self-resetting
    // pass run by the last CTA to finish
    int post;
    int* post_counter;
    float* post_x;             // vector updated/normalised by the post pass [batch][post_ld]
    int post_ld, post_dim;
    const float* post_add;     // Gemma: post_x += rmsnorm(post_add, post_add_w)
    const float* post_add_w;
    const float* post_norm_w;  // prep(rmsnorm(post_x, post_norm_w)) -> post_prep
    float eps;
    uint8_t* post_prep;
    // argmax (classifier): 64-bit keys reduced with atomicMax, decoded by the
    // last CTA, which also clears them
    unsigned long long* am_key;   // [batch], zero
    int32_t* am_out;              // [batch]
    unsigned int* err;
};

// Fills the derived launch fields (KC, stages, smem, staging mode, tensor
// maps) and launches.
int mv_launch(MvParams p, cudaStream_t stream, bool pdl);

// x [batch][K] (fp32, device) -> prep records, optionally RMS-normalised.
int prep_launch(const float* x, int ldx, int K, int batch, const float* norm_w, float eps, uint8_t* recs,
                cudaStream_t stream, bool pdl);

int num_sms();

// Tensor map over `rows` rows of `pitch` bytes viewed as 8-byte elements,
// with a box of `box_bytes` x `box_rows` (rows past the end read as zeros).
int encode_rows_map(CUtensorMap* map, const void* base, int rows, int pitch, int box_bytes, int box_rows);

}  // namespace brew
