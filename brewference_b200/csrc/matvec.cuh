// matvec.cuh — quantized matvec over unchanged GGUF blocks (host interface).
#pragma once

#include "brew_common.cuh"

namespace brew {

constexpr int MV_TILE_ROWS = 16;        // rows per tile (one m16 MMA row block)
constexpr int MV_CONSUMER_WARPS = 8;    // split a tile's blocks 8 ways
constexpr int MV_THREADS = (MV_CONSUMER_WARPS + 1) * 32;
constexpr int MV_MAX_PARTS = 4;         // CTAs that may share one tile (stream-K)
constexpr int MV_MAX_BATCH = 32;        // per launch; larger batches loop on the host
constexpr int MV_ARGMAX_MAX_BATCH = 16;

enum MvEpi { MV_EPI_STORE = 0, MV_EPI_GLU_SILU = 1, MV_EPI_GLU_GELU = 2 };
enum MvPost { MV_POST_NONE = 0, MV_POST_PREP = 1, MV_POST_ARGMAX = 2 };

// One weight matrix feeding the launch.  Tiles never straddle segments.
struct MvSeg {
    const uint8_t* w;     // packed rows of this matrix (already at its layer)
    float* y;             // output [batch][ldy]
    const float* bias;    // [rows] added to the output, or null
    const float* resid;   // [batch][ldy] residual: y = resid + v, or null
    int rows;             // output rows (GLU: output indices)
    int tile0;            // first tile of this segment
};

struct MvParams {
    MvSeg seg[3];
    int nseg;
    int type;
    int K, KB, KC, nchunks;    // columns, blocks per row, blocks per stage, stages per tile
    int64_t row_bytes;
    int batch, ldy;
    int epi;
    int total_tiles, units;    // units = total_tiles * nchunks
    int nstages, stage_bytes, slot_pitch;
    const uint8_t* prep;       // prep records of x, [KB][rec_bytes]
    int rec_bytes;
    // stream-K scratch
    float* part_buf;           // [grid][MV_MAX_PARTS][16*batch], by first CTA of a split tile
    int* tile_counters;        // [grid], zero, self-resetting
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
    // argmax (classifier): per-CTA partials then the last CTA reduces
    float* am_val;             // [gridDim][batch]
    int* am_idx;
    int32_t* am_out;           // [batch]
    unsigned int* err;
};

// Fills the derived launch fields (KC, stages, smem) and launches.
int mv_launch(MvParams p, cudaStream_t stream, bool pdl);

// Floats of stream-K part buffer a launch of `grid` CTAs needs.
size_t mv_part_floats(int grid, int batch);

// x [batch][K] (fp32, device) -> prep records, optionally RMS-normalised.
int prep_launch(const float* x, int ldx, int K, int batch, const float* norm_w, float eps, uint8_t* recs,
                cudaStream_t stream, bool pdl);

int num_sms();

}  // namespace brew
