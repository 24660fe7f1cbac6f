// decode.cuh — one decode step of the whole model as one persistent kernel.
#pragma once

#include <cuda.h>

#include "brew_common.cuh"
#include "packed.cuh"

namespace brew {

// weight families of the decode kernel, each a fragment-packed copy
// (packed.cuh) of all layers: Q|K|V rows, wo, gate/up interleaved, down, and
// the classifier
enum { PK_QKV = 0, PK_O, PK_GU, PK_DOWN, PK_OUT, PK_NFAM };

constexpr int DK_MAX_BATCH = 2;
constexpr int DK_DETAIL = 32;   // chunks of the detailed phase traced

// The vectors one layer's phases hand to each other (tagged words): the
// layer's input residual, Q|K|V, the attention output, the residual after
// attention, the gated FFN activation, and Gemma's wo / down outputs before
// their post-norms.  XIN of layer n_layers is the classifier's input.
enum { DK_TG_XIN = 0, DK_TG_QKV, DK_TG_XB, DK_TG_XMID, DK_TG_HB, DK_TG_XB2O, DK_TG_XB2D, DK_TG_N };

// Word offsets of the tagged vectors in a layer's sequence row; returns the
// row length (every vector starts on a 4-word boundary).
inline int dk_tagged_layout(int dim, int qkvw, int qw, int hidden, int* off) {
    const int len[DK_TG_N] = {dim, qkvw, qw, dim, hidden, dim, dim};
    int o = 0;
    for (int v = 0; v < DK_TG_N; ++v) {
        off[v] = o;
        o += (len[v] + 3) & ~3;
    }
    return o;
}

// K / V positions an attention item stages in shared memory per round, at
// least (decode_prepare widens it to what the attention area holds).
__host__ __device__ inline int attn_sub(int hd) { return hd <= 128 ? 32 : 16; }
// ... and at most: the warp-level rounds give each of the 8 consumer warps
// this many positions / 8 of a round.
__host__ __device__ inline int attn_sub_max(int hd) { return hd <= 128 ? 48 : 16; }

struct alignas(64) DecodeParams {
    const uint8_t* pk[PK_NFAM];         // packed weights
    int64_t pk_lb[PK_NFAM];             // bytes per layer of each family
    // dimensions
    int arch, dim, hidden, n_layers, n_heads, n_kv, hd, vocab, seq_len, window, batch;
    int type_layer, type_out;
    float eps, inv_scale;
    // weights
    const uint8_t* embed;
    int type_embed;
    const float *rms_att, *rms_ffn, *rms_final, *post_att, *post_ffn, *rms_q, *rms_k;
    const float *q_bias, *k_bias, *v_bias;
    // state
    float *kc, *vc;
    int64_t cache_bstride;
    const float *rope_cos, *rope_sin;   // [2][seq_len][hd/2]: 0 = global/default base, 1 = Gemma3 local
    // Tagged activations: [n_layers + 1][DK_MAX_BATCH][tg_ls] words, each
    // (epoch << 32) | float bits; vector v of layer l starts at word
    // tg_off[v] of the layer's sequence row (dk_tagged_layout)
    unsigned long long* tg;
    int tg_ls;
    int tg_off[DK_TG_N];
    float* logits;
    float* attn_part;                   // [2 (layer parity)][DK_MAX_BATCH][n_heads][nchunk][hd + 4]: m, l, -, -, o[hd]
    int* attn_ctr;                      // [2 (epoch parity)][n_layers][DK_MAX_BATCH][n_kv] arrival counters
    int nchunk, attn_floats;            // attn_floats: shared-memory floats of the attention area
    int attn_sub;                       // K / V positions staged per round
    unsigned long long* am_key;
    int32_t* am_out;
    const int32_t *tokens, *pos;
    // One-sequence calls from the host may pass the token and position as
    // launch parameters instead (use_imm = 1): no upload precedes the launch.
    int use_imm, tok_imm, pos_imm;
    // optional mapped pinned host memory: the last CTA writes [0] the argmax
    // id and then [1] the device error word, so a host caller needs no copy
    int32_t* host_out;
    unsigned int* seq;                  // epoch of the last completed launch
    int* done;                          // CTAs done with this launch (the last one finishes the step)
    int* abort;
    unsigned int* err;
    unsigned long long* trace;          // optional [grid][trace_slots]: %globaltimer per CTA
    int trace_slots;                    // 1 + 5 per phase (load wave landed, prep done, last weight stage in, work done, phase end)
    int detail_l, detail_ph;            // optional per-chunk trace of one (layer, phase): 3 x DK_DETAIL more slots
    // launch geometry
    int nstages, stage_bytes, vec_bytes, prep_bytes, rec_bytes, grid;
    size_t smem;
    // stage geometry per matvec phase (PH_QKV .. PH_CLS): tiles per group
    // for a CTA owning nt tiles (index min(nt, 9)), and block columns per
    // stage for a group of ng tiles (index ng <= 8)
    int8_t geo_gs[5][10];
    int16_t geo_kc[5][9];
    int16_t geo_nch[5][9];              // chunks of a group: KB / geo_kc
};

// True when the model can run on the persistent decode kernel.
bool decode_supported(const brew_config& c, int batch);
// Fills the shared-memory geometry fields (needs the dimensions, batch and nchunk).
int decode_prepare(DecodeParams* p);
int decode_launch(const DecodeParams& p, cudaStream_t stream);
// RoPE cos/sin tables [2][seq_len][hd/2] (RopeCache.precomputeAngles per position).
int rope_tables_launch(float* cos_t, float* sin_t, int seq_len, int hd, float base0, float base1, float scale,
                       cudaStream_t stream);

}  // namespace brew
