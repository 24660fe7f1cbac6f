// decode.cuh — one decode step of the whole model as one persistent kernel.
#pragma once

#include <cuda.h>

#include "brew_common.cuh"

namespace brew {

// tensor maps of the weight families (all layers concatenated)
enum { DK_MAP_Q = 0, DK_MAP_K, DK_MAP_V, DK_MAP_O, DK_MAP_GATE, DK_MAP_UP, DK_MAP_DOWN, DK_MAP_OUT, DK_NMAPS };

constexpr int DK_MAX_BATCH = 2;

struct alignas(64) DecodeParams {
    CUtensorMap maps[DK_NMAPS];
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
    float *x0, *x1;                     // residual stream (Gemma3 alternates between the two)
    float *xb, *xb2, *qkv, *hb, *logits;
    float* attn_part;
    int* attn_ctr;
    int nchunk;
    unsigned long long* am_key;
    int32_t* am_out;
    const int32_t *tokens, *pos;
    unsigned long long* bar;            // [0] arrival counter, [1] its value at step start
    int* abort;
    unsigned int* err;
    unsigned long long* trace;          // optional [grid][trace_slots]: %globaltimer per CTA
    int trace_slots;                    // 1 + 3 per phase (prep done, work done, barrier passed)
    // launch geometry
    int nstages, stage_bytes, vec_bytes, prep_bytes, rec_bytes, nb_cap, grid;
    size_t smem;
};

// True when the model can run on the persistent decode kernel.
bool decode_supported(const brew_config& c, int batch);
// Fills the geometry fields and the tensor maps (maps need `w` pointers).
int decode_prepare(DecodeParams* p, const uint8_t* wq, const uint8_t* wk, const uint8_t* wv, const uint8_t* wo,
                   const uint8_t* wgate, const uint8_t* wup, const uint8_t* wdown, const uint8_t* wout);
int decode_launch(const DecodeParams& p, cudaStream_t stream);
// RoPE cos/sin tables [2][seq_len][hd/2] (RopeCache.precomputeAngles per position).
int rope_tables_launch(float* cos_t, float* sin_t, int seq_len, int hd, float base0, float base1, float scale,
                       cudaStream_t stream);

}  // namespace brew
