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

// K / V positions an attention item stages in shared memory per round.
__host__ __device__ inline int attn_sub(int hd) { return hd <= 128 ? 32 : 16; }

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
    float *x0, *x1;                     // residual stream (Gemma3 alternates between the two)
    float *xb, *xb2, *qkv, *hb, *logits;
    float* attn_part;                   // [batch][n_heads][nchunk][hd + 4]: m, l, -, -, o[hd]
    int* attn_ctr;
    int nchunk, attn_floats;            // attn_floats: shared-memory floats of the attention area
    unsigned long long* am_key;
    int32_t* am_out;
    const int32_t *tokens, *pos;
    unsigned long long* bar;            // [0] arrival counter, [1] its value at step start
    int* abort;
    unsigned int* err;
    unsigned long long* trace;          // optional [grid][trace_slots]: %globaltimer per CTA
    int trace_slots;                    // 1 + 5 per phase (load wave landed, prep done, last weight stage in, work done, barrier passed)
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
