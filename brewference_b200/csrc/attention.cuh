// attention.cuh — batch decode attention over the fp32 KV cache (host side).
#pragma once

#include "brew_common.cuh"

namespace brew {

struct AttnParams {
    int batch, n_heads, n_kv, hd, seq_len;
    int arch;                  // BREW_ARCH_*: selects QK-norm and RoPE layout
    int window;                // > 0: sliding window start = pos - window + 1
    int rope;                  // 1: rotate q and k (0: SmolLM3's no-RoPE layers)
    float eps, rope_base, rope_scale, inv_scale;
    const float* q;            // [batch][ldq]  (after bias)
    const float* k;            // [batch][ldkv]
    const float* v;
    int ldq, ldkv;
    const float* qnorm_w;      // [hd] or null (Qwen3 / Gemma3 QK-norm)
    const float* knorm_w;
    float* kcache;             // layer base of sequence 0; + b * cache_bstride
    float* vcache;
    int64_t cache_bstride;     // floats between sequences
    const int32_t* pos;        // [batch] device
    float* xb;                 // [batch][ldxb]
    int ldxb;
    float* part;               // [batch][n_heads][nchunk][hd + 2]
    int* counters;             // [batch][n_kv], zero, self-resetting
    int nchunk;                // CTAs per (sequence, kv head)
    uint8_t* prep_out;         // prep records of xb (K = n_heads*hd) for wo
    unsigned int* err;
};

int attn_launch(const AttnParams& p, cudaStream_t stream, bool pdl);
int attn_pick_nchunk(int n_kv, int batch, int seq_len);
size_t attn_part_floats(int batch, int n_heads, int nchunk, int hd);

}  // namespace brew
