// prefill.cuh — batched prompt prefill: the T tokens of a prompt chunk go
// through each layer together, with the matrix products on the tcgen05 GEMM
// (gemm.cuh) instead of T matrix-vector products.
//
// The reference prefills token by token (GenericModelSession.prefill,
// runtime/ModelRunner.java:196-206: forward(prompt[i], i) for each i), and
// the only state that survives a prefill is the KV cache: the logits of
// prompt tokens are never read.  So the batched prefill produces exactly
// that state: for every layer the K / V rows of positions pos0 .. pos0+T-1.
// The per-element arithmetic (RMSNorm, head norm, RoPE, SwiGLU / GeGLU,
// residuals) is the same as the token-by-token path; the fp32 summation
// order of the dot products differs (results agree to fp32 rounding).
#pragma once

#include "brew_common.cuh"

namespace brew {

// x[t][i] = dequant(embed row tokens[t])[i] (* sqrt(dim) for Gemma3,
// Kernels.scaleEmbeddings), t < T.
int prefill_embed_launch(int type, const uint8_t* embed, int vocab, int dim, const int32_t* tokens, int T, bool gemma,
                         float* x, unsigned int* err, cudaStream_t s);

// Per token row t (position pos0 + t) of qkv = [q heads | k heads | v heads]:
// head-wise RMSNorm of q and k (Qwen3 / Gemma3, Kernels.headWiseRmsNorm),
// RoPE of q and k from the tables (RopeCache), q written back in place, k
// and v appended to the layer's cache rows (AttentionEngine.storeKeyValueInCache).
struct PfQkParams {
    int T, pos0, n_heads, n_kv, hd, seq_len;
    int table;                    // RoPE table: 0 global / default base, 1 Gemma3 local
    bool interleaved;             // Llama pairs (2d, 2d+1); others (d, d + hd/2)
    bool rope;                    // rotate q and k (false: SmolLM3's no-RoPE layers)
    float eps;
    float* qkv;                   // [T][ldq]
    int ldq;
    const float *qnorm_w, *knorm_w;   // [hd] each, or null
    const float *rope_cos, *rope_sin; // [2][seq_len][hd/2]
    float *kcache, *vcache;       // this layer, sequence 0: [seq_len][n_kv * hd]
};
int prefill_qk_launch(const PfQkParams& p, cudaStream_t s);

// Causal attention of the T query rows (positions pos0 + t) over the cache
// rows start .. pos0 + t (start = pos - window + 1 for Gemma3's local layers)
// (AttentionEngine.attend, transformer/attention/AttentionEngine.java:40-106):
// scores q.k / sqrt(hd), softmax, weighted sum of the values, with the
// softmax taken online over 32-position tiles.
struct PfAttnParams {
    int T, pos0, n_heads, n_kv, hd, window;
    float inv_scale;
    const float* q;               // [T][ldq], RoPE'd
    int ldq;
    const float *kcache, *vcache; // this layer, sequence 0
    float* xb;                    // [T][ldxb]
    int ldxb;
};
int prefill_attn_launch(const PfAttnParams& p, cudaStream_t s);

// Shapes the two kernels above take: hd in {64, 128, 256}, n_heads / n_kv <= 32.
bool prefill_shapes_supported(int n_heads, int n_kv, int hd);

}  // namespace brew
