// misc.cuh — small kernels: embedding + prep, dequantization, synthetic
// weights, argmax.
#pragma once

#include "brew_common.cuh"

namespace brew {

// x[b] = dequant(embed row tokens[b]) (* sqrt(dim) for Gemma3), then the prep
// records of rmsnorm(x[b], norm_w) for the first projection.
int embed_prep_launch(int type, const uint8_t* embed, int vocab, int dim, const int32_t* tokens, int batch,
                      bool gemma_scale, float* x, const float* norm_w, float eps, uint8_t* prep, unsigned int* err,
                      cudaStream_t stream, bool pdl);

// out[i] = dequant(element elem_offset + i), bit-exact with the GGML formulas.
int dequant_launch(int type, const uint8_t* w, int64_t elem_offset, int64_t n, float* out, cudaStream_t stream);

// Seeded N(0, std) values of tensor `tensor_id` quantized to `type`:
// the same bytes as the oracle's ob_synth_quantized.
int synth_launch(int type, uint64_t seed, uint32_t tensor_id, int64_t n, float std_dev, uint8_t* out,
                 cudaStream_t stream);
// fp32 synthetic values (biases).
int synth_f32_launch(uint64_t seed, uint32_t tensor_id, int64_t n, float std_dev, float* out, cudaStream_t stream);
int fill_f32_launch(float* out, int64_t n, float v, cudaStream_t stream);

// out[b] = argmax(logits[b][0..n)) with Kernels.argMax semantics; keys and
// ctr: `batch` zeroed scratch words each, left zero.
int argmax_launch(const float* logits, int ld, int n, int batch, unsigned long long* keys, int* ctr, int32_t* out,
                  cudaStream_t stream, bool pdl);

}  // namespace brew
