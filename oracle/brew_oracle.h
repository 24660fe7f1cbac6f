/*
 * brew_oracle.h — CPU restatement of the reference's hot-path arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker that the CUDA path
 * is compared against; it is loaded by the tests, by the smoke check and by
 * the CPU-baseline leg of bench.py, never by the product library.
 *
 * Parity status: the reference (Java 8) ships no tests, golden vectors or
 * fixtures, and cannot run in this environment (no JDK).  The restatement is
 * therefore pinned by (a) exhaustive fp16 decode checks, (b) the GGML block
 * formats of gguf-py 0.19.0 (quantize + dequantize fixtures under
 * tests/golden/), and (c) line-by-line citations of the Java it restates.
 * For the Java-only arithmetic (matvec order, norms, RoPE, attention,
 * activations, token feeding) parity is unpinned by the reference itself.
 */
#ifndef BREW_ORACLE_H
#define BREW_ORACLE_H

#include <stdint.h>
#include <stddef.h>
#include "../include/brew.h"

#ifdef __cplusplus
extern "C" {
#endif

/* fp16 <-> fp32 */
float    ob_half_to_float(uint16_t h);
uint16_t ob_float_to_half(float f);

/* thread count for the row-parallel / head-parallel loops (0 = all cores) */
void ob_set_threads(int n);
int  ob_get_threads(void);

/* seeded synthetic N(0, std) values (Irwin-Hall(12) on a counter hash) */
float ob_synth_value(uint64_t seed, uint32_t tensor_id, uint64_t index, float std_dev);
void  ob_synth_fill(uint64_t seed, uint32_t tensor_id, uint64_t start, int64_t n, float std_dev, float* out);

/* block formats */
int     ob_type_block(int type, int* block_elems, int* block_bytes);
int64_t ob_type_bytes(int type, int64_t n);
int ob_quantize(int type, const float* x, int64_t n, uint8_t* out);
int ob_dequantize(int type, const uint8_t* bytes, int64_t elem_offset, int64_t n, float* out);
/* synthesize rows*cols values of tensor `tensor_id` and quantize them */
int ob_synth_quantized(int type, uint64_t seed, uint32_t tensor_id, int64_t n, float std_dev, uint8_t* out);

/* Linear.matmul restatement: y[r] for r < N, element offset `woff` */
int ob_matvec(int type, const uint8_t* w, int64_t woff, const float* x, float* y, int K, int N);

/* Kernels.* restatements */
void  ob_rmsnorm(float* out, const float* in, const float* w, int n, float eps);
void  ob_headwise_rmsnorm(float* v, const float* w, int heads, int head_size, float eps);
void  ob_softmax(float* v, int n);
int   ob_argmax(const float* v, int n);
void  ob_rope(float* q, float* k, int n_heads, int n_kv_heads, int head_size,
              float base, float position, int interleaved);
void  ob_glu(float* hb, const float* hb2, int n, int gelu);

/* synthetic model + forward + greedy generation */
typedef struct ob_model ob_model;
ob_model* ob_model_synth(const brew_config* cfg, uint64_t seed);
void      ob_model_free(ob_model* m);
const uint8_t* ob_model_tensor(ob_model* m, int which, int64_t* n_bytes);
const float*   ob_model_vector(ob_model* m, int which, int64_t* n);
void      ob_model_reset(ob_model* m);
int       ob_model_forward(ob_model* m, int token, int pos, float* logits_out);
int       ob_generate(ob_model* m, const int32_t* prompt, int n_prompt, int max_new,
                      int32_t* out_tokens, int* n_out);

/* tensor ids of the synthetic generator (shared with the device generator) */
#define OB_W_EMBED   0
#define OB_W_OUTPUT  1
#define OB_W_Q       2
#define OB_W_K       3
#define OB_W_V       4
#define OB_W_O       5
#define OB_W_GATE    6
#define OB_W_UP      7
#define OB_W_DOWN    8
#define OB_B_Q       9
#define OB_B_K      10
#define OB_B_V      11
#define OB_TENSOR_ID(kind, layer) ((uint32_t)(((uint32_t)(kind) << 16) | (uint32_t)(layer)))

#ifdef __cplusplus
}
#endif
#endif
