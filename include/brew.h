/*
 * brew.h — C ABI of the B200 quantized-matmul path of brewference.
 *
 * Every entry point here replaces one piece of the reference's Java hot path
 * (paths relative to src/main/java/com/epicmonstrosity/brewference/ of the
 * reference).  The signatures use plain pointers, sizes and POD structs so a
 * JNI glue file (Java 8 has no Panama), ctypes or C++ can bind them directly.
 *
 * Conventions
 *   - Every function returns an int status: BREW_OK (0) or a negative
 *     BREW_ERR_* code.  brew_last_error() returns the message of the last
 *     failure on the calling thread.  The JNI glue maps
 *       BREW_ERR_INVALID_ARG   -> IllegalArgumentException  (Linear.java:67-74)
 *       BREW_ERR_OUT_OF_BOUNDS -> IllegalStateException     (Linear.java:46-50)
 *       BREW_ERR_CONTEXT_FULL  -> IllegalStateException     (runtime/ModelRunner.java:208-216)
 *       BREW_ERR_IO            -> IOException               (gguf/GgufWeightsLoader.java:76-78,251-253)
 *     and everything else to IllegalStateException.
 *   - Weight tensors are uploaded as the GGUF bytes, unchanged: 34-byte Q8_0,
 *     18-byte Q4_0, 144-byte Q4_K and 210-byte Q6_K blocks, rows of `cols`
 *     elements.  Element offsets (the reference's `weightsOffset`) are
 *     converted to block offsets on the device side.
 *   - Host pointers are plain host memory; functions with a _dev suffix take
 *     device pointers and a cudaStream_t passed as void*.
 */
#ifndef BREW_H
#define BREW_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define BREW_API __attribute__((visibility("default")))
#else
#define BREW_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------ */
#define BREW_OK                 0
#define BREW_ERR_INVALID_ARG   -1
#define BREW_ERR_OUT_OF_BOUNDS -2
#define BREW_ERR_CUDA          -3
#define BREW_ERR_NCCL          -4
#define BREW_ERR_TIMEOUT       -5
#define BREW_ERR_CONTEXT_FULL  -6
#define BREW_ERR_UNSUPPORTED   -7
#define BREW_ERR_IO            -8
#define BREW_ERR_NO_DEVICE     -9

/* ---- GGML tensor type ids (gguf/Reader.java:67-81 reads them as `type`) -- */
#define BREW_TYPE_F32   0
#define BREW_TYPE_F16   1
#define BREW_TYPE_Q4_0  2
#define BREW_TYPE_Q8_0  8
#define BREW_TYPE_Q4_K 12
#define BREW_TYPE_Q6_K 14

/* ---- architectures (model/ModelRunnerFactory.java:23-49) ---------------- */
#define BREW_ARCH_LLAMA  0   /* model/llama2/Llama2Transformer.java:27-79   */
#define BREW_ARCH_QWEN2  1   /* model/qwen2/Qwen2Transformer.java:27-84     */
#define BREW_ARCH_QWEN3  2   /* model/qwen3/Qwen3Transformer.java:27-85     */
#define BREW_ARCH_GEMMA3 3   /* model/gemma3/Gemma3Transformer.java:27-92   */
#define BREW_ARCH_GEMMA2 4   /* model/gemma2/Gemma2Transformer.java:27-87   */
#define BREW_ARCH_SMOLLM3 5  /* model/smollm3/SmolLM3Transformer.java:40-94 */

/* Model hyper-parameters: the fields of gguf/Config.java that the forward
 * pass reads (GgufConfigParser.java:9-59), plus the GGML type of each weight
 * matrix.  `rope_base` <= 0 selects the architecture's fallback exactly as the
 * reference's suppliers do (Llama2Transformer.java:45 and
 * SmolLM3Transformer.java:60 -> 1e4, Qwen2/Qwen3 -> 1e6,
 * Gemma3Transformer.java:51 and Gemma2Transformer.java:47 -> 1e6 global /
 * 1e4 local).  SmolLM3 skips RoPE on every 4th layer
 * (SmolLM3Transformer.java:48); Gemma2 attends globally on every 2nd layer
 * (Gemma2AttentionPattern.java:10-12), Gemma3 on every 6th. */
typedef struct brew_config {
    int32_t arch;
    int32_t dim;             /* {arch}.embedding_length                      */
    int32_t hidden_dim;      /* {arch}.feed_forward_length                   */
    int32_t n_layers;        /* {arch}.block_count                           */
    int32_t n_heads;         /* {arch}.attention.head_count                  */
    int32_t n_kv_heads;      /* {arch}.attention.head_count_kv               */
    int32_t head_size;       /* Config.getHeadSize (Qwen3 128, Gemma3 256)   */
    int32_t vocab_size;      /* size of tokenizer.ggml.tokens                */
    int32_t seq_len;         /* {arch}.context_length                        */
    int32_t sliding_window;  /* {arch}.attention.sliding_window (Gemma3)     */
    float   eps;             /* {arch}.attention.layer_norm_rms_epsilon      */
    float   rope_base;       /* {arch}.rope.freq_base (<= 0: arch fallback)  */
    float   rope_scale;      /* Config.ropeFrequencyScale (<= 0: 1.0)        */
    int32_t bos_token;
    int32_t eos_token;
    int32_t tied_embeddings; /* 1: classifier = token_embd (GgufWeightsLoader.java:159-162) */
    /* GGML type of each weight matrix family */
    int32_t type_embed, type_output;
    int32_t type_q, type_k, type_v, type_o;
    int32_t type_gate, type_up, type_down;
} brew_config;

/* ---- errors, devices ---------------------------------------------------- */

/* Copies the calling thread's last error message into buf (NUL-terminated).
 * Returns the message length. */
BREW_API int brew_last_error(char* buf, size_t buf_size);

/* Selects and initialises a CUDA device for the calling process.  Fails with
 * BREW_ERR_NO_DEVICE when no device is visible: there is no CPU fallback. */
BREW_API int brew_init(int device);

/* Library version string and the number of kernels this library launched so
 * far on this process (all kinds). */
BREW_API const char* brew_version(void);
BREW_API int64_t brew_kernel_launches(void);

/* ---- weight tensors (gguf/GgufWeightsLoader.java:228-247 readQ8Block) ---- */

typedef struct brew_tensor_s* brew_tensor;

/* Bytes that `n_elements` of GGML type `type` occupy on disk (and in HBM). */
BREW_API int64_t brew_type_bytes(int type, int64_t n_elements);
BREW_API int brew_type_block(int type, int* block_elements, int* block_bytes);

/* Uploads packed GGUF bytes unchanged to HBM.  Replaces readQ8Block +
 * concatenateQ8Blocks (GgufWeightsLoader.java:167-185,228-247): per-layer
 * tensors are uploaded one after another into one tensor so that the
 * reference's element offsets `layer*in*out` stay valid.  n_elements must be
 * a multiple of the type's block size (GgufWeightsLoader.java:229-231). */
BREW_API int brew_tensor_upload(int type, const void* bytes, int64_t n_elements, brew_tensor* out);
/* Appends more packed bytes at element offset `elem_offset` of an existing
 * tensor created with brew_tensor_alloc (for layer-by-layer loading). */
BREW_API int brew_tensor_alloc(int type, int64_t n_elements, brew_tensor* out);
BREW_API int brew_tensor_write(brew_tensor t, int64_t elem_offset, const void* bytes, int64_t n_elements);
BREW_API int brew_tensor_free(brew_tensor t);
BREW_API int brew_tensor_info(brew_tensor t, int* type, int64_t* n_elements, int64_t* n_bytes);
/* Copies the packed bytes of elements [elem_offset, elem_offset + n) back to
 * host memory (whole blocks). */
BREW_API int brew_tensor_read(brew_tensor t, int64_t elem_offset, int64_t n_elements, void* bytes);
/* Device address of the packed bytes (for callers that launch their own work). */
BREW_API int brew_tensor_device_ptr(brew_tensor t, void** dev_ptr);

/* Dequantizes `n` elements starting at element `row_offset` into host fp32
 * `out`.  Bit-exact with QuantizedWeights.dequantizeRow
 * (gguf/QuantizedWeights.java:76-85) for Q8_0 and with the GGML definitions
 * for Q4_0 / Q4_K / Q6_K. */
BREW_API int brew_dequantize_row(brew_tensor t, int64_t row_offset, int64_t n, float* out);
BREW_API int brew_dequantize_row_dev(brew_tensor t, int64_t row_offset, int64_t n, float* out_dev, void* stream);

/* ---- the hot path: Linear.matmul (transformer/math/Linear.java:40-65) --- */

/* output[row] = sum_k W[weights_offset + row*input_size + k] * input[k]
 * for row < output_size, with host fp32 arrays — the drop-in for
 * Linear.matmul(output, input, weights, weightsOffset, inputSize, outputSize).
 * Errors: BREW_ERR_INVALID_ARG for null arrays/tensor (Linear.java:67-74) or
 * an input_size that is not a whole number of blocks; BREW_ERR_OUT_OF_BOUNDS
 * when the last block read lies past the tensor (Linear.java:46-50). */
BREW_API int brew_matmul(float* output, const float* input, brew_tensor weights,
                int64_t weights_offset, int32_t input_size, int32_t output_size);

/* Batched form: `batch` input vectors [batch][input_size] -> outputs
 * [batch][output_size], device pointers, on `stream` (0 = default). */
BREW_API int brew_matmul_dev(float* output_dev, const float* input_dev, brew_tensor weights,
                    int64_t weights_offset, int32_t input_size, int32_t output_size,
                    int32_t batch, void* stream);

/* brew_matmul_dev without any allocation in the call: the quantized records
 * of the input live in a 256 KiB array that is part of the loaded module
 * (one per device), not in a buffer grown on demand.  No counterpart in the
 * reference (its Java matmul allocates nothing on a device).  For callers
 * that must not allocate device memory mid-call (a JNI critical region, a
 * server whose memory is reserved up front).  Same arguments, results and
 * errors as brew_matmul_dev, plus: brew_init must have been called
 * (BREW_ERR_INVALID_ARG otherwise); (input_size / 32) * record bytes of
 * min(batch, 16) vectors must fit in 256 KiB (input_size <= 74880 at batch
 * 1, <= 4672 at batch 16), else BREW_ERR_INVALID_ARG.  brew_init looks up
 * the array's address on its device; the kernels themselves are loaded on
 * their first launch, so make one call before entering a region that must
 * not allocate and before any stream capture starts.  Calls whose device
 * work may overlap (different unordered streams) race on the one array. */
BREW_API int brew_matmul_dev_static(float* output_dev, const float* input_dev, brew_tensor weights,
                    int64_t weights_offset, int32_t input_size, int32_t output_size,
                    int32_t batch, void* stream);

/* Prefill GEMM on the tcgen05 tensor cores: output_dev [T][N] = W x for T
 * token vectors input_dev [T][K] at once (the prompt of ModelRunner.prefill,
 * runtime/ModelRunner.java:196-206, instead of T matvecs).  N a multiple of
 * 128, any T >= 1.  Each 32-element block's integer dot product is exact
 * (24-bit limb split of x) and scaled by d_row * s_block in fp32, as
 * brew_matmul does per token.  No reference counterpart.
 *
 * brew_gemm_q8_dev: one call on a Q8_0 tensor (repacks the matrix, allocates
 * scratch, synchronises).  A plan keeps the repacked matrix (Q8_0 or Q4_0)
 * for repeated runs: brew_gemm_plan_run enqueues on `stream` without
 * synchronising (its scratch grows, with an allocation, the first time a
 * larger T is run); runs of one plan must not overlap. */
BREW_API int brew_gemm_q8_dev(float* output_dev, const float* input_dev, brew_tensor weights,
                              int64_t weights_offset, int32_t input_size, int32_t output_size,
                              int32_t tokens, void* stream);
typedef struct brew_gemm_plan_s* brew_gemm_plan;
BREW_API int brew_gemm_plan_create(brew_tensor weights, int64_t weights_offset, int32_t input_size,
                                   int32_t output_size, brew_gemm_plan* out);
BREW_API int brew_gemm_plan_run(brew_gemm_plan plan, float* output_dev, const float* input_dev, int32_t tokens,
                                void* stream);
BREW_API int brew_gemm_plan_free(brew_gemm_plan plan);

/* Two-step form for callers that multiply one input by several matrices
 * (Q, K and V share their input): brew_prepare_input_dev writes the
 * quantized-activation records of x [batch][input_size] into `prep_dev`
 * (brew_prep_bytes(input_size, batch) bytes, 16-byte aligned), and
 * brew_matmul_prepared_dev multiplies a Q8_0 or Q4_0 tensor by them. */
BREW_API int64_t brew_prep_bytes(int32_t input_size, int32_t batch);
BREW_API int brew_prepare_input_dev(const float* input_dev, int32_t input_size, int32_t batch, void* prep_dev,
                                    void* stream);
BREW_API int brew_matmul_prepared_dev(float* output_dev, const void* prep_dev, brew_tensor weights,
                                      int64_t weights_offset, int32_t input_size, int32_t output_size,
                                      int32_t batch, void* stream);

/* ---- device-resident model (TransformerGraph.forward, ModelRunner) ------ */

typedef struct brew_model_s* brew_model;

/* Per-layer weights of a model, as packed tensors whose layers are
 * concatenated like QuantizedWeights (gguf/QuantizedWeights.java:37-60).
 * Norm and bias vectors are host fp32 arrays concatenated over layers
 * (GgufWeightsLoader.java:170-179); they are copied to the device.  Unused
 * entries are NULL (e.g. biases outside Qwen2, post norms outside Gemma3). */
typedef struct brew_model_weights {
    brew_tensor token_embd, output;               /* output may be NULL when tied */
    brew_tensor wq, wk, wv, wo, w_gate, w_up, w_down;
    const float* rms_att;       /* [n_layers*dim]       */
    const float* rms_ffn;       /* [n_layers*dim]       */
    const float* rms_final;     /* [dim]                */
    const float* post_att;      /* [n_layers*dim]  Gemma3 */
    const float* post_ffn;      /* [n_layers*dim]  Gemma3 */
    const float* rms_q;         /* [n_layers*head_size] Qwen3/Gemma3 */
    const float* rms_k;         /* [n_layers*head_size] */
    const float* q_bias;        /* [n_layers*n_heads*head_size] Qwen2 */
    const float* k_bias;        /* [n_layers*kv_dim]    */
    const float* v_bias;        /* [n_layers*kv_dim]    */
} brew_model_weights;

/* Creates a device-resident model with room for `max_batch` concurrent
 * sequences (each with its own fp32 KV cache of n_layers*seq_len*kv_dim,
 * RunStateAllocator.java:48-70). */
BREW_API int brew_model_create(const brew_config* cfg, const brew_model_weights* w,
                      int32_t max_batch, brew_model* out);

/* ---- GGUF checkpoints (gguf/Reader.java, gguf/GgufConfigParser.java,
 *      gguf/GgufWeightsLoader.java) ---------------------------------------
 * brew_gguf_open memory-maps a GGUF v2/v3 file and parses its header,
 * metadata and tensor infos as Reader.read does (Reader.java:25-58); errors
 * (bad magic, version, truncation, alignment) are BREW_ERR_IO.
 * brew_gguf_config fills a brew_config the way GgufConfigParser.parseCommon
 * (GgufConfigParser.java:9-59) and the per-architecture loaders do
 * (general.architecture -> arch, vocab = length of tokenizer.ggml.tokens,
 * head size 128 for qwen3 (Qwen3CheckpointLoader.java:16), 256 for gemma2 /
 * gemma3 (Gemma2/Gemma3CheckpointLoader.java:18), else dim / heads; tied
 * when there is no output.weight, GgufWeightsLoader.java:159-162) plus the
 * GGML type of each matrix family.  brew_gguf_tensor_info lists the tensors
 * (name, GGML type, elements, absolute file offset of the data). */
typedef struct brew_gguf_s* brew_gguf;
BREW_API int brew_gguf_open(const char* path, brew_gguf* out);
BREW_API int brew_gguf_close(brew_gguf g);
BREW_API int brew_gguf_config(brew_gguf g, brew_config* cfg);
BREW_API int brew_gguf_tensor_count(brew_gguf g, int64_t* n);
BREW_API int brew_gguf_tensor_info(brew_gguf g, int64_t index, char* name, size_t name_size, int* type,
                                   int64_t* n_elements, int64_t* file_offset);
/* Loads a GGUF checkpoint into a device-resident model in one call: the
 * replacement of GgufCheckpointLoader.loadWeights + GgufWeightsLoader.load
 * (GgufWeightsLoader.java:24-165).  Packed Q8_0 / Q4_0 / Q4_K / Q6_K blocks
 * go from the memory-mapped file to HBM unchanged through pinned staging
 * buffers, each family's layers concatenated; F32 / F16 norm and bias
 * vectors (readFloatArray, :249-278) are converted to fp32.  Unlike
 * readQ8Block the tensor types are checked (BREW_ERR_UNSUPPORTED for other
 * types, or a family whose layers differ in type).  The model owns its
 * tensors. */
BREW_API int brew_model_load_gguf(const char* path, int32_t max_batch, brew_model* out);

/* Creates a model whose weights are generated on the device from `seed`
 * (seeded N(0, 0.02) quantized to the configured GGML types, norms 1.0).
 * The bytes equal those of the CPU generator used by the tests. */
BREW_API int brew_model_synthesize(const brew_config* cfg, uint64_t seed, int32_t max_batch, brew_model* out);
BREW_API int brew_model_free(brew_model m);
/* ---- tensor parallelism (one process per GPU of a box) --------------------
 * Every matrix is split by rows over the ranks of a communicator: rank r of P
 * multiplies rows [r*N/P, (r+1)*N/P) of each N-row matrix and the slices are
 * gathered after each projection (q|k|v or the attention output, wo,
 * gate|up, down, classifier; the argmax is reduced over the ranks' (value,
 * index) keys).  The gathers are peer stores into every rank's tagged slots
 * through CUDA IPC over NVLink (BREW_TP_NCCL=1: NCCL all-gathers instead).
 * Attention is sharded by kv head when the kv heads divide over the ranks
 * (each rank's q|k|v rows are its heads), else replicated; norms and
 * residuals are replicated, so every rank ends a step with the full
 * activations.  The K-quant matvecs split K for each rank's own rows, so the
 * logits match the one-GPU logits to rounding; with BREW_TP_EXACT=1 (read by
 * brew_model_set_tp) they split K as on one GPU and every output row is the
 * one-GPU row bit for bit.  N must be a multiple of P for every matrix.  The
 * row split is the one the reference's matvec parallelises over
 * (Linear.java:51-64, rows of `out`). */
typedef struct brew_comm_s* brew_comm;
/* Rows [r0, r1) of an N-row matrix that rank `rank` of `nranks` owns. */
BREW_API int brew_tp_rows(int64_t rows, int32_t nranks, int32_t rank, int64_t* r0, int64_t* r1);
/* Rank 0 creates the 128-byte NCCL unique id and shares it with the others. */
BREW_API int brew_comm_unique_id(uint8_t* id_out);
/* Collective: every rank calls it with the same id (device = brew_init's). */
BREW_API int brew_comm_init(const uint8_t* id, int32_t nranks, int32_t rank, brew_comm* out);
/* Free the models that use a communicator before the communicator. */
BREW_API int brew_comm_free(brew_comm c);
/* Shards model `m` over `comm` (same model on every rank, same seed or same
 * tensors).  The model then runs the unfused forward with the gathers. */
BREW_API int brew_model_set_tp(brew_model m, brew_comm comm);

/* The model's hyper-parameters and matrix types (as created or loaded). */
BREW_API int brew_model_config(brew_model m, brew_config* out);

/* Returns the model's tensors (borrowed handles) for inspection. */
BREW_API int brew_model_tensor(brew_model m, int which, brew_tensor* out);

/* One decode step of TransformerGraph.forward(token, pos, ...) for `batch`
 * sequences (host arrays tokens[batch], pos[batch]).  Either output may be
 * NULL: logits [batch][vocab] (host fp32) and/or argmax ids [batch] computed
 * on the device with Kernels.argMax semantics (lowest index on ties,
 * transformer/math/Kernels.java:150-162).  One sequence without logits on
 * the persistent decode kernel is one launch and one synchronize: the token
 * and position are launch parameters and the kernel writes the id and the
 * device error word into mapped pinned host memory of the model. */
BREW_API int brew_model_forward(brew_model m, const int32_t* tokens, const int32_t* pos,
                       int32_t batch, float* logits, int32_t* argmax);

/* Device-pointer form for callers that keep tokens/positions/results resident. */
BREW_API int brew_model_forward_dev(brew_model m, const int32_t* tokens_dev, const int32_t* pos_dev,
                           int32_t batch, float* logits_dev, int32_t* argmax_dev, void* stream);

/* Greedy generation for one sequence, with the token feeding order of
 * GenericModelSession.generate/prefill (runtime/ModelRunner.java:122-206):
 * each prompt token is forwarded at its position; then the last prompt token
 * is forwarded again at position n_prompt, and each generated token is fed
 * back at the next position; stops at eos or after
 * min(max_new_tokens, seq_len - n_prompt) tokens.  `out_tokens` receives the
 * generated ids; *n_out their count.  BREW_ERR_CONTEXT_FULL when the prompt
 * does not fit (ModelRunner.java:208-216). */
BREW_API int brew_session_generate(brew_model m, const int32_t* prompt, int32_t n_prompt,
                          int32_t max_new_tokens, int32_t* out_tokens, int32_t* n_out);

/* The two halves of brew_session_generate for callers that time or drive
 * them separately.  brew_session_prefill resets the session and forwards
 * prompt[i] at position i (the classifier is skipped: prompt logits are never
 * read).  brew_session_decode then runs `n_steps` greedy steps from the
 * session's pending token and position, enqueued on `stream` (NULL: the
 * library stream) without host synchronisation; when `out_tokens` is not NULL
 * it synchronises and copies the generated ids there. */
BREW_API int brew_session_prefill(brew_model m, const int32_t* prompt, int32_t n_prompt, void* stream);
BREW_API int brew_session_decode(brew_model m, int32_t n_steps, int32_t* out_tokens, void* stream);

/* How brew_session_prefill / brew_session_generate fill the KV cache with
 * the prompt.  BREW_PREFILL_TOKENS (default): forward(prompt[i], i) token by
 * token, the reference's order (ModelRunner.java:196-206).
 * BREW_PREFILL_BATCHED: chunks of up to 512 prompt tokens go through each
 * layer together, the matrices multiplied on the tcgen05 tensor cores (int8
 * MMA of the exact Q8_0 block products, fp32 block-scale epilogue).  The
 * prompt's logits are never read, so the resulting state is the KV cache,
 * equal to the token-by-token one up to fp32 summation order.  Needs every
 * layer matrix in Q8_0 or Q4_0, one GPU (no tensor parallelism), head size 64 / 128
 * / 256 and matrix row counts (q|k|v, dim, 2 * hidden_dim) that are
 * multiples of 128; otherwise BREW_ERR_UNSUPPORTED.  No reference
 * counterpart: the reference has only the token-by-token prefill. */
#define BREW_PREFILL_TOKENS 0
#define BREW_PREFILL_BATCHED 1
BREW_API int brew_model_set_prefill(brew_model m, int32_t mode);
/* Kernels in one decode step's CUDA graph (for launch accounting). */
BREW_API int brew_model_step_kernels(brew_model m, int32_t batch, int32_t* n_kernels);

/* Phase tracing of the persistent decode kernel: when on, every CTA of every
 * decode step records %globaltimer (ns) at its start and, per phase (5 per
 * layer: QKV, attention, wo, gate|up, down; then the classifier), when the
 * first load wave of its input landed, when its input preparation is done,
 * when its last weight stage arrived (0: none), when its work is done and
 * when it leaves the grid barrier: [n_ctas][1 + 5 * (5 * n_layers + 1)]
 * values.  brew_model_trace
 * copies the last step's stamps (n = 0 when the model runs the kernel-graph
 * path). */
BREW_API int brew_model_set_trace(brew_model m, int32_t on);
BREW_API int brew_model_trace(brew_model m, int64_t* ns, int32_t max_n, int32_t* n);

/* Failure-detection self-test (no reference counterpart): runs the library's
 * two bounded device waits, an mbarrier phase and the grid barrier's arrival
 * counter, against events that never happen.  Each must give up after
 * `limit_ns` (1 ns .. 1 s), record the timeout in the device error word and
 * return, as a decode step whose weight pipeline or grid barrier stalled
 * does (there the limit is 2 s).  Returns BREW_ERR_TIMEOUT when the waits
 * ended as designed; *waits_ended (optional) receives how many did (2).
 * The context stays usable afterwards. */
BREW_API int brew_selftest_wait_timeout(int64_t limit_ns, int32_t* waits_ended);

/* Clears the sequence state (ModelSession.reset, ModelRunner.java:115-120). */
BREW_API int brew_model_reset(brew_model m);

#ifdef __cplusplus
}
#endif

#endif /* BREW_H */
