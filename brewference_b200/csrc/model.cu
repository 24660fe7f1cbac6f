// model.cu — device-resident model: TransformerGraph.forward for the llama,
// qwen2, qwen3 and gemma3 graphs, captured into CUDA graphs, plus the greedy
// generation loop of GenericModelSession (runtime/ModelRunner.java:100-217).
//
// Per layer the forward is five launches, chained with programmatic
// dependent launch so each matvec streams its weights while the previous
// kernel finishes:
//   1. Q|K|V matvec (one launch over the three matrices, bias epilogue)
//   2. attention: QK-norm, RoPE, KV append, split-context softmax.V, combine,
//      prep records of xb
//   3. wo matvec (+ residual, or Gemma3 post-norm) whose last CTA
//      RMS-normalises x for the FFN and writes its prep records
//   4. gate|up matvec with the SwiGLU/GeGLU epilogue and prep records of hb
//   5. down matvec (+ residual / post-norm) whose last CTA normalises x for
//      the next layer (or the final norm)
// then the classifier matvec with a fused argmax.  The embedding lookup and
// the first RMSNorm are one more kernel.
#include "brew_internal.cuh"
#include "decode.cuh"
#include "eltwise.cuh"
#include "gemm.cuh"
#include "kqtc.cuh"
#include "prefill.cuh"
#include "tp.cuh"

#include <cmath>
#include <cstdlib>
#include <cstring>
#include <map>
#include <string>
#include <vector>

namespace brew {

namespace {

enum { T_EMBED = 0, T_OUTPUT, T_Q, T_K, T_V, T_O, T_GATE, T_UP, T_DOWN, T_COUNT };

uint32_t tensor_id(int kind, int layer) { return ((uint32_t)kind << 16) | (uint32_t)layer; }

__global__ void step_kernel(int32_t* tokens, int32_t* pos, const int32_t* tok_src, int32_t pos_val, int32_t* record,
                            const int32_t* am) {
    if (threadIdx.x == 0) {
        if (record) *record = am[0];
        tokens[0] = *tok_src;
        pos[0] = pos_val;
    }
}

}  // namespace

}  // namespace brew

using namespace brew;

struct brew_model_s {
    brew_config c;
    int max_batch = 1;
    brew_tensor t[T_COUNT] = {};
    bool owns_tensors = false;
    float *rms_att = nullptr, *rms_ffn = nullptr, *rms_final = nullptr, *post_att = nullptr, *post_ffn = nullptr;
    float *rms_q = nullptr, *rms_k = nullptr, *q_bias = nullptr, *k_bias = nullptr, *v_bias = nullptr;
    float *kc = nullptr, *vc = nullptr;
    int64_t cache_bstride = 0;
    float *x = nullptr, *xb = nullptr, *xb2 = nullptr, *qkv = nullptr, *hb = nullptr, *logits = nullptr;
    uint8_t *prep_x = nullptr, *prep_q = nullptr, *prep_h = nullptr;
    int* counters = nullptr;   // [group counters][post][attn]
    int n_counters = 0;
    float* attn_part = nullptr;
    unsigned long long* am_key = nullptr;
    int* am_ctr = nullptr;                  // [batch] arrival counters of the batched argmax
    int32_t* am_out = nullptr;
    int32_t *tokens_d = nullptr, *pos_d = nullptr;
    int32_t* gen_d = nullptr;      // generated ids of brew_session_generate
    int32_t* prompt_d = nullptr;   // prompt of brew_session_generate (+1 for bos)
    int prompt_cap = 0;
    int nchunk = 1;
    int qkvw = 0;
    std::vector<void*> allocs;
    std::map<int, cudaGraphExec_t> graphs;   // key: batch*2 + with_classifier
    std::map<int, int> graph_kernels;        // kernels captured in each graph
    // greedy session (GenericModelSession state: position, pendingToken)
    int sess_pos = 0;
    const int32_t* sess_pending = nullptr;   // device address of the pending token
    int sess_generated = 0;                  // ids recorded in gen_d since prefill
    int32_t* h_pin = nullptr;                // pinned staging (tokens, pos, argmax)
    int h_pin_cap = 0;
    int32_t* h_res = nullptr;                // mapped pinned [argmax id, device error word] of the decode kernel
    int32_t* h_res_dev = nullptr;            // ... its device address
    // persistent decode kernel (batch <= DK_MAX_BATCH)
    bool use_decode = false;
    DecodeParams dp;
    float *rope_cos = nullptr, *rope_sin = nullptr, *dk_part = nullptr;
    int* dk_actr = nullptr;                 // its attention arrival counters [2][layers][DK_MAX_BATCH][kv heads]
    size_t dk_nactr = 0;
    unsigned long long* dk_tg = nullptr;    // its tagged activations
    size_t dk_tg_words = 0;
    unsigned int* dk_seq = nullptr;         // epoch of its last completed launch
    int* dk_done = nullptr;                 // its end-of-step arrival counter
    uint8_t* pk[PK_NFAM] = {};              // fragment-packed weight copies of the decode kernel
    // unfused forward (models with K-quant matrices)
    bool unfused = false;
    float *xn = nullptr, *hb2 = nullptr;    // normed input of a matvec; the up projection
    uint8_t* prep_any = nullptr;            // x records of a Q8_0 / Q4_0 matvec in that forward
    uint8_t* kqp[T_COUNT] = {};             // K-quant matrices expanded for the tcgen05 matvec (kqtc.cuh)
    uint8_t* kqp_qkv = nullptr;             // ... Q, K and V of one type as one [q|k|v]-row family per layer
    uint8_t* kqp_gu = nullptr;              // ... gate and up of one type as one [gate|up]-row family per layer
    float* hgu = nullptr;                   // [batch][2 * hidden]: gate | up outputs of that family
    uint8_t* kq_rec = nullptr;              // x records of a K-quant matvec (kqtc.cuh)
    float* qkv_bias = nullptr;              // [layers][q|k|v rows]: the biases indexed by q|k|v family row
    // tensor parallelism: this rank's rows of the q|k|v and gate|up families
    // as families of their own ([q_R | k_R | v_R], [gate_R | up_R]), one
    // launch each; their biases; the gate|up outputs
    uint8_t* kqp_qkv_tp = nullptr;
    uint8_t* kqp_gu_tp = nullptr;
    float* qkv_bias_tp = nullptr;
    float* tp_gu = nullptr;
    float* kq_part = nullptr;               // its split-K partial sums
    int* kq_ctr = nullptr;                  // and their arrival counters
    size_t kq_nctr = 0;
    // tensor parallelism (brew_model_set_tp): this rank's row slices
    brew_comm comm = nullptr;
    float *tp_send = nullptr, *tp_recv = nullptr, *tp_g = nullptr, *tp_u = nullptr;
    // ... peer-store gathers (tp.cuh): this rank's tagged arena, every
    // rank's arena mapped here (IPC), the step counter of the tags, the
    // gathers' abort flag; words of one layer's four gather slots
    bool tp_p2p = false;
    // sharded K-quant matvecs split K for the rows they hold (all SMs busy),
    // or, with BREW_TP_EXACT=1, as the whole family does on one GPU (the
    // sharded logits then equal the one-GPU logits bit for bit)
    bool tp_exact = false;
    unsigned long long* tp_arena = nullptr;
    TpPeers tp_peers = {};
    uint32_t* tp_step = nullptr;
    int* tp_abort = nullptr;
    size_t tp_layer_words = 0;
    unsigned long long *tp_keys = nullptr, *tp_keys_all = nullptr;
    int* abort_flag = nullptr;
    unsigned long long* trace = nullptr;    // phase timestamps of the last decode step
    int trace_n = 0;
    // batched prefill (brew_model_set_prefill): GEMM-layout copies of the
    // layer matrices and the activations of one prompt chunk
    int prefill_mode = BREW_PREFILL_TOKENS;
    bool pf_ready = false;
    int pf_cap = 0;                         // tokens per chunk (multiple of GEMM_TT)
    int8_t* pf_wq[4] = {};                  // Q|K|V, wo, gate|up, down: [layer][N/128][K/32] 4 KB quant tiles
    uint16_t* pf_wd[4] = {};                // [layer][K/32][N] fp16 block scales
    float *pf_x = nullptr, *pf_xn = nullptr, *pf_qkv = nullptr, *pf_xb = nullptr, *pf_xb2 = nullptr, *pf_h = nullptr;
    int8_t* pf_limbs = nullptr;
    float* pf_lsc = nullptr;
};

namespace brew {
namespace {

template <class T>
int dalloc(brew_model_s* m, T** p, size_t count) {
    void* q = nullptr;
    BREW_CUDA(cudaMalloc(&q, count * sizeof(T) + 256));
    BREW_CUDA(cudaMemset(q, 0, count * sizeof(T) + 256));
    BREW_CUDA(cudaStreamSynchronize(0));   // legacy-stream memset: done before the non-blocking stream's kernels
    m->allocs.push_back(q);
    *p = static_cast<T*>(q);
    return BREW_OK;
}

constexpr int MODEL_MAX_BATCH = 32;   // sequences per step of the unfused forward

// Any Q4_K / Q6_K matrix: the model runs the unfused forward (separate
// norm / bias / residual / activation kernels around each matvec).
bool uses_kquants(const brew_config& c) {
    const int types[] = {c.type_q, c.type_k, c.type_v, c.type_o, c.type_gate, c.type_up, c.type_down,
                         c.tied_embeddings ? c.type_embed : c.type_output};
    for (int t : types)
        if (t == BREW_TYPE_Q4_K || t == BREW_TYPE_Q6_K) return true;
    return false;
}

int check_config(const brew_config& c, int max_batch) {
    BREW_CHECK(c.arch >= BREW_ARCH_LLAMA && c.arch <= BREW_ARCH_SMOLLM3, BREW_ERR_UNSUPPORTED, "arch %d", c.arch);
    BREW_CHECK(c.dim > 0 && c.dim % 32 == 0, BREW_ERR_INVALID_ARG, "dim %d", c.dim);
    BREW_CHECK(c.hidden_dim > 0 && c.hidden_dim % 32 == 0, BREW_ERR_INVALID_ARG, "hidden_dim %d", c.hidden_dim);
    BREW_CHECK(c.n_layers > 0 && c.n_heads > 0 && c.n_kv_heads > 0 && c.n_heads % c.n_kv_heads == 0,
               BREW_ERR_INVALID_ARG, "layers/heads %d/%d/%d", c.n_layers, c.n_heads, c.n_kv_heads);
    BREW_CHECK(c.head_size > 0 && c.head_size % 32 == 0, BREW_ERR_INVALID_ARG, "head_size %d", c.head_size);
    BREW_CHECK(c.vocab_size > 0 && c.seq_len > 0, BREW_ERR_INVALID_ARG, "vocab/seq_len");
    // the fused forward runs up to MV_MAX_BATCH sequences per step; the
    // unfused (K-quant) forward, whose matvecs loop over vector groups, up to
    // MODEL_MAX_BATCH
    const int bmax = uses_kquants(c) ? MODEL_MAX_BATCH : MV_MAX_BATCH;
    BREW_CHECK(max_batch >= 1 && max_batch <= bmax, BREW_ERR_INVALID_ARG, "max_batch %d (at most %d for this model)",
               max_batch, bmax);
    const int types[] = {c.type_q, c.type_k, c.type_v, c.type_o, c.type_gate, c.type_up, c.type_down,
                         c.tied_embeddings ? c.type_embed : c.type_output, c.type_embed};
    for (int t : types)
        BREW_CHECK(is_quant_matrix_type(t), BREW_ERR_UNSUPPORTED, "GGML type %d is not a supported weight type", t);
    if (!uses_kquants(c)) {
        // the fused forward: one type for Q/K/V and one for gate/up
        BREW_CHECK(c.type_q == c.type_k && c.type_k == c.type_v, BREW_ERR_UNSUPPORTED, "Q/K/V of different types");
        BREW_CHECK(c.type_gate == c.type_up, BREW_ERR_UNSUPPORTED, "gate/up of different types");
    } else {
        // K-quant rows are whole 256-element super-blocks
        const int qw = c.n_heads * c.head_size;
        auto kq = [](int t) { return t == BREW_TYPE_Q4_K || t == BREW_TYPE_Q6_K; };
        const int in_dim[] = {c.type_q, c.type_k, c.type_v, c.type_gate, c.type_up,
                              c.tied_embeddings ? c.type_embed : c.type_output, c.type_embed};
        for (int t : in_dim)
            BREW_CHECK(!kq(t) || c.dim % 256 == 0, BREW_ERR_UNSUPPORTED, "K-quant matrix with dim %d %% 256", c.dim);
        BREW_CHECK(!kq(c.type_o) || qw % 256 == 0, BREW_ERR_UNSUPPORTED, "K-quant wo with %d inputs", qw);
        BREW_CHECK(!kq(c.type_down) || c.hidden_dim % 256 == 0, BREW_ERR_UNSUPPORTED, "K-quant down with %d inputs",
                   c.hidden_dim);
    }
    return BREW_OK;
}

void matrix_shape(const brew_config& c, int which, int64_t* rows, int64_t* cols, int* type, int* layers) {
    const int64_t qw = (int64_t)c.n_heads * c.head_size, kvd = (int64_t)c.n_kv_heads * c.head_size;
    *layers = c.n_layers;
    switch (which) {
        case T_EMBED: *rows = c.vocab_size; *cols = c.dim; *type = c.type_embed; *layers = 1; break;
        case T_OUTPUT: *rows = c.vocab_size; *cols = c.dim; *type = c.tied_embeddings ? c.type_embed : c.type_output; *layers = 1; break;
        case T_Q: *rows = qw; *cols = c.dim; *type = c.type_q; break;
        case T_K: *rows = kvd; *cols = c.dim; *type = c.type_k; break;
        case T_V: *rows = kvd; *cols = c.dim; *type = c.type_v; break;
        case T_O: *rows = c.dim; *cols = qw; *type = c.type_o; break;
        case T_GATE: *rows = c.hidden_dim; *cols = c.dim; *type = c.type_gate; break;
        case T_UP: *rows = c.hidden_dim; *cols = c.dim; *type = c.type_up; break;
        default: *rows = c.dim; *cols = c.hidden_dim; *type = c.type_down; break;
    }
}

const uint8_t* layer_ptr(brew_tensor t, int layer, int64_t rows, int64_t cols);

// Rows of the family a K-quant matrix is multiplied with at one GPU (q|k|v,
// gate|up, or the matrix itself): its split-K count derives from this, so
// a sharded launch sums each row in the one-GPU order.
int64_t kq_basis(const brew_model_s* m, int which, int64_t rows) {
    const brew_config& c = m->c;
    const int64_t qw = (int64_t)c.n_heads * c.head_size, kvd = (int64_t)c.n_kv_heads * c.head_size;
    const int tq = c.type_q, tg = c.type_gate;
    const bool kq_qkv = (tq == BREW_TYPE_Q4_K || tq == BREW_TYPE_Q6_K) && c.type_k == tq && c.type_v == tq &&
                        qw % 16 == 0 && kvd % 16 == 0;
    const bool kq_gu = (tg == BREW_TYPE_Q4_K || tg == BREW_TYPE_Q6_K) && c.type_up == tg && c.hidden_dim % 16 == 0;
    if (kq_qkv && (which == T_Q || which == T_K || which == T_V)) return qw + 2 * kvd;
    if (kq_gu && (which == T_GATE || which == T_UP)) return 2 * (int64_t)c.hidden_dim;
    return rows;
}

// Buffers of the unfused forward (K-quant models, tensor parallelism).
int alloc_unfused(brew_model_s* m) {
    if (m->unfused) return BREW_OK;
    const brew_config& c = m->c;
    const int B = m->max_batch;
    const int64_t qw = (int64_t)c.n_heads * c.head_size;
    const int64_t kmax = std::max<int64_t>(std::max<int64_t>(c.dim, qw), c.hidden_dim);
    int rc;
    if ((rc = dalloc(m, &m->xn, (size_t)B * std::max<int64_t>(qw, c.dim)))) return rc;
    if ((rc = dalloc(m, &m->hb2, (size_t)B * c.hidden_dim))) return rc;
    if ((rc = dalloc(m, &m->prep_any, (size_t)(kmax / 32) * prep_rec_bytes(std::min(B, MV_MAX_BATCH))))) return rc;
    // the K-quant matrices, repacked once for the int8 MMA matvec; Q, K and
    // V of one K-quant type as one family (rows q | k | v per layer), so that
    // one launch multiplies all three
    const int64_t kvd = (int64_t)c.n_kv_heads * c.head_size;
    const bool kq_qkv = (c.type_q == BREW_TYPE_Q4_K || c.type_q == BREW_TYPE_Q6_K) && c.type_k == c.type_q &&
                        c.type_v == c.type_q && qw % 16 == 0 && kvd % 16 == 0;
    if (kq_qkv) {
        const int64_t nf = qw + 2 * kvd;
        const size_t per = kx_bytes(c.type_q, nf, c.dim);
        if ((rc = dalloc(m, &m->kqp_qkv, per * c.n_layers))) return rc;
        for (int l = 0; l < c.n_layers; ++l) {
            uint8_t* base = m->kqp_qkv + per * l;
            if ((rc = kx_pack_launch(c.type_q, layer_ptr(m->t[T_Q], l, qw, c.dim), qw, c.dim, base, nf, 0,
                                     ctx().stream)) ||
                (rc = kx_pack_launch(c.type_q, layer_ptr(m->t[T_K], l, kvd, c.dim), kvd, c.dim, base, nf, qw,
                                     ctx().stream)) ||
                (rc = kx_pack_launch(c.type_q, layer_ptr(m->t[T_V], l, kvd, c.dim), kvd, c.dim, base, nf, qw + kvd,
                                     ctx().stream)))
                return rc;
        }
        if (m->q_bias) {   // the family launch adds the bias in its epilogue
            BREW_CUDA(cudaDeviceSynchronize());
            if ((rc = dalloc(m, &m->qkv_bias, (size_t)nf * c.n_layers))) return rc;
            for (int l = 0; l < c.n_layers; ++l) {
                float* fb = m->qkv_bias + (size_t)nf * l;
                BREW_CUDA(cudaMemcpy(fb, m->q_bias + (size_t)qw * l, qw * sizeof(float), cudaMemcpyDeviceToDevice));
                BREW_CUDA(cudaMemcpy(fb + qw, m->k_bias + (size_t)kvd * l, kvd * sizeof(float), cudaMemcpyDeviceToDevice));
                BREW_CUDA(cudaMemcpy(fb + qw + kvd, m->v_bias + (size_t)kvd * l, kvd * sizeof(float),
                                     cudaMemcpyDeviceToDevice));
            }
        }
    }
    // gate and up likewise (rows gate | up), their outputs side by side
    const int64_t hid = c.hidden_dim;
    const bool kq_gu = (c.type_gate == BREW_TYPE_Q4_K || c.type_gate == BREW_TYPE_Q6_K) && c.type_up == c.type_gate &&
                       hid % 16 == 0;
    if (kq_gu) {
        const size_t per = kx_bytes(c.type_gate, 2 * hid, c.dim);
        if ((rc = dalloc(m, &m->kqp_gu, per * c.n_layers)) || (rc = dalloc(m, &m->hgu, (size_t)B * 2 * hid)))
            return rc;
        for (int l = 0; l < c.n_layers; ++l) {
            uint8_t* base = m->kqp_gu + per * l;
            if ((rc = kx_pack_launch(c.type_gate, layer_ptr(m->t[T_GATE], l, hid, c.dim), hid, c.dim, base, 2 * hid, 0,
                                     ctx().stream)) ||
                (rc = kx_pack_launch(c.type_gate, layer_ptr(m->t[T_UP], l, hid, c.dim), hid, c.dim, base, 2 * hid, hid,
                                     ctx().stream)))
                return rc;
        }
    }
    // scratch of the K-quant matvecs: x records, and the split-K partial
    // sums of the largest launch (kq_basis gives each matrix's split)
    size_t kq_part = 0, kq_ctr = 0;
    bool any_kq = false;
    for (int which = T_OUTPUT; which < T_COUNT; ++which) {
        int64_t rows, cols;
        int type, layers;
        matrix_shape(c, which, &rows, &cols, &type, &layers);
        if (type != BREW_TYPE_Q4_K && type != BREW_TYPE_Q6_K) continue;
        any_kq = true;
        const int64_t basis = kq_basis(m, which, rows);
        const int sp = kq_splits(cols, basis);
        if (sp > 1) kq_part = std::max(kq_part, (size_t)sp * KX_MAX_VECTORS * (size_t)((basis + KX_TM - 1) / KX_TM * KX_TM));
        kq_ctr = std::max(kq_ctr, (size_t)((basis + KX_TM - 1) / KX_TM));
    }
    if (any_kq) {
        if ((rc = dalloc(m, &m->kq_rec, kx_rec_bytes(std::min(B, KX_MAX_VECTORS), kmax))) ||
            (rc = dalloc(m, &m->kq_part, std::max<size_t>(kq_part, 1))) ||
            (rc = dalloc(m, &m->kq_ctr, std::max<size_t>(kq_ctr, 1))))
            return rc;
        m->kq_nctr = std::max<size_t>(kq_ctr, 1);
    }
    for (int which = T_OUTPUT; which < T_COUNT; ++which) {
        int64_t rows, cols;
        int type, layers;
        matrix_shape(c, which, &rows, &cols, &type, &layers);
        if (type != BREW_TYPE_Q4_K && type != BREW_TYPE_Q6_K) continue;
        if (kq_qkv && (which == T_Q || which == T_K || which == T_V)) continue;
        if (kq_gu && (which == T_GATE || which == T_UP)) continue;
        const size_t per = kx_bytes(type, rows, cols);
        if ((rc = dalloc(m, &m->kqp[which], per * layers))) return rc;
        for (int l = 0; l < layers; ++l)
            if ((rc = kx_pack_launch(type, layer_ptr(m->t[which], l, rows, cols), rows, (int)cols, m->kqp[which] + per * l,
                                     rows, 0, ctx().stream)))
                return rc;
    }
    BREW_CUDA(cudaStreamSynchronize(ctx().stream));
    m->unfused = true;
    return BREW_OK;
}

int alloc_state(brew_model_s* m) {
    const brew_config& c = m->c;
    const int B = m->max_batch;
    const int64_t qw = (int64_t)c.n_heads * c.head_size, kvd = (int64_t)c.n_kv_heads * c.head_size;
    m->qkvw = (int)(qw + 2 * kvd);
    m->cache_bstride = (int64_t)c.n_layers * c.seq_len * kvd;
    int rc;
    if ((rc = dalloc(m, &m->kc, (size_t)B * m->cache_bstride))) return rc;
    if ((rc = dalloc(m, &m->vc, (size_t)B * m->cache_bstride))) return rc;
    if ((rc = dalloc(m, &m->x, (size_t)B * c.dim))) return rc;
    if ((rc = dalloc(m, &m->xb, (size_t)B * std::max<int64_t>(qw, c.dim)))) return rc;
    if ((rc = dalloc(m, &m->xb2, (size_t)B * c.dim))) return rc;
    if ((rc = dalloc(m, &m->qkv, (size_t)B * m->qkvw))) return rc;
    if ((rc = dalloc(m, &m->hb, (size_t)B * c.hidden_dim))) return rc;
    if ((rc = dalloc(m, &m->logits, (size_t)B * c.vocab_size))) return rc;
    const size_t rec = prep_rec_bytes(B);
    if ((rc = dalloc(m, &m->prep_x, (size_t)(c.dim / 32) * rec))) return rc;
    if ((rc = dalloc(m, &m->prep_q, (size_t)(qw / 32) * rec))) return rc;
    if ((rc = dalloc(m, &m->prep_h, (size_t)(c.hidden_dim / 32) * rec))) return rc;
    m->n_counters = c.hidden_dim / 32 + 8 + B * c.n_kv_heads;
    if ((rc = dalloc(m, &m->counters, (size_t)m->n_counters))) return rc;
    m->nchunk = attn_pick_nchunk(c.n_kv_heads, B, c.seq_len);
    if ((rc = dalloc(m, &m->attn_part, attn_part_floats(B, c.n_heads, m->nchunk, c.head_size)))) return rc;
    if ((rc = dalloc(m, &m->am_key, (size_t)B))) return rc;
    if ((rc = dalloc(m, &m->am_ctr, (size_t)B))) return rc;
    if ((rc = dalloc(m, &m->am_out, (size_t)B))) return rc;
    // tokens and positions side by side: one upload per forward call
    if ((rc = dalloc(m, &m->tokens_d, (size_t)2 * B))) return rc;
    m->pos_d = m->tokens_d + B;
    if ((rc = dalloc(m, &m->gen_d, (size_t)c.seq_len + 1))) return rc;
    if (uses_kquants(c) && (rc = alloc_unfused(m))) return rc;
    m->h_pin_cap = std::max(4 * B, 64);
    BREW_CUDA(cudaMallocHost(&m->h_pin, (size_t)m->h_pin_cap * sizeof(int32_t)));
    return BREW_OK;
}

int upload_vec(brew_model_s* m, float** dst, const float* src, size_t n) {
    if (!src) return BREW_OK;
    int rc = dalloc(m, dst, n);
    if (rc) return rc;
    BREW_CUDA(cudaMemcpy(*dst, src, n * sizeof(float), cudaMemcpyHostToDevice));
    BREW_CUDA(cudaStreamSynchronize(0));   // pageable copy on the legacy stream: landed before the model's kernels
    return BREW_OK;
}

int fill_vec(brew_model_s* m, float** dst, size_t n, float v) {
    int rc = dalloc(m, dst, n);
    if (rc) return rc;
    return fill_f32_launch(*dst, (int64_t)n, v, ctx().stream);
}

const uint8_t* layer_ptr(brew_tensor t, int layer, int64_t rows, int64_t cols) {
    TypeInfo ti;
    type_info(t->type, &ti);
    return t->d + (int64_t)layer * (rows * cols / ti.block_elems) * ti.block_bytes;
}

int64_t row_bytes_of(int type, int64_t cols) {
    TypeInfo ti;
    type_info(type, &ti);
    return cols / ti.block_elems * ti.block_bytes;
}

// Enqueues one forward pass for `B` sequences reading tokens_d / pos_d.
// y[b][0:N] = W x[b] for any supported type: the K-quant kernel, or the
// int8-MMA matvec after preparing x's records.
int mv_any(brew_model_s* m, int type, const uint8_t* w, const float* x, int ldx, int K, int N, float* y, int ldy, int B,
           cudaStream_t s) {
    const int64_t rb = row_bytes_of(type, K);
    if (type == BREW_TYPE_Q4_K || type == BREW_TYPE_Q6_K)
        return kquant_matvec_launch(type, w, rb, x, ldx, K, N, y, ldy, B, s, false);
    for (int b0 = 0; b0 < B; b0 += MV_MAX_BATCH) {   // the MMA matvec takes up to MV_MAX_BATCH vectors
        const int nb = std::min(MV_MAX_BATCH, B - b0);
        int rc = prep_launch(x + (int64_t)b0 * ldx, ldx, K, nb, nullptr, 0.0f, m->prep_any, s, false);
        if (rc) return rc;
        MvParams p = {};
        p.type = type;
        p.K = K;
        p.row_bytes = rb;
        p.batch = nb;
        p.ldy = ldy;
        p.epi = MV_EPI_STORE;
        p.nseg = 1;
        p.seg[0] = {w, y + (int64_t)b0 * ldy, nullptr, nullptr, N, 0};
        p.prep = m->prep_any;
        p.err = ctx().err_word;
        if ((rc = mv_launch(p, s, false))) return rc;
    }
    return BREW_OK;
}

// The expanded copy holding rows row0.. of matrix `which` (layer l, rows x
// K): the copy of its family (q|k|v, gate|up) or its own, with the rows'
// offset in it; base null when the matrix has none.
struct KxRef {
    const uint8_t* base;
    int64_t N, row0;
    int64_t basis;   // rows of the one-GPU family: its split of K
};

KxRef kx_ref(const brew_model_s* m, int which, int l, int64_t rows, int K, int64_t row0) {
    const brew_config& c = m->c;
    const int type = m->t[which]->type;
    if (m->kqp_qkv && (which == T_Q || which == T_K || which == T_V)) {
        const int64_t qw = (int64_t)c.n_heads * c.head_size, kvd = (int64_t)c.n_kv_heads * c.head_size, nf = qw + 2 * kvd;
        const int64_t off = which == T_Q ? 0 : which == T_K ? qw : qw + kvd;   // rows before it in the family
        return {m->kqp_qkv + (size_t)l * kx_bytes(type, nf, K), nf, off + row0, nf};
    }
    if (m->kqp_gu && (which == T_GATE || which == T_UP)) {
        const int64_t hid = c.hidden_dim;
        return {m->kqp_gu + (size_t)l * kx_bytes(type, 2 * hid, K), 2 * hid, (which == T_GATE ? 0 : hid) + row0, 2 * hid};
    }
    if (!m->kqp[which]) return {nullptr, 0, 0, 0};
    return {m->kqp[which] + (size_t)l * kx_bytes(type, rows, K), rows, row0, rows};
}

// y[b][0:n] = rows r.row0 .. r.row0 + n - 1 of the expanded copy r times
// x[b] (+ the family-indexed bias), in groups of KX_MAX_VECTORS vectors
// (the x records of a group, then the tcgen05 matvec); `rec`: the records
// of all B <= KX_MAX_VECTORS vectors, made already by the kernel that
// produced x.  The split of K follows the family's rows, so a sharded
// launch sums each row as the one-GPU launch does.
int kq_run(brew_model_s* m, int type, const KxRef& r, int n, int K, const float* x, int ldx, float* y, int ldy, int B,
           cudaStream_t s, const uint8_t* rec = nullptr, const float* bias = nullptr) {
    const int splits = kq_splits(K, (m->comm && m->comm->nranks > 1 && !m->tp_exact) ? (int64_t)n : r.basis);
    if (rec) {
        BREW_CHECK(B <= KX_MAX_VECTORS, BREW_ERR_INVALID_ARG, "records of %d vectors", B);
        return kx_mma_launch(type, r.base, r.N, r.row0, n, K, rec, B, splits, m->kq_part, m->kq_ctr, bias, y, ldy,
                             ctx().err_word, s);
    }
    for (int b0 = 0; b0 < B; b0 += KX_MAX_VECTORS) {
        const int nb = std::min(KX_MAX_VECTORS, B - b0);
        int rc = kx_prep_launch(x + (int64_t)b0 * ldx, ldx, K, nb, m->kq_rec, s);
        if (!rc)
            rc = kx_mma_launch(type, r.base, r.N, r.row0, n, K, m->kq_rec, nb, splits, m->kq_part, m->kq_ctr, bias,
                               y + (int64_t)b0 * ldy, ldy, ctx().err_word, s);
        if (rc) return rc;
    }
    return BREW_OK;
}

// One matvec of the unfused forward; `rec` (records of x for a tcgen05
// K-quant matvec, or null) is used when the matrix runs on that path.
int mv_w(brew_model_s* m, int which, int l, int64_t rows, int K, int64_t row0, int n, const float* x, int ldx, float* y,
         int ldy, int B, cudaStream_t s, const uint8_t* rec = nullptr) {
    brew_tensor t = m->t[which];
    const int type = t->type;
    const KxRef r = kx_ref(m, which, l, rows, K, row0);
    if (r.base) return kq_run(m, type, r, n, K, x, ldx, y, ldy, B, s, rec);
    return mv_any(m, type, layer_ptr(t, l, rows, K) + row0 * row_bytes_of(type, K), x, ldx, K, n, y, ldy, B, s);
}

// The forward of a model with K-quant matrices (the Qwen2.5-7B Q4_K/Q6_K
// config) and of tensor-parallel models: per layer, residual + RMSNorm (+ the
// next tcgen05 K-quant matvec's x records) in one kernel, the q|k|v matvec
// (bias in its epilogue when q|k|v is one family), attention, wo, residual +
// RMSNorm, gate|up, GLU (+ records), down; each residual is applied by the
// next norm kernel.  Op order of the reference's forward methods
// (model/*/...Transformer.java).
int enqueue_forward_unfused(brew_model_s* m, int B, bool with_classifier, cudaStream_t s) {
    const brew_config& c = m->c;
    const int L = c.n_layers, dim = c.dim, hd = c.head_size, hid = c.hidden_dim;
    const int qw = c.n_heads * hd, kvd = c.n_kv_heads * hd;
    const bool gemma = arch_gemma(c.arch);
    const bool qknorm = arch_qknorm(c.arch);
    unsigned int* err = ctx().err_word;
    int* attn_ctr = m->counters + hid / 32 + 8;
    int rc;
    // tensor parallelism: this rank multiplies rows [R*N/P, (R+1)*N/P) of
    // every matrix and the slices are all-gathered
    const int P = m->comm ? m->comm->nranks : 1, R = m->comm ? m->comm->rank : 0;
    // gather site k of layer l (k: 0 q|k|v, 1 wo, 2 gate|up, 3 down; the
    // logits are site 4 L): peer stores into every rank's tagged slot, or an
    // NCCL all-gather and an unshard kernel
    const size_t mb = (size_t)m->max_batch;
    auto site_off = [&](int site) -> size_t {
        if (site == 4 * L) return (size_t)L * m->tp_layer_words;
        const size_t o[4] = {0, mb * m->qkvw, mb * (m->qkvw + dim), mb * (m->qkvw + dim + hid)};
        return (size_t)(site / 4) * m->tp_layer_words + o[site % 4];
    };
    auto gather_from = [&](const float* src, int slice, const TpSeg* segs, int nseg, float* dst, int ldd, int site) {
        if (m->tp_p2p) {
            const size_t off = site_off(site);
            int r = tp_push_launch(src, B, slice, segs, nseg, ldd, m->tp_peers, P, R, off, m->tp_step, site, s);
            if (!r) r = tp_pull_launch(m->tp_arena + off, B, ldd, dst, m->tp_step, site, m->tp_abort, err, s);
            return r;
        }
        int r = tp_allgather(m->comm, src, m->tp_recv, (size_t)B * slice, s);
        if (!r) r = tp_unshard_launch(m->tp_recv, P, B, slice, segs, nseg, dst, ldd, s);
        return r;
    };
    auto gather = [&](int slice, const TpSeg* segs, int nseg, float* dst, int ldd, int site) {
        return gather_from(m->tp_send, slice, segs, nseg, dst, ldd, site);
    };
    // attention sharded by kv head when the kv heads divide over the ranks:
    // rank R's q|k|v rows are exactly its heads' q, k and v, so attention
    // runs on them locally (its K/V cache holds only those heads) and the
    // attention output is gathered instead of q|k|v
    const bool shard_attn = P > 1 && c.n_kv_heads % P == 0;
    const int qs = qw / P, ks = kvd / P, sl = qs + 2 * ks;
    if (P > 1 && m->tp_p2p && (rc = tp_step_launch(m->tp_step, s))) return rc;
    // embedding row (scaled for Gemma3); its records are not used here
    if ((rc = embed_prep_launch(c.type_embed, m->t[T_EMBED]->d, c.vocab_size, dim, m->tokens_d, B, gemma, m->x,
                                m->rms_att, c.eps, m->prep_x, err, s, false)))
        return rc;
    // The x records of a tcgen05 K-quant matvec's input are made by the
    // kernel that produces the input (norm_prep / glu_prep) when the next
    // matvec runs on that path; the residual of each sub-layer is applied by
    // the next norm_prep.
    auto rec_for = [&](int which, int l, int64_t rows, int K) -> uint8_t* {
        return B <= KX_MAX_VECTORS && kx_ref(m, which, l, rows, K, 0).base ? m->kq_rec : nullptr;
    };
    for (int l = 0; l < L; ++l) {
        // the previous layer's FFN residual, then the attention RMSNorm
        uint8_t* rq = rec_for(T_Q, l, qw, dim);
        if ((rc = norm_prep_launch(m->x, dim, l ? m->xb2 : nullptr, dim,
                                   gemma && l ? m->post_ffn + (int64_t)(l - 1) * dim : nullptr,
                                   m->rms_att + (int64_t)l * dim, c.eps, dim, B, m->xn, dim, rq, s)))
            return rc;
        float* q = m->qkv;
        float* k = m->qkv + qw;
        float* v = m->qkv + qw + kvd;
        if (P == 1) {
            if (m->kqp_qkv) {   // q | k | v in one launch per vector group, the bias in its epilogue
                const float* fb = m->qkv_bias ? m->qkv_bias + (int64_t)l * (qw + 2 * kvd) : nullptr;
                if ((rc = kq_run(m, c.type_q, kx_ref(m, T_Q, l, qw, dim, 0), m->qkvw, dim, m->xn, dim, q, m->qkvw, B,
                                 s, rq, fb)))
                    return rc;
            } else if ((rc = mv_w(m, T_Q, l, qw, dim, 0, qw, m->xn, dim, q, m->qkvw, B, s, rq)) ||
                       (rc = mv_w(m, T_K, l, kvd, dim, 0, kvd, m->xn, dim, k, m->qkvw, B, s, rq)) ||
                       (rc = mv_w(m, T_V, l, kvd, dim, 0, kvd, m->xn, dim, v, m->qkvw, B, s, rq)))
                return rc;
            if (m->q_bias && !(m->kqp_qkv && m->qkv_bias) &&
                ((rc = add_bias_launch(q, m->qkvw, m->q_bias + (int64_t)l * qw, qw, B, s)) ||
                 (rc = add_bias_launch(k, m->qkvw, m->k_bias + (int64_t)l * kvd, kvd, B, s)) ||
                 (rc = add_bias_launch(v, m->qkvw, m->v_bias + (int64_t)l * kvd, kvd, B, s))))
                return rc;
        } else {
            // slices [q_R | k_R | v_R] per rank, gathered into q | k | v
            // (unless attention is sharded)
            float* sq = m->tp_send;
            if (m->kqp_qkv_tp) {   // this rank's q|k|v rows: one launch, the bias in its epilogue
                const KxRef r = {m->kqp_qkv_tp + (size_t)l * kx_bytes(c.type_q, sl, dim), sl, 0, qw + 2 * kvd};
                if ((rc = kq_run(m, c.type_q, r, sl, dim, m->xn, dim, sq, sl, B, s, rq,
                                 m->qkv_bias_tp ? m->qkv_bias_tp + (int64_t)l * sl : nullptr)))
                    return rc;
            } else if ((rc = mv_w(m, T_Q, l, qw, dim, (int64_t)R * qs, qs, m->xn, dim, sq, sl, B, s, rq)) ||
                (rc = mv_w(m, T_K, l, kvd, dim, (int64_t)R * ks, ks, m->xn, dim, sq + qs, sl, B, s, rq)) ||
                (rc = mv_w(m, T_V, l, kvd, dim, (int64_t)R * ks, ks, m->xn, dim, sq + qs + ks, sl, B, s, rq)))
                return rc;
            if (m->q_bias && !(m->kqp_qkv_tp && m->qkv_bias_tp) &&
                ((rc = add_bias_launch(sq, sl, m->q_bias + (int64_t)l * qw + (int64_t)R * qs, qs, B, s)) ||
                 (rc = add_bias_launch(sq + qs, sl, m->k_bias + (int64_t)l * kvd + (int64_t)R * ks, ks, B, s)) ||
                 (rc = add_bias_launch(sq + qs + ks, sl, m->v_bias + (int64_t)l * kvd + (int64_t)R * ks, ks, B, s))))
                return rc;
            const TpSeg segs[3] = {{qs, 0, 0}, {ks, qs, qw}, {ks, qs + ks, qw + kvd}};
            if (!shard_attn && (rc = gather(sl, segs, 3, m->qkv, m->qkvw, 4 * l))) return rc;
        }
        {
            AttnParams a = {};
            a.batch = B;
            a.n_heads = c.n_heads;
            a.n_kv = c.n_kv_heads;
            a.hd = hd;
            a.seq_len = c.seq_len;
            a.arch = c.arch;
            a.window = arch_window(c.arch, l, c.sliding_window);   // Gemma2/Gemma3AttentionPattern.java:10-16
            a.rope = arch_rope_layer(c.arch, l) ? 1 : 0;
            a.eps = c.eps;
            a.rope_base = arch_rope_base(c.arch, c.rope_base, gemma && !arch_global_layer(c.arch, l));
            a.rope_scale = c.rope_scale > 0.0f ? c.rope_scale : 1.0f;
            a.inv_scale = 1.0f / (float)std::sqrt((double)hd);   // AttentionEngine.java:18-19
            a.q = q;
            a.k = k;
            a.v = v;
            a.ldq = a.ldkv = m->qkvw;
            a.qnorm_w = qknorm ? m->rms_q + (int64_t)l * hd : nullptr;
            a.knorm_w = qknorm ? m->rms_k + (int64_t)l * hd : nullptr;
            a.kcache = m->kc + (int64_t)l * c.seq_len * kvd;
            a.vcache = m->vc + (int64_t)l * c.seq_len * kvd;
            a.cache_bstride = m->cache_bstride;
            a.pos = m->pos_d;
            a.xb = m->xb;
            a.ldxb = qw;
            a.part = m->attn_part;
            a.counters = attn_ctr;
            a.nchunk = m->nchunk;
            a.prep_out = nullptr;   // the matvecs of this forward make their own x records
            a.err = err;
            if (shard_attn) {   // this rank's heads; the cache holds [layer][position][its kv heads]
                a.n_heads = c.n_heads / P;
                a.n_kv = c.n_kv_heads / P;
                a.q = m->tp_send;
                a.k = m->tp_send + qs;
                a.v = m->tp_send + qs + ks;
                a.ldq = a.ldkv = sl;
                a.kcache = m->kc + (int64_t)l * c.seq_len * ks;
                a.vcache = m->vc + (int64_t)l * c.seq_len * ks;
                a.xb = m->tp_g;
                a.ldxb = qs;
            }
            if ((rc = attn_launch(a, s, false))) return rc;
            const TpSeg xseg = {qs, 0, 0};
            if (shard_attn && (rc = gather_from(m->tp_g, qs, &xseg, 1, m->xb, qw, 4 * l))) return rc;
        }
        if (P == 1) {
            if ((rc = mv_w(m, T_O, l, dim, qw, 0, dim, m->xb, qw, m->xb2, dim, B, s)))
                return rc;
        } else {
            const TpSeg seg = {dim / P, 0, 0};
            if ((rc = mv_w(m, T_O, l, dim, qw, (int64_t)R * (dim / P), dim / P, m->xb, qw, m->tp_send, dim / P, B, s)) ||
                (rc = gather(dim / P, &seg, 1, m->xb2, dim, 4 * l + 1)))
                return rc;
        }
        // the attention residual, then the FFN RMSNorm
        uint8_t* rg = rec_for(T_GATE, l, hid, dim);
        if ((rc = norm_prep_launch(m->x, dim, m->xb2, dim, gemma ? m->post_att + (int64_t)l * dim : nullptr,
                                   m->rms_ffn + (int64_t)l * dim, c.eps, dim, B, m->xn, dim, rg, s)))
            return rc;
        uint8_t* rd = rec_for(T_DOWN, l, dim, hid);
        if (P == 1 && m->kqp_gu) {
            // gate | up in one launch per vector group; GLU into the gate half
            if ((rc = kq_run(m, c.type_gate, kx_ref(m, T_GATE, l, hid, dim, 0), 2 * hid, dim, m->xn, dim, m->hgu,
                             2 * hid, B, s, rg)) ||
                (rc = glu_prep_launch(m->hgu, m->hgu, m->hgu + hid, 2 * hid, hid, B, gemma, rd, s)) ||
                (rc = mv_w(m, T_DOWN, l, dim, hid, 0, dim, m->hgu, 2 * hid, m->xb2, dim, B, s, rd)))
                return rc;
        } else if (P == 1) {
            if ((rc = mv_w(m, T_GATE, l, hid, dim, 0, hid, m->xn, dim, m->hb, hid, B, s, rg)) ||
                (rc = mv_w(m, T_UP, l, hid, dim, 0, hid, m->xn, dim, m->hb2, hid, B, s, rg)) ||
                (rc = glu_prep_launch(m->hb, m->hb, m->hb2, hid, hid, B, gemma, rd, s)) ||
                (rc = mv_w(m, T_DOWN, l, dim, hid, 0, dim, m->hb, hid, m->xb2, dim, B, s, rd)))
                return rc;
        } else {
            const int hs = hid / P;
            const TpSeg hseg = {hs, 0, 0}, dseg = {dim / P, 0, 0};
            if (m->kqp_gu_tp) {   // this rank's gate|up rows: one launch, then the GLU of the local slice
                const KxRef r = {m->kqp_gu_tp + (size_t)l * kx_bytes(c.type_gate, 2 * hs, dim), 2 * hs, 0, 2 * hid};
                if ((rc = kq_run(m, c.type_gate, r, 2 * hs, dim, m->xn, dim, m->tp_gu, 2 * hs, B, s, rg)) ||
                    (rc = glu_launch(m->tp_send, m->tp_gu, m->tp_gu + hs, 2 * hs, hs, B, gemma, s, hs)))
                    return rc;
            } else if ((rc = mv_w(m, T_GATE, l, hid, dim, (int64_t)R * hs, hs, m->xn, dim, m->tp_g, hs, B, s, rg)) ||
                       (rc = mv_w(m, T_UP, l, hid, dim, (int64_t)R * hs, hs, m->xn, dim, m->tp_u, hs, B, s, rg)) ||
                       (rc = glu_launch(m->tp_send, m->tp_g, m->tp_u, hs, hs, B, gemma, s))) {
                return rc;
            }
            if ((rc = gather(hs, &hseg, 1, m->hb, hid, 4 * l + 2)) ||
                (rc = mv_w(m, T_DOWN, l, dim, hid, (int64_t)R * (dim / P), dim / P, m->hb, hid, m->tp_send, dim / P, B,
                           s)) ||
                (rc = gather(dim / P, &dseg, 1, m->xb2, dim, 4 * l + 3)))
                return rc;
        }
    }
    const float* post_last = gemma ? m->post_ffn + (int64_t)(L - 1) * dim : nullptr;
    if (!with_classifier) return residual_launch(m->x, dim, m->xb2, dim, post_last, c.eps, dim, B, s);
    const int V = c.vocab_size;
    // the last FFN residual, then the final RMSNorm
    uint8_t* rcls = rec_for(T_OUTPUT, 0, V, dim);
    if ((rc = norm_prep_launch(m->x, dim, m->xb2, dim, post_last, m->rms_final, c.eps, dim, B, m->xn, dim, rcls, s)))
        return rc;
    if (P == 1) {
        if ((rc = mv_w(m, T_OUTPUT, 0, V, dim, 0, V, m->xn, dim, m->logits, V, B, s, rcls))) return rc;
        return argmax_launch(m->logits, V, V, B, m->am_key, m->am_ctr, m->am_out, s, false);
    }
    // sharded classifier: per-rank argmax keys, gathered and reduced; the
    // logits slices are gathered too (brew_model_forward returns them)
    const int vs = V / P;
    const TpSeg vseg = {vs, 0, 0};
    if ((rc = mv_w(m, T_OUTPUT, 0, V, dim, (int64_t)R * vs, vs, m->xn, dim, m->tp_send, vs, B, s, rcls)) ||
        (rc = tp_argmax_keys_launch(m->tp_send, vs, vs, B, R * vs, m->tp_keys, s)) ||
        (rc = tp_allgather_u64(m->comm, m->tp_keys, m->tp_keys_all, (size_t)B, s)) ||
        (rc = tp_argmax_reduce_launch(m->tp_keys_all, P, B, m->am_out, s)) ||
        (rc = gather(vs, &vseg, 1, m->logits, V, 4 * L)))
        return rc;
    return BREW_OK;
}

int enqueue_forward(brew_model_s* m, int B, bool with_classifier, cudaStream_t s) {
    if (m->unfused) return enqueue_forward_unfused(m, B, with_classifier, s);
    const brew_config& c = m->c;
    const int L = c.n_layers, dim = c.dim, hd = c.head_size, hid = c.hidden_dim;
    const int qw = c.n_heads * hd, kvd = c.n_kv_heads * hd;
    const bool gemma = arch_gemma(c.arch);
    const bool qknorm = arch_qknorm(c.arch);
    unsigned int* err = ctx().err_word;
    int* group_ctr = m->counters;
    int* post_ctr = group_ctr + hid / 32;
    int* attn_ctr = post_ctr + 8;
    int rc;

    rc = embed_prep_launch(c.type_embed, m->t[T_EMBED]->d, c.vocab_size, dim, m->tokens_d, B, gemma, m->x, m->rms_att,
                           c.eps, m->prep_x, err, s, true);
    if (rc) return rc;

    for (int l = 0; l < L; ++l) {
        // 1. Q|K|V
        {
            MvParams p = {};
            p.type = c.type_q;
            p.K = dim;
            p.row_bytes = row_bytes_of(c.type_q, dim);
            p.batch = B;
            p.ldy = m->qkvw;
            p.epi = MV_EPI_STORE;
            p.nseg = 3;
            p.seg[0] = {layer_ptr(m->t[T_Q], l, qw, dim), m->qkv, m->q_bias ? m->q_bias + (int64_t)l * qw : nullptr,
                        nullptr, qw, 0};
            p.seg[1] = {layer_ptr(m->t[T_K], l, kvd, dim), m->qkv + qw, m->k_bias ? m->k_bias + (int64_t)l * kvd : nullptr,
                        nullptr, kvd, 0};
            p.seg[2] = {layer_ptr(m->t[T_V], l, kvd, dim), m->qkv + qw + kvd,
                        m->v_bias ? m->v_bias + (int64_t)l * kvd : nullptr, nullptr, kvd, 0};
            p.prep = m->prep_x;
            p.err = err;
            if ((rc = mv_launch(p, s, true))) return rc;
        }
        // 2. attention
        {
            AttnParams a = {};
            a.batch = B;
            a.n_heads = c.n_heads;
            a.n_kv = c.n_kv_heads;
            a.hd = hd;
            a.seq_len = c.seq_len;
            a.arch = c.arch;
            a.window = arch_window(c.arch, l, c.sliding_window);   // Gemma2/Gemma3AttentionPattern.java:10-16
            a.rope = arch_rope_layer(c.arch, l) ? 1 : 0;
            a.eps = c.eps;
            a.rope_base = arch_rope_base(c.arch, c.rope_base, gemma && !arch_global_layer(c.arch, l));
            a.rope_scale = c.rope_scale > 0.0f ? c.rope_scale : 1.0f;
            a.inv_scale = 1.0f / (float)std::sqrt((double)hd);   // AttentionEngine.java:18-19
            a.q = m->qkv;
            a.k = m->qkv + qw;
            a.v = m->qkv + qw + kvd;
            a.ldq = a.ldkv = m->qkvw;
            a.qnorm_w = qknorm ? m->rms_q + (int64_t)l * hd : nullptr;
            a.knorm_w = qknorm ? m->rms_k + (int64_t)l * hd : nullptr;
            a.kcache = m->kc + (int64_t)l * c.seq_len * kvd;
            a.vcache = m->vc + (int64_t)l * c.seq_len * kvd;
            a.cache_bstride = m->cache_bstride;
            a.pos = m->pos_d;
            a.xb = m->xb;
            a.ldxb = qw;
            a.part = m->attn_part;
            a.counters = attn_ctr;
            a.nchunk = m->nchunk;
            a.prep_out = m->prep_q;
            a.err = err;
            if ((rc = attn_launch(a, s, true))) return rc;
        }
        // 3. wo (+ residual or Gemma3 post-attention norm), then FFN norm
        {
            MvParams p = {};
            p.type = c.type_o;
            p.K = qw;
            p.row_bytes = row_bytes_of(c.type_o, qw);
            p.batch = B;
            p.ldy = dim;
            p.epi = MV_EPI_STORE;
            p.nseg = 1;
            p.seg[0] = {layer_ptr(m->t[T_O], l, dim, qw), gemma ? m->xb2 : m->x, nullptr, gemma ? nullptr : m->x, dim, 0};
            p.prep = m->prep_q;
            p.post = MV_POST_PREP;
            p.post_counter = post_ctr;
            p.post_x = m->x;
            p.post_ld = dim;
            p.post_dim = dim;
            p.post_add = gemma ? m->xb2 : nullptr;
            p.post_add_w = gemma ? m->post_att + (int64_t)l * dim : nullptr;
            p.post_norm_w = m->rms_ffn + (int64_t)l * dim;
            p.eps = c.eps;
            p.post_prep = m->prep_x;
            p.err = err;
            if ((rc = mv_launch(p, s, true))) return rc;
        }
        // 4. gate|up with the gated activation
        {
            MvParams p = {};
            p.type = c.type_gate;
            p.K = dim;
            p.row_bytes = row_bytes_of(c.type_gate, dim);
            p.batch = B;
            p.ldy = hid;
            p.epi = gemma ? MV_EPI_GLU_GELU : MV_EPI_GLU_SILU;
            p.nseg = 2;
            p.seg[0] = {layer_ptr(m->t[T_GATE], l, hid, dim), m->hb, nullptr, nullptr, hid, 0};
            p.seg[1] = {layer_ptr(m->t[T_UP], l, hid, dim), nullptr, nullptr, nullptr, hid, 0};
            p.prep = m->prep_x;
            p.next_prep = m->prep_h;
            p.group_counters = group_ctr;
            p.err = err;
            if ((rc = mv_launch(p, s, true))) return rc;
        }
        // 5. down (+ residual or Gemma3 post-FFN norm), then the next norm
        {
            MvParams p = {};
            p.type = c.type_down;
            p.K = hid;
            p.row_bytes = row_bytes_of(c.type_down, hid);
            p.batch = B;
            p.ldy = dim;
            p.epi = MV_EPI_STORE;
            p.nseg = 1;
            p.seg[0] = {layer_ptr(m->t[T_DOWN], l, dim, hid), gemma ? m->xb2 : m->x, nullptr, gemma ? nullptr : m->x, dim, 0};
            p.prep = m->prep_h;
            p.post = MV_POST_PREP;
            p.post_counter = post_ctr;
            p.post_x = m->x;
            p.post_ld = dim;
            p.post_dim = dim;
            p.post_add = gemma ? m->xb2 : nullptr;
            p.post_add_w = gemma ? m->post_ffn + (int64_t)l * dim : nullptr;
            p.post_norm_w = l + 1 < L ? m->rms_att + (int64_t)(l + 1) * dim : m->rms_final;
            p.eps = c.eps;
            p.post_prep = m->prep_x;
            p.err = err;
            if ((rc = mv_launch(p, s, true))) return rc;
        }
    }
    if (!with_classifier) return BREW_OK;
    {
        const int otype = c.tied_embeddings ? c.type_embed : c.type_output;
        MvParams p = {};
        p.type = otype;
        p.K = dim;
        p.row_bytes = row_bytes_of(otype, dim);
        p.batch = B;
        p.ldy = c.vocab_size;
        p.epi = MV_EPI_STORE;
        p.nseg = 1;
        p.seg[0] = {m->t[T_OUTPUT]->d, m->logits, nullptr, nullptr, c.vocab_size, 0};
        p.prep = m->prep_x;
        const bool fused = B <= MV_ARGMAX_MAX_BATCH;
        p.post = fused ? MV_POST_ARGMAX : MV_POST_NONE;
        p.post_counter = post_ctr;
        p.am_key = m->am_key;
        p.am_out = m->am_out;
        p.err = err;
        if ((rc = mv_launch(p, s, true))) return rc;
        if (!fused && (rc = argmax_launch(m->logits, c.vocab_size, c.vocab_size, B, m->am_key, m->am_ctr, m->am_out, s,
                                          true)))
            return rc;
    }
    return BREW_OK;
}

int get_graph(brew_model_s* m, int B, bool with_classifier, cudaGraphExec_t* out) {
    const int key = B * 2 + (with_classifier ? 1 : 0);
    auto it = m->graphs.find(key);
    if (it != m->graphs.end()) {
        *out = it->second;
        return BREW_OK;
    }
    cudaStream_t s = ctx().stream;
    cudaGraph_t g = nullptr;
    const int64_t before = brew_kernel_launches();
    BREW_CUDA(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
    int rc = enqueue_forward(m, B, with_classifier, s);
    cudaError_t e = cudaStreamEndCapture(s, &g);
    // captured kernels do not run yet: count them per replay instead
    const int nk = (int)(brew_kernel_launches() - before);
    count_launch(-nk);
    m->graph_kernels[key] = nk;
    if (rc) {
        if (g) cudaGraphDestroy(g);
        return rc;
    }
    BREW_CUDA(e);
    cudaGraphExec_t exec = nullptr;
    e = cudaGraphInstantiate(&exec, g, 0);
    cudaGraphDestroy(g);
    BREW_CUDA(e);
    m->graphs[key] = exec;
    *out = exec;
    return BREW_OK;
}

int launch_graph(brew_model_s* m, int B, bool with_classifier, cudaStream_t s) {
    cudaGraphExec_t g;
    int rc = get_graph(m, B, with_classifier, &g);
    if (rc) return rc;
    BREW_CUDA(cudaGraphLaunch(g, s));
    count_launch(m->graph_kernels[B * 2 + (with_classifier ? 1 : 0)]);
    return BREW_OK;
}

int launch_forward(brew_model_s* m, int B, bool with_classifier, cudaStream_t s) {
    if (m->use_decode && B == 1) {
        // the decode kernel always runs the classifier (prefill logits are
        // simply not read)
        return decode_launch(m->dp, s);
    }
    return launch_graph(m, B, with_classifier, s);
}

int launch_step(brew_model_s* m, const int32_t* tok_src, int pos, int32_t* record, cudaStream_t s) {
    step_kernel<<<1, 32, 0, s>>>(m->tokens_d, m->pos_d, tok_src, pos, record, m->am_out);
    BREW_CUDA(cudaGetLastError());
    count_launch();
    return BREW_OK;
}

// ---- batched prefill (prefill.cuh) ----

constexpr int PF_CHUNK = 512;   // prompt tokens per pass through the layers

bool prefill_supported(const brew_config& c, std::string* why) {
    const int qw = c.n_heads * c.head_size, kvd = c.n_kv_heads * c.head_size;
    const int types[] = {c.type_q, c.type_k, c.type_v, c.type_o, c.type_gate, c.type_up, c.type_down};
    for (int t : types)
        if (t != BREW_TYPE_Q8_0 && t != BREW_TYPE_Q4_0) {
            *why = "the batched prefill takes Q8_0 or Q4_0 layer matrices";
            return false;
        }
    if ((qw + 2 * kvd) % GEMM_TM || c.dim % GEMM_TM || (2 * c.hidden_dim) % GEMM_TM) {
        *why = "the batched prefill needs q|k|v, dim and 2*hidden_dim rows in multiples of 128";
        return false;
    }
    if (!prefill_shapes_supported(c.n_heads, c.n_kv_heads, c.head_size)) {
        *why = "the batched prefill takes head size 64, 128 or 256 and at most 32 q heads per kv head";
        return false;
    }
    return true;
}

// RoPE tables [2][seq_len][hd/2] (0: global / default base, 1: Gemma3 local).
int ensure_rope_tables(brew_model_s* m) {
    if (m->rope_cos) return BREW_OK;
    const brew_config& c = m->c;
    const int hd = c.head_size, half = hd / 2;
    int rc;
    if ((rc = dalloc(m, &m->rope_cos, (size_t)2 * c.seq_len * half))) return rc;
    if ((rc = dalloc(m, &m->rope_sin, (size_t)2 * c.seq_len * half))) return rc;
    const float base0 = arch_rope_base(c.arch, c.rope_base, false);   // global / only table
    const float base1 = arch_rope_base(c.arch, c.rope_base, true);    // Gemma local layers
    const float scale = c.rope_scale > 0.0f ? c.rope_scale : 1.0f;
    return rope_tables_launch(m->rope_cos, m->rope_sin, c.seq_len, hd, base0, base1, scale, ctx().stream);
}

// GEMM-layout copies of every layer's matrices (Q|K|V and gate|up each
// concatenated by rows) and the buffers of one chunk.
int setup_prefill(brew_model_s* m) {
    if (m->pf_ready) return BREW_OK;
    const brew_config& c = m->c;
    const int L = c.n_layers, dim = c.dim, hid = c.hidden_dim;
    const int qw = c.n_heads * c.head_size, kvd = c.n_kv_heads * c.head_size, qkvw = qw + 2 * kvd;
    int rc;
    if ((rc = ensure_rope_tables(m))) return rc;
    const int N[4] = {qkvw, dim, 2 * hid, dim}, K[4] = {dim, qw, dim, hid};
    for (int f = 0; f < 4; ++f) {
        if ((rc = dalloc(m, &m->pf_wq[f], (size_t)L * N[f] * K[f]))) return rc;
        if ((rc = dalloc(m, &m->pf_wd[f], (size_t)L * N[f] * (K[f] / 32)))) return rc;
    }
    cudaStream_t s = ctx().stream;
    // one GGUF matrix (rows x cols) of layer l into rows [row0, row0 + rows) of family f
    auto pack = [&](int f, int l, int row0, int which, int rows, int cols) {
        int8_t* wq = m->pf_wq[f] + (int64_t)l * N[f] * K[f];            // this layer's quant tiles
        uint16_t* wd = m->pf_wd[f] + (int64_t)l * N[f] * (K[f] / 32);   // this layer's [K/32][N] scales
        return gemm_pack_launch(m->t[which]->type, layer_ptr(m->t[which], l, rows, cols), rows, cols, wq, wd, N[f],
                                row0, s);
    };
    for (int l = 0; l < L; ++l) {
        if ((rc = pack(0, l, 0, T_Q, qw, dim)) || (rc = pack(0, l, qw, T_K, kvd, dim)) ||
            (rc = pack(0, l, qw + kvd, T_V, kvd, dim)) || (rc = pack(1, l, 0, T_O, dim, qw)) ||
            (rc = pack(2, l, 0, T_GATE, hid, dim)) || (rc = pack(2, l, hid, T_UP, hid, dim)) ||
            (rc = pack(3, l, 0, T_DOWN, dim, hid)))
            return rc;
    }
    const int cap = std::min(PF_CHUNK, (c.seq_len + GEMM_TT - 1) / GEMM_TT * GEMM_TT);
    const int kmax = std::max(std::max(dim, qw), hid);
    if ((rc = dalloc(m, &m->pf_x, (size_t)cap * dim)) || (rc = dalloc(m, &m->pf_xn, (size_t)cap * dim)) ||
        (rc = dalloc(m, &m->pf_qkv, (size_t)cap * qkvw)) || (rc = dalloc(m, &m->pf_xb, (size_t)cap * qw)) ||
        (rc = dalloc(m, &m->pf_xb2, (size_t)cap * dim)) || (rc = dalloc(m, &m->pf_h, (size_t)cap * 2 * hid)) ||
        (rc = dalloc(m, &m->pf_limbs, (size_t)(kmax / 32) * 3 * cap * 32)) ||
        (rc = dalloc(m, &m->pf_lsc, (size_t)(kmax / 32) * cap)))
        return rc;
    BREW_CUDA(cudaStreamSynchronize(s));
    m->pf_cap = cap;
    m->pf_ready = true;
    return BREW_OK;
}

// The prompt tokens tok_d[0 .. n) at positions 0 .. n-1 through every layer,
// in chunks of pf_cap tokens: the K / V cache rows of sequence 0 (the
// prompt's logits are not computed; the last layer stops after attention).
// Per layer, the op order of the reference's forward methods
// (model/*/...Transformer.java), each step over the chunk's rows.
int prefill_batched(brew_model_s* m, const int32_t* tok_d, int n, cudaStream_t s) {
    const brew_config& c = m->c;
    const int L = c.n_layers, dim = c.dim, hid = c.hidden_dim, hd = c.head_size;
    const int qw = c.n_heads * hd, kvd = c.n_kv_heads * hd, qkvw = qw + 2 * kvd;
    const bool gemma = arch_gemma(c.arch);
    const bool qknorm = arch_qknorm(c.arch);
    unsigned int* err = ctx().err_word;
    const int N[4] = {qkvw, dim, 2 * hid, dim}, K[4] = {dim, qw, dim, hid};
    int rc;
    for (int c0 = 0; c0 < n; c0 += m->pf_cap) {
        const int T = std::min(m->pf_cap, n - c0), Tp = (T + GEMM_TT - 1) / GEMM_TT * GEMM_TT;
        // y [Tp][N[f]] = W_f(layer l) x, x [T][ldx]
        auto gemm = [&](int f, int l, const float* x, int ldx, float* y) {
            int r = gemm_limbs_launch(x, ldx, T, Tp, K[f], m->pf_limbs, m->pf_lsc, s);
            if (!r)
                r = gemm_q8_launch(m->pf_wq[f] + (int64_t)l * N[f] * K[f], m->pf_wd[f] + (int64_t)l * N[f] * (K[f] / 32),
                                   m->pf_limbs, m->pf_lsc, N[f], K[f], Tp, T, y, err, s);
            return r;
        };
        if ((rc = prefill_embed_launch(c.type_embed, m->t[T_EMBED]->d, c.vocab_size, dim, tok_d + c0, T, gemma, m->pf_x,
                                       err, s)))
            return rc;
        for (int l = 0; l < L; ++l) {
            const bool global = arch_global_layer(c.arch, l);
            if ((rc = rmsnorm_launch(m->pf_x, dim, m->rms_att + (int64_t)l * dim, c.eps, dim, T, m->pf_xn, dim, s)) ||
                (rc = gemm(0, l, m->pf_xn, dim, m->pf_qkv)))
                return rc;
            if (m->q_bias &&
                ((rc = add_bias_launch(m->pf_qkv, qkvw, m->q_bias + (int64_t)l * qw, qw, T, s)) ||
                 (rc = add_bias_launch(m->pf_qkv + qw, qkvw, m->k_bias + (int64_t)l * kvd, kvd, T, s)) ||
                 (rc = add_bias_launch(m->pf_qkv + qw + kvd, qkvw, m->v_bias + (int64_t)l * kvd, kvd, T, s))))
                return rc;
            float* kcache = m->kc + (int64_t)l * c.seq_len * kvd;
            float* vcache = m->vc + (int64_t)l * c.seq_len * kvd;
            PfQkParams qk = {};
            qk.T = T;
            qk.pos0 = c0;
            qk.n_heads = c.n_heads;
            qk.n_kv = c.n_kv_heads;
            qk.hd = hd;
            qk.seq_len = c.seq_len;
            qk.table = (gemma && !global) ? 1 : 0;
            qk.interleaved = arch_interleaved(c.arch);
            qk.rope = arch_rope_layer(c.arch, l);
            qk.eps = c.eps;
            qk.qkv = m->pf_qkv;
            qk.ldq = qkvw;
            qk.qnorm_w = qknorm ? m->rms_q + (int64_t)l * hd : nullptr;
            qk.knorm_w = qknorm ? m->rms_k + (int64_t)l * hd : nullptr;
            qk.rope_cos = m->rope_cos;
            qk.rope_sin = m->rope_sin;
            qk.kcache = kcache;
            qk.vcache = vcache;
            if ((rc = prefill_qk_launch(qk, s))) return rc;
            PfAttnParams at = {};
            at.T = T;
            at.pos0 = c0;
            at.n_heads = c.n_heads;
            at.n_kv = c.n_kv_heads;
            at.hd = hd;
            at.window = (gemma && !global) ? c.sliding_window : 0;
            at.inv_scale = 1.0f / (float)std::sqrt((double)hd);   // AttentionEngine.java:18-19
            at.q = m->pf_qkv;
            at.ldq = qkvw;
            at.kcache = kcache;
            at.vcache = vcache;
            at.xb = m->pf_xb;
            at.ldxb = qw;
            if ((rc = prefill_attn_launch(at, s))) return rc;
            if (l == L - 1) break;   // the rest of the last layer feeds only the logits
            if ((rc = gemm(1, l, m->pf_xb, qw, m->pf_xb2)) ||
                (rc = residual_launch(m->pf_x, dim, m->pf_xb2, dim, gemma ? m->post_att + (int64_t)l * dim : nullptr,
                                      c.eps, dim, T, s)) ||
                (rc = rmsnorm_launch(m->pf_x, dim, m->rms_ffn + (int64_t)l * dim, c.eps, dim, T, m->pf_xn, dim, s)) ||
                (rc = gemm(2, l, m->pf_xn, dim, m->pf_h)) ||
                (rc = glu_launch(m->pf_h, m->pf_h, m->pf_h + hid, 2 * hid, hid, T, gemma, s)) ||
                (rc = gemm(3, l, m->pf_h, 2 * hid, m->pf_xb2)) ||
                (rc = residual_launch(m->pf_x, dim, m->pf_xb2, dim, gemma ? m->post_ffn + (int64_t)l * dim : nullptr,
                                      c.eps, dim, T, s)))
                return rc;
        }
    }
    return BREW_OK;
}

// GenericModelSession.prefill (runtime/ModelRunner.java:196-206) from a reset
// session: forward(prompt[i], i) for each prompt token (or the same cache
// state from the batched prefill).
int session_prefill(brew_model_s* m, const int32_t* prompt, int n_prompt, cudaStream_t s) {
    const brew_config& c = m->c;
    BREW_CHECK(n_prompt >= 0 && (prompt || n_prompt == 0), BREW_ERR_INVALID_ARG, "bad prompt");
    BREW_CHECK(n_prompt <= c.seq_len, BREW_ERR_CONTEXT_FULL, "The session has reached its context limit of %d tokens.",
               c.seq_len);
    for (int i = 0; i < n_prompt; ++i)
        BREW_CHECK(prompt[i] >= 0 && prompt[i] < c.vocab_size, BREW_ERR_INVALID_ARG, "prompt token %d out of range",
                   prompt[i]);
    if (m->prompt_cap < n_prompt + 1) {
        if (m->prompt_d) cudaFree(m->prompt_d);
        m->prompt_d = nullptr;
        BREW_CUDA(cudaMalloc(&m->prompt_d, (size_t)(n_prompt + 1) * sizeof(int32_t)));
        m->prompt_cap = n_prompt + 1;
    }
    // the prompt plus reset()'s pending token (BOS, ModelRunner.java:119)
    std::vector<int32_t> staged(prompt, prompt + n_prompt);
    staged.push_back(c.bos_token);
    BREW_CUDA(cudaMemcpyAsync(m->prompt_d, staged.data(), staged.size() * sizeof(int32_t), cudaMemcpyHostToDevice, s));
    BREW_CUDA(cudaStreamSynchronize(s));
    int rc;
    if (m->prefill_mode == BREW_PREFILL_BATCHED) {
        if ((rc = prefill_batched(m, m->prompt_d, n_prompt, s))) return rc;
    } else {
        for (int i = 0; i < n_prompt; ++i) {
            if ((rc = launch_step(m, m->prompt_d + i, i, nullptr, s))) return rc;
            if ((rc = launch_forward(m, 1, false, s))) return rc;
        }
    }
    m->sess_pos = n_prompt;
    m->sess_pending = n_prompt > 0 ? m->prompt_d + n_prompt - 1 : m->prompt_d + n_prompt;
    m->sess_generated = 0;
    return BREW_OK;
}

// The decode loop of GenericModelSession.generate (:141-152): forward the
// pending token at the current position, take the argmax as the next
// pending token.  Each step's id is recorded in gen_d on the device.
int session_decode(brew_model_s* m, int n_steps, cudaStream_t s) {
    const brew_config& c = m->c;
    BREW_CHECK(m->sess_pending, BREW_ERR_INVALID_ARG, "no session: call brew_session_prefill first");
    BREW_CHECK(n_steps >= 0, BREW_ERR_INVALID_ARG, "n_steps %d", n_steps);
    BREW_CHECK(m->sess_pos + n_steps <= c.seq_len, BREW_ERR_CONTEXT_FULL,
               "The session has reached its context limit of %d tokens.", c.seq_len);
    int rc;
    for (int k = 0; k < n_steps; ++k) {
        const int g = m->sess_generated;
        if ((rc = launch_step(m, m->sess_pending, m->sess_pos, g > 0 ? m->gen_d + g - 1 : nullptr, s))) return rc;
        if ((rc = launch_forward(m, 1, true, s))) return rc;
        m->sess_pending = m->am_out;
        m->sess_pos++;
        m->sess_generated++;
    }
    // record the last step's id
    if (n_steps > 0 && (rc = launch_step(m, m->am_out, m->sess_pos, m->gen_d + m->sess_generated - 1, s))) return rc;
    return BREW_OK;
}

// Sets up the persistent decode kernel when the shapes allow it.
int setup_decode(brew_model_s* m) {
    const brew_config& c = m->c;
    if (!decode_supported(c, 1) || getenv("BREW_NO_DECODE_KERNEL")) return BREW_OK;
    const int B = std::min(m->max_batch, DK_MAX_BATCH);
    const int hd = c.head_size, half = hd / 2;
    int rc;
    if ((rc = dalloc(m, &m->rope_cos, (size_t)2 * c.seq_len * half))) return rc;
    if ((rc = dalloc(m, &m->rope_sin, (size_t)2 * c.seq_len * half))) return rc;
    if ((rc = dalloc(m, &m->abort_flag, 1))) return rc;
    if ((rc = dalloc(m, &m->dk_seq, 1))) return rc;
    if ((rc = dalloc(m, &m->dk_done, 1))) return rc;
    BREW_CUDA(cudaHostAlloc(&m->h_res, 2 * sizeof(int32_t), cudaHostAllocMapped));
    BREW_CUDA(cudaHostGetDevicePointer((void**)&m->h_res_dev, m->h_res, 0));
    const float base0 = arch_rope_base(c.arch, c.rope_base, false);   // global / only table
    const float base1 = arch_rope_base(c.arch, c.rope_base, true);    // Gemma local layers
    const float scale = c.rope_scale > 0.0f ? c.rope_scale : 1.0f;
    if ((rc = rope_tables_launch(m->rope_cos, m->rope_sin, c.seq_len, hd, base0, base1, scale, ctx().stream))) return rc;
    DecodeParams& p = m->dp;
    p = DecodeParams{};
    p.arch = c.arch;
    p.dim = c.dim;
    p.hidden = c.hidden_dim;
    p.n_layers = c.n_layers;
    p.n_heads = c.n_heads;
    p.n_kv = c.n_kv_heads;
    p.hd = hd;
    p.vocab = c.vocab_size;
    p.seq_len = c.seq_len;
    p.window = c.sliding_window;
    p.batch = 1;
    p.type_layer = c.type_q;
    p.type_out = c.tied_embeddings ? c.type_embed : c.type_output;
    p.eps = c.eps;
    p.inv_scale = 1.0f / (float)std::sqrt((double)hd);   // AttentionEngine.java:18-19
    p.embed = m->t[T_EMBED]->d;
    p.type_embed = c.type_embed;
    p.rms_att = m->rms_att;
    p.rms_ffn = m->rms_ffn;
    p.rms_final = m->rms_final;
    p.post_att = m->post_att;
    p.post_ffn = m->post_ffn;
    p.rms_q = m->rms_q;
    p.rms_k = m->rms_k;
    p.q_bias = m->q_bias;
    p.k_bias = m->k_bias;
    p.v_bias = m->v_bias;
    p.kc = m->kc;
    p.vc = m->vc;
    p.cache_bstride = m->cache_bstride;
    p.rope_cos = m->rope_cos;
    p.rope_sin = m->rope_sin;
    {   // tagged activations: every layer's vectors, plus the classifier's input
        const int qw = c.n_heads * hd, qkvw = qw + 2 * c.n_kv_heads * hd;
        p.tg_ls = dk_tagged_layout(c.dim, qkvw, qw, c.hidden_dim, p.tg_off);
        m->dk_tg_words = (size_t)(c.n_layers + 1) * DK_MAX_BATCH * p.tg_ls;
        if ((rc = dalloc(m, &m->dk_tg, m->dk_tg_words))) return rc;
        p.tg = m->dk_tg;
    }
    p.logits = m->logits;
    p.nchunk = std::max(1, std::min(64, num_sms() / (B * c.n_kv_heads)));
    if ((rc = dalloc(m, &m->dk_part, (size_t)2 * DK_MAX_BATCH * c.n_heads * p.nchunk * (hd + 4)))) return rc;
    p.attn_part = m->dk_part;
    m->dk_nactr = (size_t)2 * c.n_layers * DK_MAX_BATCH * c.n_kv_heads;
    if ((rc = dalloc(m, &m->dk_actr, m->dk_nactr))) return rc;
    p.attn_ctr = m->dk_actr;
    p.am_key = m->am_key;
    p.am_out = m->am_out;
    p.tokens = m->tokens_d;
    p.pos = m->pos_d;
    p.seq = m->dk_seq;
    p.done = m->dk_done;
    p.abort = m->abort_flag;
    p.err = ctx().err_word;
    p.trace_slots = 1 + 5 * (5 * c.n_layers + 1) + 3 * DK_DETAIL;
    p.detail_l = -1;
    p.detail_ph = -1;
    if (const char* e = getenv("BREW_TRACE_DETAIL")) sscanf(e, "%d,%d", &p.detail_l, &p.detail_ph);
    m->trace_n = num_sms() * p.trace_slots;
    if ((rc = dalloc(m, &m->trace, (size_t)m->trace_n))) return rc;
    p.trace = getenv("BREW_TRACE") ? m->trace : nullptr;
    rc = decode_prepare(&p);
    if (rc == BREW_ERR_UNSUPPORTED) return BREW_OK;   // fall back to the kernel graph
    if (rc) return rc;
    // fragment-packed copies of the weights (the GGUF-layout tensors stay for
    // the kernel-graph path and for read-back)
    const int qw = c.n_heads * hd, kvd = c.n_kv_heads * hd;
    PackSpec spec[PK_NFAM] = {};
    spec[PK_QKV] = {{m->t[T_Q]->d, m->t[T_K]->d, m->t[T_V]->d}, {qw, kvd, kvd}, PK_ROWS, c.type_q, c.dim, c.n_layers};
    spec[PK_O] = {{m->t[T_O]->d, nullptr, nullptr}, {c.dim, 0, 0}, PK_ROWS, c.type_o, qw, c.n_layers};
    spec[PK_GU] = {{m->t[T_GATE]->d, m->t[T_UP]->d, nullptr}, {c.hidden_dim, 0, 0}, PK_GLU, c.type_gate, c.dim,
                   c.n_layers};
    spec[PK_DOWN] = {{m->t[T_DOWN]->d, nullptr, nullptr}, {c.dim, 0, 0}, PK_ROWS, c.type_down, c.hidden_dim,
                     c.n_layers};
    spec[PK_OUT] = {{m->t[T_OUTPUT]->d, nullptr, nullptr}, {c.vocab_size, 0, 0}, PK_ROWS, p.type_out, c.dim, 1};
    for (int f = 0; f < PK_NFAM; ++f) {
        p.pk_lb[f] = (int64_t)pk_layer_bytes(spec[f]);
        if ((rc = dalloc(m, &m->pk[f], (size_t)spec[f].layers * pk_layer_bytes(spec[f])))) return rc;
        if ((rc = pack_tiles_launch(m->pk[f], spec[f], ctx().stream))) return rc;
        p.pk[f] = m->pk[f];
    }
    m->use_decode = true;
    return BREW_OK;
}

// One forward of `B` sequences reading tokens_d / pos_d: the persistent
// decode kernel when available, else the captured kernel graph.
int launch_forward(brew_model_s* m, int B, bool with_classifier, cudaStream_t s);

// After a device-side error the decode kernel's counters may be left raised
// and its tagged words half written with an epoch the next launch reuses:
// clear them (and the abort flag) so the next step starts clean.
int after_step_check(brew_model_s* m, const char* where) {
    const int rc = check_device_error(where);
    if (rc && m->kq_ctr) {   // a K-quant matvec that stopped early may leave split counters raised
        cudaMemset(m->kq_ctr, 0, m->kq_nctr * sizeof(int));
        cudaDeviceSynchronize();
    }
    if (rc && m->tp_abort) {   // a peer-store gather that gave up
        cudaMemset(m->tp_abort, 0, sizeof(int));
        cudaDeviceSynchronize();
    }
    if (rc && m->use_decode) {
        cudaMemset(m->dk_done, 0, sizeof(int));
        cudaMemset(m->dk_actr, 0, m->dk_nactr * sizeof(int));
        cudaMemset(m->dk_tg, 0, m->dk_tg_words * sizeof(unsigned long long));
        cudaMemset(m->abort_flag, 0, sizeof(int));
        cudaMemset(m->am_key, 0, (size_t)m->max_batch * sizeof(unsigned long long));
        cudaMemset(m->am_ctr, 0, (size_t)m->max_batch * sizeof(int));
        cudaDeviceSynchronize();
    }
    return rc;
}

int model_finish_create(brew_model_s* m) {
    int rc = alloc_state(m);
    if (rc) return rc;
    if ((rc = setup_decode(m))) return rc;
    BREW_CUDA(cudaStreamSynchronize(ctx().stream));
    BREW_CUDA(cudaDeviceSynchronize());
    return BREW_OK;
}

void model_destroy(brew_model_s* m);

}  // namespace

void model_adopt_tensors(brew_model_s* m) {
    if (m->c.tied_embeddings) {   // the classifier becomes a view of the embedding
        brew_tensor v = new brew_tensor_s(*m->t[T_EMBED]);
        v->owned = false;
        m->t[T_OUTPUT] = v;
    }
    m->owns_tensors = true;
}

namespace {

void model_destroy(brew_model_s* m) {
    if (!m) return;
    for (auto& kv : m->graphs) cudaGraphExecDestroy(kv.second);
    if (m->tp_p2p) {   // the other ranks' arenas mapped here
        cudaDeviceSynchronize();
        for (int r = 0; r < TP_MAX_RANKS; ++r)
            if (m->tp_peers.p[r] && m->tp_peers.p[r] != m->tp_arena) cudaIpcCloseMemHandle(m->tp_peers.p[r]);
    }
    for (void* p : m->allocs) cudaFree(p);
    if (m->h_pin) cudaFreeHost(m->h_pin);
    if (m->h_res) cudaFreeHost(m->h_res);
    if (m->prompt_d) cudaFree(m->prompt_d);
    if (m->owns_tensors)
        for (int i = 0; i < T_COUNT; ++i)
            if (m->t[i]) brew_tensor_free(m->t[i]);
    delete m;
}

}  // namespace
}  // namespace brew

extern "C" {

int brew_model_create(const brew_config* cfg, const brew_model_weights* w, int32_t max_batch, brew_model* out) {
    BREW_CHECK(cfg && w && out, BREW_ERR_INVALID_ARG, "null argument");
    *out = nullptr;
    int rc = check_config(*cfg, max_batch);
    if (rc) return rc;
    if ((rc = ensure_init())) return rc;
    std::lock_guard<std::mutex> lk(api_mutex());
    const brew_config& c = *cfg;
    brew_tensor ts[T_COUNT] = {w->token_embd, c.tied_embeddings ? w->token_embd : w->output, w->wq, w->wk, w->wv, w->wo,
                               w->w_gate, w->w_up, w->w_down};
    for (int i = 0; i < T_COUNT; ++i) {
        BREW_CHECK(ts[i], BREW_ERR_INVALID_ARG, "weight tensor %d is null", i);
        int64_t rows, cols;
        int type, layers;
        matrix_shape(c, i, &rows, &cols, &type, &layers);
        BREW_CHECK(ts[i]->type == type, BREW_ERR_INVALID_ARG, "tensor %d has type %d, config says %d", i, ts[i]->type, type);
        BREW_CHECK(ts[i]->n == rows * cols * layers, BREW_ERR_INVALID_ARG, "tensor %d has %lld elements, expected %lld", i,
                   (long long)ts[i]->n, (long long)(rows * cols * layers));
    }
    const bool gemma = arch_gemma(c.arch), qk = arch_qknorm(c.arch), bias = c.arch == BREW_ARCH_QWEN2;
    BREW_CHECK(w->rms_att && w->rms_ffn && w->rms_final, BREW_ERR_INVALID_ARG, "norm weights missing");
    BREW_CHECK(!gemma || (w->post_att && w->post_ffn), BREW_ERR_INVALID_ARG, "Gemma post-norm weights missing");
    BREW_CHECK(!qk || (w->rms_q && w->rms_k), BREW_ERR_INVALID_ARG, "QK-norm weights missing");
    BREW_CHECK(!bias || (w->q_bias && w->k_bias && w->v_bias), BREW_ERR_INVALID_ARG, "QKV bias missing");
    brew_model_s* m = new brew_model_s();
    m->c = c;
    m->max_batch = max_batch;
    for (int i = 0; i < T_COUNT; ++i) m->t[i] = ts[i];
    const size_t L = c.n_layers, dim = c.dim, hs = c.head_size;
    const size_t qw = (size_t)c.n_heads * hs, kvd = (size_t)c.n_kv_heads * hs;
    if ((rc = upload_vec(m, &m->rms_att, w->rms_att, L * dim)) || (rc = upload_vec(m, &m->rms_ffn, w->rms_ffn, L * dim)) ||
        (rc = upload_vec(m, &m->rms_final, w->rms_final, dim)) ||
        (gemma && ((rc = upload_vec(m, &m->post_att, w->post_att, L * dim)) || (rc = upload_vec(m, &m->post_ffn, w->post_ffn, L * dim)))) ||
        (qk && ((rc = upload_vec(m, &m->rms_q, w->rms_q, L * hs)) || (rc = upload_vec(m, &m->rms_k, w->rms_k, L * hs)))) ||
        (bias && ((rc = upload_vec(m, &m->q_bias, w->q_bias, L * qw)) || (rc = upload_vec(m, &m->k_bias, w->k_bias, L * kvd)) ||
                  (rc = upload_vec(m, &m->v_bias, w->v_bias, L * kvd)))) ||
        (rc = model_finish_create(m))) {
        model_destroy(m);
        return rc;
    }
    *out = m;
    return BREW_OK;
}

int brew_model_synthesize(const brew_config* cfg, uint64_t seed, int32_t max_batch, brew_model* out) {
    BREW_CHECK(cfg && out, BREW_ERR_INVALID_ARG, "null argument");
    *out = nullptr;
    int rc = check_config(*cfg, max_batch);
    if (rc) return rc;
    if ((rc = ensure_init())) return rc;
    std::lock_guard<std::mutex> lk(api_mutex());
    const brew_config& c = *cfg;
    brew_model_s* m = new brew_model_s();
    m->c = c;
    m->max_batch = max_batch;
    m->owns_tensors = true;
    cudaStream_t s = ctx().stream;
    for (int i = 0; i < T_COUNT && !rc; ++i) {
        if (i == T_OUTPUT && c.tied_embeddings) continue;
        int64_t rows, cols;
        int type, layers;
        matrix_shape(c, i, &rows, &cols, &type, &layers);
        rc = brew_tensor_alloc(type, rows * cols * layers, &m->t[i]);
        if (rc) break;
        const int64_t per = brew_type_bytes(type, rows * cols);
        for (int l = 0; l < layers && !rc; ++l)
            rc = synth_launch(type, seed, tensor_id(i, l), rows * cols, 0.02f, m->t[i]->d + per * l, s);
    }
    if (!rc && c.tied_embeddings) {
        brew_tensor v = new brew_tensor_s(*m->t[T_EMBED]);
        v->owned = false;
        m->t[T_OUTPUT] = v;
    }
    const size_t L = c.n_layers, dim = c.dim, hs = c.head_size;
    const size_t qw = (size_t)c.n_heads * hs, kvd = (size_t)c.n_kv_heads * hs;
    if (!rc) rc = fill_vec(m, &m->rms_att, L * dim, 1.0f);
    if (!rc) rc = fill_vec(m, &m->rms_ffn, L * dim, 1.0f);
    if (!rc) rc = fill_vec(m, &m->rms_final, dim, 1.0f);
    if (!rc && arch_gemma(c.arch)) {
        rc = fill_vec(m, &m->post_att, L * dim, 1.0f);
        if (!rc) rc = fill_vec(m, &m->post_ffn, L * dim, 1.0f);
    }
    if (!rc && arch_qknorm(c.arch)) {
        rc = fill_vec(m, &m->rms_q, L * hs, 1.0f);
        if (!rc) rc = fill_vec(m, &m->rms_k, L * hs, 1.0f);
    }
    if (!rc && c.arch == BREW_ARCH_QWEN2) {
        rc = dalloc(m, &m->q_bias, L * qw);
        if (!rc) rc = dalloc(m, &m->k_bias, L * kvd);
        if (!rc) rc = dalloc(m, &m->v_bias, L * kvd);
        for (size_t l = 0; l < L && !rc; ++l) {
            rc = synth_f32_launch(seed, tensor_id(9, (int)l), qw, 0.02f, m->q_bias + l * qw, s);
            if (!rc) rc = synth_f32_launch(seed, tensor_id(10, (int)l), kvd, 0.02f, m->k_bias + l * kvd, s);
            if (!rc) rc = synth_f32_launch(seed, tensor_id(11, (int)l), kvd, 0.02f, m->v_bias + l * kvd, s);
        }
    }
    if (!rc) rc = model_finish_create(m);
    if (rc) {
        model_destroy(m);
        return rc;
    }
    *out = m;
    return BREW_OK;
}

int brew_model_config(brew_model m, brew_config* out) {
    BREW_CHECK(m && out, BREW_ERR_INVALID_ARG, "null argument");
    *out = m->c;
    return BREW_OK;
}

int brew_model_free(brew_model m) {
    if (!m) return BREW_OK;
    std::lock_guard<std::mutex> lk(api_mutex());
    cudaDeviceSynchronize();
    model_destroy(m);
    return BREW_OK;
}

int brew_model_set_prefill(brew_model m, int32_t mode) {
    BREW_CHECK(m, BREW_ERR_INVALID_ARG, "null argument");
    BREW_CHECK(mode == BREW_PREFILL_TOKENS || mode == BREW_PREFILL_BATCHED, BREW_ERR_INVALID_ARG, "prefill mode %d",
               mode);
    std::lock_guard<std::mutex> lk(api_mutex());
    int rc = ensure_init();
    if (rc) return rc;
    if (mode == BREW_PREFILL_BATCHED) {
        std::string why;
        BREW_CHECK(prefill_supported(m->c, &why), BREW_ERR_UNSUPPORTED, "%s", why.c_str());
        BREW_CHECK(!m->comm, BREW_ERR_UNSUPPORTED, "the batched prefill runs on one GPU (the model is sharded)");
        if ((rc = setup_prefill(m))) return rc;
    }
    m->prefill_mode = mode;
    return BREW_OK;
}

int brew_model_set_tp(brew_model m, brew_comm comm) {
    BREW_CHECK(m && comm, BREW_ERR_INVALID_ARG, "null argument");
    BREW_CHECK(!m->comm, BREW_ERR_INVALID_ARG, "the model is already sharded");
    const brew_config& c = m->c;
    const int P = comm->nranks;
    const int qw = c.n_heads * c.head_size, kvd = c.n_kv_heads * c.head_size;
    const int rows[] = {qw, kvd, c.dim, c.hidden_dim, c.vocab_size};
    for (int n : rows)
        BREW_CHECK(n % P == 0, BREW_ERR_UNSUPPORTED, "%d rows do not split over %d ranks", n, P);
    std::lock_guard<std::mutex> lk(api_mutex());
    int rc = ensure_init();
    if (rc) return rc;
    BREW_CHECK(comm->device == ctx().device, BREW_ERR_INVALID_ARG, "communicator on device %d, model on %d",
               comm->device, ctx().device);
    BREW_CUDA(cudaDeviceSynchronize());
    // the forward changes: drop captured graphs and the one-GPU decode kernel
    for (auto& kv : m->graphs) cudaGraphExecDestroy(kv.second);
    m->graphs.clear();
    m->graph_kernels.clear();
    m->use_decode = false;
    m->prefill_mode = BREW_PREFILL_TOKENS;
    if ((rc = alloc_unfused(m))) return rc;
    const int B = m->max_batch;
    const int slice = std::max(std::max((qw + 2 * kvd) / P, c.dim / P), std::max(c.hidden_dim / P, c.vocab_size / P));
    if ((rc = dalloc(m, &m->tp_send, (size_t)B * slice)) || (rc = dalloc(m, &m->tp_recv, (size_t)P * B * slice)) ||
        (rc = dalloc(m, &m->tp_g, (size_t)B * (std::max(c.hidden_dim, qw) / P))) ||   // also a sharded attention's output
        (rc = dalloc(m, &m->tp_u, (size_t)B * (c.hidden_dim / P))) || (rc = dalloc(m, &m->tp_keys, (size_t)B)) ||
        (rc = dalloc(m, &m->tp_keys_all, (size_t)P * B)))
        return rc;
    // this rank's rows of the K-quant q|k|v and gate|up families as families
    // of their own (one launch each; the split of K stays the one-GPU one)
    const int R = comm->rank;
    if (P > 1 && m->kqp_qkv) {
        const int qs = qw / P, ks = kvd / P, sl = qs + 2 * ks;
        const size_t per = kx_bytes(c.type_q, sl, c.dim);
        const int64_t rb = row_bytes_of(c.type_q, c.dim);
        if ((rc = dalloc(m, &m->kqp_qkv_tp, per * c.n_layers))) return rc;
        for (int l = 0; l < c.n_layers && !rc; ++l) {
            uint8_t* base = m->kqp_qkv_tp + per * l;
            rc = kx_pack_launch(c.type_q, layer_ptr(m->t[T_Q], l, qw, c.dim) + (int64_t)R * qs * rb, qs, c.dim, base, sl,
                                0, ctx().stream);
            if (!rc)
                rc = kx_pack_launch(c.type_q, layer_ptr(m->t[T_K], l, kvd, c.dim) + (int64_t)R * ks * rb, ks, c.dim,
                                    base, sl, qs, ctx().stream);
            if (!rc)
                rc = kx_pack_launch(c.type_q, layer_ptr(m->t[T_V], l, kvd, c.dim) + (int64_t)R * ks * rb, ks, c.dim,
                                    base, sl, qs + ks, ctx().stream);
        }
        if (rc) return rc;
        if (m->q_bias) {
            BREW_CUDA(cudaDeviceSynchronize());
            if ((rc = dalloc(m, &m->qkv_bias_tp, (size_t)sl * c.n_layers))) return rc;
            for (int l = 0; l < c.n_layers; ++l) {
                float* fb = m->qkv_bias_tp + (size_t)sl * l;
                BREW_CUDA(cudaMemcpy(fb, m->q_bias + (size_t)qw * l + (size_t)R * qs, qs * sizeof(float),
                                     cudaMemcpyDeviceToDevice));
                BREW_CUDA(cudaMemcpy(fb + qs, m->k_bias + (size_t)kvd * l + (size_t)R * ks, ks * sizeof(float),
                                     cudaMemcpyDeviceToDevice));
                BREW_CUDA(cudaMemcpy(fb + qs + ks, m->v_bias + (size_t)kvd * l + (size_t)R * ks, ks * sizeof(float),
                                     cudaMemcpyDeviceToDevice));
            }
        }
    }
    if (P > 1 && m->kqp_gu) {
        const int hs = c.hidden_dim / P;
        const size_t per = kx_bytes(c.type_gate, 2 * hs, c.dim);
        const int64_t rb = row_bytes_of(c.type_gate, c.dim);
        if ((rc = dalloc(m, &m->kqp_gu_tp, per * c.n_layers)) || (rc = dalloc(m, &m->tp_gu, (size_t)B * 2 * hs)))
            return rc;
        for (int l = 0; l < c.n_layers && !rc; ++l) {
            uint8_t* base = m->kqp_gu_tp + per * l;
            rc = kx_pack_launch(c.type_gate, layer_ptr(m->t[T_GATE], l, c.hidden_dim, c.dim) + (int64_t)R * hs * rb, hs,
                                c.dim, base, 2 * hs, 0, ctx().stream);
            if (!rc)
                rc = kx_pack_launch(c.type_gate, layer_ptr(m->t[T_UP], l, c.hidden_dim, c.dim) + (int64_t)R * hs * rb,
                                    hs, c.dim, base, 2 * hs, hs, ctx().stream);
        }
        if (rc) return rc;
    }
    // split-K scratch for the sharded launches' own splits
    m->tp_exact = getenv("BREW_TP_EXACT") != nullptr;
    if (P > 1 && !m->tp_exact && m->kq_part) {
        const int hs = c.hidden_dim / P, sl = (qw + 2 * kvd) / P;
        const int64_t shapes[5][2] = {{sl, c.dim}, {c.dim / P, qw}, {2 * hs, c.dim}, {c.dim / P, c.hidden_dim},
                                      {c.vocab_size / P, c.dim}};
        size_t need = 0;
        for (const auto& sh : shapes) {
            const int sp = kq_splits(sh[1], sh[0]);
            if (sp > 1) need = std::max(need, (size_t)sp * KX_MAX_VECTORS * (size_t)((sh[0] + KX_TM - 1) / KX_TM * KX_TM));
        }
        if (need && (rc = dalloc(m, &m->kq_part, need))) return rc;
    }
    // peer-store gathers (tp.cuh): one tagged slot per gather site, every
    // rank's arena mapped into this process through CUDA IPC, the handles
    // exchanged over the communicator.  BREW_TP_NCCL=1 keeps the NCCL
    // all-gathers.
    if (P > 1 && P <= TP_MAX_RANKS && !getenv("BREW_TP_NCCL")) {
        const int V = c.vocab_size, L = c.n_layers;
        BREW_CHECK(4 * L + 1 <= 256, BREW_ERR_UNSUPPORTED, "peer gathers: %d layers (at most 63)", L);
        m->tp_layer_words = (size_t)B * (m->qkvw + 2 * (size_t)c.dim + c.hidden_dim);
        const size_t words = (size_t)L * m->tp_layer_words + (size_t)B * V;
        if ((rc = dalloc(m, &m->tp_arena, words)) || (rc = dalloc(m, &m->tp_step, 1)) ||
            (rc = dalloc(m, &m->tp_abort, 1)))
            return rc;
        cudaIpcMemHandle_t own;
        BREW_CUDA(cudaIpcGetMemHandle(&own, m->tp_arena));
        static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
        float* hbuf = nullptr;   // [P][16] floats: the handles' bytes
        if ((rc = dalloc(m, &hbuf, (size_t)(P + 1) * 16))) return rc;
        BREW_CUDA(cudaMemcpy(hbuf + (size_t)P * 16, &own, 64, cudaMemcpyHostToDevice));
        if ((rc = tp_allgather(comm, hbuf + (size_t)P * 16, hbuf, 16, ctx().stream))) return rc;
        BREW_CUDA(cudaStreamSynchronize(ctx().stream));
        std::vector<cudaIpcMemHandle_t> all(P);
        BREW_CUDA(cudaMemcpy(all.data(), hbuf, (size_t)P * 64, cudaMemcpyDeviceToHost));
        for (int r = 0; r < P; ++r) {
            if (r == R) {
                m->tp_peers.p[r] = m->tp_arena;
                continue;
            }
            void* ptr = nullptr;
            BREW_CUDA(cudaIpcOpenMemHandle(&ptr, all[r], cudaIpcMemLazyEnablePeerAccess));
            m->tp_peers.p[r] = static_cast<unsigned long long*>(ptr);
        }
        m->tp_p2p = true;
    }
    BREW_CUDA(cudaStreamSynchronize(ctx().stream));
    m->comm = comm;
    return BREW_OK;
}

int brew_model_tensor(brew_model m, int which, brew_tensor* out) {
    BREW_CHECK(m && out && which >= 0 && which < T_COUNT, BREW_ERR_INVALID_ARG, "bad argument");
    *out = m->t[which];
    return BREW_OK;
}

int brew_model_trace(brew_model m, int64_t* ns, int32_t max_n, int32_t* n) {
    BREW_CHECK(m && ns && n, BREW_ERR_INVALID_ARG, "null argument");
    *n = 0;
    if (!m->use_decode || !m->dp.trace) return BREW_OK;
    std::lock_guard<std::mutex> lk(api_mutex());
    const int k = std::min(max_n, m->trace_n);
    BREW_CUDA(cudaStreamSynchronize(ctx().stream));
    BREW_CUDA(cudaMemcpy(ns, m->trace, (size_t)k * sizeof(int64_t), cudaMemcpyDeviceToHost));
    *n = k;
    return BREW_OK;
}

int brew_model_set_trace(brew_model m, int32_t on) {
    BREW_CHECK(m, BREW_ERR_INVALID_ARG, "null model");
    if (m->use_decode) m->dp.trace = on ? m->trace : nullptr;
    return BREW_OK;
}

int brew_model_reset(brew_model m) {
    BREW_CHECK(m, BREW_ERR_INVALID_ARG, "null model");
    std::lock_guard<std::mutex> lk(api_mutex());
    BREW_CUDA(cudaMemsetAsync(m->kc, 0, (size_t)m->max_batch * m->cache_bstride * sizeof(float), ctx().stream));
    BREW_CUDA(cudaMemsetAsync(m->vc, 0, (size_t)m->max_batch * m->cache_bstride * sizeof(float), ctx().stream));
    BREW_CUDA(cudaStreamSynchronize(ctx().stream));
    return BREW_OK;
}

int brew_model_forward_dev(brew_model m, const int32_t* tokens_dev, const int32_t* pos_dev, int32_t batch,
                           float* logits_dev, int32_t* argmax_dev, void* stream) {
    BREW_CHECK(m && tokens_dev && pos_dev, BREW_ERR_INVALID_ARG, "null argument");
    BREW_CHECK(batch >= 1 && batch <= m->max_batch, BREW_ERR_INVALID_ARG, "batch %d (max %d)", batch, m->max_batch);
    int rc = ensure_init();
    if (rc) return rc;
    std::lock_guard<std::mutex> lk(api_mutex());
    cudaStream_t s = ctx().stream;
    cudaStream_t us = static_cast<cudaStream_t>(stream);
    cudaEvent_t ev;
    if (us) {
        BREW_CUDA(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
        BREW_CUDA(cudaEventRecord(ev, us));
        BREW_CUDA(cudaStreamWaitEvent(s, ev));
    }
    BREW_CUDA(cudaMemcpyAsync(m->tokens_d, tokens_dev, batch * sizeof(int32_t), cudaMemcpyDeviceToDevice, s));
    BREW_CUDA(cudaMemcpyAsync(m->pos_d, pos_dev, batch * sizeof(int32_t), cudaMemcpyDeviceToDevice, s));
    if ((rc = launch_forward(m, batch, true, s))) return rc;
    if (logits_dev)
        BREW_CUDA(cudaMemcpyAsync(logits_dev, m->logits, (size_t)batch * m->c.vocab_size * sizeof(float),
                                  cudaMemcpyDeviceToDevice, s));
    if (argmax_dev) BREW_CUDA(cudaMemcpyAsync(argmax_dev, m->am_out, batch * sizeof(int32_t), cudaMemcpyDeviceToDevice, s));
    if (us) {
        BREW_CUDA(cudaEventRecord(ev, s));
        BREW_CUDA(cudaStreamWaitEvent(us, ev));
        cudaEventDestroy(ev);
    }
    return BREW_OK;
}

int brew_model_forward(brew_model m, const int32_t* tokens, const int32_t* pos, int32_t batch, float* logits,
                       int32_t* argmax) {
    BREW_CHECK(m && tokens && pos, BREW_ERR_INVALID_ARG, "null argument");
    BREW_CHECK(batch >= 1 && batch <= m->max_batch, BREW_ERR_INVALID_ARG, "batch %d (max %d)", batch, m->max_batch);
    for (int b = 0; b < batch; ++b) {
        BREW_CHECK(tokens[b] >= 0 && tokens[b] < m->c.vocab_size, BREW_ERR_INVALID_ARG, "token %d out of range", tokens[b]);
        BREW_CHECK(pos[b] >= 0, BREW_ERR_INVALID_ARG, "position %d", pos[b]);
        BREW_CHECK(pos[b] < m->c.seq_len, BREW_ERR_CONTEXT_FULL,
                   "The session has reached its context limit of %d tokens.", m->c.seq_len);
    }
    int rc = ensure_init();
    if (rc) return rc;
    std::lock_guard<std::mutex> lk(api_mutex());
    cudaStream_t s = ctx().stream;
    if (m->use_decode && batch == 1 && !logits && m->h_res) {
        // one sequence, argmax only: the token and position travel as launch
        // parameters and the kernel's last CTA writes the id and the error
        // word into mapped pinned memory, so the call is one launch and one
        // synchronize (no copy either way)
        DecodeParams dp = m->dp;
        dp.use_imm = 1;
        dp.tok_imm = tokens[0];
        dp.pos_imm = pos[0];
        dp.host_out = m->h_res_dev;
        volatile int32_t* hr = m->h_res;
        hr[0] = -1;
        hr[1] = -1;   // stays -1 when the kernel stops early
        if ((rc = decode_launch(dp, s))) return rc;
        BREW_CUDA(cudaStreamSynchronize(s));
        const int32_t id = hr[0], ew = hr[1];
        if (argmax) argmax[0] = id;
        if (ew == 0) return BREW_OK;
        return after_step_check(m, "brew_model_forward");
    }
    // pinned staging: [tokens | positions] as laid out on the device (one
    // upload), then the argmax ids and the device error word (read back
    // with the ids: the error path runs only when it is set)
    const int mb = m->max_batch;
    int32_t* hp = m->h_pin;
    memcpy(hp, tokens, batch * sizeof(int32_t));
    memcpy(hp + mb, pos, batch * sizeof(int32_t));
    BREW_CUDA(cudaMemcpyAsync(m->tokens_d, hp, (size_t)(mb + batch) * sizeof(int32_t), cudaMemcpyHostToDevice, s));
    if ((rc = launch_forward(m, batch, true, s))) return rc;
    if (logits)
        BREW_CUDA(cudaMemcpyAsync(logits, m->logits, (size_t)batch * m->c.vocab_size * sizeof(float), cudaMemcpyDeviceToHost, s));
    if (argmax) BREW_CUDA(cudaMemcpyAsync(hp + 2 * mb, m->am_out, batch * sizeof(int32_t), cudaMemcpyDeviceToHost, s));
    int32_t* herr = hp + 3 * mb;
    *herr = 0;
    if (ctx().err_word) BREW_CUDA(cudaMemcpyAsync(herr, ctx().err_word, sizeof(int32_t), cudaMemcpyDeviceToHost, s));
    BREW_CUDA(cudaStreamSynchronize(s));
    if (argmax) memcpy(argmax, hp + 2 * mb, batch * sizeof(int32_t));
    if (*herr == 0) return BREW_OK;
    return after_step_check(m, "brew_model_forward");
}

int brew_session_prefill(brew_model m, const int32_t* prompt, int32_t n_prompt, void* stream) {
    BREW_CHECK(m, BREW_ERR_INVALID_ARG, "null model");
    int rc = ensure_init();
    if (rc) return rc;
    std::lock_guard<std::mutex> lk(api_mutex());
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : ctx().stream;
    return session_prefill(m, prompt, n_prompt, s);
}

int brew_session_decode(brew_model m, int32_t n_steps, int32_t* out, void* stream) {
    BREW_CHECK(m, BREW_ERR_INVALID_ARG, "null model");
    int rc = ensure_init();
    if (rc) return rc;
    std::lock_guard<std::mutex> lk(api_mutex());
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : ctx().stream;
    const int first = m->sess_generated;
    if ((rc = session_decode(m, n_steps, s))) return rc;
    if (!out) return BREW_OK;
    if (n_steps > 0)
        BREW_CUDA(cudaMemcpyAsync(out, m->gen_d + first, (size_t)n_steps * sizeof(int32_t), cudaMemcpyDeviceToHost, s));
    BREW_CUDA(cudaStreamSynchronize(s));
    return after_step_check(m, "brew_session_decode");
}

int brew_model_step_kernels(brew_model m, int32_t batch, int32_t* n) {
    BREW_CHECK(m && n, BREW_ERR_INVALID_ARG, "null argument");
    BREW_CHECK(batch >= 1 && batch <= m->max_batch, BREW_ERR_INVALID_ARG, "batch %d", batch);
    int rc = ensure_init();
    if (rc) return rc;
    std::lock_guard<std::mutex> lk(api_mutex());
    if (m->use_decode && batch == 1) {
        *n = 1;
        return BREW_OK;
    }
    cudaGraphExec_t g;
    if ((rc = get_graph(m, batch, true, &g))) return rc;
    *n = m->graph_kernels[batch * 2 + 1];
    return BREW_OK;
}

int brew_session_generate(brew_model m, const int32_t* prompt, int32_t n_prompt, int32_t max_new, int32_t* out,
                          int32_t* n_out) {
    BREW_CHECK(m && n_out && (prompt || n_prompt == 0), BREW_ERR_INVALID_ARG, "null argument");
    BREW_CHECK(n_prompt >= 0, BREW_ERR_INVALID_ARG, "n_prompt %d", n_prompt);
    const brew_config& c = m->c;
    // ensureContextAvailable (runtime/ModelRunner.java:208-216)
    BREW_CHECK(n_prompt <= c.seq_len, BREW_ERR_CONTEXT_FULL,
               "The session has reached its context limit of %d tokens.", c.seq_len);
    const int remaining = c.seq_len - n_prompt;              // :132-135
    const int limit = max_new <= 0 ? remaining : std::min(max_new, remaining);
    BREW_CHECK(limit == 0 || out, BREW_ERR_INVALID_ARG, "out is null");
    int rc = ensure_init();
    if (rc) return rc;
    std::lock_guard<std::mutex> lk(api_mutex());
    cudaStream_t s = ctx().stream;
    if ((rc = session_prefill(m, prompt, n_prompt, s))) return rc;
    if ((rc = session_decode(m, limit, s))) return rc;
    std::vector<int32_t> gen(limit);
    if (limit > 0) BREW_CUDA(cudaMemcpyAsync(gen.data(), m->gen_d, limit * sizeof(int32_t), cudaMemcpyDeviceToHost, s));
    BREW_CUDA(cudaStreamSynchronize(s));
    rc = after_step_check(m, "brew_session_generate");
    if (rc) return rc;
    // stop at the first EOS, inclusive (:149-151)
    int n = 0;
    for (; n < limit; ++n) {
        out[n] = gen[n];
        if (gen[n] == c.eos_token) {
            ++n;
            break;
        }
    }
    *n_out = n;
    return BREW_OK;
}

}  // extern "C"
