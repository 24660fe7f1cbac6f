// gguf.cu — GGUF checkpoint reading and loading straight into HBM (host code).
//
// Replaces the reference's load path:
//   gguf/Reader.java:25-58,60-125     header, metadata key/values, tensor infos,
//                                      aligned data offset
//   gguf/GgufConfigParser.java:9-59   the config fields the forward pass reads
//   model/*/...CheckpointLoader.java   per-architecture head size (Qwen3 128,
//                                      Gemma2 / Gemma3 256, else dim / heads)
//   gguf/GgufWeightsLoader.java:24-165,228-278
//                                      tensors by name, layers concatenated,
//                                      F32 / F16 norm and bias vectors, the
//                                      classifier tied to the embedding when
//                                      the file has no output.weight
// The file is memory-mapped; each packed weight tensor goes to the device
// unchanged through two pinned staging buffers (one is filled from the mapping
// while the other's copy engine transfer runs).  Unlike readQ8Block, the
// tensor type is checked: Q8_0, Q4_0, Q4_K and Q6_K matrices are accepted.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cstring>
#include <string>
#include <unordered_map>
#include <vector>

#include "brew_internal.cuh"

struct brew_gguf_s {
    int fd = -1;
    const uint8_t* base = nullptr;
    size_t size = 0;
    uint32_t version = 0;
    uint64_t data_offset = 0;
    struct Value {
        int type = -1;          // GGUF value type (0..12)
        int64_t i = 0;          // integer types and bool
        double f = 0.0;         // FLOAT32 / FLOAT64
        std::string s;          // STRING
        int elem_type = -1;     // ARRAY: element type and count
        int64_t count = 0;
    };
    std::unordered_map<std::string, Value> meta;
    struct Tensor {
        std::string name;
        std::vector<int64_t> dims;
        int type = 0;
        uint64_t offset = 0;    // relative to data_offset
        int64_t n = 0;          // elements
        int64_t bytes = 0;
    };
    std::vector<Tensor> tensors;
    std::unordered_map<std::string, size_t> by_name;
};

namespace brew {
namespace {

// Bounds-checked little-endian reader over the mapped file.
struct Cursor {
    const uint8_t* p;
    size_t size, off = 0;
    bool ok = true;
    bool take(void* dst, size_t n) {
        if (!ok || n > size - off) {
            ok = false;
            return false;
        }
        memcpy(dst, p + off, n);
        off += n;
        return true;
    }
    bool skip(size_t n) {
        if (!ok || n > size - off) return ok = false;
        off += n;
        return true;
    }
    template <typename T>
    T get() {
        T v{};
        take(&v, sizeof(T));
        return v;
    }
    bool str(std::string* s) {
        const int64_t len = get<int64_t>();
        if (!ok || len < 0 || (uint64_t)len > size - off) return ok = false;   // Reader.java:128-136
        if (s) s->assign(reinterpret_cast<const char*>(p + off), (size_t)len);
        off += (size_t)len;
        return true;
    }
};

int scalar_bytes(int type) {
    switch (type) {
        case 0: case 1: case 7: return 1;     // UINT8, INT8, BOOL
        case 2: case 3: return 2;             // UINT16, INT16
        case 4: case 5: case 6: return 4;     // UINT32, INT32, FLOAT32
        case 10: case 11: case 12: return 8;  // UINT64, INT64, FLOAT64
        default: return 0;
    }
}

// Reader.readValue (gguf/Reader.java:83-125); arrays keep their element type
// and count (the loader needs only the token list's length).
bool read_value(Cursor& c, int type, brew_gguf_s::Value* v) {
    v->type = type;
    switch (type) {
        case 0: v->i = c.get<uint8_t>(); break;
        case 1: v->i = c.get<int8_t>(); break;
        case 2: v->i = c.get<uint16_t>(); break;
        case 3: v->i = c.get<int16_t>(); break;
        case 4: v->i = c.get<uint32_t>(); break;
        case 5: v->i = c.get<int32_t>(); break;
        case 6: v->f = c.get<float>(); break;
        case 7: v->i = c.get<uint8_t>() != 0; break;
        case 8: c.str(&v->s); break;
        case 9: {
            v->elem_type = c.get<int32_t>();
            v->count = c.get<int64_t>();
            if (!c.ok || v->count < 0 || v->count > 0x7fffffffLL) return c.ok = false;   // Reader.java:112-114
            const int eb = scalar_bytes(v->elem_type);
            if (eb) {
                c.skip((size_t)v->count * eb);
            } else if (v->elem_type == 8) {
                for (int64_t k = 0; k < v->count && c.ok; ++k) c.str(nullptr);
            } else if (v->elem_type == 9) {
                brew_gguf_s::Value inner;
                for (int64_t k = 0; k < v->count && c.ok; ++k) read_value(c, 9, &inner);
            } else {
                return c.ok = false;
            }
            break;
        }
        case 10: v->i = (int64_t)c.get<uint64_t>(); break;
        case 11: v->i = c.get<int64_t>(); break;
        case 12: v->f = c.get<double>(); break;
        default: return c.ok = false;   // "Unknown GGUF metadata type"
    }
    return c.ok;
}

int gguf_parse(brew_gguf_s* g) {
    Cursor c{g->base, g->size};
    const uint32_t magic = c.get<uint32_t>();
    BREW_CHECK(c.ok && magic == 0x46554747u, BREW_ERR_IO, "Not a GGUF file (bad magic number): 0x%x", magic);
    g->version = c.get<uint32_t>();
    BREW_CHECK(g->version == 2 || g->version == 3, BREW_ERR_IO,
               "Unsupported GGUF version: %u, expected 2 or 3 (Little Endian)", g->version);
    const int64_t n_tensors = c.get<int64_t>(), n_meta = c.get<int64_t>();
    BREW_CHECK(c.ok && n_tensors >= 0 && n_meta >= 0, BREW_ERR_IO, "GGUF header truncated");
    for (int64_t i = 0; i < n_meta; ++i) {
        std::string key;
        c.str(&key);
        const int type = c.get<int32_t>();
        brew_gguf_s::Value v;
        BREW_CHECK(read_value(c, type, &v), BREW_ERR_IO, "GGUF metadata entry %lld (%s): bad value or EOF",
                   (long long)i, key.c_str());
        g->meta[key] = v;
    }
    for (int64_t i = 0; i < n_tensors; ++i) {   // Reader.readTensorInfo (:67-81)
        brew_gguf_s::Tensor t;
        c.str(&t.name);
        const int32_t nd = c.get<int32_t>();
        BREW_CHECK(c.ok && nd >= 0 && nd <= 8, BREW_ERR_IO, "Unreasonable tensor n_dims=%d for tensor: %s", nd,
                   t.name.c_str());
        t.n = 1;
        for (int d = 0; d < nd; ++d) {
            const int64_t v = c.get<int64_t>();
            BREW_CHECK(c.ok && v > 0 && v <= 0x7fffffffLL, BREW_ERR_IO, "Bad tensor dim in %s: %lld", t.name.c_str(),
                       (long long)v);
            t.dims.push_back(v);
            t.n *= v;
        }
        t.type = c.get<int32_t>();
        t.offset = c.get<uint64_t>();
        BREW_CHECK(c.ok, BREW_ERR_IO, "GGUF tensor info %lld truncated", (long long)i);
        TypeInfo ti;
        t.bytes = (type_info(t.type, &ti) && t.n % ti.block_elems == 0) ? t.n / ti.block_elems * ti.block_bytes : -1;
        g->by_name[t.name] = g->tensors.size();
        g->tensors.push_back(t);
    }
    int64_t align = 32;   // general.alignment, default 32 (Reader.java:51-55)
    auto it = g->meta.find("general.alignment");
    if (it != g->meta.end() && it->second.type != 8 && it->second.type != 9) align = it->second.i;
    BREW_CHECK(align > 0 && (align & (align - 1)) == 0, BREW_ERR_IO,
               "Invalid general.alignment: %lld (must be power of two)", (long long)align);
    g->data_offset = (c.off + (uint64_t)align - 1) & ~((uint64_t)align - 1);
    for (const auto& t : g->tensors)
        if (t.bytes >= 0)
            BREW_CHECK(g->data_offset + t.offset + (uint64_t)t.bytes <= g->size, BREW_ERR_IO,
                       "tensor %s runs past the end of the file", t.name.c_str());
    return BREW_OK;
}

const brew_gguf_s::Value* meta_get(const brew_gguf_s* g, const std::string& key) {
    auto it = g->meta.find(key);
    return it == g->meta.end() ? nullptr : &it->second;
}

// writeConfigInt / writeConfigFloat (GgufConfigParser.java:65-90): any
// numeric value type; absent keys leave the default.
bool meta_num(const brew_gguf_s* g, const std::string& key, double* out) {
    const auto* v = meta_get(g, key);
    if (!v || v->type == 8 || v->type == 9) return false;
    *out = (v->type == 6 || v->type == 12) ? v->f : (double)v->i;
    return true;
}

int arch_from_name(const std::string& a, int* id) {
    // model/ModelRunnerFactory.java:29-47
    if (a == "llama" || a == "llama2") *id = BREW_ARCH_LLAMA;
    else if (a == "qwen2") *id = BREW_ARCH_QWEN2;
    else if (a == "qwen3") *id = BREW_ARCH_QWEN3;
    else if (a == "gemma3") *id = BREW_ARCH_GEMMA3;
    else if (a == "gemma2") *id = BREW_ARCH_GEMMA2;
    else if (a == "smollm3") *id = BREW_ARCH_SMOLLM3;
    else return set_error(BREW_ERR_UNSUPPORTED, "Unsupported architecture: %s", a.c_str());
    return BREW_OK;
}

const brew_gguf_s::Tensor* tensor_get(const brew_gguf_s* g, const std::string& name) {
    auto it = g->by_name.find(name);
    return it == g->by_name.end() ? nullptr : &g->tensors[it->second];
}

int gguf_config(const brew_gguf_s* g, brew_config* cfg) {
    brew_config c = {};
    const auto* av = meta_get(g, "general.architecture");
    BREW_CHECK(av && av->type == 8, BREW_ERR_IO, "general.architecture missing");
    int rc = arch_from_name(av->s, &c.arch);
    if (rc) return rc;
    const std::string p = av->s + ".";
    double v;
    auto need = [&](const char* k, double* out) {
        if (meta_num(g, p + k, out)) return BREW_OK;
        return set_error(BREW_ERR_IO, "GGUF metadata %s%s missing", p.c_str(), k);
    };
    if ((rc = need("embedding_length", &v))) return rc;
    c.dim = (int32_t)v;
    if ((rc = need("feed_forward_length", &v))) return rc;
    c.hidden_dim = (int32_t)v;
    if ((rc = need("block_count", &v))) return rc;
    c.n_layers = (int32_t)v;
    if ((rc = need("context_length", &v))) return rc;
    c.seq_len = (int32_t)v;
    if ((rc = need("attention.head_count", &v))) return rc;
    c.n_heads = (int32_t)v;
    c.n_kv_heads = meta_num(g, p + "attention.head_count_kv", &v) ? (int32_t)v : c.n_heads;
    c.eps = meta_num(g, p + "attention.layer_norm_rms_epsilon", &v) ? (float)v : 0.0f;
    c.sliding_window = meta_num(g, p + "attention.sliding_window", &v) ? (int32_t)v : 0;
    c.rope_base = meta_num(g, p + "rope.freq_base", &v) ? (float)v : 0.0f;
    c.rope_scale = 0.0f;   // not read from GGUF by the reference
    // head size: Qwen3CheckpointLoader.java:16, Gemma2/3CheckpointLoader.java:18, Config.getHeadSize
    if (c.arch == BREW_ARCH_QWEN3) c.head_size = 128;
    else if (arch_gemma(c.arch)) c.head_size = 256;
    else c.head_size = c.n_heads > 0 ? c.dim / c.n_heads : 0;
    const auto* tok = meta_get(g, "tokenizer.ggml.tokens");   // vocab = size of the token list
    BREW_CHECK(tok && tok->type == 9, BREW_ERR_IO, "tokenizer.ggml.tokens missing");
    c.vocab_size = (int32_t)tok->count;
    c.bos_token = meta_num(g, "tokenizer.ggml.bos_token_id", &v) ? (int32_t)v : -1;
    c.eos_token = meta_num(g, "tokenizer.ggml.eos_token_id", &v) ? (int32_t)v : -1;
    // tensor types; the classifier is the embedding when output.weight is absent
    const auto* te = tensor_get(g, "token_embd.weight");
    BREW_CHECK(te, BREW_ERR_IO, "token_embd.weight missing");
    c.type_embed = te->type;
    const auto* to = tensor_get(g, "output.weight");
    c.tied_embeddings = to ? 0 : 1;
    c.type_output = to ? to->type : te->type;
    const char* tails[7] = {"attn_q.weight", "attn_k.weight", "attn_v.weight", "attn_output.weight",
                            "ffn_gate.weight", "ffn_up.weight", "ffn_down.weight"};
    int32_t* types[7] = {&c.type_q, &c.type_k, &c.type_v, &c.type_o, &c.type_gate, &c.type_up, &c.type_down};
    for (int k = 0; k < 7; ++k) {
        const auto* t = tensor_get(g, std::string("blk.0.") + tails[k]);
        BREW_CHECK(t, BREW_ERR_IO, "blk.0.%s missing", tails[k]);
        *types[k] = t->type;
    }
    *cfg = c;
    return BREW_OK;
}

// Copies `bytes` bytes at `src` (in the mapping) to `dst` on the device
// through the two pinned staging buffers.
struct Uploader {
    static constexpr size_t CHUNK = 32u << 20;
    uint8_t* pin[2] = {nullptr, nullptr};
    cudaEvent_t ev[2] = {nullptr, nullptr};
    cudaStream_t s = nullptr;
    int k = 0;
    int init() {
        for (int i = 0; i < 2; ++i) {
            BREW_CUDA(cudaHostAlloc(reinterpret_cast<void**>(&pin[i]), CHUNK, cudaHostAllocDefault));
            BREW_CUDA(cudaEventCreateWithFlags(&ev[i], cudaEventDisableTiming));
        }
        BREW_CUDA(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking));
        return BREW_OK;
    }
    int copy(uint8_t* dst, const uint8_t* src, size_t bytes) {
        for (size_t o = 0; o < bytes; o += CHUNK) {
            const size_t n = std::min(CHUNK, bytes - o);
            BREW_CUDA(cudaEventSynchronize(ev[k]));   // this buffer's previous transfer is done
            memcpy(pin[k], src + o, n);
            BREW_CUDA(cudaMemcpyAsync(dst + o, pin[k], n, cudaMemcpyHostToDevice, s));
            BREW_CUDA(cudaEventRecord(ev[k], s));
            k ^= 1;
        }
        return BREW_OK;
    }
    int finish() {
        if (s) BREW_CUDA(cudaStreamSynchronize(s));
        return BREW_OK;
    }
    ~Uploader() {
        if (s) {
            cudaStreamSynchronize(s);
            cudaStreamDestroy(s);
        }
        for (int i = 0; i < 2; ++i) {
            if (ev[i]) cudaEventDestroy(ev[i]);
            if (pin[i]) cudaFreeHost(pin[i]);
        }
    }
};

// readFloatArray (GgufWeightsLoader.java:249-278): F32 or F16, else IOException.
int read_vector(const brew_gguf_s* g, const brew_gguf_s::Tensor& t, float* out) {
    const uint8_t* src = g->base + g->data_offset + t.offset;
    if (t.type == BREW_TYPE_F32) {
        memcpy(out, src, (size_t)t.n * 4);
    } else if (t.type == BREW_TYPE_F16) {
        for (int64_t i = 0; i < t.n; ++i) {
            uint16_t h;
            memcpy(&h, src + 2 * i, 2);
            out[i] = __half2float(__ushort_as_half(h));   // exact fp16 -> fp32 (HalfPrecisionFloat.toFloat)
        }
    } else {
        return set_error(BREW_ERR_IO, "Unexpected tensor type %d for %s", t.type, t.name.c_str());
    }
    return BREW_OK;
}

int gguf_load_model(const brew_gguf_s* g, int32_t max_batch, brew_model* out) {
    brew_config c;
    int rc = gguf_config(g, &c);
    if (rc) return rc;
    const int L = c.n_layers;
    const int64_t dim = c.dim, hs = c.head_size, hid = c.hidden_dim;
    const int64_t qw = (int64_t)c.n_heads * hs, kvd = (int64_t)c.n_kv_heads * hs;
    // matrix families (GgufWeightsLoader.java:88-117) and their per-layer shapes
    struct Fam {
        const char* tail;
        int type;
        int64_t n;   // elements per layer
        brew_tensor t;
    } fam[7] = {{"attn_q.weight", c.type_q, qw * dim, nullptr},      {"attn_k.weight", c.type_k, kvd * dim, nullptr},
                {"attn_v.weight", c.type_v, kvd * dim, nullptr},     {"attn_output.weight", c.type_o, dim * qw, nullptr},
                {"ffn_gate.weight", c.type_gate, hid * dim, nullptr}, {"ffn_up.weight", c.type_up, hid * dim, nullptr},
                {"ffn_down.weight", c.type_down, dim * hid, nullptr}};
    brew_tensor embd = nullptr, outw = nullptr;
    Uploader up;
    auto cleanup = [&]() {
        for (auto& f : fam) brew_tensor_free(f.t);
        brew_tensor_free(embd);
        brew_tensor_free(outw);
    };
    auto matrix = [&](const brew_gguf_s::Tensor* t, int type, int64_t n, const char* what) -> int {
        BREW_CHECK(t, BREW_ERR_IO, "tensor %s missing", what);
        BREW_CHECK(is_quant_matrix_type(t->type), BREW_ERR_UNSUPPORTED, "tensor %s has GGML type %d", t->name.c_str(),
                   t->type);
        BREW_CHECK(t->type == type, BREW_ERR_UNSUPPORTED, "tensor %s has GGML type %d, layer 0 has %d",
                   t->name.c_str(), t->type, type);
        BREW_CHECK(t->n == n, BREW_ERR_IO, "tensor %s has %lld elements, expected %lld", t->name.c_str(),
                   (long long)t->n, (long long)n);
        return BREW_OK;
    };
    if ((rc = up.init())) return rc;
    // embedding and classifier
    const auto* te = tensor_get(g, "token_embd.weight");
    if ((rc = matrix(te, c.type_embed, (int64_t)c.vocab_size * dim, "token_embd.weight")) ||
        (rc = brew_tensor_alloc(te->type, te->n, &embd)) ||
        (rc = up.copy(embd->d, g->base + g->data_offset + te->offset, (size_t)te->bytes))) {
        cleanup();
        return rc;
    }
    if (!c.tied_embeddings) {
        const auto* to = tensor_get(g, "output.weight");
        if ((rc = matrix(to, c.type_output, (int64_t)c.vocab_size * dim, "output.weight")) ||
            (rc = brew_tensor_alloc(to->type, to->n, &outw)) ||
            (rc = up.copy(outw->d, g->base + g->data_offset + to->offset, (size_t)to->bytes))) {
            cleanup();
            return rc;
        }
    }
    // layer matrices, concatenated over layers (concatenateQ8Blocks)
    for (auto& f : fam) {
        if ((rc = brew_tensor_alloc(f.type, f.n * L, &f.t))) {
            cleanup();
            return rc;
        }
        const int64_t lbytes = brew_type_bytes(f.type, f.n);
        for (int l = 0; l < L; ++l) {
            const std::string name = "blk." + std::to_string(l) + "." + f.tail;
            const auto* t = tensor_get(g, name);
            if ((rc = matrix(t, f.type, f.n, name.c_str())) ||
                (rc = up.copy(f.t->d + lbytes * l, g->base + g->data_offset + t->offset, (size_t)lbytes))) {
                cleanup();
                return rc;
            }
        }
    }
    if ((rc = up.finish())) {
        cleanup();
        return rc;
    }
    // norm and bias vectors (F32 / F16), concatenated over layers
    auto vec = [&](const char* tail, int64_t per, bool layered, std::vector<float>* dst, bool required) -> int {
        const int nl = layered ? L : 1;
        dst->assign((size_t)(per * nl), 0.0f);
        for (int l = 0; l < nl; ++l) {
            const std::string name = layered ? "blk." + std::to_string(l) + "." + tail : std::string(tail);
            const auto* t = tensor_get(g, name);
            if (!t) {
                if (required) return set_error(BREW_ERR_IO, "tensor %s missing", name.c_str());
                dst->clear();
                return BREW_OK;
            }
            BREW_CHECK(t->n == per, BREW_ERR_IO, "tensor %s has %lld elements, expected %lld", name.c_str(),
                       (long long)t->n, (long long)per);
            const int r = read_vector(g, *t, dst->data() + per * l);
            if (r) return r;
        }
        return BREW_OK;
    };
    const bool gemma = arch_gemma(c.arch), qk = arch_qknorm(c.arch), bias = c.arch == BREW_ARCH_QWEN2;
    std::vector<float> rms_att, rms_ffn, rms_final, post_att, post_ffn, rms_q, rms_k, qb, kb, vb;
    if ((rc = vec("attn_norm.weight", dim, true, &rms_att, true)) ||
        (rc = vec("ffn_norm.weight", dim, true, &rms_ffn, true)) ||
        (rc = vec("output_norm.weight", dim, false, &rms_final, true)) ||
        (rc = vec("post_attention_norm.weight", dim, true, &post_att, gemma)) ||
        (rc = vec("post_ffw_norm.weight", dim, true, &post_ffn, gemma)) ||
        (rc = vec("attn_q_norm.weight", hs, true, &rms_q, qk)) ||
        (rc = vec("attn_k_norm.weight", hs, true, &rms_k, qk)) ||
        (rc = vec("attn_q.bias", qw, true, &qb, bias)) || (rc = vec("attn_k.bias", kvd, true, &kb, bias)) ||
        (rc = vec("attn_v.bias", kvd, true, &vb, bias))) {
        cleanup();
        return rc;
    }
    auto ptr = [](const std::vector<float>& v) -> const float* { return v.empty() ? nullptr : v.data(); };
    brew_model_weights w = {};
    w.token_embd = embd;
    w.output = outw;
    w.wq = fam[0].t;
    w.wk = fam[1].t;
    w.wv = fam[2].t;
    w.wo = fam[3].t;
    w.w_gate = fam[4].t;
    w.w_up = fam[5].t;
    w.w_down = fam[6].t;
    w.rms_att = ptr(rms_att);
    w.rms_ffn = ptr(rms_ffn);
    w.rms_final = ptr(rms_final);
    w.post_att = ptr(post_att);
    w.post_ffn = ptr(post_ffn);
    w.rms_q = ptr(rms_q);
    w.rms_k = ptr(rms_k);
    w.q_bias = ptr(qb);
    w.k_bias = ptr(kb);
    w.v_bias = ptr(vb);
    if ((rc = brew_model_create(&c, &w, max_batch, out))) {
        cleanup();
        return rc;
    }
    model_adopt_tensors(*out);
    return BREW_OK;
}

}  // namespace
}  // namespace brew

using namespace brew;

extern "C" {

int brew_gguf_open(const char* path, brew_gguf* out) {
    BREW_CHECK(path && out, BREW_ERR_INVALID_ARG, "null argument");
    *out = nullptr;
    const int fd = open(path, O_RDONLY);
    BREW_CHECK(fd >= 0, BREW_ERR_IO, "cannot open %s", path);
    struct stat st;
    if (fstat(fd, &st) != 0 || st.st_size < 24) {
        close(fd);
        return set_error(BREW_ERR_IO, "%s: not a GGUF file (too short)", path);
    }
    void* base = mmap(nullptr, (size_t)st.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
    if (base == MAP_FAILED) {
        close(fd);
        return set_error(BREW_ERR_IO, "cannot map %s", path);
    }
    madvise(base, (size_t)st.st_size, MADV_SEQUENTIAL);
    brew_gguf g = new brew_gguf_s();
    g->fd = fd;
    g->base = static_cast<const uint8_t*>(base);
    g->size = (size_t)st.st_size;
    const int rc = gguf_parse(g);
    if (rc) {
        brew_gguf_close(g);
        return rc;
    }
    *out = g;
    return BREW_OK;
}

int brew_gguf_close(brew_gguf g) {
    if (!g) return BREW_OK;
    if (g->base) munmap(const_cast<uint8_t*>(g->base), g->size);
    if (g->fd >= 0) close(g->fd);
    delete g;
    return BREW_OK;
}

int brew_gguf_config(brew_gguf g, brew_config* cfg) {
    BREW_CHECK(g && cfg, BREW_ERR_INVALID_ARG, "null argument");
    return gguf_config(g, cfg);
}

int brew_gguf_tensor_count(brew_gguf g, int64_t* n) {
    BREW_CHECK(g && n, BREW_ERR_INVALID_ARG, "null argument");
    *n = (int64_t)g->tensors.size();
    return BREW_OK;
}

int brew_gguf_tensor_info(brew_gguf g, int64_t i, char* name, size_t name_size, int* type, int64_t* n_elements,
                          int64_t* file_offset) {
    BREW_CHECK(g, BREW_ERR_INVALID_ARG, "null argument");
    BREW_CHECK(i >= 0 && i < (int64_t)g->tensors.size(), BREW_ERR_OUT_OF_BOUNDS, "tensor index %lld", (long long)i);
    const auto& t = g->tensors[(size_t)i];
    if (name && name_size) snprintf(name, name_size, "%s", t.name.c_str());
    if (type) *type = t.type;
    if (n_elements) *n_elements = t.n;
    if (file_offset) *file_offset = (int64_t)(g->data_offset + t.offset);
    return BREW_OK;
}

int brew_model_load_gguf(const char* path, int32_t max_batch, brew_model* out) {
    BREW_CHECK(path && out, BREW_ERR_INVALID_ARG, "null argument");
    *out = nullptr;
    brew_gguf g = nullptr;
    int rc = brew_gguf_open(path, &g);
    if (rc) return rc;
    rc = gguf_load_model(g, max_batch, out);
    brew_gguf_close(g);
    return rc;
}

}  // extern "C"
