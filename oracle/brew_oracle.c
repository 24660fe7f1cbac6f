/*
 * brew_oracle.c — CPU restatement of brewference's hot path (the oracle).
 *
 * TEST INFRASTRUCTURE ONLY: the tests, the smoke check and bench.py's
 * CPU-baseline leg load this file's library as the checker.  The product
 * library never links it.
 *
 * Floating-point rules follow the Java sources: every float operation is an
 * IEEE binary32 operation rounded on its own (compile with -ffp-contract=off,
 * no fast-math; Java has no implicit FMA), and the places where Java widens
 * to double (Math.sqrt/exp/pow/sin/cos/tanh and double literals) widen here
 * too.  Citations are relative to src/main/java/com/epicmonstrosity/
 * brewference/ of the reference.
 *
 * Formats the reference does not decode (Q4_0, Q4_K, Q6_K) follow GGML's
 * block layout as implemented by gguf-py 0.19.0 (gguf/quants.py), whose
 * quantize/dequantize outputs are committed as fixtures under tests/golden/.
 */
#include "brew_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

/* ======================================================================= */
/* fp16                                                                      */
/* ======================================================================= */

/* HalfPrecisionFloat.toFloat (gguf/HalfPrecisionFloat.java:21-59): exact
 * widening, including subnormals (normalised by shifting), inf and NaN
 * (mantissa carried into the top of the fp32 mantissa). */
float ob_half_to_float(uint16_t half) {
    const uint32_t h = half;
    const uint32_t sign = ((h >> 15) & 1u) << 31;
    int exponent = (int)((h >> 10) & 0x1F);
    uint32_t mantissa = h & 0x3FF;
    uint32_t bits;
    if (exponent == 0) {
        if (mantissa == 0) {
            bits = sign;
        } else {
            int e = 1;                                  /* :43-52 */
            while ((mantissa & 0x400) == 0) { mantissa <<= 1; e--; }
            mantissa &= 0x3FF;
            bits = sign | ((uint32_t)(e + 127 - 15) << 23) | (mantissa << 13);
        }
    } else if (exponent == 0x1F) {
        bits = sign | (0xFFu << 23) | (mantissa << 13);
    } else {
        bits = sign | ((uint32_t)(exponent + 127 - 15) << 23) | (mantissa << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* fp32 -> fp16, round to nearest even (numpy's astype(np.float16), which
 * gguf-py uses to store block scales). */
uint16_t ob_float_to_half(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t a = x & 0x7FFFFFFFu;
    if (a >= 0x7F800000u) {                       /* inf / nan */
        if (a == 0x7F800000u) return (uint16_t)(sign | 0x7C00u);
        return (uint16_t)(sign | 0x7E00u | ((a >> 13) & 0x3FFu));
    }
    if (a >= 0x477FF000u) return (uint16_t)(sign | 0x7C00u);   /* >= 65520: inf */
    if (a < 0x38800000u) {                        /* half subnormal or zero */
        if (a < 0x33000000u) return (uint16_t)sign;            /* < 2^-25 */
        const uint32_t e = a >> 23;
        const uint32_t m = (a & 0x7FFFFFu) | 0x800000u;
        const uint32_t shift = 126u - e;          /* 14..24 */
        uint32_t mh = m >> shift;
        const uint32_t rem = m & ((1u << shift) - 1u);
        const uint32_t halfway = 1u << (shift - 1u);
        if (rem > halfway || (rem == halfway && (mh & 1u))) mh++;
        return (uint16_t)(sign | mh);
    }
    uint32_t h = ((((a >> 23) - 112u) << 10) | ((a >> 13) & 0x3FFu));
    const uint32_t rem = a & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;
    return (uint16_t)(sign | h);
}

/* ======================================================================= */
/* thread pool (stands in for the JVM ForkJoin common pool,                  */
/* transformer/math/Linear.java:59-63 and the head-parallel attention)       */
/* ======================================================================= */

typedef void (*ob_task)(void* ctx, int64_t begin, int64_t end);

static int g_threads = 0;
static pthread_mutex_t g_mu = PTHREAD_MUTEX_INITIALIZER;
static pthread_cond_t g_cv_job = PTHREAD_COND_INITIALIZER;
static pthread_cond_t g_cv_done = PTHREAD_COND_INITIALIZER;
static int g_pool_size = 0;          /* worker threads (excluding caller) */
static uint64_t g_generation = 0;
static ob_task g_fn;
static void* g_ctx;
static int64_t g_n, g_grain, g_next;
static int g_active;

static int ob_hw_threads(void) {
    long n = sysconf(_SC_NPROCESSORS_ONLN);
    return n > 0 ? (int)n : 1;
}

void ob_set_threads(int n) { g_threads = n; }
int ob_get_threads(void) { return g_threads > 0 ? g_threads : ob_hw_threads(); }

static void run_chunks(ob_task fn, void* ctx) {
    for (;;) {
        int64_t b;
        pthread_mutex_lock(&g_mu);
        b = g_next;
        g_next += g_grain;
        pthread_mutex_unlock(&g_mu);
        if (b >= g_n) break;
        int64_t e = b + g_grain < g_n ? b + g_grain : g_n;
        fn(ctx, b, e);
    }
}

static void* worker_main(void* arg) {
    (void)arg;
    uint64_t seen = 0;
    for (;;) {
        pthread_mutex_lock(&g_mu);
        while (g_generation == seen) pthread_cond_wait(&g_cv_job, &g_mu);
        seen = g_generation;
        ob_task fn = g_fn;
        void* ctx = g_ctx;
        pthread_mutex_unlock(&g_mu);
        run_chunks(fn, ctx);
        pthread_mutex_lock(&g_mu);
        if (--g_active == 0) pthread_cond_signal(&g_cv_done);
        pthread_mutex_unlock(&g_mu);
    }
    return NULL;
}

static pthread_mutex_t g_call_mu = PTHREAD_MUTEX_INITIALIZER;

static void parallel_for(int64_t n, int64_t grain, ob_task fn, void* ctx) {
    int want = ob_get_threads() - 1;
    if (n <= grain || want <= 0) { fn(ctx, 0, n); return; }
    pthread_mutex_lock(&g_call_mu);
    pthread_mutex_lock(&g_mu);
    while (g_pool_size < want) {
        pthread_t t;
        if (pthread_create(&t, NULL, worker_main, NULL) != 0) break;
        pthread_detach(t);
        g_pool_size++;
    }
    g_fn = fn; g_ctx = ctx; g_n = n; g_grain = grain; g_next = 0;
    g_active = g_pool_size;
    g_generation++;
    pthread_cond_broadcast(&g_cv_job);
    pthread_mutex_unlock(&g_mu);
    run_chunks(fn, ctx);
    pthread_mutex_lock(&g_mu);
    while (g_active > 0) pthread_cond_wait(&g_cv_done, &g_mu);
    pthread_mutex_unlock(&g_mu);
    pthread_mutex_unlock(&g_call_mu);
}

/* ======================================================================= */
/* synthetic values                                                          */
/* ======================================================================= */

static inline uint64_t mix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

/* Irwin-Hall sum of twelve 16-bit uniforms, centred: mean 0, variance 1.
 * Integer arithmetic up to one exact and one rounded fp32 multiply, so the
 * device generator reproduces it bit for bit. */
float ob_synth_value(uint64_t seed, uint32_t tensor_id, uint64_t index, float std_dev) {
    const uint64_t key = mix64(seed ^ ((uint64_t)tensor_id << 32) ^ 0x5851F42D4C957F2Dull);
    int32_t s = 0;
    for (int j = 0; j < 3; j++) {
        uint64_t h = mix64(key + 3ull * index + (uint64_t)j);
        s += (int32_t)(h & 0xFFFF) + (int32_t)((h >> 16) & 0xFFFF)
           + (int32_t)((h >> 32) & 0xFFFF) + (int32_t)((h >> 48) & 0xFFFF);
    }
    const int32_t num = 2 * s + 12 - 12 * 65536;     /* sum of (2u+1-65536) */
    const float z = (float)num * 7.62939453125e-06f;  /* * 2^-17, exact */
    return z * std_dev;
}

void ob_synth_fill(uint64_t seed, uint32_t tensor_id, uint64_t start, int64_t n, float std_dev, float* out) {
    for (int64_t i = 0; i < n; i++) out[i] = ob_synth_value(seed, tensor_id, start + (uint64_t)i, std_dev);
}

/* ======================================================================= */
/* block formats                                                             */
/* ======================================================================= */

int ob_type_block(int type, int* be, int* bb) {
    switch (type) {
        case BREW_TYPE_F32:  *be = 1;   *bb = 4;   return 0;
        case BREW_TYPE_F16:  *be = 1;   *bb = 2;   return 0;
        case BREW_TYPE_Q4_0: *be = 32;  *bb = 18;  return 0;
        case BREW_TYPE_Q8_0: *be = 32;  *bb = 34;  return 0;
        case BREW_TYPE_Q4_K: *be = 256; *bb = 144; return 0;
        case BREW_TYPE_Q6_K: *be = 256; *bb = 210; return 0;
        default: return -1;
    }
}

int64_t ob_type_bytes(int type, int64_t n) {
    int be, bb;
    if (ob_type_block(type, &be, &bb) != 0 || n % be != 0) return -1;
    return n / be * bb;
}

static inline void put_half(uint8_t* p, float f) {
    uint16_t h = ob_float_to_half(f);
    p[0] = (uint8_t)(h & 0xFF);
    p[1] = (uint8_t)(h >> 8);
}
static inline float get_half(const uint8_t* p) {
    return ob_half_to_float((uint16_t)(p[0] | (p[1] << 8)));
}

/* gguf-py Q8_0.quantize_blocks (quants.py:380-393): d = amax/127,
 * q = round-half-away(x * (1/d)), d stored as fp16. */
static void quant_q8_0(const float* x, uint8_t* out) {
    float amax = 0.0f;
    for (int i = 0; i < 32; i++) { float a = fabsf(x[i]); if (a > amax) amax = a; }
    const float d = amax / 127.0f;
    const float id = d == 0.0f ? 0.0f : 1.0f / d;
    put_half(out, d);
    for (int i = 0; i < 32; i++) {
        float v = roundf(x[i] * id);
        out[2 + i] = (uint8_t)(int8_t)(int)v;
    }
}

/* gguf-py Q4_0.quantize_blocks (quants.py:222-238): d = x[argmax|x|] / -8,
 * q = clip(trunc(x * (1/d) + 8.5), 0, 15), element j in the low nibble and
 * j+16 in the high nibble of byte j. */
static void quant_q4_0(const float* x, uint8_t* out) {
    int imax = 0;
    float amax = fabsf(x[0]);
    for (int i = 1; i < 32; i++) { float a = fabsf(x[i]); if (a > amax) { amax = a; imax = i; } }
    const float d = x[imax] / -8.0f;
    const float id = d == 0.0f ? 0.0f : 1.0f / d;
    uint8_t q[32];
    for (int i = 0; i < 32; i++) {
        float t = truncf(x[i] * id + 8.5f);
        int qi = (int)t;
        if (qi < 0) qi = 0;
        if (qi > 15) qi = 15;
        q[i] = (uint8_t)qi;
    }
    put_half(out, d);
    for (int j = 0; j < 16; j++) out[2 + j] = (uint8_t)(q[j] | (q[j + 16] << 4));
}

static inline int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

/* Q4_K quantizer of this project (gguf-py has none): per 32-element
 * sub-block scale = (max - min(0,min)) / 15 and min = -min(0,min), six-bit
 * sub-scales against fp16 super-scales d = max(scale)/63, dmin =
 * max(min)/63.  Layout per GGML block_q4_K: d, dmin, 12 packed scale bytes
 * (get_scale_min_k4), 128 nibble bytes (chunk c of 64 elements: low nibbles
 * = sub-block 2c, high nibbles = 2c+1). */
static void quant_q4_k(const float* x, uint8_t* out) {
    float scale[8], minv[8];
    float maxscale = 0.0f, maxmin = 0.0f;
    for (int s = 0; s < 8; s++) {
        float mn = 0.0f, mx = x[32 * s];
        for (int i = 0; i < 32; i++) {
            float v = x[32 * s + i];
            if (v < mn) mn = v;
            if (v > mx) mx = v;
        }
        if (mx < mn) mx = mn;
        scale[s] = (mx - mn) / 15.0f;
        minv[s] = -mn;
        if (scale[s] > maxscale) maxscale = scale[s];
        if (minv[s] > maxmin) maxmin = minv[s];
    }
    const float d = maxscale / 63.0f, dmin = maxmin / 63.0f;
    put_half(out + 0, d);
    put_half(out + 2, dmin);
    const float df = get_half(out + 0), dminf = get_half(out + 2);
    int sc[8], m[8];
    for (int s = 0; s < 8; s++) {
        sc[s] = df > 0.0f ? clampi((int)roundf(scale[s] / df), 0, 63) : 0;
        m[s] = dminf > 0.0f ? clampi((int)roundf(minv[s] / dminf), 0, 63) : 0;
    }
    uint8_t* sb = out + 4;
    for (int j = 0; j < 4; j++) {
        sb[j] = (uint8_t)(sc[j] | ((sc[j + 4] >> 4) << 6));
        sb[j + 4] = (uint8_t)(m[j] | ((m[j + 4] >> 4) << 6));
        sb[j + 8] = (uint8_t)((sc[j + 4] & 15) | ((m[j + 4] & 15) << 4));
    }
    uint8_t q[256];
    for (int s = 0; s < 8; s++) {
        const float es = df * (float)sc[s];
        const float em = dminf * (float)m[s];
        for (int i = 0; i < 32; i++) {
            int qi = 0;
            if (es > 0.0f) qi = clampi((int)roundf((x[32 * s + i] + em) / es), 0, 15);
            q[32 * s + i] = (uint8_t)qi;
        }
    }
    uint8_t* qs = out + 16;
    for (int c = 0; c < 4; c++)
        for (int i = 0; i < 32; i++)
            qs[32 * c + i] = (uint8_t)(q[64 * c + i] | (q[64 * c + 32 + i] << 4));
}

/* Q6_K quantizer of this project: per 16-element sub-block scale = amax/31,
 * int8 sub-scales against the fp16 super-scale d = max(scale)/127,
 * q = clamp(round(x / (d*sc)), -32, 31) + 32.  Layout per GGML block_q6_K:
 * ql[128], qh[64], int8 scales[16], d. */
static void quant_q6_k(const float* x, uint8_t* out) {
    float scale[16];
    float maxsc = 0.0f;
    for (int s = 0; s < 16; s++) {
        float amax = 0.0f;
        for (int i = 0; i < 16; i++) { float a = fabsf(x[16 * s + i]); if (a > amax) amax = a; }
        scale[s] = amax / 31.0f;
        if (scale[s] > maxsc) maxsc = scale[s];
    }
    const float d = maxsc / 127.0f;
    put_half(out + 208, d);
    const float df = get_half(out + 208);
    int sc[16];
    for (int s = 0; s < 16; s++) sc[s] = df > 0.0f ? clampi((int)roundf(scale[s] / df), -128, 127) : 0;
    uint8_t u[256];
    for (int s = 0; s < 16; s++) {
        const float e = df * (float)sc[s];
        for (int i = 0; i < 16; i++) {
            int qi = 0;
            if (e > 0.0f) qi = clampi((int)roundf(x[16 * s + i] / e), -32, 31);
            u[16 * s + i] = (uint8_t)(qi + 32);
        }
    }
    uint8_t* ql = out;
    uint8_t* qh = out + 128;
    int8_t* scales = (int8_t*)(out + 192);
    for (int s = 0; s < 16; s++) scales[s] = (int8_t)sc[s];
    for (int h = 0; h < 2; h++) {
        for (int l = 0; l < 32; l++) {
            const int u1 = u[128 * h + l], u2 = u[128 * h + 32 + l];
            const int u3 = u[128 * h + 64 + l], u4 = u[128 * h + 96 + l];
            ql[64 * h + l] = (uint8_t)((u1 & 15) | ((u3 & 15) << 4));
            ql[64 * h + 32 + l] = (uint8_t)((u2 & 15) | ((u4 & 15) << 4));
            qh[32 * h + l] = (uint8_t)((u1 >> 4) | ((u2 >> 4) << 2) | ((u3 >> 4) << 4) | ((u4 >> 4) << 6));
        }
    }
}

int ob_quantize(int type, const float* x, int64_t n, uint8_t* out) {
    int be, bb;
    if (ob_type_block(type, &be, &bb) != 0 || n % be != 0) return -1;
    const int64_t nb = n / be;
    for (int64_t b = 0; b < nb; b++) {
        const float* xb = x + b * be;
        uint8_t* ob = out + b * bb;
        switch (type) {
            case BREW_TYPE_Q8_0: quant_q8_0(xb, ob); break;
            case BREW_TYPE_Q4_0: quant_q4_0(xb, ob); break;
            case BREW_TYPE_Q4_K: quant_q4_k(xb, ob); break;
            case BREW_TYPE_Q6_K: quant_q6_k(xb, ob); break;
            case BREW_TYPE_F32: memcpy(ob, xb, 4); break;
            case BREW_TYPE_F16: put_half(ob, xb[0]); break;
            default: return -1;
        }
    }
    return 0;
}

/* Dequantizes one whole block into out[be].
 *   Q8_0: q * d                     QuantizedWeights.java:76-85 (and gguf-py)
 *   Q4_0: d * (q - 8)               gguf-py Q4_0.dequantize_blocks
 *   Q4_K: (d*sc) * q - (dmin*m)     gguf-py Q4_K.dequantize_blocks
 *   Q6_K: (d*sc) * (q - 32)         gguf-py Q6_K.dequantize_blocks */
static void dequant_block(int type, const uint8_t* b, float* out) {
    switch (type) {
        case BREW_TYPE_Q8_0: {
            const float d = get_half(b);
            for (int i = 0; i < 32; i++) out[i] = (float)(int8_t)b[2 + i] * d;
            break;
        }
        case BREW_TYPE_Q4_0: {
            const float d = get_half(b);
            for (int j = 0; j < 16; j++) {
                out[j] = d * (float)((int)(b[2 + j] & 15) - 8);
                out[j + 16] = d * (float)((int)(b[2 + j] >> 4) - 8);
            }
            break;
        }
        case BREW_TYPE_Q4_K: {
            const float d = get_half(b), dmin = get_half(b + 2);
            const uint8_t* sb = b + 4;
            const uint8_t* qs = b + 16;
            for (int s = 0; s < 8; s++) {
                int sc, m;
                if (s < 4) { sc = sb[s] & 63; m = sb[s + 4] & 63; }
                else {
                    sc = (sb[s + 4] & 0xF) | ((sb[s - 4] >> 6) << 4);
                    m = (sb[s + 4] >> 4) | ((sb[s] >> 6) << 4);
                }
                const float t = d * (float)sc, u = dmin * (float)m;
                const int c = s / 2, hi = s & 1;
                for (int i = 0; i < 32; i++) {
                    const int q = hi ? (qs[32 * c + i] >> 4) : (qs[32 * c + i] & 15);
                    out[32 * s + i] = t * (float)q - u;
                }
            }
            break;
        }
        case BREW_TYPE_Q6_K: {
            const uint8_t* ql = b;
            const uint8_t* qh = b + 128;
            const int8_t* sc = (const int8_t*)(b + 192);
            const float d = get_half(b + 208);
            for (int e = 0; e < 256; e++) {
                const int h = e / 128, r = e % 128, grp = r / 32, l = r % 32;
                const int lq = ql[64 * h + (grp & 1) * 32 + l];
                const int low = grp < 2 ? (lq & 15) : (lq >> 4);
                const int high = (qh[32 * h + l] >> (2 * grp)) & 3;
                const int q = (low | (high << 4)) - 32;
                const float t = d * (float)sc[e / 16];
                out[e] = t * (float)q;
            }
            break;
        }
        case BREW_TYPE_F32: memcpy(out, b, 4); break;
        case BREW_TYPE_F16: out[0] = get_half(b); break;
    }
}

int ob_dequantize(int type, const uint8_t* bytes, int64_t off, int64_t n, float* out) {
    int be, bb;
    if (ob_type_block(type, &be, &bb) != 0) return -1;
    float tmp[256];
    int64_t i = 0;
    while (i < n) {
        const int64_t e = off + i;
        const int64_t blk = e / be;
        const int in = (int)(e % be);
        dequant_block(type, bytes + blk * bb, tmp);
        int take = be - in;
        if (take > n - i) take = (int)(n - i);
        memcpy(out + i, tmp + in, (size_t)take * sizeof(float));
        i += take;
    }
    return 0;
}

typedef struct { int type; uint64_t seed; uint32_t id; float sd; uint8_t* out; int be, bb; } synthq_ctx;

static void synthq_task(void* vctx, int64_t b0, int64_t b1) {
    synthq_ctx* c = (synthq_ctx*)vctx;
    float x[256];
    for (int64_t b = b0; b < b1; b++) {
        ob_synth_fill(c->seed, c->id, (uint64_t)(b * c->be), c->be, c->sd, x);
        ob_quantize(c->type, x, c->be, c->out + b * c->bb);
    }
}

int ob_synth_quantized(int type, uint64_t seed, uint32_t tensor_id, int64_t n, float sd, uint8_t* out) {
    synthq_ctx c;
    if (ob_type_block(type, &c.be, &c.bb) != 0 || n % c.be != 0) return -1;
    c.type = type; c.seed = seed; c.id = tensor_id; c.sd = sd; c.out = out;
    parallel_for(n / c.be, 4096, synthq_task, &c);
    return 0;
}

/* ======================================================================= */
/* Linear.matmul (transformer/math/Linear.java:40-99)                        */
/* ======================================================================= */

/* computeRowDotProduct (Linear.java:76-99): per 32-element block a
 * sequential fp32 sum of (float)q * x, then rowSum += blockSum * scale.
 * Q4_0 uses the same form with (q - 8).  K-quants (no reference code): per
 * 32-element group a sequential fp32 sum of dequant(w) * x, added to rowSum. */
static float row_dot(int type, const uint8_t* w, int64_t row_elem, const float* x, int K) {
    float rowSum = 0.0f;
    if (type == BREW_TYPE_Q8_0 || type == BREW_TYPE_Q4_0) {
        const int bb = type == BREW_TYPE_Q8_0 ? 34 : 18;
        const uint8_t* b = w + (row_elem / 32) * bb;
        for (int blk = 0; blk < K / 32; blk++, b += bb) {
            const float scale = get_half(b);
            float blockSum = 0.0f;
            if (type == BREW_TYPE_Q8_0) {
                for (int i = 0; i < 32; i++) blockSum += (float)(int8_t)b[2 + i] * x[blk * 32 + i];
            } else {
                for (int i = 0; i < 32; i++) {
                    const int q = i < 16 ? (b[2 + i] & 15) : (b[2 + i - 16] >> 4);
                    blockSum += (float)(q - 8) * x[blk * 32 + i];
                }
            }
            rowSum += blockSum * scale;
        }
        return rowSum;
    }
    float tmp[256];
    int be, bb;
    ob_type_block(type, &be, &bb);
    for (int k0 = 0; k0 < K; k0 += be) {
        dequant_block(type, w + ((row_elem + k0) / be) * bb, tmp);
        for (int g = 0; g < be; g += 32) {
            float blockSum = 0.0f;
            for (int i = 0; i < 32; i++) blockSum += tmp[g + i] * x[k0 + g + i];
            rowSum += blockSum;
        }
    }
    return rowSum;
}

typedef struct { int type; const uint8_t* w; int64_t woff; const float* x; float* y; int K; } mv_ctx;

static void mv_task(void* vctx, int64_t r0, int64_t r1) {
    mv_ctx* c = (mv_ctx*)vctx;
    for (int64_t r = r0; r < r1; r++) c->y[r] = row_dot(c->type, c->w, c->woff + r * (int64_t)c->K, c->x, c->K);
}

int ob_matvec(int type, const uint8_t* w, int64_t woff, const float* x, float* y, int K, int N) {
    int be, bb;
    if (ob_type_block(type, &be, &bb) != 0 || K % be != 0 || woff % be != 0) return -1;
    mv_ctx c = {type, w, woff, x, y, K};
    if (N < 256) mv_task(&c, 0, N);          /* Linear.java:52-57: sequential */
    else parallel_for(N, 64, mv_task, &c);   /* :58-63: row-parallel        */
    return 0;
}

/* ======================================================================= */
/* Kernels.* (transformer/math/Kernels.java)                                 */
/* ======================================================================= */

/* inverseRootMeanSquare (:77-88) + rmsNorm (:47-58): in place allowed. */
void ob_rmsnorm(float* out, const float* in, const float* w, int n, float eps) {
    float ss = 0.0f;
    for (int i = 0; i < n; i++) { const float v = in[i]; ss += v * v; }
    const float meanSquare = ss / (float)n;
    const float scale = (float)(1.0 / sqrt((double)(meanSquare + eps)));
    for (int i = 0; i < n; i++) out[i] = in[i] * scale * w[i];
}

/* headWiseRmsNorm (:22-30): weight slice shared by all heads. */
void ob_headwise_rmsnorm(float* v, const float* w, int heads, int hs, float eps) {
    for (int h = 0; h < heads; h++) ob_rmsnorm(v + h * hs, v + h * hs, w, hs, eps);
}

/* softMax (:100-126) */
void ob_softmax(float* v, int n) {
    float mx = v[0];
    for (int i = 1; i < n; i++) if (v[i] > mx) mx = v[i];
    float sum = 0.0f;
    for (int i = 0; i < n; i++) { const float e = (float)exp((double)(v[i] - mx)); v[i] = e; sum += e; }
    const float inv = 1.0f / sum;
    for (int i = 0; i < n; i++) v[i] *= inv;
}

/* argMax (:150-162): first index of the maximum */
int ob_argmax(const float* v, int n) {
    int mi = 0;
    float mv = v[0];
    for (int i = 1; i < n; i++) if (v[i] > mv) { mv = v[i]; mi = i; }
    return mi;
}

/* RopeCache.precomputeAngles (transformer/rope/RopeCache.java:15-26) and
 * InterleavedRope / NonInterleavedRope.applyToHeads. */
static void rope_heads(float* v, int heads, int hs, const float* cs, const float* sn, int interleaved) {
    const int half = hs / 2;
    for (int h = 0; h < heads; h++) {
        float* p = v + h * hs;
        for (int d = 0; d < half; d++) {
            const int i0 = interleaved ? 2 * d : d;
            const int i1 = interleaved ? 2 * d + 1 : d + half;
            const float a = p[i0], b = p[i1];
            p[i0] = a * cs[d] - b * sn[d];
            p[i1] = a * sn[d] + b * cs[d];
        }
    }
}

void ob_rope(float* q, float* k, int nh, int nkv, int hs, float base, float position, int interleaved) {
    const int half = hs / 2;
    float cs[512], sn[512];
    for (int p = 0; p < half; p++) {
        const float invf = (float)(1.0 / pow((double)base, (double)((float)(2 * p) / (float)hs)));
        const float ang = position * invf;
        cs[p] = (float)cos((double)ang);
        sn[p] = (float)sin((double)ang);
    }
    rope_heads(q, nh, hs, cs, sn, interleaved);
    rope_heads(k, nkv, hs, cs, sn, interleaved);
}

/* FfnActivation.swiGlu / geGlu (transformer/ffn/FfnActivation.java:23-58) */
void ob_glu(float* hb, const float* hb2, int n, int gelu) {
    const float c0 = 0.7978845608028654f, c1 = 0.044715f;
    for (int i = 0; i < n; i++) {
        const double v = (double)hb[i];
        double a;
        if (gelu) {
            const double inner = (double)c0 * (v + (double)c1 * v * v * v);
            a = 0.5 * v * (1.0 + tanh(inner));
        } else {
            a = v / (1.0 + exp(-v));
        }
        hb[i] = (float)a * hb2[i];
    }
}

/* ======================================================================= */
/* model                                                                     */
/* ======================================================================= */

struct ob_model {
    brew_config c;
    uint8_t* t[9];        /* packed tensors by OB_W_* (output aliases embed when tied) */
    int64_t tbytes[9];
    float *rms_att, *rms_ffn, *rms_final, *post_att, *post_ffn, *rms_q, *rms_k;
    float *q_bias, *k_bias, *v_bias;
    /* RunState (transformer/RunState.java) */
    float *x, *xb, *xb2, *hb, *hb2, *q, *k, *v, *att, *logits, *kc, *vc;
};

static int type_of(const brew_config* c, int which) {
    switch (which) {
        case OB_W_EMBED: return c->type_embed;
        case OB_W_OUTPUT: return c->tied_embeddings ? c->type_embed : c->type_output;
        case OB_W_Q: return c->type_q;
        case OB_W_K: return c->type_k;
        case OB_W_V: return c->type_v;
        case OB_W_O: return c->type_o;
        case OB_W_GATE: return c->type_gate;
        case OB_W_UP: return c->type_up;
        default: return c->type_down;
    }
}

/* rows x cols of one layer's matrix (ne1 = out, ne0 = in) */
static void shape_of(const brew_config* c, int which, int64_t* rows, int64_t* cols) {
    const int64_t qw = (int64_t)c->n_heads * c->head_size, kvd = (int64_t)c->n_kv_heads * c->head_size;
    switch (which) {
        case OB_W_EMBED: case OB_W_OUTPUT: *rows = c->vocab_size; *cols = c->dim; break;
        case OB_W_Q: *rows = qw; *cols = c->dim; break;
        case OB_W_K: case OB_W_V: *rows = kvd; *cols = c->dim; break;
        case OB_W_O: *rows = c->dim; *cols = qw; break;
        case OB_W_GATE: case OB_W_UP: *rows = c->hidden_dim; *cols = c->dim; break;
        default: *rows = c->dim; *cols = c->hidden_dim; break;
    }
}

static float* filled(int64_t n, float v) {
    float* p = (float*)malloc((size_t)n * sizeof(float));
    for (int64_t i = 0; i < n; i++) p[i] = v;
    return p;
}

ob_model* ob_model_synth(const brew_config* cfg, uint64_t seed) {
    ob_model* m = (ob_model*)calloc(1, sizeof(ob_model));
    m->c = *cfg;
    const brew_config* c = &m->c;
    const int L = c->n_layers;
    for (int w = 0; w < 9; w++) {
        if (w == OB_W_OUTPUT && c->tied_embeddings) continue;
        int64_t rows, cols;
        shape_of(c, w, &rows, &cols);
        const int type = type_of(c, w);
        const int layers = (w == OB_W_EMBED || w == OB_W_OUTPUT) ? 1 : L;
        const int64_t per = ob_type_bytes(type, rows * cols);
        if (per < 0) { ob_model_free(m); return NULL; }
        m->tbytes[w] = per * layers;
        m->t[w] = (uint8_t*)malloc((size_t)m->tbytes[w] + 64);
        for (int l = 0; l < layers; l++)
            ob_synth_quantized(type, seed, OB_TENSOR_ID(w, l), rows * cols, 0.02f, m->t[w] + per * l);
    }
    if (c->tied_embeddings) { m->t[OB_W_OUTPUT] = m->t[OB_W_EMBED]; m->tbytes[OB_W_OUTPUT] = m->tbytes[OB_W_EMBED]; }
    const int64_t dim = c->dim, hs = c->head_size, qw = (int64_t)c->n_heads * hs, kvd = (int64_t)c->n_kv_heads * hs;
    m->rms_att = filled(L * dim, 1.0f);
    m->rms_ffn = filled(L * dim, 1.0f);
    m->rms_final = filled(dim, 1.0f);
    if (c->arch == BREW_ARCH_GEMMA3 || c->arch == BREW_ARCH_GEMMA2) {
        m->post_att = filled(L * dim, 1.0f);
        m->post_ffn = filled(L * dim, 1.0f);
    }
    if (c->arch == BREW_ARCH_QWEN3 || c->arch == BREW_ARCH_GEMMA3) { m->rms_q = filled(L * hs, 1.0f); m->rms_k = filled(L * hs, 1.0f); }
    if (c->arch == BREW_ARCH_QWEN2) {
        m->q_bias = (float*)malloc((size_t)(L * qw) * sizeof(float));
        m->k_bias = (float*)malloc((size_t)(L * kvd) * sizeof(float));
        m->v_bias = (float*)malloc((size_t)(L * kvd) * sizeof(float));
        for (int l = 0; l < L; l++) {
            ob_synth_fill(seed, OB_TENSOR_ID(OB_B_Q, l), 0, qw, 0.02f, m->q_bias + l * qw);
            ob_synth_fill(seed, OB_TENSOR_ID(OB_B_K, l), 0, kvd, 0.02f, m->k_bias + l * kvd);
            ob_synth_fill(seed, OB_TENSOR_ID(OB_B_V, l), 0, kvd, 0.02f, m->v_bias + l * kvd);
        }
    }
    const int64_t xbd = qw > dim ? qw : dim;
    m->x = filled(dim, 0); m->xb = filled(xbd, 0); m->xb2 = filled(dim, 0);
    m->hb = filled(c->hidden_dim, 0); m->hb2 = filled(c->hidden_dim, 0);
    m->q = filled(qw, 0); m->k = filled(kvd, 0); m->v = filled(kvd, 0);
    m->att = filled((int64_t)c->n_heads * c->seq_len, 0);
    m->logits = filled(c->vocab_size, 0);
    m->kc = filled((int64_t)L * c->seq_len * kvd, 0);
    m->vc = filled((int64_t)L * c->seq_len * kvd, 0);
    return m;
}

void ob_model_free(ob_model* m) {
    if (!m) return;
    for (int w = 0; w < 9; w++) if (!(w == OB_W_OUTPUT && m->c.tied_embeddings)) free(m->t[w]);
    float* fs[] = {m->rms_att, m->rms_ffn, m->rms_final, m->post_att, m->post_ffn, m->rms_q, m->rms_k,
                   m->q_bias, m->k_bias, m->v_bias, m->x, m->xb, m->xb2, m->hb, m->hb2, m->q, m->k, m->v,
                   m->att, m->logits, m->kc, m->vc};
    for (size_t i = 0; i < sizeof(fs) / sizeof(fs[0]); i++) free(fs[i]);
    free(m);
}

const uint8_t* ob_model_tensor(ob_model* m, int which, int64_t* n_bytes) {
    if (which < 0 || which > 8) return NULL;
    if (n_bytes) *n_bytes = m->tbytes[which];
    return m->t[which];
}

/* vectors: 0 rms_att 1 rms_ffn 2 rms_final 3 post_att 4 post_ffn 5 rms_q 6 rms_k 7 q_bias 8 k_bias 9 v_bias */
const float* ob_model_vector(ob_model* m, int which, int64_t* n) {
    const brew_config* c = &m->c;
    const int64_t L = c->n_layers, dim = c->dim, hs = c->head_size;
    const int64_t qw = (int64_t)c->n_heads * hs, kvd = (int64_t)c->n_kv_heads * hs;
    const float* p = NULL;
    int64_t len = 0;
    switch (which) {
        case 0: p = m->rms_att; len = L * dim; break;
        case 1: p = m->rms_ffn; len = L * dim; break;
        case 2: p = m->rms_final; len = dim; break;
        case 3: p = m->post_att; len = L * dim; break;
        case 4: p = m->post_ffn; len = L * dim; break;
        case 5: p = m->rms_q; len = L * hs; break;
        case 6: p = m->rms_k; len = L * hs; break;
        case 7: p = m->q_bias; len = L * qw; break;
        case 8: p = m->k_bias; len = L * kvd; break;
        case 9: p = m->v_bias; len = L * kvd; break;
    }
    if (n) *n = p ? len : 0;
    return p;
}

void ob_model_reset(ob_model* m) {
    const brew_config* c = &m->c;
    const int64_t kvd = (int64_t)c->n_kv_heads * c->head_size;
    memset(m->kc, 0, (size_t)((int64_t)c->n_layers * c->seq_len * kvd) * sizeof(float));
    memset(m->vc, 0, (size_t)((int64_t)c->n_layers * c->seq_len * kvd) * sizeof(float));
}

/* AttentionEngine.attend (transformer/attention/AttentionEngine.java:50-106) */
typedef struct { ob_model* m; int layer, pos, start; int64_t layer_off; float inv_scale; } attn_ctx;

static void attn_task(void* vctx, int64_t h0, int64_t h1) {
    attn_ctx* a = (attn_ctx*)vctx;
    ob_model* m = a->m;
    const brew_config* c = &m->c;
    const int hs = c->head_size, kvd = c->n_kv_heads * hs;
    const int kv_mul = c->n_heads / c->n_kv_heads;
    for (int64_t h = h0; h < h1; h++) {
        const int qoff = (int)h * hs;
        float* att = m->att + h * c->seq_len;
        const int kvoff = (int)(h / kv_mul) * hs;
        for (int t = a->start; t <= a->pos; t++) {
            const float* kr = m->kc + a->layer_off + (int64_t)t * kvd + kvoff;
            float score = 0.0f;
            for (int i = 0; i < hs; i++) score += m->q[qoff + i] * kr[i];
            att[t] = score * a->inv_scale;
        }
        ob_softmax(att + a->start, a->pos - a->start + 1);
        float* xb = m->xb + qoff;
        for (int i = 0; i < hs; i++) xb[i] = 0.0f;
        for (int t = a->start; t <= a->pos; t++) {
            const float aw = att[t];
            const float* vr = m->vc + a->layer_off + (int64_t)t * kvd + kvoff;
            for (int i = 0; i < hs; i++) xb[i] += aw * vr[i];
        }
    }
}

static void accum(float* a, const float* b, int n) { for (int i = 0; i < n; i++) a[i] += b[i]; }

/* The six forward passes (model/llama2/Llama2Transformer.java:27-79,
 * model/qwen2/Qwen2Transformer.java:27-84, model/qwen3/Qwen3Transformer.java:27-85,
 * model/gemma3/Gemma3Transformer.java:27-92, model/gemma2/Gemma2Transformer.java:28-87,
 * model/smollm3/SmolLM3Transformer.java:28-81) share this body; the switches
 * mark where they differ.  Gemma2 is Gemma3 without the head-wise q/k norms
 * and with a global layer every 2nd layer; SmolLM3 is Llama2 without RoPE on
 * every 4th layer. */
int ob_model_forward(ob_model* m, int token, int pos, float* logits_out) {
    const brew_config* c = &m->c;
    const int dim = c->dim, hs = c->head_size, hid = c->hidden_dim;
    const int qw = c->n_heads * hs, kvd = c->n_kv_heads * hs;
    const int arch = c->arch;
    const int gemma = arch == BREW_ARCH_GEMMA3 || arch == BREW_ARCH_GEMMA2;
    const int interleaved = arch == BREW_ARCH_LLAMA || arch == BREW_ARCH_SMOLLM3;
    if (token < 0 || token >= c->vocab_size || pos < 0 || pos >= c->seq_len) return -1;

    ob_dequantize(c->type_embed, m->t[OB_W_EMBED], (int64_t)token * dim, dim, m->x);
    if (gemma) {                                          /* Kernels.scaleEmbeddings */
        const float s = (float)sqrt((double)dim);
        for (int i = 0; i < dim; i++) m->x[i] *= s;
    }
    const float inv_scale = 1.0f / (float)sqrt((double)hs);  /* AttentionPattern.java:8-10 */
    for (int l = 0; l < c->n_layers; l++) {
        const int64_t layer_off = (int64_t)l * c->seq_len * kvd;
        ob_rmsnorm(m->xb, m->x, m->rms_att + (int64_t)l * dim, dim, c->eps);
        ob_matvec(c->type_q, m->t[OB_W_Q], (int64_t)l * dim * qw, m->xb, m->q, dim, qw);
        ob_matvec(c->type_k, m->t[OB_W_K], (int64_t)l * dim * kvd, m->xb, m->k, dim, kvd);
        ob_matvec(c->type_v, m->t[OB_W_V], (int64_t)l * dim * kvd, m->xb, m->v, dim, kvd);
        if (arch == BREW_ARCH_QWEN2) {                    /* Qwen2Transformer.java:45-47 */
            accum(m->q, m->q_bias + (int64_t)l * qw, qw);
            accum(m->k, m->k_bias + (int64_t)l * kvd, kvd);
            accum(m->v, m->v_bias + (int64_t)l * kvd, kvd);
        }
        if (arch == BREW_ARCH_QWEN3 || arch == BREW_ARCH_GEMMA3) {
            ob_headwise_rmsnorm(m->q, m->rms_q + (int64_t)l * hs, c->n_heads, hs, c->eps);
            ob_headwise_rmsnorm(m->k, m->rms_k + (int64_t)l * hs, c->n_kv_heads, hs, c->eps);
        }
        int global = 1;
        if (arch == BREW_ARCH_GEMMA3) global = ((l + 1) % 6) == 0;       /* Gemma3AttentionPattern.java:10-12 */
        else if (arch == BREW_ARCH_GEMMA2) global = ((l + 1) % 2) == 0;  /* Gemma2AttentionPattern.java:10-12 */
        float base;
        if (c->rope_base > 0.0f) base = c->rope_base;
        else if (interleaved) base = 10000.0f;            /* Llama2Transformer.java:45, SmolLM3Transformer.java:47 */
        else if (gemma) base = global ? 1000000.0f : 10000.0f;  /* Gemma3Transformer.java:51, Gemma2Transformer.java:47 */
        else base = 1000000.0f;
        const float position = (float)pos * (c->rope_scale > 0.0f ? c->rope_scale : 1.0f);
        /* SmolLM3Transformer.java:35,46-47: no RoPE on every 4th layer */
        if (!(arch == BREW_ARCH_SMOLLM3 && (l + 1) % 4 == 0))
            ob_rope(m->q, m->k, c->n_heads, c->n_kv_heads, hs, base, position, interleaved);
        /* storeKeyValueInCache (AttentionEngine.java:34-38) */
        memcpy(m->kc + layer_off + (int64_t)pos * kvd, m->k, (size_t)kvd * sizeof(float));
        memcpy(m->vc + layer_off + (int64_t)pos * kvd, m->v, (size_t)kvd * sizeof(float));
        int start = 0;                                    /* Gemma3AttentionPattern.java:14-16 */
        if (gemma && !global) {
            start = pos - c->sliding_window + 1;
            if (start < 0) start = 0;
        }
        attn_ctx ac = {m, l, pos, start, layer_off, inv_scale};
        parallel_for(c->n_heads, 1, attn_task, &ac);
        ob_matvec(c->type_o, m->t[OB_W_O], (int64_t)l * dim * qw, m->xb, m->xb2, qw, dim);
        if (gemma) ob_rmsnorm(m->xb2, m->xb2, m->post_att + (int64_t)l * dim, dim, c->eps);
        accum(m->x, m->xb2, dim);
        ob_rmsnorm(m->xb, m->x, m->rms_ffn + (int64_t)l * dim, dim, c->eps);
        ob_matvec(c->type_gate, m->t[OB_W_GATE], (int64_t)l * dim * hid, m->xb, m->hb, dim, hid);
        ob_matvec(c->type_up, m->t[OB_W_UP], (int64_t)l * dim * hid, m->xb, m->hb2, dim, hid);
        ob_glu(m->hb, m->hb2, hid, gemma);
        ob_matvec(c->type_down, m->t[OB_W_DOWN], (int64_t)l * dim * hid, m->hb, m->xb, hid, dim);
        if (gemma) ob_rmsnorm(m->xb, m->xb, m->post_ffn + (int64_t)l * dim, dim, c->eps);
        accum(m->x, m->xb, dim);
    }
    ob_rmsnorm(m->x, m->x, m->rms_final, dim, c->eps);
    ob_matvec(type_of(c, OB_W_OUTPUT), m->t[OB_W_OUTPUT], 0, m->x, m->logits, dim, c->vocab_size);
    if (logits_out) memcpy(logits_out, m->logits, (size_t)c->vocab_size * sizeof(float));
    return 0;
}

/* GenericModelSession.generate / prefill / sampleNextToken with temperature
 * <= 0 (runtime/ModelRunner.java:115-206). */
int ob_generate(ob_model* m, const int32_t* prompt, int n_prompt, int max_new, int32_t* out, int* n_out) {
    const brew_config* c = &m->c;
    int position = 0;
    int pending = c->bos_token;                           /* reset(), :119 */
    ob_model_reset(m);
    for (int i = 0; i < n_prompt; i++) {                  /* prefill, :196-206 */
        if (position >= c->seq_len) return -2;            /* ensureContextAvailable */
        if (ob_model_forward(m, prompt[i], position, NULL) != 0) return -1;
        pending = prompt[i];
        position++;
    }
    const int remaining = c->seq_len - position;          /* :132-135 */
    const int limit = max_new <= 0 ? remaining : (max_new < remaining ? max_new : remaining);
    int count = 0;
    int eos = 0;
    while (!eos && count < limit) {                       /* :141-152 */
        if (ob_model_forward(m, pending, position, NULL) != 0) return -1;
        const int tok = ob_argmax(m->logits, c->vocab_size);
        out[count] = tok;
        pending = tok;
        position++;
        count++;
        if (tok == c->eos_token) eos = 1;
    }
    *n_out = count;
    return 0;
}
