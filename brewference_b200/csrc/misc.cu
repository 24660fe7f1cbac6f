// misc.cu — embedding + prep, dequantization, synthetic weights, argmax.
#include "brew_internal.cuh"
#include "misc.cuh"
#include "mv_device.cuh"
#include "prep.cuh"
#include "quant_device.cuh"

#include <algorithm>

namespace brew {

namespace {

__global__ void __launch_bounds__(256) embed_prep_kernel(int type, const uint8_t* embed, int vocab, int dim,
                                                          const int32_t* tokens, bool gemma, float* x,
                                                          const float* nw, float eps, uint8_t* prep, int batch,
                                                          unsigned int* err) {
    __shared__ float red[32];
    pdl_launch_dependents();
    pdl_wait();
    const int b = blockIdx.x;
    int tok = tokens[b];
    if (tok < 0 || tok >= vocab) {
        if (threadIdx.x == 0) atomicOr(err, BREW_DEVERR_BAD_TOKEN);
        tok = 0;
    }
    float* xb = x + (int64_t)b * dim;
    // Kernels.scaleEmbeddings: x *= (float)Math.sqrt(size)
    const float es = gemma ? (float)sqrt((double)dim) : 1.0f;
    for (int i = threadIdx.x; i < dim; i += blockDim.x) {
        float v = dequant_elem(type, embed, (int64_t)tok * dim + i);
        if (gemma) v = __fmul_rn(v, es);
        __stcg(&xb[i], v);
    }
    __threadfence();
    __syncthreads();
    prep_vector_cta(xb, dim, nw, eps, prep, prep_rec_bytes(batch), batch, b, red);
}

__global__ void dequant_kernel(int type, const uint8_t* w, int64_t off, int64_t n, float* out) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) out[i] = dequant_elem(type, w, off + i);
}

// ---- synthetic values: the device copy of the oracle's generator -------
__device__ __forceinline__ uint64_t mix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

__device__ __forceinline__ float synth_value(uint64_t key, uint64_t index, float sd) {
    int32_t s = 0;
#pragma unroll
    for (int j = 0; j < 3; j++) {
        const uint64_t h = mix64(key + 3ull * index + (uint64_t)j);
        s += (int32_t)(h & 0xFFFF) + (int32_t)((h >> 16) & 0xFFFF) + (int32_t)((h >> 32) & 0xFFFF) +
             (int32_t)((h >> 48) & 0xFFFF);
    }
    const int32_t num = 2 * s + 12 - 12 * 65536;
    return __fmul_rn(__fmul_rn((float)num, 7.62939453125e-06f), sd);
}

__device__ __forceinline__ uint64_t synth_key(uint64_t seed, uint32_t id) {
    return mix64(seed ^ ((uint64_t)id << 32) ^ 0x5851F42D4C957F2Dull);
}

// Block scales sit at even offsets of blocks whose sizes are even, so one
// 16-bit store writes them.
__device__ __forceinline__ void put_half(uint8_t* p, float f) {
    *reinterpret_cast<uint16_t*>(p) = __half_as_ushort(__float2half_rn(f));
}

__device__ __forceinline__ int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

// Quantizers: the same arithmetic, in the same order, as the oracle's
// quant_q8_0 / quant_q4_0 (gguf-py) and quant_q4_k / quant_q6_k.
__device__ void quant_block(int type, const float* x, uint8_t* out) {
    if (type == BREW_TYPE_Q8_0) {
        float amax = 0.0f;
        for (int i = 0; i < 32; i++) amax = fmaxf(amax, fabsf(x[i]));
        const float d = __fdiv_rn(amax, 127.0f);
        const float id = d == 0.0f ? 0.0f : __fdiv_rn(1.0f, d);
        put_half(out, d);
        for (int i = 0; i < 32; i++) out[2 + i] = (uint8_t)(int8_t)(int)roundf(__fmul_rn(x[i], id));
    } else if (type == BREW_TYPE_Q4_0) {
        int imax = 0;
        float amax = fabsf(x[0]);
        for (int i = 1; i < 32; i++) {
            const float a = fabsf(x[i]);
            if (a > amax) { amax = a; imax = i; }
        }
        const float d = __fdiv_rn(x[imax], -8.0f);
        const float id = d == 0.0f ? 0.0f : __fdiv_rn(1.0f, d);
        uint8_t q[32];
        for (int i = 0; i < 32; i++) q[i] = (uint8_t)clampi((int)truncf(__fadd_rn(__fmul_rn(x[i], id), 8.5f)), 0, 15);
        put_half(out, d);
        for (int j = 0; j < 16; j++) out[2 + j] = (uint8_t)(q[j] | (q[j + 16] << 4));
    } else if (type == BREW_TYPE_Q4_K) {
        float scale[8], minv[8];
        float maxscale = 0.0f, maxmin = 0.0f;
        for (int s = 0; s < 8; s++) {
            float mn = 0.0f, mx = x[32 * s];
            for (int i = 0; i < 32; i++) {
                const float v = x[32 * s + i];
                if (v < mn) mn = v;
                if (v > mx) mx = v;
            }
            if (mx < mn) mx = mn;
            scale[s] = __fdiv_rn(__fsub_rn(mx, mn), 15.0f);
            minv[s] = -mn;
            if (scale[s] > maxscale) maxscale = scale[s];
            if (minv[s] > maxmin) maxmin = minv[s];
        }
        put_half(out + 0, __fdiv_rn(maxscale, 63.0f));
        put_half(out + 2, __fdiv_rn(maxmin, 63.0f));
        const float df = ld_half(out), dminf = ld_half(out + 2);
        int sc[8], m[8];
        for (int s = 0; s < 8; s++) {
            sc[s] = df > 0.0f ? clampi((int)roundf(__fdiv_rn(scale[s], df)), 0, 63) : 0;
            m[s] = dminf > 0.0f ? clampi((int)roundf(__fdiv_rn(minv[s], dminf)), 0, 63) : 0;
        }
        uint8_t* sb = out + 4;
        for (int j = 0; j < 4; j++) {
            sb[j] = (uint8_t)(sc[j] | ((sc[j + 4] >> 4) << 6));
            sb[j + 4] = (uint8_t)(m[j] | ((m[j + 4] >> 4) << 6));
            sb[j + 8] = (uint8_t)((sc[j + 4] & 15) | ((m[j + 4] & 15) << 4));
        }
        uint8_t* qs = out + 16;
        for (int c = 0; c < 4; c++) {
            for (int i = 0; i < 32; i++) {
                int qv[2];
                for (int hsel = 0; hsel < 2; hsel++) {
                    const int s = 2 * c + hsel;
                    const float es = __fmul_rn(df, (float)sc[s]);
                    const float em = __fmul_rn(dminf, (float)m[s]);
                    qv[hsel] = es > 0.0f ? clampi((int)roundf(__fdiv_rn(__fadd_rn(x[32 * s + i], em), es)), 0, 15) : 0;
                }
                qs[32 * c + i] = (uint8_t)(qv[0] | (qv[1] << 4));
            }
        }
    } else if (type == BREW_TYPE_Q6_K) {
        float scale[16];
        float maxsc = 0.0f;
        for (int s = 0; s < 16; s++) {
            float amax = 0.0f;
            for (int i = 0; i < 16; i++) amax = fmaxf(amax, fabsf(x[16 * s + i]));
            scale[s] = __fdiv_rn(amax, 31.0f);
            if (scale[s] > maxsc) maxsc = scale[s];
        }
        put_half(out + 208, __fdiv_rn(maxsc, 127.0f));
        const float df = ld_half(out + 208);
        int sc[16];
        for (int s = 0; s < 16; s++) sc[s] = df > 0.0f ? clampi((int)roundf(__fdiv_rn(scale[s], df)), -128, 127) : 0;
        for (int s = 0; s < 16; s++) out[192 + s] = (uint8_t)(int8_t)sc[s];
        uint8_t u[256];
        for (int s = 0; s < 16; s++) {
            const float e = __fmul_rn(df, (float)sc[s]);
            for (int i = 0; i < 16; i++) {
                const int qi = e > 0.0f ? clampi((int)roundf(__fdiv_rn(x[16 * s + i], e)), -32, 31) : 0;
                u[16 * s + i] = (uint8_t)(qi + 32);
            }
        }
        for (int h = 0; h < 2; h++) {
            for (int l = 0; l < 32; l++) {
                const int u1 = u[128 * h + l], u2 = u[128 * h + 32 + l];
                const int u3 = u[128 * h + 64 + l], u4 = u[128 * h + 96 + l];
                out[64 * h + l] = (uint8_t)((u1 & 15) | ((u3 & 15) << 4));
                out[64 * h + 32 + l] = (uint8_t)((u2 & 15) | ((u4 & 15) << 4));
                out[128 + 32 * h + l] = (uint8_t)((u1 >> 4) | ((u2 >> 4) << 2) | ((u3 >> 4) << 4) | ((u4 >> 4) << 6));
            }
        }
    }
}

__global__ void synth_kernel(int type, uint64_t seed, uint32_t id, int64_t nblocks, int be, int bb, float sd,
                             uint8_t* out) {
    const int64_t blk = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (blk >= nblocks) return;
    const uint64_t key = synth_key(seed, id);
    float x[256];
    for (int i = 0; i < be; i++) x[i] = synth_value(key, (uint64_t)(blk * be + i), sd);
    quant_block(type, x, out + blk * bb);
}

__global__ void synth_f32_kernel(uint64_t seed, uint32_t id, int64_t n, float sd, float* out) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) out[i] = synth_value(synth_key(seed, id), (uint64_t)i, sd);
}

__global__ void fill_kernel(float* out, int64_t n, float v) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) out[i] = v;
}

// Kernels.argMax (transformer/math/Kernels.java:150-162): first index of the
// maximum, strict '>' so ties keep the lowest index (and a NaN is never the
// maximum).  CTA (chunk, sequence) reduces `chunk` logits to an orderable
// key (value, then lower index) and merges it into keys[b] with atomicMax;
// the last CTA of the sequence writes out[b] and leaves keys[b] and ctr[b]
// zero again.
constexpr int AM_THREADS = 256;

__global__ void __launch_bounds__(AM_THREADS) argmax_kernel(const float* logits, int ld, int n, int chunk,
                                                            unsigned long long* keys, int* ctr, int32_t* out) {
    __shared__ unsigned long long red[AM_THREADS / 32];
    __shared__ int s_last;
    pdl_launch_dependents();
    pdl_wait();
    const int b = blockIdx.y;
    const float* l = logits + (int64_t)b * ld;
    const int i0 = blockIdx.x * chunk, i1 = min(n, i0 + chunk);
    unsigned long long best = 0ull;
    for (int i = i0 + threadIdx.x; i < i1; i += AM_THREADS) {
        const float v = l[i];
        const unsigned long long k = v == v ? argmax_key(v, i) : 0ull;
        best = k > best ? k : best;
    }
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long v = __shfl_xor_sync(0xffffffffu, best, o);
        best = v > best ? v : best;
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (lane == 0) red[warp] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < AM_THREADS / 32; ++w) best = red[w] > best ? red[w] : best;
        atomicMax(&keys[b], best);
        __threadfence();
        s_last = atomicAdd(&ctr[b], 1) == (int)gridDim.x - 1;
        if (s_last) {
            __threadfence();
            const unsigned long long k = atomicExch(&keys[b], 0ull);
            ctr[b] = 0;
            out[b] = k == 0ull ? 0 : (int32_t)(0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull));
        }
    }
}

cudaLaunchConfig_t make_cfg(dim3 grid, dim3 block, size_t smem, cudaStream_t s, bool pdl, cudaLaunchAttribute* attr) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cfg;
}

}  // namespace

int embed_prep_launch(int type, const uint8_t* embed, int vocab, int dim, const int32_t* tokens, int batch,
                      bool gemma_scale, float* x, const float* norm_w, float eps, uint8_t* prep, unsigned int* err,
                      cudaStream_t stream, bool pdl) {
    BREW_CHECK(dim % 32 == 0, BREW_ERR_INVALID_ARG, "embed: dim %d", dim);
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = make_cfg(dim3(batch), dim3(256), 0, stream, pdl, attr);
    BREW_CUDA(cudaLaunchKernelEx(&cfg, embed_prep_kernel, type, embed, vocab, dim, tokens, gemma_scale, x, norm_w,
                                 eps, prep, batch, err));
    count_launch();
    return BREW_OK;
}

int dequant_launch(int type, const uint8_t* w, int64_t off, int64_t n, float* out, cudaStream_t stream) {
    if (n <= 0) return BREW_OK;
    const int64_t blocks = (n + 255) / 256;
    dequant_kernel<<<(unsigned)blocks, 256, 0, stream>>>(type, w, off, n, out);
    BREW_CUDA(cudaGetLastError());
    count_launch();
    return BREW_OK;
}

int synth_launch(int type, uint64_t seed, uint32_t id, int64_t n, float sd, uint8_t* out, cudaStream_t stream) {
    TypeInfo ti;
    BREW_CHECK(type_info(type, &ti) && ti.block_elems > 1, BREW_ERR_UNSUPPORTED, "synth: type %d", type);
    BREW_CHECK(n % ti.block_elems == 0, BREW_ERR_INVALID_ARG, "synth: %lld elements", (long long)n);
    const int64_t nb = n / ti.block_elems;
    const int threads = 128;
    synth_kernel<<<(unsigned)((nb + threads - 1) / threads), threads, 0, stream>>>(type, seed, id, nb, ti.block_elems,
                                                                                 ti.block_bytes, sd, out);
    BREW_CUDA(cudaGetLastError());
    count_launch();
    return BREW_OK;
}

int synth_f32_launch(uint64_t seed, uint32_t id, int64_t n, float sd, float* out, cudaStream_t stream) {
    if (n <= 0) return BREW_OK;
    synth_f32_kernel<<<(unsigned)((n + 255) / 256), 256, 0, stream>>>(seed, id, n, sd, out);
    BREW_CUDA(cudaGetLastError());
    count_launch();
    return BREW_OK;
}

int fill_f32_launch(float* out, int64_t n, float v, cudaStream_t stream) {
    if (n <= 0) return BREW_OK;
    fill_kernel<<<(unsigned)((n + 255) / 256), 256, 0, stream>>>(out, n, v);
    BREW_CUDA(cudaGetLastError());
    count_launch();
    return BREW_OK;
}

int argmax_launch(const float* logits, int ld, int n, int batch, unsigned long long* keys, int* ctr, int32_t* out,
                  cudaStream_t stream, bool pdl) {
    constexpr int chunk = 16 * AM_THREADS;   // logits per CTA
    const int chunks = std::max(1, (n + chunk - 1) / chunk);
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = make_cfg(dim3(chunks, batch), dim3(AM_THREADS), 0, stream, pdl, attr);
    BREW_CUDA(cudaLaunchKernelEx(&cfg, argmax_kernel, logits, ld, n, chunk, keys, ctr, out));
    count_launch();
    return BREW_OK;
}

}  // namespace brew

// ---------------------------------------------------------------------------
// Failure-detection self-test: the two bounded waits every pipeline of this
// library uses (an mbarrier phase, the grid barrier's counter) run against
// events that never happen and must give up after `limit_ns`, record the
// timeout in the device error word and return, leaving the context usable.
// ---------------------------------------------------------------------------
namespace brew {
namespace {

__device__ unsigned long long g_selftest_counter;   // nothing ever adds to it

__global__ void selftest_wait_kernel(unsigned int* err, uint64_t limit_ns, int* status) {
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);   // one arrival completes the phase; none comes
        fence_mbar_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        const bool a = mbar_wait_bounded(&bar, 0, err, BREW_DEVERR_TIMEOUT_FULL, limit_ns);
        const bool b = wait_counter_bounded(&g_selftest_counter, 1ull, nullptr, limit_ns);
        if (!b) atomicOr(err, BREW_DEVERR_TIMEOUT_EMPTY);
        status[0] = a ? 1 : 0;
        status[1] = b ? 1 : 0;
    }
}

}  // namespace
}  // namespace brew

using namespace brew;

extern "C" int brew_selftest_wait_timeout(int64_t limit_ns, int32_t* waits_ended) {
    BREW_CHECK(limit_ns > 0 && limit_ns <= 1000000000LL, BREW_ERR_INVALID_ARG, "limit %lld ns (1 ns .. 1 s)",
               (long long)limit_ns);
    int rc = ensure_init();
    if (rc) return rc;
    int* st = nullptr;
    BREW_CUDA(cudaMalloc(&st, 2 * sizeof(int)));
    cudaStream_t s = ctx().stream;
    selftest_wait_kernel<<<1, 32, 0, s>>>(ctx().err_word, (uint64_t)limit_ns, st);
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    int h[2] = {-1, -1};
    if (e == cudaSuccess) e = cudaMemcpy(h, st, sizeof(h), cudaMemcpyDeviceToHost);
    cudaFree(st);
    if (e != cudaSuccess) return cuda_error(e, "selftest_wait_kernel");
    count_launch();
    if (waits_ended) *waits_ended = (h[0] == 0 ? 1 : 0) + (h[1] == 0 ? 1 : 0);
    return check_device_error("brew_selftest_wait_timeout");
}
