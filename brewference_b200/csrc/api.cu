// api.cu — C ABI: errors, device context, packed weight tensors, Linear.matmul.
#include "brew_internal.cuh"

#include <atomic>
#include <cstdarg>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>

__device__ unsigned int g_brew_device_error;

namespace brew {

namespace {
thread_local std::string t_last_error;
std::atomic<int64_t> g_launches{0};
Context g_ctx;
std::mutex g_mu;
}  // namespace

int set_error(int code, const char* fmt, ...) {
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    t_last_error = buf;
    return code;
}

int cuda_error(cudaError_t e, const char* what) {
    return set_error(BREW_ERR_CUDA, "CUDA error %d (%s) in %s", (int)e, cudaGetErrorString(e), what);
}

void count_launch(int n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

Context& ctx() { return g_ctx; }
std::mutex& api_mutex() { return g_mu; }

unsigned int* device_error_word() { return g_ctx.err_word; }

int check_device_error(const char* where) {
    if (!g_ctx.err_word) return BREW_OK;
    unsigned int v = 0;
    BREW_CUDA(cudaMemcpyFromSymbol(&v, g_brew_device_error, sizeof(v)));
    if (v == 0) return BREW_OK;
    const unsigned int zero = 0;
    cudaMemcpyToSymbol(g_brew_device_error, &zero, sizeof(zero));
    if (v & (BREW_DEVERR_TIMEOUT_FULL | BREW_DEVERR_TIMEOUT_EMPTY))
        return set_error(BREW_ERR_TIMEOUT, "%s: a bounded device wait timed out (flags 0x%x)", where, v);
    if (v & BREW_DEVERR_BAD_TOKEN) return set_error(BREW_ERR_INVALID_ARG, "%s: token id out of range", where);
    return set_error(BREW_ERR_OUT_OF_BOUNDS, "%s: device index check failed (flags 0x%x)", where, v);
}

int ensure_init() {
    if (g_ctx.initialized) {
        BREW_CUDA(cudaSetDevice(g_ctx.device));
        return BREW_OK;
    }
    return brew_init(-1);
}

int Scratch::reserve(size_t need_bytes) {
    if (need_bytes <= bytes) return BREW_OK;
    if (ptr) cudaFree(ptr);
    ptr = nullptr;
    bytes = 0;
    BREW_CUDA(cudaMalloc(&ptr, need_bytes));
    // cudaMemset runs on the legacy default stream, which does not order
    // against the library's non-blocking streams: wait for it, or it could
    // land after the kernels that use the buffer next
    BREW_CUDA(cudaMemset(ptr, 0, need_bytes));
    BREW_CUDA(cudaStreamSynchronize(0));
    bytes = need_bytes;
    return BREW_OK;
}

// ---- generic GPU matvec for the K-quants ---------------------------------
// One warp per output row; each 32-element group is dequantized with the
// GGML formulas and summed in fp32 (the oracle's K-quant order per group).
namespace {
__device__ __forceinline__ float ldh(const uint8_t* p) { return half_bits_to_float((uint16_t)(p[0] | (p[1] << 8))); }

// One warp per output row for up to MAXB vectors: each weight is dequantized
// once and multiplied into every vector's sum (the per-vector summation
// order is the same for any batch).
template <int MAXB>
__global__ void kquant_matvec_kernel(int type, const uint8_t* w, int64_t row_bytes, const float* x, int ldx, int K,
                                     int N, float* y, int ldy, int batch) {
    pdl_launch_dependents();
    pdl_wait();
    const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    const int b0 = blockIdx.y * MAXB;
    if (row >= N) return;
    const uint8_t* wr = w + (int64_t)row * row_bytes;
    float acc[MAXB];
#pragma unroll
    for (int b = 0; b < MAXB; ++b) acc[b] = 0.0f;
    for (int k0 = 0; k0 < K; k0 += 256) {
        const int s = lane >> 2;  // 8 sub-blocks of 32 per super-block, 4 lanes each
        const uint8_t* blk = wr + (int64_t)(k0 / 256) * (type == BREW_TYPE_Q4_K ? 144 : 210);
        float part[MAXB];
#pragma unroll
        for (int b = 0; b < MAXB; ++b) part[b] = 0.0f;
        for (int i = (lane & 3) * 8; i < (lane & 3) * 8 + 8; ++i) {
            const int r = s * 32 + i;
            float wv;
            if (type == BREW_TYPE_Q4_K) {
                const uint8_t* sb = blk + 4;
                int sc, m;
                if (s < 4) { sc = sb[s] & 63; m = sb[s + 4] & 63; }
                else { sc = (sb[s + 4] & 0xF) | ((sb[s - 4] >> 6) << 4); m = (sb[s + 4] >> 4) | ((sb[s] >> 6) << 4); }
                const uint8_t qb = blk[16 + 32 * (s / 2) + i];
                const int q = (s & 1) ? (qb >> 4) : (qb & 15);
                wv = __fsub_rn(__fmul_rn(__fmul_rn(ldh(blk), (float)sc), (float)q), __fmul_rn(ldh(blk + 2), (float)m));
            } else {
                const int h = r / 128, rr = r % 128, grp = rr / 32, l = rr % 32;
                const int lq = blk[64 * h + (grp & 1) * 32 + l];
                const int low = grp < 2 ? (lq & 15) : (lq >> 4);
                const int high = (blk[128 + 32 * h + l] >> (2 * grp)) & 3;
                const int q = (low | (high << 4)) - 32;
                wv = __fmul_rn(__fmul_rn(ldh(blk + 208), (float)(int8_t)blk[192 + r / 16]), (float)q);
            }
#pragma unroll
            for (int b = 0; b < MAXB; ++b)
                if (b0 + b < batch) part[b] += wv * x[(int64_t)(b0 + b) * ldx + k0 + r];
        }
#pragma unroll
        for (int b = 0; b < MAXB; ++b) acc[b] += part[b];
    }
#pragma unroll
    for (int b = 0; b < MAXB; ++b) {
        const float v = warp_sum(acc[b]);
        if (lane == 0 && b0 + b < batch) y[(int64_t)(b0 + b) * ldy + row] = v;
    }
}
}  // namespace

int kquant_matvec_launch(int type, const uint8_t* w, int64_t row_bytes, const float* x, int ldx, int K, int N, float* y,
                         int ldy, int batch, cudaStream_t stream, bool pdl) {
    BREW_CHECK(K % 256 == 0, BREW_ERR_INVALID_ARG, "K-quant matvec: K=%d not a multiple of 256", K);
    const int maxb = batch <= 1 ? 1 : (batch <= 4 ? 4 : 16);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((N + 7) / 8, (batch + maxb - 1) / maxb);
    cfg.blockDim = dim3(256);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    if (maxb == 1)
        BREW_CUDA(cudaLaunchKernelEx(&cfg, kquant_matvec_kernel<1>, type, w, row_bytes, x, ldx, K, N, y, ldy, batch));
    else if (maxb == 4)
        BREW_CUDA(cudaLaunchKernelEx(&cfg, kquant_matvec_kernel<4>, type, w, row_bytes, x, ldx, K, N, y, ldy, batch));
    else
        BREW_CUDA(cudaLaunchKernelEx(&cfg, kquant_matvec_kernel<16>, type, w, row_bytes, x, ldx, K, N, y, ldy, batch));
    count_launch();
    return BREW_OK;
}

// Runs one matvec (any supported type) on device buffers: the shared core of
// brew_matmul / brew_matmul_dev.  The prep records of x live in a growable
// scratch buffer of the context.
int run_matvec(brew_tensor t, int64_t weights_offset, const float* x_dev, int K, int N, float* y_dev, int batch,
               cudaStream_t stream) {
    TypeInfo ti;
    type_info(t->type, &ti);
    const int64_t row_bytes = (int64_t)K / ti.block_elems * ti.block_bytes;
    const uint8_t* w = t->d + weights_offset / ti.block_elems * ti.block_bytes;
    if (t->type == BREW_TYPE_Q4_K || t->type == BREW_TYPE_Q6_K)
        return kquant_matvec_launch(t->type, w, row_bytes, x_dev, K, K, N, y_dev, N, batch, stream, false);
    Context& c = g_ctx;
    for (int b0 = 0; b0 < batch; b0 += MV_MAX_BATCH) {
        const int nb = std::min(MV_MAX_BATCH, batch - b0);
        const size_t prep_bytes = (size_t)(K / 32) * prep_rec_bytes(nb);
        int rc = c.mv_scratch.reserve(prep_bytes + 256);
        if (rc) return rc;
        uint8_t* prep = static_cast<uint8_t*>(c.mv_scratch.ptr);
        rc = prep_launch(x_dev + (int64_t)b0 * K, K, K, nb, nullptr, 0.0f, prep, stream, false);
        if (rc) return rc;
        rc = launch_prepared(t, w, row_bytes, prep, K, N, y_dev + (int64_t)b0 * N, nb, stream);
        if (rc) return rc;
    }
    return BREW_OK;
}

int launch_prepared(brew_tensor t, const uint8_t* w, int64_t row_bytes, const uint8_t* prep, int K, int N, float* y,
                    int nb, cudaStream_t stream) {
    MvParams p = {};
    p.nseg = 1;
    p.seg[0].w = w;
    p.seg[0].y = y;
    p.seg[0].rows = N;
    p.type = t->type;
    p.K = K;
    p.row_bytes = row_bytes;
    p.batch = nb;
    p.ldy = N;
    p.epi = MV_EPI_STORE;
    p.prep = prep;
    p.post = MV_POST_NONE;
    p.err = g_ctx.err_word;
    return mv_launch(p, stream, false);
}

int run_matvec_prepared(brew_tensor t, int64_t weights_offset, const uint8_t* prep, int K, int N, float* y, int batch,
                        cudaStream_t stream) {
    TypeInfo ti;
    type_info(t->type, &ti);
    const int64_t row_bytes = (int64_t)K / ti.block_elems * ti.block_bytes;
    const uint8_t* w = t->d + weights_offset / ti.block_elems * ti.block_bytes;
    return launch_prepared(t, w, row_bytes, prep, K, N, y, batch, stream);
}

}  // namespace brew

using namespace brew;

extern "C" {

int brew_last_error(char* buf, size_t n) {
    const std::string& s = t_last_error;
    if (buf && n) {
        const size_t m = std::min(n - 1, s.size());
        memcpy(buf, s.data(), m);
        buf[m] = 0;
    }
    return (int)s.size();
}

const char* brew_version(void) { return "brewference_b200 0.1.0 (sm_100a)"; }

int64_t brew_kernel_launches(void) { return g_launches.load(); }

int brew_init(int device) {
    std::lock_guard<std::mutex> lk(g_mu);
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess || n == 0) {
        cudaGetLastError();
        return set_error(BREW_ERR_NO_DEVICE, "no CUDA device visible (%s); this library has no CPU path",
                         e == cudaSuccess ? "0 devices" : cudaGetErrorString(e));
    }
    if (device < 0) {
        const char* env = getenv("LOCAL_RANK");
        device = env ? atoi(env) % n : 0;
    }
    BREW_CHECK(device < n, BREW_ERR_INVALID_ARG, "device %d of %d", device, n);
    if (g_ctx.initialized && g_ctx.device == device) return BREW_OK;
    BREW_CUDA(cudaSetDevice(device));
    cudaDeviceProp prop;
    BREW_CUDA(cudaGetDeviceProperties(&prop, device));
    BREW_CHECK(prop.major == 10, BREW_ERR_UNSUPPORTED, "device %d is sm_%d%d; this library is built for sm_100a",
               device, prop.major, prop.minor);
    g_ctx.device = device;
    BREW_CUDA(cudaStreamCreateWithFlags(&g_ctx.stream, cudaStreamNonBlocking));
    void* p = nullptr;
    BREW_CUDA(cudaGetSymbolAddress(&p, g_brew_device_error));
    g_ctx.err_word = static_cast<unsigned int*>(p);
    const unsigned int zero = 0;
    BREW_CUDA(cudaMemcpyToSymbol(g_brew_device_error, &zero, sizeof(zero)));
    g_ctx.initialized = true;
    return BREW_OK;
}

int64_t brew_type_bytes(int type, int64_t n) {
    TypeInfo ti;
    if (!type_info(type, &ti) || n < 0 || n % ti.block_elems) return -1;
    return n / ti.block_elems * ti.block_bytes;
}

int brew_type_block(int type, int* be, int* bb) {
    TypeInfo ti;
    if (!type_info(type, &ti)) return set_error(BREW_ERR_UNSUPPORTED, "unknown GGML type %d", type);
    if (be) *be = ti.block_elems;
    if (bb) *bb = ti.block_bytes;
    return BREW_OK;
}

int brew_tensor_alloc(int type, int64_t n, brew_tensor* out) {
    BREW_CHECK(out, BREW_ERR_INVALID_ARG, "out is null");
    *out = nullptr;
    TypeInfo ti;
    BREW_CHECK(type_info(type, &ti), BREW_ERR_UNSUPPORTED, "unsupported GGML type %d", type);
    BREW_CHECK(n > 0 && n % ti.block_elems == 0, BREW_ERR_IO,
               "tensor has %lld elements, not a multiple of the block size %d", (long long)n, ti.block_elems);
    int rc = ensure_init();
    if (rc) return rc;
    brew_tensor t = new brew_tensor_s();
    t->type = type;
    t->n = n;
    t->bytes = n / ti.block_elems * ti.block_bytes;
    // +256: bulk copies are rounded out to 16-byte bounds
    cudaError_t e = cudaMalloc(&t->d, (size_t)t->bytes + 256);
    if (e != cudaSuccess) {
        delete t;
        return cuda_error(e, "cudaMalloc(tensor)");
    }
    cudaMemset(t->d + t->bytes, 0, 256);
    cudaStreamSynchronize(0);   // legacy-stream memset: finish it before any non-blocking stream uses t
    *out = t;
    return BREW_OK;
}

int brew_tensor_write(brew_tensor t, int64_t off, const void* bytes, int64_t n) {
    BREW_CHECK(t && bytes, BREW_ERR_INVALID_ARG, "null tensor or bytes");
    TypeInfo ti;
    type_info(t->type, &ti);
    BREW_CHECK(off >= 0 && n >= 0 && off % ti.block_elems == 0 && n % ti.block_elems == 0, BREW_ERR_INVALID_ARG,
               "write at %lld of %lld elements: not whole blocks", (long long)off, (long long)n);
    BREW_CHECK(off + n <= t->n, BREW_ERR_OUT_OF_BOUNDS, "write past the tensor end");
    int rc = ensure_init();
    if (rc) return rc;
    // a pageable host->device cudaMemcpy may return before its DMA has
    // landed, and it runs on the legacy stream, which the library's
    // non-blocking streams do not wait for: wait for it here
    BREW_CUDA(cudaMemcpy(t->d + off / ti.block_elems * ti.block_bytes, bytes, (size_t)(n / ti.block_elems * ti.block_bytes),
                         cudaMemcpyHostToDevice));
    BREW_CUDA(cudaStreamSynchronize(0));
    return BREW_OK;
}

int brew_tensor_upload(int type, const void* bytes, int64_t n, brew_tensor* out) {
    BREW_CHECK(bytes, BREW_ERR_INVALID_ARG, "bytes is null");
    int rc = brew_tensor_alloc(type, n, out);
    if (rc) return rc;
    rc = brew_tensor_write(*out, 0, bytes, n);
    if (rc) {
        brew_tensor_free(*out);
        *out = nullptr;
    }
    return rc;
}

int brew_tensor_free(brew_tensor t) {
    if (!t) return BREW_OK;
    if (t->owned) cudaFree(t->d);
    delete t;
    return BREW_OK;
}

int brew_tensor_info(brew_tensor t, int* type, int64_t* n, int64_t* nb) {
    BREW_CHECK(t, BREW_ERR_INVALID_ARG, "null tensor");
    if (type) *type = t->type;
    if (n) *n = t->n;
    if (nb) *nb = t->bytes;
    return BREW_OK;
}

int brew_tensor_read(brew_tensor t, int64_t off, int64_t n, void* bytes) {
    BREW_CHECK(t && bytes, BREW_ERR_INVALID_ARG, "null tensor or bytes");
    TypeInfo ti;
    type_info(t->type, &ti);
    BREW_CHECK(off >= 0 && n >= 0 && off % ti.block_elems == 0 && n % ti.block_elems == 0, BREW_ERR_INVALID_ARG,
               "read at %lld of %lld elements: not whole blocks", (long long)off, (long long)n);
    BREW_CHECK(off + n <= t->n, BREW_ERR_OUT_OF_BOUNDS, "read past the tensor end");
    int rc = ensure_init();
    if (rc) return rc;
    // kernels on non-blocking streams may still be writing t: the legacy
    // stream's copy does not wait for them
    BREW_CUDA(cudaDeviceSynchronize());
    BREW_CUDA(cudaMemcpy(bytes, t->d + off / ti.block_elems * ti.block_bytes, (size_t)(n / ti.block_elems * ti.block_bytes),
                         cudaMemcpyDeviceToHost));
    return BREW_OK;
}

int brew_tensor_device_ptr(brew_tensor t, void** p) {
    BREW_CHECK(t && p, BREW_ERR_INVALID_ARG, "null argument");
    *p = t->d;
    return BREW_OK;
}

int brew_dequantize_row_dev(brew_tensor t, int64_t off, int64_t n, float* out, void* stream) {
    BREW_CHECK(t && out, BREW_ERR_INVALID_ARG, "null argument");
    BREW_CHECK(off >= 0 && n >= 0 && off + n <= t->n, BREW_ERR_OUT_OF_BOUNDS, "dequantize [%lld, +%lld) of %lld",
               (long long)off, (long long)n, (long long)t->n);
    int rc = ensure_init();
    if (rc) return rc;
    return dequant_launch(t->type, t->d, off, n, out, static_cast<cudaStream_t>(stream));
}

int brew_dequantize_row(brew_tensor t, int64_t off, int64_t n, float* out) {
    BREW_CHECK(t && out, BREW_ERR_INVALID_ARG, "null argument");
    int rc = ensure_init();
    if (rc) return rc;
    std::lock_guard<std::mutex> lk(g_mu);
    Context& c = g_ctx;
    rc = c.io_scratch.reserve((size_t)n * sizeof(float) + 256);
    if (rc) return rc;
    float* d = static_cast<float*>(c.io_scratch.ptr);
    rc = brew_dequantize_row_dev(t, off, n, d, c.stream);
    if (rc) return rc;
    BREW_CUDA(cudaMemcpyAsync(out, d, (size_t)n * sizeof(float), cudaMemcpyDeviceToHost, c.stream));
    BREW_CUDA(cudaStreamSynchronize(c.stream));
    return BREW_OK;
}

static int matmul_checks(const void* output, const void* input, brew_tensor w, int64_t off, int32_t K, int32_t N) {
    // Linear.validateMatmulArguments (transformer/math/Linear.java:67-74)
    BREW_CHECK(w, BREW_ERR_INVALID_ARG, "Weight block cannot be null");
    BREW_CHECK(w->d, BREW_ERR_INVALID_ARG, "Weight block scales and data must be initialized");
    BREW_CHECK(input && output, BREW_ERR_INVALID_ARG, "Input and output arrays cannot be null");
    TypeInfo ti;
    type_info(w->type, &ti);
    BREW_CHECK(is_quant_matrix_type(w->type), BREW_ERR_UNSUPPORTED, "matmul on GGML type %d", w->type);
    BREW_CHECK(K > 0 && K % ti.block_elems == 0, BREW_ERR_INVALID_ARG,
               "inputSize %d is not a whole number of %d-element blocks", K, ti.block_elems);
    BREW_CHECK(N >= 0 && off >= 0 && off % ti.block_elems == 0, BREW_ERR_INVALID_ARG,
               "weightsOffset %lld is not at a block boundary", (long long)off);
    // Linear.java:46-50: the last block read must lie inside the tensor
    BREW_CHECK(off + (int64_t)N * K <= w->n, BREW_ERR_OUT_OF_BOUNDS,
               "matmul scale index out of bounds (wOffset=%lld, n=%d, d=%d)", (long long)off, K, N);
    return BREW_OK;
}

int64_t brew_prep_bytes(int32_t K, int32_t batch) {
    if (K <= 0 || K % 32 || batch < 1 || batch > MV_MAX_BATCH) return -1;
    return (int64_t)(K / 32) * prep_rec_bytes(batch);
}

int brew_prepare_input_dev(const float* x, int32_t K, int32_t batch, void* prep, void* stream) {
    BREW_CHECK(x && prep, BREW_ERR_INVALID_ARG, "null argument");
    BREW_CHECK(K > 0 && K % 32 == 0, BREW_ERR_INVALID_ARG, "inputSize %d is not a multiple of 32", K);
    BREW_CHECK(batch >= 1 && batch <= MV_MAX_BATCH, BREW_ERR_INVALID_ARG, "batch %d", batch);
    BREW_CHECK(((uintptr_t)prep & 15) == 0, BREW_ERR_INVALID_ARG, "prep buffer not 16-byte aligned");
    int rc = ensure_init();
    if (rc) return rc;
    return prep_launch(x, K, K, batch, nullptr, 0.0f, static_cast<uint8_t*>(prep), static_cast<cudaStream_t>(stream),
                       false);
}

int brew_matmul_prepared_dev(float* y, const void* prep, brew_tensor w, int64_t off, int32_t K, int32_t N,
                             int32_t batch, void* stream) {
    int rc = matmul_checks(y, prep, w, off, K, N);
    if (rc) return rc;
    BREW_CHECK(w->type == BREW_TYPE_Q8_0 || w->type == BREW_TYPE_Q4_0, BREW_ERR_UNSUPPORTED,
               "prepared matmul needs Q8_0 or Q4_0 weights");
    BREW_CHECK(batch >= 1 && batch <= MV_MAX_BATCH, BREW_ERR_INVALID_ARG, "batch %d", batch);
    BREW_CHECK(((uintptr_t)prep & 15) == 0, BREW_ERR_INVALID_ARG, "prep buffer not 16-byte aligned");
    if (N == 0) return BREW_OK;
    if ((rc = ensure_init())) return rc;
    std::lock_guard<std::mutex> lk(g_mu);
    return run_matvec_prepared(w, off, static_cast<const uint8_t*>(prep), K, N, y, batch,
                               static_cast<cudaStream_t>(stream));
}

int brew_matmul_dev(float* y, const float* x, brew_tensor w, int64_t off, int32_t K, int32_t N, int32_t batch,
                    void* stream) {
    int rc = matmul_checks(y, x, w, off, K, N);
    if (rc) return rc;
    BREW_CHECK(batch >= 1, BREW_ERR_INVALID_ARG, "batch %d", batch);
    if (N == 0) return BREW_OK;
    rc = ensure_init();
    if (rc) return rc;
    std::lock_guard<std::mutex> lk(g_mu);
    return run_matvec(w, off, x, K, N, y, batch, static_cast<cudaStream_t>(stream));
}

int brew_matmul(float* output, const float* input, brew_tensor w, int64_t off, int32_t K, int32_t N) {
    int rc = matmul_checks(output, input, w, off, K, N);
    if (rc) return rc;
    if (N == 0) return BREW_OK;
    rc = ensure_init();
    if (rc) return rc;
    std::lock_guard<std::mutex> lk(g_mu);
    Context& c = g_ctx;
    const size_t xb = ((size_t)K * sizeof(float) + 255) & ~size_t(255);
    rc = c.io_scratch.reserve(xb + (size_t)N * sizeof(float));
    if (rc) return rc;
    float* dx = static_cast<float*>(c.io_scratch.ptr);
    float* dy = reinterpret_cast<float*>(static_cast<uint8_t*>(c.io_scratch.ptr) + xb);
    BREW_CUDA(cudaMemcpyAsync(dx, input, (size_t)K * sizeof(float), cudaMemcpyHostToDevice, c.stream));
    rc = run_matvec(w, off, dx, K, N, dy, 1, c.stream);
    if (rc) return rc;
    BREW_CUDA(cudaMemcpyAsync(output, dy, (size_t)N * sizeof(float), cudaMemcpyDeviceToHost, c.stream));
    BREW_CUDA(cudaStreamSynchronize(c.stream));
    return check_device_error("brew_matmul");
}

}  // extern "C"
