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

// ---- GPU matvec for the K-quants -----------------------------------------
// Q4_K / Q6_K rows (super-blocks of 256 elements) times up to 16 fp32
// vectors per launch, on CUDA cores.  Each weight is dequantized once, with
// the GGML formulas and their fp32 rounding per element
// (d*sc*q - dmin*m for Q4_K, d*scale*(q - 32) for Q6_K), and multiplied into
// every vector's sum.
//
// A warp owns RW rows (4, or 2 with 16 vectors, whose accumulators would
// not fit the registers of two CTAs per SM otherwise) and walks their super-blocks; lane l owns 4 bytes
// of each super-block's quant array (so a warp's weight reads are one
// coalesced 128-byte run per row) and the 8 elements they hold:
//   Q4_K  qs bytes 4l .. 4l+3: elements 4 (l % 8) + 0..3 of sub-block
//         2 (l / 8) (low nibbles) and of the next sub-block (high nibbles);
//   Q6_K  ql bytes 4l .. 4l+3: elements 128 h + 32 g + 4 (l % 8) + 0..3
//         (h = l / 16, g = (l / 8) % 2; low nibbles, high bits of qh at 2g)
//         and the same + 64 (high nibbles, qh bits at 2g + 4).
// The vectors' matching 4-element pieces are read as float4 (L1-cached:
// every warp of the CTA reads them), and the lanes' partial sums meet in a
// warp reduction at the end.
namespace {
constexpr int KQ_WARPS = 8;       // warps per CTA
constexpr int KQ_MAXV = 16;       // vectors per launch

__device__ __forceinline__ uint32_t byte_of(uint32_t w, int i) { return (w >> (8 * i)) & 0xFFu; }

// 6-bit scale and min of Q4_K sub-block s from the 12 scale bytes (held in
// the header words h1 = bytes 4..7, h2 = 8..11, h3 = 12..15 of the block):
// GGML's get_scale_min_k4.
__device__ __forceinline__ void q4k_sm(uint32_t h1, uint32_t h2, uint32_t h3, int s, int& sc, int& m) {
    auto sb = [&](int i) -> int { return (int)byte_of(i < 4 ? h1 : (i < 8 ? h2 : h3), i & 3); };
    if (s < 4) {
        sc = sb(s) & 63;
        m = sb(s + 4) & 63;
    } else {
        sc = (sb(s + 4) & 0xF) | ((sb(s - 4) >> 6) << 4);
        m = (sb(s + 4) >> 4) | ((sb(s) >> 6) << 4);
    }
}

__device__ __forceinline__ uint32_t ld_u16(const uint8_t* p) { return *reinterpret_cast<const uint16_t*>(p); }

// The raw bytes of lane l's share of one super-block of a row (loaded one
// super-block ahead of their use, so the weight stream's latency overlaps
// the multiplication):
//   Q4_K  hd = d, dmin, scales[12]; q = the lane's 4 quant bytes
//   Q6_K  q = 4 ql bytes, h = the 4 qh bytes over them, hd.x = the two
//         scale bytes (low, high set) and d
struct KqRaw {
    uint4 hd;
    uint32_t q, h;
};

template <int TYPE>
__device__ __forceinline__ void kq_load(const uint8_t* blk, int lane, KqRaw& r) {
    if (TYPE == BREW_TYPE_Q4_K) {
        r.hd = __ldg(reinterpret_cast<const uint4*>(blk));
        r.q = __ldg(reinterpret_cast<const uint32_t*>(blk + 16 + 4 * lane));
    } else {
        // 210-byte super-blocks are only 2-byte aligned: 16-bit loads
        const int h = lane >> 4, g = (lane >> 3) & 1, e0 = 4 * (lane & 7);
        const int rlo = 128 * h + 32 * g + e0;
        r.q = ld_u16(blk + 4 * lane) | (ld_u16(blk + 4 * lane + 2) << 16);
        const uint8_t* qhp = blk + 128 + 32 * h + e0;
        r.h = ld_u16(qhp) | (ld_u16(qhp + 2) << 16);
        r.hd.x = (uint32_t)blk[192 + (rlo >> 4)] | ((uint32_t)blk[192 + ((rlo + 64) >> 4)] << 8) |
                 (ld_u16(blk + 208) << 16);
    }
}

// Dequantized elements of lane l: w[0..3] at super-block offset lo, w[4..7]
// at hi (kq_offsets).
template <int TYPE>
__device__ __forceinline__ void kq_decode(const KqRaw& r, int lane, float (&w)[8]) {
    if (TYPE == BREW_TYPE_Q4_K) {
        const float d = half_bits_to_float((uint16_t)(r.hd.x & 0xFFFFu));
        const float dmin = half_bits_to_float((uint16_t)(r.hd.x >> 16));
        const int s0 = 2 * (lane >> 3);
        int sc0, m0, sc1, m1;
        q4k_sm(r.hd.y, r.hd.z, r.hd.w, s0, sc0, m0);
        q4k_sm(r.hd.y, r.hd.z, r.hd.w, s0 + 1, sc1, m1);
        const float D0 = __fmul_rn(d, (float)sc0), M0 = __fmul_rn(dmin, (float)m0);
        const float D1 = __fmul_rn(d, (float)sc1), M1 = __fmul_rn(dmin, (float)m1);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            w[j] = __fsub_rn(__fmul_rn(D0, (float)((r.q >> (8 * j)) & 15u)), M0);
            w[4 + j] = __fsub_rn(__fmul_rn(D1, (float)((r.q >> (8 * j + 4)) & 15u)), M1);
        }
    } else {
        const int g = (lane >> 3) & 1;
        const float d = half_bits_to_float((uint16_t)(r.hd.x >> 16));
        const float Dlo = __fmul_rn(d, (float)(int8_t)(r.hd.x & 0xFFu));
        const float Dhi = __fmul_rn(d, (float)(int8_t)((r.hd.x >> 8) & 0xFFu));
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint32_t qb = byte_of(r.q, j), hb = byte_of(r.h, j);
            const int qlo = (int)((qb & 15u) | (((hb >> (2 * g)) & 3u) << 4)) - 32;
            const int qhi = (int)((qb >> 4) | (((hb >> (2 * g + 4)) & 3u) << 4)) - 32;
            w[j] = __fmul_rn(Dlo, (float)qlo);
            w[4 + j] = __fmul_rn(Dhi, (float)qhi);
        }
    }
}

template <int TYPE>
__device__ __forceinline__ void kq_offsets(int lane, int& lo, int& hi) {
    if (TYPE == BREW_TYPE_Q4_K) {
        lo = 64 * (lane >> 3) + 4 * (lane & 7);
        hi = lo + 32;
    } else {
        lo = 128 * (lane >> 4) + 32 * ((lane >> 3) & 1) + 4 * (lane & 7);
        hi = lo + 64;
    }
}

template <int TYPE, int NV, int RW = (NV >= 16 ? 2 : 4)>
__global__ void __launch_bounds__(KQ_WARPS * 32, 2) kq_matvec_kernel(const uint8_t* w, int64_t row_bytes, const float* x,
                                                                   int ldx, int K, int N, float* y, int ldy, int batch) {
    pdl_launch_dependents();
    pdl_wait();
    constexpr int SB = TYPE == BREW_TYPE_Q4_K ? 144 : 210;
    const int lane = threadIdx.x & 31;
    const int row0 = (blockIdx.x * KQ_WARPS + (threadIdx.x >> 5)) * RW;
    const int b0 = blockIdx.y * KQ_MAXV;
    const int nv = min(NV, batch - b0);
    if (row0 >= N) return;   // whole warps
    int lo, hi;
    kq_offsets<TYPE>(lane, lo, hi);
    float acc[RW][NV];
#pragma unroll
    for (int r = 0; r < RW; ++r)
#pragma unroll
        for (int v = 0; v < NV; ++v) acc[r][v] = 0.0f;
    const int nsb = K / 256;
    const uint8_t* wr[RW];
#pragma unroll
    for (int r = 0; r < RW; ++r)   // rows past N compute row N-1 again and are not stored
        wr[r] = w + (int64_t)min(row0 + r, N - 1) * row_bytes;
    KqRaw raw[RW];
#pragma unroll
    for (int r = 0; r < RW; ++r) kq_load<TYPE>(wr[r], lane, raw[r]);
    for (int sbi = 0; sbi < nsb; ++sbi) {
        float wv[RW][8];
#pragma unroll
        for (int r = 0; r < RW; ++r) kq_decode<TYPE>(raw[r], lane, wv[r]);
        if (sbi + 1 < nsb) {
#pragma unroll
            for (int r = 0; r < RW; ++r) kq_load<TYPE>(wr[r] + (int64_t)(sbi + 1) * SB, lane, raw[r]);
        }
        const float* xs = x + (int64_t)b0 * ldx + (int64_t)sbi * 256;
#pragma unroll
        for (int v = 0; v < NV; ++v) {
            if (v < nv) {
                const float4 a = __ldg(reinterpret_cast<const float4*>(xs + (int64_t)v * ldx + lo));
                const float4 c = __ldg(reinterpret_cast<const float4*>(xs + (int64_t)v * ldx + hi));
#pragma unroll
                for (int r = 0; r < RW; ++r) {
                    float t = acc[r][v];
                    t = fmaf(wv[r][0], a.x, t);
                    t = fmaf(wv[r][1], a.y, t);
                    t = fmaf(wv[r][2], a.z, t);
                    t = fmaf(wv[r][3], a.w, t);
                    t = fmaf(wv[r][4], c.x, t);
                    t = fmaf(wv[r][5], c.y, t);
                    t = fmaf(wv[r][6], c.z, t);
                    t = fmaf(wv[r][7], c.w, t);
                    acc[r][v] = t;
                }
            }
        }
    }
#pragma unroll
    for (int r = 0; r < RW; ++r)
#pragma unroll
        for (int v = 0; v < NV; ++v) {
            const float s = warp_sum(acc[r][v]);
            if (lane == 0 && v < nv && row0 + r < N) y[(int64_t)(b0 + v) * ldy + row0 + r] = s;
        }
}

template <int TYPE>
int kq_launch(const uint8_t* w, int64_t row_bytes, const float* x, int ldx, int K, int N, float* y, int ldy, int batch,
              cudaStream_t stream, bool pdl) {
    const int per = std::min(batch, KQ_MAXV);
    cudaLaunchConfig_t cfg = {};
    const int rw = per >= 16 ? 2 : 4;   // the kernel's RW for this vector count
    cfg.gridDim = dim3((N + KQ_WARPS * rw - 1) / (KQ_WARPS * rw), (batch + KQ_MAXV - 1) / KQ_MAXV);
    cfg.blockDim = dim3(KQ_WARPS * 32);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    if (per == 1)
        BREW_CUDA(cudaLaunchKernelEx(&cfg, kq_matvec_kernel<TYPE, 1>, w, row_bytes, x, ldx, K, N, y, ldy, batch));
    else if (per <= 2)
        BREW_CUDA(cudaLaunchKernelEx(&cfg, kq_matvec_kernel<TYPE, 2>, w, row_bytes, x, ldx, K, N, y, ldy, batch));
    else if (per <= 4)
        BREW_CUDA(cudaLaunchKernelEx(&cfg, kq_matvec_kernel<TYPE, 4>, w, row_bytes, x, ldx, K, N, y, ldy, batch));
    else if (per <= 8)
        BREW_CUDA(cudaLaunchKernelEx(&cfg, kq_matvec_kernel<TYPE, 8>, w, row_bytes, x, ldx, K, N, y, ldy, batch));
    else
        BREW_CUDA(cudaLaunchKernelEx(&cfg, kq_matvec_kernel<TYPE, 16>, w, row_bytes, x, ldx, K, N, y, ldy, batch));
    count_launch();
    return BREW_OK;
}
}  // namespace

int kquant_matvec_launch(int type, const uint8_t* w, int64_t row_bytes, const float* x, int ldx, int K, int N, float* y,
                         int ldy, int batch, cudaStream_t stream, bool pdl) {
    BREW_CHECK(K % 256 == 0, BREW_ERR_INVALID_ARG, "K-quant matvec: K=%d not a multiple of 256", K);
    BREW_CHECK(type == BREW_TYPE_Q4_K || type == BREW_TYPE_Q6_K, BREW_ERR_INVALID_ARG, "K-quant matvec: type %d", type);
    // the float4 reads of x need 16-byte aligned vectors
    BREW_CHECK((reinterpret_cast<uintptr_t>(x) & 15) == 0 && ldx % 4 == 0, BREW_ERR_INVALID_ARG,
               "K-quant matvec: x must be 16-byte aligned with a row pitch that is a multiple of 4 floats");
    if (batch <= 0 || N <= 0) return BREW_OK;
    if (type == BREW_TYPE_Q4_K) return kq_launch<BREW_TYPE_Q4_K>(w, row_bytes, x, ldx, K, N, y, ldy, batch, stream, pdl);
    return kq_launch<BREW_TYPE_Q6_K>(w, row_bytes, x, ldx, K, N, y, ldy, batch, stream, pdl);
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
    // programmatic dependent launch: the kernel streams its weight tiles
    // before griddepcontrol.wait and reads x / writes y only after it, so
    // back-to-back calls on one stream overlap one call's weight fetch with
    // the previous call's tail (a preceding kernel that does not trigger
    // early still completes first)
    return mv_launch(p, stream, true);
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
    return static_scratch_setup();
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
