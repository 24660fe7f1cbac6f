// eltwise.cu — per-row vector kernels of the unfused (K-quant) forward pass.
#include "eltwise.cuh"
#include "mv_device.cuh"
#include "prep.cuh"
#include "kqtc.cuh"

namespace brew {
namespace {

constexpr int EW_THREADS = 256;

// Sum over the CTA (EW_THREADS threads); `red` has 32 floats.
__device__ float cta_sum(float v, float* red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    v = warp_sum(v);
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float t = 0.0f;
    for (int w = 0; w < EW_THREADS / 32; ++w) t += red[w];
    __syncthreads();
    return t;
}

// One CTA per row b.
__global__ void __launch_bounds__(EW_THREADS) rmsnorm_kernel(const float* x, int ldx, const float* w, float eps, int K,
                                                             float* out, int ldo) {
    __shared__ float red[32];
    const float* xr = x + (int64_t)blockIdx.x * ldx;
    float* orow = out + (int64_t)blockIdx.x * ldo;
    float ss = 0.0f;
    for (int i = threadIdx.x; i < K; i += EW_THREADS) ss += xr[i] * xr[i];
    const float scale = rms_scale(cta_sum(ss, red), K, eps);
    for (int i = threadIdx.x; i < K; i += EW_THREADS) orow[i] = xr[i] * scale * w[i];
}

__global__ void add_bias_kernel(float* y, int ldy, const float* bias, int N) {
    float* yr = y + (int64_t)blockIdx.y * ldy;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < N; i += gridDim.x * blockDim.x) yr[i] = yr[i] + bias[i];
}

__global__ void __launch_bounds__(EW_THREADS) residual_kernel(float* x, int ldx, const float* t, int ldt,
                                                              const float* norm_w, float eps, int K) {
    __shared__ float red[32];
    float* xr = x + (int64_t)blockIdx.x * ldx;
    const float* tr = t + (int64_t)blockIdx.x * ldt;
    float scale = 1.0f;
    if (norm_w) {
        float ss = 0.0f;
        for (int i = threadIdx.x; i < K; i += EW_THREADS) ss += tr[i] * tr[i];
        scale = rms_scale(cta_sum(ss, red), K, eps);
    }
    for (int i = threadIdx.x; i < K; i += EW_THREADS) xr[i] = xr[i] + (norm_w ? tr[i] * scale * norm_w[i] : tr[i]);
}

__global__ void glu_kernel(float* hb, int ldo, const float* g, const float* u, int ld, int N, int epi) {
    const int64_t off = (int64_t)blockIdx.y * ld, oo = (int64_t)blockIdx.y * ldo;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < N; i += gridDim.x * blockDim.x)
        hb[oo + i] = act_glu(g[off + i], epi) * u[off + i];
}

constexpr int NP_THREADS = 1024;   // norm_prep: one CTA of 32 warps per vector

// Sum over the NP_THREADS threads of the CTA; `red` has 32 floats.
__device__ float cta_sum_np(float v, float* red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    v = warp_sum(v);
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float t = 0.0f;
    for (int w = 0; w < NP_THREADS / 32; ++w) t += red[w];
    __syncthreads();
    return t;
}

// One CTA per vector (CTAs past B only write zero records).
__global__ void __launch_bounds__(NP_THREADS) norm_prep_kernel(float* x, int ldx, const float* t, int ldt,
                                                               const float* post_w, const float* w, float eps, int K,
                                                               int B, float* out, int ldo, uint8_t* rec, int nvp) {
    extern __shared__ float xv[];   // K floats
    __shared__ float red[32];
    const int b = blockIdx.x, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (b < B) {
        float* xr = x + (int64_t)b * ldx;
        if (t) {   // the residual: x += t, or x += rmsnorm(t, post_w) (Gemma3's post-norm)
            const float* tr = t + (int64_t)b * ldt;
            float scale = 1.0f;
            if (post_w) {
                float ss = 0.0f;
                for (int i = threadIdx.x; i < K; i += NP_THREADS) ss += tr[i] * tr[i];
                scale = rms_scale(cta_sum_np(ss, red), K, eps);
            }
            for (int i = threadIdx.x; i < K; i += NP_THREADS) {
                const float v = xr[i] + (post_w ? tr[i] * scale * post_w[i] : tr[i]);
                xr[i] = v;
                xv[i] = v;
            }
        } else {
            for (int i = threadIdx.x; i < K; i += NP_THREADS) xv[i] = xr[i];
        }
        // the RMSNorm (each thread reads back the elements it wrote)
        float ss = 0.0f;
        for (int i = threadIdx.x; i < K; i += NP_THREADS) ss += xv[i] * xv[i];
        const float scale = rms_scale(cta_sum_np(ss, red), K, eps);
        float* orow = out + (int64_t)b * ldo;
        for (int i = threadIdx.x; i < K; i += NP_THREADS) {
            const float v = xv[i] * scale * w[i];
            orow[i] = v;
            xv[i] = v;
        }
    }
    if (!rec) return;
    __syncthreads();
    for (int sb = warp; sb < K / 256; sb += NP_THREADS / 32) {   // the records, warp w: super-blocks w, w + 32, ...
        float xs[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) xs[i] = b < B ? xv[sb * 256 + 8 * lane + i] : 0.0f;
        kx_emit_sb(rec, K, nvp, b, sb, xs);
    }
}

// One warp per (vector, super-block): the gated activation of its 256
// elements, then their records (vectors past B: zero records).
__global__ void glu_prep_kernel(float* hb, const float* g, const float* u, int ld, int N, int B, int epi, uint8_t* rec,
                                int nvp) {
    const int lane = threadIdx.x & 31;
    const int64_t wid = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int KSB = N / 256;
    if (wid >= (int64_t)nvp * KSB) return;
    const int b = (int)(wid / KSB), sb = (int)(wid % KSB);
    float xs[8];
    if (b < B) {
        const int64_t o = (int64_t)b * ld + (int64_t)sb * 256 + 8 * lane;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            xs[i] = act_glu(g[o + i], epi) * u[o + i];
            hb[o + i] = xs[i];
        }
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) xs[i] = 0.0f;
    }
    kx_emit_sb(rec, N, nvp, b, sb, xs);
}

int grid_for(int n) { return std::max(1, std::min(148 * 4, (n + 255) / 256)); }

}  // namespace

int norm_prep_launch(float* x, int ldx, const float* t, int ldt, const float* post_w, const float* w, float eps, int K,
                     int B, float* out, int ldo, uint8_t* rec, cudaStream_t s) {
    BREW_CHECK(B >= 1 && (!rec || (B <= KX_MAX_VECTORS && K % 256 == 0)), BREW_ERR_INVALID_ARG,
               "norm+records: B=%d K=%d", B, K);
    const size_t smem = (size_t)K * sizeof(float);
    static uint64_t attr_devs = 0;
    int dev = 0;
    BREW_CUDA(cudaGetDevice(&dev));
    if (smem > 48 * 1024 && dev < 64 && !(attr_devs >> dev & 1)) {
        BREW_CUDA(cudaFuncSetAttribute(norm_prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024));
        attr_devs |= 1ull << dev;
    }
    BREW_CHECK(smem <= 160 * 1024, BREW_ERR_INVALID_ARG, "norm+records: K=%d", K);
    const int nvp = rec ? (B + 15) / 16 * 16 : B;
    norm_prep_kernel<<<nvp, NP_THREADS, smem, s>>>(x, ldx, t, ldt, post_w, w, eps, K, B, out, ldo, rec, nvp);
    BREW_CUDA(cudaGetLastError());
    count_launch();
    return BREW_OK;
}

int glu_prep_launch(float* hb, const float* g, const float* u, int ld, int N, int B, bool gelu, uint8_t* rec,
                    cudaStream_t s) {
    if (!rec) return glu_launch(hb, g, u, ld, N, B, gelu, s);
    BREW_CHECK(B >= 1 && B <= KX_MAX_VECTORS && N % 256 == 0, BREW_ERR_INVALID_ARG, "glu+records: B=%d N=%d", B, N);
    const int nvp = (B + 15) / 16 * 16;
    const int64_t warps = (int64_t)nvp * (N / 256);
    glu_prep_kernel<<<(unsigned)((warps * 32 + 255) / 256), 256, 0, s>>>(hb, g, u, ld, N, B,
                                                                          gelu ? MV_EPI_GLU_GELU : MV_EPI_GLU_SILU, rec,
                                                                          nvp);
    BREW_CUDA(cudaGetLastError());
    count_launch();
    return BREW_OK;
}

int rmsnorm_launch(const float* x, int ldx, const float* w, float eps, int K, int B, float* out, int ldo,
                   cudaStream_t s) {
    rmsnorm_kernel<<<B, EW_THREADS, 0, s>>>(x, ldx, w, eps, K, out, ldo);
    BREW_CUDA(cudaGetLastError());
    count_launch();
    return BREW_OK;
}

int add_bias_launch(float* y, int ldy, const float* bias, int N, int B, cudaStream_t s) {
    add_bias_kernel<<<dim3(grid_for(N), B), 256, 0, s>>>(y, ldy, bias, N);
    BREW_CUDA(cudaGetLastError());
    count_launch();
    return BREW_OK;
}

int residual_launch(float* x, int ldx, const float* t, int ldt, const float* norm_w, float eps, int K, int B,
                    cudaStream_t s) {
    residual_kernel<<<B, EW_THREADS, 0, s>>>(x, ldx, t, ldt, norm_w, eps, K);
    BREW_CUDA(cudaGetLastError());
    count_launch();
    return BREW_OK;
}

int glu_launch(float* hb, const float* g, const float* u, int ld, int N, int B, bool gelu, cudaStream_t s, int ldo) {
    glu_kernel<<<dim3(grid_for(N), B), 256, 0, s>>>(hb, ldo > 0 ? ldo : ld, g, u, ld, N,
                                                     gelu ? MV_EPI_GLU_GELU : MV_EPI_GLU_SILU);
    BREW_CUDA(cudaGetLastError());
    count_launch();
    return BREW_OK;
}

}  // namespace brew
