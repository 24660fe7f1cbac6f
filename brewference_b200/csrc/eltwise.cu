// eltwise.cu — per-row vector kernels of the unfused (K-quant) forward pass.
#include "eltwise.cuh"
#include "mv_device.cuh"
#include "prep.cuh"

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

__global__ void glu_kernel(float* hb, const float* g, const float* u, int ld, int N, int epi) {
    const int64_t off = (int64_t)blockIdx.y * ld;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < N; i += gridDim.x * blockDim.x)
        hb[off + i] = act_glu(g[off + i], epi) * u[off + i];
}

int grid_for(int n) { return std::max(1, std::min(148 * 4, (n + 255) / 256)); }

}  // namespace

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

int glu_launch(float* hb, const float* g, const float* u, int ld, int N, int B, bool gelu, cudaStream_t s) {
    glu_kernel<<<dim3(grid_for(N), B), 256, 0, s>>>(hb, g, u, ld, N, gelu ? MV_EPI_GLU_GELU : MV_EPI_GLU_SILU);
    BREW_CUDA(cudaGetLastError());
    count_launch();
    return BREW_OK;
}

}  // namespace brew
