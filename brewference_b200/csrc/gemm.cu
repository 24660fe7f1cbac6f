// gemm.cu — the prefill GEMM on tcgen05 (layout and arithmetic in gemm.cuh).
#include "brew_internal.cuh"
#include "gemm.cuh"
#include "prep.cuh"

namespace brew {
namespace {

// ---- tcgen05 helpers (PTX forms as in CUTLASS's sm100 MMA / TMEM atoms) ----
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Shared-memory matrix descriptor, K-major, no swizzle: core matrices of
// 8 rows x 16 bytes (128 contiguous bytes), the two 16-byte K halves of a
// 32-byte block `lbo` bytes apart, groups of 8 rows `sbo` bytes apart.
__device__ __forceinline__ uint64_t umma_desc_k(uint32_t smem_addr, uint32_t lbo, uint32_t sbo) {
    uint64_t d = 0;
    d |= (uint64_t)((smem_addr >> 4) & 0x3FFFu);
    d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
    d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
    d |= (uint64_t)1 << 46;   // descriptor version of sm_100
    return d;                  // base offset 0, layout type 0 (no swizzle)
}

// Instruction descriptor of kind::i8: D s32, A s8, B s8, both K-major.
constexpr uint32_t umma_idesc_s8(int M, int N) {
    return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void umma_s8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                        uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
        : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&v)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
                 : "r"(taddr)
                 : "memory");
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

constexpr int GEMM_N = 3 * GEMM_TT;       // limb columns per CTA (96)
constexpr int GEMM_TMEM_COLS = 128;       // power of two >= GEMM_N
constexpr int GEMM_SMEM = 48 * 1024;      // requested dynamic shared memory: at most 4 CTAs (4 x 128 TMEM columns) per SM

__global__ void gemm_pack_q8_kernel(const uint8_t* w, int N, int K, int8_t* wq, uint16_t* wd) {
    const int KB = K / 32;
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (int64_t)N * KB) return;
    const int64_t row = i / KB, kb = i % KB;
    const uint8_t* b = w + (row * KB + kb) * 34;
    wd[row * KB + kb] = (uint16_t)(b[0] | (b[1] << 8));
    int8_t* q = wq + row * K + kb * 32;
#pragma unroll 8
    for (int j = 0; j < 32; ++j) q[j] = (int8_t)b[2 + j];
}

// One warp per (token, block); tokens T .. Tp-1 are zero padding.
__global__ void gemm_limbs_kernel(const float* x, int ldx, int T, int Tp, int K, int8_t* limbs, float* scales) {
    const int lane = threadIdx.x & 31;
    const int64_t wid = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int KB = K / 32;
    if (wid >= (int64_t)Tp * KB) return;
    const int t = (int)(wid / KB), kb = (int)(wid % KB);
    const float v = t < T ? x[(int64_t)t * ldx + 32 * kb + lane] : 0.0f;
    const float amax = warp_max(fabsf(v));
    const float inv = amax > 0.0f ? PREP_RANGE / amax : 0.0f;
    const int q = __float2int_rn(v * inv);
    const int lo = ((q + 128) & 255) - 128;
    const int q1 = (q - lo) >> 8;
    const int mid = ((q1 + 128) & 255) - 128;
    const int hi = (q1 - mid) >> 8;
    int8_t* base = limbs + ((int64_t)kb * 3 * Tp + 3 * t) * 32;
    base[lane] = (int8_t)hi;
    base[32 + lane] = (int8_t)mid;
    base[64 + lane] = (int8_t)lo;
    if (lane == 0) scales[(int64_t)kb * Tp + t] = amax / PREP_RANGE;
}

// CTA = 128 weight rows x 32 tokens, 4 warps; thread i owns tensor-memory
// lane i (= weight row row0 + i) and accumulates its 32 outputs in fp32.
__global__ void __launch_bounds__(128) gemm_q8_kernel(const int8_t* wq, const uint16_t* wd, const int8_t* limbs,
                                                      const float* scales, int N, int K, int T, float* y,
                                                      unsigned int* err) {
    extern __shared__ __align__(1024) uint8_t smem[];
    uint8_t* sa = smem;                                          // A: 128 rows x 32 B (4096 B)
    uint8_t* sb = smem + 4096;                                   // B: 96 limb columns x 32 B (3072 B)
    float* ss = reinterpret_cast<float*>(smem + 7168);           // the block's token scales [32]
    uint64_t* mbar = reinterpret_cast<uint64_t*>(smem + 7296);   // MMA completion
    uint32_t* tslot = reinterpret_cast<uint32_t*>(smem + 7360);  // tensor-memory base address
    const int tid = threadIdx.x, warp = tid >> 5;
    const int row0 = blockIdx.x * GEMM_TM, t0 = blockIdx.y * GEMM_TT;
    const int KB = K / 32;
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tslot)),
                     "r"(GEMM_TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (tid == 0) {
        mbar_init(mbar, 1);
        fence_mbar_init();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;
    const uint32_t taddr = tmem + ((uint32_t)(warp * 32) << 16);   // this warp's 32 lanes
    const int row = row0 + tid;
    constexpr uint32_t idesc = umma_idesc_s8(GEMM_TM, GEMM_N);
    float acc[GEMM_TT];
#pragma unroll
    for (int t = 0; t < GEMM_TT; ++t) acc[t] = 0.0f;
    bool ok = true;
    for (int kb = 0; kb < KB; ++kb) {
        // stage the block column: A 256 and B 192 pieces of 16 B, in the
        // K-major core-matrix layout (row r at (r/8)*256 + half*128 + (r%8)*16)
        for (int c = tid; c < 2 * GEMM_TM + 2 * GEMM_N; c += 128) {
            if (c < 2 * GEMM_TM) {
                const int m = c >> 1, h = c & 1;
                cp_async16(sa + (m >> 3) * 256 + h * 128 + (m & 7) * 16,
                           wq + (int64_t)(row0 + m) * K + (int64_t)kb * 32 + h * 16);
            } else {
                const int n = (c - 2 * GEMM_TM) >> 1, h = (c - 2 * GEMM_TM) & 1;
                cp_async16(sb + (n >> 3) * 256 + h * 128 + (n & 7) * 16,
                           limbs + ((int64_t)kb * 3 * T + 3 * t0 + n) * 32 + h * 16);
            }
        }
        if (tid < GEMM_TT) ss[tid] = scales[(int64_t)kb * T + t0 + tid];
        const float d = half_bits_to_float(wd[(int64_t)row * KB + kb]);
        cp_async_wait_all();
        fence_proxy_async_smem();   // the copies are read by the tensor cores (async proxy)
        __syncthreads();
        if (tid == 0) {
            tc_fence_after();
            umma_s8(tmem, umma_desc_k(smem_u32(sa), 128, 256), umma_desc_k(smem_u32(sb), 128, 256), idesc, 0u);
            umma_commit(mbar);
        }
        __syncwarp();
        if (ok && !mbar_wait_bounded(mbar, kb & 1, err, BREW_DEVERR_TIMEOUT_FULL)) ok = false;
        ok = __all_sync(0xffffffffu, ok);   // tcgen05.ld is warp-collective
        tc_fence_after();
        if (ok) {
            // columns 3t, 3t+1, 3t+2: limbs hi, mid, lo of token t
#pragma unroll
            for (int j = 0; j < GEMM_N / 24; ++j) {
                uint32_t v0[8], v1[8], v2[8];
                tmem_ld8(taddr + 24 * j, v0);
                tmem_ld8(taddr + 24 * j + 8, v1);
                tmem_ld8(taddr + 24 * j + 16, v2);
                tmem_ld_wait();
                uint32_t v[24];
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    v[e] = v0[e];
                    v[8 + e] = v1[e];
                    v[16 + e] = v2[e];
                }
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    const int t = 8 * j + u;
                    const float hi = (float)(int)v[3 * u], mid = (float)(int)v[3 * u + 1], lo = (float)(int)v[3 * u + 2];
                    acc[t] = fmaf((lo + mid * 256.0f) + hi * 65536.0f, d * ss[t], acc[t]);
                }
            }
        }
        tc_fence_before();
        __syncthreads();   // tensor memory and the staged tiles are free again
    }
#pragma unroll
    for (int t = 0; t < GEMM_TT; ++t) y[(int64_t)(t0 + t) * N + row] = acc[t];
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(GEMM_TMEM_COLS)
                     : "memory");
    }
}

}  // namespace

int gemm_pack_q8_launch(const uint8_t* w, int N, int K, int8_t* wq, uint16_t* wd, cudaStream_t stream) {
    const int64_t n = (int64_t)N * (K / 32);
    gemm_pack_q8_kernel<<<(unsigned)((n + 255) / 256), 256, 0, stream>>>(w, N, K, wq, wd);
    BREW_CUDA(cudaGetLastError());
    count_launch();
    return BREW_OK;
}

int gemm_limbs_launch(const float* x, int ldx, int T, int Tp, int K, int8_t* limbs, float* scales,
                      cudaStream_t stream) {
    BREW_CHECK(T >= 0 && Tp >= T && K % 32 == 0, BREW_ERR_INVALID_ARG, "gemm limbs: T=%d Tp=%d K=%d", T, Tp, K);
    const int64_t warps = (int64_t)Tp * (K / 32);
    if (warps == 0) return BREW_OK;
    gemm_limbs_kernel<<<(unsigned)((warps * 32 + 255) / 256), 256, 0, stream>>>(x, ldx, T, Tp, K, limbs, scales);
    BREW_CUDA(cudaGetLastError());
    count_launch();
    return BREW_OK;
}

int gemm_q8_launch(const int8_t* wq, const uint16_t* wd, const int8_t* limbs, const float* scales, int N, int K, int T,
                   float* y, unsigned int* err, cudaStream_t stream) {
    BREW_CHECK(N % GEMM_TM == 0 && T % GEMM_TT == 0 && K % 32 == 0 && K > 0, BREW_ERR_INVALID_ARG,
               "gemm: N=%d (multiple of %d), T=%d (multiple of %d), K=%d (multiple of 32)", N, GEMM_TM, T, GEMM_TT, K);
    static bool attr = false;
    if (!attr) {
        BREW_CUDA(cudaFuncSetAttribute(gemm_q8_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, GEMM_SMEM));
        attr = true;
    }
    gemm_q8_kernel<<<dim3(N / GEMM_TM, T / GEMM_TT), 128, GEMM_SMEM, stream>>>(wq, wd, limbs, scales, N, K, T, y, err);
    BREW_CUDA(cudaGetLastError());
    count_launch();
    return BREW_OK;
}

}  // namespace brew

using namespace brew;

extern "C" int brew_gemm_q8_dev(float* y, const float* x, brew_tensor w, int64_t off, int32_t K, int32_t N,
                                int32_t T, void* stream) {
    BREW_CHECK(y && x && w && w->d, BREW_ERR_INVALID_ARG, "null argument");
    BREW_CHECK(w->type == BREW_TYPE_Q8_0, BREW_ERR_UNSUPPORTED, "the prefill GEMM takes Q8_0 weights");
    BREW_CHECK(K > 0 && K % 32 == 0 && off >= 0 && off % 32 == 0, BREW_ERR_INVALID_ARG, "K=%d off=%lld", K,
               (long long)off);
    BREW_CHECK(off + (int64_t)N * K <= w->n, BREW_ERR_OUT_OF_BOUNDS, "matrix past the tensor end");
    BREW_CHECK(N % GEMM_TM == 0 && T % GEMM_TT == 0 && T > 0, BREW_ERR_INVALID_ARG,
               "gemm: N=%d must be a multiple of %d and T=%d of %d", N, GEMM_TM, T, GEMM_TT);
    int rc = ensure_init();
    if (rc) return rc;
    std::lock_guard<std::mutex> lk(api_mutex());
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int KB = K / 32;
    int8_t *wq = nullptr, *limbs = nullptr;
    uint16_t* wd = nullptr;
    float* sc = nullptr;
    BREW_CUDA(cudaMalloc(&wq, (size_t)N * K));
    BREW_CUDA(cudaMalloc(&wd, (size_t)N * KB * 2));
    BREW_CUDA(cudaMalloc(&limbs, (size_t)KB * 3 * T * 32));
    BREW_CUDA(cudaMalloc(&sc, (size_t)KB * T * 4));
    rc = gemm_pack_q8_launch(w->d + off / 32 * 34, N, K, wq, wd, s);
    if (!rc) rc = gemm_limbs_launch(x, K, T, T, K, limbs, sc, s);
    if (!rc) rc = gemm_q8_launch(wq, wd, limbs, sc, N, K, T, y, ctx().err_word, s);
    cudaStreamSynchronize(s);
    cudaFree(wq);
    cudaFree(wd);
    cudaFree(limbs);
    cudaFree(sc);
    if (rc) return rc;
    return check_device_error("brew_gemm_q8_dev");
}
