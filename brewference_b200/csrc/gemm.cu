// gemm.cu — the prefill GEMM on tcgen05 (layout and arithmetic in gemm.cuh).
#include "brew_internal.cuh"
#include "gemm.cuh"
#include "prep.cuh"
#include "tc_device.cuh"

namespace brew {
namespace {

constexpr int GEMM_N = 3 * GEMM_TT;        // limb columns per tile (96)
constexpr int GEMM_STAGES = 4;             // shared-memory ring
constexpr int GEMM_A_BYTES = GEMM_TM * 32; // one block column of 128 rows
constexpr int GEMM_B_BYTES = GEMM_N * 32;  // and of the 96 limb columns
constexpr int GEMM_STAGE_BYTES = GEMM_A_BYTES + GEMM_B_BYTES;
constexpr int GEMM_TMEM_COLS = 256;        // two accumulator buffers of 128 columns
// requested dynamic shared memory: also caps residency at two CTAs per SM,
// so the CTAs of one SM never ask for more than its 512 tensor-memory columns
constexpr int GEMM_SMEM = 96 * 1024;
constexpr int GEMM_EPI_WARPS = 8;          // two per tensor-memory lane quadrant (16 tokens each)
constexpr int GEMM_THREADS = 64 + 32 * GEMM_EPI_WARPS;   // loader warp, MMA warp, epilogue warps

// Bounded mbarrier wait for the pipeline's short hand-offs: polls without
// sleeping at first (try_wait itself suspends the thread for a while),
// then backs off; ~2 s in all before it records `code` and gives up.
__device__ __forceinline__ bool gemm_wait(uint64_t* bar, uint32_t parity, unsigned int* err, unsigned int code) {
    for (int i = 0; i < 32; ++i)
        if (mbar_try_wait(bar, parity)) return true;
    return mbar_wait_bounded(bar, parity, err, code);
}


// Q8_0 blocks (34 B: fp16 d, 32 int8 q) or Q4_0 blocks (18 B: fp16 d, 32
// nibbles, value d * (q - 8)): the integer factors q (Q8_0) or q - 8 (Q4_0)
// as int8, the scales d as they are.
template <int TYPE>
__global__ void gemm_pack_kernel(const uint8_t* w, int rows, int K, int8_t* wq, uint16_t* wd, int ldn, int row0) {
    constexpr int BB = TYPE == BREW_TYPE_Q8_0 ? 34 : 18;
    const int KB = K / 32;
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (int64_t)rows * KB) return;
    const int64_t row = i / KB, kb = i % KB;
    const uint8_t* b = w + (row * KB + kb) * BB;
    const int64_t grow = row0 + row;
    wd[kb * ldn + grow] = (uint16_t)(b[0] | (b[1] << 8));
    int8_t* tile = wq + ((grow / GEMM_TM) * KB + kb) * 4096;
    const int r = (int)(grow % GEMM_TM);
#pragma unroll 8
    for (int j = 0; j < 32; ++j) {
        const int q = TYPE == BREW_TYPE_Q8_0 ? (int)(int8_t)b[2 + j] : (j < 16 ? (b[2 + j] & 15) : (b[2 + j - 16] >> 4)) - 8;
        tile[tc_tile_off(r, j)] = (int8_t)q;
    }
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
    const float inv = prep_block_inv(amax);
    const int q = __float2int_rn(v * inv);
    const int lo = ((q + 128) & 255) - 128;
    const int q1 = (q - lo) >> 8;
    const int mid = ((q1 + 128) & 255) - 128;
    const int hi = (q1 - mid) >> 8;
    // limb column of (token t, limb l) inside its tile of 32 tokens: token
    // pairs side by side, 6 (t / 2) + 2 l + (t % 2), so the epilogue reads
    // both tokens of a pair from adjacent tensor-memory columns
    int8_t* tile = limbs + (int64_t)kb * 3 * Tp * 32 + (int64_t)(t >> 5) * 3072;
    const int c0 = 6 * ((t & 31) >> 1) + (t & 1);
    tile[tc_tile_off(c0, lane)] = (int8_t)hi;
    tile[tc_tile_off(c0 + 2, lane)] = (int8_t)mid;
    tile[tc_tile_off(c0 + 4, lane)] = (int8_t)lo;
    if (lane == 0) scales[(int64_t)kb * Tp + t] = prep_block_scale(amax);
}

// CTA = 128 weight rows x 32 tokens, warp-specialised:
//   warp 0      one lane loads block column kb (A: 128 rows x 32 B, B: 96
//               limb columns x 32 B) into ring stage kb % 4: two bulk copies,
//               since both are stored in the K-major core-matrix layout
//               (tc_tile_off) already; all 4 stages can be in flight;
//   warp 1      one thread issues tcgen05.mma for block column kb into tensor-
//               memory buffer kb % 2 (each column needs its own product: the
//               block scales differ per column) and commits to the stage's
//               "empty" and the buffer's "full" barriers;
//   warps 2-9   read the buffer back (warp w owns tensor-memory lanes
//               32 (w % 4) ..: rows row0 + 32 (w % 4) + lane, and 16 of the
//               32 tokens), release it as soon as it is in registers, and add
//               d_row * s_token * ((lo + mid 2^8) + hi 2^16) to fp32
//               accumulators.
// So the loads run ahead, and the MMA of column kb + 1 overlaps the
// epilogue of column kb.
__global__ void __launch_bounds__(GEMM_THREADS, 2) gemm_q8_kernel(const int8_t* wq, const uint16_t* wd,
                                                               const int8_t* limbs, const float* scales, int N, int K,
                                                               int T, int Tvalid, float* y, unsigned int* err) {
    extern __shared__ __align__(1024) uint8_t smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + GEMM_STAGES * GEMM_STAGE_BYTES);
    uint64_t* empty = full + GEMM_STAGES;
    uint64_t* tfull = empty + GEMM_STAGES;
    uint64_t* tempty = tfull + 2;
    uint32_t* tslot = reinterpret_cast<uint32_t*>(tempty + 2);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int row0 = blockIdx.x * GEMM_TM, t0 = blockIdx.y * GEMM_TT;
    const int KB = K / 32;
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tslot)),
                     "r"(GEMM_TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (tid == 0) {
        for (int i = 0; i < GEMM_STAGES; ++i) {
            mbar_init(&full[i], 1);    // the loader's arrive.expect_tx (+ the copies' bytes)
            mbar_init(&empty[i], 1);   // tcgen05.commit
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&tfull[i], 1);   // tcgen05.commit
            mbar_init(&tempty[i], GEMM_EPI_WARPS);   // one arrival per epilogue warp
        }
        fence_mbar_init();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;
    if (warp == 0) {
        // ---------------------------------- loader ----------------------------------
        // two bulk copies per block column: the weight tile and the limb tile
        // are stored in the shared-memory layout already
        if (lane == 0) {
            const int8_t* asrc = wq + (int64_t)blockIdx.x * KB * GEMM_A_BYTES;
            const int8_t* bsrc = limbs + (int64_t)blockIdx.y * GEMM_B_BYTES;
            for (int kb = 0; kb < KB; ++kb) {
                const int s = kb % GEMM_STAGES;
                if (!gemm_wait(&empty[s], ((kb / GEMM_STAGES) + 1) & 1, err, BREW_DEVERR_TIMEOUT_EMPTY)) break;
                uint8_t* sa = smem + s * GEMM_STAGE_BYTES;
                mbar_arrive_expect_tx(&full[s], GEMM_STAGE_BYTES);
                bulk_g2s(sa, asrc + (int64_t)kb * GEMM_A_BYTES, GEMM_A_BYTES, &full[s]);
                bulk_g2s(sa + GEMM_A_BYTES, bsrc + (int64_t)kb * 3 * T * 32, GEMM_B_BYTES, &full[s]);
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        // ------------------------------------ MMA ------------------------------------
        if (lane == 0) {
            constexpr uint32_t idesc = umma_idesc_s8(GEMM_TM, GEMM_N);
            for (int kb = 0; kb < KB; ++kb) {
                const int s = kb % GEMM_STAGES, b = kb & 1;
                if (!gemm_wait(&full[s], (kb / GEMM_STAGES) & 1, err, BREW_DEVERR_TIMEOUT_FULL)) break;
                if (!gemm_wait(&tempty[b], (kb >> 1) & 1, err, BREW_DEVERR_TIMEOUT_EMPTY)) break;
                tc_fence_after();
                const uint32_t sa = smem_u32(smem + s * GEMM_STAGE_BYTES);
                umma_s8(tmem + b * 128, umma_desc_k(sa, 128, 256), umma_desc_k(sa + GEMM_A_BYTES, 128, 256), idesc,
                        1u);   // onto the magic-number start value
                umma_commit(&empty[s]);
                umma_commit(&tfull[b]);
            }
        }
        __syncwarp();
    } else {
        // ---------------------------------- epilogue ----------------------------------
        // warp w: tensor-memory lanes 32 (w % 4) .. (rows row0 + 32 (w % 4) +
        // lane) and tokens 16 hh .. 16 hh + 15 (columns 48 hh .. 48 hh + 47)
        const int q = warp & 3, hh = (warp - 2) >> 2;
        const int row = row0 + 32 * q + lane;
        const uint32_t tq = tmem + ((uint32_t)(32 * q) << 16) + 48 * hh;
        // both buffers start at the magic value (their first "release")
#pragma unroll
        for (int b = 0; b < 2; ++b)
#pragma unroll
            for (int c = 0; c < 3; ++c) tmem_st16_const(tq + b * 128 + 16 * c, TC_MAGIC);
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
            mbar_arrive(&tempty[0]);
            mbar_arrive(&tempty[1]);
        }
        uint64_t acc[8];   // token pairs (2p, 2p + 1)
#pragma unroll
        for (int p = 0; p < 8; ++p) acc[p] = 0ull;
        const uint64_t negc = f2_packf(-TC_MAGIC_F, -TC_MAGIC_F);
        const uint64_t neg257c = f2_packf(-257.0f * TC_MAGIC_F, -257.0f * TC_MAGIC_F);
        const uint64_t k256 = f2_packf(256.0f, 256.0f), k65536 = f2_packf(65536.0f, 65536.0f);
        // this column's weight scale and token scales, loaded one column ahead
        uint16_t dbits = wd[row];
        float4 sn[4];
        const float* sbase = scales + t0 + 16 * hh;
#pragma unroll
        for (int g = 0; g < 4; ++g) sn[g] = __ldg(reinterpret_cast<const float4*>(sbase) + g);
        for (int kb = 0; kb < KB; ++kb) {
            const int b = kb & 1;
            bool ok = gemm_wait(&tfull[b], (kb >> 1) & 1, err, BREW_DEVERR_TIMEOUT_FULL);
            ok = __all_sync(0xffffffffu, ok);   // tcgen05.ld / st are warp-collective
            if (!ok) break;
            tc_fence_after();
            const float d = half_bits_to_float(dbits);
            const uint64_t d2 = f2_packf(d, d);
            // two halves of 24 columns (8 tokens): read, reset to the magic
            // value, and after the second half release the buffer
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const uint32_t ta = tq + b * 128 + 24 * e;
                uint32_t v[24];
                tmem_ld8(ta, v);
                tmem_ld8(ta + 8, v + 8);
                tmem_ld8(ta + 16, v + 16);
                tmem_ld_wait();
                tmem_st16_const(ta, TC_MAGIC);
                tmem_st8_const(ta + 16, TC_MAGIC);
                if (e == 1) {
                    tmem_st_wait();
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&tempty[b]);
                }
#pragma unroll
                for (int pp = 0; pp < 4; ++pp) {
                    // tokens 2p, 2p + 1 of this warp's 16: columns 6 pp + (0, 1) hi,
                    // (2, 3) mid, (4, 5) lo of this half
                    const int p = 4 * e + pp;
                    const float4 sg = sn[p >> 1];
                    const uint64_t s2 = (p & 1) ? f2_packf(sg.z, sg.w) : f2_packf(sg.x, sg.y);
                    // (lo + mid 2^8) + hi 2^16 from the three magic-biased
                    // sums: hi - c is exact; mid 2^8 + lo rounds once (to a
                    // multiple of 2^8 near 257 c: error <= 2^7), and taking
                    // 257 c = 771 * 2^22 from it is exact
                    const uint64_t hi = f2_add(f2_pack(v[6 * pp], v[6 * pp + 1]), negc);
                    const uint64_t ml = f2_add(f2_fma(f2_pack(v[6 * pp + 2], v[6 * pp + 3]), k256,
                                                      f2_pack(v[6 * pp + 4], v[6 * pp + 5])),
                                               neg257c);
                    const uint64_t val = f2_fma(hi, k65536, ml);
                    acc[p] = f2_fma(val, f2_mul(d2, s2), acc[p]);
                }
            }
            if (kb + 1 < KB) {   // the next column's scales, while the next MMA runs
                dbits = wd[(int64_t)(kb + 1) * N + row];
#pragma unroll
                for (int g = 0; g < 4; ++g)
                    sn[g] = __ldg(reinterpret_cast<const float4*>(sbase + (int64_t)(kb + 1) * T) + g);
            }
        }
#pragma unroll
        for (int p = 0; p < 8; ++p) {   // tokens past Tvalid are padding: not stored
            const float a0 = __uint_as_float((uint32_t)acc[p]), a1 = __uint_as_float((uint32_t)(acc[p] >> 32));
            const int tk = t0 + 16 * hh + 2 * p;
            if (tk < Tvalid) y[(int64_t)tk * N + row] = a0;
            if (tk + 1 < Tvalid) y[(int64_t)(tk + 1) * N + row] = a1;
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(GEMM_TMEM_COLS)
                     : "memory");
    }
}

}  // namespace

int gemm_pack_launch(int type, const uint8_t* w, int rows, int K, int8_t* wq, uint16_t* wd, int ldn, int row0,
                     cudaStream_t stream) {
    BREW_CHECK(type == BREW_TYPE_Q8_0 || type == BREW_TYPE_Q4_0, BREW_ERR_UNSUPPORTED,
               "the GEMM takes Q8_0 or Q4_0 blocks (type %d)", type);
    const int64_t n = (int64_t)rows * (K / 32);
    const unsigned blocks = (unsigned)((n + 255) / 256);
    if (type == BREW_TYPE_Q8_0) gemm_pack_kernel<BREW_TYPE_Q8_0><<<blocks, 256, 0, stream>>>(w, rows, K, wq, wd, ldn, row0);
    else gemm_pack_kernel<BREW_TYPE_Q4_0><<<blocks, 256, 0, stream>>>(w, rows, K, wq, wd, ldn, row0);
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
                   int Tvalid, float* y, unsigned int* err, cudaStream_t stream) {
    BREW_CHECK(N % GEMM_TM == 0 && T % GEMM_TT == 0 && K % 32 == 0 && K > 0, BREW_ERR_INVALID_ARG,
               "gemm: N=%d (multiple of %d), T=%d (multiple of %d), K=%d (multiple of 32)", N, GEMM_TM, T, GEMM_TT, K);
    static uint64_t attr_devs = 0;   // devices whose attribute is set
    int dev = 0;
    BREW_CUDA(cudaGetDevice(&dev));
    if (dev < 64 && !(attr_devs >> dev & 1)) {
        BREW_CUDA(cudaFuncSetAttribute(gemm_q8_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, GEMM_SMEM));
        attr_devs |= 1ull << dev;
    }
    gemm_q8_kernel<<<dim3(N / GEMM_TM, T / GEMM_TT), GEMM_THREADS, GEMM_SMEM, stream>>>(wq, wd, limbs, scales, N, K,
                                                                                        T, Tvalid, y, err);
    BREW_CUDA(cudaGetLastError());
    count_launch();
    return BREW_OK;
}

}  // namespace brew

using namespace brew;

// A GEMM-layout copy of one Q8_0 / Q4_0 matrix and the activation scratch of
// its runs.
struct brew_gemm_plan_s {
    int type = 0, K = 0, N = 0, device = -1;
    int8_t* wq = nullptr;       // [N/128][K/32] quant tiles
    uint16_t* wd = nullptr;     // [K/32][N] block scales
    int8_t* limbs = nullptr;    // [K/32][cap/32][3072 B]
    float* scales = nullptr;    // [K/32][cap]
    int cap = 0;                // tokens the scratch holds (multiple of GEMM_TT)
};

namespace {

void plan_release(brew_gemm_plan p) {
    if (!p) return;
    cudaFree(p->wq);
    cudaFree(p->wd);
    cudaFree(p->limbs);
    cudaFree(p->scales);
    delete p;
}

int plan_create(brew_tensor w, int64_t off, int K, int N, bool q8_only, brew_gemm_plan* out) {
    BREW_CHECK(w && w->d && out, BREW_ERR_INVALID_ARG, "null argument");
    *out = nullptr;
    BREW_CHECK(w->type == BREW_TYPE_Q8_0 || (!q8_only && w->type == BREW_TYPE_Q4_0), BREW_ERR_UNSUPPORTED,
               "the GEMM takes %s weights (type %d)", q8_only ? "Q8_0" : "Q8_0 or Q4_0", w->type);
    BREW_CHECK(K > 0 && K % 32 == 0 && off >= 0 && off % 32 == 0, BREW_ERR_INVALID_ARG, "K=%d off=%lld", K,
               (long long)off);
    BREW_CHECK(N > 0 && N % GEMM_TM == 0, BREW_ERR_INVALID_ARG, "gemm: N=%d must be a multiple of %d", N, GEMM_TM);
    BREW_CHECK(off + (int64_t)N * K <= w->n, BREW_ERR_OUT_OF_BOUNDS, "matrix past the tensor end");
    int rc = ensure_init();
    if (rc) return rc;
    brew_gemm_plan p = new brew_gemm_plan_s();
    p->type = w->type;
    p->K = K;
    p->N = N;
    p->device = ctx().device;
    cudaStream_t s = ctx().stream;
    const int bb = w->type == BREW_TYPE_Q8_0 ? 34 : 18;
    if (cudaMalloc(&p->wq, (size_t)N * K) != cudaSuccess || cudaMalloc(&p->wd, (size_t)N * (K / 32) * 2) != cudaSuccess) {
        plan_release(p);
        return set_error(BREW_ERR_CUDA, "gemm plan: out of device memory");
    }
    rc = gemm_pack_launch(w->type, w->d + off / 32 * bb, N, K, p->wq, p->wd, N, 0, s);
    if (!rc && cudaStreamSynchronize(s) != cudaSuccess) rc = set_error(BREW_ERR_CUDA, "gemm plan: pack failed");
    if (rc) {
        plan_release(p);
        return rc;
    }
    *out = p;
    return BREW_OK;
}

int plan_run(brew_gemm_plan p, float* y, const float* x, int T, cudaStream_t s) {
    BREW_CHECK(p && y && x, BREW_ERR_INVALID_ARG, "null argument");
    BREW_CHECK(T >= 1, BREW_ERR_INVALID_ARG, "gemm: T=%d", T);
    BREW_CHECK(p->device == ctx().device, BREW_ERR_INVALID_ARG, "gemm plan of device %d used on device %d", p->device,
               ctx().device);
    const int Tp = (T + GEMM_TT - 1) / GEMM_TT * GEMM_TT, KB = p->K / 32;
    if (Tp > p->cap) {   // the scratch grows to the largest T seen
        cudaStreamSynchronize(s);
        cudaFree(p->limbs);
        cudaFree(p->scales);
        p->limbs = nullptr;
        p->scales = nullptr;
        p->cap = 0;
        BREW_CUDA(cudaMalloc(&p->limbs, (size_t)KB * 3 * Tp * 32));
        BREW_CUDA(cudaMalloc(&p->scales, (size_t)KB * Tp * 4));
        p->cap = Tp;
    }
    int rc = gemm_limbs_launch(x, p->K, T, Tp, p->K, p->limbs, p->scales, s);
    if (!rc) rc = gemm_q8_launch(p->wq, p->wd, p->limbs, p->scales, p->N, p->K, Tp, T, y, ctx().err_word, s);
    return rc;
}

}  // namespace

extern "C" {

int brew_gemm_plan_create(brew_tensor w, int64_t off, int32_t K, int32_t N, brew_gemm_plan* out) {
    std::lock_guard<std::mutex> lk(api_mutex());
    return plan_create(w, off, K, N, false, out);
}

int brew_gemm_plan_run(brew_gemm_plan p, float* y, const float* x, int32_t T, void* stream) {
    std::lock_guard<std::mutex> lk(api_mutex());
    return plan_run(p, y, x, T, static_cast<cudaStream_t>(stream));
}

int brew_gemm_plan_free(brew_gemm_plan p) {
    std::lock_guard<std::mutex> lk(api_mutex());
    if (p) cudaDeviceSynchronize();   // no run of this plan still in flight
    plan_release(p);
    return BREW_OK;
}

int brew_gemm_q8_dev(float* y, const float* x, brew_tensor w, int64_t off, int32_t K, int32_t N, int32_t T,
                     void* stream) {
    BREW_CHECK(y && x && w && w->d, BREW_ERR_INVALID_ARG, "null argument");
    BREW_CHECK(T > 0, BREW_ERR_INVALID_ARG, "gemm: T=%d", T);
    std::lock_guard<std::mutex> lk(api_mutex());
    brew_gemm_plan p = nullptr;
    int rc = plan_create(w, off, K, N, true, &p);
    if (rc) return rc;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    rc = plan_run(p, y, x, T, s);
    cudaStreamSynchronize(s);
    plan_release(p);
    if (rc) return rc;
    return check_device_error("brew_gemm_q8_dev");
}

}  // extern "C"
