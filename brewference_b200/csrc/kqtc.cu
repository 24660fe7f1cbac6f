// kqtc.cu — the K-quant matvec on tcgen05 (layouts and arithmetic in kqtc.cuh).
#include "brew_internal.cuh"
#include "kqtc.cuh"
#include "prep.cuh"
#include "tc_device.cuh"

namespace brew {
namespace {

__device__ __forceinline__ float kx_half(const uint8_t* p) {
    return half_bits_to_float((uint16_t)(p[0] | (p[1] << 8)));
}

// 6-bit scale and min of Q4_K sub-block s (GGML's get_scale_min_k4).
__device__ __forceinline__ void kx_scale_min(const uint8_t* sb, int s, int& sc, int& m) {
    if (s < 4) {
        sc = sb[s] & 63;
        m = sb[s + 4] & 63;
    } else {
        sc = (sb[s + 4] & 0xF) | ((sb[s - 4] >> 6) << 4);
        m = (sb[s + 4] >> 4) | ((sb[s] >> 6) << 4);
    }
}

// One thread per (row, 32-element sub-block j of super-block sb).
template <int TYPE>
__global__ void kx_pack_kernel(const uint8_t* w, int64_t rows, int K, uint8_t* base, int64_t pitch, int64_t row_off,
                               size_t m_off, size_t f_off) {
    constexpr int SB = TYPE == BREW_TYPE_Q4_K ? 144 : 210;
    const int KB = K / 32, KSB = K / 256;
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= rows * KB) return;
    const int64_t row = i / KB;
    const int kb = (int)(i % KB), sb = kb / 8, j = kb % 8;
    const uint8_t* blk = w + row * (int64_t)KSB * SB + (int64_t)sb * SB;
    const int64_t prow = row_off + row;
    uint32_t h[8], l[8];   // 32 bytes each
    int mv = 0;
    float d, dmin = 0.0f;
    if (TYPE == BREW_TYPE_Q4_K) {
        int sc;
        kx_scale_min(blk + 4, j, sc, mv);
        d = kx_half(blk);
        dmin = kx_half(blk + 2);
        const int sh = sc >> 3, sl = sc & 7;
#pragma unroll
        for (int w4 = 0; w4 < 8; ++w4) {
            uint32_t hv = 0u, lv = 0u;
#pragma unroll
            for (int b = 0; b < 4; ++b) {
                const int k = 4 * w4 + b;
                const int q = (blk[16 + 32 * (j / 2) + k] >> (4 * (j & 1))) & 15;
                hv |= (uint32_t)(q * sh) << (8 * b);
                lv |= (uint32_t)(q * sl) << (8 * b);
            }
            h[w4] = hv;
            l[w4] = lv;
        }
    } else {
        d = kx_half(blk + 208);
        const int s_lo = (int8_t)blk[192 + 2 * j], s_hi = (int8_t)blk[192 + 2 * j + 1];
#pragma unroll
        for (int w4 = 0; w4 < 8; ++w4) {
            uint32_t hv = 0u, lv = 0u;
#pragma unroll
            for (int b = 0; b < 4; ++b) {
                const int k = 4 * w4 + b;
                const int r = 32 * j + k, hb = r / 128, rr = r % 128, grp = rr / 32, ll = rr % 32;
                const int lq = blk[64 * hb + (grp & 1) * 32 + ll];
                const int low = grp < 2 ? (lq & 15) : (lq >> 4);
                const int high = (blk[128 + 32 * hb + ll] >> (2 * grp)) & 3;
                const int v = (k < 16 ? s_lo : s_hi) * ((low | (high << 4)) - 32);   // [-4064, 4096]
                hv |= (uint32_t)((v >> 6) & 255) << (8 * b);
                lv |= (uint32_t)(v & 63) << (8 * b);
            }
            h[w4] = hv;
            l[w4] = lv;
        }
    }
    uint8_t* hp = base;
    uint8_t* lp = base + (size_t)K * pitch;
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
        const int64_t o = ((int64_t)(2 * kb + hf) * pitch + prow) * 16;
        *reinterpret_cast<uint4*>(hp + o) = make_uint4(h[4 * hf], h[4 * hf + 1], h[4 * hf + 2], h[4 * hf + 3]);
        *reinterpret_cast<uint4*>(lp + o) = make_uint4(l[4 * hf], l[4 * hf + 1], l[4 * hf + 2], l[4 * hf + 3]);
    }
    if (TYPE == BREW_TYPE_Q4_K) base[m_off + ((int64_t)sb * pitch + prow) * 16 + j] = (uint8_t)mv;
    if (j == 0) reinterpret_cast<float2*>(base + f_off)[(int64_t)sb * pitch + prow] = make_float2(d, dmin);
}


// One warp per (vector t < nvp, super-block): lane i holds elements
// 8i .. 8i + 7 (sub-block i / 4); vectors past nv are zero.
__global__ void kx_prep_kernel(const float* x, int ldx, int K, int nv, int nvp, uint8_t* rec) {
    const int lane = threadIdx.x & 31;
    const int64_t wid = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int KSB = K / 256;
    if (wid >= (int64_t)nvp * KSB) return;
    const int t = (int)(wid / KSB), sb = (int)(wid % KSB);
    float xs[8];
    if (t < nv) {
        const float4* p = reinterpret_cast<const float4*>(x + (int64_t)t * ldx + (int64_t)sb * 256 + 8 * lane);
        const float4 a = p[0], b = p[1];
        xs[0] = a.x; xs[1] = a.y; xs[2] = a.z; xs[3] = a.w;
        xs[4] = b.x; xs[5] = b.y; xs[6] = b.z; xs[7] = b.w;
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) xs[i] = 0.0f;
    }
    kx_emit_sb(rec, K, nvp, t, sb, xs);
}

// Shared memory of one stage (one super-block): the 8 sub-blocks' h and l
// tiles (128 rows x 32 k each: K-half 0 then K-half 1, 2 KB apart), the
// min tile (K-half 0 = m_0..m_7, 0; K-half 1 = a zero area never copied
// into), then the records' 8 limb tiles and 2 min-term tiles.
constexpr int KX_AH = 0, KX_AL = 32768, KX_AM = 65536, KX_Z = 67584, KX_B = 69632;
constexpr int KX_STAGE = KX_B + 10 * 96 * 32;   // 100352
constexpr int KX_SMEM = 2 * KX_STAGE + 128;
constexpr int KX_EPI = 16;                      // epilogue warps: 4 per tensor-memory lane quadrant
constexpr int KX_THREADS = 64 + 32 * KX_EPI;    // loader warp, MMA warp, epilogue warps
constexpr int KX_TMEM_COLS = 512;               // h, l, min-Xl, min-Xh accumulators at 0, 128, 256, 384

__device__ __forceinline__ bool kx_wait(uint64_t* bar, uint32_t parity, unsigned int* err, unsigned int code) {
    for (int i = 0; i < 32; ++i)
        if (mbar_try_wait(bar, parity)) return true;
    return mbar_wait_bounded(bar, parity, err, code);
}

// CTA = 128 rows (row0 + 128 blockIdx.x ..) x all vectors x the
// super-blocks of split blockIdx.y.  Per super-block:
//   warp 0      one lane bulk-copies the stage (33 copies: 32 K-half runs
//               of h and l, the min tile, the records) into one of 2 stages;
//   warp 1      one thread issues, per sub-block j, the MMAs h_j x B_j and
//               l_j x B_j into the h and l accumulators (Q4_K: then the min
//               tile against the two min-term tiles), all onto the preset
//               magic value, and commits to the stage's "empty" and the
//               accumulators' "full" barriers;
//   warps 2-17  read the four accumulators back (warp w: lanes 32 (w % 4),
//               a quarter of the columns), reset them, release them, and add
//               s_v (d (F h + l) - dmin (m1 + 256 m2)) to fp32 accumulators
//               per (vector, limb).
// The copies of the next super-block overlap the MMAs and the readout.
template <int TYPE, int NVG>
__global__ void __launch_bounds__(KX_THREADS, 1)
    kx_mma_kernel(const uint8_t* base, int64_t pitch, int64_t row0, int n, int K, size_t m_off, size_t f_off,
                  const uint8_t* rec, int nv, int S, float* part, int* ctr, const float* bias, float* y, int ldy,
                  unsigned int* err) {
    constexpr bool Q4 = TYPE == BREW_TYPE_Q4_K;
    constexpr int NVP = 16 * NVG, NC = 3 * NVP;   // vectors and limb columns of the MMA
    constexpr int CW = NC / (KX_EPI / 4), TPW = CW / 3;   // columns and vectors per epilogue warp
    constexpr int NACC = Q4 ? 4 : 2;
    extern __shared__ __align__(1024) uint8_t smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + 2 * KX_STAGE);
    uint64_t* empty = full + 2;
    uint64_t* tfull = empty + 2;
    uint64_t* tempty = tfull + 1;
    uint32_t* tslot = reinterpret_cast<uint32_t*>(tempty + 1);
    __shared__ int s_last;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int KSB = K / 256, split = blockIdx.y;
    const int sb0 = (int)((int64_t)split * KSB / S), sb1 = (int)((int64_t)(split + 1) * KSB / S);
    const int64_t r0 = row0 + (int64_t)blockIdx.x * KX_TM;   // the CTA's first row in the family
    const int rec_tile = 10 * NC * 32;
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tslot)),
                     "r"(KX_TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (tid == 0) {
        for (int i = 0; i < 2; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1);
        }
        mbar_init(tfull, 1);
        mbar_init(tempty, KX_EPI);
        fence_mbar_init();
    }
    if (Q4) {   // the min tile's second K-half: zeros, read by the tensor cores
        for (int i = tid; i < 2 * 512; i += KX_THREADS)
            reinterpret_cast<uint32_t*>(smem + (i / 512) * KX_STAGE + KX_Z)[i % 512] = 0u;
        fence_proxy_async();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;
    if (warp == 0) {
        // ---------------------------------- loader ----------------------------------
        if (lane == 0) {
            const uint64_t pol = l2_evict_first_policy();
            const uint8_t* hp = base;
            const uint8_t* lp = base + (size_t)K * pitch;
            const uint32_t bbytes = (Q4 ? 10 : 8) * NC * 32;
            const uint32_t bytes = 16 * 4096 + (Q4 ? 2048 : 0) + bbytes;
            int it = 0;
            for (int sb = sb0; sb < sb1; ++sb, ++it) {
                const int st = it & 1;
                if (it >= 2 && !kx_wait(&empty[st], ((it >> 1) - 1) & 1, err, BREW_DEVERR_TIMEOUT_EMPTY)) break;
                uint8_t* s0 = smem + st * KX_STAGE;
                mbar_arrive_expect_tx(&full[st], bytes);
                for (int hk = 0; hk < 16; ++hk) {   // K-half hk of the super-block: sub-block hk / 2
                    const int64_t o = ((int64_t)(16 * sb + hk) * pitch + r0) * 16;
                    const int so = (hk >> 1) * 4096 + (hk & 1) * 2048;
                    bulk_g2s_hint(s0 + KX_AH + so, hp + o, 2048, &full[st], pol);
                    bulk_g2s_hint(s0 + KX_AL + so, lp + o, 2048, &full[st], pol);
                }
                if (Q4) bulk_g2s_hint(s0 + KX_AM, base + m_off + ((int64_t)sb * pitch + r0) * 16, 2048, &full[st], pol);
                bulk_g2s(s0 + KX_B, rec + (int64_t)sb * rec_tile, bbytes, &full[st]);
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        // ------------------------------------ MMA ------------------------------------
        if (lane == 0) {
            constexpr uint32_t idesc = umma_idesc_s8(KX_TM, NC);
            int it = 0;
            for (int sb = sb0; sb < sb1; ++sb, ++it) {
                const int st = it & 1;
                if (!kx_wait(&full[st], (it >> 1) & 1, err, BREW_DEVERR_TIMEOUT_FULL)) break;
                if (!kx_wait(tempty, it & 1, err, BREW_DEVERR_TIMEOUT_EMPTY)) break;
                tc_fence_after();
                const uint32_t s0 = smem_u32(smem + st * KX_STAGE);
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const uint64_t bd = umma_desc_k(s0 + KX_B + j * NC * 32, 128, 256);
                    umma_s8(tmem, umma_desc_k(s0 + KX_AH + j * 4096, 2048, 128), bd, idesc, 1u);
                    umma_s8(tmem + 128, umma_desc_k(s0 + KX_AL + j * 4096, 2048, 128), bd, idesc, 1u);
                }
                if (Q4) {
                    const uint64_t ad = umma_desc_k(s0 + KX_AM, 2048, 128);
                    umma_s8(tmem + 256, ad, umma_desc_k(s0 + KX_B + 8 * NC * 32, 128, 256), idesc, 1u);
                    umma_s8(tmem + 384, ad, umma_desc_k(s0 + KX_B + 9 * NC * 32, 128, 256), idesc, 1u);
                }
                umma_commit(&empty[st]);
                umma_commit(tfull);
            }
        }
        __syncwarp();
    } else {
        // ---------------------------------- epilogue ----------------------------------
        const int q = warp & 3, hh = (warp - 2) >> 2;
        const int lrow = (int)(r0 - row0) + 32 * q + lane;   // row within the launch
        const int64_t frow = r0 + 32 * q + lane;             // row within the family (< pitch)
        const uint32_t tq = tmem + ((uint32_t)(32 * q) << 16) + CW * hh;
#pragma unroll
        for (int a = 0; a < NACC; ++a) {   // exactly this warp's CW columns (a multiple of 4)
#pragma unroll
            for (int c = 0; c + 8 <= CW; c += 8) tmem_st8_const(tq + 128 * a + c, TC_MAGIC);
            if (CW % 8) tmem_st4_const(tq + 128 * a + CW - 4, TC_MAGIC);
        }
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(tempty);
        uint64_t acc[TPW / 2][3];   // vector pairs x limbs (hi, mid, lo)
#pragma unroll
        for (int p = 0; p < TPW / 2; ++p) acc[p][0] = acc[p][1] = acc[p][2] = 0ull;
        const uint64_t negc = f2_packf(-TC_MAGIC_F, -TC_MAGIC_F);
        const uint64_t kF = Q4 ? f2_packf(8.0f, 8.0f) : f2_packf(64.0f, 64.0f);
        const uint64_t k256 = f2_packf(256.0f, 256.0f), k65536 = f2_packf(65536.0f, 65536.0f);
        const float2* fpl = reinterpret_cast<const float2*>(base + f_off);
        const float* scl = reinterpret_cast<const float*>(rec + (int64_t)KSB * rec_tile);
        float2 fr = sb0 < sb1 ? __ldg(fpl + (int64_t)sb0 * pitch + frow) : make_float2(0.0f, 0.0f);
        int it = 0;
        for (int sb = sb0; sb < sb1; ++sb, ++it) {
            bool ok = kx_wait(tfull, it & 1, err, BREW_DEVERR_TIMEOUT_FULL);
            ok = __all_sync(0xffffffffu, ok);   // tcgen05.ld / st are warp-collective
            if (!ok) break;
            tc_fence_after();
            float sv[TPW];
#pragma unroll
            for (int g = 0; g < TPW / 4; ++g) {
                const float4 s4 = __ldg(reinterpret_cast<const float4*>(scl + (int64_t)sb * NVP + TPW * hh) + g);
                sv[4 * g] = s4.x;
                sv[4 * g + 1] = s4.y;
                sv[4 * g + 2] = s4.z;
                sv[4 * g + 3] = s4.w;
            }
            const uint64_t d2 = f2_packf(fr.x, fr.x), nm2 = f2_packf(-fr.y, -fr.y);
            if (sb + 1 < sb1) fr = __ldg(fpl + (int64_t)(sb + 1) * pitch + frow);
#pragma unroll
            for (int e = 0; e < CW / 12; ++e) {   // 12 columns (2 vector pairs) at a time
                const uint32_t ta = tq + 12 * e;
                uint32_t v[NACC][12];
#pragma unroll
                for (int a = 0; a < NACC; ++a) {
                    tmem_ld8(ta + 128 * a, v[a]);
                    tmem_ld4(ta + 128 * a + 8, v[a] + 8);
                }
                tmem_ld_wait();
#pragma unroll
                for (int a = 0; a < NACC; ++a) {
                    tmem_st8_const(ta + 128 * a, TC_MAGIC);
                    tmem_st4_const(ta + 128 * a + 8, TC_MAGIC);
                }
#pragma unroll
                for (int pp = 0; pp < 2; ++pp) {
                    const int p = 2 * e + pp;
                    const uint64_t s2 = f2_packf(sv[2 * p], sv[2 * p + 1]);
#pragma unroll
                    for (int l = 0; l < 3; ++l) {
                        const int c = 6 * pp + 2 * l;
                        const uint64_t H = f2_add(f2_pack(v[0][c], v[0][c + 1]), negc);
                        const uint64_t L = f2_add(f2_pack(v[1][c], v[1][c + 1]), negc);
                        const uint64_t val = f2_fma(H, kF, L);   // F h + l
                        uint64_t tv;
                        if (Q4) {
                            const uint64_t M1 = f2_add(f2_pack(v[2 % NACC][c], v[2 % NACC][c + 1]), negc);
                            const uint64_t M2 = f2_add(f2_pack(v[3 % NACC][c], v[3 % NACC][c + 1]), negc);
                            tv = f2_fma(d2, val, f2_mul(nm2, f2_fma(M2, k256, M1)));
                        } else {
                            tv = f2_mul(d2, val);
                        }
                        acc[p][l] = f2_fma(s2, tv, acc[p][l]);
                    }
                }
            }
            tmem_st_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(tempty);
        }
        // limbs meet: (lo + mid 2^8) + hi 2^16
        const int64_t npad = (int64_t)gridDim.x * KX_TM;
#pragma unroll
        for (int p = 0; p < TPW / 2; ++p) {
            const uint64_t r = f2_fma(acc[p][0], k65536, f2_fma(acc[p][1], k256, acc[p][2]));
            const float a0 = __uint_as_float((uint32_t)r), a1 = __uint_as_float((uint32_t)(r >> 32));
            const int tk = TPW * hh + 2 * p;
            if (lrow < n) {
                if (S == 1) {
                    const float bv = bias ? __ldg(bias + frow) : 0.0f;
                    if (tk < nv) y[(int64_t)tk * ldy + lrow] = bias ? a0 + bv : a0;
                    if (tk + 1 < nv) y[(int64_t)(tk + 1) * ldy + lrow] = bias ? a1 + bv : a1;
                } else {
                    if (tk < nv) part[((int64_t)split * nv + tk) * npad + lrow] = a0;
                    if (tk + 1 < nv) part[((int64_t)split * nv + tk + 1) * npad + lrow] = a1;
                }
            }
        }
        if (S > 1) {   // the last CTA of this row group adds the splits in split order
            __threadfence();
            asm volatile("bar.sync 1, %0;" ::"n"(32 * KX_EPI) : "memory");
            if (tid == 64) {
                const int old = atomicAdd(&ctr[blockIdx.x], 1);
                s_last = old == S - 1;
                if (s_last) ctr[blockIdx.x] = 0;   // every split has arrived: ready for the next launch
            }
            asm volatile("bar.sync 1, %0;" ::"n"(32 * KX_EPI) : "memory");
            if (s_last) {
                __threadfence();
                const int rbase = (int)(r0 - row0);
                for (int i = tid - 64; i < nv * KX_TM; i += 32 * KX_EPI) {
                    const int tk = i / KX_TM, lr = rbase + i % KX_TM;
                    if (lr >= n) continue;
                    float sum = 0.0f;
                    for (int sp = 0; sp < S; ++sp) sum += __ldcg(part + ((int64_t)sp * nv + tk) * npad + lr);
                    y[(int64_t)tk * ldy + lr] = bias ? sum + __ldg(bias + row0 + lr) : sum;
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(KX_TMEM_COLS)
                     : "memory");
    }
}

template <int TYPE, int NVG>
int kx_launch_t(const uint8_t* base, int64_t N, int64_t row0, int n, int K, const uint8_t* rec, int nv, int S,
                float* part, int* ctr, const float* bias, float* y, int ldy, unsigned int* err, cudaStream_t stream) {
    static uint64_t attr_devs = 0;   // devices whose attribute is set
    int dev = 0;
    BREW_CUDA(cudaGetDevice(&dev));
    if (dev < 64 && !(attr_devs >> dev & 1)) {
        BREW_CUDA(cudaFuncSetAttribute(kx_mma_kernel<TYPE, NVG>, cudaFuncAttributeMaxDynamicSharedMemorySize, KX_SMEM));
        attr_devs |= 1ull << dev;
    }
    const dim3 grid((unsigned)((n + KX_TM - 1) / KX_TM), (unsigned)S);
    kx_mma_kernel<TYPE, NVG><<<grid, KX_THREADS, KX_SMEM, stream>>>(base, kx_pitch(N), row0, n, K, kx_m_off(N, K),
                                                                    kx_f_off(TYPE, N, K), rec, nv, S, part, ctr, bias,
                                                                    y, ldy, err);
    BREW_CUDA(cudaGetLastError());
    count_launch();
    return BREW_OK;
}

}  // namespace

int kq_splits(int64_t K, int64_t n_basis) {
    // as many splits as keep the family's 128-row groups within one wave of
    // one CTA per SM of a B200 (148 SMs), at least two super-blocks each
    constexpr int64_t wave = 148;
    const int64_t groups = std::max<int64_t>(1, (n_basis + KX_TM - 1) / KX_TM), ksb = K / 256;
    int64_t s = wave / groups;
    s = std::min<int64_t>(s, std::max<int64_t>(1, ksb / 2));
    return (int)std::max<int64_t>(1, s);
}

int kx_pack_launch(int type, const uint8_t* w, int64_t rows, int K, uint8_t* base, int64_t N, int64_t row_off,
                   cudaStream_t stream) {
    BREW_CHECK((type == BREW_TYPE_Q4_K || type == BREW_TYPE_Q6_K) && K % 256 == 0 && K > 0 && rows > 0 &&
                   row_off >= 0 && row_off + rows <= N,
               BREW_ERR_INVALID_ARG, "K-quant expand: type %d rows=%lld K=%d", type, (long long)rows, K);
    const int64_t cnt = rows * (K / 32);
    const unsigned blocks = (unsigned)((cnt + 255) / 256);
    if (type == BREW_TYPE_Q4_K)
        kx_pack_kernel<BREW_TYPE_Q4_K><<<blocks, 256, 0, stream>>>(w, rows, K, base, kx_pitch(N), row_off,
                                                                   kx_m_off(N, K), kx_f_off(type, N, K));
    else
        kx_pack_kernel<BREW_TYPE_Q6_K><<<blocks, 256, 0, stream>>>(w, rows, K, base, kx_pitch(N), row_off,
                                                                   kx_m_off(N, K), kx_f_off(type, N, K));
    BREW_CUDA(cudaGetLastError());
    count_launch();
    return BREW_OK;
}

int kx_prep_launch(const float* x, int ldx, int K, int nv, uint8_t* rec, cudaStream_t stream) {
    BREW_CHECK(nv >= 1 && nv <= KX_MAX_VECTORS && K % 256 == 0 && K > 0 && ldx % 4 == 0 &&
                   (reinterpret_cast<uintptr_t>(x) & 15) == 0,
               BREW_ERR_INVALID_ARG, "K-quant records: nv=%d K=%d ldx=%d (x 16-byte aligned)", nv, K, ldx);
    const int nvp = (nv + 15) / 16 * 16;
    const int64_t warps = (int64_t)nvp * (K / 256);
    kx_prep_kernel<<<(unsigned)((warps * 32 + 255) / 256), 256, 0, stream>>>(x, ldx, K, nv, nvp, rec);
    BREW_CUDA(cudaGetLastError());
    count_launch();
    return BREW_OK;
}

int kx_mma_launch(int type, const uint8_t* base, int64_t N, int64_t row0, int n, int K, const uint8_t* rec, int nv,
                  int splits, float* part, int* ctr, const float* bias, float* y, int ldy, unsigned int* err,
                  cudaStream_t stream) {
    BREW_CHECK(nv >= 1 && nv <= KX_MAX_VECTORS && K % 256 == 0 && K > 0 && n > 0 && row0 >= 0 && row0 + n <= N &&
                   splits >= 1 && splits <= K / 256 && (splits == 1 || (part && ctr)),
               BREW_ERR_INVALID_ARG, "K-quant MMA matvec: nv=%d n=%d K=%d splits=%d", nv, n, K, splits);
    BREW_CHECK(type == BREW_TYPE_Q4_K || type == BREW_TYPE_Q6_K, BREW_ERR_INVALID_ARG, "K-quant MMA matvec: type %d",
               type);
    const bool q4 = type == BREW_TYPE_Q4_K;
    if (nv <= 16)
        return q4 ? kx_launch_t<BREW_TYPE_Q4_K, 1>(base, N, row0, n, K, rec, nv, splits, part, ctr, bias, y, ldy, err, stream)
                  : kx_launch_t<BREW_TYPE_Q6_K, 1>(base, N, row0, n, K, rec, nv, splits, part, ctr, bias, y, ldy, err, stream);
    return q4 ? kx_launch_t<BREW_TYPE_Q4_K, 2>(base, N, row0, n, K, rec, nv, splits, part, ctr, bias, y, ldy, err, stream)
              : kx_launch_t<BREW_TYPE_Q6_K, 2>(base, N, row0, n, K, rec, nv, splits, part, ctr, bias, y, ldy, err, stream);
}

}  // namespace brew
