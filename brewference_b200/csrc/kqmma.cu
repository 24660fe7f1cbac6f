// kqmma.cu — K-quant matvec on the int8 tensor cores (layouts in kqmma.cuh).
#include "brew_internal.cuh"
#include "kqmma.cuh"
#include "mv_device.cuh"
#include "prep.cuh"

namespace brew {
namespace {

__device__ __forceinline__ float kq_half(const uint8_t* p) {
    return half_bits_to_float((uint16_t)(p[0] | (p[1] << 8)));
}

// 6-bit scale and min of Q4_K sub-block s (GGML's get_scale_min_k4).
__device__ __forceinline__ void q4k_scale_min(const uint8_t* sb, int s, int& sc, int& m) {
    if (s < 4) {
        sc = sb[s] & 63;
        m = sb[s + 4] & 63;
    } else {
        sc = (sb[s + 4] & 0xF) | ((sb[s - 4] >> 6) << 4);
        m = (sb[s + 4] >> 4) | ((sb[s] >> 6) << 4);
    }
}

// One thread per (row, 32-element sub-block): decodes the sub-block's
// quants and factors and writes them at their places in the tile-superblock.
template <int TYPE>
__global__ void kq_pack_kernel(const uint8_t* w, int64_t N, int K, uint8_t* out) {
    constexpr int TSB = kq_sb_bytes(TYPE), SB = TYPE == BREW_TYPE_Q4_K ? 144 : 210;
    const int KB = K / 32, KSB = K / 256;
    const int64_t rows = (N + 15) / 16 * 16;
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= rows * KB) return;
    const int64_t row = i / KB;
    const int kb = (int)(i % KB), sb = kb / 8, j = kb % 8;
    const int rt = (int)(row % 16), g = rt % 8, upper = rt / 8;
    uint8_t* base = out + ((row / 16) * KSB + sb) * TSB;
    int q[32];
    int s0 = 0, s1 = 0;       // Q4_K: sc, m; Q6_K: scales of the two halves
    float f0 = 0.0f, f1 = 0.0f;   // Q4_K: d, dmin; Q6_K: d
    if (row < N) {
        const uint8_t* blk = w + row * (int64_t)KSB * SB + (int64_t)sb * SB;
        if (TYPE == BREW_TYPE_Q4_K) {
            q4k_scale_min(blk + 4, j, s0, s1);
            f0 = kq_half(blk);
            f1 = kq_half(blk + 2);
            for (int k = 0; k < 32; ++k) q[k] = (blk[16 + 32 * (j / 2) + k] >> (4 * (j & 1))) & 15;
        } else {
            f0 = kq_half(blk + 208);
            s0 = (int8_t)blk[192 + 2 * j];
            s1 = (int8_t)blk[192 + 2 * j + 1];
            for (int k = 0; k < 32; ++k) {
                const int r = 32 * j + k, h = r / 128, rr = r % 128, grp = rr / 32, l = rr % 32;
                const int lq = blk[64 * h + (grp & 1) * 32 + l];
                const int low = grp < 2 ? (lq & 15) : (lq >> 4);
                const int high = (blk[128 + 32 * h + l] >> (2 * grp)) & 3;
                q[k] = (low | (high << 4)) - 32;
            }
        }
    } else {
        for (int k = 0; k < 32; ++k) q[k] = 0;
    }
    if (TYPE == BREW_TYPE_Q4_K) {
        for (int t = 0; t < 4; ++t)
            for (int jj = 0; jj < 4; ++jj)
                base[j * 256 + (g * 4 + t) * 8 + 4 * upper + jj] = (uint8_t)(q[4 * t + jj] | (q[16 + 4 * t + jj] << 4));
        base[2048 + j * 32 + g * 4 + 2 * upper] = (uint8_t)s0;
        base[2048 + j * 32 + g * 4 + 2 * upper + 1] = (uint8_t)s1;
        if (j == 0) {
            float* f = reinterpret_cast<float*>(base + 2304 + 16 * g + 8 * upper);
            f[0] = f0;
            f[1] = f1;
        }
    } else {
        for (int k = 0; k < 32; ++k) {
            const int t = (k % 16) / 4, half = k / 16;
            base[j * 512 + (g * 4 + t) * 16 + 4 * (upper + 2 * half) + (k % 4)] = (uint8_t)(int8_t)q[k];
        }
        base[4096 + j * 32 + g * 4 + 2 * upper] = (uint8_t)(int8_t)s0;
        base[4096 + j * 32 + g * 4 + 2 * upper + 1] = (uint8_t)(int8_t)s1;
        if (j == 0) reinterpret_cast<float*>(base + 4352 + 8 * g)[upper] = f0;
    }
}

constexpr int KQ_XS_OFF = 12288, KQ_S_OFF = 13056;

__device__ __forceinline__ uint64_t kq_pack8(const int (&v)[8]) {
    uint32_t lo = 0u, hi = 0u;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        lo |= (uint32_t)(v[i] & 255) << (8 * i);
        hi |= (uint32_t)(v[4 + i] & 255) << (8 * i);
    }
    return (uint64_t)lo | ((uint64_t)hi << 32);
}

// One warp per (vector, super-block): lane i holds elements 8i .. 8i + 7
// (sub-block i / 4).  Vectors nv .. 16 ceil(nv / 16) - 1 are written as zeros.
__global__ void kq_prep_kernel(const float* x, int ldx, int K, int nv, int nvp, uint8_t* rec) {
    const int lane = threadIdx.x & 31;
    const int64_t wid = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int KSB = K / 256;
    if (wid >= (int64_t)nvp * KSB) return;
    const int v = (int)(wid / KSB), sb = (int)(wid % KSB);
    const int vg = v / 16, vl = v % 16;
    float xs[8];
    if (v < nv) {
        const float4* p = reinterpret_cast<const float4*>(x + (int64_t)v * ldx + (int64_t)sb * 256 + 8 * lane);
        const float4 a = p[0], b = p[1];
        xs[0] = a.x; xs[1] = a.y; xs[2] = a.z; xs[3] = a.w;
        xs[4] = b.x; xs[5] = b.y; xs[6] = b.z; xs[7] = b.w;
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) xs[i] = 0.0f;
    }
    float am = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) am = fmaxf(am, fabsf(xs[i]));
    am = warp_max(am);
    const float inv = am > 0.0f ? PREP_RANGE / am : 0.0f;
    int hi[8], mid[8], lo[8];
    int sh = 0, sm = 0, sl = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int q = __float2int_rn(xs[i] * inv);
        lo[i] = ((q + 128) & 255) - 128;
        const int q1 = (q - lo[i]) >> 8;
        mid[i] = ((q1 + 128) & 255) - 128;
        hi[i] = (q1 - mid[i]) >> 8;
        sh += hi[i];
        sm += mid[i];
        sl += lo[i];
    }
    uint8_t* r = rec + ((int64_t)vg * KSB + sb) * KQ_REC;
    const int j = lane >> 2, k0 = 8 * (lane & 3);
    const int phys = (k0 >> 4) ^ (vl & 1);   // odd vectors: halves swapped
    uint8_t* row0 = r + j * 1536 + (3 * vl) * 32 + phys * 16 + (k0 & 15);
    *reinterpret_cast<uint64_t*>(row0) = kq_pack8(hi);
    *reinterpret_cast<uint64_t*>(row0 + 32) = kq_pack8(mid);
    *reinterpret_cast<uint64_t*>(row0 + 64) = kq_pack8(lo);
    // sub-block sums over its 4 lanes
#pragma unroll
    for (int o = 1; o < 4; o <<= 1) {
        sh += __shfl_xor_sync(0xffffffffu, sh, o);
        sm += __shfl_xor_sync(0xffffffffu, sm, o);
        sl += __shfl_xor_sync(0xffffffffu, sl, o);
    }
    if ((lane & 3) == 0) {
        const int X[3] = {sh, sm, sl};
#pragma unroll
        for (int l = 0; l < 3; ++l) {
            const int xl = ((X[l] + 128) & 255) - 128;
            const int xh = (X[l] - xl) >> 8;
            uint8_t* xr = r + KQ_XS_OFF + (3 * vl + l) * 16;
            xr[j] = (uint8_t)xl;
            xr[8 + j] = (uint8_t)xh;
        }
    }
    if (lane == 0) reinterpret_cast<float*>(r + KQ_S_OFF)[vl] = am / PREP_RANGE;
}

// int8 MMA over 16 elements: a0 / a1 hold rows g / g + 8, k = 4t .. 4t + 3;
// b holds k = 4t .. 4t + 3 of column g.
__device__ __forceinline__ void mma_s8s8_k16(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t b) {
    asm("mma.sync.aligned.m16n8k16.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%7,%8,%9,%10};"
        : "=r"(c[0]), "=r"(c[1]), "=r"(c[2]), "=r"(c[3])
        : "r"(a0), "r"(a1), "r"(b), "r"(0), "r"(0), "r"(0), "r"(0));
}

__device__ __forceinline__ uint32_t lds_u32(const uint8_t* p) { return *reinterpret_cast<const uint32_t*>(p); }

constexpr int KQ_TILES = 8;                  // 16-row tiles per CTA
constexpr int KQ_SMEM_BUDGET = 200 * 1024;   // ring of stages

template <int TYPE>
struct KqGeo {
    static constexpr int TSB = kq_sb_bytes(TYPE);
    static constexpr int W_BYTES = KQ_TILES * TSB;
    static constexpr int STAGE = W_BYTES + KQ_REC;   // one super-block: weights of 8 tiles, x records of 16 vectors
    static constexpr int NS = KQ_SMEM_BUDGET / STAGE < 6 ? KQ_SMEM_BUDGET / STAGE : 6;
    static constexpr int SMEM = NS * STAGE + 2 * NS * 8;
    static constexpr int CONSUMERS = KQ_TILES;        // warp a: tile a
    static constexpr int THREADS = 32 * (CONSUMERS + 1);
    static_assert(STAGE % 16 == 0 && NS >= 2, "stage geometry");
};

// Bounded wait with a short poll first (the hand-off is usually imminent).
__device__ __forceinline__ bool kq_wait(uint64_t* bar, uint32_t parity, unsigned int* err, unsigned int code) {
    for (int i = 0; i < 16; ++i)
        if (mbar_try_wait(bar, parity)) return true;
    return mbar_wait_bounded(bar, parity, err, code);
}

// CTA = 8 16-row tiles (128 rows) x one group of 16 vectors (vg) x the
// super-blocks [sb0, sb1) of split blockIdx.y; blockIdx.x = tg * nvg + vg,
// so the CTAs of the vector groups of one row group run side by side and
// the second reads the weights from L2.  The last warp streams each
// super-block's tile-superblocks and x records into a ring of shared-memory
// stages with bulk copies; consumer warp a multiplies tile a by the 16
// vectors (8 n8 tiles of 2 vectors x 4 limb columns): per sub-block one MMA
// (two half MMAs for Q6_K) per n8 tile, the sub-block scales applied to the
// int32 results with integer multiply-adds, and per super-block one fp32
// step (scales d, dmin and the vector's scale).  With splits > 1, each CTA
// writes its partial sums and the last CTA of a (row group, vector group)
// adds the splits in split order.
template <int TYPE>
__global__ void __launch_bounds__(KqGeo<TYPE>::THREADS, 1)
    kq_mma_kernel(const uint8_t* pk, int tiles, int KSB, int N, const uint8_t* rec, int nv, int nvg, int S,
                  float* part, int* ctr, float* y, int ldy, unsigned int* err) {
    using G = KqGeo<TYPE>;
    constexpr int VG = 1;
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + G::NS * G::STAGE);
    uint64_t* empty = full + G::NS;
    __shared__ int s_last;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tg = blockIdx.x / nvg, vg = blockIdx.x % nvg, split = blockIdx.y;
    const int tile0 = tg * KQ_TILES, ntile = min(KQ_TILES, tiles - tile0);
    const int sb0 = (int)((int64_t)split * KSB / S), sb1 = (int)((int64_t)(split + 1) * KSB / S);
    if (threadIdx.x == 0) {
        for (int i = 0; i < G::NS; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], G::CONSUMERS);
        }
        fence_mbar_init();
    }
    __syncthreads();
    if (warp == G::CONSUMERS) {
        // ---------------------------------- producer ----------------------------------
        if (lane == 0) {
            const uint64_t pol = l2_evict_first_policy();
            const uint32_t bytes = (uint32_t)(ntile * G::TSB + VG * KQ_REC);
            int it = 0;
            for (int sb = sb0; sb < sb1; ++sb, ++it) {
                const int st = it % G::NS;
                if (it >= G::NS && !kq_wait(&empty[st], ((it / G::NS) - 1) & 1, err, BREW_DEVERR_TIMEOUT_EMPTY)) break;
                uint8_t* dst = smem + st * G::STAGE;
                mbar_arrive_expect_tx(&full[st], bytes);
                for (int a = 0; a < ntile; ++a)
                    bulk_g2s_hint(dst + a * G::TSB, pk + ((int64_t)(tile0 + a) * KSB + sb) * G::TSB, G::TSB, &full[st],
                                  pol);
                bulk_g2s(dst + G::W_BYTES, rec + ((int64_t)vg * KSB + sb) * KQ_REC, KQ_REC, &full[st]);
            }
        }
        return;
    }
    // ---------------------------------- consumers ----------------------------------
    const int a = warp;
    const int g = lane >> 2, t = lane & 3;
    const bool tile_ok = a < ntile;
    // B column g of n8 tile n: vector 2n + par, limb lB (3: the zero column)
    const int par = g >> 2, lB = g & 3;
    const bool hasB = lB < 3;
    const uint32_t rowB = (uint32_t)(3 * par + lB) * 32;
    const uint32_t boff0 = rowB + (par ? 16u : 0u) + 4 * t, boff1 = rowB + (par ? 0u : 16u) + 4 * t;
    const uint32_t xoff = KQ_XS_OFF + (uint32_t)(3 * par + lB) * 16 + 4 * t;
    // accumulator columns 2t, 2t + 1 belong to vector 2n + (t >> 1)
    const uint32_t soff = KQ_S_OFF + 4 * (t >> 1);
    float accf[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n) accf[n][0] = accf[n][1] = accf[n][2] = accf[n][3] = 0.0f;
    int it = 0;
    for (int sb = sb0; sb < sb1; ++sb, ++it) {
        const int st = it % G::NS;
        const bool ok = __all_sync(0xffffffffu, kq_wait(&full[st], (it / G::NS) & 1, err, BREW_DEVERR_TIMEOUT_FULL));
        if (!ok) break;
        const uint8_t* W = smem + st * G::STAGE + a * G::TSB;
        const uint8_t* R = smem + st * G::STAGE + G::W_BYTES;
        if (tile_ok) {
            int acci[8][4];
#pragma unroll
            for (int n = 0; n < 8; ++n) acci[n][0] = acci[n][1] = acci[n][2] = acci[n][3] = 0;
#pragma unroll 2
            for (int j = 0; j < 8; ++j) {
                const uint8_t* Rj = R + j * 1536;
                if (TYPE == BREW_TYPE_Q4_K) {
                    const uint2 Wq = *reinterpret_cast<const uint2*>(W + j * 256 + lane * 8);
                    const uint32_t a0 = Wq.x & 0x0F0F0F0Fu, a1 = Wq.y & 0x0F0F0F0Fu;
                    const uint32_t a2 = (Wq.x >> 4) & 0x0F0F0F0Fu, a3 = (Wq.y >> 4) & 0x0F0F0F0Fu;
                    const uint32_t scm = lds_u32(W + 2048 + j * 32 + g * 4);
                    const int sc0 = (int)(scm & 0xFFu), sc1 = (int)((scm >> 16) & 0xFFu);
#pragma unroll
                    for (int n = 0; n < 8; ++n) {
                        const uint32_t b0 = hasB ? lds_u32(Rj + 192 * n + boff0) : 0u;
                        const uint32_t b1 = hasB ? lds_u32(Rj + 192 * n + boff1) : 0u;
                        int c[4];
                        mma_u8s8(c, a0, a1, a2, a3, b0, b1);
                        acci[n][0] += sc0 * c[0];
                        acci[n][1] += sc0 * c[1];
                        acci[n][2] += sc1 * c[2];
                        acci[n][3] += sc1 * c[3];
                    }
                } else {
                    const uint4 A = *reinterpret_cast<const uint4*>(W + j * 512 + lane * 16);
                    const uint32_t scs = lds_u32(W + 4096 + j * 32 + g * 4);
                    const int slo0 = (int)(int8_t)(scs & 0xFFu), shi0 = (int)(int8_t)((scs >> 8) & 0xFFu);
                    const int slo1 = (int)(int8_t)((scs >> 16) & 0xFFu), shi1 = (int)(int8_t)(scs >> 24);
#pragma unroll
                    for (int n = 0; n < 8; ++n) {
                        const uint32_t b0 = hasB ? lds_u32(Rj + 192 * n + boff0) : 0u;
                        const uint32_t b1 = hasB ? lds_u32(Rj + 192 * n + boff1) : 0u;
                        int cl[4], ch[4];
                        mma_s8s8_k16(cl, A.x, A.y, b0);   // k 0..15
                        mma_s8s8_k16(ch, A.z, A.w, b1);   // k 16..31
                        acci[n][0] += slo0 * cl[0] + shi0 * ch[0];
                        acci[n][1] += slo0 * cl[1] + shi0 * ch[1];
                        acci[n][2] += slo1 * cl[2] + shi1 * ch[2];
                        acci[n][3] += slo1 * cl[3] + shi1 * ch[3];
                    }
                }
            }
            // the super-block's fp32 step
            if (TYPE == BREW_TYPE_Q4_K) {
                const float4 f = *reinterpret_cast<const float4*>(W + 2304 + 16 * g);   // d, dmin of rows g, g + 8
                // min term: A = m_j of rows g, g + 8 at k = 4 (t & 1) + 0..3,
                // once against Xl (lanes t < 2) and once against Xh (t >= 2)
                uint32_t mg = 0u, mg8 = 0u;
#pragma unroll
                for (int jj = 0; jj < 4; ++jj) {
                    const uint32_t wv = lds_u32(W + 2048 + (4 * (t & 1) + jj) * 32 + g * 4);
                    mg |= ((wv >> 8) & 0xFFu) << (8 * jj);
                    mg8 |= ((wv >> 24) & 0xFFu) << (8 * jj);
                }
                const uint32_t al = t < 2 ? mg : 0u, al8 = t < 2 ? mg8 : 0u;
                const uint32_t ah = t < 2 ? 0u : mg, ah8 = t < 2 ? 0u : mg8;
#pragma unroll
                for (int n = 0; n < 8; ++n) {
                    const uint32_t bx = hasB ? lds_u32(R + xoff + 96 * n) : 0u;
                    int cl[4], ch[4];
                    mma_s8s8_k16(cl, al, al8, bx);
                    mma_s8s8_k16(ch, ah, ah8, bx);
                    const float s = *reinterpret_cast<const float*>(R + soff + 8 * n);
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const float d = i < 2 ? f.x : f.z, dm = i < 2 ? f.y : f.w;
                        const float msum = (float)(cl[i] + 256 * ch[i]);
                        accf[n][i] = fmaf(s, fmaf(d, (float)acci[n][i], -dm * msum), accf[n][i]);
                    }
                }
            } else {
                const float2 f = *reinterpret_cast<const float2*>(W + 4352 + 8 * g);   // d of rows g, g + 8
#pragma unroll
                for (int n = 0; n < 8; ++n) {
                    const float s = *reinterpret_cast<const float*>(R + soff + 8 * n);
                    accf[n][0] = fmaf(s * f.x, (float)acci[n][0], accf[n][0]);
                    accf[n][1] = fmaf(s * f.x, (float)acci[n][1], accf[n][1]);
                    accf[n][2] = fmaf(s * f.y, (float)acci[n][2], accf[n][2]);
                    accf[n][3] = fmaf(s * f.y, (float)acci[n][3], accf[n][3]);
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[st]);
    }
    // limbs hi / mid (lane t even) and lo (lane t + 1) -> one value per row
    // and vector: (lo + mid 2^8) + hi 2^16
    const int64_t npad = (int64_t)(gridDim.x / nvg) * 128;
    if (tile_ok) {
#pragma unroll
        for (int n = 0; n < 8; ++n) {
            const float lo0 = __shfl_down_sync(0xffffffffu, accf[n][0], 1);
            const float lo1 = __shfl_down_sync(0xffffffffu, accf[n][2], 1);
            const int v = 16 * vg + 2 * n + (t >> 1);
            if ((t & 1) == 0 && v < nv) {
                const int r0 = (tile0 + a) * 16 + g;
                const float y0 = (lo0 + accf[n][1] * 256.0f) + accf[n][0] * 65536.0f;
                const float y1 = (lo1 + accf[n][3] * 256.0f) + accf[n][2] * 65536.0f;
                if (S == 1) {
                    if (r0 < N) y[(int64_t)v * ldy + r0] = y0;
                    if (r0 + 8 < N) y[(int64_t)v * ldy + r0 + 8] = y1;
                } else {
                    float* p = part + ((int64_t)split * nv + v) * npad;
                    p[r0] = y0;
                    p[r0 + 8] = y1;
                }
            }
        }
    }
    if (S == 1) return;
    // split-K: the last CTA of this row group adds the partial sums in split order
    __threadfence();
    asm volatile("bar.sync 1, %0;" ::"r"(32 * G::CONSUMERS) : "memory");
    if (threadIdx.x == 0) {
        const int old = atomicAdd(&ctr[blockIdx.x], 1);
        s_last = old == S - 1;
        if (s_last) ctr[blockIdx.x] = 0;   // every split has arrived: ready for the next launch
    }
    asm volatile("bar.sync 1, %0;" ::"r"(32 * G::CONSUMERS) : "memory");
    if (!s_last) return;
    __threadfence();
    const int nvl = min(16, nv - 16 * vg);
    for (int i = threadIdx.x; i < nvl * 128; i += 32 * G::CONSUMERS) {
        const int v = 16 * vg + i / 128, row = tile0 * 16 + i % 128;
        if (row >= N) continue;
        float sum = 0.0f;
        for (int sp = 0; sp < S; ++sp) sum += __ldcg(part + ((int64_t)sp * nv + v) * npad + row);
        y[(int64_t)v * ldy + row] = sum;
    }
}

template <int TYPE>
int kq_mma_launch_t(const uint8_t* packed, int64_t N, int K, const uint8_t* rec, int nv, int S, float* part, int* ctr,
                    float* y, int ldy, unsigned int* err, cudaStream_t stream) {
    using G = KqGeo<TYPE>;
    static uint64_t attr_devs = 0;   // devices whose attribute is set
    int dev = 0;
    BREW_CUDA(cudaGetDevice(&dev));
    if (dev < 64 && !(attr_devs >> dev & 1)) {
        BREW_CUDA(cudaFuncSetAttribute(kq_mma_kernel<TYPE>, cudaFuncAttributeMaxDynamicSharedMemorySize, G::SMEM));
        attr_devs |= 1ull << dev;
    }
    const int tiles = (int)((N + 15) / 16);
    const int nvg = (nv + 15) / 16;
    const dim3 grid((unsigned)((tiles + KQ_TILES - 1) / KQ_TILES * nvg), (unsigned)S);
    kq_mma_kernel<TYPE><<<grid, G::THREADS, G::SMEM, stream>>>(packed, tiles, K / 256, (int)N, rec, nv, nvg, S, part,
                                                               ctr, y, ldy, err);
    BREW_CUDA(cudaGetLastError());
    count_launch();
    return BREW_OK;
}

}  // namespace

int kq_splits(int64_t K, int64_t n_basis) {
    // as many splits as keep the family's 128-row groups within one wave of
    // one CTA per SM of a B200 (148 SMs), at least two super-blocks each
    constexpr int64_t wave = 148;
    const int64_t groups = std::max<int64_t>(1, (n_basis + 127) / 128), ksb = K / 256;
    int64_t s = wave / groups;
    s = std::min<int64_t>(s, std::max<int64_t>(1, ksb / 2));
    return (int)std::max<int64_t>(1, s);
}

int kq_pack_launch(int type, const uint8_t* w, int64_t N, int K, uint8_t* out, cudaStream_t stream) {
    BREW_CHECK((type == BREW_TYPE_Q4_K || type == BREW_TYPE_Q6_K) && K % 256 == 0 && K > 0 && N > 0,
               BREW_ERR_INVALID_ARG, "K-quant pack: type %d N=%lld K=%d", type, (long long)N, K);
    const int64_t n = (N + 15) / 16 * 16 * (K / 32);
    const unsigned blocks = (unsigned)((n + 255) / 256);
    if (type == BREW_TYPE_Q4_K) kq_pack_kernel<BREW_TYPE_Q4_K><<<blocks, 256, 0, stream>>>(w, N, K, out);
    else kq_pack_kernel<BREW_TYPE_Q6_K><<<blocks, 256, 0, stream>>>(w, N, K, out);
    BREW_CUDA(cudaGetLastError());
    count_launch();
    return BREW_OK;
}

int kq_prep_launch(const float* x, int ldx, int K, int nv, uint8_t* rec, cudaStream_t stream) {
    BREW_CHECK(nv >= 1 && nv <= KQ_MAX_VECTORS && K % 256 == 0 && K > 0 && ldx % 4 == 0 &&
                   (reinterpret_cast<uintptr_t>(x) & 15) == 0,
               BREW_ERR_INVALID_ARG, "K-quant records: nv=%d K=%d ldx=%d (x 16-byte aligned)", nv, K, ldx);
    const int nvp = (nv + 15) / 16 * 16;
    const int64_t warps = (int64_t)nvp * (K / 256);
    kq_prep_kernel<<<(unsigned)((warps * 32 + 255) / 256), 256, 0, stream>>>(x, ldx, K, nv, nvp, rec);
    BREW_CUDA(cudaGetLastError());
    count_launch();
    return BREW_OK;
}

int kq_mma_launch(int type, const uint8_t* packed, int64_t N, int K, const uint8_t* rec, int nv, int splits,
                  float* part, int* ctr, float* y, int ldy, unsigned int* err, cudaStream_t stream) {
    BREW_CHECK(nv >= 1 && nv <= KQ_MAX_VECTORS && K % 256 == 0 && K > 0 && N > 0 && splits >= 1 &&
                   splits <= K / 256 && (splits == 1 || (part && ctr)),
               BREW_ERR_INVALID_ARG, "K-quant MMA matvec: nv=%d N=%lld K=%d splits=%d", nv, (long long)N, K, splits);
    if (type == BREW_TYPE_Q4_K)
        return kq_mma_launch_t<BREW_TYPE_Q4_K>(packed, N, K, rec, nv, splits, part, ctr, y, ldy, err, stream);
    BREW_CHECK(type == BREW_TYPE_Q6_K, BREW_ERR_INVALID_ARG, "K-quant MMA matvec: type %d", type);
    return kq_mma_launch_t<BREW_TYPE_Q6_K>(packed, N, K, rec, nv, splits, part, ctr, y, ldy, err, stream);
}

}  // namespace brew
