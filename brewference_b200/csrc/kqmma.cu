// kqmma.cu — K-quant matvec on the int8 tensor cores (layout in kqmma.cuh).
#include "brew_internal.cuh"
#include "kqmma.cuh"
#include "matvec.cuh"
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

// One thread per (row, 32-element block): decodes the block's quants and
// factors and writes them at their fragment positions.
template <int TYPE>
__global__ void kq_pack_kernel(const uint8_t* w, int64_t N, int K, uint8_t* out) {
    constexpr int TB = kq_tile_bytes(TYPE), SB = TYPE == BREW_TYPE_Q4_K ? 144 : 210;
    const int KB = K / 32;
    const int64_t rows = (N + 15) / 16 * 16;
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= rows * KB) return;
    const int64_t row = i / KB;
    const int kb = (int)(i % KB);
    const int rt = (int)(row % 16), g = rt % 8, upper = rt / 8;
    uint8_t* base = out + ((row / 16) * KB + kb) * TB;
    int q[32];
    float f0 = 0.0f, f1 = 0.0f;   // Q4_K: D, M; Q6_K: D_lo, D_hi
    if (row < N) {
        const uint8_t* blk = w + row * (int64_t)(K / 256) * SB + (int64_t)(kb / 8) * SB;
        const int s = kb % 8;   // the 32-element sub-block of the super-block
        if (TYPE == BREW_TYPE_Q4_K) {
            int sc, m;
            q4k_scale_min(blk + 4, s, sc, m);
            f0 = __fmul_rn(kq_half(blk), (float)sc);       // d * sc
            f1 = __fmul_rn(kq_half(blk + 2), (float)m);    // dmin * m
            for (int k = 0; k < 32; ++k) q[k] = (blk[16 + 32 * (s / 2) + k] >> (4 * (s & 1))) & 15;
        } else {
            const float d = kq_half(blk + 208);
            f0 = __fmul_rn(d, (float)(int8_t)blk[192 + 2 * s]);
            f1 = __fmul_rn(d, (float)(int8_t)blk[192 + 2 * s + 1]);
            for (int k = 0; k < 32; ++k) {
                const int r = 32 * s + k, h = r / 128, rr = r % 128, grp = rr / 32, l = rr % 32;
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
        // byte (lane, upper, j): q[4t + j] low nibble, q[16 + 4t + j] high nibble
        for (int t = 0; t < 4; ++t)
            for (int j = 0; j < 4; ++j)
                base[(g * 4 + t) * 8 + 4 * upper + j] = (uint8_t)(q[4 * t + j] | (q[16 + 4 * t + j] << 4));
        float* sc = reinterpret_cast<float*>(base + 256 + 16 * g + 8 * upper);
        sc[0] = f0;
        sc[1] = f1;
    } else {
        for (int k = 0; k < 32; ++k) {
            const int t = (k % 16) / 4, half = k / 16;
            base[(g * 4 + t) * 16 + 4 * (upper + 2 * half) + (k % 4)] = (uint8_t)(int8_t)q[k];
        }
        float* sc = reinterpret_cast<float*>(base + 512 + 16 * g + 8 * upper);
        sc[0] = f0;
        sc[1] = f1;
    }
}

constexpr int KQM_WARPS = 8;

// int8 MMA over 16 of the block's 32 elements (one Q6_K scale's half):
// a0 / a1 hold rows g / g + 8, k = 4t .. 4t + 3; b holds k = 4t .. 4t + 3.
__device__ __forceinline__ void mma_s8s8_k16(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t b) {
    asm("mma.sync.aligned.m16n8k16.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%7,%8,%9,%10};"
        : "=r"(c[0]), "=r"(c[1]), "=r"(c[2]), "=r"(c[3])
        : "r"(a0), "r"(a1), "r"(b), "r"(0), "r"(0), "r"(0), "r"(0));
}

// An int32 block sum |i| < 2^22 as a float, exactly, with full-rate adds
// (the bits of 1.5 * 2^23 plus i are the float 1.5 * 2^23 + i).
__device__ __forceinline__ float kq_i2f(int i) { return __int_as_float(i + 0x4B400000) - 12582912.0f; }

// CTA = NG 16-row tiles (2 for matrices of many tiles, 1 otherwise, so that
// a 3584-row matrix still spreads over 224 CTAs) x up to 2 NT vectors.  The 8 warps split the
// block columns (warp w takes kb = w, w + 8, ...), each keeping fp32
// accumulators per limb column; at the end each warp combines its limbs,
// the warps' sums meet in shared memory and 256 threads write the outputs.
template <int TYPE, int NT, int KQM_NG>
__global__ void __launch_bounds__(KQM_WARPS * 32, 2) kq_mma_kernel(const uint8_t* pk, int KB, int tiles, int N,
                                                                   const uint8_t* prep, int rec_bytes, int nv,
                                                                   float* y, int ldy) {
    constexpr int TB = kq_tile_bytes(TYPE), SO = TYPE == BREW_TYPE_Q4_K ? 256 : 512;
    __shared__ float red[KQM_WARPS][KQM_NG][16][16];   // [warp][tile][row][vector]
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, t = lane & 3;
    const int tile0 = blockIdx.x * KQM_NG;
    const int ng = min(KQM_NG, tiles - tile0);
    // x operand of n8 tile n (prep.cuh): B column g = limb (g & 3) of vector
    // 2n + (g >> 2); accumulator columns 2t, 2t + 1 = limbs (2t) & 3, +1 of
    // vector 2n + (t >> 1)
    uint32_t boff[NT], soff[NT], loff0[NT], loff1[NT];
    bool vB[NT], vC[NT];
    const int l0 = (2 * t) & 3;
#pragma unroll
    for (int n = 0; n < NT; ++n) {
        const int bB = 2 * n + (g >> 2), lB = g & 3, bC = 2 * n + (t >> 1);
        vB[n] = lB < 3 && bB < nv;
        vC[n] = bC < nv;
        const int bCs = vC[n] ? bC : 0;
        boff[n] = (vB[n] ? (3 * bB + lB) * 32 : 0) + 4 * t;
        soff[n] = prep_s_off(nv) + 4 * bCs;
        loff0[n] = prep_lsum_off(nv) + 4 * (3 * bCs + l0);
        loff1[n] = prep_lsum_off(nv) + 4 * (3 * bCs + 1);
    }
    float acc[KQM_NG][NT][4];
#pragma unroll
    for (int a = 0; a < KQM_NG; ++a)
#pragma unroll
        for (int n = 0; n < NT; ++n) acc[a][n][0] = acc[a][n][1] = acc[a][n][2] = acc[a][n][3] = 0.0f;
    for (int kb = warp; kb < KB; kb += KQM_WARPS) {
        const uint8_t* rec = prep + (int64_t)kb * rec_bytes;
        uint32_t b0[NT], b1[NT];
        float s[NT], ml0[NT], ml1[NT];
#pragma unroll
        for (int n = 0; n < NT; ++n) {
            b0[n] = vB[n] ? __ldg(reinterpret_cast<const uint32_t*>(rec + boff[n])) : 0u;
            b1[n] = vB[n] ? __ldg(reinterpret_cast<const uint32_t*>(rec + boff[n] + 16)) : 0u;
            s[n] = vC[n] ? __ldg(reinterpret_cast<const float*>(rec + soff[n])) : 0.0f;
            if (TYPE == BREW_TYPE_Q4_K) {   // limb sums of the two columns (the zero column: 0)
                ml0[n] = vC[n] ? (float)__ldg(reinterpret_cast<const int*>(rec + loff0[n])) : 0.0f;
                ml1[n] = (vC[n] && l0 == 0) ? (float)__ldg(reinterpret_cast<const int*>(rec + loff1[n])) : 0.0f;
            }
        }
#pragma unroll
        for (int a = 0; a < KQM_NG; ++a) {
            if (a < ng) {
                const uint8_t* blk = pk + ((int64_t)(tile0 + a) * KB + kb) * TB;
                const float4 f = __ldg(reinterpret_cast<const float4*>(blk + SO + 16 * g));
                if (TYPE == BREW_TYPE_Q4_K) {
                    const uint2 W = __ldg(reinterpret_cast<const uint2*>(blk + lane * 8));
                    const uint32_t a0 = W.x & 0x0F0F0F0Fu, a1 = W.y & 0x0F0F0F0Fu;
                    const uint32_t a2 = (W.x >> 4) & 0x0F0F0F0Fu, a3 = (W.y >> 4) & 0x0F0F0F0Fu;
#pragma unroll
                    for (int n = 0; n < NT; ++n) {
                        int c[4];
                        mma_u8s8(c, a0, a1, a2, a3, b0[n], b1[n]);
                        // s * (D * sum(q limb) - M * sum(limb)); rows g (D, M = f.x, f.y), g + 8 (f.z, f.w)
                        acc[a][n][0] = fmaf(s[n], fmaf(f.x, kq_i2f(c[0]), -f.y * ml0[n]), acc[a][n][0]);
                        acc[a][n][1] = fmaf(s[n], fmaf(f.x, kq_i2f(c[1]), -f.y * ml1[n]), acc[a][n][1]);
                        acc[a][n][2] = fmaf(s[n], fmaf(f.z, kq_i2f(c[2]), -f.w * ml0[n]), acc[a][n][2]);
                        acc[a][n][3] = fmaf(s[n], fmaf(f.z, kq_i2f(c[3]), -f.w * ml1[n]), acc[a][n][3]);
                    }
                } else {
                    const uint4 A = __ldg(reinterpret_cast<const uint4*>(blk + lane * 16));
#pragma unroll
                    for (int n = 0; n < NT; ++n) {
                        int cl[4], ch[4];
                        mma_s8s8_k16(cl, A.x, A.y, b0[n]);   // k 0..15
                        mma_s8s8_k16(ch, A.z, A.w, b1[n]);   // k 16..31
                        // s * (D_lo * sum_lo + D_hi * sum_hi); rows g (f.x, f.y), g + 8 (f.z, f.w)
                        acc[a][n][0] = fmaf(s[n], fmaf(f.y, kq_i2f(ch[0]), f.x * kq_i2f(cl[0])), acc[a][n][0]);
                        acc[a][n][1] = fmaf(s[n], fmaf(f.y, kq_i2f(ch[1]), f.x * kq_i2f(cl[1])), acc[a][n][1]);
                        acc[a][n][2] = fmaf(s[n], fmaf(f.w, kq_i2f(ch[2]), f.z * kq_i2f(cl[2])), acc[a][n][2]);
                        acc[a][n][3] = fmaf(s[n], fmaf(f.w, kq_i2f(ch[3]), f.z * kq_i2f(cl[3])), acc[a][n][3]);
                    }
                }
            }
        }
    }
    // limbs hi / mid (lane t even) and lo (lane t + 1) -> one value per row
    // and vector: (lo + mid 2^8) + hi 2^16
#pragma unroll
    for (int a = 0; a < KQM_NG; ++a)
#pragma unroll
        for (int n = 0; n < NT; ++n) {
            const float lo0 = __shfl_down_sync(0xffffffffu, acc[a][n][0], 1);
            const float lo1 = __shfl_down_sync(0xffffffffu, acc[a][n][2], 1);
            if ((t & 1) == 0) {
                const int v = 2 * n + (t >> 1);
                red[warp][a][g][v] = (lo0 + acc[a][n][1] * 256.0f) + acc[a][n][0] * 65536.0f;
                red[warp][a][g + 8][v] = (lo1 + acc[a][n][3] * 256.0f) + acc[a][n][2] * 65536.0f;
            }
        }
    __syncthreads();
    for (int i = threadIdx.x; i < KQM_NG * 16 * nv; i += KQM_WARPS * 32) {
        const int v = i % nv, row = (i / nv) % 16, a = i / (16 * nv);
        const int r = (tile0 + a) * 16 + row;
        if (a < ng && r < N) {
            float sum = 0.0f;
#pragma unroll
            for (int w = 0; w < KQM_WARPS; ++w) sum += red[w][a][row][v];
            y[(int64_t)v * ldy + r] = sum;
        }
    }
}

template <int TYPE, int NT>
int kq_mma_launch_t(const uint8_t* packed, int64_t N, int K, const uint8_t* prep, int nv, float* y, int ldy,
                    cudaStream_t stream) {
    const int tiles = (int)((N + 15) / 16);
    if (tiles >= 4 * num_sms())
        kq_mma_kernel<TYPE, NT, 2><<<(tiles + 1) / 2, KQM_WARPS * 32, 0, stream>>>(packed, K / 32, tiles, (int)N, prep,
                                                                                  prep_rec_bytes(nv), nv, y, ldy);
    else
        kq_mma_kernel<TYPE, NT, 1><<<tiles, KQM_WARPS * 32, 0, stream>>>(packed, K / 32, tiles, (int)N, prep,
                                                                        prep_rec_bytes(nv), nv, y, ldy);
    BREW_CUDA(cudaGetLastError());
    count_launch();
    return BREW_OK;
}

template <int TYPE>
int kq_mma_dispatch(const uint8_t* packed, int64_t N, int K, const uint8_t* prep, int nv, float* y, int ldy,
                    cudaStream_t stream) {
    const int nt = (nv + 1) / 2;
    if (nt <= 1) return kq_mma_launch_t<TYPE, 1>(packed, N, K, prep, nv, y, ldy, stream);
    if (nt <= 2) return kq_mma_launch_t<TYPE, 2>(packed, N, K, prep, nv, y, ldy, stream);
    if (nt <= 4) return kq_mma_launch_t<TYPE, 4>(packed, N, K, prep, nv, y, ldy, stream);
    return kq_mma_launch_t<TYPE, 8>(packed, N, K, prep, nv, y, ldy, stream);
}

}  // namespace

int kq_pack_launch(int type, const uint8_t* w, int64_t N, int K, uint8_t* out, cudaStream_t stream) {
    BREW_CHECK((type == BREW_TYPE_Q4_K || type == BREW_TYPE_Q6_K) && K % 256 == 0 && N > 0, BREW_ERR_INVALID_ARG,
               "K-quant pack: type %d K=%d", type, K);
    const int64_t n = (N + 15) / 16 * 16 * (K / 32);
    const unsigned blocks = (unsigned)((n + 255) / 256);
    if (type == BREW_TYPE_Q4_K) kq_pack_kernel<BREW_TYPE_Q4_K><<<blocks, 256, 0, stream>>>(w, N, K, out);
    else kq_pack_kernel<BREW_TYPE_Q6_K><<<blocks, 256, 0, stream>>>(w, N, K, out);
    BREW_CUDA(cudaGetLastError());
    count_launch();
    return BREW_OK;
}

int kq_mma_launch(int type, const uint8_t* packed, int64_t N, int K, const uint8_t* prep, int nv, float* y, int ldy,
                  cudaStream_t stream) {
    BREW_CHECK(nv >= 1 && nv <= 16 && K % 256 == 0, BREW_ERR_INVALID_ARG, "K-quant MMA matvec: nv=%d K=%d", nv, K);
    if (type == BREW_TYPE_Q4_K) return kq_mma_dispatch<BREW_TYPE_Q4_K>(packed, N, K, prep, nv, y, ldy, stream);
    BREW_CHECK(type == BREW_TYPE_Q6_K, BREW_ERR_INVALID_ARG, "K-quant MMA matvec: type %d", type);
    return kq_mma_dispatch<BREW_TYPE_Q6_K>(packed, N, K, prep, nv, y, ldy, stream);
}

}  // namespace brew
