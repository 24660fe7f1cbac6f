// prep.cuh — activation "prep records": the operand format the quantized
// matvec consumes on the x side.
//
// A matvec against GGUF blocks needs, per 32-element block j of x, the dot
// product sum_i q[r][32j+i] * x[32j+i].  x is fp32; the tensor cores only
// multiply integers exactly.  So each 32-element block of x is rewritten as
// a 24-bit block fixed-point number v_i = rint(x_i * 8290000 / max|x_block|)
// and v_i is split into three balanced signed bytes
//     v = hi * 2^16 + mid * 2^8 + lo,   hi, mid, lo in [-128, 127].
// With those three "limb" columns as the B operand of an int8 MMA, the
// per-block integer sums are exact; the fp32 epilogue multiplies them by the
// block's fp16 weight scale and s_j, and the limb weights 2^16 / 2^8 / 1 are
// applied (exactly) when the columns are combined.  The x rounding error is
// 2^-24 relative to the block maximum, i.e. at the level of fp32 itself.
//
// Record of block j for `batch` vectors, padded to a multiple of 16 bytes:
//     int8   limbs[3*batch][32]   limb l of vector b at row 3*b + l
//     float  s[batch]             block scale of vector b
//     int32  lsum[3*batch]        sum_i limbs[3*b+l][i]  (zero-point correction, Q4_0)
// In the MMA, vector b occupies the four B columns 4*b .. 4*b+3 (limbs
// hi, mid, lo and a zero column), so each thread's pair of accumulator
// columns belongs to one vector.
#pragma once

#include "brew_common.cuh"

namespace brew {

constexpr float PREP_RANGE = 8290000.0f;   // |v| <= 8290001 keeps hi in [-127, 127]

// The two scales of a block whose largest magnitude is am: inv = R / am
// (x * inv is the block fixed-point value) and s = am / R (its weight in the
// product).  inv comes from the fast approximate division (within 2 ulp, no
// IEEE slow path on the critical path of every phase's input), s from a
// multiply by the constant 1 / R; |x * inv| <= R * (1 + 2^-21) keeps the top
// limb in [-127, 127], and the products stay exact to fp32 rounding.  Blocks
// whose maximum is below 1e-30 (R / am would overflow) are taken as zero.
constexpr float PREP_TINY = 1e-30f;
__host__ __device__ inline float prep_block_scale(float am) { return am * (1.0f / PREP_RANGE); }
#ifdef __CUDACC__
__device__ __forceinline__ float prep_block_inv(float am) { return am > PREP_TINY ? __fdividef(PREP_RANGE, am) : 0.0f; }
#endif

// n8 MMA column tiles for `batch` vectors (4 columns per vector)
__host__ __device__ inline int prep_nt(int batch) { return (batch + 1) / 2; }
__host__ __device__ inline int prep_rec_bytes(int batch) { return (batch * (3 * 32 + 4 + 3 * 4) + 15) & ~15; }
__host__ __device__ inline int prep_s_off(int batch) { return 3 * batch * 32; }
__host__ __device__ inline int prep_lsum_off(int batch) { return 3 * batch * 32 + 4 * batch; }

#ifdef __CUDACC__

// One warp writes the record entries of vector b for one block: lane i
// holds x[32j + i].
__device__ __forceinline__ void prep_emit_warp(uint8_t* rec, int batch, int b, float x) {
    const int lane = threadIdx.x & 31;
    const float amax = warp_max(fabsf(x));
    const float inv = prep_block_inv(amax);
    const float s = prep_block_scale(amax);
    const int v = __float2int_rn(x * inv);
    const int lo = ((v + 128) & 255) - 128;
    const int v1 = (v - lo) >> 8;
    const int mid = ((v1 + 128) & 255) - 128;
    const int hi = (v1 - mid) >> 8;
    int8_t* limbs = reinterpret_cast<int8_t*>(rec);
    limbs[(3 * b + 0) * 32 + lane] = (int8_t)hi;
    limbs[(3 * b + 1) * 32 + lane] = (int8_t)mid;
    limbs[(3 * b + 2) * 32 + lane] = (int8_t)lo;
    const int shi = warp_sum_i(hi), smid = warp_sum_i(mid), slo = warp_sum_i(lo);
    if (lane == 0) {
        reinterpret_cast<float*>(rec + prep_s_off(batch))[b] = s;
        int* ls = reinterpret_cast<int*>(rec + prep_lsum_off(batch));
        ls[3 * b + 0] = shi;
        ls[3 * b + 1] = smid;
        ls[3 * b + 2] = slo;
    }
}

// The same record entries as prep_emit_warp, written by eight lanes per
// block: lane group (lane >> 3) of the warp holds one block, lane (lane & 7)
// its elements 4*(lane & 7) .. +3 in x.  Every lane of the warp calls it (the
// group max is a shuffle); `ok` masks the shared-memory stores.  `lsum`
// selects whether the limb sums (used only by the Q4_0 zero-point
// correction) are produced.
__device__ __forceinline__ void prep_emit_quad(uint8_t* rec, int batch, int b, float4 x, bool ok, bool lsum) {
    const int lane = threadIdx.x & 31, e = (lane & 7) * 4;
    float am = fmaxf(fmaxf(fabsf(x.x), fabsf(x.y)), fmaxf(fabsf(x.z), fabsf(x.w)));
    am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 1));
    am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 2));
    am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 4));
    const float inv = prep_block_inv(am);
    const float s = prep_block_scale(am);
    const float xs[4] = {x.x, x.y, x.z, x.w};
    uint32_t phi = 0u, pmid = 0u, plo = 0u;
    int shi = 0, smid = 0, slo = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const int v = __float2int_rn(xs[k] * inv);
        const int lo = ((v + 128) & 255) - 128;
        const int v1 = (v - lo) >> 8;
        const int mid = ((v1 + 128) & 255) - 128;
        const int hi = (v1 - mid) >> 8;
        phi |= (uint32_t)(hi & 255) << (8 * k);
        pmid |= (uint32_t)(mid & 255) << (8 * k);
        plo |= (uint32_t)(lo & 255) << (8 * k);
        shi += hi;
        smid += mid;
        slo += lo;
    }
    if (ok) {
        *reinterpret_cast<uint32_t*>(rec + (3 * b + 0) * 32 + e) = phi;
        *reinterpret_cast<uint32_t*>(rec + (3 * b + 1) * 32 + e) = pmid;
        *reinterpret_cast<uint32_t*>(rec + (3 * b + 2) * 32 + e) = plo;
    }
    if (lsum) {
        // four limbs per lane: each lane sum is in [-512, 508]; hi and mid
        // share one word with a bias of 512 per lane (eight lanes < 2^16)
        int hm = (shi + 512) | ((smid + 512) << 16);
#pragma unroll
        for (int o = 1; o < 8; o <<= 1) {
            hm += __shfl_xor_sync(0xffffffffu, hm, o);
            slo += __shfl_xor_sync(0xffffffffu, slo, o);
        }
        if (ok && (lane & 7) == 0) {
            int* ls = reinterpret_cast<int*>(rec + prep_lsum_off(batch));
            ls[3 * b + 0] = (hm & 0xFFFF) - 8 * 512;
            ls[3 * b + 1] = (hm >> 16) - 8 * 512;
            ls[3 * b + 2] = slo;
        }
    }
    if (ok && (lane & 7) == 0) reinterpret_cast<float*>(rec + prep_s_off(batch))[b] = s;
}

// Block-wide sum (all threads of the CTA call it; red has >= 32 floats).
__device__ __forceinline__ float block_sum(float v, float* red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
    v = warp_sum(v);
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float t = 0.0f;
    if (warp == 0) {
        t = lane < nw ? red[lane] : 0.0f;
        t = warp_sum(t);
        if (lane == 0) red[0] = t;
    }
    __syncthreads();
    t = red[0];
    __syncthreads();
    return t;
}

// inverseRootMeanSquare (transformer/math/Kernels.java:77-88): the sum of
// squares in fp32, meanSquare = ss / n in fp32 (IEEE division), then the
// scale (float)(1.0 / Math.sqrt((double)(meanSquare + eps))).  The last step
// is the correctly rounded fp32 reciprocal square root of the fp32 sum: the
// reference's double result is within 2^-52 of the exact value before its
// rounding to fp32, so the two round to the same float except for arguments
// within 2^-52 of a rounding midpoint (about 4e-9 of them), where they differ
// by one ulp.  One correctly rounded instruction sequence instead of a double
// square root and a double division on every phase's critical path.
__device__ __forceinline__ float rms_scale(float ss, int n, float eps) {
    const float meanSquare = __fdiv_rn(ss, (float)n);
    return __frsqrt_rn(__fadd_rn(meanSquare, eps));
}

// Whole-CTA prep of one vector x[K] (read through L2: it may have been
// written by other CTAs of the same kernel) (optionally RMS-normalised with weight
// nw: x * scale * nw, Kernels.java:47-58) into records[K/32].
static __device__ void prep_vector_cta(const float* x, int K, const float* nw, float eps, uint8_t* recs, int rec_bytes,
                                int batch, int b, float* red) {
    float scale = 1.0f;
    if (nw) {
        float ss = 0.0f;
        for (int i = threadIdx.x; i < K; i += blockDim.x) {
            const float v = __ldcg(&x[i]);
            ss += v * v;
        }
        ss = block_sum(ss, red);
        scale = rms_scale(ss, K, eps);
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw_ = blockDim.x >> 5;
    for (int j = warp; j < K / 32; j += nw_) {
        float v = __ldcg(&x[32 * j + lane]);
        if (nw) v = v * scale * nw[32 * j + lane];
        prep_emit_warp(recs + (size_t)j * rec_bytes, batch, b, v);
    }
}

#endif

}  // namespace brew
