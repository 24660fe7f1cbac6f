// mv_device.cuh — device building blocks of the packed-block matvec, shared
// by the stand-alone matvec kernel and the persistent decode kernel.
#pragma once

#include "brew_common.cuh"
#include "matvec.cuh"
#include "prep.cuh"

namespace brew {

// Shared-memory loads as plain C++ loads (not volatile asm): the compiler may
// overlap the loads of the next block pair with the current one's MMA and
// epilogue.  Ordering against the mbarrier waits is kept by their "memory"
// clobbers.  Addresses are 32-bit shared-window offsets turned back into
// generic pointers.
__device__ __forceinline__ const uint8_t* sptr(uint32_t a) {
    return reinterpret_cast<const uint8_t*>(__cvta_shared_to_generic(a));
}
__device__ __forceinline__ uint32_t lds32(uint32_t a) { return *reinterpret_cast<const uint32_t*>(sptr(a)); }
__device__ __forceinline__ uint32_t lds16(uint32_t a) { return *reinterpret_cast<const uint16_t*>(sptr(a)); }
__device__ __forceinline__ float ldsf(uint32_t a) { return *reinterpret_cast<const float*>(sptr(a)); }

// 4 bytes at a 2-byte aligned shared-memory address: two aligned words and a
// funnel shift (shift 0 or 16).
__device__ __forceinline__ uint32_t lds32_a2(uint32_t a) {
    const uint32_t b = a & ~3u;
    return __funnelshift_r(lds32(b), lds32(b + 4), (a & 3u) * 8u);
}

__device__ __forceinline__ void mma_s8s8(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%11,%12,%13};"
        : "=r"(c[0]), "=r"(c[1]), "=r"(c[2]), "=r"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0), "r"(0), "r"(0), "r"(0));
}

__device__ __forceinline__ void mma_u8s8(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%11,%12,%13};"
        : "=r"(c[0]), "=r"(c[1]), "=r"(c[2]), "=r"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0), "r"(0), "r"(0), "r"(0));
}

__device__ __forceinline__ void consumer_bar() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

__device__ __forceinline__ float act_glu(float g, int epi) {
    // FfnActivation.silu / geluPytorchTanh evaluated in double, cast to float
    // (transformer/ffn/FfnActivation.java:43-58).
    const double v = (double)g;
    double a;
    if (epi == MV_EPI_GLU_GELU) {
        const double inner = (double)0.7978845608028654f * (v + (double)0.044715f * v * v * v);
        a = 0.5 * v * (1.0 + tanh(inner));
    } else {
        a = v / (1.0 + exp(-v));
    }
    return (float)a;
}

// Orderable 64-bit argmax key: larger value first, then smaller index
// (Kernels.argMax keeps the first maximum).
__device__ __forceinline__ unsigned long long argmax_key(float v, int idx) {
    uint32_t u = __float_as_uint(v);
    u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return ((unsigned long long)u << 32) | (0xFFFFFFFFu - (uint32_t)idx);
}

// One 16-row x 32-element block: the int8 MMA of the weight fragment against
// the limb columns of every vector, then acc += C * (d_row * s_vector).  Lane
// (g, t) holds accumulator columns 8n+2t and 8n+2t+1 of rows g and g+8; both
// columns belong to vector (8n+2t)/4 (4 columns per vector, see prep.cuh).
template <int TYPE, int NT>
__device__ __forceinline__ void mma_block(float (&acc)[NT][4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          float d0, float d1, uint32_t rec, int batch, int g, int t) {
    const uint32_t soff = prep_s_off(batch), loff = prep_lsum_off(batch);
#pragma unroll
    for (int n = 0; n < NT; ++n) {
        const int cB = n * 8 + g, bB = cB >> 2, lB = cB & 3;
        const bool vB = lB < 3 && bB < batch;
        const uint32_t ba = rec + (vB ? (3 * bB + lB) * 32 : 0) + 4 * t;
        uint32_t b0 = lds32(ba), b1 = lds32(ba + 16);
        if (!vB) b0 = b1 = 0u;
        const int bC = (n * 8 + 2 * t) >> 2;
        const int l0 = (2 * t) & 3;               // 0 or 2
        const bool vC = bC < batch;
        const int bCs = vC ? bC : 0;
        int c[4];
        if (TYPE == BREW_TYPE_Q8_0) {
            mma_s8s8(c, a0, a1, a2, a3, b0, b1);
        } else {
            mma_u8s8(c, a0, a1, a2, a3, b0, b1);
            // Q4_0 quants are stored as q+8: subtract 8 * sum(limbs)
            const int ls0 = vC ? (int)lds32(rec + loff + 4 * (3 * bCs + l0)) : 0;
            const int ls1 = (vC && l0 == 0) ? (int)lds32(rec + loff + 4 * (3 * bCs + 1)) : 0;
            c[0] -= 8 * ls0;
            c[1] -= 8 * ls1;
            c[2] -= 8 * ls0;
            c[3] -= 8 * ls1;
        }
        const float s = vC ? ldsf(rec + soff + 4 * bCs) : 0.0f;
        const float ds0 = d0 * s, ds1 = d1 * s;
        acc[n][0] = fmaf((float)c[0], ds0, acc[n][0]);
        acc[n][1] = fmaf((float)c[1], ds0, acc[n][1]);
        acc[n][2] = fmaf((float)c[2], ds1, acc[n][2]);
        acc[n][3] = fmaf((float)c[3], ds1, acc[n][3]);
    }
}

__device__ __forceinline__ float h2f_lo(uint32_t w) { return __half2float(__ushort_as_half((uint16_t)(w & 0xFFFFu))); }
__device__ __forceinline__ float h2f_hi(uint32_t w) { return __half2float(__ushort_as_half((uint16_t)(w >> 16))); }

// Multiplies one staged TMA chunk of a tile: boxes are [16 rows][8 blocks]
// (box row = 8*BB bytes), walked in block pairs (68 / 36 bytes, word
// aligned: only the even block's quants need a byte permute).  Warp `sub` of
// `ws` takes pairs sub, sub+ws, ...; prep0 is the record of the chunk's first
// block.
template <int TYPE, int NT>
__device__ __forceinline__ void tma_tile_stage(float (&acc)[NT][4], uint32_t sb, uint32_t prep0, int rec_bytes, int tw,
                                               int nb, int sub, int ws, int g, int t, int batch) {
    constexpr int BB = TYPE == BREW_TYPE_Q8_0 ? 34 : 18;
    constexpr int BOXW = 8 * BB, PAIR = 2 * BB;
    const int npairs = nb * 4;
#pragma unroll 4
    for (int pp = sub; pp < npairs; pp += ws) {
        const int bi = pp >> 2, pi = pp & 3;
        const uint32_t R0 = sb + ((tw * nb + bi) * 16 + g) * BOXW + pi * PAIR;
        const uint32_t R1 = R0 + 8 * BOXW;
        const uint32_t recA = prep0 + (bi * 8 + pi * 2) * rec_bytes;
        const uint32_t recB = recA + rec_bytes;
        if (TYPE == BREW_TYPE_Q8_0) {
            const uint32_t dA0 = lds32(R0), dA1 = lds32(R1);
            const uint32_t dB0 = lds32(R0 + 32), dB1 = lds32(R1 + 32);
            const uint32_t a0 = __byte_perm(lds32(R0 + 4 * t), lds32(R0 + 4 * t + 4), 0x5432);
            const uint32_t a1 = __byte_perm(lds32(R1 + 4 * t), lds32(R1 + 4 * t + 4), 0x5432);
            const uint32_t a2 = __byte_perm(lds32(R0 + 4 * t + 16), lds32(R0 + 4 * t + 20), 0x5432);
            const uint32_t a3 = __byte_perm(lds32(R1 + 4 * t + 16), lds32(R1 + 4 * t + 20), 0x5432);
            mma_block<TYPE, NT>(acc, a0, a1, a2, a3, h2f_lo(dA0), h2f_lo(dA1), recA, batch, g, t);
            mma_block<TYPE, NT>(acc, lds32(R0 + 36 + 4 * t), lds32(R1 + 36 + 4 * t), lds32(R0 + 52 + 4 * t),
                                lds32(R1 + 52 + 4 * t), h2f_hi(dB0), h2f_hi(dB1), recB, batch, g, t);
        } else {
            const uint32_t dA0 = lds32(R0), dA1 = lds32(R1);
            const uint32_t dB0 = lds32(R0 + 16), dB1 = lds32(R1 + 16);
            const uint32_t w0 = __byte_perm(lds32(R0 + 4 * t), lds32(R0 + 4 * t + 4), 0x5432);
            const uint32_t w1 = __byte_perm(lds32(R1 + 4 * t), lds32(R1 + 4 * t + 4), 0x5432);
            mma_block<TYPE, NT>(acc, w0 & 0x0F0F0F0Fu, w1 & 0x0F0F0F0Fu, (w0 >> 4) & 0x0F0F0F0Fu,
                                (w1 >> 4) & 0x0F0F0F0Fu, h2f_lo(dA0), h2f_lo(dA1), recA, batch, g, t);
            const uint32_t v0 = lds32(R0 + 20 + 4 * t), v1 = lds32(R1 + 20 + 4 * t);
            mma_block<TYPE, NT>(acc, v0 & 0x0F0F0F0Fu, v1 & 0x0F0F0F0Fu, (v0 >> 4) & 0x0F0F0F0Fu,
                                (v1 >> 4) & 0x0F0F0F0Fu, h2f_hi(dB0), h2f_hi(dB1), recB, batch, g, t);
        }
    }
}

// Stage geometry of a CTA that owns `nt` tiles: gs tiles staged together,
// ws warps per tile (splitting its blocks), nb TMA boxes of 8 blocks per tile
// per stage (nb <= nb_cap, gs*nb <= MV_MAX_BOXES), KC blocks per stage.
struct Geom {
    int gs, ws, nb, KC, nchunks;
};

__device__ __forceinline__ Geom tma_geom(int nt, int KB, int nb_cap) {
    Geom g;
    g.gs = min(MV_MAX_BOXES, nt);
    // warps per tile: the largest power of two with gs * ws <= 8 (8 consumer warps)
    g.ws = g.gs >= 5 ? 1 : (g.gs >= 3 ? 2 : (g.gs == 2 ? 4 : 8));
    const int nbmax = min(nb_cap, max(1, MV_MAX_BOXES / g.gs));
    const int nbox = KB / 8;
    g.nb = 1;
    for (int d = nbmax; d >= 1; --d)
        if (nbox % d == 0) { g.nb = d; break; }
    g.KC = 8 * g.nb;
    g.nchunks = KB / g.KC;
    return g;
}

}  // namespace brew
