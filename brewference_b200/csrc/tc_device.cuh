// tc_device.cuh — device helpers of the tcgen05 kernels: shared-memory
// matrix and instruction descriptors, the int8 MMA, tensor-memory loads and
// stores, and packed fp32 pair arithmetic.
#pragma once

#include "brew_common.cuh"

namespace brew {

// ---- tcgen05 helpers (PTX forms as in CUTLASS's sm100 MMA / TMEM atoms) ----
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

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

__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// tcgen05.st of one 32-bit constant to 16 / 8 columns of this warp's 32 lanes.
__device__ __forceinline__ void tmem_st16_const(uint32_t taddr, uint32_t c) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, "
        "%1};" ::"r"(taddr),
        "r"(c)
        : "memory");
}
__device__ __forceinline__ void tmem_st8_const(uint32_t taddr, uint32_t c) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %1, %1, %1, %1, %1, %1, %1};" ::"r"(taddr), "r"(c)
                 : "memory");
}
__device__ __forceinline__ void tmem_st4_const(uint32_t taddr, uint32_t c) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1, %1, %1, %1};" ::"r"(taddr), "r"(c) : "memory");
}
__device__ __forceinline__ void tmem_ld4(uint32_t taddr, uint32_t* v) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3])
                 : "r"(taddr)
                 : "memory");
}
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t* v) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
                 : "r"(taddr)
                 : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Packed fp32 pairs (sm_100 f32x2 arithmetic): each half is an ordinary
// IEEE fp32 operation with round-to-nearest, two per instruction.
__device__ __forceinline__ uint64_t f2_pack(uint32_t lo, uint32_t hi) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "r"(lo), "r"(hi));
    return r;
}
__device__ __forceinline__ uint64_t f2_packf(float lo, float hi) {
    return f2_pack(__float_as_uint(lo), __float_as_uint(hi));
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
    uint64_t r;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
    uint64_t r;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
    return r;
}

// The int32 accumulators start at the bits of the float 1.5 * 2^23 instead
// of 0: the MMAs add an integer sum i (|i| < 2^22) to it, and the result's
// bits are the float 1.5 * 2^23 + i, exactly (the well-known magic-number
// conversion).  Subtracting 1.5 * 2^23 gives i as a float.
constexpr uint32_t TC_MAGIC = 0x4B400000u;
constexpr float TC_MAGIC_F = 12582912.0f;

// Byte offset of quant j (0..31) of row r (0..127) inside a 4096-byte
// block-column tile: the K-major core-matrix layout the MMA's shared-memory
// descriptor reads (8-row groups of 256 B, the two 16-byte K halves 128 B
// apart), so a stage is one contiguous copy.
__host__ __device__ __forceinline__ int tc_tile_off(int r, int j) {
    return (r >> 3) * 256 + (j >> 4) * 128 + (r & 7) * 16 + (j & 15);
}

}  // namespace brew
