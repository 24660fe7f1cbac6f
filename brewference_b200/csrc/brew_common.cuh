// brew_common.cuh — shared device/host helpers of libbrew (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <stdio.h>

#include "../../include/brew.h"

// ---------------------------------------------------------------------------
// host-side error plumbing
// ---------------------------------------------------------------------------
namespace brew {

int set_error(int code, const char* fmt, ...);
int cuda_error(cudaError_t e, const char* what);
void count_launch(int n = 1);

#define BREW_CUDA(call)                                                   \
    do {                                                                  \
        cudaError_t _e = (call);                                          \
        if (_e != cudaSuccess) return ::brew::cuda_error(_e, #call);      \
    } while (0)

#define BREW_CHECK(cond, code, ...)                                       \
    do {                                                                  \
        if (!(cond)) return ::brew::set_error((code), __VA_ARGS__);       \
    } while (0)

// GGML block geometry
struct TypeInfo {
    int block_elems;
    int block_bytes;
};

inline bool type_info(int type, TypeInfo* ti) {
    switch (type) {
        case BREW_TYPE_F32: *ti = {1, 4}; return true;
        case BREW_TYPE_F16: *ti = {1, 2}; return true;
        case BREW_TYPE_Q4_0: *ti = {32, 18}; return true;
        case BREW_TYPE_Q8_0: *ti = {32, 34}; return true;
        case BREW_TYPE_Q4_K: *ti = {256, 144}; return true;
        case BREW_TYPE_Q6_K: *ti = {256, 210}; return true;
        default: return false;
    }
}

inline bool is_quant_matrix_type(int type) {
    return type == BREW_TYPE_Q4_0 || type == BREW_TYPE_Q8_0 || type == BREW_TYPE_Q4_K || type == BREW_TYPE_Q6_K;
}

// Per-architecture rules of the reference's forward methods
// (model/*/...Transformer.java and their AttentionPattern classes).
// Gemma family: embeddings scaled by sqrt(dim), post-attention and post-FFN
// norms, GeGLU, local (sliding-window, base 1e4) and global (base 1e6) layers.
__host__ __device__ inline bool arch_gemma(int a) { return a == BREW_ARCH_GEMMA3 || a == BREW_ARCH_GEMMA2; }
// head-wise RMSNorm of q and k (Qwen3Transformer.java, Gemma3Transformer.java:42-43)
__host__ __device__ inline bool arch_qknorm(int a) { return a == BREW_ARCH_QWEN3 || a == BREW_ARCH_GEMMA3; }
// InterleavedRope pairs (2d, 2d+1) (Llama2Transformer.java:45, SmolLM3Transformer.java:60)
__host__ __device__ inline bool arch_interleaved(int a) { return a == BREW_ARCH_LLAMA || a == BREW_ARCH_SMOLLM3; }
// global attention layer: Gemma3AttentionPattern.java:10-12 (every 6th),
// Gemma2AttentionPattern.java:10-12 (every 2nd); other architectures attend
// to every position
__host__ __device__ inline bool arch_global_layer(int a, int l) {
    return a == BREW_ARCH_GEMMA3 ? (l + 1) % 6 == 0 : a == BREW_ARCH_GEMMA2 ? (l + 1) % 2 == 0 : true;
}
// RoPE applied at layer l (SmolLM3Transformer.java:48: not on every 4th layer)
__host__ __device__ inline bool arch_rope_layer(int a, int l) { return a != BREW_ARCH_SMOLLM3 || (l + 1) % 4 != 0; }
// sliding window of layer l (0: none)
__host__ __device__ inline int arch_window(int a, int l, int window) {
    return (arch_gemma(a) && !arch_global_layer(a, l)) ? window : 0;
}
// RoPE base of the global (or only) table and of the Gemma local table: the
// configured base when > 0, else the architecture's supplier value
inline float arch_rope_base(int a, float cfg_base, bool local) {
    if (cfg_base > 0.0f) return cfg_base;
    if (a == BREW_ARCH_LLAMA || a == BREW_ARCH_SMOLLM3) return 10000.0f;
    if (arch_gemma(a)) return local ? 10000.0f : 1000000.0f;
    return 1000000.0f;
}

// device-side error flags (one word per device, written by bounded waits)
#define BREW_DEVERR_TIMEOUT_FULL   1u
#define BREW_DEVERR_TIMEOUT_EMPTY  2u
#define BREW_DEVERR_BAD_INDEX      4u
#define BREW_DEVERR_BAD_TOKEN      8u

unsigned int* device_error_word();      // device pointer of this device's flag word
int check_device_error(const char* where);  // reads + clears the flag (synchronising)

// Sets a kernel's dynamic shared-memory limit on the current device the first
// time that device launches it.  The attribute is per device, so `done` keeps
// one bit per device ordinal (devices 64 and up set it on every call).
inline cudaError_t smem_attr_per_device(const void* fn, int bytes, unsigned long long* done) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 64 && ((*done >> dev) & 1ull)) return cudaSuccess;
    e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e == cudaSuccess && dev < 64) *done |= 1ull << dev;
    return e;
}

}  // namespace brew

// ---------------------------------------------------------------------------
// device helpers
// ---------------------------------------------------------------------------
#ifdef __CUDACC__

namespace brew {

// Bounded spin limits: a wait that exceeds them records an error flag and
// gives up instead of hanging the GPU.
#define BREW_SPIN_LIMIT (1u << 24)

__device__ __forceinline__ float half_bits_to_float(uint16_t h) {
    return __half2float(__ushort_as_half(h));
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---- mbarrier ------------------------------------------------------------
// 16-byte asynchronous global -> shared copy through L2 (sees the writes of
// other CTAs published by a grid barrier); completed by cp_async_wait_all.
__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gsrc) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
// Closes this thread's group of cp.async copies issued since the last commit.
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
// Waits until at most N of this thread's committed groups are still in flight.
template <int N>
__device__ __forceinline__ void cp_async_wait_group() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Waits for phase `parity` of `bar` for at most ~2 s (and at most
// BREW_SPIN_LIMIT polls); on timeout records `err` in the device error word
// and returns false, so a broken pipeline ends instead of hanging the GPU.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, unsigned int* err_word,
                                                  unsigned int err, uint64_t limit_ns = 2000000000ull) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    for (uint32_t it = 0; it < BREW_SPIN_LIMIT; ++it) {
        if (mbar_try_wait(bar, parity)) return true;
        __nanosleep(64);   // leave issue slots to the warps that compute
        if ((it & 255u) == 255u && global_ns() - t0 > limit_ns) break;
    }
    if (err_word) atomicOr(err_word, err);
    return false;
}

__device__ __forceinline__ unsigned long long ld_acquire_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ int ld_volatile_int(const int* p) { return *reinterpret_cast<const volatile int*>(p); }

// Waits until the counter *ctr reaches `target` (acquire), for at most
// limit_ns, or until *abort is set by another CTA that gave up.  Returns
// false on timeout or abort: the grid barrier's wait, which must end instead
// of hanging the GPU when an arrival never comes.
__device__ __forceinline__ bool wait_counter_bounded(const unsigned long long* ctr, unsigned long long target,
                                                     const int* abort, uint64_t limit_ns) {
    const uint64_t t0 = global_ns();
    uint32_t it = 0;
    while (ld_acquire_u64(ctr) < target) {
        __nanosleep(32);
        if ((++it & 63u) == 0u && (global_ns() - t0 > limit_ns || (abort && ld_volatile_int(abort)))) return false;
    }
    return true;
}

// Waits until the int counter reaches `target` (acquire), bounded like
// wait_counter_bounded.
__device__ __forceinline__ bool wait_int_bounded(const int* ctr, int target, const int* abort, uint64_t limit_ns) {
    const uint64_t t0 = global_ns();
    uint32_t it = 0;
    for (;;) {
        int v;
        asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(ctr) : "memory");
        if (v >= target) return true;
        __nanosleep(32);
        if ((++it & 63u) == 0u && (global_ns() - t0 > limit_ns || (abort && ld_volatile_int(abort)))) return false;
    }
}

// Bulk prefetch of `bytes` (multiple of 16, 16-byte aligned) into L2.
__device__ __forceinline__ void prefetch_l2(const void* src_gmem, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src_gmem), "r"(bytes) : "memory");
}

// ---- bulk async copy global -> this CTA's shared memory (TMA, non-tensor) ----
__device__ __forceinline__ void bulk_g2s(void* dst_smem, const void* src_gmem, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst_smem)),
        "l"(src_gmem), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// L2 policy for data read once per step (streamed weights): evict first, so
// that the KV rows and activations stay resident.
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}

// bulk_g2s with an L2 cache policy.
__device__ __forceinline__ void bulk_g2s_hint(void* dst_smem, const void* src_gmem, uint32_t bytes, uint64_t* bar,
                                              uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
            smem_u32(dst_smem)),
        "l"(src_gmem), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

// 2-D tiled TMA load through a tensor map into this CTA's shared memory: box at element
// coordinates (x, y) into shared memory, completing on `bar`.
__device__ __forceinline__ void tma_load_2d(void* dst_smem, const void* tmap, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(dst_smem)),
        "l"(tmap), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// ---- programmatic dependent launch -------------------------------------
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;"); }

// ---- misc ----------------------------------------------------------------
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ int warp_sum_i(int v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

}  // namespace brew

#endif  // __CUDACC__
