// decode.cu — one decode step (TransformerGraph.forward + argmax) of the whole
// model as ONE persistent kernel on all SMs.
//
// Why: at batch 1 the step streams every weight byte once (1.83 GB for the
// Qwen3-1.7B shape) and the per-layer dependency chain (norm -> QKV ->
// attention -> wo -> norm -> gate/up -> down) is long.  As separate kernels
// each link pays a launch/ramp/drain gap and the HBM idles in between.  Here:
//   * one CTA per SM (cooperative launch); the last warp of every CTA is a producer
//     that streams the CTA's share of EVERY phase's weight tiles into a ring
//     of shared-memory stages, running ahead across phase boundaries.  The
//     weights are a fragment-packed copy (packed.cuh): a tile's block columns
//     are contiguous, so a stage is one 1-D bulk copy per tile into this
//     CTA's own shared memory;
//   * the other DK_CW warps consume: each phase starts by building its own prep records
//     (RMSNorm + limb split of the input vector, prep.cuh) in shared memory,
//     then multiplies the staged tiles (int8 MMA, warp w taking block columns
//     w, w + DK_CW, ... of every tile) and writes its output rows after a
//     cross-warp sum;
//   * no grid barrier separates the phases: every vector one phase hands to
//     the next is stored as tagged words (value | launch epoch, one 8-byte
//     store each) in its own slot per layer, and a reader polls the words it
//     needs until they carry this launch's epoch, so the wait for the data
//     is the data load itself (bounded wait);
//   * attention (QK-norm, RoPE from precomputed tables, KV append, chunked
//     softmax.V with a last-arriver combine) runs between the QKV and wo
//     phases on the consumer warps while the producer keeps streaming.
// Reference: model/*/...Transformer.java forward(), transformer/math/Linear.java,
// transformer/attention/AttentionEngine.java, Kernels.java.
#include "decode.cuh"

#include <cudaTypedefs.h>

#include <algorithm>
#include <cmath>

#include "matvec.cuh"
#include "mv_device.cuh"
#include "prep.cuh"
#include "quant_device.cuh"

namespace brew {

namespace {

enum { PH_QKV = 0, PH_O, PH_GU, PH_DOWN, PH_CLS, PH_ATTN };

constexpr int ATTN_MIN_POS = 32;   // positions per attention CTA at least
// dynamic shared memory of the decode kernel, at most: 226 KB of the 227 KB a
// block may opt in to (the kernel's static shared variables take the rest)
constexpr size_t DK_SMEM_BUDGET = 226 * 1024;
// consumer warps per CTA (one more warp streams the weights)
#ifndef DK_CONSUMER_WARPS
#define DK_CONSUMER_WARPS 8
#endif
constexpr int DK_CW = DK_CONSUMER_WARPS;
constexpr int DK_CT = DK_CW * 32;             // consumer threads
constexpr int DK_GMAX = 4;                    // tiles per group at most
constexpr int DK_PVK = 1024 / DK_CT;          // attention outputs per thread ([G][hd] <= 1024)
constexpr int DK_RED_BYTES = DK_CW * DK_GMAX * 16 * 2 * 4;   // cross-warp partial sums of a tile group

// Named barrier among the consumer warps.
__device__ __forceinline__ void dk_bar() { asm volatile("bar.sync 1, %0;" ::"n"(DK_CT) : "memory"); }
// The same barrier, returning the OR of v over the consumer threads: a wait
// that gave up in one thread stops the whole CTA at the same phase boundary
// (a thread leaving alone would strand the others at the next barrier).
__device__ __forceinline__ bool dk_bar_or(bool v) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\tbar.red.or.pred q, 1, %2, p;\n\tselp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)v), "n"(DK_CT)
        : "memory");
    return r != 0;
}

// ---- tagged activations ----
// A word is (epoch << 32) | the float's bits, stored and loaded as one
// aligned 8-byte access (single-copy atomic), so a reader that sees the
// epoch also sees the value written with it.  Each (layer, vector) slot is
// written once per launch, and the epoch changes every launch: a word from
// an earlier launch never passes for this one's, and no word is overwritten
// while another CTA may still read it.
typedef unsigned long long u64;

__shared__ uint32_t s_ep;   // this launch's epoch (never 0: the arena starts zeroed)

// Slot v of layer l; word i of sequence b is at [b * tg_ls + i].
__device__ __forceinline__ u64* tgp(const DecodeParams& P, int l, int v) {
    return P.tg + (int64_t)l * DK_MAX_BATCH * P.tg_ls + P.tg_off[v];
}
__device__ __forceinline__ u64 tag_word(float v, uint32_t ep) { return ((u64)ep << 32) | __float_as_uint(v); }
__device__ __forceinline__ bool tag_is(u64 w, uint32_t ep) { return (uint32_t)(w >> 32) == ep; }
__device__ __forceinline__ float tag_val(u64 w) { return __uint_as_float((uint32_t)w); }
__device__ __forceinline__ void st_tag(u64* p, float v, uint32_t ep) {
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(tag_word(v, ep)));
}
// four consecutive words (p 16-byte aligned)
__device__ __forceinline__ void st_tag4(u64* p, float4 v, uint32_t ep) {
    asm volatile("st.relaxed.gpu.global.v2.u64 [%0], {%1, %2};" ::"l"(p), "l"(tag_word(v.x, ep)), "l"(tag_word(v.y, ep)));
    asm volatile("st.relaxed.gpu.global.v2.u64 [%0], {%1, %2};" ::"l"(p + 2), "l"(tag_word(v.z, ep)),
                 "l"(tag_word(v.w, ep)));
}
__device__ __forceinline__ u64 ld_tag(const u64* p) {
    u64 a;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(a) : "l"(p));
    return a;
}
// two consecutive words (p 16-byte aligned): each is its own atomic access
__device__ __forceinline__ void ld_tag2(const u64* p, u64& a, u64& b) {
    asm volatile("ld.relaxed.gpu.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p));
}

// A wait for tagged data that gave up: error word and abort flag (the other
// CTAs' waits see the flag and end too).
__device__ __noinline__ void tag_fail(const DecodeParams& P) {
    atomicOr(P.err, BREW_DEVERR_TIMEOUT_FULL);
    atomicExch(P.abort, 1);
}

// Polls the word pair at p until both words carry epoch ep.  Bounded: gives
// up after 2 s, or as soon as the abort flag is raised; false then.
__device__ __noinline__ bool tag_wait2(const DecodeParams& P, const u64* p, uint32_t ep, u64& a, u64& b) {
    const uint64_t t0 = global_ns();
    for (uint32_t it = 1;; ++it) {
        ld_tag2(p, a, b);
        if (tag_is(a, ep) && tag_is(b, ep)) return true;
        if ((it & 63u) == 0 && (global_ns() - t0 > 2000000000ull || ld_volatile_int(P.abort))) {
            tag_fail(P);
            return false;
        }
    }
}

// The same for one word.
__device__ __noinline__ bool tag_wait1(const DecodeParams& P, const u64* p, uint32_t ep, u64& a) {
    const uint64_t t0 = global_ns();
    for (uint32_t it = 1;; ++it) {
        a = ld_tag(p);
        if (tag_is(a, ep)) return true;
        if ((it & 63u) == 0 && (global_ns() - t0 > 2000000000ull || ld_volatile_int(P.abort))) {
            tag_fail(P);
            return false;
        }
    }
}

// Reads this thread's word pairs i = threadIdx.x + DK_CT k (k < 32) of
// [0, n2), pair i at addr(i) (16-byte aligned), and hands each to
// use(i, x, y) once both words carry epoch ep.  A sweep walks the pairs
// still pending in order, four loads in flight; when some are unwritten,
// the first of them is polled alone and the rest are swept again after it
// lands (the producers' stores arrive close together).  False when a wait
// gave up.
template <class A, class U>
__device__ __forceinline__ bool tag_pairs(const DecodeParams& P, int n2, uint32_t ep, A addr, U use) {
    constexpr int W = 4;
    const int tid = threadIdx.x;
    const int nk = tid < n2 ? min(32, (n2 - tid + DK_CT - 1) / DK_CT) : 0;   // this thread's pairs
    uint32_t pend = nk == 32 ? 0xFFFFFFFFu : (1u << nk) - 1u;
    for (;;) {
        uint32_t left = 0;
        #pragma unroll 1
        for (int k0 = 0; k0 < nk; k0 += W) {
            if (((pend >> k0) & ((1u << W) - 1u)) == 0u) continue;
            u64 a[W], b[W];
#pragma unroll
            for (int u = 0; u < W; ++u)
                if ((pend >> (k0 + u)) & 1u) ld_tag2(addr(tid + DK_CT * (k0 + u)), a[u], b[u]);
#pragma unroll
            for (int u = 0; u < W; ++u) {
                if (!((pend >> (k0 + u)) & 1u)) continue;
                if (tag_is(a[u], ep) && tag_is(b[u], ep)) use(tid + DK_CT * (k0 + u), tag_val(a[u]), tag_val(b[u]));
                else left |= 1u << (k0 + u);
            }
        }
        if (!left) return true;
        const int k = __ffs(left) - 1;
        u64 a, b;
        if (!tag_wait2(P, addr(tid + DK_CT * k), ep, a, b)) return false;
        use(tid + DK_CT * k, tag_val(a), tag_val(b));
        pend = left & (left - 1u);
        if (!pend) return true;
    }
}
constexpr int DK_STAGE_BYTES = 64 * 544;           // one pipeline stage: 64 Q8_0 block-tiles

// One matvec phase over fragment-packed tiles (packed.cuh): y = W x for the
// tiles of this layer's family, split over the CTAs by whole tiles.
struct DPhase {
    const uint8_t* w;        // this layer's packed tiles
    int KB, tiles, rows, epi, ldy, tt, ph;
    bool argmax;
    float* y;                // the classifier's logits (plain floats)
    u64* ty;                 // the other phases' outputs (tagged words, sequence stride tg_ls)
    const u64* tresid;       // STORE: y = resid + (W x + bias), resid tagged
    const float* bias[3];    // bias of rows [r0[k], r0[k + 1]) is bias[k][row - r0[k]]
    int r0[4];
};

__device__ __forceinline__ DPhase make_phase(const DecodeParams& P, int l, int ph) {
    DPhase f = {};
    const int qw = P.n_heads * P.hd, kvd = P.n_kv * P.hd;
    const bool gem = arch_gemma(P.arch);
    f.epi = MV_EPI_STORE;
    f.tt = P.type_layer;
    f.ph = ph;
    switch (ph) {
        case PH_QKV:
            f.w = P.pk[PK_QKV] + (int64_t)l * P.pk_lb[PK_QKV];
            f.KB = P.dim / 32;
            f.rows = qw + 2 * kvd;
            f.ty = tgp(P, l, DK_TG_QKV);
            f.ldy = P.tg_ls;
            f.bias[0] = P.q_bias ? P.q_bias + (int64_t)l * qw : nullptr;
            f.bias[1] = P.k_bias ? P.k_bias + (int64_t)l * kvd : nullptr;
            f.bias[2] = P.v_bias ? P.v_bias + (int64_t)l * kvd : nullptr;
            f.r0[0] = 0;
            f.r0[1] = qw;
            f.r0[2] = qw + kvd;
            f.r0[3] = qw + 2 * kvd;
            f.tiles = f.rows / 16;
            break;
        case PH_O:
            f.w = P.pk[PK_O] + (int64_t)l * P.pk_lb[PK_O];
            f.KB = qw / 32;
            f.rows = P.dim;
            f.ty = tgp(P, l, gem ? DK_TG_XB2O : DK_TG_XMID);
            f.tresid = gem ? nullptr : tgp(P, l, DK_TG_XIN);
            f.ldy = P.tg_ls;
            f.tiles = P.dim / 16;
            break;
        case PH_GU:
            f.w = P.pk[PK_GU] + (int64_t)l * P.pk_lb[PK_GU];
            f.KB = P.dim / 32;
            f.rows = P.hidden;
            f.epi = gem ? MV_EPI_GLU_GELU : MV_EPI_GLU_SILU;
            f.ty = tgp(P, l, DK_TG_HB);
            f.ldy = P.tg_ls;
            f.tiles = P.hidden / 8;
            break;
        case PH_DOWN:
            f.w = P.pk[PK_DOWN] + (int64_t)l * P.pk_lb[PK_DOWN];
            f.KB = P.hidden / 32;
            f.rows = P.dim;
            f.ty = gem ? tgp(P, l, DK_TG_XB2D) : tgp(P, l + 1, DK_TG_XIN);
            f.tresid = gem ? nullptr : tgp(P, l, DK_TG_XMID);
            f.ldy = P.tg_ls;
            f.tiles = P.dim / 16;
            break;
        default:  // PH_CLS
            f.w = P.pk[PK_OUT];
            f.KB = P.dim / 32;
            f.rows = P.vocab;
            f.tt = P.type_out;
            f.argmax = true;
            f.y = P.logits;
            f.ldy = P.vocab;
            f.tiles = (P.vocab + 15) / 16;
            break;
    }
    return f;
}

// Stage geometry of a group of tiles: KC block columns of each tile per
// stage (a multiple of 8 dividing KB: warp w takes columns w, w + 8, ...).
// The group sizes and KC come from tables that decode_prepare fills (they
// maximise the bytes a stage carries).
struct PGeom {
    int KC, nchunks;
};

__device__ __forceinline__ int pk_gs(const DecodeParams& P, int ph, int nt) { return P.geo_gs[ph][min(nt, 9)]; }

// Tile groups hold 1, 2 or 4 tiles (the largest of those <= n): three
// instantiations of the group loop keep the kernel's code small enough for
// the instruction caches.
__device__ __forceinline__ int ng_pow2(int n) { return n >= 4 ? 4 : n >= 2 ? 2 : 1; }

// This CTA's tile range [t0, t1) of each matvec phase (PH_QKV .. PH_CLS): the
// tiles are split over the CTAs in order, computed once at kernel start.
__shared__ int s_tiles[5][2];

__device__ __forceinline__ PGeom pk_geom(const DecodeParams& P, int ph, int ng, int KB) {
    PGeom g;
    g.KC = P.geo_kc[ph][ng];
    g.nchunks = P.geo_nch[ph][ng];
    return g;
}


// Sum over the consumer threads.
__device__ __forceinline__ float consumer_sum(float v, float* red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    v = warp_sum(v);
    if (lane == 0) red[warp] = v;
    dk_bar();
    float t = 0.0f;
#pragma unroll
    for (int w = 0; w < DK_CW; ++w) t += red[w];
    dk_bar();
    return t;
}

enum { SRC_EMBED = 0, SRC_PLAIN = 1, SRC_GEMMA_ADD = 2 };

// Copies n4 float4 from global memory (through L2: the data may have been
// written by other CTAs of this kernel) to shared memory, and optionally a
// second array beside it, as asynchronous copies that are all in flight at
// once (completed by cp_async_wait_all).
__device__ __forceinline__ void stage_async(float4* d0, const float4* s0, float4* d1, const float4* s1, int n4) {
    #pragma unroll 1
    for (int i = threadIdx.x; i < n4; i += DK_CT) {
        if (s0) cp_async16(d0 + i, s0 + i);
        if (s1) cp_async16(d1 + i, s1 + i);
    }
}

// Builds the prep records of one phase's input vector(s) in shared memory.
//   SRC_EMBED      v = dequant(token row) (* sqrt(dim), Gemma3); written to xout
//   SRC_PLAIN      v = src
//   SRC_GEMMA_ADD  v = src + rmsnorm(t, tw)   (Gemma3 post-norm residual); written to xout
// then records of rmsnorm(v, nw) (nw != null) or of v.  src, t and xout are
// tagged slots (sequence stride tg_ls).  The vector is staged in shared
// memory (`vec`, K floats) and the norm weight beside it (K more floats).
// xout writes are split over the CTAs by block (block j by CTA j % G), so
// each element has one writer.  `lsum`: the consumer multiplies Q4_0 blocks
// (needs the limb sums).  `nw_staged` (SRC_PLAIN): this thread already
// issued the copy of nw into the weight half of `vec` (stage_norm).  False
// when a wait for tagged input gave up.
__device__ bool prep_phase(const DecodeParams& P, int mode, const u64* src, int K, const float* nw, const u64* t,
                           const float* tw, u64* xout, uint8_t* prep, float* vec, float* red, bool lsum,
                           unsigned long long* t_wave, bool nw_staged, uint32_t ep) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int KB = K / 32, K4 = K / 4, K2 = K / 2;
    const int G = gridDim.x;
    const int ls = P.tg_ls;
    float4* v4 = reinterpret_cast<float4*>(vec);
    float2* v2 = reinterpret_cast<float2*>(vec);
    float4* w4 = v4 + K4;
    const float2* w2 = reinterpret_cast<const float2*>(vec + K);
    const float4* nw4 = reinterpret_cast<const float4*>(nw);
    bool ok_all = true;
    #pragma unroll 1
    for (int b = 0; b < P.batch; ++b) {
        float ss = 0.0f;
        if (mode == SRC_EMBED) {
            int tok = P.use_imm ? P.tok_imm : P.tokens[b];
            if (tok < 0 || tok >= P.vocab) {
                if (threadIdx.x == 0) atomicOr(P.err, BREW_DEVERR_BAD_TOKEN);
                tok = 0;
            }
            const float es = (float)sqrt((double)K);   // Kernels.scaleEmbeddings
            #pragma unroll 1
            for (int i = threadIdx.x; i < K; i += DK_CT) {
                float v = dequant_elem(P.type_embed, P.embed, (int64_t)tok * K + i);
                vec[i] = arch_gemma(P.arch) ? __fmul_rn(v, es) : v;
            }
            if (nw) stage_async(w4, nullptr, w4, nw4, K4);
            cp_async_wait_all();
            dk_bar();
            #pragma unroll 1
            for (int i = threadIdx.x; i < K; i += DK_CT) ss += vec[i] * vec[i];
        } else if (mode == SRC_GEMMA_ADD) {
            stage_async(w4, nullptr, w4, reinterpret_cast<const float4*>(tw), K4);
            const u64* tb = t + (int64_t)b * ls;
            float tss = 0.0f;
            ok_all &= tag_pairs(P, K2, ep, [&](int i) { return tb + 2 * i; },
                                [&](int i, float x, float y) {
                                    v2[i] = make_float2(x, y);
                                    tss += x * x + y * y;
                                });
            cp_async_wait_all();
            const float tsc = rms_scale(consumer_sum(tss, red), K, P.eps);
            // each thread combines the pairs it staged itself
            const u64* sb = src + (int64_t)b * ls;
            ok_all &= tag_pairs(P, K2, ep, [&](int i) { return sb + 2 * i; },
                                [&](int i, float x, float y) {
                                    const float2 tv = v2[i], w = w2[i];
                                    v2[i] = make_float2(x + tv.x * tsc * w.x, y + tv.y * tsc * w.y);
                                });
            dk_bar();   // every thread is done with tw before nw replaces it
            if (nw) stage_async(w4, nullptr, w4, nw4, K4);
            cp_async_wait_all();
            #pragma unroll 1
            for (int i = threadIdx.x; i < K2; i += DK_CT) {
                const float2 v = v2[i];
                ss += v.x * v.x + v.y * v.y;
            }
        } else {
            if (nw && !(nw_staged && b == 0)) stage_async(w4, nullptr, w4, nw4, K4);
            const u64* sb = src + (int64_t)b * ls;
            ok_all &= tag_pairs(P, K2, ep, [&](int i) { return sb + 2 * i; },
                                [&](int i, float x, float y) {
                                    v2[i] = make_float2(x, y);
                                    ss += x * x + y * y;
                                });
            cp_async_wait_all();
        }
        // one barrier publishes the staged vector and the partial sums
        if (nw) {
            ss = warp_sum(ss);
            if (lane == 0) red[warp] = ss;
        }
        dk_bar();
        if (t_wave && b == 0) *t_wave = global_ns();
        float scale = 1.0f;
        if (nw) {
            float tot = 0.0f;
#pragma unroll
            for (int w = 0; w < DK_CW; ++w) tot += red[w];
            scale = rms_scale(tot, K, P.eps);
        }
        // two independent block quads per iteration (their shuffle and
        // divide chains overlap)
        const int gq = lane >> 3, e = (lane & 7) * 4;
        #pragma unroll 1
        for (int j0 = warp * 4; j0 < KB; j0 += 8 * DK_CW) {
            int jj[2];
            bool ok[2];
            float4 v[2];
#pragma unroll
            for (int u = 0; u < 2; ++u) {
                const int j = j0 + 4 * DK_CW * u + gq;
                ok[u] = j < KB;
                jj[u] = ok[u] ? j : KB - 1;
                v[u] = v4[(32 * jj[u] + e) >> 2];
                if (xout && ok[u] && (j % G) == (int)blockIdx.x) st_tag4(xout + (int64_t)b * ls + 32 * j + e, v[u], ep);
                if (nw) {
                    const float4 w = w4[(32 * jj[u] + e) >> 2];
                    v[u].x = v[u].x * scale * w.x;
                    v[u].y = v[u].y * scale * w.y;
                    v[u].z = v[u].z * scale * w.z;
                    v[u].w = v[u].w * scale * w.w;
                }
            }
#pragma unroll
            for (int u = 0; u < 2; ++u) prep_emit_quad(prep + (size_t)jj[u] * P.rec_bytes, P.batch, b, v[u], ok[u], lsum);
        }
        dk_bar();
    }
    return ok_all;
}

struct Ring {
    uint64_t* full;
    uint64_t* empty;
    uint8_t* stages;
    int ns, stage_bytes;
};

// Position in the ring: the stage counter q, its slot q % ns and the parity
// (q / ns) & 1 of the slot's barrier phase, advanced without divisions.
struct RingPos {
    int q = 0, slot = 0;
    uint32_t par = 0;
    __device__ __forceinline__ void advance(int ns) {
        ++q;
        if (++slot == ns) {
            slot = 0;
            par ^= 1u;
        }
    }
};


// This lane's operand offsets inside a prep record (prep.cuh): B column g =
// limb (g & 3) of vector g >> 2; accumulator columns 2t, 2t+1 belong to
// vector t >> 1 (limbs (2t) & 3 and (2t + 1) & 3).
struct LaneOps {
    uint32_t boff, soff, loff0, loff1;
    bool vB, vC;
    int l0, bC;
};

// The stages of one tile group of NG tiles, then the limb combine of each
// warp's partial sums into `red`.  NG is a compile-time count: the tile loop
// is straight-line code, so the compiler schedules every tile's loads ahead
// of the MMAs (with a run-time count and predicated tile slots, the loop
// measured 2.5-3x slower per block column for one and two tiles).
template <int TT, int NG>
__device__ __forceinline__ void mv_group(const DecodeParams& P, const PGeom& geo, const Ring& ring, RingPos& rp,
                                         uint32_t prep_s, const LaneOps& o, float* red, bool& aborted,
                                         unsigned long long* t_full, unsigned long long* detail, int& dch) {
    constexpr int BS = pk_block_bytes(TT), SO = pk_scale_off(TT);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, t = lane & 3;
    float acc[NG][4];
#pragma unroll
    for (int k = 0; k < NG; ++k) acc[k][0] = acc[k][1] = acc[k][2] = acc[k][3] = 0.0f;
    for (int chunk = 0; chunk < geo.nchunks; ++chunk, rp.advance(ring.ns)) {
        const int stage = rp.slot;
        if (!aborted && !mbar_wait_bounded(&ring.full[stage], rp.par, P.err, BREW_DEVERR_TIMEOUT_FULL))
            aborted = true;
        if (t_full && warp == 0) *t_full = global_ns();
        if (detail && tid == 0 && dch < DK_DETAIL) detail[DK_DETAIL + dch] = global_ns();
        if (!aborted) {
            const uint32_t sb = smem_u32(ring.stages + (size_t)stage * ring.stage_bytes);
            for (int kb = warp; kb < geo.KC; kb += DK_CW) {
                const uint32_t rec = prep_s + (chunk * geo.KC + kb) * P.rec_bytes;
                uint32_t b0 = lds32(rec + o.boff), b1 = lds32(rec + o.boff + 16);
                if (!o.vB) b0 = b1 = 0u;
                const float s = o.vC ? ldsf(rec + o.soff) : 0.0f;
                int ls0 = 0, ls1 = 0;
                if (TT == BREW_TYPE_Q4_0) {   // Q4_0 quants are stored as q + 8
                    ls0 = o.vC ? 8 * (int)lds32(rec + o.loff0) : 0;
                    ls1 = (o.vC && o.l0 == 0) ? 8 * (int)lds32(rec + o.loff1) : 0;
                }
#pragma unroll
                for (int k = 0; k < NG; ++k) {
                    const uint32_t blk = sb + (k * geo.KC + kb) * BS;
                    int c[4];
                    if (TT == BREW_TYPE_Q8_0) {
                        const uint4 A = *reinterpret_cast<const uint4*>(sptr(blk + lane * 16));
                        mma_s8s8(c, A.x, A.y, A.z, A.w, b0, b1);
                    } else {
                        const uint2 W = *reinterpret_cast<const uint2*>(sptr(blk + lane * 8));
                        mma_u8s8(c, W.x & 0x0F0F0F0Fu, W.y & 0x0F0F0F0Fu, (W.x >> 4) & 0x0F0F0F0Fu,
                                 (W.y >> 4) & 0x0F0F0F0Fu, b0, b1);
                        c[0] -= ls0;
                        c[1] -= ls1;
                        c[2] -= ls0;
                        c[3] -= ls1;
                    }
                    const uint32_t dd = lds32(blk + SO + 4 * g);
                    const float ds0 = h2f_lo(dd) * s, ds1 = h2f_hi(dd) * s;
                    acc[k][0] = fmaf((float)c[0], ds0, acc[k][0]);
                    acc[k][1] = fmaf((float)c[1], ds0, acc[k][1]);
                    acc[k][2] = fmaf((float)c[2], ds1, acc[k][2]);
                    acc[k][3] = fmaf((float)c[3], ds1, acc[k][3]);
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&ring.empty[stage]);
        if (detail && tid == 0 && dch < DK_DETAIL) detail[2 * DK_DETAIL + dch] = global_ns();
        ++dch;
    }
    // limbs hi / mid (lane t even) and lo (lane t + 1) -> one value per row
    // and vector: v = (lo + mid * 2^8) + hi * 2^16
#pragma unroll
    for (int k = 0; k < NG; ++k) {
        const float lo0 = __shfl_down_sync(0xffffffffu, acc[k][0], 1);
        const float lo1 = __shfl_down_sync(0xffffffffu, acc[k][2], 1);
        if ((t & 1) == 0 && o.vC) {
            red[((warp * DK_GMAX + k) * 16 + g) * 2 + o.bC] = (lo0 + acc[k][1] * 256.0f) + acc[k][0] * 65536.0f;
            red[((warp * DK_GMAX + k) * 16 + g + 8) * 2 + o.bC] = (lo1 + acc[k][3] * 256.0f) + acc[k][2] * 65536.0f;
        }
    }
}

// Consumer side of one matvec phase: this CTA's tiles in groups of up to 8,
// stage by stage.  Warp w multiplies block columns w, w + 8, ... of the stage
// for every tile of the group (the x operand of a column is loaded once and
// used for all tiles).  At the end of a group the warps' partial sums meet
// in shared memory (`red`, [8 warps][8 tiles][16 rows][2 vectors]) and each
// of the 256 threads finishes one output.
template <int TT, int NT>
__device__ void mv_phase(const DecodeParams& P, const DPhase& f, const Ring& ring, RingPos& rp, uint32_t prep_s,
                         float* red, unsigned long long* s_best, bool& aborted, unsigned long long* t_full,
                         unsigned long long* detail, uint32_t ep) {
    int dch = 0;
    static_assert(NT == 1, "decode batch <= 2: one n8 column tile");
    constexpr int BS = pk_block_bytes(TT);
    const int tid = threadIdx.x, lane = tid & 31;
    const int g = lane >> 2, t = lane & 3;
    const int t0 = s_tiles[f.ph][0], t1 = s_tiles[f.ph][1];
    const int nt = t1 - t0;
    if (nt <= 0) return;
    const int batch = P.batch;
    const int gs = pk_gs(P, f.ph, nt);
    const bool glu = f.epi != MV_EPI_STORE;
    const int lg_tile = (glu ? 3 : 4) + (batch == 2 ? 1 : 0);   // log2 of the outputs per tile
    LaneOps o;
    {
        const int bB = g >> 2, lB = g & 3;
        o.vB = lB < 3 && bB < batch;
        o.boff = (o.vB ? (3 * bB + lB) * 32 : 0) + 4 * t;
        o.bC = t >> 1;
        o.vC = o.bC < batch;
        const int bCs = o.vC ? o.bC : 0;
        o.l0 = (2 * t) & 3;
        o.soff = prep_s_off(batch) + 4 * bCs;
        o.loff0 = prep_lsum_off(batch) + 4 * (3 * bCs + o.l0);
        o.loff1 = prep_lsum_off(batch) + 4 * (3 * bCs + 1);
    }
    for (int tg0 = t0; tg0 < t1; tg0 += ng_pow2(min(gs, t1 - tg0))) {
        const int ng = ng_pow2(min(gs, t1 - tg0));
        const PGeom geo = pk_geom(P, f.ph, ng, f.KB);
        // this thread's output of the group: its bias and residual are read
        // now, so that their latency overlaps the MMA loop
        // per_tile = (8 or 16) * batch, batch 1 or 2: powers of two
        const int ok = tid >> lg_tile, orem = tid & ((1 << lg_tile) - 1);
        const int orow = batch == 2 ? orem >> 1 : orem, ob = batch == 2 ? (orem & 1) : 0;
        float pb = 0.0f;
        u64 rw = 0;   // the residual's tagged word (checked after the MMA loop)
        if (!glu && ok < ng) {
            const int row = (tg0 + ok) * 16 + orow;
            if (row < f.rows) {
                for (int k = 0; k < 3; ++k)
                    if (f.bias[k] && row >= f.r0[k] && row < f.r0[k + 1]) pb = __ldg(&f.bias[k][row - f.r0[k]]);
                if (f.tresid) rw = ld_tag(&f.tresid[(int64_t)ob * f.ldy + row]);
            }
        }
        switch (ng) {
            case 1: mv_group<TT, 1>(P, geo, ring, rp, prep_s, o, red, aborted, t_full, detail, dch); break;
            case 2: mv_group<TT, 2>(P, geo, ring, rp, prep_s, o, red, aborted, t_full, detail, dch); break;
            default: mv_group<TT, 4>(P, geo, ring, rp, prep_s, o, red, aborted, t_full, detail, dch); break;
        }
        dk_bar();
        if (ok < ng) {
            auto V = [&](int r) {
                float v = 0.0f;
#pragma unroll
                for (int w = 0; w < DK_CW; ++w) v += red[((w * DK_GMAX + ok) * 16 + r) * 2 + ob];
                return v;
            };
            if (!glu) {
                const int row = (tg0 + ok) * 16 + orow;
                if (row < f.rows) {
                    float v = V(orow);
                    bool hb = false;
                    for (int k = 0; k < 3; ++k) hb |= f.bias[k] && row >= f.r0[k] && row < f.r0[k + 1];
                    if (hb) v = v + pb;
                    if (f.tresid) {
                        const u64* rp_ = &f.tresid[(int64_t)ob * f.ldy + row];
                        if (!tag_is(rw, ep) && !tag_wait1(P, rp_, ep, rw)) aborted = true;
                        v = tag_val(rw) + v;
                    }
                    if (f.argmax) {
                        f.y[(int64_t)ob * f.ldy + row] = v;
                        atomicMax(&s_best[ob], argmax_key(v, row));
                    } else {
                        st_tag(&f.ty[(int64_t)ob * f.ldy + row], v, ep);
                    }
                }
            } else {
                const int i = (tg0 + ok) * 8 + orow;
                st_tag(&f.ty[(int64_t)ob * f.ldy + i], act_glu(V(orow), f.epi) * V(orow + 8), ep);
            }
        }
        dk_bar();
    }
}

// Producer side of one matvec phase: the same tiles and stages, in order;
// one bulk copy per tile per stage (the tile's KC block-tiles are contiguous).
template <int TT>
__device__ void produce_phase(const DecodeParams& P, const DPhase& f, const Ring& ring, RingPos& rp,
                                           unsigned long long* detail) {
    int dch = 0;
    const uint64_t pol = l2_evict_first_policy();
    constexpr int BS = pk_block_bytes(TT);
    const int lane = threadIdx.x & 31;
    const int t0 = s_tiles[f.ph][0], t1 = s_tiles[f.ph][1];
    const int nt = t1 - t0;
    if (nt <= 0) return;
    const int gs = pk_gs(P, f.ph, nt);
    for (int tg0 = t0; tg0 < t1; tg0 += ng_pow2(min(gs, t1 - tg0))) {
        const int ng = ng_pow2(min(gs, t1 - tg0));
        const PGeom geo = pk_geom(P, f.ph, ng, f.KB);
        const uint32_t cbytes = (uint32_t)geo.KC * BS;
        for (int chunk = 0; chunk < geo.nchunks; ++chunk, rp.advance(ring.ns)) {
            const int stage = rp.slot;
            if (rp.q >= ring.ns) {   // wait for the consumers to release the slot's previous use
                bool ok = false;
                const uint64_t t0ns = global_ns();
                for (uint32_t it = 0;; ++it) {
                    if (mbar_try_wait(&ring.empty[stage], rp.par ^ 1u)) { ok = true; break; }
                    __nanosleep(128);   // the ring is full: do not steal issue slots from the consumers
                    if ((it & 255u) == 255u && (global_ns() - t0ns > 2000000000ull || ld_volatile_int(P.abort))) break;
                }
                if (!ok) {
                    if (lane == 0) {
                        atomicOr(P.err, BREW_DEVERR_TIMEOUT_EMPTY);
                        atomicExch(P.abort, 1);
                    }
                    rp.q = 1 << 30;   // stop producing
                    return;
                }
            }
            uint8_t* sbase = ring.stages + (size_t)stage * ring.stage_bytes;
            if (detail && lane == 0 && dch < DK_DETAIL) detail[dch] = global_ns();
            ++dch;
            if (lane == 0) mbar_arrive_expect_tx(&ring.full[stage], (uint32_t)ng * cbytes);
            __syncwarp();
            if (lane < ng)
                bulk_g2s_hint(sbase + (size_t)lane * cbytes,
                         f.w + ((int64_t)(tg0 + lane) * f.KB + (int64_t)chunk * geo.KC) * BS, cbytes, &ring.full[stage], pol);
            __syncwarp();
        }
    }
}

// Attention for the items of this CTA (AttentionEngine.attend), then the
// last CTA of each (sequence, kv head) combines the chunks into xb.
//
// An item is (sequence, kv head, chunk of positions).  Everything it reads
// (its q heads, the new k and v, the head-norm weights, the RoPE row and the
// K / V rows of the chunk) is fetched with asynchronous global->shared copies
// issued together, so the item waits for one memory round trip instead of
// one per dependent load.  Chunks longer than P.attn_sub positions are
// walked in rounds with a running (online) softmax.  `sm` is the attention
// area of shared memory (P.attn_floats floats):
//   K rows [SUB][hd] | V rows [SUB][hd] | q [G][hd] | k [hd] | v [hd] |
//   q-norm w [hd] | k-norm w [hd] | cos [hd/2] | sin [hd/2] |
//   scores [G][SUB] | per head: running max, running sum, round rescale, -
// and, for the combine, the partials [heads][nchunk][hd + 4].
// Head-wise RMSNorm (when w is given: Kernels.headWiseRmsNorm) and RoPE (when
// rope: InterleavedRope pairs (2d, 2d+1) or NonInterleavedRope pairs
// (d, d + hd/2), RopeCache cos / sin rows cs, sn) of one head vector in shared
// memory by one warp: lane holds elements lane + 32 r, r < R = hd / 32.
template <int R>
__device__ __forceinline__ void norm_rope_warp_t(float* v, const float* w, float eps, bool rope, bool inter,
                                                 const float* cs, const float* sn) {
    const int lane = threadIdx.x & 31;
    float x[R];
#pragma unroll
    for (int r = 0; r < R; ++r) x[r] = v[lane + 32 * r];
    if (w) {
        float ss = 0.0f;
#pragma unroll
        for (int r = 0; r < R; ++r) ss += x[r] * x[r];
        const float scale = rms_scale(warp_sum(ss), 32 * R, eps);
#pragma unroll
        for (int r = 0; r < R; ++r) x[r] = x[r] * scale * w[lane + 32 * r];
    }
    if (rope) {
        if (inter) {   // partner element i ^ 1: the neighbouring lane, same register
#pragma unroll
            for (int r = 0; r < R; ++r) {
                const float other = __shfl_xor_sync(0xffffffffu, x[r], 1);
                const int i = lane + 32 * r, d = i >> 1;
                const float c = cs[d], s = sn[d];
                x[r] = (i & 1) == 0 ? __fsub_rn(__fmul_rn(x[r], c), __fmul_rn(other, s))
                                    : __fadd_rn(__fmul_rn(other, s), __fmul_rn(x[r], c));
            }
        } else {       // partner element i + hd/2: register r + R/2 of the same lane
#pragma unroll
            for (int r = 0; r < R / 2; ++r) {
                const int d = lane + 32 * r;
                const float a = x[r], b = x[r + R / 2], c = cs[d], s = sn[d];
                x[r] = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s));
                x[r + R / 2] = __fadd_rn(__fmul_rn(a, s), __fmul_rn(b, c));
            }
        }
    }
    __syncwarp();
#pragma unroll
    for (int r = 0; r < R; ++r) v[lane + 32 * r] = x[r];
    __syncwarp();
}

__device__ __noinline__ void norm_rope_warp(float* v, int hd, const float* w, float eps, bool rope, bool inter,
                                            const float* cs, const float* sn) {
    if (hd == 64) norm_rope_warp_t<2>(v, w, eps, rope, inter, cs, sn);
    else if (hd == 128) norm_rope_warp_t<4>(v, w, eps, rope, inter, cs, sn);
    else norm_rope_warp_t<8>(v, w, eps, rope, inter, cs, sn);
}

// One attention item: sequence b, kv head hk, chunk c of the positions
// start .. pos (Gemma3's local layers: the last `window` positions), split
// into chunks of `per` positions; `used` chunks are non-empty.
struct AttnItem {
    int c, hk, b, pos, p0, n, used;
};

// This step's position of each sequence, read from P.pos once at kernel start.
__shared__ int s_pos[DK_MAX_BATCH];

// Chunk geometry of each sequence's attention for this step, computed once
// at kernel start: [sequence][0: all positions, 1: sliding window] =
// {start, positions per chunk, used chunks} (used = 0: no valid position).
__shared__ int s_attg[DK_MAX_BATCH][2][3];
// (chunk, kv head, sequence) of this CTA's first attention item (blockIdx.x)
__shared__ int s_item0[3];

__device__ __forceinline__ void attn_geometry(const DecodeParams& P, int b, int windowed, int* g) {
    const int pos = b < P.batch ? (P.use_imm ? P.pos_imm : P.pos[b]) : -1;
    g[0] = g[1] = g[2] = 0;
    if (pos < 0 || pos >= P.seq_len) return;
    const int nch = P.nchunk;
    const int start = (windowed && P.window > 0) ? max(0, pos - P.window + 1) : 0;
    const int len = pos - start + 1;
    const int per = max(ATTN_MIN_POS, (len + nch - 1) / nch);
    g[0] = start;
    g[1] = per;
    g[2] = (len + per - 1) / per;
}

__device__ __forceinline__ bool attn_item(const DecodeParams& P, int l, int item, AttnItem& it) {
    const int nch = P.nchunk;
    const bool windowed = arch_window(P.arch, l, P.window) > 0;   // Gemma2/Gemma3AttentionPattern.java:10-16
    if (item == (int)blockIdx.x) {
        it.c = s_item0[0];
        it.hk = s_item0[1];
        it.b = s_item0[2];
    } else {
        it.c = item % nch;
        it.hk = (item / nch) % P.n_kv;
        it.b = item / (nch * P.n_kv);
    }
    it.pos = s_pos[it.b];
    const int* g = s_attg[it.b][windowed ? 1 : 0];
    if (it.pos < 0 || it.pos >= P.seq_len || g[2] == 0) return false;
    const int start = g[0], per = g[1];
    it.used = g[2];
    it.p0 = start + it.c * per;
    it.n = max(0, min(it.pos + 1, it.p0 + per) - it.p0);
    return true;
}

// Asynchronous copies of the cached K / V rows of positions p0 + r0 ..
// p0 + r0 + SUB - 1 of an item into shared memory (kb, vb: [SUB][hd]); the
// row of this step's position is skipped (it comes from this step's k / v).
__device__ __forceinline__ void attn_issue_kv(const DecodeParams& P, int l, const AttnItem& it, int r0, float* kb,
                                              float* vb) {
    const int hd = P.hd, hd4 = hd / 4, kvd = P.n_kv * hd;
    const int lg4 = 31 - __clz(hd4);   // hd is a power of two
    const int ns = min(P.attn_sub, it.n - r0);
    const float* kc = P.kc + (int64_t)it.b * P.cache_bstride + (int64_t)l * P.seq_len * kvd;
    const float* vc = P.vc + (int64_t)it.b * P.cache_bstride + (int64_t)l * P.seq_len * kvd;
    #pragma unroll 1
    for (int i = threadIdx.x; i < ns * hd4; i += DK_CT) {
        const int r = i >> lg4, ci = i & (hd4 - 1);
        const int p = it.p0 + r0 + r;
        if (p == it.pos) continue;
        const int64_t off = (int64_t)p * kvd + (int64_t)it.hk * hd + 4 * ci;
        cp_async16(kb + r * hd + 4 * ci, kc + off);
        cp_async16(vb + r * hd + 4 * ci, vc + off);
    }
}

// Loads E consecutive floats (E = 2, 4 or 8: 8-, 16- or 2x16-byte aligned).
template <int E>
__device__ __forceinline__ void lds_vec(const float* p, float* v) {
    if constexpr (E == 2) {
        const float2 a = *reinterpret_cast<const float2*>(p);
        v[0] = a.x; v[1] = a.y;
    } else {
#pragma unroll
        for (int k = 0; k < E; k += 4) {
            const float4 a = *reinterpret_cast<const float4*>(p + k);
            v[k] = a.x; v[k + 1] = a.y; v[k + 2] = a.z; v[k + 3] = a.w;
        }
    }
}

// The rounds of one attention item with the positions split over the warps:
// warp w takes positions w, w + 8, ... of each round (K / V rows staged in
// shared memory, kb / vb [SUB][hd]); lane holds elements lane * E .. + E - 1
// of every row, q and the unnormalised output of each of the G <= GM heads in
// registers, and an online softmax (running max m and sum l per head) over
// the warp's positions, so no CTA barrier separates scores, softmax and the
// weighted sum.  At the end the warps' (m, l, o) meet in shared memory (the
// K staging area) and the CTA's partial for chunk c is written to pbase in
// the layout of the cross-CTA combine: [head][chunk][m, l, -, -, o[hd]].
template <int E, int GM, int JM>
__device__ __forceinline__ void attn_rounds_warp(const DecodeParams& P, int l, const AttnItem& it, float* kb, float* vb,
                                 const float* qs, const float* ks, const float* vs, float* pbase, int nch,
                                 unsigned long long* detail) {
    const int G = P.n_heads / P.n_kv, hd = 32 * E, SUB = P.attn_sub;   // SUB <= 8 JM
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int n = it.n, p0 = it.p0, pos = it.pos, c = it.c;
    const bool has_pos = pos >= p0 && pos < p0 + n;
    const float NEG = -INFINITY;
    float qr[GM][E], o[GM][E], m[GM], ls[GM];
#pragma unroll
    for (int h = 0; h < GM; ++h) {
        m[h] = NEG;
        ls[h] = 0.0f;
#pragma unroll
        for (int e = 0; e < E; ++e) o[h][e] = 0.0f;
    }
    #pragma unroll 1
    for (int r0 = 0; r0 < n; r0 += SUB) {
        const int ns = min(SUB, n - r0);
        if (r0 > 0) {
            attn_issue_kv(P, l, it, r0, kb, vb);
            cp_async_wait_all();
            if (has_pos && pos - p0 >= r0 && pos - p0 < r0 + ns) {
                const int r = pos - p0 - r0;
                #pragma unroll 1
                for (int i = tid; i < hd; i += DK_CT) {
                    kb[r * hd + i] = ks[i];
                    vb[r * hd + i] = vs[i];
                }
            }
        }
        dk_bar();
        if (r0 == 0) {
            if (detail && tid == 0) detail[9] = global_ns();
#pragma unroll
            for (int h = 0; h < GM; ++h)
                if (h < G) lds_vec<E>(qs + h * hd + lane * E, qr[h]);
        }
        // scores q.k / sqrt(hd) of this warp's positions
        float sc[JM][GM];
#pragma unroll
        for (int j = 0; j < JM; ++j) {
            const int t = warp + 8 * j;
            float kt[E];
            if (t < ns) lds_vec<E>(kb + t * hd + lane * E, kt);
            else
#pragma unroll
                for (int e = 0; e < E; ++e) kt[e] = 0.0f;
#pragma unroll
            for (int h = 0; h < GM; ++h) {
                float a = 0.0f;
                if (h < G)
#pragma unroll
                    for (int e = 0; e < E; ++e) a = fmaf(qr[h][e], kt[e], a);
                sc[j][h] = a;
            }
        }
#pragma unroll
        for (int j = 0; j < JM; ++j)
#pragma unroll
            for (int h = 0; h < GM; ++h) {
                const float v = warp_sum(sc[j][h]) * P.inv_scale;
                sc[j][h] = (warp + 8 * j < ns) ? v : NEG;
            }
        // online softmax and the weighted sum of this warp's V rows
#pragma unroll
        for (int h = 0; h < GM; ++h) {
            if (h >= G) continue;
            float mx = m[h];
#pragma unroll
            for (int j = 0; j < JM; ++j) mx = fmaxf(mx, sc[j][h]);
            if (mx == NEG) continue;   // no position of this warp yet
            const float corr = expf(m[h] - mx);
            ls[h] *= corr;
#pragma unroll
            for (int e = 0; e < E; ++e) o[h][e] *= corr;
            m[h] = mx;
#pragma unroll
            for (int j = 0; j < JM; ++j) {
                const int t = warp + 8 * j;
                if (t < ns) {
                    const float pj = expf(sc[j][h] - mx);
                    ls[h] += pj;
                    float vt[E];
                    lds_vec<E>(vb + t * hd + lane * E, vt);
#pragma unroll
                    for (int e = 0; e < E; ++e) o[h][e] = fmaf(pj, vt[e], o[h][e]);
                }
            }
        }
        dk_bar();   // the next round's copies overwrite kb / vb
    }
    // the warps' partials meet in the staging area: [warp][head][m, l, o[hd]]
    const int wst = hd + 2;
#pragma unroll
    for (int h = 0; h < GM; ++h) {
        if (h >= G) continue;
        float* wp = kb + (warp * G + h) * wst;
        if (lane == 0) {
            wp[0] = m[h];
            wp[1] = ls[h];
        }
#pragma unroll
        for (int e = 0; e < E; ++e) wp[2 + lane * E + e] = o[h][e];
    }
    dk_bar();
    const int stride = hd + 4;
    #pragma unroll 1
    for (int idx = tid; idx < G * hd; idx += DK_CT) {
        const int h = idx / hd, i = idx - h * hd;
        float M = NEG;
#pragma unroll
        for (int w = 0; w < 8; ++w) M = fmaxf(M, kb[(w * G + h) * wst]);
        float L = 0.0f, O = 0.0f;
#pragma unroll
        for (int w = 0; w < 8; ++w) {
            const float* wp = kb + (w * G + h) * wst;
            if (wp[0] == NEG) continue;
            const float f = expf(wp[0] - M);
            L = fmaf(f, wp[1], L);
            O = fmaf(f, wp[2 + i], O);
        }
        float* dst = pbase + ((int64_t)h * nch + c) * stride;
        __stcg(&dst[4 + i], O);
        if (i == 0) {
            __stcg(&dst[0], M);
            __stcg(&dst[1], L);
        }
    }
}



__device__ void attn_phase(const DecodeParams& P, int l, float* sm, unsigned long long* t_wave,
                           unsigned long long* detail, uint32_t ep, bool& aborted) {
    const int G = P.n_heads / P.n_kv, hd = P.hd, half = hd / 2, hd4 = hd / 4;
    const int kvd = P.n_kv * hd, qw = P.n_heads * hd;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int table = (arch_gemma(P.arch) && !arch_global_layer(P.arch, l)) ? 1 : 0;   // local-layer base
    const bool inter = arch_interleaved(P.arch);
    const bool rope_on = arch_rope_layer(P.arch, l);
    const int nch = P.nchunk;
    const int SUB = P.attn_sub;
    const int stride = hd + 4;   // partial: m, l, 2 spare, o[hd]
    int tpp = 1;                 // lanes per (position, head) score (power of two <= 8)
    while (tpp < 8 && 2 * tpp * G * SUB <= DK_CT) tpp *= 2;
    // (pc * gmagic) >> 16 == pc / G for the pair indices pc < G * SUB (<= 256), G <= 8
    const int gmagic = (65536 + G - 1) / G;
    float* kb = sm;
    float* vb = kb + SUB * hd;
    float* qs = vb + SUB * hd;
    float* ks = qs + G * hd;
    float* vs = ks + hd;
    float* wq = vs + hd;
    float* wk = wq + hd;
    float* cs = wk + hd;   // RoPE cos / sin of this item's position (RopeCache.precomputeAngles rows)
    float* sn = cs + half;
    float* sc = sn + half;
    float* st = sc + G * SUB;
    __shared__ int s_all;   // every chunk of the item's (sequence, kv head) has arrived
    // detail trace (first item of the CTA): 0 start, 1 wave landed, 2 head
    // norm, 3 RoPE, 4 rounds done, 5 all chunks arrived, 6 the slice's
    // partials staged, 7 slice combined, 8 phase end
    unsigned long long* const det0 = detail;
    auto stamp = [&](int k) {
        if (detail && tid == 0) detail[k] = global_ns();
    };
    stamp(0);
    const int items = P.batch * P.n_kv * nch;
    // every item CTA waits for all chunks of its (sequence, kv head): one
    // item per CTA at most (decode_prepare sizes nchunk so), else stop
    if (items > (int)gridDim.x) {
        if (tid == 0 && blockIdx.x == 0) {
            atomicOr(P.err, BREW_DEVERR_BAD_INDEX);
            atomicExch(P.abort, 1);
        }
        aborted = true;
        return;
    }
    #pragma unroll 1
    for (int item = blockIdx.x; item < items; item += gridDim.x) {
        AttnItem it;
        if (!attn_item(P, l, item, it)) {   // a position outside the context: stop the step
            if (tid == 0) {
                atomicOr(P.err, BREW_DEVERR_BAD_INDEX);
                atomicExch(P.abort, 1);
            }
            aborted = true;
            continue;
        }
        const int c = it.c, hk = it.hk, b = it.b, pos = it.pos, used = it.used, p0 = it.p0, n = it.n;
        // partials alternate between two buffers by layer parity: layer l + 2's
        // items start only after every combine of layer l has produced its
        // output (their inputs depend on it), so no partial is overwritten
        // while it is read
        float* pbase = P.attn_part + (int64_t)(l & 1) * DK_MAX_BATCH * P.n_heads * nch * stride +
                       ((int64_t)b * P.n_heads + (int64_t)hk * G) * nch * stride;
        float* kc = P.kc + (int64_t)b * P.cache_bstride + (int64_t)l * P.seq_len * kvd;
        float* vc = P.vc + (int64_t)b * P.cache_bstride + (int64_t)l * P.seq_len * kvd;
        if (c < used) {
            const u64* qsrc = tgp(P, l, DK_TG_QKV) + (int64_t)b * P.tg_ls + (int64_t)hk * G * hd;
            const u64* ksrc = tgp(P, l, DK_TG_QKV) + (int64_t)b * P.tg_ls + qw + (int64_t)hk * hd;
            const u64* vsrc = ksrc + kvd;
            #pragma unroll 1
            for (int i = tid; i < hd4; i += DK_CT) {
                if (P.rms_q) {
                    cp_async16(wq + 4 * i, P.rms_q + (int64_t)l * hd + 4 * i);
                    cp_async16(wk + 4 * i, P.rms_k + (int64_t)l * hd + 4 * i);
                }
            }
            if (rope_on) {
                const int64_t ro = ((int64_t)table * P.seq_len + pos) * half;
                #pragma unroll 1
                for (int i = tid; i < half / 4; i += DK_CT) {
                    cp_async16(cs + 4 * i, P.rope_cos + ro + 4 * i);
                    cp_async16(sn + 4 * i, P.rope_sin + ro + 4 * i);
                }
            }
            cp_async_commit();                 // group: norm weights, RoPE row
            attn_issue_kv(P, l, it, 0, kb, vb);
            cp_async_commit();                 // group: the first round's cached K / V rows
            if (tid < G) {
                st[4 * tid + 0] = -INFINITY;
                st[4 * tid + 1] = 0.0f;
            }
            // this step's q heads, k and v (tagged words, written by the Q|K|V
            // phase): pairs [0, G hd / 2) of q, then hd / 2 of k and of v, into
            // qs | ks | vs (contiguous)
            {
                const int nq2 = G * hd / 2, h2 = hd / 2, np = nq2 + 2 * h2;
                auto pair = [&](int i) {
                    return i < nq2 ? qsrc + 2 * i : i < nq2 + h2 ? ksrc + 2 * (i - nq2) : vsrc + 2 * (i - nq2 - h2);
                };
                #pragma unroll 1
                for (int i0 = tid; i0 < np; i0 += 2 * DK_CT) {   // two pairs in flight per thread
                    const int i1 = i0 + DK_CT;
                    u64 a0, b0, a1 = 0, b1 = 0;
                    ld_tag2(pair(i0), a0, b0);
                    if (i1 < np) ld_tag2(pair(i1), a1, b1);
                    if (!(tag_is(a0, ep) && tag_is(b0, ep)) && !tag_wait2(P, pair(i0), ep, a0, b0)) aborted = true;
                    qs[2 * i0] = tag_val(a0);
                    qs[2 * i0 + 1] = tag_val(b0);
                    if (i1 < np) {
                        if (!(tag_is(a1, ep) && tag_is(b1, ep)) && !tag_wait2(P, pair(i1), ep, a1, b1)) aborted = true;
                        qs[2 * i1] = tag_val(a1);
                        qs[2 * i1 + 1] = tag_val(b1);
                    }
                }
            }
            cp_async_wait_group<1>();          // weights / RoPE landed; the K / V rows may still be in flight
            dk_bar();
            if (t_wave) *t_wave = global_ns();
            stamp(1);
            // one warp per vector (the G q heads, then k): head-wise RMSNorm
            // (Kernels.headWiseRmsNorm, Qwen3 / Gemma3) and RoPE in registers,
            // lane holding elements lane + 32 r; the k warp also appends this
            // step's k and v to the cache (storeKeyValueInCache,
            // AttentionEngine.java:34-38) and, when this position is in the
            // first round, writes them into that round's K / V rows
            const bool has_pos = pos >= p0 && pos < p0 + n;
            #pragma unroll 1
            for (int hh = warp; hh <= G; hh += DK_CW) {
                float* vecp = hh < G ? qs + hh * hd : ks;
                norm_rope_warp(vecp, hd, P.rms_q ? (hh < G ? wq : wk) : nullptr, P.eps, rope_on, inter, cs, sn);
                if (hh == G && has_pos) {
                    const int r = pos - p0;
                    float* kcr = kc + (int64_t)pos * kvd + hk * hd;
                    float* vcr = vc + (int64_t)pos * kvd + hk * hd;
                    #pragma unroll 1
                    for (int i = lane; i < hd; i += 32) {
                        const float kv = ks[i], vv = vs[i];
                        kcr[i] = kv;
                        vcr[i] = vv;
                        if (r < SUB) {
                            kb[r * hd + i] = kv;
                            vb[r * hd + i] = vv;
                        }
                    }
                }
            }
            stamp(2);
            cp_async_wait_group<0>();
            stamp(3);
            // warp-level rounds where q and the output of the kv head's
            // query heads fit 8 to 16 registers per lane; else the CTA-wide rounds
            if (DK_CW == 8 && hd == 128 && G <= 2) {
                attn_rounds_warp<4, 2, 6>(P, l, it, kb, vb, qs, ks, vs, pbase, nch, detail);
            } else if (DK_CW == 8 && hd == 64 && G <= 4) {
                attn_rounds_warp<2, 4, 6>(P, l, it, kb, vb, qs, ks, vs, pbase, nch, detail);
            } else if (DK_CW == 8 && hd == 256 && G <= 2) {
                attn_rounds_warp<8, 2, 2>(P, l, it, kb, vb, qs, ks, vs, pbase, nch, detail);
            } else {
                float acc[DK_PVK] = {};   // outputs tid + DK_CT k of [G][hd] (G * hd <= 1024)
                #pragma unroll 1
                for (int r0 = 0; r0 < n; r0 += SUB) {
                    const int ns = min(SUB, n - r0);
                    if (r0 > 0) {
                        attn_issue_kv(P, l, it, r0, kb, vb);
                        cp_async_wait_all();
                    }
                    if (r0 > 0 && has_pos && pos - p0 >= r0 && pos - p0 < r0 + ns) {
                        const int r = pos - p0 - r0;
                        #pragma unroll 1
                        for (int i = tid; i < hd; i += DK_CT) {
                            kb[r * hd + i] = ks[i];
                            vb[r * hd + i] = vs[i];
                        }
                    }
                    dk_bar();
                    if (r0 == 0) stamp(9);
                    // scores q.k / sqrt(hd): tpp lanes per (position, head) pair,
                    // each summing every tpp-th float4 of the row, then a shuffle
                    // sum over the pair's lanes.  Every lane runs the same number
                    // of iterations (the shuffles need the whole warp).
                    {
                        const int npair = G * ns, ppi = DK_CT / tpp;
                        const int j = tid & (tpp - 1);
                        #pragma unroll 1
                        for (int p00 = 0; p00 < npair; p00 += ppi) {
                            const int pr = p00 + tid / tpp;
                            const int pc = pr < npair ? pr : npair - 1;
                            const int tt = (pc * gmagic) >> 16, h = pc - tt * G;   // pc / G, pc % G
                            const float4* q4 = reinterpret_cast<const float4*>(qs + h * hd);
                            const float4* k4 = reinterpret_cast<const float4*>(kb + tt * hd);
                            float s0 = 0.0f, s1 = 0.0f;
                            #pragma unroll 1
                            for (int m = j; m < hd4; m += 2 * tpp) {
                                const float4 a = q4[m], kk = k4[m];
                                s0 = fmaf(a.x, kk.x, s0);
                                s0 = fmaf(a.y, kk.y, s0);
                                s0 = fmaf(a.z, kk.z, s0);
                                s0 = fmaf(a.w, kk.w, s0);
                                if (m + tpp < hd4) {
                                    const float4 a1 = q4[m + tpp], k1 = k4[m + tpp];
                                    s1 = fmaf(a1.x, k1.x, s1);
                                    s1 = fmaf(a1.y, k1.y, s1);
                                    s1 = fmaf(a1.z, k1.z, s1);
                                    s1 = fmaf(a1.w, k1.w, s1);
                                }
                            }
                            float sv = s0 + s1;
                            for (int o = tpp >> 1; o > 0; o >>= 1) sv += __shfl_xor_sync(0xffffffffu, sv, o);
                            if (j == 0 && pr < npair) sc[h * SUB + tt] = sv * P.inv_scale;
                        }
                    }
                    dk_bar();
                    if (r0 == 0) stamp(10);
                    // running softmax: weights of this round relative to the new maximum
                    #pragma unroll 1
                    for (int h = warp; h < G; h += DK_CW) {
                        float m = -INFINITY;
                        #pragma unroll 1
                        for (int tt = lane; tt < ns; tt += 32) m = fmaxf(m, sc[h * SUB + tt]);
                        m = warp_max(m);
                        const float mo = st[4 * h], mn = fmaxf(mo, m);
                        float ls = 0.0f;
                        #pragma unroll 1
                        for (int tt = lane; tt < ns; tt += 32) {
                            const float e = expf(sc[h * SUB + tt] - mn);
                            sc[h * SUB + tt] = e;
                            ls += e;
                        }
                        ls = warp_sum(ls);
                        __syncwarp();
                        if (lane == 0) {
                            const float corr = expf(mo - mn);
                            st[4 * h + 2] = corr;
                            st[4 * h + 0] = mn;
                            st[4 * h + 1] = st[4 * h + 1] * corr + ls;
                        }
                    }
                    dk_bar();
                    if (r0 == 0) stamp(11);
    #pragma unroll
                    for (int k = 0; k < DK_PVK; ++k) {
                        const int idx = tid + DK_CT * k;
                        if (idx < G * hd) {
                            const int h = idx / hd, i = idx % hd;
                            const float* sh = sc + h * SUB;
                            const float* vcol = vb + i;
                            float a0 = acc[k] * st[4 * h + 2], a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
                            int tt = 0;
                            #pragma unroll 1
                            for (; tt + 4 <= ns; tt += 4) {
                                a0 = fmaf(sh[tt], vcol[tt * hd], a0);
                                a1 = fmaf(sh[tt + 1], vcol[(tt + 1) * hd], a1);
                                a2 = fmaf(sh[tt + 2], vcol[(tt + 2) * hd], a2);
                                a3 = fmaf(sh[tt + 3], vcol[(tt + 3) * hd], a3);
                            }
                            #pragma unroll 1
                            for (; tt < ns; ++tt) a0 = fmaf(sh[tt], vcol[tt * hd], a0);
                            acc[k] = (a0 + a1) + (a2 + a3);
                        }
                    }
                    dk_bar();
                    if (r0 == 0) stamp(12);
                }
                stamp(4);
    #pragma unroll
                for (int k = 0; k < DK_PVK; ++k) {
                    const int idx = tid + DK_CT * k;
                    if (idx < G * hd) {
                        const int h = idx / hd, i = idx % hd;
                        __stcg(&pbase[((int64_t)h * nch + c) * stride + 4 + i], acc[k]);
                    }
                }
                if (tid < G) {
                    __stcg(&pbase[((int64_t)tid * nch + c) * stride + 0], st[4 * tid + 0]);
                    __stcg(&pbase[((int64_t)tid * nch + c) * stride + 1], st[4 * tid + 1]);
                }
            }
        }
        // Arrival, then every item CTA of (b, hk) combines its slice of the
        // G hd outputs (AttentionEngine.attend's softmax over all positions,
        // regrouped by chunk).  The counters of this launch are the set of
        // its epoch's parity (cleared by the previous launch), so all chunks
        // are in when the count reaches nch.  The barrier orders every
        // thread's partial stores before thread 0's release; the acquire
        // orders the other chunks' partials before the slice is read.
        dk_bar();
        int* ctr = &P.attn_ctr[(((int)(ep & 1u) * P.n_layers + l) * DK_MAX_BATCH + b) * P.n_kv + hk];
        if (tid == 0) {
            int prev;
            asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], 1;" : "=r"(prev) : "l"(ctr) : "memory");
            int ok = 1;
            if (prev + 1 < nch && !wait_int_bounded(ctr, nch, P.abort, 2000000000ull)) {
                atomicOr(P.err, BREW_DEVERR_TIMEOUT_FULL);
                atomicExch(P.abort, 1);
                ok = 0;
            }
            s_all = ok;
        }
        dk_bar();
        if (!s_all) aborted = true;
        stamp(5);
        {
            const int tot = G * hd, S = (tot + nch - 1) / nch;   // outputs per CTA
            const int o0 = c * S, o1 = min(tot, o0 + S);
            if (o0 < o1 && s_all) {
                const int lgh = 31 - __clz(hd);   // hd is a power of two
                const int h0 = o0 >> lgh, nh = ((o1 - 1) >> lgh) - h0 + 1;   // heads of the slice
                // stage the slice's heads: every used chunk's record [m, l, -, -, o[hd]]
                // (contiguous per head), then the weights and 1 / L per head
                float* srec = sm;                       // [nh][used][stride]
                float* swt = srec + nh * used * stride; // [nh][used], then [nh] 1 / L
                const int n4 = used * stride / 4;
                #pragma unroll 1
                for (int hh = 0; hh < nh; ++hh) {
                    const float* src = pbase + (int64_t)(h0 + hh) * nch * stride;
                    #pragma unroll 1
                    for (int j = tid; j < n4; j += DK_CT) cp_async16(srec + 4 * (hh * n4 + j), src + 4 * j);
                }
                cp_async_wait_all();
                dk_bar();
                stamp(6);
                // one warp per head of the slice: the largest running max, the
                // chunks' weights and 1 / L
                #pragma unroll 1
                for (int hh = warp; hh < nh; hh += DK_CW) {
                    const float* ph = srec + hh * used * stride;
                    float M = -INFINITY;
                    #pragma unroll 1
                    for (int k = lane; k < used; k += 32) M = fmaxf(M, ph[k * stride]);
                    M = warp_max(M);
                    float Ls = 0.0f;
                    #pragma unroll 1
                    for (int k = lane; k < used; k += 32) {
                        const float w = expf(ph[k * stride] - M);
                        swt[hh * used + k] = w;
                        Ls += w * ph[k * stride + 1];
                    }
                    Ls = warp_sum(Ls);
                    if (lane == 0) swt[nh * used + hh] = __frcp_rn(Ls);   // = 1.0f / Ls, correctly rounded
                }
                dk_bar();
                #pragma unroll 1
                for (int t = tid; t < o1 - o0; t += DK_CT) {
                    const int oi = o0 + t, hh = (oi >> lgh) - h0, i = oi & (hd - 1);
                    const float* ph = srec + hh * used * stride + 4 + i;
                    const float* wt = swt + hh * used;
                    // four independent partial sums over the chunks (k mod 4)
                    float o4[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                    int k = 0;
                    #pragma unroll 1
                    for (; k + 4 <= used; k += 4) {
#pragma unroll
                        for (int u = 0; u < 4; ++u) o4[u] += wt[k + u] * ph[(k + u) * stride];
                    }
                    #pragma unroll 1
                    for (; k < used; ++k) o4[0] += wt[k] * ph[k * stride];
                    const float o = (o4[0] + o4[1]) + (o4[2] + o4[3]);
                    st_tag(tgp(P, l, DK_TG_XB) + (int64_t)b * P.tg_ls + (int64_t)hk * G * hd + oi,
                           o * swt[nh * used + hh], ep);
                }
                stamp(7);
            }
        }
        dk_bar();
        detail = nullptr;   // stamps of the first item only
    }
    if (det0 && tid == 0) det0[8] = global_ns();
}

template <int TYPE, int CTYPE, int NT>
__global__ void __launch_bounds__(DK_CT + 32, 1) decode_kernel(const __grid_constant__ DecodeParams P) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int NS = P.nstages;
    Ring ring;
    ring.full = reinterpret_cast<uint64_t*>(smem);
    ring.empty = ring.full + NS;
    ring.ns = NS;
    ring.stage_bytes = P.stage_bytes;
    unsigned long long* s_best = reinterpret_cast<unsigned long long*>(smem + 512);   // [16]
    __shared__ int s_last;
    float* s_red = reinterpret_cast<float*>(smem + 640);                               // [32]
    float* red = reinterpret_cast<float*>(smem + 768);                                 // [DK_CW][DK_GMAX][16][2]
    float* vec = reinterpret_cast<float*>(smem + 768 + DK_RED_BYTES);
    vec = reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(vec) + 127) & ~uintptr_t(127));
    uint8_t* prep = reinterpret_cast<uint8_t*>(vec) + P.vec_bytes;
    ring.stages = prep + P.prep_bytes;
    ring.stages = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(ring.stages) + 127) & ~uintptr_t(127));
    const uint32_t prep_s = smem_u32(prep);

    const int tid = threadIdx.x, warp = tid >> 5;
    const int L = P.n_layers;
    if (tid == 0) {
        for (int s = 0; s < NS; ++s) {
            mbar_init(&ring.full[s], 1);
            mbar_init(&ring.empty[s], DK_CW);
        }
        fence_mbar_init();
        // this launch's epoch: one past the last completed launch's, never 0
        // (after 2^32 - 1 comes 2: the parity keeps alternating)
        const uint32_t e = *P.seq + 1u;
        s_ep = e ? e : 2u;
    }
    if (tid < 16) s_best[tid] = 0ull;
    if (blockIdx.x == 0) {   // the attention counters of the next launch's parity (the previous launch used them)
        const uint32_t e = *P.seq + 1u, par = (e ? e : 2u) & 1u;
        const int n = P.n_layers * DK_MAX_BATCH * P.n_kv;
        int* nxt = P.attn_ctr + (int)(par ^ 1u) * n;
        for (int i = tid; i < n; i += blockDim.x) nxt[i] = 0;
    }
    if (tid < DK_MAX_BATCH) s_pos[tid] = tid < P.batch ? (P.use_imm ? P.pos_imm : P.pos[tid]) : -1;
    if (tid < 5) {
        const int qw = P.n_heads * P.hd, kvd = P.n_kv * P.hd;
        const int tiles = tid == PH_QKV ? (qw + 2 * kvd) / 16
                          : tid == PH_O  ? P.dim / 16
                          : tid == PH_GU ? P.hidden / 8
                          : tid == PH_DOWN ? P.dim / 16
                                           : (P.vocab + 15) / 16;
        s_tiles[tid][0] = (int)((int64_t)blockIdx.x * tiles / gridDim.x);
        s_tiles[tid][1] = (int)((int64_t)(blockIdx.x + 1) * tiles / gridDim.x);
    }
    if (tid >= 8 && tid < 8 + 2 * DK_MAX_BATCH) attn_geometry(P, (tid - 8) >> 1, tid & 1, s_attg[(tid - 8) >> 1][tid & 1]);
    if (tid == 12) {
        const int item = blockIdx.x, nch = P.nchunk;
        s_item0[0] = item % nch;
        s_item0[1] = (item / nch) % P.n_kv;
        s_item0[2] = min(item / (nch * P.n_kv), DK_MAX_BATCH - 1);
    }
    __syncthreads();

    if (warp == DK_CW) {
        // ------------------------------- producer -------------------------------
        RingPos rp;
        unsigned long long* dtr =
            P.trace ? P.trace + (size_t)blockIdx.x * P.trace_slots + P.trace_slots - 3 * DK_DETAIL : nullptr;
        // the consumers' phase steps, without attention (no weights)
        for (int s = 0; s < 5 * L + 1 && rp.q < (1 << 29); ++s) {
            const int l = s / 5, ph = s - 5 * l;
            const bool cls = s == 5 * L;
            if (ph == 1) continue;
            const int mph = cls ? PH_CLS : ph == 0 ? PH_QKV : ph == 2 ? PH_O : ph == 3 ? PH_GU : PH_DOWN;
            const DPhase f = make_phase(P, l, mph);
            unsigned long long* d = (l == P.detail_l && mph == P.detail_ph) ? dtr : nullptr;
            if constexpr (TYPE == CTYPE) {
                produce_phase<TYPE>(P, f, ring, rp, d);
            } else {
                if (cls)
                    produce_phase<CTYPE>(P, f, ring, rp, d);
                else
                    produce_phase<TYPE>(P, f, ring, rp, d);
            }
        }
        return;
    }

    // --------------------------------- consumers ---------------------------------
    const uint32_t ep = s_ep;
    RingPos rp;
    bool aborted = false;
    const bool gem = arch_gemma(P.arch);
    constexpr bool lsum_l = TYPE == BREW_TYPE_Q4_0, lsum_c = CTYPE == BREW_TYPE_Q4_0;
    // trace (P.trace set): per CTA, slot 0 = start, then slots 1 + 5 s + k of
    // step s: k = 0 load wave landed, 1 prep done, 2 last weight stage in,
    // 3 work done, 4 phase end.  The wave / weight stamps pass through shared
    // memory, and every address is formed from P when it is used: tracing
    // holds no registers across the step loop.
    __shared__ unsigned long long s_tw[2];   // [0] wave landed, [1] last weight stage in
    auto stamp = [&](int st, int k, unsigned long long v) {
        if (P.trace && tid == 0) P.trace[(size_t)blockIdx.x * P.trace_slots + 1 + 5 * st + k] = v;
    };
    auto det = [&](int l, int ph) {
        return (P.trace && l == P.detail_l && ph == P.detail_ph)
                   ? P.trace + (size_t)blockIdx.x * P.trace_slots + P.trace_slots - 3 * DK_DETAIL
                   : nullptr;
    };
    if (P.trace && tid == 0) {
        P.trace[(size_t)blockIdx.x * P.trace_slots] = global_ns();
        s_tw[0] = s_tw[1] = 0ull;
    }
    // the end of a phase: a wait that gave up in any consumer thread stops the CTA
    auto phase_end = [&](int st) {
        stamp(st, 3, global_ns());
        aborted = dk_bar_or(aborted);
        stamp(st, 4, global_ns());
    };
    // The next phase's RMSNorm weight is copied into shared memory, beside
    // the input vector where prep_phase reads it, while this phase
    // multiplies (issued after this phase's prep, when `vec` is free again;
    // waited for by the next prep_phase).  Not for Gemma3, whose prep also
    // stages its post-norm weight there.
    auto stage_norm = [&](const float* nw) {
        if (!gem) stage_async(reinterpret_cast<float4*>(vec) + P.dim / 4, reinterpret_cast<const float4*>(nw), nullptr,
                              nullptr, P.dim / 4);
    };
    // One step per phase: s = 5 l + p, p = 0 Q|K|V, 1 attention, 2 wo,
    // 3 gate|up, 4 down; s = 5 L is the classifier.  Every phase function
    // has one call site (the kernel's code stays small: its instruction
    // fetches compete with the weight stream for L2).  A phase waits only for
    // its own inputs (tagged words), never for the whole grid.
    const int nsteps = 5 * L + 1;
    for (int s = 0; s < nsteps && !aborted; ++s) {
        const int l = s / 5, ph = s - 5 * l;
        const bool cls = s == 5 * L;
        if (ph == 0 && !cls && blockIdx.x == 0 && tid == 0) {
            // the head-norm weights go to L2 one phase ahead (HBM misses
            // otherwise; fetched earlier the weight stream would evict them)
            if (P.rms_q) prefetch_l2(P.rms_q + (int64_t)l * P.hd, (uint32_t)P.hd * 4u);
            if (P.rms_k) prefetch_l2(P.rms_k + (int64_t)l * P.hd, (uint32_t)P.hd * 4u);
        }
        if (ph == 1) {
            cp_async_wait_all();   // no staged norm weight may land in the attention area
            attn_phase(P, l, vec, P.trace ? &s_tw[0] : nullptr, det(l, PH_ATTN), ep, aborted);
            if (P.trace && tid == 0) {
                stamp(s, 0, s_tw[0]);   // the first load wave landed
                s_tw[0] = 0ull;
            }
            phase_end(s);
            continue;
        }
        // the phase's input vector -> prep records in shared memory
        //   non-Gemma: XIN(l) -> Q|K|V; XB -> wo (+ XIN) -> XMID -> gate|up ->
        //   HB -> down (+ XMID) -> XIN(l + 1)
        //   Gemma3:    XIN(l) = XMID(l - 1) + norm(XB2D(l - 1)) (QKV prep);
        //   wo -> XB2O; XMID(l) = XIN(l) + norm(XB2O) (gate|up prep); down -> XB2D
        int mode = SRC_PLAIN, K = P.dim, mph;
        const u64 *src = nullptr, *t = nullptr;
        const float *nw = nullptr, *tw = nullptr, *next_norm = nullptr;
        u64* xout = nullptr;
        bool staged = false;
        if (ph == 0) {   // RMSNorm + Q|K|V, or the final RMSNorm + classifier
            mph = cls ? PH_CLS : PH_QKV;
            nw = cls ? P.rms_final : P.rms_att + (int64_t)l * P.dim;
            if (l == 0) {
                mode = SRC_EMBED;
                xout = tgp(P, 0, DK_TG_XIN);
            } else if (gem) {   // the previous layer's post-FFN norm + residual
                mode = SRC_GEMMA_ADD;
                src = tgp(P, l - 1, DK_TG_XMID);
                t = tgp(P, l - 1, DK_TG_XB2D);
                tw = P.post_ffn + (int64_t)(l - 1) * P.dim;
                xout = cls ? nullptr : tgp(P, l, DK_TG_XIN);
            } else {
                src = tgp(P, l, DK_TG_XIN);
                staged = true;
            }
        } else if (ph == 2) {   // wo (+ residual)
            mph = PH_O;
            src = tgp(P, l, DK_TG_XB);
            K = P.n_heads * P.hd;
            next_norm = P.rms_ffn + (int64_t)l * P.dim;
        } else if (ph == 3) {   // RMSNorm (FFN) + gate|up
            mph = PH_GU;
            nw = P.rms_ffn + (int64_t)l * P.dim;
            if (gem) {   // post-attention norm + residual
                mode = SRC_GEMMA_ADD;
                src = tgp(P, l, DK_TG_XIN);
                t = tgp(P, l, DK_TG_XB2O);
                tw = P.post_att + (int64_t)l * P.dim;
                xout = tgp(P, l, DK_TG_XMID);
            } else {
                src = tgp(P, l, DK_TG_XMID);
                staged = true;
            }
        } else {   // down (+ residual)
            mph = PH_DOWN;
            src = tgp(P, l, DK_TG_HB);
            K = P.hidden;
            next_norm = l + 1 < L ? P.rms_att + (int64_t)(l + 1) * P.dim : P.rms_final;
        }
        // a CTA without tiles in this phase needs no input (unless it owns
        // blocks of the residual the prep writes)
        const bool need = s_tiles[mph][1] > s_tiles[mph][0] || (xout && (int)blockIdx.x < K / 32);
        if (need && !prep_phase(P, mode, src, K, nw, t, tw, xout, prep, vec, s_red, cls ? lsum_c : lsum_l,
                                P.trace ? &s_tw[0] : nullptr, staged, ep))
            aborted = true;
        if (next_norm) stage_norm(next_norm);
        if (P.trace && tid == 0) {   // the prep's load wave landed, then the prep is done
            stamp(s, 0, s_tw[0]);
            stamp(s, 1, global_ns());
            s_tw[0] = 0ull;
        }
        const DPhase f = make_phase(P, l, mph);
        if constexpr (TYPE == CTYPE) {
            mv_phase<TYPE, NT>(P, f, ring, rp, prep_s, red, s_best, aborted, P.trace ? &s_tw[1] : nullptr, det(l, mph), ep);
        } else {
            if (cls)
                mv_phase<CTYPE, NT>(P, f, ring, rp, prep_s, red, s_best, aborted, P.trace ? &s_tw[1] : nullptr, det(l, mph),
                                    ep);
            else
                mv_phase<TYPE, NT>(P, f, ring, rp, prep_s, red, s_best, aborted, P.trace ? &s_tw[1] : nullptr, det(l, mph),
                                   ep);
        }
        if (P.trace && tid == 0) {
            stamp(s, 2, s_tw[1]);
            s_tw[1] = 0ull;
        }
        if (cls) {
            dk_bar();
            if (tid < P.batch) atomicMax(&P.am_key[tid], s_best[tid]);
        }
        phase_end(s);
    }
    if (aborted) return;
    // the last CTA to finish writes the argmax and opens the next epoch; the
    // barrier orders the CTA's argmax updates before thread 0's release
    dk_bar();
    if (tid == 0) {
        int prev;
        asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], 1;" : "=r"(prev) : "l"(P.done) : "memory");
        s_last = prev == (int)gridDim.x - 1;
    }
    dk_bar();
    if (s_last) {
        if (tid < P.batch) {
            const unsigned long long k = atomicExch(&P.am_key[tid], 0ull);
            P.am_out[tid] = (int32_t)(0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull));
        }
        if (tid == 0) {
            *P.done = 0;
            *P.seq = ep;
            if (P.host_out) {   // id first, then the error word: the host waits on the latter
                P.host_out[0] = P.am_out[0];
                __threadfence_system();
                P.host_out[1] = (int32_t)*reinterpret_cast<volatile unsigned int*>(P.err);
            }
        }
    }
}

__global__ void rope_table_kernel(float* cos_t, float* sin_t, int seq_len, int hd, float base0, float base1,
                                  float scale) {
    // RopeCache.precomputeAngles (transformer/rope/RopeCache.java:15-26), per position
    const int half = hd / 2;
    const int64_t n = 2LL * seq_len * half;
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int tb = (int)(i / ((int64_t)seq_len * half));
    const int pos = (int)((i / half) % seq_len);
    const int p = (int)(i % half);
    const float base = tb == 0 ? base0 : base1;
    const float invf = (float)(1.0 / pow((double)base, (double)((float)(2 * p) / (float)hd)));
    const float ang = ((float)pos * scale) * invf;
    cos_t[i] = (float)cos((double)ang);
    sin_t[i] = (float)sin((double)ang);
}

template <int TYPE, int CTYPE, int NT>
int launch_decode(const DecodeParams& p, cudaStream_t stream) {
    // the attribute is per device; it is set to the whole budget, so every
    // model's size (p.smem <= DK_SMEM_BUDGET) is covered
    static unsigned long long attr_set = 0;   // one bit per device
    int dev = 0;
    BREW_CUDA(cudaGetDevice(&dev));
    if (dev >= 64 || !(attr_set >> dev & 1ull)) {
        BREW_CUDA(cudaFuncSetAttribute(decode_kernel<TYPE, CTYPE, NT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)DK_SMEM_BUDGET));
        if (dev < 64) attr_set |= 1ull << dev;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.grid);
    cfg.blockDim = dim3(DK_CT + 32);
    cfg.dynamicSmemBytes = p.smem;
    cfg.stream = stream;
    cudaLaunchAttribute a[1];
    a[0].id = cudaLaunchAttributeCooperative;
    a[0].val.cooperative = 1;
    cfg.attrs = a;
    cfg.numAttrs = 1;
    BREW_CUDA(cudaLaunchKernelEx(&cfg, decode_kernel<TYPE, CTYPE, NT>, p));
    count_launch();
    return BREW_OK;
}

}  // namespace

bool decode_supported(const brew_config& c, int batch) {
    if (batch < 1 || batch > DK_MAX_BATCH) return false;
    const int qw = c.n_heads * c.head_size;
    const int types[] = {c.type_q, c.type_k, c.type_v, c.type_o, c.type_gate, c.type_up, c.type_down};
    for (int t : types)
        if (t != c.type_q || (t != BREW_TYPE_Q8_0 && t != BREW_TYPE_Q4_0)) return false;
    const int tout = c.tied_embeddings ? c.type_embed : c.type_output;
    if (tout != BREW_TYPE_Q8_0 && tout != BREW_TYPE_Q4_0) return false;
    // whole 32-element blocks (a stage holds a divisor of a row's block count)
    if (c.dim % 32 || qw % 32 || c.hidden_dim % 32) return false;
    if ((c.n_kv_heads * c.head_size) % 16) return false;
    // attention: a CTA holds the G * hd outputs of a kv head's queries in
    // four registers per thread; 16-byte copies of half rows
    if ((c.n_heads / c.n_kv_heads) * c.head_size > 1024 || c.head_size % 8) return false;
    // 64, 128 or 256: shift-based indexing, two to eight registers per lane in norm_rope_warp
    if (c.head_size != 64 && c.head_size != 128 && c.head_size != 256) return false;
    // a prep's tagged input: at most 32 word pairs per consumer thread
    if (std::max(std::max(c.dim, qw), c.hidden_dim) > 64 * DK_CT) return false;
    return true;
}

int rope_tables_launch(float* cos_t, float* sin_t, int seq_len, int hd, float base0, float base1, float scale,
                       cudaStream_t stream) {
    const int64_t n = 2LL * seq_len * (hd / 2);
    rope_table_kernel<<<(unsigned)((n + 255) / 256), 256, 0, stream>>>(cos_t, sin_t, seq_len, hd, base0, base1, scale);
    BREW_CUDA(cudaGetLastError());
    count_launch();
    return BREW_OK;
}

int decode_prepare(DecodeParams* p) {
    const int qw = p->n_heads * p->hd;
    p->rec_bytes = prep_rec_bytes(p->batch);
    const int kmax = std::max(std::max(p->dim, qw), p->hidden);
    const int G = p->n_heads / p->n_kv;
    // attention area (vec and prep are contiguous): the item layout of
    // attn_phase, or one head's partials of all chunks for the combine
    const int SUB = attn_sub(p->hd);
    // the combine of a CTA's slice of the G hd outputs stages the chunk
    // records of the slice's heads (one or two) plus their weights
    size_t comb_fl = 0;
    {
        const int tot = G * p->hd, S = (tot + p->nchunk - 1) / p->nchunk;
        for (int c = 0; c < p->nchunk; ++c) {
            const int o0 = c * S, o1 = std::min(tot, o0 + S);
            if (o0 >= o1) break;
            const int nh = (o1 - 1) / p->hd - o0 / p->hd + 1;
            comb_fl = std::max(comb_fl, (size_t)nh * ((size_t)p->nchunk * (p->hd + 4) + p->nchunk) + nh);
        }
    }
    const size_t attn_fl = std::max((size_t)2 * SUB * p->hd + (size_t)G * p->hd + 5 * (size_t)p->hd +
                                        (size_t)G * SUB + 4 * (size_t)G + 64,
                                    comb_fl);
    // staged input vector and the norm weight beside it
    p->vec_bytes = (int)(((size_t)std::max(kmax, 2 * p->dim) * 4 + 127) & ~size_t(127));
    const size_t prep_need = (size_t)(kmax / 32) * p->rec_bytes;
    const size_t attn_need = attn_fl * 4 > (size_t)p->vec_bytes ? attn_fl * 4 - p->vec_bytes : 0;
    p->prep_bytes = (int)((std::max(prep_need, attn_need) + 127) & ~size_t(127));
    p->attn_floats = (p->vec_bytes + p->prep_bytes) / 4;
    // widen the K / V staging to what the area holds (one round per chunk
    // of up to attn_sub_max positions)
    {
        const size_t fixed_fl = (size_t)G * p->hd + 5 * (size_t)p->hd + 4 * (size_t)G + 64;
        const size_t fit = ((size_t)p->attn_floats - fixed_fl) / (2 * (size_t)p->hd + G);
        p->attn_sub = std::max(SUB, (int)std::min<size_t>(fit, (size_t)attn_sub_max(p->hd)));
    }

    p->stage_bytes = DK_STAGE_BYTES;
    const size_t fixed = 768 + (size_t)DK_RED_BYTES + 128 + p->vec_bytes + p->prep_bytes + 128;
    const size_t budget = DK_SMEM_BUDGET;
    BREW_CHECK(fixed + 2 * (size_t)p->stage_bytes <= budget, BREW_ERR_UNSUPPORTED, "decode kernel: shapes too large");
    p->nstages = (int)std::min<size_t>(32, (budget - fixed) / p->stage_bytes);
    p->smem = fixed + (size_t)p->nstages * p->stage_bytes;
    // stage geometry per phase: for a group of ng tiles the widest KC (a
    // multiple of 8 dividing KB) whose ng * KC blocks fit a stage; for a CTA
    // of nt tiles the group size (<= 8) whose stages carry the most bytes
    // (ties: the larger group, whose x operand is loaded once for more tiles)
    const int phase_kb[5] = {p->dim / 32, qw / 32, p->dim / 32, p->hidden / 32, p->dim / 32};
    for (int ph = 0; ph < 5; ++ph) {
        const int KB = phase_kb[ph];
        const int bs = pk_block_bytes(ph == PH_CLS ? p->type_out : p->type_layer);
        int kc[9] = {0};
        for (int ng = 1; ng <= 8; ++ng) {
            const int cap = std::min(KB, p->stage_bytes / (ng * bs));
            // a multiple of the consumer warp count when one fits (every warp
            // takes the same number of block columns), else of 8
            kc[ng] = 8;
            bool found = false;
            for (int c = (cap / DK_CW) * DK_CW; c >= DK_CW && !found; c -= DK_CW)
                if (KB % c == 0) {
                    kc[ng] = c;
                    found = true;
                }
            for (int c = (cap / 8) * 8; c >= 8 && !found; c -= 8)
                if (KB % c == 0) {
                    kc[ng] = c;
                    found = true;
                }
            for (int c = cap; c >= 1 && !found; --c)   // any divisor (rows of 36 blocks, ...)
                if (KB % c == 0) {
                    kc[ng] = c;
                    found = true;
                }
            BREW_CHECK(ng * kc[ng] * bs <= p->stage_bytes && kc[ng] < 32768, BREW_ERR_UNSUPPORTED,
                       "decode kernel: stage geometry");
            p->geo_kc[ph][ng] = (int16_t)kc[ng];
            p->geo_nch[ph][ng] = (int16_t)(KB / kc[ng]);
        }
        p->geo_kc[ph][0] = 8;
        p->geo_nch[ph][0] = (int16_t)(KB / 8);
        p->geo_gs[ph][0] = 1;
        for (int nt = 1; nt <= 9; ++nt) {
            int best = 1, fill = 0;
            for (int gs = DK_GMAX; gs >= 1; gs >>= 1)
                if (gs <= nt && gs * kc[gs] * bs > fill) {
                    fill = gs * kc[gs] * bs;
                    best = gs;
                }
            p->geo_gs[ph][nt] = (int8_t)best;
        }
    }
    int dev = 0, coop = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev);
    BREW_CHECK(coop, BREW_ERR_UNSUPPORTED, "decode kernel: cooperative launch unsupported");
    p->grid = num_sms();
    // the attention combine waits for all chunks of a kv head: one item per CTA
    BREW_CHECK((int64_t)p->batch * p->n_kv * p->nchunk <= p->grid, BREW_ERR_UNSUPPORTED, "decode kernel: %d attention items for %d CTAs", p->batch * p->n_kv * p->nchunk,
               p->grid);
    return BREW_OK;
}

int decode_launch(const DecodeParams& p, cudaStream_t stream) {
    const int tl = p.type_layer, to = p.type_out;
    if (tl == BREW_TYPE_Q8_0 && to == BREW_TYPE_Q8_0) return launch_decode<BREW_TYPE_Q8_0, BREW_TYPE_Q8_0, 1>(p, stream);
    if (tl == BREW_TYPE_Q4_0 && to == BREW_TYPE_Q8_0) return launch_decode<BREW_TYPE_Q4_0, BREW_TYPE_Q8_0, 1>(p, stream);
    if (tl == BREW_TYPE_Q8_0 && to == BREW_TYPE_Q4_0) return launch_decode<BREW_TYPE_Q8_0, BREW_TYPE_Q4_0, 1>(p, stream);
    return launch_decode<BREW_TYPE_Q4_0, BREW_TYPE_Q4_0, 1>(p, stream);
}

}  // namespace brew
