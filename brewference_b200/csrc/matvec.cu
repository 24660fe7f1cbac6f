// matvec.cu — y = W x for W in unchanged GGUF Q8_0 / Q4_0 blocks (sm_100a).
//
// Replaces Linear.matmul (transformer/math/Linear.java:40-99).  Design:
//   * Weights stay in their 34-byte (Q8_0) / 18-byte (Q4_0) blocks.  One
//     producer warp streams 16-row tiles, KC blocks at a time, from HBM into
//     a ring of shared-memory stages with cp.async.bulk (the TMA bulk-copy
//     engine; no multicast), each row copy rounded out to 16-byte bounds.
//   * The x side arrives as prep records (prep.cuh): per 32-block three
//     int8 limb columns per batch element.  One mma.sync m16n8k32 int8 MMA
//     then produces the exact integer block dot products of 16 rows x 8
//     columns; the fp32 epilogue multiplies by the block's fp16 weight scale
//     and the limb's scale and accumulates.  That is ~0.06 instructions per
//     weight byte, so the kernel is bound by HBM, not by issue.
//   * Work is split "stream-K": the grid is persistent (<= #SMs CTAs) and
//     each CTA takes an equal contiguous share of (tile, stage) units; tiles
//     cut between CTAs combine their partial sums in a fixed order, so the
//     result is deterministic.
//   * Fused epilogues: bias, residual add, SwiGLU/GeGLU (gate and up rows in
//     one tile), the next matvec's prep records, and a "last CTA" pass that
//     RMS-normalises the finished vector for the next layer or reduces the
//     classifier argmax.
//   * Programmatic dependent launch: weight copies are issued before
//     griddepcontrol.wait, so they overlap the previous kernel's tail.
#include "matvec.cuh"
#include "prep.cuh"

#include <algorithm>
#include <mutex>

namespace brew {

namespace {

// shared-memory loads by 32-bit shared-window address
__device__ __forceinline__ uint32_t lds32(uint32_t a) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ uint32_t lds16(uint32_t a) {
    uint16_t v;
    asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ float ldsf(uint32_t a) { return __uint_as_float(lds32(a)); }

// 4 bytes at a 2-byte aligned shared-memory address: two aligned words and a
// funnel shift (shift 0 or 16).
__device__ __forceinline__ uint32_t lds32_a2(uint32_t a) {
    const uint32_t b = a & ~3u;
    return __funnelshift_r(lds32(b), lds32(b + 4), (a & 3u) * 8u);
}

__device__ __forceinline__ void mma_s8s8(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%11,%12,%13};"
        : "=r"(c[0]), "=r"(c[1]), "=r"(c[2]), "=r"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0), "r"(0), "r"(0), "r"(0));
}

__device__ __forceinline__ void mma_u8s8(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%11,%12,%13};"
        : "=r"(c[0]), "=r"(c[1]), "=r"(c[2]), "=r"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0), "r"(0), "r"(0), "r"(0));
}

__device__ __forceinline__ void consumer_bar() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

// Global address of row r (0..15) of `tile`, or null past the matrix end.
__device__ __forceinline__ const uint8_t* tile_row_ptr(const MvParams& p, int tile, int r) {
    if (p.epi != MV_EPI_STORE) {
        const int local = (tile - p.seg[0].tile0) * 8 + (r & 7);
        if (local >= p.seg[0].rows) return nullptr;
        return p.seg[r >> 3].w + (int64_t)local * p.row_bytes;
    }
    int s = 0;
    if (p.nseg > 1 && tile >= p.seg[1].tile0) s = 1;
    if (p.nseg > 2 && tile >= p.seg[2].tile0) s = 2;
    const int local = (tile - p.seg[s].tile0) * MV_TILE_ROWS + r;
    if (local >= p.seg[s].rows) return nullptr;
    return p.seg[s].w + (int64_t)local * p.row_bytes;
}

__device__ __forceinline__ int cta_of_unit(int64_t x, int units, int grid) {
    return (int)(((x + 1) * (int64_t)grid - 1) / units);
}

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

struct ArgBest {
    float v;
    int i;
};

__device__ __forceinline__ void argbest_update(ArgBest& b, float v, int i) {
    if (v > b.v || (v == b.v && i < b.i)) { b.v = v; b.i = i; }
}

// Writes the final values of one tile (vals[16][batch] in shared memory).
__device__ void tile_epilogue(const MvParams& p, int tile, const float* vals, int ctid, ArgBest& best) {
    if (p.epi == MV_EPI_STORE) {
        int s = 0;
        if (p.nseg > 1 && tile >= p.seg[1].tile0) s = 1;
        if (p.nseg > 2 && tile >= p.seg[2].tile0) s = 2;
        const MvSeg& sg = p.seg[s];
        const int rb = (tile - sg.tile0) * MV_TILE_ROWS;
        for (int idx = ctid; idx < MV_TILE_ROWS * p.batch; idx += 256) {
            const int r = idx & 15, b = idx >> 4;
            const int row = rb + r;
            if (row >= sg.rows) continue;
            float v = vals[idx];
            if (sg.bias) v = v + sg.bias[row];
            if (sg.resid) v = sg.resid[(int64_t)b * p.ldy + row] + v;
            sg.y[(int64_t)b * p.ldy + row] = v;
            if (p.post == MV_POST_ARGMAX) argbest_update(best, v, row);
        }
    } else {
        const int i0 = (tile - p.seg[0].tile0) * 8;
        for (int idx = ctid; idx < 8 * p.batch; idx += 256) {
            const int r = idx & 7, b = idx >> 3;
            const int i = i0 + r;
            if (i >= p.seg[0].rows) continue;
            const float g = vals[b * 16 + r], u = vals[b * 16 + 8 + r];
            p.seg[0].y[(int64_t)b * p.ldy + i] = act_glu(g, p.epi) * u;
        }
        if (p.next_prep) {
            // when all four tiles of a 32-wide group are written, emit the
            // group's prep record for the next matvec
            __shared__ int s_last;
            __threadfence();
            consumer_bar();
            const int group = i0 >> 5;
            if (ctid == 0) {
                const int old = atomicAdd(&p.group_counters[group], 1);
                s_last = (old == 3);
            }
            consumer_bar();
            if (s_last) {
                __threadfence();
                const int warp = ctid >> 5, lane = ctid & 31;
                const int ncol = 3 * p.batch;
                for (int b = warp; b < p.batch; b += MV_CONSUMER_WARPS) {
                    const float v = __ldcg(&p.seg[0].y[(int64_t)b * p.ldy + group * 32 + lane]);
                    prep_emit_warp(p.next_prep + (size_t)group * p.rec_bytes, ncol, b, v);
                }
                if (ctid == 0) p.group_counters[group] = 0;
            }
        }
    }
}

template <int TYPE, int NT>
__global__ void __launch_bounds__(MV_THREADS, 1) mv_kernel(const __grid_constant__ MvParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr int NTC = NT * 8;
    constexpr int BB = TYPE == BREW_TYPE_Q8_0 ? 34 : 18;
    const int NS = p.nstages;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);
    uint64_t* empty = full + NS;
    float* red = reinterpret_cast<float*>(smem + 256);               // [16][NTC]
    float* vals = red + 16 * NTC;                                      // [16*batch]
    uint8_t* stages = smem + 256 + (16 * NTC + 16 * MV_MAX_BATCH) * 4;
    stages = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(stages) + 127) & ~uintptr_t(127));

    const int tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    const int G = gridDim.x;
    const int u0 = (int)((int64_t)blockIdx.x * p.units / G);
    const int u1 = (int)((int64_t)(blockIdx.x + 1) * p.units / G);
    const int CB = p.KC * BB;
    const int stage_w = MV_TILE_ROWS * p.slot_pitch;
    const int prep_bytes = p.KC * p.rec_bytes;

    if (tid == 0) {
        for (int s = 0; s < NS; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], MV_CONSUMER_WARPS);
        }
        fence_mbar_init();
    }
    for (int i = tid; i < 16 * NTC; i += blockDim.x) red[i] = 0.0f;
    __syncthreads();

    if (warp == MV_CONSUMER_WARPS) {
        // ------------------------------ producer ------------------------------
        auto issue_weights = [&](int q) {
            const int u = u0 + q;
            const int stage = q % NS;
            const int tile = u / p.nchunks, chunk = u % p.nchunks;
            uint8_t* sbase = stages + (size_t)stage * p.stage_bytes;
            uint32_t len = 0;
            const uint8_t* src = nullptr;
            uint32_t lead = 0;
            if (lane < MV_TILE_ROWS) {
                const uint8_t* rp = tile_row_ptr(p, tile, lane);
                if (rp) {
                    src = rp + (int64_t)chunk * CB;
                    lead = (uint32_t)(reinterpret_cast<uintptr_t>(src) & 15u);
                    len = (lead + CB + 15u) & ~15u;
                }
            }
            uint32_t total = len;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) total += __shfl_xor_sync(0xffffffffu, total, o);
            if (lane == 0) mbar_arrive_expect_tx(&full[stage], total + prep_bytes);
            __syncwarp();
            if (len) bulk_g2s(sbase + lane * p.slot_pitch, src - lead, len, &full[stage]);
        };
        auto issue_prep = [&](int q) {
            if (lane == 0) {
                const int u = u0 + q;
                const int chunk = u % p.nchunks;
                uint8_t* sbase = stages + (size_t)(q % NS) * p.stage_bytes;
                bulk_g2s(sbase + stage_w, p.prep + (size_t)chunk * p.KC * p.rec_bytes, prep_bytes,
                         &full[q % NS]);
            }
        };
        const int nq = u1 - u0;
        const int pre = nq < NS ? nq : NS;
        for (int q = 0; q < pre; ++q) issue_weights(q);
        pdl_launch_dependents();
        pdl_wait();
        for (int q = 0; q < pre; ++q) issue_prep(q);
        for (int q = NS; q < nq; ++q) {
            const int stage = q % NS;
            const uint32_t parity = ((q / NS) - 1) & 1;
            if (!mbar_wait_bounded(&empty[stage], parity, p.err, BREW_DEVERR_TIMEOUT_EMPTY)) break;
            issue_weights(q);
            issue_prep(q);
        }
    } else {
        // ------------------------------ consumers -----------------------------
        pdl_launch_dependents();
        pdl_wait();
        const int g = lane >> 2, t = lane & 3;
        const int ctid = tid;  // 0..255
        const int ncol = 3 * p.batch;
        float acc[NT][4];
#pragma unroll
        for (int n = 0; n < NT; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.0f;
        ArgBest best{-INFINITY, 0x7fffffff};
        bool aborted = false;

        int q = 0;
        for (int u = u0; u < u1; ++u, ++q) {
            const int stage = q % NS;
            const uint32_t parity = (q / NS) & 1;
            const int tile = u / p.nchunks, chunk = u % p.nchunks;
            if (!aborted && !mbar_wait_bounded(&full[stage], parity, p.err, BREW_DEVERR_TIMEOUT_FULL)) aborted = true;
            const uint8_t* sbase = stages + (size_t)stage * p.stage_bytes;
            const uint8_t* sprep = sbase + stage_w;
            // rows g and g+8 of this tile: where their chunk starts in smem
            const uint8_t* rp0 = tile_row_ptr(p, tile, g);
            const uint8_t* rp1 = tile_row_ptr(p, tile, g + 8);
            const uint32_t lead0 = rp0 ? (uint32_t)((reinterpret_cast<uintptr_t>(rp0) + (int64_t)chunk * CB) & 15u) : 0u;
            const uint32_t lead1 = rp1 ? (uint32_t)((reinterpret_cast<uintptr_t>(rp1) + (int64_t)chunk * CB) & 15u) : 0u;
            const uint32_t row0 = smem_u32(sbase) + g * p.slot_pitch + lead0;
            const uint32_t row1 = smem_u32(sbase) + (g + 8) * p.slot_pitch + lead1;
            const uint32_t prep0 = smem_u32(sprep);
            if (!aborted) {
#pragma unroll 2
                for (int j = warp; j < p.KC; j += MV_CONSUMER_WARPS) {
                    const uint32_t b0p = row0 + j * BB;
                    const uint32_t b1p = row1 + j * BB;
                    uint32_t a0, a1, a2, a3;
                    if (TYPE == BREW_TYPE_Q8_0) {
                        a0 = lds32_a2(b0p + 2 + 4 * t);
                        a1 = lds32_a2(b1p + 2 + 4 * t);
                        a2 = lds32_a2(b0p + 18 + 4 * t);
                        a3 = lds32_a2(b1p + 18 + 4 * t);
                    } else {
                        const uint32_t w0 = lds32_a2(b0p + 2 + 4 * t);
                        const uint32_t w1 = lds32_a2(b1p + 2 + 4 * t);
                        a0 = w0 & 0x0F0F0F0Fu;
                        a1 = w1 & 0x0F0F0F0Fu;
                        a2 = (w0 >> 4) & 0x0F0F0F0Fu;
                        a3 = (w1 >> 4) & 0x0F0F0F0Fu;
                    }
                    const float d0 = half_bits_to_float((uint16_t)lds16(b0p));
                    const float d1 = half_bits_to_float((uint16_t)lds16(b1p));
                    const uint32_t rec = prep0 + j * p.rec_bytes;
                    const uint32_t sw = rec + ncol * 32;
                    const uint32_t ls = rec + ncol * 36;
#pragma unroll
                    for (int n = 0; n < NT; ++n) {
                        // columns past 3*batch are not stored: feed zeros
                        // (indices are clamped so no load leaves the record)
                        const int cb = n * 8 + g;
                        const bool vb = cb < ncol;
                        const int cbs = vb ? cb : 0;
                        uint32_t bf0 = lds32(rec + cbs * 32 + 4 * t);
                        uint32_t bf1 = lds32(rec + cbs * 32 + 16 + 4 * t);
                        if (!vb) bf0 = bf1 = 0u;
                        const int c0 = n * 8 + 2 * t, c1 = c0 + 1;
                        const bool v0 = c0 < ncol, v1 = c1 < ncol;
                        const int c0s = v0 ? c0 : 0, c1s = v1 ? c1 : 0;
                        int c[4];
                        if (TYPE == BREW_TYPE_Q8_0) {
                            mma_s8s8(c, a0, a1, a2, a3, bf0, bf1);
                        } else {
                            mma_u8s8(c, a0, a1, a2, a3, bf0, bf1);
                            const int l0 = v0 ? (int)lds32(ls + 4 * c0s) : 0;
                            const int l1 = v1 ? (int)lds32(ls + 4 * c1s) : 0;
                            c[0] -= 8 * l0;
                            c[1] -= 8 * l1;
                            c[2] -= 8 * l0;
                            c[3] -= 8 * l1;
                        }
                        const float s0 = v0 ? ldsf(sw + 4 * c0s) : 0.0f;
                        const float s1 = v1 ? ldsf(sw + 4 * c1s) : 0.0f;
                        acc[n][0] = fmaf((float)c[0], d0 * s0, acc[n][0]);
                        acc[n][1] = fmaf((float)c[1], d0 * s1, acc[n][1]);
                        acc[n][2] = fmaf((float)c[2], d1 * s0, acc[n][2]);
                        acc[n][3] = fmaf((float)c[3], d1 * s1, acc[n][3]);
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[stage]);

            const bool tile_end = (chunk == p.nchunks - 1) || (u == u1 - 1);
            if (!tile_end) continue;

            // ---- this CTA's share of the tile is done: reduce ----
#pragma unroll
            for (int n = 0; n < NT; ++n) {
                atomicAdd(&red[g * NTC + n * 8 + 2 * t], acc[n][0]);
                atomicAdd(&red[g * NTC + n * 8 + 2 * t + 1], acc[n][1]);
                atomicAdd(&red[(g + 8) * NTC + n * 8 + 2 * t], acc[n][2]);
                atomicAdd(&red[(g + 8) * NTC + n * 8 + 2 * t + 1], acc[n][3]);
                acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.0f;
            }
            consumer_bar();
            for (int idx = ctid; idx < 16 * p.batch; idx += 256) {
                const int r = idx & 15, b = idx >> 4;
                float* rr = red + r * NTC + 3 * b;
                vals[idx] = (rr[2] + rr[1]) + rr[0];
                rr[0] = rr[1] = rr[2] = 0.0f;
            }
            const int64_t t0 = (int64_t)tile * p.nchunks;
            const int first_cta = cta_of_unit(t0, p.units, G);
            const int last_cta = cta_of_unit(t0 + p.nchunks - 1, p.units, G);
            if (first_cta == last_cta) {
                consumer_bar();
                tile_epilogue(p, tile, vals, ctid, best);
            } else {
                // partial tile: publish, the last arriving CTA combines in order
                __shared__ int s_last;
                // a split tile is identified by its first CTA: CTA ranges are
                // contiguous, so no two split tiles share a first CTA
                const int part = blockIdx.x - first_cta;
                const int nparts = last_cta - first_cta + 1;
                if (nparts > MV_MAX_PARTS) {   // the host sizes the grid so this cannot happen
                    if (ctid == 0) atomicOr(p.err, BREW_DEVERR_BAD_INDEX);
                    consumer_bar();
                    continue;
                }
                float* pb = p.part_buf + ((size_t)first_cta * MV_MAX_PARTS) * 16 * p.batch;
                for (int idx = ctid; idx < 16 * p.batch; idx += 256) __stcg(&pb[part * 16 * p.batch + idx], vals[idx]);
                __threadfence();
                consumer_bar();
                if (ctid == 0) {
                    const int old = atomicAdd(&p.tile_counters[first_cta], 1);
                    s_last = (old == nparts - 1);
                }
                consumer_bar();
                if (s_last) {
                    __threadfence();
                    for (int idx = ctid; idx < 16 * p.batch; idx += 256) {
                        float v = __ldcg(&pb[idx]);
                        for (int k = 1; k < nparts; ++k) v += __ldcg(&pb[k * 16 * p.batch + idx]);
                        vals[idx] = v;
                    }
                    consumer_bar();
                    tile_epilogue(p, tile, vals, ctid, best);
                    if (ctid == 0) p.tile_counters[first_cta] = 0;
                }
            }
            consumer_bar();
        }

        if (p.post == MV_POST_ARGMAX) {
            // per-CTA best per batch element: threads 16b..16b+15 hold batch b
            ArgBest bb = best;
#pragma unroll
            for (int o = 8; o > 0; o >>= 1) {
                const float ov = __shfl_xor_sync(0xffffffffu, bb.v, o);
                const int oi = __shfl_xor_sync(0xffffffffu, bb.i, o);
                argbest_update(bb, ov, oi);
            }
            const int b = ctid >> 4;
            if ((ctid & 15) == 0 && b < p.batch) {
                p.am_val[blockIdx.x * p.batch + b] = bb.v;
                p.am_idx[blockIdx.x * p.batch + b] = bb.i;
            }
        }
    }

    // ------------------------------ post pass --------------------------------
    if (p.post == MV_POST_NONE) return;
    __shared__ int s_post_last;
    __shared__ float s_red[32];
    __threadfence();
    __syncthreads();
    if (tid == 0) {
        const int old = atomicAdd(p.post_counter, 1);
        s_post_last = (old == G - 1);
    }
    __syncthreads();
    if (!s_post_last) return;
    __threadfence();
    if (p.post == MV_POST_ARGMAX) {
        if (tid < 32) {
            for (int b = 0; b < p.batch; ++b) {
                ArgBest bb{-INFINITY, 0x7fffffff};
                for (int c = tid; c < G; c += 32) argbest_update(bb, __ldcg(&p.am_val[c * p.batch + b]), __ldcg(&p.am_idx[c * p.batch + b]));
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) {
                    const float ov = __shfl_xor_sync(0xffffffffu, bb.v, o);
                    const int oi = __shfl_xor_sync(0xffffffffu, bb.i, o);
                    argbest_update(bb, ov, oi);
                }
                if (tid == 0) p.am_out[b] = bb.i == 0x7fffffff ? 0 : bb.i;
            }
        }
    } else {
        const int ncol = 3 * p.batch;
        for (int b = 0; b < p.batch; ++b) {
            float* x = p.post_x + (int64_t)b * p.post_ld;
            if (p.post_add) {
                // Gemma3 post-norm: x += rmsnorm(t, w)  (Gemma3Transformer.java:62-65,81-84)
                const float* tv = p.post_add + (int64_t)b * p.ldy;
                float ss = 0.0f;
                for (int i = tid; i < p.post_dim; i += blockDim.x) {
                    const float v = __ldcg(&tv[i]);
                    ss += v * v;
                }
                ss = block_sum(ss, s_red);
                const float sc = rms_scale(ss, p.post_dim, p.eps);
                for (int i = tid; i < p.post_dim; i += blockDim.x)
                    __stcg(&x[i], __ldcg(&x[i]) + __ldcg(&tv[i]) * sc * p.post_add_w[i]);
                __threadfence();
                __syncthreads();
            }
            prep_vector_cta(x, p.post_dim, p.post_norm_w, p.eps, p.post_prep, p.rec_bytes, ncol, b, s_red);
        }
    }
    __syncthreads();
    if (tid == 0) *p.post_counter = 0;
}

__global__ void __launch_bounds__(256) prep_kernel(const float* x, int ldx, int K, int batch, const float* nw, float eps,
                                                    uint8_t* recs) {
    __shared__ float red[32];
    pdl_launch_dependents();
    pdl_wait();
    const int b = blockIdx.y;
    const int ncol = 3 * batch;
    const int rec_bytes = prep_rec_bytes(batch);
    const float* xb = x + (int64_t)b * ldx;
    float scale = 1.0f;
    if (nw) {
        float ss = 0.0f;
        for (int i = threadIdx.x; i < K; i += blockDim.x) {
            const float v = __ldcg(&xb[i]);
            ss += v * v;
        }
        ss = block_sum(ss, red);
        scale = rms_scale(ss, K, eps);
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nwarp = blockDim.x >> 5;
    for (int j = blockIdx.x * nwarp + warp; j < K / 32; j += gridDim.x * nwarp) {
        float v = __ldcg(&xb[32 * j + lane]);
        if (nw) v = v * scale * nw[32 * j + lane];
        prep_emit_warp(recs + (size_t)j * rec_bytes, ncol, b, v);
    }
}

template <int TYPE, int NT>
int launch_typed(const MvParams& p, cudaStream_t stream, bool pdl, int grid, size_t smem) {
    static std::once_flag once;
    static cudaError_t attr_err = cudaSuccess;
    std::call_once(once, [] {
        attr_err = cudaFuncSetAttribute(mv_kernel<TYPE, NT>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    });
    BREW_CUDA(attr_err);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(MV_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    BREW_CUDA(cudaLaunchKernelEx(&cfg, mv_kernel<TYPE, NT>, p));
    count_launch();
    return BREW_OK;
}

template <int TYPE>
int launch_nt(const MvParams& p, cudaStream_t stream, bool pdl, int grid, size_t smem) {
    switch (prep_nt(p.batch)) {
        case 1: return launch_typed<TYPE, 1>(p, stream, pdl, grid, smem);
        case 2: return launch_typed<TYPE, 2>(p, stream, pdl, grid, smem);
        case 3: return launch_typed<TYPE, 3>(p, stream, pdl, grid, smem);
        case 4: case 5: case 6: return launch_typed<TYPE, 6>(p, stream, pdl, grid, smem);
        default: return launch_typed<TYPE, 12>(p, stream, pdl, grid, smem);
    }
}

// Largest number of CTAs that share one tile for a given grid (stream-K).
int max_parts(int units, int nchunks, int grid) {
    int worst = 1;
    for (int c = 0; c < grid; ++c) {
        // the tile containing this CTA's first unit, and the CTAs covering it
        const int64_t u0 = (int64_t)c * units / grid;
        const int64_t t0 = u0 / nchunks * nchunks;
        const int64_t first = ((t0 + 1) * grid - 1) / units;
        const int64_t last = ((t0 + nchunks) * grid - 1) / units;
        worst = std::max(worst, (int)(last - first + 1));
    }
    return worst;
}

}  // namespace

int num_sms() {
    static int n = 0;
    if (n == 0) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (n <= 0) n = 148;
    }
    return n;
}

size_t mv_part_floats(int grid, int batch) {
    return (size_t)grid * MV_MAX_PARTS * 16 * (size_t)batch;
}

int mv_launch(MvParams p, cudaStream_t stream, bool pdl) {
    TypeInfo ti;
    BREW_CHECK(type_info(p.type, &ti), BREW_ERR_UNSUPPORTED, "matvec: unsupported type %d", p.type);
    BREW_CHECK(p.type == BREW_TYPE_Q8_0 || p.type == BREW_TYPE_Q4_0, BREW_ERR_UNSUPPORTED,
               "matvec: type %d is not handled by the int8 MMA matvec", p.type);
    BREW_CHECK(p.K > 0 && p.K % 32 == 0, BREW_ERR_INVALID_ARG, "matvec: K=%d is not a multiple of 32", p.K);
    BREW_CHECK(p.batch >= 1 && p.batch <= MV_MAX_BATCH, BREW_ERR_INVALID_ARG, "matvec: batch %d", p.batch);
    BREW_CHECK(p.post != MV_POST_ARGMAX || p.batch <= MV_ARGMAX_MAX_BATCH, BREW_ERR_INVALID_ARG,
               "matvec: fused argmax needs batch <= %d", MV_ARGMAX_MAX_BATCH);
    p.KB = p.K / 32;
    p.rec_bytes = prep_rec_bytes(p.batch);
    // stage = 16 rows x KC blocks (+ their prep records); KC divides KB
    const int BB = ti.block_bytes;
    int KC = 1;
    for (int c = 1; c <= p.KB; ++c) {
        if (p.KB % c) continue;
        const int cb = c * BB;
        const int slot = (cb + 47) & ~15;
        const int st = MV_TILE_ROWS * slot + c * p.rec_bytes;
        if (cb <= 1184 && st <= 40 * 1024) KC = c;
    }
    p.KC = KC;
    p.nchunks = p.KB / KC;
    p.slot_pitch = (KC * BB + 47) & ~15;
    p.stage_bytes = MV_TILE_ROWS * p.slot_pitch + KC * p.rec_bytes;
    const int NTC = prep_nt(p.batch) * 8;
    const size_t fixed = 256 + (size_t)(16 * NTC + 16 * MV_MAX_BATCH) * 4 + 128;
    const size_t budget = 112 * 1024;
    int ns = (int)((budget - fixed) / p.stage_bytes);
    ns = std::max(2, std::min(ns, 8));
    p.nstages = ns;
    const size_t smem = fixed + (size_t)ns * p.stage_bytes;
    // tiles per segment
    int tiles = 0;
    for (int s = 0; s < p.nseg; ++s) {
        p.seg[s].tile0 = tiles;
        if (p.epi == MV_EPI_STORE) tiles += (p.seg[s].rows + MV_TILE_ROWS - 1) / MV_TILE_ROWS;
    }
    if (p.epi != MV_EPI_STORE) {
        BREW_CHECK(p.nseg == 2 && p.seg[0].rows == p.seg[1].rows, BREW_ERR_INVALID_ARG, "matvec: GLU needs 2 equal segments");
        p.seg[1].tile0 = 0;
        tiles = (p.seg[0].rows + 7) / 8;
        BREW_CHECK(!p.next_prep || p.seg[0].rows % 32 == 0, BREW_ERR_INVALID_ARG, "matvec: GLU prep needs rows %% 32 == 0");
    }
    p.total_tiles = tiles;
    p.units = tiles * p.nchunks;
    // grid: persistent, at most one CTA per SM, and no tile split more than
    // MV_MAX_PARTS ways
    int grid = std::min(num_sms(), p.units);
    grid = std::min(grid, std::max(1, (MV_MAX_PARTS - 1) * p.units / p.nchunks));
    grid = std::max(grid, 1);
    while (grid > 1 && max_parts(p.units, p.nchunks, grid) > MV_MAX_PARTS) --grid;
    if (p.post == MV_POST_ARGMAX) BREW_CHECK(p.am_val && p.am_idx && p.am_out, BREW_ERR_INVALID_ARG, "argmax buffers");
    if (p.type == BREW_TYPE_Q8_0) return launch_nt<BREW_TYPE_Q8_0>(p, stream, pdl, grid, smem);
    return launch_nt<BREW_TYPE_Q4_0>(p, stream, pdl, grid, smem);
}

int prep_launch(const float* x, int ldx, int K, int batch, const float* norm_w, float eps, uint8_t* recs,
                cudaStream_t stream, bool pdl) {
    BREW_CHECK(K % 32 == 0, BREW_ERR_INVALID_ARG, "prep: K=%d not a multiple of 32", K);
    cudaLaunchConfig_t cfg = {};
    const int blocks_x = norm_w ? 1 : std::max(1, std::min(64, K / 32 / 8));
    cfg.gridDim = dim3(blocks_x, batch);
    cfg.blockDim = dim3(256);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    BREW_CUDA(cudaLaunchKernelEx(&cfg, prep_kernel, x, ldx, K, batch, norm_w, eps, recs));
    count_launch();
    return BREW_OK;
}

}  // namespace brew
