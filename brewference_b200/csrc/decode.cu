// decode.cu — one decode step (TransformerGraph.forward + argmax) of the whole
// model as ONE persistent kernel on all SMs.
//
// Why: at batch 1 the step streams every weight byte once (1.83 GB for the
// Qwen3-1.7B shape) and the per-layer dependency chain (norm -> QKV ->
// attention -> wo -> norm -> gate/up -> down) is long.  As separate kernels
// each link pays a launch/ramp/drain gap and the HBM idles in between.  Here:
//   * one CTA per SM (cooperative launch); warp 8 of every CTA is a producer
//     that streams the CTA's share of EVERY phase's weight tiles (TMA boxes of
//     16 rows x 8 blocks through per-family tensor maps, no multicast) into a
//     ring of shared-memory stages, running ahead across phase boundaries;
//   * warps 0-7 consume: each phase starts by building its own prep records
//     (RMSNorm + limb split of the input vector, prep.cuh) in shared memory,
//     then multiplies the staged tiles (int8 MMA, mv_device.cuh) and writes
//     its output rows;
//   * phases are separated by a grid barrier among the consumer warps
//     (acquire/release counter in global memory, bounded wait);
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

enum { PH_QKV = 0, PH_O, PH_GU, PH_DOWN, PH_CLS };

constexpr int ATTN_MIN_POS = 32;   // positions per attention CTA at least

struct DSeg {
    int rows, tile0, map, yoff;
    float* y;
    const float* bias;
    const float* resid;
};

struct DPhase {
    int K, KB, tiles, nseg, epi, ldy, tt;
    bool argmax;
    DSeg s[3];
};

__device__ __forceinline__ DPhase make_phase(const DecodeParams& P, int l, int ph, float* xcur) {
    DPhase f = {};
    const int qw = P.n_heads * P.hd, kvd = P.n_kv * P.hd;
    const bool gem = P.arch == BREW_ARCH_GEMMA3;
    f.epi = MV_EPI_STORE;
    f.tt = P.type_layer;
    switch (ph) {
        case PH_QKV:
            f.K = P.dim;
            f.nseg = 3;
            f.ldy = qw + 2 * kvd;
            f.s[0] = {qw, 0, DK_MAP_Q, l * qw, P.qkv, P.q_bias ? P.q_bias + (int64_t)l * qw : nullptr, nullptr};
            f.s[1] = {kvd, qw / 16, DK_MAP_K, l * kvd, P.qkv + qw, P.k_bias ? P.k_bias + (int64_t)l * kvd : nullptr, nullptr};
            f.s[2] = {kvd, qw / 16 + kvd / 16, DK_MAP_V, l * kvd, P.qkv + qw + kvd,
                      P.v_bias ? P.v_bias + (int64_t)l * kvd : nullptr, nullptr};
            f.tiles = qw / 16 + 2 * (kvd / 16);
            break;
        case PH_O:
            f.K = qw;
            f.nseg = 1;
            f.ldy = P.dim;
            f.s[0] = {P.dim, 0, DK_MAP_O, l * P.dim, gem ? P.xb2 : xcur, nullptr, gem ? nullptr : xcur};
            f.tiles = P.dim / 16;
            break;
        case PH_GU:
            f.K = P.dim;
            f.nseg = 2;
            f.epi = gem ? MV_EPI_GLU_GELU : MV_EPI_GLU_SILU;
            f.ldy = P.hidden;
            f.s[0] = {P.hidden, 0, DK_MAP_GATE, l * P.hidden, P.hb, nullptr, nullptr};
            f.s[1] = {P.hidden, 0, DK_MAP_UP, l * P.hidden, nullptr, nullptr, nullptr};
            f.tiles = P.hidden / 8;
            break;
        case PH_DOWN:
            f.K = P.hidden;
            f.nseg = 1;
            f.ldy = P.dim;
            f.s[0] = {P.dim, 0, DK_MAP_DOWN, l * P.dim, gem ? P.xb2 : xcur, nullptr, gem ? nullptr : xcur};
            f.tiles = P.dim / 16;
            break;
        default:  // PH_CLS
            f.K = P.dim;
            f.nseg = 1;
            f.ldy = P.vocab;
            f.tt = P.type_out;
            f.argmax = true;
            f.s[0] = {P.vocab, 0, DK_MAP_OUT, 0, P.logits, nullptr, nullptr};
            f.tiles = (P.vocab + 15) / 16;
            break;
    }
    f.KB = f.K / 32;
    return f;
}

__device__ __forceinline__ int seg_of(const DPhase& f, int tile) {
    int s = 0;
    if (f.nseg > 1 && f.epi == MV_EPI_STORE && tile >= f.s[1].tile0) s = 1;
    if (f.nseg > 2 && tile >= f.s[2].tile0) s = 2;
    return s;
}

__device__ __forceinline__ unsigned long long ld_acquire_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ int ld_volatile_int(const int* p) { return *reinterpret_cast<const volatile int*>(p); }

// Grid barrier among the consumer warps of all CTAs.  Bounded: after ~2 s
// (or when another CTA already gave up) it records a timeout and raises the
// abort flag instead of waiting forever.
__device__ bool grid_sync(const DecodeParams& P, unsigned long long target, int* s_ok) {
    consumer_bar();   // the CTA's writes happen before thread 0's release
    if (threadIdx.x == 0) {
        int ok = 1;
        asm volatile("red.release.gpu.global.add.u64 [%0], 1;" ::"l"(P.bar) : "memory");
        const uint64_t t0 = global_ns();
        uint32_t it = 0;
        while (ld_acquire_u64(&P.bar[0]) < target) {
            __nanosleep(32);
            if ((++it & 63u) == 0u && (global_ns() - t0 > 2000000000ull || ld_volatile_int(P.abort))) {
                atomicOr(P.err, BREW_DEVERR_TIMEOUT_FULL);
                atomicExch(P.abort, 1);
                ok = 0;
                break;
            }
        }
        *s_ok = ok;
    }
    consumer_bar();   // ... and the acquire happens before every thread's reads
    return *s_ok != 0;
}

// Sum over the 256 consumer threads.
__device__ __forceinline__ float consumer_sum(float v, float* red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    v = warp_sum(v);
    if (lane == 0) red[warp] = v;
    consumer_bar();
    float t = 0.0f;
#pragma unroll
    for (int w = 0; w < 8; ++w) t += red[w];
    consumer_bar();
    return t;
}

enum { SRC_EMBED = 0, SRC_PLAIN = 1, SRC_GEMMA_ADD = 2 };

// Loads K floats (K % 4 == 0, 16-byte aligned) into shared memory with every
// load in flight at once (through L2: the data was written by other CTAs).
__device__ __forceinline__ void stage_vec(float* dst, const float* src, int K) {
    const float4* s4 = reinterpret_cast<const float4*>(src);
    float4* d4 = reinterpret_cast<float4*>(dst);
    const int n4 = K / 4;
#pragma unroll 4
    for (int i = threadIdx.x; i < n4; i += 256) d4[i] = __ldcg(&s4[i]);
}

// Builds the prep records of one phase's input vector(s) in shared memory.
//   SRC_EMBED      v = dequant(token row) (* sqrt(dim), Gemma3); written to xout
//   SRC_PLAIN      v = src
//   SRC_GEMMA_ADD  v = src + rmsnorm(t, tw)   (Gemma3 post-norm residual); written to xout
// then records of rmsnorm(v, nw) (nw != null) or of v.  The vector is first
// staged in shared memory (`vec`, K floats).  xout writes are split over the
// CTAs by block (block j by CTA j % G), so each element has one writer.
__device__ void prep_phase(const DecodeParams& P, int mode, const float* src, int ld, int K, const float* nw,
                           const float* t, const float* tw, float* xout, uint8_t* prep, float* vec, float* red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int KB = K / 32;
    const int G = gridDim.x;
    for (int b = 0; b < P.batch; ++b) {
        if (mode == SRC_EMBED) {
            int tok = P.tokens[b];
            if (tok < 0 || tok >= P.vocab) {
                if (threadIdx.x == 0) atomicOr(P.err, BREW_DEVERR_BAD_TOKEN);
                tok = 0;
            }
            const float es = (float)sqrt((double)K);   // Kernels.scaleEmbeddings
            for (int i = threadIdx.x; i < K; i += 256) {
                float v = dequant_elem(P.type_embed, P.embed, (int64_t)tok * K + i);
                vec[i] = P.arch == BREW_ARCH_GEMMA3 ? __fmul_rn(v, es) : v;
            }
            consumer_bar();
        } else if (mode == SRC_GEMMA_ADD) {
            stage_vec(vec, t + (int64_t)b * ld, K);
            consumer_bar();
            float ss = 0.0f;
            for (int i = threadIdx.x; i < K; i += 256) ss += vec[i] * vec[i];
            const float tsc = rms_scale(consumer_sum(ss, red), K, P.eps);
            const float* sb = src + (int64_t)b * ld;
            for (int i = threadIdx.x; i < K; i += 256) vec[i] = __ldcg(&sb[i]) + vec[i] * tsc * tw[i];
            consumer_bar();
        } else {
            stage_vec(vec, src + (int64_t)b * ld, K);
            consumer_bar();
        }
        float scale = 1.0f;
        if (nw) {
            float ss = 0.0f;
            for (int i = threadIdx.x; i < K; i += 256) ss += vec[i] * vec[i];
            scale = rms_scale(consumer_sum(ss, red), K, P.eps);
        }
        for (int j = warp; j < KB; j += 8) {
            const float v = vec[32 * j + lane];
            if (xout && (j % G) == (int)blockIdx.x) __stcg(&xout[(int64_t)b * ld + 32 * j + lane], v);
            const float r = nw ? v * scale * nw[32 * j + lane] : v;
            prep_emit_warp(prep + (size_t)j * P.rec_bytes, P.batch, b, r);
        }
        consumer_bar();
    }
}

// Writes one finished tile of a phase (values summed over the tile's ws warps
// and the three limb columns).
template <int NTC>
__device__ void phase_tile_out(const DecodeParams& P, const DPhase& f, int tile, const float* red, int warp0, int ws,
                               int lane, unsigned long long* s_best) {
    auto V = [&](int r, int b) {
        float v = 0.0f;
        for (int s = 0; s < ws; ++s) {
            const float* rr = red + ((warp0 + s) * 16 + r) * NTC + 4 * b;
            v += (rr[2] + rr[1] * 256.0f) + rr[0] * 65536.0f;
        }
        return v;
    };
    if (f.epi == MV_EPI_STORE) {
        const DSeg& sg = f.s[seg_of(f, tile)];
        const int rb = (tile - sg.tile0) * 16;
        for (int idx = lane; idx < 16 * P.batch; idx += 32) {
            const int r = idx & 15, b = idx >> 4;
            const int row = rb + r;
            if (row >= sg.rows) continue;
            float v = V(r, b);
            if (sg.bias) v = v + sg.bias[row];
            if (sg.resid) v = __ldcg(&sg.resid[(int64_t)b * f.ldy + row]) + v;
            sg.y[(int64_t)b * f.ldy + row] = v;
            if (f.argmax) atomicMax(&s_best[b], argmax_key(v, row));
        }
        return;
    }
    const int i0 = tile * 8;
    for (int idx = lane; idx < 8 * P.batch; idx += 32) {
        const int r = idx & 7, b = idx >> 3;
        f.s[0].y[(int64_t)b * f.ldy + i0 + r] = act_glu(V(r, b), f.epi) * V(r + 8, b);
    }
}

struct Ring {
    uint64_t* full;
    uint64_t* empty;
    uint8_t* stages;
    int ns, stage_bytes;
};

// Consumer side of one matvec phase: this CTA's tiles, stage by stage.
template <int TT, int NT>
__device__ void mv_phase(const DecodeParams& P, const DPhase& f, const Ring& ring, int& q, uint32_t prep_s,
                         float* red, unsigned long long* s_best, bool& aborted) {
    constexpr int NTC = NT * 8;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, t = lane & 3;
    const int G = gridDim.x;
    const int t0 = (int)((int64_t)blockIdx.x * f.tiles / G);
    const int t1 = (int)((int64_t)(blockIdx.x + 1) * f.tiles / G);
    const int nt = t1 - t0;
    if (nt <= 0) return;
    const Geom geo = tma_geom(nt, f.KB, P.nb_cap);
    const int ngroups = (nt + geo.gs - 1) / geo.gs;
    const int tw = warp / geo.ws, sub = warp % geo.ws;
    float acc[NT][4];
#pragma unroll
    for (int n = 0; n < NT; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.0f;
    for (int grp = 0; grp < ngroups; ++grp) {
        const int tg0 = t0 + grp * geo.gs;
        const int ng = min(geo.gs, t1 - tg0);
        for (int chunk = 0; chunk < geo.nchunks; ++chunk, ++q) {
            const int stage = q % ring.ns;
            if (!aborted && !mbar_wait_bounded(&ring.full[stage], (q / ring.ns) & 1, P.err, BREW_DEVERR_TIMEOUT_FULL))
                aborted = true;
            if (!aborted && tw < ng) {
                const uint32_t sb = smem_u32(ring.stages + (size_t)stage * ring.stage_bytes);
                tma_tile_stage<TT, NT>(acc, sb, prep_s + chunk * geo.KC * P.rec_bytes, P.rec_bytes, tw, geo.nb, sub,
                                       geo.ws, g, t, P.batch);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&ring.empty[stage]);
        }
        float* myred = red + warp * 16 * NTC;
        if (tw < ng) {
#pragma unroll
            for (int n = 0; n < NT; ++n) {
                myred[g * NTC + n * 8 + 2 * t] = acc[n][0];
                myred[g * NTC + n * 8 + 2 * t + 1] = acc[n][1];
                myred[(g + 8) * NTC + n * 8 + 2 * t] = acc[n][2];
                myred[(g + 8) * NTC + n * 8 + 2 * t + 1] = acc[n][3];
                acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.0f;
            }
        }
        consumer_bar();
        if (tw < ng && sub == 0) phase_tile_out<NTC>(P, f, tg0 + tw, red, warp, geo.ws, lane, s_best);
        consumer_bar();
    }
}

// Producer side of one matvec phase: the same tiles and stages, in order.
template <int TT>
__device__ void produce_phase(const DecodeParams& P, const DPhase& f, const Ring& ring, int& q) {
    constexpr int BB = TT == BREW_TYPE_Q8_0 ? 34 : 18;
    constexpr int BOXW = 8 * BB;
    const int lane = threadIdx.x & 31;
    const int G = gridDim.x;
    const int t0 = (int)((int64_t)blockIdx.x * f.tiles / G);
    const int t1 = (int)((int64_t)(blockIdx.x + 1) * f.tiles / G);
    const int nt = t1 - t0;
    if (nt <= 0) return;
    const Geom geo = tma_geom(nt, f.KB, P.nb_cap);
    const int ngroups = (nt + geo.gs - 1) / geo.gs;
    const bool glu = f.epi != MV_EPI_STORE;
    for (int grp = 0; grp < ngroups; ++grp) {
        const int tg0 = t0 + grp * geo.gs;
        const int ng = min(geo.gs, t1 - tg0);
        for (int chunk = 0; chunk < geo.nchunks; ++chunk, ++q) {
            const int stage = q % ring.ns;
            if (q >= ring.ns) {
                bool ok = false;
                const uint64_t t0ns = global_ns();
                for (uint32_t it = 0;; ++it) {
                    if (mbar_try_wait(&ring.empty[stage], ((q / ring.ns) - 1) & 1)) { ok = true; break; }
                    __nanosleep(128);   // the ring is full: do not steal issue slots from the consumers
                    if ((it & 255u) == 255u && (global_ns() - t0ns > 2000000000ull || ld_volatile_int(P.abort))) break;
                }
                if (!ok) {
                    if (lane == 0) {
                        atomicOr(P.err, BREW_DEVERR_TIMEOUT_EMPTY);
                        atomicExch(P.abort, 1);
                    }
                    q = 1 << 30;   // stop producing
                    return;
                }
            }
            uint8_t* sbase = ring.stages + (size_t)stage * ring.stage_bytes;
            const int nbox = ng * geo.nb * (glu ? 2 : 1);
            if (lane == 0) mbar_arrive_expect_tx(&ring.full[stage], ng * geo.nb * 16 * BOXW);
            __syncwarp();
            for (int k = lane; k < nbox; k += 32) {
                const int half = glu ? (k & 1) : 0;
                const int kb = glu ? (k >> 1) : k;
                const int ts = kb / geo.nb, bi = kb % geo.nb;
                const int tile = tg0 + ts;
                const int x = (chunk * geo.KC + bi * 8) * BB / 8;
                uint8_t* dst = sbase + ((ts * geo.nb + bi) * 16 + half * 8) * BOXW;
                if (glu) {
                    const DSeg& sg = f.s[half];
                    tma_load_2d(dst, &P.maps[sg.map], x, sg.yoff + tile * 8, &ring.full[stage]);
                } else {
                    const DSeg& sg = f.s[seg_of(f, tile)];
                    tma_load_2d(dst, &P.maps[sg.map], x, sg.yoff + (tile - sg.tile0) * 16, &ring.full[stage]);
                }
            }
            __syncwarp();
        }
    }
}

// Positions of K / V staged in shared memory at a time.
__device__ __forceinline__ int attn_sub(int hd) { return hd <= 128 ? 64 : 32; }

// Attention for the items of this CTA (AttentionEngine.attend), then the
// last CTA of each (sequence, kv head) combines the chunks into xb.  K and V
// rows of a chunk are staged in shared memory (`kv`, attn_sub(hd) positions
// at a time) with every load in flight.
__device__ void attn_phase(const DecodeParams& P, int l, float* sm, float* kv) {
    const int G = P.n_heads / P.n_kv, hd = P.hd, half = hd / 2;
    const int kvd = P.n_kv * hd, qw = P.n_heads * hd, ldq = qw + 2 * kvd;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const bool gem = P.arch == BREW_ARCH_GEMMA3;
    const bool global = ((l + 1) % 6) == 0;   // Gemma3AttentionPattern.java:10-12
    const int window = (gem && !global) ? P.window : 0;
    const int table = (gem && !global) ? 1 : 0;
    const int nch = P.nchunk;
    const int cap = max(ATTN_MIN_POS, (P.seq_len + nch - 1) / nch);
    const int SUB = attn_sub(hd);
    float* qs = sm;                // [G][hd]
    float* ks = qs + G * hd;       // [hd]
    float* sc = ks + hd;           // [G][cap]
    float* wc = sc + G * cap;      // [G][nch]
    float* sml = wc + G * nch;     // [2][16]: m, l / 1/L
    int* s_last = reinterpret_cast<int*>(sml + 32);
    const int items = P.batch * P.n_kv * nch;
    for (int item = blockIdx.x; item < items; item += gridDim.x) {
        const int c = item % nch, hk = (item / nch) % P.n_kv, b = item / (nch * P.n_kv);
        const int pos = P.pos[b];
        if (pos < 0 || pos >= P.seq_len) {
            if (tid == 0) atomicOr(P.err, BREW_DEVERR_BAD_INDEX);
            continue;
        }
        const int start = window > 0 ? max(0, pos - window + 1) : 0;
        const int len = pos - start + 1;
        const int per = max(ATTN_MIN_POS, (len + nch - 1) / nch);
        const int used = (len + per - 1) / per;
        const int p0 = start + c * per;
        const int n = min(cap, max(0, min(pos + 1, p0 + per) - p0));
        const int stride = hd + 2;
        float* pbase = P.attn_part + ((int64_t)b * P.n_heads + (int64_t)hk * G) * nch * stride;
        float* kc = P.kc + (int64_t)b * P.cache_bstride + (int64_t)l * P.seq_len * kvd;
        float* vc = P.vc + (int64_t)b * P.cache_bstride + (int64_t)l * P.seq_len * kvd;
        if (c < used) {
            const float* qsrc = P.qkv + (int64_t)b * ldq + (int64_t)hk * G * hd;
            for (int i = tid; i < G * hd; i += 256) qs[i] = __ldcg(&qsrc[i]);
            const float* ksrc = P.qkv + (int64_t)b * ldq + qw + (int64_t)hk * hd;
            for (int i = tid; i < hd; i += 256) ks[i] = __ldcg(&ksrc[i]);
            consumer_bar();
            if (P.rms_q) {   // Kernels.headWiseRmsNorm (Qwen3, Gemma3)
                for (int hh = warp; hh <= G; hh += 8) {
                    float* vecp = hh < G ? qs + hh * hd : ks;
                    const float* w = (hh < G ? P.rms_q : P.rms_k) + (int64_t)l * hd;
                    float ss = 0.0f;
                    for (int i = lane; i < hd; i += 32) ss += vecp[i] * vecp[i];
                    const float scale = rms_scale(warp_sum(ss), hd, P.eps);
                    __syncwarp();
                    for (int i = lane; i < hd; i += 32) vecp[i] = vecp[i] * scale * w[i];
                }
                consumer_bar();
            }
            const float* cs = P.rope_cos + ((int64_t)table * P.seq_len + pos) * half;
            const float* sn = P.rope_sin + ((int64_t)table * P.seq_len + pos) * half;
            const bool inter = P.arch == BREW_ARCH_LLAMA;
            for (int idx = tid; idx < (G + 1) * half; idx += 256) {
                const int hh = idx / half, d = idx % half;
                float* vecp = hh < G ? qs + hh * hd : ks;
                const int i0 = inter ? 2 * d : d;
                const int i1 = inter ? 2 * d + 1 : d + half;
                const float a = vecp[i0], bb = vecp[i1], cc = cs[d], ss = sn[d];
                vecp[i0] = __fsub_rn(__fmul_rn(a, cc), __fmul_rn(bb, ss));
                vecp[i1] = __fadd_rn(__fmul_rn(a, ss), __fmul_rn(bb, cc));
            }
            consumer_bar();
            if (pos >= p0 && pos < p0 + n) {   // storeKeyValueInCache (AttentionEngine.java:34-38)
                const float* vsrc = P.qkv + (int64_t)b * ldq + qw + kvd + (int64_t)hk * hd;
                for (int i = tid; i < hd; i += 256) {
                    kc[(int64_t)pos * kvd + hk * hd + i] = ks[i];
                    vc[(int64_t)pos * kvd + hk * hd + i] = __ldcg(&vsrc[i]);
                }
            }
            consumer_bar();
            const int hd4 = hd / 4;
            // scores q.k / sqrt(hd), K staged SUB positions at a time
            for (int s0 = 0; s0 < n; s0 += SUB) {
                const int ns = min(SUB, n - s0);
                for (int i = tid; i < ns * hd4; i += 256) {
                    const int r = i / hd4, cidx = i % hd4;
                    reinterpret_cast<float4*>(kv)[i] =
                        __ldcg(reinterpret_cast<const float4*>(kc + (int64_t)(p0 + s0 + r) * kvd + hk * hd) + cidx);
                }
                consumer_bar();
                for (int tt = warp; tt < ns; tt += 8) {
                    const float* kr = kv + tt * hd;
                    for (int h = 0; h < G; ++h) {
                        float s = 0.0f;
                        for (int i = lane; i < hd; i += 32) s += qs[h * hd + i] * kr[i];
                        s = warp_sum(s);
                        if (lane == 0) sc[h * cap + s0 + tt] = s * P.inv_scale;
                    }
                }
                consumer_bar();
            }
            for (int h = warp; h < G; h += 8) {
                float m = -INFINITY;
                for (int tt = lane; tt < n; tt += 32) m = fmaxf(m, sc[h * cap + tt]);
                m = warp_max(m);
                float lsum = 0.0f;
                for (int tt = lane; tt < n; tt += 32) {
                    const float e = expf(sc[h * cap + tt] - m);
                    sc[h * cap + tt] = e;
                    lsum += e;
                }
                lsum = warp_sum(lsum);
                if (lane == 0) {
                    sml[h] = m;
                    sml[16 + h] = lsum;
                }
            }
            consumer_bar();
            // P.V with V staged SUB positions at a time; thread owns outputs idx
            float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};   // G*hd <= 1024 outputs over 256 threads
            for (int s0 = 0; s0 < n; s0 += SUB) {
                const int ns = min(SUB, n - s0);
                for (int i = tid; i < ns * hd4; i += 256) {
                    const int r = i / hd4, cidx = i % hd4;
                    reinterpret_cast<float4*>(kv)[i] =
                        __ldcg(reinterpret_cast<const float4*>(vc + (int64_t)(p0 + s0 + r) * kvd + hk * hd) + cidx);
                }
                consumer_bar();
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const int idx = tid + 256 * k;
                    if (idx < G * hd) {
                        const int h = idx / hd, i = idx % hd;
                        float a = acc[k];
                        for (int tt = 0; tt < ns; ++tt) a += sc[h * cap + s0 + tt] * kv[tt * hd + i];
                        acc[k] = a;
                    }
                }
                consumer_bar();
            }
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int idx = tid + 256 * k;
                if (idx < G * hd) {
                    const int h = idx / hd, i = idx % hd;
                    __stcg(&pbase[((int64_t)h * nch + c) * stride + 2 + i], acc[k]);
                }
            }
            if (tid < G) {
                __stcg(&pbase[((int64_t)tid * nch + c) * stride + 0], sml[tid]);
                __stcg(&pbase[((int64_t)tid * nch + c) * stride + 1], sml[16 + tid]);
            }
        }
        // arrival; the last CTA of (b, hk) combines the used chunks in order
        __threadfence();
        consumer_bar();
        int* ctr = &P.attn_ctr[b * P.n_kv + hk];
        if (tid == 0) *s_last = (atomicAdd(ctr, 1) == nch - 1);
        consumer_bar();
        if (*s_last) {
            __threadfence();
            for (int h = warp; h < G; h += 8) {
                float M = -INFINITY;
                for (int k = lane; k < used; k += 32) M = fmaxf(M, __ldcg(&pbase[((int64_t)h * nch + k) * stride]));
                M = warp_max(M);
                float L = 0.0f;
                for (int k = lane; k < used; k += 32) {
                    const float w = expf(__ldcg(&pbase[((int64_t)h * nch + k) * stride]) - M);
                    wc[h * nch + k] = w;
                    L += w * __ldcg(&pbase[((int64_t)h * nch + k) * stride + 1]);
                }
                L = warp_sum(L);
                if (lane == 0) sml[16 + h] = 1.0f / L;
            }
            consumer_bar();
            for (int idx = tid; idx < G * hd; idx += 256) {
                const int h = idx / hd, i = idx % hd;
                const float* src = pbase + (int64_t)h * nch * stride + 2 + i;
                float o0 = 0.0f, o1 = 0.0f, o2 = 0.0f, o3 = 0.0f;
                int k = 0;
                for (; k + 4 <= used; k += 4) {   // independent loads in flight
                    const float v0 = __ldcg(src + (int64_t)k * stride), v1 = __ldcg(src + (int64_t)(k + 1) * stride);
                    const float v2 = __ldcg(src + (int64_t)(k + 2) * stride), v3 = __ldcg(src + (int64_t)(k + 3) * stride);
                    o0 += wc[h * nch + k] * v0;
                    o1 += wc[h * nch + k + 1] * v1;
                    o2 += wc[h * nch + k + 2] * v2;
                    o3 += wc[h * nch + k + 3] * v3;
                }
                for (; k < used; ++k) o0 += wc[h * nch + k] * __ldcg(src + (int64_t)k * stride);
                P.xb[(int64_t)b * qw + (int64_t)hk * G * hd + idx] = ((o0 + o1) + (o2 + o3)) * sml[16 + h];
            }
            if (tid == 0) *ctr = 0;
        }
        consumer_bar();
    }
}

template <int TYPE, int CTYPE, int NT>
__global__ void __launch_bounds__(288, 1) decode_kernel(const __grid_constant__ DecodeParams P) {
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr int NTC = NT * 8;
    const int NS = P.nstages;
    Ring ring;
    ring.full = reinterpret_cast<uint64_t*>(smem);
    ring.empty = ring.full + NS;
    ring.ns = NS;
    ring.stage_bytes = P.stage_bytes;
    unsigned long long* s_best = reinterpret_cast<unsigned long long*>(smem + 512);   // [16]
    __shared__ unsigned long long s_base;
    __shared__ int s_ok;
    float* s_red = reinterpret_cast<float*>(smem + 640);                               // [32]
    float* red = reinterpret_cast<float*>(smem + 768);                                 // [8][16][NTC]
    float* vec = reinterpret_cast<float*>(smem + 768 + 8 * 16 * NTC * 4);
    vec = reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(vec) + 127) & ~uintptr_t(127));
    uint8_t* prep = reinterpret_cast<uint8_t*>(vec) + P.vec_bytes;
    ring.stages = prep + P.prep_bytes;
    ring.stages = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(ring.stages) + 127) & ~uintptr_t(127));

    const int tid = threadIdx.x, warp = tid >> 5;
    const int L = P.n_layers;
    if (tid == 0) {
        for (int s = 0; s < NS; ++s) {
            mbar_init(&ring.full[s], 1);
            mbar_init(&ring.empty[s], 8);
        }
        fence_mbar_init();
        s_base = P.bar[1];
    }
    if (tid < 16) s_best[tid] = 0ull;
    __syncthreads();

    if (warp == 8) {
        // ------------------------------- producer -------------------------------
        int q = 0;
        for (int l = 0; l < L && q < (1 << 29); ++l) {
            for (int ph = PH_QKV; ph <= PH_DOWN && q < (1 << 29); ++ph) {
                const DPhase f = make_phase(P, l, ph, P.x0);
                produce_phase<TYPE>(P, f, ring, q);
            }
        }
        if (q < (1 << 29)) {
            const DPhase f = make_phase(P, 0, PH_CLS, P.x0);
            produce_phase<CTYPE>(P, f, ring, q);
        }
        return;
    }

    // --------------------------------- consumers ---------------------------------
    const uint32_t prep_s = smem_u32(prep);
    const int Gc = gridDim.x;
    unsigned long long target = s_base;
    int q = 0;
    bool aborted = false;
    const bool gem = P.arch == BREW_ARCH_GEMMA3;
    float* xcur = P.x0;
    float* xalt = P.x1;
    // trace: per CTA, slot 0 = start, then per phase (prep done, work done,
    // barrier passed)
    int nev = 0;
    unsigned long long* tr = P.trace ? P.trace + (size_t)blockIdx.x * P.trace_slots : nullptr;
    auto mark = [&]() {
        if (tr && tid == 0 && nev < P.trace_slots) tr[nev] = global_ns();
        ++nev;
    };
    mark();
    auto barrier = [&]() {
        mark();
        target += (unsigned long long)Gc;
        if (!grid_sync(P, target, &s_ok)) aborted = true;
        mark();
    };
    for (int l = 0; l < L && !aborted; ++l) {
        // ---- RMSNorm (attention) + Q|K|V ----
        if (l == 0) {
            prep_phase(P, SRC_EMBED, xcur, P.dim, P.dim, P.rms_att, nullptr, nullptr, xcur, prep, vec, s_red);
        } else if (gem) {
            prep_phase(P, SRC_GEMMA_ADD, xcur, P.dim, P.dim, P.rms_att + (int64_t)l * P.dim, P.xb2,
                       P.post_ffn + (int64_t)(l - 1) * P.dim, xalt, prep, vec, s_red);
            float* tmp = xcur; xcur = xalt; xalt = tmp;
        } else {
            prep_phase(P, SRC_PLAIN, xcur, P.dim, P.dim, P.rms_att + (int64_t)l * P.dim, nullptr, nullptr, nullptr, prep,
                       vec, s_red);
        }
        mark();
        {
            const DPhase f = make_phase(P, l, PH_QKV, xcur);
            mv_phase<TYPE, NT>(P, f, ring, q, prep_s, red, s_best, aborted);
        }
        barrier();
        if (aborted) break;
        // ---- attention ----
        mark();
        attn_phase(P, l, reinterpret_cast<float*>(prep), vec);
        barrier();
        if (aborted) break;
        // ---- wo (+ residual) ----
        prep_phase(P, SRC_PLAIN, P.xb, P.n_heads * P.hd, P.n_heads * P.hd, nullptr, nullptr, nullptr, nullptr, prep,
                   vec, s_red);
        mark();
        {
            const DPhase f = make_phase(P, l, PH_O, xcur);
            mv_phase<TYPE, NT>(P, f, ring, q, prep_s, red, s_best, aborted);
        }
        barrier();
        if (aborted) break;
        // ---- RMSNorm (FFN) + gate|up ----
        if (gem) {
            prep_phase(P, SRC_GEMMA_ADD, xcur, P.dim, P.dim, P.rms_ffn + (int64_t)l * P.dim, P.xb2,
                       P.post_att + (int64_t)l * P.dim, xalt, prep, vec, s_red);
            float* tmp = xcur; xcur = xalt; xalt = tmp;
        } else {
            prep_phase(P, SRC_PLAIN, xcur, P.dim, P.dim, P.rms_ffn + (int64_t)l * P.dim, nullptr, nullptr, nullptr, prep,
                       vec, s_red);
        }
        mark();
        {
            const DPhase f = make_phase(P, l, PH_GU, xcur);
            mv_phase<TYPE, NT>(P, f, ring, q, prep_s, red, s_best, aborted);
        }
        barrier();
        if (aborted) break;
        // ---- down (+ residual) ----
        prep_phase(P, SRC_PLAIN, P.hb, P.hidden, P.hidden, nullptr, nullptr, nullptr, nullptr, prep, vec, s_red);
        mark();
        {
            const DPhase f = make_phase(P, l, PH_DOWN, xcur);
            mv_phase<TYPE, NT>(P, f, ring, q, prep_s, red, s_best, aborted);
        }
        barrier();
    }
    if (!aborted) {
        // ---- final RMSNorm + classifier + argmax ----
        if (gem)
            prep_phase(P, SRC_GEMMA_ADD, xcur, P.dim, P.dim, P.rms_final, P.xb2, P.post_ffn + (int64_t)(L - 1) * P.dim,
                       nullptr, prep, vec, s_red);
        else
            prep_phase(P, SRC_PLAIN, xcur, P.dim, P.dim, P.rms_final, nullptr, nullptr, nullptr, prep, vec, s_red);
        mark();
        const DPhase f = make_phase(P, 0, PH_CLS, xcur);
        mv_phase<CTYPE, NT>(P, f, ring, q, prep_s, red, s_best, aborted);
        consumer_bar();
        if (tid < P.batch) atomicMax(&P.am_key[tid], s_best[tid]);
        barrier();
        if (!aborted && blockIdx.x == 0) {
            if (tid < P.batch) {
                const unsigned long long k = atomicExch(&P.am_key[tid], 0ull);
                P.am_out[tid] = (int32_t)(0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull));
            }
            if (tid == 0) P.bar[1] = target;   // arrival count at the start of the next step
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
    static bool attr = false;
    if (!attr) {
        BREW_CUDA(cudaFuncSetAttribute(decode_kernel<TYPE, CTYPE, NT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)p.smem));
        attr = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.grid);
    cfg.blockDim = dim3(288);
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
    // TMA boxes of 8 blocks over 16-byte row pitches: K multiple of 256
    if (c.dim % 256 || qw % 256 || c.hidden_dim % 256) return false;
    if ((c.n_kv_heads * c.head_size) % 16) return false;
    if (c.n_heads / c.n_kv_heads > 16 || c.head_size > 512) return false;
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

int decode_prepare(DecodeParams* p, const uint8_t* wq, const uint8_t* wk, const uint8_t* wv, const uint8_t* wo,
                   const uint8_t* wgate, const uint8_t* wup, const uint8_t* wdown, const uint8_t* wout) {
    TypeInfo tl, to;
    type_info(p->type_layer, &tl);
    type_info(p->type_out, &to);
    const int qw = p->n_heads * p->hd, kvd = p->n_kv * p->hd, L = p->n_layers;
    const int Pd = p->dim / 32 * tl.block_bytes, Pq = qw / 32 * tl.block_bytes, Ph = p->hidden / 32 * tl.block_bytes;
    const int Po = p->dim / 32 * to.block_bytes;
    int rc;
    if ((rc = encode_rows_map(&p->maps[DK_MAP_Q], wq, L * qw, Pd, 8 * tl.block_bytes, 16)) ||
        (rc = encode_rows_map(&p->maps[DK_MAP_K], wk, L * kvd, Pd, 8 * tl.block_bytes, 16)) ||
        (rc = encode_rows_map(&p->maps[DK_MAP_V], wv, L * kvd, Pd, 8 * tl.block_bytes, 16)) ||
        (rc = encode_rows_map(&p->maps[DK_MAP_O], wo, L * p->dim, Pq, 8 * tl.block_bytes, 16)) ||
        (rc = encode_rows_map(&p->maps[DK_MAP_GATE], wgate, L * p->hidden, Pd, 8 * tl.block_bytes, 8)) ||
        (rc = encode_rows_map(&p->maps[DK_MAP_UP], wup, L * p->hidden, Pd, 8 * tl.block_bytes, 8)) ||
        (rc = encode_rows_map(&p->maps[DK_MAP_DOWN], wdown, L * p->dim, Ph, 8 * tl.block_bytes, 16)) ||
        (rc = encode_rows_map(&p->maps[DK_MAP_OUT], wout, p->vocab, Po, 8 * to.block_bytes, 16)))
        return rc;
    p->rec_bytes = prep_rec_bytes(p->batch);
    p->nb_cap = std::max(1, std::min(MV_MAX_BOXES, (8 * 1024) / (8 * p->rec_bytes)));
    const int kmax = std::max(std::max(p->dim, qw), p->hidden);
    const int G = p->n_heads / p->n_kv;
    const int cap = std::max(ATTN_MIN_POS, (p->seq_len + p->nchunk - 1) / p->nchunk);
    const size_t attn_floats = (size_t)G * p->hd + p->hd + (size_t)G * cap + (size_t)G * p->nchunk + 64;
    p->prep_bytes = (int)((std::max((size_t)(kmax / 32) * p->rec_bytes, attn_floats * 4) + 127) & ~size_t(127));
    // staged input vector, or K / V rows of an attention sub-chunk
    p->vec_bytes = (int)((std::max((size_t)kmax * 4, (size_t)(p->hd <= 128 ? 64 : 32) * p->hd * 4) + 127) & ~size_t(127));
    const int boxw = 8 * std::max(tl.block_bytes, to.block_bytes);
    p->stage_bytes = MV_MAX_BOXES * 16 * boxw;
    const int NT = 1;   // DK_MAX_BATCH <= 2
    const size_t fixed = 768 + (size_t)8 * 16 * NT * 8 * 4 + 128 + p->vec_bytes + p->prep_bytes + 128;
    const size_t budget = 224 * 1024;
    BREW_CHECK(fixed + 2 * (size_t)p->stage_bytes <= budget, BREW_ERR_UNSUPPORTED, "decode kernel: shapes too large");
    p->nstages = (int)std::min<size_t>(32, (budget - fixed) / p->stage_bytes);
    p->smem = fixed + (size_t)p->nstages * p->stage_bytes;
    int dev = 0, coop = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev);
    BREW_CHECK(coop, BREW_ERR_UNSUPPORTED, "decode kernel: cooperative launch unsupported");
    p->grid = num_sms();
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
