// matvec.cu — y = W x for W in unchanged GGUF Q8_0 / Q4_0 blocks (sm_100a).
//
// Replaces Linear.matmul (transformer/math/Linear.java:40-99).  Design:
//   * Weights stay in their 34-byte (Q8_0) / 18-byte (Q4_0) blocks.  One
//     producer warp streams them into a ring of shared-memory stages with TMA:
//     cp.async.bulk.tensor.2d boxes of 16 rows x 8 blocks through a tensor map
//     (row pitch a multiple of 16 bytes; each CTA loads only for itself), or bulk copies of whole
//     rows otherwise.
//   * The x side arrives as prep records (prep.cuh): per 32-block three int8
//     limb columns per vector.  One mma.sync m16n8k32 int8 MMA gives the exact
//     integer block dot products of 16 rows; the fp32 epilogue multiplies by
//     the block's fp16 weight scale and the vector's block scale.
//   * Each CTA owns whole 16-row tiles (no cross-CTA reduction).  With many
//     tiles a warp owns a tile; with few, 2/4/8 warps split a tile's blocks and
//     combine through shared memory in a fixed order: the result is
//     deterministic.
//   * Fused epilogues: bias, residual add, SwiGLU/GeGLU (gate and up rows in
//     one tile) with the next matvec's prep records, a last-CTA pass that
//     RMS-normalises the finished vector, and the classifier argmax.
//   * Programmatic dependent launch: weight copies are issued before
//     griddepcontrol.wait, so they overlap the previous kernel's tail.
#include "matvec.cuh"
#include "mv_device.cuh"
#include "prep.cuh"

#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

namespace brew {

namespace {

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

__device__ __forceinline__ Geom cta_geom(const MvParams& p, int nt) {
    if (p.mode == MV_MODE_TMA) return tma_geom(nt, p.KB, p.nb_cap);
    Geom g;
    g.gs = 1;
    g.ws = 8;
    g.nb = 1;
    g.KC = p.mode == MV_MODE_CONTIG ? p.KB : p.kcb;
    g.nchunks = p.KB / g.KC;
    return g;
}

// Writes one finished tile: vals are summed over the ws warps of the tile
// (red slices warp0 .. warp0+ws-1, in order) and the three limb columns.
template <int NTC>
__device__ void tile_out(const MvParams& p, int tile, const float* red, int warp0, int ws, int lane,
                         unsigned long long* s_best) {
    auto V = [&](int r, int b) {
        // limb columns hi, mid, lo of vector b carry weights 2^16, 2^8, 1
        float v = 0.0f;
        for (int s = 0; s < ws; ++s) {
            const float* rr = red + ((warp0 + s) * 16 + r) * NTC + 4 * b;
            v += (rr[2] + rr[1] * 256.0f) + rr[0] * 65536.0f;
        }
        return v;
    };
    if (p.epi == MV_EPI_STORE) {
        int s = 0;
        if (p.nseg > 1 && tile >= p.seg[1].tile0) s = 1;
        if (p.nseg > 2 && tile >= p.seg[2].tile0) s = 2;
        const MvSeg& sg = p.seg[s];
        const int rb = (tile - sg.tile0) * MV_TILE_ROWS;
        for (int idx = lane; idx < MV_TILE_ROWS * p.batch; idx += 32) {
            const int r = idx & 15, b = idx >> 4;
            const int row = rb + r;
            if (row >= sg.rows) continue;
            float v = V(r, b);
            if (sg.bias) v = v + sg.bias[row];
            if (sg.resid) v = sg.resid[(int64_t)b * p.ldy + row] + v;
            sg.y[(int64_t)b * p.ldy + row] = v;
            if (p.post == MV_POST_ARGMAX) atomicMax(&s_best[b], argmax_key(v, row));
        }
        return;
    }
    const int i0 = (tile - p.seg[0].tile0) * 8;
    for (int idx = lane; idx < 8 * p.batch; idx += 32) {
        const int r = idx & 7, b = idx >> 3;
        const int i = i0 + r;
        if (i >= p.seg[0].rows) continue;
        p.seg[0].y[(int64_t)b * p.ldy + i] = act_glu(V(r, b), p.epi) * V(r + 8, b);
    }
    if (p.next_prep) {
        // the fourth tile of a 32-wide group to finish emits its prep record
        __threadfence();
        __syncwarp();
        int last = 0;
        const int group = i0 >> 5;
        if (lane == 0) last = atomicAdd(&p.group_counters[group], 1) == 3;
        last = __shfl_sync(0xffffffffu, last, 0);
        if (last) {
            __threadfence();
            for (int b = 0; b < p.batch; ++b) {
                const float v = __ldcg(&p.seg[0].y[(int64_t)b * p.ldy + group * 32 + lane]);
                prep_emit_warp(p.next_prep + (size_t)group * p.rec_bytes, p.batch, b, v);
            }
            if (lane == 0) p.group_counters[group] = 0;
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
    unsigned long long* s_best = reinterpret_cast<unsigned long long*>(smem + 256);   // [16]
    float* red = reinterpret_cast<float*>(smem + 384);                               // [8][16][NTC]
    uint8_t* stages = smem + 384 + MV_CONSUMER_WARPS * 16 * NTC * 4;
    stages = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(stages) + 127) & ~uintptr_t(127));

    const int tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    const int G = gridDim.x;
    const int t0 = (int)((int64_t)blockIdx.x * p.total_tiles / G);
    const int t1 = (int)((int64_t)(blockIdx.x + 1) * p.total_tiles / G);
    const int nt = t1 - t0;
    const Geom geo = cta_geom(p, nt);
    const int ngroups = (nt + geo.gs - 1) / geo.gs;
    const int nq = ngroups * geo.nchunks;
    const int BOXW = p.kcb * BB;                 // TMA box row bytes
    const int prep_bytes = geo.KC * p.rec_bytes;
    const bool glu = p.epi != MV_EPI_STORE;

    if (tid == 0) {
        for (int s = 0; s < NS; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], MV_CONSUMER_WARPS);
        }
        fence_mbar_init();
    }
    if (tid < 16) s_best[tid] = 0ull;
    __syncthreads();

    if (warp == MV_CONSUMER_WARPS) {
        // ------------------------------ producer ------------------------------
        auto issue_weights = [&](int q) {
            const int stage = q % NS;
            const int grp = q / geo.nchunks, chunk = q % geo.nchunks;
            const int tg0 = t0 + grp * geo.gs;
            const int ng = min(geo.gs, t1 - tg0);
            uint8_t* sbase = stages + (size_t)stage * p.stage_bytes;
            if (p.mode == MV_MODE_TMA) {
                const int nbox = ng * geo.nb * (glu ? 2 : 1);
                if (lane == 0) mbar_arrive_expect_tx(&full[stage], ng * geo.nb * MV_TILE_ROWS * BOXW + prep_bytes);
                __syncwarp();
                for (int k = lane; k < nbox; k += 32) {
                    const int half = glu ? (k & 1) : 0;
                    const int kb = glu ? (k >> 1) : k;
                    const int ts = kb / geo.nb, bi = kb % geo.nb;
                    const int tile = tg0 + ts;
                    const int x = (chunk * geo.KC + bi * p.kcb) * BB / 8;
                    uint8_t* dst = sbase + ((ts * geo.nb + bi) * MV_TILE_ROWS + half * 8) * BOXW;
                    if (glu) {
                        tma_load_2d(dst, &p.tmap[half], x, (tile - p.seg[0].tile0) * 8, &full[stage]);
                    } else {
                        int s = 0;
                        if (p.nseg > 1 && tile >= p.seg[1].tile0) s = 1;
                        if (p.nseg > 2 && tile >= p.seg[2].tile0) s = 2;
                        tma_load_2d(dst, &p.tmap[s], x, (tile - p.seg[s].tile0) * MV_TILE_ROWS, &full[stage]);
                    }
                }
                return;
            }
            const int tile = tg0;   // gs == 1
            if (p.mode == MV_MODE_CONTIG) {
                // whole rows: region 0 = rows 0..15 (GLU: gate rows), region 1 = up rows
                uint32_t len = 0, lead = 0;
                const uint8_t* src = nullptr;
                const int nreg = glu ? 2 : 1;
                if (lane < nreg) {
                    const int r0 = lane * 8;
                    const uint8_t* rp = tile_row_ptr(p, tile, r0);
                    if (rp) {
                        int nv = 1;
                        const int span = glu ? 8 : MV_TILE_ROWS;
                        while (nv < span && tile_row_ptr(p, tile, r0 + nv)) ++nv;
                        lead = (uint32_t)(reinterpret_cast<uintptr_t>(rp) & 15u);
                        len = (lead + (uint32_t)(nv * p.row_bytes) + 15u) & ~15u;
                        src = rp - lead;
                    }
                }
                const uint32_t total = __shfl_sync(0xffffffffu, len, 0) + __shfl_sync(0xffffffffu, len, 1);
                if (lane == 0) mbar_arrive_expect_tx(&full[stage], total + prep_bytes);
                __syncwarp();
                if (len) bulk_g2s(sbase + lane * p.region_stride, src, len, &full[stage]);
                return;
            }
            // MV_MODE_ROW: one copy per row
            uint32_t len = 0, lead = 0;
            const uint8_t* src = nullptr;
            const int CB = geo.KC * BB;
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
                const int chunk = q % geo.nchunks;
                uint8_t* sbase = stages + (size_t)(q % NS) * p.stage_bytes;
                bulk_g2s(sbase + p.stage_w, p.prep + (size_t)chunk * geo.KC * p.rec_bytes, prep_bytes, &full[q % NS]);
            }
        };
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
        const int tw = warp / geo.ws, sub = warp % geo.ws;   // tile slot, split index
        float acc[NT][4];
#pragma unroll
        for (int n = 0; n < NT; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.0f;
        bool aborted = false;

        for (int q = 0; q < nq; ++q) {
            const int stage = q % NS;
            const uint32_t parity = (q / NS) & 1;
            const int grp = q / geo.nchunks, chunk = q % geo.nchunks;
            const int tg0 = t0 + grp * geo.gs;
            const int ng = min(geo.gs, t1 - tg0);
            if (!aborted && !mbar_wait_bounded(&full[stage], parity, p.err, BREW_DEVERR_TIMEOUT_FULL)) aborted = true;
            const uint8_t* sbase = stages + (size_t)stage * p.stage_bytes;
            const uint32_t sb = smem_u32(sbase);
            const uint32_t prep0 = sb + p.stage_w;
            if (!aborted && tw < ng) {
                const int tile = tg0 + tw;
                if (p.mode == MV_MODE_TMA) {
                    tma_tile_stage<TYPE, NT>(acc, sb, prep0, p.rec_bytes, tw, geo.nb, sub, geo.ws, g, t, p.batch);
                } else {
                    // CONTIG / ROW: rows at arbitrary 2-byte alignment, block by block
                    uint32_t row0, row1;
                    if (p.mode == MV_MODE_CONTIG) {
                        const uint8_t* ra = tile_row_ptr(p, tile, 0);
                        const uint32_t la = ra ? (uint32_t)(reinterpret_cast<uintptr_t>(ra) & 15u) : 0u;
                        row0 = sb + la + g * (uint32_t)p.row_bytes;
                        if (glu) {
                            const uint8_t* rb = tile_row_ptr(p, tile, 8);
                            const uint32_t lb = rb ? (uint32_t)(reinterpret_cast<uintptr_t>(rb) & 15u) : 0u;
                            row1 = sb + p.region_stride + lb + g * (uint32_t)p.row_bytes;
                        } else {
                            row1 = sb + la + (g + 8) * (uint32_t)p.row_bytes;
                        }
                    } else {
                        const int CB = geo.KC * BB;
                        const uint8_t* rp0 = tile_row_ptr(p, tile, g);
                        const uint8_t* rp1 = tile_row_ptr(p, tile, g + 8);
                        const uint32_t l0 = rp0 ? (uint32_t)((reinterpret_cast<uintptr_t>(rp0) + (int64_t)chunk * CB) & 15u) : 0u;
                        const uint32_t l1 = rp1 ? (uint32_t)((reinterpret_cast<uintptr_t>(rp1) + (int64_t)chunk * CB) & 15u) : 0u;
                        row0 = sb + g * p.slot_pitch + l0;
                        row1 = sb + (g + 8) * p.slot_pitch + l1;
                    }
                    for (int j = sub; j < geo.KC; j += geo.ws) {
                        const uint32_t b0p = row0 + j * BB, b1p = row1 + j * BB;
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
                        mma_block<TYPE, NT>(acc, a0, a1, a2, a3, half_bits_to_float((uint16_t)lds16(b0p)),
                                            half_bits_to_float((uint16_t)lds16(b1p)), prep0 + j * p.rec_bytes, p.batch,
                                            g, t);
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[stage]);
            if (chunk != geo.nchunks - 1) continue;

            // ---- group end: every tile of the group is complete in this CTA ----
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
            if (geo.ws > 1) consumer_bar(); else __syncwarp();
            if (tw < ng && sub == 0) tile_out<NTC>(p, tg0 + tw, red, warp, geo.ws, lane, s_best);
            if (geo.ws > 1) consumer_bar(); else __syncwarp();
        }
        if (p.post == MV_POST_ARGMAX) {
            consumer_bar();
            if (tid < p.batch) atomicMax(&p.am_key[tid], s_best[tid]);
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
        if (tid < p.batch) {
            const unsigned long long k = atomicExch(&p.am_key[tid], 0ull);
            p.am_out[tid] = (int32_t)(0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull));
        }
    } else {
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
            prep_vector_cta(x, p.post_dim, p.post_norm_w, p.eps, p.post_prep, p.rec_bytes, p.batch, b, s_red);
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
        prep_emit_warp(recs + (size_t)j * rec_bytes, batch, b, v);
    }
}

template <int TYPE, int NT>
int launch_typed(const MvParams& p, cudaStream_t stream, bool pdl, int grid, size_t smem) {
    static std::mutex mu;
    static unsigned long long attr_set = 0;   // one bit per device
    {
        std::lock_guard<std::mutex> lk(mu);
        BREW_CUDA(smem_attr_per_device((const void*)mv_kernel<TYPE, NT>, 200 * 1024, &attr_set));
    }
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

// The kernel is instantiated for NT in {1, 2, 4, 8}: the n8 MMA tiles (4
// columns per vector) rounded up.  Host-side shared-memory sizing must use
// this same value.
int nt_instance(int batch) {
    const int nt = prep_nt(batch);
    return nt <= 2 ? nt : (nt <= 4 ? 4 : 8);
}

template <int TYPE>
int launch_nt(const MvParams& p, cudaStream_t stream, bool pdl, int grid, size_t smem) {
    switch (nt_instance(p.batch)) {
        case 1: return launch_typed<TYPE, 1>(p, stream, pdl, grid, smem);
        case 2: return launch_typed<TYPE, 2>(p, stream, pdl, grid, smem);
        case 4: return launch_typed<TYPE, 4>(p, stream, pdl, grid, smem);
        default: return launch_typed<TYPE, 8>(p, stream, pdl, grid, smem);
    }
}

}  // namespace

// Tensor map over `rows` rows of `pitch` bytes as 8-byte elements, box of
// `box_bytes` x `box_rows`.  Rows past the end read as zeros.
int encode_rows_map(CUtensorMap* map, const void* base, int rows, int pitch, int box_bytes, int box_rows) {
    static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
    if (!encode) {
        cudaDriverEntryPointQueryResult q;
        void* fn = nullptr;
        BREW_CUDA(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q));
        BREW_CHECK(fn && q == cudaDriverEntryPointSuccess, BREW_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
        encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
    const cuuint64_t dims[2] = {(cuuint64_t)(pitch / 8), (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)pitch};
    const cuuint32_t box[2] = {(cuuint32_t)(box_bytes / 8), (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    BREW_CHECK(r == CUDA_SUCCESS, BREW_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d): rows %d pitch %d box %dx%d", (int)r,
               rows, pitch, box_bytes, box_rows);
    return BREW_OK;
}

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
    const int BB = ti.block_bytes;
    const int P = p.KB * BB;
    const bool glu = p.epi != MV_EPI_STORE;
    // tiles per segment
    int tiles = 0;
    for (int s = 0; s < p.nseg; ++s) {
        p.seg[s].tile0 = tiles;
        if (!glu) tiles += (p.seg[s].rows + MV_TILE_ROWS - 1) / MV_TILE_ROWS;
    }
    if (glu) {
        BREW_CHECK(p.nseg == 2 && p.seg[0].rows == p.seg[1].rows, BREW_ERR_INVALID_ARG, "matvec: GLU needs 2 equal segments");
        p.seg[1].tile0 = 0;
        tiles = (p.seg[0].rows + 7) / 8;
        BREW_CHECK(!p.next_prep || p.seg[0].rows % 32 == 0, BREW_ERR_INVALID_ARG, "matvec: GLU prep needs rows %% 32 == 0");
    }
    p.total_tiles = tiles;
    // staging mode (see MvMode)
    bool aligned = (P % 16) == 0 && p.KB % 8 == 0;
    for (int s = 0; s < p.nseg; ++s) aligned = aligned && ((reinterpret_cast<uintptr_t>(p.seg[s].w) & 15) == 0);
    const int contig_rs = (8 * P + 30) & ~15;
    if (aligned) {
        p.mode = MV_MODE_TMA;
        p.kcb = 8;                                   // box: 16 rows x 8 blocks (272 or 144 bytes)
        const int boxw = p.kcb * BB;
        p.nb_cap = std::max(1, std::min(MV_MAX_BOXES, (8 * 1024) / (p.kcb * p.rec_bytes)));
        p.stage_w = MV_MAX_BOXES * MV_TILE_ROWS * boxw;
        p.stage_bytes = (p.stage_w + p.nb_cap * p.kcb * p.rec_bytes + 127) & ~127;
    } else if (2 * contig_rs + p.KB * p.rec_bytes <= 56 * 1024) {
        p.mode = MV_MODE_CONTIG;
        p.kcb = p.KB;
        p.nb_cap = 1;
        p.region_stride = contig_rs;
        p.stage_w = 2 * contig_rs;
        p.stage_bytes = (p.stage_w + p.KB * p.rec_bytes + 127) & ~127;
    } else {
        p.mode = MV_MODE_ROW;
        int KC = 1;
        for (int c = 1; c <= p.KB; ++c) {
            if (p.KB % c) continue;
            const int cb = c * BB;
            const int slot = (cb + 47) & ~15;
            if (cb <= 1184 && MV_TILE_ROWS * slot + c * p.rec_bytes <= 40 * 1024) KC = c;
        }
        p.kcb = KC;
        p.nb_cap = 1;
        p.slot_pitch = (KC * BB + 47) & ~15;
        p.stage_w = MV_TILE_ROWS * p.slot_pitch;
        p.stage_bytes = (p.stage_w + KC * p.rec_bytes + 127) & ~127;
    }
    const int NTC = nt_instance(p.batch) * 8;     // as the kernel instance lays it out
    const size_t fixed = 384 + (size_t)MV_CONSUMER_WARPS * 16 * NTC * 4 + 128;
    const size_t budget = 112 * 1024;
    int ns = budget > fixed ? (int)((budget - fixed) / p.stage_bytes) : 0;
    ns = std::max(2, std::min(ns, 12));
    p.nstages = ns;
    const size_t smem = fixed + (size_t)ns * p.stage_bytes;
    BREW_CHECK(smem <= 200 * 1024, BREW_ERR_INVALID_ARG, "matvec: %zu bytes of shared memory", smem);
    if (p.mode == MV_MODE_TMA) {
        const int box_rows = glu ? 8 : MV_TILE_ROWS;
        for (int s = 0; s < p.nseg; ++s) {
            const int rc = encode_rows_map(&p.tmap[s], p.seg[s].w, p.seg[s].rows, P, p.kcb * BB, box_rows);
            if (rc) return rc;
        }
    }
    // grid: persistent, at most one CTA per SM, each owning whole tiles
    const int grid = std::max(1, std::min(num_sms(), tiles));
    if (p.post == MV_POST_ARGMAX)
        BREW_CHECK(p.am_key && p.am_out && p.batch <= MV_ARGMAX_MAX_BATCH, BREW_ERR_INVALID_ARG, "argmax buffers");
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
