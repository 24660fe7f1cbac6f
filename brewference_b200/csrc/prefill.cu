// prefill.cu — the per-token kernels of the batched prefill (prefill.cuh).
#include <algorithm>

#include "brew_internal.cuh"
#include "prefill.cuh"
#include "prep.cuh"
#include "quant_device.cuh"

namespace brew {
namespace {

__global__ void prefill_embed_kernel(int type, const uint8_t* embed, int vocab, int dim, const int32_t* tokens,
                                     bool gemma, float* x, unsigned int* err) {
    const int t = blockIdx.x;
    int tok = tokens[t];
    if (tok < 0 || tok >= vocab) {
        if (threadIdx.x == 0) atomicOr(err, BREW_DEVERR_BAD_TOKEN);
        tok = 0;
    }
    const float es = gemma ? (float)sqrt((double)dim) : 1.0f;   // Kernels.scaleEmbeddings
    float* xr = x + (int64_t)t * dim;
    for (int i = threadIdx.x; i < dim; i += blockDim.x) {
        const float v = dequant_elem(type, embed, (int64_t)tok * dim + i);
        xr[i] = gemma ? __fmul_rn(v, es) : v;
    }
}

// One warp per (token, head vector); element i of the head is held by lane
// i % 32 in register i / 32.  R = hd / 32.
template <int R>
__global__ void __launch_bounds__(256) prefill_qk_kernel(const __grid_constant__ PfQkParams p) {
    const int lane = threadIdx.x & 31;
    const int nvec = p.n_heads + 2 * p.n_kv;
    const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (gw >= (int64_t)p.T * nvec) return;   // whole warps
    const int t = (int)(gw / nvec), v = (int)(gw % nvec);
    const int pos = p.pos0 + t;
    const int hd = p.hd, half = hd / 2, kvd = p.n_kv * hd;
    float* src = p.qkv + (int64_t)t * p.ldq + (int64_t)v * hd;   // q heads, then k heads, then v heads
    float x[R];
#pragma unroll
    for (int r = 0; r < R; ++r) x[r] = src[lane + 32 * r];
    if (v >= p.n_heads + p.n_kv) {   // value head: appended unchanged
        float* dst = p.vcache + (int64_t)pos * kvd + (int64_t)(v - p.n_heads - p.n_kv) * hd;
#pragma unroll
        for (int r = 0; r < R; ++r) dst[lane + 32 * r] = x[r];
        return;
    }
    const bool isq = v < p.n_heads;
    const float* w = isq ? p.qnorm_w : p.knorm_w;
    if (w) {   // Kernels.headWiseRmsNorm: the decode path's order of the sum
        float ss = 0.0f;
#pragma unroll
        for (int r = 0; r < R; ++r) ss += x[r] * x[r];
        const float scale = rms_scale(warp_sum(ss), hd, p.eps);
#pragma unroll
        for (int r = 0; r < R; ++r) x[r] = x[r] * scale * w[lane + 32 * r];
    }
    const float* ct = p.rope_cos + ((int64_t)p.table * p.seq_len + pos) * half;
    const float* st = p.rope_sin + ((int64_t)p.table * p.seq_len + pos) * half;
    if (!p.rope) {
        // no rotation on this layer
    } else if (p.interleaved) {
        // pair (2d, 2d + 1): partner in the neighbouring lane, same register
#pragma unroll
        for (int r = 0; r < R; ++r) {
            const int i = lane + 32 * r, d = i >> 1;
            const float other = __shfl_xor_sync(0xffffffffu, x[r], 1);
            const float c = ct[d], s = st[d];
            if ((i & 1) == 0) x[r] = __fsub_rn(__fmul_rn(x[r], c), __fmul_rn(other, s));
            else x[r] = __fadd_rn(__fmul_rn(other, s), __fmul_rn(x[r], c));
        }
    } else {
        // pair (d, d + hd/2): registers r and r + R/2 of the same lane
#pragma unroll
        for (int r = 0; r < R / 2; ++r) {
            const int d = lane + 32 * r;
            const float a = x[r], b = x[r + R / 2], c = ct[d], s = st[d];
            x[r] = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s));
            x[r + R / 2] = __fadd_rn(__fmul_rn(a, s), __fmul_rn(b, c));
        }
    }
    float* dst = isq ? src : p.kcache + (int64_t)pos * kvd + (int64_t)(v - p.n_heads) * hd;
#pragma unroll
    for (int r = 0; r < R; ++r) dst[lane + 32 * r] = x[r];
}

constexpr int PF_TILE = 32;    // key positions per tile (one per lane)
constexpr int PF_PAIRS = 32;   // (query, head) pairs per CTA: 4 per warp
constexpr int PF_KS = 33;      // float4 stride between the K^T rows of a tile

// CTA = (kv head hk, block of qb query tokens); the qb * G (query, q head)
// pairs share each 32-position K / V tile in shared memory, double-buffered
// with asynchronous copies (tile k + 1 lands while tile k is used).  K is
// stored transposed by quads: float4 kt[i/4][j] = k_j[i .. i+3], so lane j
// reads key j's quads without bank conflicts; V row-major.  Warp w owns
// pairs 4w .. 4w + 3.  Scores: lane j computes q.k_j; the softmax is online
// over tiles (running max m, sum l); the weighted sum keeps hd/32 outputs
// per lane.
template <int R>
__global__ void __launch_bounds__(256) prefill_attn_kernel(const __grid_constant__ PfAttnParams p, int qb) {
    extern __shared__ __align__(16) float sm[];
    constexpr int hd = R * 32, hd4 = hd / 4;
    const int G = p.n_heads / p.n_kv, kvd = p.n_kv * hd;
    const int hk = blockIdx.x, t0 = blockIdx.y * qb;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    float4* qs = reinterpret_cast<float4*>(sm);          // [PF_PAIRS][hd/4]
    float4* kt = qs + PF_PAIRS * hd4;                    // [2][hd/4][PF_KS]
    float4* vt = kt + 2 * hd4 * PF_KS;                   // [2][PF_TILE][hd/4]
    const int npairs = qb * G;
    for (int e = tid; e < npairs * hd4; e += 256) {
        const int pi = e / hd4, i4 = e % hd4, qi = pi / G, h = pi % G;
        qs[e] = (t0 + qi < p.T)
                    ? *reinterpret_cast<const float4*>(p.q + (int64_t)(t0 + qi) * p.ldq + (int64_t)(hk * G + h) * hd + 4 * i4)
                    : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    }
    int qpos[4];
    bool act[4];
#pragma unroll
    for (int r = 0; r < 4; ++r) {
        const int pi = warp * 4 + r, qi = pi / G;
        act[r] = pi < npairs && t0 + qi < p.T;
        qpos[r] = p.pos0 + t0 + qi;
    }
    const int tlast = min(p.T, t0 + qb) - 1;
    const int kmax = p.pos0 + tlast;                                          // last key any query sees
    const int kmin = p.window > 0 ? max(0, p.pos0 + t0 - p.window + 1) : 0;   // first key any query sees
    const float* kc = p.kcache + (int64_t)hk * hd;
    const float* vc = p.vcache + (int64_t)hk * hd;
    // tile at key k0 into buffer bf: keys past kmax are zero (never scored,
    // and their zero values keep the weighted sum finite)
    auto load_tile = [&](int k0, int bf) {
        float4* ktb = kt + bf * hd4 * PF_KS;
        float4* vtb = vt + bf * PF_TILE * hd4;
        for (int e = tid; e < PF_TILE * hd4; e += 256) {
            const int j = e / hd4, i4 = e % hd4, key = k0 + j;
            if (key <= kmax) {
                cp_async16(ktb + i4 * PF_KS + j, kc + (int64_t)key * kvd + 4 * i4);
                cp_async16(vtb + j * hd4 + i4, vc + (int64_t)key * kvd + 4 * i4);
            } else {
                ktb[i4 * PF_KS + j] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                vtb[j * hd4 + i4] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            }
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    float m[4], l[4], o[4][R];
#pragma unroll
    for (int r = 0; r < 4; ++r) {
        m[r] = -INFINITY;
        l[r] = 0.0f;
#pragma unroll
        for (int c = 0; c < R; ++c) o[r][c] = 0.0f;
    }
    load_tile(kmin, 0);
    int bf = 0;
    for (int k0 = kmin; k0 <= kmax; k0 += PF_TILE, bf ^= 1) {
        if (k0 + PF_TILE <= kmax) {   // the next tile into the other buffer (freed by the last barrier)
            load_tile(k0 + PF_TILE, bf ^ 1);
            asm volatile("cp.async.wait_group 1;" ::: "memory");
        } else {
            asm volatile("cp.async.wait_group 0;" ::: "memory");
        }
        __syncthreads();
        const float4* ktb = kt + bf * hd4 * PF_KS;
        const float* vtb = reinterpret_cast<const float*>(vt + bf * PF_TILE * hd4);
        const int key = k0 + lane;
        float s[4];
#pragma unroll
        for (int r = 0; r < 4; ++r) s[r] = 0.0f;
        for (int i4 = 0; i4 < hd4; ++i4) {
            const float4 kv = ktb[i4 * PF_KS + lane];
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                const float4 qv = qs[(warp * 4 + r) * hd4 + i4];
                s[r] = fmaf(qv.x, kv.x, s[r]);
                s[r] = fmaf(qv.y, kv.y, s[r]);
                s[r] = fmaf(qv.z, kv.z, s[r]);
                s[r] = fmaf(qv.w, kv.w, s[r]);
            }
        }
        float pj[4];
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            const bool valid = act[r] && key <= qpos[r] && (p.window <= 0 || key > qpos[r] - p.window);
            const float sv = valid ? s[r] * p.inv_scale : -INFINITY;
            const float tmax = warp_max(sv);
            if (tmax == -INFINITY) {   // no key of this tile for this pair (uniform over the warp)
                pj[r] = 0.0f;
                continue;
            }
            const float mn = fmaxf(m[r], tmax);
            const float corr = expf(m[r] - mn);
            pj[r] = valid ? expf(sv - mn) : 0.0f;
            l[r] = l[r] * corr + warp_sum(pj[r]);
            m[r] = mn;
#pragma unroll
            for (int c = 0; c < R; ++c) o[r][c] *= corr;
        }
        for (int j = 0; j < PF_TILE; ++j) {
            float vj[R];
#pragma unroll
            for (int c = 0; c < R; ++c) vj[c] = vtb[j * hd + lane + 32 * c];
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                const float w = __shfl_sync(0xffffffffu, pj[r], j);
#pragma unroll
                for (int c = 0; c < R; ++c) o[r][c] = fmaf(w, vj[c], o[r][c]);
            }
        }
        __syncthreads();   // this buffer is refilled two tiles later
    }
#pragma unroll
    for (int r = 0; r < 4; ++r) {
        if (!act[r]) continue;
        const int pi = warp * 4 + r, qi = pi / G, h = pi % G;
        const float inv = 1.0f / l[r];
        float* dst = p.xb + (int64_t)(t0 + qi) * p.ldxb + (int64_t)(hk * G + h) * hd;
#pragma unroll
        for (int c = 0; c < R; ++c) dst[lane + 32 * c] = o[r][c] * inv;
    }
}

template <int R>
size_t pf_attn_smem() {
    constexpr int hd4 = R * 8;
    return sizeof(float4) * ((size_t)PF_PAIRS * hd4 + 2 * (size_t)hd4 * PF_KS + 2 * (size_t)PF_TILE * hd4);
}

template <int R>
int attn_launch_r(const PfAttnParams& p, cudaStream_t s) {
    const int G = p.n_heads / p.n_kv;
    const int qb = std::max(1, PF_PAIRS / G);
    const size_t smem = pf_attn_smem<R>();
    static int attr_dev = -1;   // the attribute is per device
    int dev = 0;
    cudaGetDevice(&dev);
    if (attr_dev != dev) {
        BREW_CUDA(cudaFuncSetAttribute(prefill_attn_kernel<R>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        attr_dev = dev;
    }
    const dim3 grid(p.n_kv, (p.T + qb - 1) / qb);
    prefill_attn_kernel<R><<<grid, 256, smem, s>>>(p, qb);
    BREW_CUDA(cudaGetLastError());
    count_launch();
    return BREW_OK;
}

}  // namespace

bool prefill_shapes_supported(int n_heads, int n_kv, int hd) {
    return (hd == 64 || hd == 128 || hd == 256) && n_kv > 0 && n_heads % n_kv == 0 && n_heads / n_kv <= PF_PAIRS;
}

int prefill_embed_launch(int type, const uint8_t* embed, int vocab, int dim, const int32_t* tokens, int T, bool gemma,
                         float* x, unsigned int* err, cudaStream_t s) {
    if (T <= 0) return BREW_OK;
    prefill_embed_kernel<<<T, 256, 0, s>>>(type, embed, vocab, dim, tokens, gemma, x, err);
    BREW_CUDA(cudaGetLastError());
    count_launch();
    return BREW_OK;
}

int prefill_qk_launch(const PfQkParams& p, cudaStream_t s) {
    BREW_CHECK(prefill_shapes_supported(p.n_heads, p.n_kv, p.hd), BREW_ERR_UNSUPPORTED, "prefill: head size %d", p.hd);
    if (p.T <= 0) return BREW_OK;
    const int64_t warps = (int64_t)p.T * (p.n_heads + 2 * p.n_kv);
    const unsigned blocks = (unsigned)((warps + 7) / 8);
    if (p.hd == 64) prefill_qk_kernel<2><<<blocks, 256, 0, s>>>(p);
    else if (p.hd == 128) prefill_qk_kernel<4><<<blocks, 256, 0, s>>>(p);
    else prefill_qk_kernel<8><<<blocks, 256, 0, s>>>(p);
    BREW_CUDA(cudaGetLastError());
    count_launch();
    return BREW_OK;
}

int prefill_attn_launch(const PfAttnParams& p, cudaStream_t s) {
    BREW_CHECK(prefill_shapes_supported(p.n_heads, p.n_kv, p.hd), BREW_ERR_UNSUPPORTED, "prefill: head size %d", p.hd);
    if (p.T <= 0) return BREW_OK;
    if (p.hd == 64) return attn_launch_r<2>(p, s);
    if (p.hd == 128) return attn_launch_r<4>(p, s);
    return attn_launch_r<8>(p, s);
}

}  // namespace brew
