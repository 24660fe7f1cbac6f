// attention.cu — decode attention for `batch` sequences at their own
// positions (AttentionEngine.attend, transformer/attention/AttentionEngine.java:34-106).
//
// One CTA per (kv head, context chunk, sequence):
//   1. loads the G = n_heads/n_kv query heads of its KV group and the new key,
//      applies per-head RMSNorm (Qwen3/Gemma3, Kernels.headWiseRmsNorm) and
//      RoPE (interleaved for llama, NeoX otherwise; RopeCache.java:15-26),
//   2. the CTA whose chunk holds `pos` appends k, v to the fp32 cache
//      (storeKeyValueInCache, :34-38),
//   3. scores q.k * (1/sqrt(hd)) over its chunk, chunk-local softmax and P.V,
//   4. the last CTA of the (sequence, kv head) to finish combines the chunks
//      in a fixed order, writes xb and the prep records of xb for wo.
// Products in RoPE are rounded separately (no FMA), as in the Java source.
#include "attention.cuh"
#include "prep.cuh"

#include <algorithm>
#include <mutex>

namespace brew {

namespace {

constexpr int ATTN_MIN_CHUNK = 64;

__global__ void __launch_bounds__(128) attn_kernel(const __grid_constant__ AttnParams p, int cap) {
    extern __shared__ float sm[];
    const int hk = blockIdx.x, c = blockIdx.y, b = blockIdx.z;
    const int G = p.n_heads / p.n_kv, hd = p.hd, half = hd / 2;
    const int kvd = p.n_kv * hd;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    float* qs = sm;                  // [G][hd]
    float* ks = qs + G * hd;         // [hd]
    float* sc = ks + hd;             // [G][cap]
    float* red = sc + G * cap;       // [32]
    float* cs = red + 32;            // [half]
    float* sn = cs + half;           // [half]
    float* wc = sn + half;           // [G][nchunk]
    __shared__ int s_last;
    __shared__ float s_m[16], s_l[16];

    pdl_launch_dependents();
    pdl_wait();

    const int pos = p.pos[b];
    if (pos < 0 || pos >= p.seq_len) {
        if (tid == 0) atomicOr(p.err, BREW_DEVERR_BAD_INDEX);
        return;
    }
    const int start = p.window > 0 ? max(0, pos - p.window + 1) : 0;
    const int len = pos - start + 1;
    // at least ATTN_MIN_CHUNK positions per CTA: short contexts use few
    // chunks (the others only check in), long ones spread over all
    const int per = max(ATTN_MIN_CHUNK, (len + p.nchunk - 1) / p.nchunk);
    const int used = (len + per - 1) / per;
    const int p0 = start + c * per;
    const int p1 = min(pos + 1, p0 + per);
    const int n = min(cap, max(0, p1 - p0));   // per <= cap by construction
    const int stride = hd + 2;
    float* pbase = p.part + ((int64_t)b * p.n_heads + (int64_t)hk * G) * p.nchunk * stride;
    int* ctr = &p.counters[b * p.n_kv + hk];
    if (c >= used) goto arrive;
    {

    // RoPE table for this position (RopeCache.precomputeAngles)
    const float posf = (float)pos * p.rope_scale;
    for (int i = tid; i < half; i += blockDim.x) {
        const float invf = (float)(1.0 / pow((double)p.rope_base, (double)((float)(2 * i) / (float)hd)));
        const float ang = posf * invf;
        cs[i] = (float)cos((double)ang);
        sn[i] = (float)sin((double)ang);
    }
    const float* qsrc = p.q + (int64_t)b * p.ldq + (int64_t)hk * G * hd;
    for (int i = tid; i < G * hd; i += blockDim.x) qs[i] = qsrc[i];
    const float* ksrc = p.k + (int64_t)b * p.ldkv + (int64_t)hk * hd;
    for (int i = tid; i < hd; i += blockDim.x) ks[i] = ksrc[i];
    __syncthreads();

    if (p.qnorm_w) {
        for (int hh = warp; hh <= G; hh += 4) {
            float* vec = hh < G ? qs + hh * hd : ks;
            const float* w = hh < G ? p.qnorm_w : p.knorm_w;
            float ss = 0.0f;
            for (int i = lane; i < hd; i += 32) ss += vec[i] * vec[i];
            ss = warp_sum(ss);
            const float scale = rms_scale(ss, hd, p.eps);
            __syncwarp();
            for (int i = lane; i < hd; i += 32) vec[i] = vec[i] * scale * w[i];
        }
        __syncthreads();
    }
    const bool inter = arch_interleaved(p.arch);
    for (int idx = tid; p.rope && idx < (G + 1) * half; idx += blockDim.x) {
        const int hh = idx / half, d = idx % half;
        float* vec = hh < G ? qs + hh * hd : ks;
        const int i0 = inter ? 2 * d : d;
        const int i1 = inter ? 2 * d + 1 : d + half;
        const float a = vec[i0], bb = vec[i1];
        vec[i0] = __fsub_rn(__fmul_rn(a, cs[d]), __fmul_rn(bb, sn[d]));
        vec[i1] = __fadd_rn(__fmul_rn(a, sn[d]), __fmul_rn(bb, cs[d]));
    }
    __syncthreads();

    float* kc = p.kcache + (int64_t)b * p.cache_bstride;
    float* vc = p.vcache + (int64_t)b * p.cache_bstride;
    if (pos >= p0 && pos < p1) {
        const float* vsrc = p.v + (int64_t)b * p.ldkv + (int64_t)hk * hd;
        for (int i = tid; i < hd; i += blockDim.x) {
            kc[(int64_t)pos * kvd + hk * hd + i] = ks[i];
            vc[(int64_t)pos * kvd + hk * hd + i] = vsrc[i];
        }
    }
    __syncthreads();

    // scores: one position per thread, its K row against up to 4 heads per
    // pass (q from shared memory, the same address for all lanes)
    for (int t = tid; t < n; t += blockDim.x) {
        const float4* kr = reinterpret_cast<const float4*>(kc + (int64_t)(p0 + t) * kvd + hk * hd);
        for (int h0 = 0; h0 < G; h0 += 4) {
            float s[4] = {0.0f, 0.0f, 0.0f, 0.0f};
            for (int i = 0; i < hd / 4; ++i) {
                const float4 kv = kr[i];
#pragma unroll
                for (int hh = 0; hh < 4; ++hh) {
                    if (h0 + hh < G) {
                        const float4 qv = reinterpret_cast<const float4*>(qs + (h0 + hh) * hd)[i];
                        s[hh] += qv.x * kv.x + qv.y * kv.y + qv.z * kv.z + qv.w * kv.w;
                    }
                }
            }
#pragma unroll
            for (int hh = 0; hh < 4; ++hh)
                if (h0 + hh < G) sc[(h0 + hh) * cap + t] = s[hh] * p.inv_scale;
        }
    }
    __syncthreads();
    // chunk-local softmax numerators
    for (int h = warp; h < G; h += 4) {
        float m = -INFINITY;
        for (int t = lane; t < n; t += 32) m = fmaxf(m, sc[h * cap + t]);
        m = warp_max(m);
        float l = 0.0f;
        for (int t = lane; t < n; t += 32) {
            const float e = n > 0 ? expf(sc[h * cap + t] - m) : 0.0f;
            sc[h * cap + t] = e;
            l += e;
        }
        l = warp_sum(l);
        if (lane == 0) { s_m[h] = m; s_l[h] = l; }
    }
    __syncthreads();
    for (int idx = tid; idx < G * hd; idx += blockDim.x) {
        const int h = idx / hd, i = idx % hd;
        const float* vr = vc + (int64_t)p0 * kvd + hk * hd + i;
        const float* sh = sc + h * cap;
        float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;   // four chains of positions in flight
        int t = 0;
        for (; t + 4 <= n; t += 4) {
            a0 += sh[t] * vr[(int64_t)t * kvd];
            a1 += sh[t + 1] * vr[(int64_t)(t + 1) * kvd];
            a2 += sh[t + 2] * vr[(int64_t)(t + 2) * kvd];
            a3 += sh[t + 3] * vr[(int64_t)(t + 3) * kvd];
        }
        for (; t < n; ++t) a0 += sh[t] * vr[(int64_t)t * kvd];
        __stcg(&pbase[((int64_t)h * p.nchunk + c) * stride + 2 + i], (a0 + a1) + (a2 + a3));
    }
    if (tid < G) {
        __stcg(&pbase[((int64_t)tid * p.nchunk + c) * stride + 0], n > 0 ? s_m[tid] : -INFINITY);
        __stcg(&pbase[((int64_t)tid * p.nchunk + c) * stride + 1], n > 0 ? s_l[tid] : 0.0f);
    }
    }
arrive:
    __syncthreads();   // the CTA's partials are written before thread 0's fence and arrival
    if (tid == 0) {
        __threadfence();
        s_last = (atomicAdd(ctr, 1) == p.nchunk - 1);
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();

    // combine the used chunks in order
    for (int h = warp; h < G; h += 4) {
        float M = -INFINITY;
        for (int k = lane; k < used; k += 32) M = fmaxf(M, __ldcg(&pbase[((int64_t)h * p.nchunk + k) * stride]));
        M = warp_max(M);
        float L = 0.0f;
        for (int k = lane; k < used; k += 32) {
            const float mk = __ldcg(&pbase[((int64_t)h * p.nchunk + k) * stride]);
            const float w = mk == -INFINITY ? 0.0f : expf(mk - M);
            wc[h * p.nchunk + k] = w;
            L += w * __ldcg(&pbase[((int64_t)h * p.nchunk + k) * stride + 1]);
        }
        L = warp_sum(L);
        if (lane == 0) s_l[h] = 1.0f / L;
    }
    __syncthreads();
    for (int idx = tid; idx < G * hd; idx += blockDim.x) {
        const int h = idx / hd, i = idx % hd;
        const float* src = pbase + (int64_t)h * p.nchunk * stride + 2 + i;
        const float* wh = wc + h * p.nchunk;
        float o = 0.0f;
        int k = 0;
        for (; k + 4 <= used; k += 4) {   // independent loads in flight
            const float v0 = __ldcg(src + (int64_t)k * stride), v1 = __ldcg(src + (int64_t)(k + 1) * stride);
            const float v2 = __ldcg(src + (int64_t)(k + 2) * stride), v3 = __ldcg(src + (int64_t)(k + 3) * stride);
            o += wh[k] * v0;
            o += wh[k + 1] * v1;
            o += wh[k + 2] * v2;
            o += wh[k + 3] * v3;
        }
        for (; k < used; ++k) o += wh[k] * __ldcg(src + (int64_t)k * stride);
        o *= s_l[h];
        qs[idx] = o;
        p.xb[(int64_t)b * p.ldxb + (int64_t)hk * G * hd + idx] = o;
    }
    __syncthreads();
    if (p.prep_out) {
        const int rec_bytes = prep_rec_bytes(p.batch);
        const int blk0 = hk * G * hd / 32;
        for (int kb = warp; kb < G * hd / 32; kb += 4)
            prep_emit_warp(p.prep_out + (size_t)(blk0 + kb) * rec_bytes, p.batch, b, qs[kb * 32 + lane]);
    }
    if (tid == 0) *ctr = 0;
}

}  // namespace

int attn_pick_nchunk(int n_kv, int batch, int seq_len) {
    // about two CTAs per SM for the whole batch, and at most 256 positions
    // per CTA at a full context (a CTA walks its positions one after another)
    int nc = std::max((2 * 148) / std::max(1, n_kv * batch), (seq_len + 255) / 256);
    nc = std::max(1, std::min(nc, 64));
    while (nc < 256 && (seq_len + nc - 1) / nc > 2048) nc *= 2;
    return nc;
}

size_t attn_part_floats(int batch, int n_heads, int nchunk, int hd) {
    return (size_t)batch * n_heads * nchunk * (hd + 2);
}

int attn_launch(const AttnParams& p, cudaStream_t stream, bool pdl) {
    BREW_CHECK(p.n_kv > 0 && p.n_heads % p.n_kv == 0, BREW_ERR_INVALID_ARG, "attention: heads %d kv %d", p.n_heads, p.n_kv);
    BREW_CHECK(p.hd % 32 == 0 && p.hd <= 512, BREW_ERR_INVALID_ARG, "attention: head size %d", p.hd);
    const int G = p.n_heads / p.n_kv;
    BREW_CHECK(G <= 16, BREW_ERR_INVALID_ARG, "attention: %d query heads per kv head", G);
    // positions one CTA may hold: the kernel uses max(ATTN_MIN_CHUNK, ceil(len / nchunk))
    const int cap = std::max(ATTN_MIN_CHUNK, (p.seq_len + p.nchunk - 1) / p.nchunk);
    const size_t smem = sizeof(float) * ((size_t)G * p.hd + p.hd + (size_t)G * cap + 32 + p.hd + (size_t)G * p.nchunk);
    BREW_CHECK(smem <= 200 * 1024, BREW_ERR_INVALID_ARG, "attention: %zu bytes of shared memory", smem);
    static std::mutex mu;
    static unsigned long long attr_set = 0;   // one bit per device
    {
        std::lock_guard<std::mutex> lk(mu);
        BREW_CUDA(smem_attr_per_device((const void*)attn_kernel, 200 * 1024, &attr_set));
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.n_kv, p.nchunk, p.batch);
    cfg.blockDim = dim3(128);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    BREW_CUDA(cudaLaunchKernelEx(&cfg, attn_kernel, p, cap));
    count_launch();
    return BREW_OK;
}

}  // namespace brew
