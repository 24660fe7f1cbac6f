// kqtc.cu — the K-quant matvec on tcgen05 (layouts and arithmetic in kqtc.cuh).
#include "brew_internal.cuh"
#include "kqtc.cuh"
#include "prep.cuh"
#include "tc_device.cuh"

namespace brew {
namespace {

__device__ __forceinline__ float kx_half(const uint8_t* p) {
    return half_bits_to_float((uint16_t)(p[0] | (p[1] << 8)));
}

// 6-bit scale and min of Q4_K sub-block s (GGML's get_scale_min_k4).
__device__ __forceinline__ void kx_scale_min(const uint8_t* sb, int s, int& sc, int& m) {
    if (s < 4) {
        sc = sb[s] & 63;
        m = sb[s + 4] & 63;
    } else {
        sc = (sb[s + 4] & 0xF) | ((sb[s - 4] >> 6) << 4);
        m = (sb[s + 4] >> 4) | ((sb[s] >> 6) << 4);
    }
}

// The 8 sub-block mins m_j of a Q4_K block (its 12 scale bytes at sb), one
// byte each: m_0 .. m_3 in x, m_4 .. m_7 in y.
__device__ __forceinline__ uint2 kx_mins(const uint8_t* sb) {
    uint32_t w[2] = {0u, 0u};
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        int sc, mj;
        kx_scale_min(sb, j, sc, mj);
        w[j >> 2] |= (uint32_t)mj << (8 * (j & 3));
    }
    return make_uint2(w[0], w[1]);
}

// Byte k of w as a float (exact: the bits of 2^23 + byte, minus 2^23).
__device__ __forceinline__ float kx_byte_f(uint32_t w, int k) {
    return __uint_as_float(0x4B000000u | ((w >> (8 * k)) & 255u)) - 8388608.0f;
}

// Q6_K expanded copy: one thread per (row, 32-element sub-block j of
// super-block sb).
__global__ void kx_pack_kernel(const uint8_t* w, int64_t rows, int K, uint8_t* base, int64_t pitch, int64_t row_off,
                               size_t f_off) {
    constexpr int SB = 210;
    const int KB = K / 32, KSB = K / 256;
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= rows * KB) return;
    const int64_t row = i / KB;
    const int kb = (int)(i % KB), sb = kb / 8, j = kb % 8;
    const uint8_t* blk = w + row * (int64_t)KSB * SB + (int64_t)sb * SB;
    const int64_t prow = row_off + row;
    uint32_t h[8], l[8];   // 32 bytes each
    const float d = kx_half(blk + 208);
    const int s_lo = (int8_t)blk[192 + 2 * j], s_hi = (int8_t)blk[192 + 2 * j + 1];
#pragma unroll
    for (int w4 = 0; w4 < 8; ++w4) {
        uint32_t hv = 0u, lv = 0u;
#pragma unroll
        for (int b = 0; b < 4; ++b) {
            const int k = 4 * w4 + b;
            const int r = 32 * j + k, hb = r / 128, rr = r % 128, grp = rr / 32, ll = rr % 32;
            const int lq = blk[64 * hb + (grp & 1) * 32 + ll];
            const int low = grp < 2 ? (lq & 15) : (lq >> 4);
            const int high = (blk[128 + 32 * hb + ll] >> (2 * grp)) & 3;
            const int v = (k < 16 ? s_lo : s_hi) * ((low | (high << 4)) - 32);   // [-4064, 4096]
            hv |= (uint32_t)((v >> 6) & 255) << (8 * b);
            lv |= (uint32_t)(v & 63) << (8 * b);
        }
        h[w4] = hv;
        l[w4] = lv;
    }
    uint8_t* hp = base;
    uint8_t* lp = base + (size_t)K * pitch;
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
        const int64_t o = ((int64_t)(2 * kb + hf) * pitch + prow) * 16;
        *reinterpret_cast<uint4*>(hp + o) = make_uint4(h[4 * hf], h[4 * hf + 1], h[4 * hf + 2], h[4 * hf + 3]);
        *reinterpret_cast<uint4*>(lp + o) = make_uint4(l[4 * hf], l[4 * hf + 1], l[4 * hf + 2], l[4 * hf + 3]);
    }
    if (j == 0) reinterpret_cast<float2*>(base + f_off)[(int64_t)sb * pitch + prow] = make_float2(d, 0.0f);
}

// Q4_K compact copy: one thread per 16-byte word of a block (9 per block):
// block (row, sb) of the GGUF matrix -> [sb][row_off + row] of the copy.
__global__ void kc_pack_kernel(const uint8_t* w, int64_t rows, int K, uint8_t* base, int64_t pitch, int64_t row_off) {
    const int KSB = K / 256;
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= rows * KSB * 9) return;
    const int64_t blk = i / 9;
    const int wd = (int)(i % 9);
    const int64_t row = blk / KSB;
    const int sb = (int)(blk % KSB);
    const uint4 v = reinterpret_cast<const uint4*>(w + blk * 144)[wd];
    reinterpret_cast<uint4*>(base + ((int64_t)sb * pitch + row_off + row) * 144)[wd] = v;
}

// One warp per (vector t < nvp, super-block): lane i holds elements
// 8i .. 8i + 7 (sub-block i / 4); vectors past nv are zero.
__global__ void kx_prep_kernel(const float* x, int ldx, int K, int nv, int nvp, uint8_t* rec) {
    const int lane = threadIdx.x & 31;
    const int64_t wid = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int KSB = K / 256;
    if (wid >= (int64_t)nvp * KSB) return;
    const int t = (int)(wid / KSB), sb = (int)(wid % KSB);
    float xs[8];
    if (t < nv) {
        const float4* p = reinterpret_cast<const float4*>(x + (int64_t)t * ldx + (int64_t)sb * 256 + 8 * lane);
        const float4 a = p[0], b = p[1];
        xs[0] = a.x; xs[1] = a.y; xs[2] = a.z; xs[3] = a.w;
        xs[4] = b.x; xs[5] = b.y; xs[6] = b.z; xs[7] = b.w;
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) xs[i] = 0.0f;
    }
    kx_emit_sb(rec, K, nvp, t, sb, xs);
}

// Shared memory of one stage (one super-block): the 8 sub-blocks' h and l
// tiles (128 rows x 32 k each: K-half 0 then K-half 1, 2 KB apart), then
// the records' 8 limb tiles.
constexpr int KX_AH = 0, KX_AL = 32768, KX_B = 65536;
constexpr int KX_STAGE = KX_B + 8 * 96 * 32;    // 90112
constexpr int KX_SMEM = 2 * KX_STAGE + 128;
constexpr int KX_EPI = 16;                      // epilogue warps: 4 per tensor-memory lane quadrant
constexpr int KX_THREADS = 64 + 32 * KX_EPI;    // loader warp, MMA warp, epilogue warps
constexpr int KX_TMEM_COLS = 512;               // two sets of the h, l accumulators: at 0, 128 and 256, 384
// Q4_K (compact stream): one expanded area (h, l at the offsets above), then
// two stages of records and two of raw block runs (128 rows x 144 bytes),
// then the barriers.
constexpr int KC_REC = 8 * 96 * 32;             // records of one super-block (up to 32 vectors)
constexpr int KC_REC0 = KX_B;
constexpr int KC_RAW = 128 * 144;
constexpr int KC_RAW0 = KC_REC0 + 2 * KC_REC;
constexpr int KC_BAR = KC_RAW0 + 2 * KC_RAW;
constexpr int KC_SMEM = KC_BAR + 128;

// Q4_K: expands item e (0 .. 511) of a raw run of 128 rows: row e % 128,
// sub-blocks 2 (e / 128) and 2 (e / 128) + 1, into the h / l tiles (the
// layout of the expanded planes: sub-block j at j 4096, K-half hk 2048
// further, row r 16 bytes each).
// Element value d (8 h + l) - dmin m_j with h = q (sc >> 3), l = q (sc & 7)
// (GGML's d sc q - dmin m), q the element's nibble.
__device__ __forceinline__ void kc_expand(uint8_t* xa, const uint8_t* raw, int e) {
    const int row = e & 127, pr = e >> 7;
    const uint8_t* blk = raw + row * 144;
    int sc[2], mn[2];
    kx_scale_min(blk + 4, 2 * pr, sc[0], mn[0]);
    kx_scale_min(blk + 4, 2 * pr + 1, sc[1], mn[1]);
    const uint4 qa = *reinterpret_cast<const uint4*>(blk + 16 + 32 * pr);
    const uint4 qb = *reinterpret_cast<const uint4*>(blk + 32 + 32 * pr);
    const uint32_t w[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
#pragma unroll
    for (int sub = 0; sub < 2; ++sub) {   // sub-block 2 pr: low nibbles; 2 pr + 1: high nibbles
        const uint32_t sh = (uint32_t)(sc[sub] >> 3), sl = (uint32_t)(sc[sub] & 7);
#pragma unroll
        for (int hk = 0; hk < 2; ++hk) {
            uint32_t hv[4], lv[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const uint32_t qv = (sub ? (w[4 * hk + u] >> 4) : w[4 * hk + u]) & 0x0F0F0F0Fu;
                hv[u] = qv * sh;   // bytewise: q s <= 105, no carry between the bytes
                lv[u] = qv * sl;
            }
            const int so = (2 * pr + sub) * 4096 + hk * 2048 + row * 16;
            *reinterpret_cast<uint4*>(xa + KX_AH + so) = make_uint4(hv[0], hv[1], hv[2], hv[3]);
            *reinterpret_cast<uint4*>(xa + KX_AL + so) = make_uint4(lv[0], lv[1], lv[2], lv[3]);
        }
    }
}

__device__ __forceinline__ bool kx_wait(uint64_t* bar, uint32_t parity, unsigned int* err, unsigned int code) {
    for (int i = 0; i < 32; ++i)
        if (mbar_try_wait(bar, parity)) return true;
    return mbar_wait_bounded(bar, parity, err, code);
}

// CTA = 128 rows (row0 + 128 blockIdx.x ..) x all vectors x the
// super-blocks of split blockIdx.y.  Per super-block:
//   warp 0      one lane bulk-copies the stage into one of 2 stages: Q4_K
//               the 128 rows' raw blocks (one 18 KB run) and the records;
//               Q6_K 33 copies (32 K-half runs of h and l, the records);
//   (Q4_K)      the epilogue warps expand the raw run into the h, l and min
//               tiles (one (row, sub-block pair) per thread) and each
//               thread keeps its readout row's (d, dmin); the expanded area
//               is single: the next expansion starts after the readout,
//               which waits for the MMAs;
//   warp 1      one thread issues, per sub-block j, the MMAs h_j x B_j and
//               l_j x B_j into the h and l accumulators of set i % 2 (two
//               sets, 256 tensor-memory columns apart), all onto the preset
//               magic value, and commits to the stage's "empty" and the
//               set's "full" barriers;
//   warps 2-17  (Q4_K) expand super-block i + 1 as soon as the MMAs of i
//               have read the expanded area, then read set i back (warp w:
//               lanes 32 (w % 4), a quarter of the columns), reset and
//               release it, and add s_v d (F h + l) to fp32 accumulators per
//               (vector, limb), and -dmin sum_j m_j X_j (the records' fp32
//               sub-block sums) to one per vector.
// The copies of the next super-block overlap the MMAs and the readout, and
// the MMAs of super-block i + 1 overlap the readout of i.
template <int TYPE, int NVG>
__global__ void __launch_bounds__(KX_THREADS, 1)
    kx_mma_kernel(const uint8_t* base, int64_t pitch, int64_t row0, int n, int K, size_t f_off,
                  const uint8_t* rec, int nv, int S, float* part, int* ctr, const float* bias, float* y, int ldy,
                  unsigned int* err) {
    constexpr bool Q4 = TYPE == BREW_TYPE_Q4_K;
    constexpr int NVP = 16 * NVG, NC = 3 * NVP;   // vectors and limb columns of the MMA
    constexpr int CW = NC / (KX_EPI / 4), TPW = CW / 3;   // columns and vectors per epilogue warp
    constexpr int NACC = 2;   // h, l
    extern __shared__ __align__(1024) uint8_t smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + (Q4 ? KC_BAR : 2 * KX_STAGE));
    uint64_t* empty = full + 2;
    uint64_t* tfull = empty + 2;     // [2] per accumulator set
    uint64_t* tempty = tfull + 2;    // [2]
    uint64_t* xready = tempty + 2;   // Q4_K: the expanded tiles are in place
    uint32_t* tslot = reinterpret_cast<uint32_t*>(xready + 1);
    __shared__ int s_last;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int KSB = K / 256, split = blockIdx.y;
    const int sb0 = (int)((int64_t)split * KSB / S), sb1 = (int)((int64_t)(split + 1) * KSB / S);
    const int64_t r0 = row0 + (int64_t)blockIdx.x * KX_TM;   // the CTA's first row in the family
    const int rec_tile = 8 * NC * 32;
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tslot)),
                     "r"(KX_TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (tid == 0) {
        for (int i = 0; i < 2; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], Q4 ? 1 + KX_EPI : 1);   // Q4_K: the MMAs' commit and every expanding warp
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&tfull[i], 1);
            mbar_init(&tempty[i], KX_EPI);
        }
        mbar_init(xready, KX_EPI);
        fence_mbar_init();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;
    if (warp == 0) {
        // ---------------------------------- loader ----------------------------------
        if (lane == 0) {
            const uint64_t pol = l2_evict_first_policy();
            const uint8_t* hp = base;
            const uint8_t* lp = base + (size_t)K * pitch;
            const uint32_t bbytes = 8 * NC * 32;   // the 8 limb tiles
            const uint32_t bytes = 16 * 4096 + bbytes;   // Q6_K: the h and l tiles and the records
            int it = 0;
            for (int sb = sb0; sb < sb1; ++sb, ++it) {
                const int st = it & 1;
                if (it >= 2 && !kx_wait(&empty[st], ((it >> 1) - 1) & 1, err, BREW_DEVERR_TIMEOUT_EMPTY)) break;
                if (Q4) {   // the raw blocks of rows r0 .. r0 + 127 of super-block sb: one contiguous run
                    mbar_arrive_expect_tx(&full[st], KC_RAW + bbytes);
                    bulk_g2s_hint(smem + KC_RAW0 + st * KC_RAW, base + ((int64_t)sb * pitch + r0) * 144, KC_RAW,
                                  &full[st], pol);
                    bulk_g2s(smem + KC_REC0 + st * KC_REC, rec + (int64_t)sb * rec_tile, bbytes, &full[st]);
                    continue;
                }
                uint8_t* s0 = smem + st * KX_STAGE;
                mbar_arrive_expect_tx(&full[st], bytes);
                for (int hk = 0; hk < 16; ++hk) {   // K-half hk of the super-block: sub-block hk / 2
                    const int64_t o = ((int64_t)(16 * sb + hk) * pitch + r0) * 16;
                    const int so = (hk >> 1) * 4096 + (hk & 1) * 2048;
                    bulk_g2s_hint(s0 + KX_AH + so, hp + o, 2048, &full[st], pol);
                    bulk_g2s_hint(s0 + KX_AL + so, lp + o, 2048, &full[st], pol);
                }
                bulk_g2s(s0 + KX_B, rec + (int64_t)sb * rec_tile, bbytes, &full[st]);
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        // ------------------------------------ MMA ------------------------------------
        if (lane == 0) {
            constexpr uint32_t idesc = umma_idesc_s8(KX_TM, NC);
            int it = 0;
            for (int sb = sb0; sb < sb1; ++sb, ++it) {
                const int st = it & 1;
                if (!kx_wait(&full[st], (it >> 1) & 1, err, BREW_DEVERR_TIMEOUT_FULL)) break;
                if (Q4 && !kx_wait(xready, it & 1, err, BREW_DEVERR_TIMEOUT_FULL)) break;
                const int b = it & 1;
                if (!kx_wait(&tempty[b], (it >> 1) & 1, err, BREW_DEVERR_TIMEOUT_EMPTY)) break;
                const uint32_t tb = tmem + 256 * b;
                tc_fence_after();
                // Q4_K: the expanded tiles at 0, the stage's records apart
                const uint32_t s0 = smem_u32(smem + (Q4 ? 0 : st * KX_STAGE));
                const uint32_t sr = Q4 ? smem_u32(smem + KC_REC0 + st * KC_REC) : s0 + KX_B;
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const uint64_t bd = umma_desc_k(sr + j * NC * 32, 128, 256);
                    umma_s8(tb, umma_desc_k(s0 + KX_AH + j * 4096, 2048, 128), bd, idesc, 1u);
                    umma_s8(tb + 128, umma_desc_k(s0 + KX_AL + j * 4096, 2048, 128), bd, idesc, 1u);
                }
                umma_commit(&empty[st]);
                umma_commit(&tfull[b]);
            }
        }
        __syncwarp();
    } else {
        // ---------------------------------- epilogue ----------------------------------
        const int q = warp & 3, hh = (warp - 2) >> 2;
        const int lrow = (int)(r0 - row0) + 32 * q + lane;   // row within the launch
        const int64_t frow = r0 + 32 * q + lane;             // row within the family (< pitch)
        const uint32_t tq = tmem + ((uint32_t)(32 * q) << 16) + CW * hh;
#pragma unroll
        for (int b = 0; b < 2; ++b)
#pragma unroll
            for (int a = 0; a < NACC; ++a) {   // exactly this warp's CW columns (a multiple of 4)
#pragma unroll
                for (int c = 0; c + 8 <= CW; c += 8) tmem_st8_const(tq + 256 * b + 128 * a + c, TC_MAGIC);
                if (CW % 8) tmem_st4_const(tq + 256 * b + 128 * a + CW - 4, TC_MAGIC);
            }
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
            mbar_arrive(&tempty[0]);
            mbar_arrive(&tempty[1]);
        }
        uint64_t acc[TPW / 2][3];   // vector pairs x limbs (hi, mid, lo; Q4_K's min term joins lo)
#pragma unroll
        for (int p = 0; p < TPW / 2; ++p) acc[p][0] = acc[p][1] = acc[p][2] = 0ull;
        const uint64_t negc = f2_packf(-TC_MAGIC_F, -TC_MAGIC_F);
        const uint64_t kF = Q4 ? f2_packf(8.0f, 8.0f) : f2_packf(64.0f, 64.0f);
        const uint64_t k256 = f2_packf(256.0f, 256.0f), k65536 = f2_packf(65536.0f, 65536.0f);
        const float2* fpl = reinterpret_cast<const float2*>(base + f_off);
        const float* scl = reinterpret_cast<const float*>(rec + (int64_t)KSB * rec_tile);
        const float* xsum = scl + (int64_t)KSB * NVP;   // [sb][NVP][8] fp32 sub-block sums
        float2 fr = (!Q4 && sb0 < sb1) ? __ldg(fpl + (int64_t)sb0 * pitch + frow) : make_float2(0.0f, 0.0f);
        // the vectors' scales of a super-block, loaded one super-block ahead
        // (their L2 round trip overlaps the previous readout)
        float4 svn[TPW / 4];
        auto load_scales = [&](int sbl) {
#pragma unroll
            for (int g = 0; g < TPW / 4; ++g)
                svn[g] = __ldg(reinterpret_cast<const float4*>(scl + (int64_t)sbl * NVP + TPW * hh) + g);
        };
        // this warp's vectors' sub-block sums of super-block sbl into L1
        // (TPW x 8 fp32: 256 bytes), read by the readout one super-block on
        auto prefetch_sums = [&](int sbl) {
            if (lane < TPW / 4)
                asm volatile("prefetch.global.L1 [%0];" ::"l"(xsum + ((int64_t)sbl * NVP + TPW * hh) * 8 + 32 * lane));
        };
        // Q4_K: expand super-block sb0 + i of its raw run into the expanded
        // area, and keep the readout row's (d, dmin) and mins
        float2 frn = make_float2(0.0f, 0.0f);
        uint2 mnn = make_uint2(0u, 0u);
        auto expand = [&](int i) -> bool {
            const int st = i & 1;
            bool okx = kx_wait(&full[st], (i >> 1) & 1, err, BREW_DEVERR_TIMEOUT_FULL);
            okx = __all_sync(0xffffffffu, okx);
            if (!okx) return false;
            const uint8_t* raw = smem + KC_RAW0 + st * KC_RAW;
            kc_expand(smem, raw, tid - 64);
            const uint8_t* rb = raw + (32 * q + lane) * 144;
            frn = make_float2(kx_half(rb), kx_half(rb + 2));
            mnn = kx_mins(rb + 4);
            fence_proxy_async();   // the generic-proxy stores, before the tensor cores read them
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(xready);
                mbar_arrive(&empty[st]);   // the raw run is consumed
            }
            return true;
        };
        if (sb0 < sb1) {
            load_scales(sb0);
            if (Q4) prefetch_sums(sb0);
        }
        bool alive = !(Q4 && sb0 < sb1) || expand(0);
        int it = 0;
        for (int sb = sb0; alive && sb < sb1; ++sb, ++it) {
            const int b = it & 1;
            bool ok = kx_wait(&tfull[b], (it >> 1) & 1, err, BREW_DEVERR_TIMEOUT_FULL);
            ok = __all_sync(0xffffffffu, ok);   // tcgen05.ld / st are warp-collective
            if (!ok) break;
            tc_fence_after();
            uint2 mnb = make_uint2(0u, 0u);
            if (Q4) {   // this super-block's factors; the MMAs are done with the expanded area: the next one
                fr = frn;
                mnb = mnn;
                if (sb + 1 < sb1 && !expand(it + 1)) break;
                if (sb + 1 < sb1) prefetch_sums(sb + 1);
            }
            float sv[TPW];
#pragma unroll
            for (int g = 0; g < TPW / 4; ++g) {
                sv[4 * g] = svn[g].x;
                sv[4 * g + 1] = svn[g].y;
                sv[4 * g + 2] = svn[g].z;
                sv[4 * g + 3] = svn[g].w;
            }
            if (sb + 1 < sb1) load_scales(sb + 1);
            const uint64_t d2 = f2_packf(fr.x, fr.x);
            const float ndm = -fr.y;
            if (!Q4 && sb + 1 < sb1) fr = __ldg(fpl + (int64_t)(sb + 1) * pitch + frow);
            const float* xs = xsum + ((int64_t)sb * NVP + TPW * hh) * 8;
#pragma unroll
            for (int e = 0; e < CW / 12; ++e) {   // 12 columns (2 vector pairs) at a time
                const uint32_t ta = tq + 256 * b + 12 * e;
                uint32_t v[NACC][12];
#pragma unroll
                for (int a = 0; a < NACC; ++a) {
                    tmem_ld8(ta + 128 * a, v[a]);
                    tmem_ld4(ta + 128 * a + 8, v[a] + 8);
                }
                tmem_ld_wait();
#pragma unroll
                for (int a = 0; a < NACC; ++a) {
                    tmem_st8_const(ta + 128 * a, TC_MAGIC);
                    tmem_st4_const(ta + 128 * a + 8, TC_MAGIC);
                }
#pragma unroll
                for (int pp = 0; pp < 2; ++pp) {
                    const int p = 2 * e + pp;
                    const uint64_t s2 = f2_packf(sv[2 * p], sv[2 * p + 1]);
#pragma unroll
                    for (int l = 0; l < 3; ++l) {
                        const int c = 6 * pp + 2 * l;
                        const uint64_t H = f2_add(f2_pack(v[0][c], v[0][c + 1]), negc);
                        const uint64_t L = f2_add(f2_pack(v[1][c], v[1][c + 1]), negc);
                        const uint64_t val = f2_fma(H, kF, L);   // F h + l
                        acc[p][l] = f2_fma(s2, f2_mul(d2, val), acc[p][l]);
                    }
                }
            }
            tmem_st_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[b]);
            if (Q4) {   // - dmin sum_j m_j X_j per vector, into the lo accumulators
                float mn[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) mn[j] = kx_byte_f(j < 4 ? mnb.x : mnb.y, j & 3);
#pragma unroll
                for (int p = 0; p < TPW / 2; ++p) {
                    float mx[2];
#pragma unroll
                    for (int u = 0; u < 2; ++u) {
                        const float4 x0 = __ldg(reinterpret_cast<const float4*>(xs + 8 * (2 * p + u)));
                        const float4 x1 = __ldg(reinterpret_cast<const float4*>(xs + 8 * (2 * p + u)) + 1);
                        float t = mn[0] * x0.x;
                        t = fmaf(mn[1], x0.y, t);
                        t = fmaf(mn[2], x0.z, t);
                        t = fmaf(mn[3], x0.w, t);
                        t = fmaf(mn[4], x1.x, t);
                        t = fmaf(mn[5], x1.y, t);
                        t = fmaf(mn[6], x1.z, t);
                        mx[u] = fmaf(mn[7], x1.w, t);
                    }
                    acc[p][2] = f2_fma(f2_packf(ndm, ndm), f2_packf(mx[0], mx[1]), acc[p][2]);
                }
            }
        }
        // limbs meet: (lo + mid 2^8) + hi 2^16
        const int64_t npad = (int64_t)gridDim.x * KX_TM;
#pragma unroll
        for (int p = 0; p < TPW / 2; ++p) {
            const uint64_t r = f2_fma(acc[p][0], k65536, f2_fma(acc[p][1], k256, acc[p][2]));
            const float a0 = __uint_as_float((uint32_t)r), a1 = __uint_as_float((uint32_t)(r >> 32));
            const int tk = TPW * hh + 2 * p;
            if (lrow < n) {
                if (S == 1) {
                    const float bv = bias ? __ldg(bias + frow) : 0.0f;
                    if (tk < nv) y[(int64_t)tk * ldy + lrow] = bias ? a0 + bv : a0;
                    if (tk + 1 < nv) y[(int64_t)(tk + 1) * ldy + lrow] = bias ? a1 + bv : a1;
                } else {
                    if (tk < nv) part[((int64_t)split * nv + tk) * npad + lrow] = a0;
                    if (tk + 1 < nv) part[((int64_t)split * nv + tk + 1) * npad + lrow] = a1;
                }
            }
        }
        if (S > 1) {   // the last CTA of this row group adds the splits in split order
            __threadfence();
            asm volatile("bar.sync 1, %0;" ::"n"(32 * KX_EPI) : "memory");
            if (tid == 64) {
                const int old = atomicAdd(&ctr[blockIdx.x], 1);
                s_last = old == S - 1;
                if (s_last) ctr[blockIdx.x] = 0;   // every split has arrived: ready for the next launch
            }
            asm volatile("bar.sync 1, %0;" ::"n"(32 * KX_EPI) : "memory");
            if (s_last) {
                __threadfence();
                const int rbase = (int)(r0 - row0);
                for (int i = tid - 64; i < nv * KX_TM; i += 32 * KX_EPI) {
                    const int tk = i / KX_TM, lr = rbase + i % KX_TM;
                    if (lr >= n) continue;
                    float sum = 0.0f;
                    for (int sp = 0; sp < S; ++sp) sum += __ldcg(part + ((int64_t)sp * nv + tk) * npad + lr);
                    y[(int64_t)tk * ldy + lr] = bias ? sum + __ldg(bias + row0 + lr) : sum;
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(KX_TMEM_COLS)
                     : "memory");
    }
}

template <int TYPE, int NVG>
int kx_launch_t(const uint8_t* base, int64_t N, int64_t row0, int n, int K, const uint8_t* rec, int nv, int S,
                float* part, int* ctr, const float* bias, float* y, int ldy, unsigned int* err, cudaStream_t stream) {
    static uint64_t attr_devs = 0;   // devices whose attribute is set
    constexpr int SMEM = TYPE == BREW_TYPE_Q4_K ? KC_SMEM : KX_SMEM;
    int dev = 0;
    BREW_CUDA(cudaGetDevice(&dev));
    if (dev < 64 && !(attr_devs >> dev & 1)) {
        BREW_CUDA(cudaFuncSetAttribute(kx_mma_kernel<TYPE, NVG>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM));
        attr_devs |= 1ull << dev;
    }
    const dim3 grid((unsigned)((n + KX_TM - 1) / KX_TM), (unsigned)S);
    kx_mma_kernel<TYPE, NVG><<<grid, KX_THREADS, SMEM, stream>>>(base, kx_pitch(N), row0, n, K,
                                                                    kx_f_off(N, K), rec, nv, S, part, ctr, bias,
                                                                    y, ldy, err);
    BREW_CUDA(cudaGetLastError());
    count_launch();
    return BREW_OK;
}

}  // namespace

int kq_splits(int64_t K, int64_t n_basis) {
    // as many splits as keep the family's 128-row groups within one wave of
    // one CTA per SM of a B200 (148 SMs), at least two super-blocks each
    constexpr int64_t wave = 148;
    const int64_t groups = std::max<int64_t>(1, (n_basis + KX_TM - 1) / KX_TM), ksb = K / 256;
    int64_t s = wave / groups;
    s = std::min<int64_t>(s, std::max<int64_t>(1, ksb / 2));
    return (int)std::max<int64_t>(1, s);
}

int kx_pack_launch(int type, const uint8_t* w, int64_t rows, int K, uint8_t* base, int64_t N, int64_t row_off,
                   cudaStream_t stream) {
    BREW_CHECK((type == BREW_TYPE_Q4_K || type == BREW_TYPE_Q6_K) && K % 256 == 0 && K > 0 && rows > 0 &&
                   row_off >= 0 && row_off + rows <= N,
               BREW_ERR_INVALID_ARG, "K-quant expand: type %d rows=%lld K=%d", type, (long long)rows, K);
    if (type == BREW_TYPE_Q4_K) {   // the compact copy: blocks reordered super-block-major
        BREW_CHECK((reinterpret_cast<uintptr_t>(w) & 15) == 0, BREW_ERR_INVALID_ARG,
                   "K-quant copy: Q4_K rows must start 16-byte aligned");
        const int64_t words = rows * (K / 256) * 9;
        kc_pack_kernel<<<(unsigned)((words + 255) / 256), 256, 0, stream>>>(w, rows, K, base, kx_pitch(N), row_off);
        BREW_CUDA(cudaGetLastError());
        count_launch();
        return BREW_OK;
    }
    const int64_t cnt = rows * (K / 32);
    const unsigned blocks = (unsigned)((cnt + 255) / 256);
    kx_pack_kernel<<<blocks, 256, 0, stream>>>(w, rows, K, base, kx_pitch(N), row_off, kx_f_off(N, K));
    BREW_CUDA(cudaGetLastError());
    count_launch();
    return BREW_OK;
}

int kx_prep_launch(const float* x, int ldx, int K, int nv, uint8_t* rec, cudaStream_t stream) {
    BREW_CHECK(nv >= 1 && nv <= KX_MAX_VECTORS && K % 256 == 0 && K > 0 && ldx % 4 == 0 &&
                   (reinterpret_cast<uintptr_t>(x) & 15) == 0,
               BREW_ERR_INVALID_ARG, "K-quant records: nv=%d K=%d ldx=%d (x 16-byte aligned)", nv, K, ldx);
    const int nvp = (nv + 15) / 16 * 16;
    const int64_t warps = (int64_t)nvp * (K / 256);
    kx_prep_kernel<<<(unsigned)((warps * 32 + 255) / 256), 256, 0, stream>>>(x, ldx, K, nv, nvp, rec);
    BREW_CUDA(cudaGetLastError());
    count_launch();
    return BREW_OK;
}

int kx_mma_launch(int type, const uint8_t* base, int64_t N, int64_t row0, int n, int K, const uint8_t* rec, int nv,
                  int splits, float* part, int* ctr, const float* bias, float* y, int ldy, unsigned int* err,
                  cudaStream_t stream) {
    BREW_CHECK(nv >= 1 && nv <= KX_MAX_VECTORS && K % 256 == 0 && K > 0 && n > 0 && row0 >= 0 && row0 + n <= N &&
                   splits >= 1 && splits <= K / 256 && (splits == 1 || (part && ctr)),
               BREW_ERR_INVALID_ARG, "K-quant MMA matvec: nv=%d n=%d K=%d splits=%d", nv, n, K, splits);
    BREW_CHECK(type == BREW_TYPE_Q4_K || type == BREW_TYPE_Q6_K, BREW_ERR_INVALID_ARG, "K-quant MMA matvec: type %d",
               type);
    const bool q4 = type == BREW_TYPE_Q4_K;
    if (nv <= 16)
        return q4 ? kx_launch_t<BREW_TYPE_Q4_K, 1>(base, N, row0, n, K, rec, nv, splits, part, ctr, bias, y, ldy, err, stream)
                  : kx_launch_t<BREW_TYPE_Q6_K, 1>(base, N, row0, n, K, rec, nv, splits, part, ctr, bias, y, ldy, err, stream);
    return q4 ? kx_launch_t<BREW_TYPE_Q4_K, 2>(base, N, row0, n, K, rec, nv, splits, part, ctr, bias, y, ldy, err, stream)
              : kx_launch_t<BREW_TYPE_Q6_K, 2>(base, N, row0, n, K, rec, nv, splits, part, ctr, bias, y, ldy, err, stream);
}

}  // namespace brew
