// kqtc.cuh — the K-quant matvec of the forward (Q4_K / Q6_K matrices, the
// 7B config) on the 5th-generation tensor cores: tcgen05.mma kind::i8 with
// the accumulators in tensor memory, 1..32 vectors per launch.
//
// Weights (Q4_K): a compact copy of each matrix (or row family of N rows),
// the GGUF 144-byte blocks unchanged but ordered super-block-major,
//   [K/256][P][144]  (P = N + 128 rows, the last 128 zero),
// so the 128 rows a CTA multiplies for one super-block are one contiguous
// 18,432-byte run: one bulk copy per stage, 0.5625 bytes per weight as in
// the file.  The CTA expands the run in shared memory into the two int8
// limb planes below (the epilogue warps, just before the MMA).
// Weights (Q6_K): an expanded copy in HBM (its 210-byte blocks are only
// 2-byte aligned, which rules out bulk copies of the rows).
// Expanded planes: every element's integer factor carries its sub-block
// scale, split into two int8 limbs, so that a whole 256-element
// super-block is summed in integers by the MMA and its fp32 factors are
// applied once:
//   Q4_K  sc * q = 8 h + l,  h = q (sc >> 3), l = q (sc & 7)  (0..105),
//         and the min term sum_j m_j X_j (X_j the sub-block sum of x) on
//         the CUDA cores from the records' fp32 sums, so that the two
//         tensor-memory accumulators (h, l) fit twice in the 512 columns;
//         element value d (8 h + l) - dmin m_j  (GGML: d sc q - dmin m);
//   Q6_K  sc * (q - 32) = 64 h + l,  h in [-64, 63], l in [0, 63];
//         element value d (64 h + l)  (GGML: d sc (q - 32)).
// Expanded planes of one matrix (or row family) of N rows, pitch P = N + 128
// rows (the last 128 rows zero, so a 128-row box never leaves the buffer;
// in HBM for Q6_K; Q4_K's h and l tiles are built in shared memory for one
// super-block of 128 rows at a time, and its d, dmin and m_j read from the
// raw blocks):
//   h, l  [K/16][P][16]  int8: the 16-element K-halves of every row, row
//                         after row, so the 128 rows of a CTA's K-half are
//                         one contiguous 2 KB run (an MMA operand's core
//                         matrices: 8 rows x 16 B);
//   f     [K/256][P]     float2 (d, 0) (Q6_K).
//
// Activations: per vector and super-block, 24-bit fixed point relative to
// the super-block's max|x|, split into limbs hi / mid / lo (the prep.cuh
// split).  Records of a launch ([K/256] super-blocks, then the scales):
//   per super-block: 8 limb tiles (one per sub-block: NC = 48 per 16
//   vectors columns x 32 k, K-major core-matrix layout tc_tile_off, column
//   6 (t / 2) + 2 l + (t % 2) for vector t, limb l);
//   scales [K/256][16 ceil(nv / 16)] fp32 (vectors past nv: zero);
//   sub-block sums [K/256][16 ceil(nv / 16)][8] fp32: the sum of the
//   vector's 32 limb-split elements of sub-block j, scale applied.
// Every integer sum of a super-block stays below 2^22 in magnitude, so the
// tensor-memory cells, preset to the bits of 1.5 * 2^23, read back as
// exact floats.
#pragma once

#include "brew_common.cuh"
#include "prep.cuh"
#include "tc_device.cuh"

namespace brew {

constexpr int KX_TM = 128;            // rows per CTA
constexpr int KX_MAX_VECTORS = 32;    // per launch

inline int64_t kx_pitch(int64_t N) { return N + 128; }
inline size_t kx_plane_bytes(int64_t N, int64_t K) { return (size_t)K * (size_t)kx_pitch(N); }   // h or l
inline size_t kx_f_off(int64_t N, int64_t K) { return 2 * kx_plane_bytes(N, K); }   // Q6_K
// Bytes of the weight copy of an N x K matrix (or row family): compact
// (Q4_K) or expanded (Q6_K).
inline size_t kx_bytes(int type, int64_t N, int64_t K) {
    if (type == BREW_TYPE_Q4_K) return (size_t)(K / 256) * kx_pitch(N) * 144;
    return kx_f_off(N, K) + (size_t)(K / 256) * kx_pitch(N) * 8;
}
// Bytes of the x records of nv vectors of K elements (tiles, then scales).
inline size_t kx_rec_tile_bytes(int nv) { return (size_t)8 * 48 * ((nv + 15) / 16) * 32; }   // per super-block
inline size_t kx_rec_bytes(int nv, int64_t K) {
    return (size_t)(K / 256) * (kx_rec_tile_bytes(nv) + 4 * 9 * 16 * (size_t)((nv + 15) / 16));
}

// Split of the super-blocks over CTAs for a matrix whose row family has
// n_basis rows: a function of the full (unsharded) shape only, so that a
// row is summed in the same order whatever share of the rows a launch has
// (tensor-parallel ranks reproduce the one-GPU outputs bit for bit).
int kq_splits(int64_t K, int64_t n_basis);

// Rows [0, rows) of GGUF matrix w (rows x K) -> rows [row_off, row_off + rows)
// of the weight copy `base` (compact or expanded, kx_bytes) of a family of
// N rows (zeroed beforehand).
int kx_pack_launch(int type, const uint8_t* w, int64_t rows, int K, uint8_t* base, int64_t N, int64_t row_off,
                   cudaStream_t stream);
// x [nv][ldx] (nv <= 32) -> records.
int kx_prep_launch(const float* x, int ldx, int K, int nv, uint8_t* rec, cudaStream_t stream);
// y[v][i] = sum_k W[row0 + i][k] x_v[k] (+ bias[row0 + i], the bias indexed
// by family row, when given), i < n, for the expanded copy `base` of a
// family of N rows; `splits` as kq_splits; splits > 1 needs `part`
// (splits x 32 x ceil(n / 128) x 128 floats) and `ctr` (ceil(n / 128)
// ints, zero on entry, left zero).
int kx_mma_launch(int type, const uint8_t* base, int64_t N, int64_t row0, int n, int K, const uint8_t* rec, int nv,
                  int splits, float* part, int* ctr, const float* bias, float* y, int ldy, unsigned int* err,
                  cudaStream_t stream);

#ifdef __CUDACC__

__device__ __forceinline__ uint64_t kx_pack8(const int (&v)[8]) {
    uint32_t lo = 0u, hi = 0u;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        lo |= (uint32_t)(v[i] & 255) << (8 * i);
        hi |= (uint32_t)(v[4 + i] & 255) << (8 * i);
    }
    return (uint64_t)lo | ((uint64_t)hi << 32);
}

// Writes the record entries of vector t (< nvp, the launch's vectors
// rounded up to 16) for super-block sb; called by a whole warp, lane i
// holding elements 8i .. 8i + 7 of the super-block in xs.
__device__ __forceinline__ void kx_emit_sb(uint8_t* rec, int K, int nvp, int t, int sb, const float (&xs)[8]) {
    const int lane = threadIdx.x & 31;
    const int KSB = K / 256, NC = 3 * nvp;
    float am = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) am = fmaxf(am, fabsf(xs[i]));
    am = warp_max(am);
    const float inv = prep_block_inv(am);
    int lim[3][8];
    int sum[3] = {0, 0, 0};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int q = __float2int_rn(xs[i] * inv);
        const int lo = ((q + 128) & 255) - 128;
        const int q1 = (q - lo) >> 8;
        const int mid = ((q1 + 128) & 255) - 128;
        lim[0][i] = (q1 - mid) >> 8;
        lim[1][i] = mid;
        lim[2][i] = lo;
        sum[0] += lim[0][i];
        sum[1] += mid;
        sum[2] += lo;
    }
    uint8_t* r = rec + (int64_t)sb * (8 * NC * 32);
    const int j = lane >> 2, k0 = 8 * (lane & 3);
    const int c0 = 6 * (t >> 1) + (t & 1);   // limb l: column c0 + 2 l
    uint8_t* tile = r + j * NC * 32;
#pragma unroll
    for (int l = 0; l < 3; ++l) *reinterpret_cast<uint64_t*>(tile + tc_tile_off(c0 + 2 * l, k0)) = kx_pack8(lim[l]);
#pragma unroll
    for (int o = 1; o < 4; o <<= 1)
#pragma unroll
        for (int l = 0; l < 3; ++l) sum[l] += __shfl_xor_sync(0xffffffffu, sum[l], o);
    if ((lane & 3) == 0) {
        // the fp32 sub-block sum: the limbs' sums meet exactly in an int
        // (|.| < 2^28), then one rounding to fp32 and the scale
        const int st = sum[0] * 65536 + sum[1] * 256 + sum[2];
        float* xsum = reinterpret_cast<float*>(rec + (int64_t)KSB * 8 * NC * 32) + (int64_t)KSB * nvp;
        xsum[((int64_t)sb * nvp + t) * 8 + j] = (float)st * prep_block_scale(am);
    }
    if (lane == 0) reinterpret_cast<float*>(rec + (int64_t)KSB * 8 * NC * 32)[(int64_t)sb * nvp + t] = prep_block_scale(am);
}

#endif  // __CUDACC__

}  // namespace brew
