// kqmma.cuh — the K-quant matvec of the forward of models with Q4_K / Q6_K
// matrices (the 7B config), on the int8 tensor cores, for 1..32 vectors.
//
// Weights.  A K-quant matrix is repacked once into 16-row tiles; a tile's
// 256-element super-blocks are contiguous ([tiles][K/256][kq_sb_bytes]).
// One tile-superblock holds
//   Q4_K  2432 B:  8 x 256 B  the 32 quants q in [0, 15] of each 32-element
//                             sub-block j, as nibbles in the MMA A-fragment
//                             order (lane (g, t): 8 bytes, low nibbles
//                             k = 4t.., high nibbles k = 16 + 4t.., rows g
//                             and g + 8);
//                 8 x 32 B    per sub-block j and lane group g the bytes
//                             (sc_g, m_g, sc_g+8, m_g+8), GGML's 6-bit
//                             scale and min (get_scale_min_k4);
//                 128 B       per g the floats (d_g, dmin_g, d_g+8, dmin_g+8);
//   Q6_K  4416 B:  8 x 512 B  the quants q - 32 in [-32, 31] as int8 in the
//                             fragment order (16 bytes per lane: rows g,
//                             g + 8, halves k < 16 and k >= 16);
//                 8 x 32 B    per sub-block j and g the int8 scales of its
//                             two 16-element halves (lo_g, hi_g, lo_g+8, hi_g+8);
//                 64 B        per g the floats (d_g, d_g+8).
// Rows past N in the last tile are zero.
//
// Activations.  Per vector and super-block, x is a 24-bit fixed-point
// number relative to the super-block's max|x| (v = rint(x * 8290000 / max),
// split into balanced bytes v = hi 2^16 + mid 2^8 + lo), so that the integer
// products of a whole super-block can be summed exactly before any scale is
// applied.  The record of 16 vectors for one super-block (kq_rec_bytes) is
//   [0, 12288)      per sub-block j (1536 B): limb rows 3 v + l (hi, mid,
//                   lo) of 32 bytes; for odd v the two 16-byte halves are
//                   swapped (so that the B-fragment loads of the two vectors
//                   of an n8 tile hit different shared-memory banks);
//   [12288, 13056)  per limb row 16 bytes: the sub-block sums
//                   X_j = sum_i limb_i split as X_j = 256 Xh_j + Xl_j
//                   (Xl_0..7, then Xh_0..7), the B operand of the Q4_K
//                   min term;
//   [13056, 13120)  the 16 vectors' scales max / 8290000.
// Vectors past nv are zero.
//
// Arithmetic, per super-block and output (row, vector, limb):
//   Q4_K  d * sum_j sc_j * sum_k(q * limb) - dmin * sum_j m_j * X_j
//   Q6_K  d * sum_h sc_h * sum_k(q * limb)
// with every sum over integers (int32, exact), then times the vector's
// scale and accumulated in fp32; the limbs meet at the end as
// (lo + mid 2^8) + hi 2^16.  This is the reference's per-element
// d * sc * q - dmin * m (Q4_K) and d * sc * q (Q6_K) products summed in
// another order.
#pragma once

#include "brew_common.cuh"

namespace brew {

constexpr int KQ_MAX_VECTORS = 32;   // per launch
constexpr int KQ_REC = 13120;        // x record of 16 vectors and one super-block

__host__ __device__ constexpr int kq_sb_bytes(int type) { return type == BREW_TYPE_Q4_K ? 2432 : 4416; }
// Bytes of one 16-row tile of a K-column matrix.
inline size_t kq_tile_bytes(int type, int64_t K) { return (size_t)(K / 256) * (size_t)kq_sb_bytes(type); }
// Bytes of the repacked copy of an N x K matrix (N rounded up to 16 rows).
inline size_t kq_packed_bytes(int type, int64_t N, int64_t K) { return (size_t)((N + 15) / 16) * kq_tile_bytes(type, K); }
// Bytes of the x records of nv vectors of K elements.
inline size_t kq_rec_bytes(int nv, int64_t K) { return (size_t)((nv + 15) / 16) * (size_t)(K / 256) * KQ_REC; }

// Split of the super-blocks over CTAs for a matrix whose row family has
// n_basis rows: a function of the full (unsharded) shape only, so that a
// row is summed in the same order whatever share of the rows a launch has
// (tensor-parallel ranks reproduce the one-GPU outputs bit for bit).
int kq_splits(int64_t K, int64_t n_basis);
// fp32 scratch of a launch with `splits` > 1 over n rows, and its counters.
inline size_t kq_part_floats(int splits, int64_t n) {
    return splits > 1 ? (size_t)splits * KQ_MAX_VECTORS * (size_t)((n + 127) / 128 * 128) : 0;
}
inline size_t kq_counters(int64_t n) { return (size_t)((n + 127) / 128) * (KQ_MAX_VECTORS / 16); }

// GGUF rows [N][K/256 super-blocks] -> the tile layout above.
int kq_pack_launch(int type, const uint8_t* w, int64_t N, int K, uint8_t* out, cudaStream_t stream);
// x [nv][ldx] (K elements each, nv <= 32) -> records [ceil(nv/16)][K/256][KQ_REC].
int kq_prep_launch(const float* x, int ldx, int K, int nv, uint8_t* rec, cudaStream_t stream);
// y[v][i] = W x_v for the nv vectors whose records are `rec`, over the
// packed tiles of rows [0, N).  splits > 1 needs `part` (kq_part_floats)
// and `ctr` (kq_counters, zero on entry; left zero).
int kq_mma_launch(int type, const uint8_t* packed, int64_t N, int K, const uint8_t* rec, int nv, int splits,
                  float* part, int* ctr, float* y, int ldy, unsigned int* err, cudaStream_t stream);

}  // namespace brew
