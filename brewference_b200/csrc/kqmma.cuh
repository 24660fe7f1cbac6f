// kqmma.cuh — the K-quant matvec on the int8 tensor-core path, for the
// forward of models with Q4_K / Q6_K matrices (the 7B config).
//
// A K-quant matrix is repacked once into fragment-ordered tiles: for every
// 16-row tile and 32-element block column, the MMA A-fragment bytes of the
// block's integer quants and fp32 factors beside them:
//   Q4_K  384 B: the 32 quants q in [0, 15] as nibbles in the Q4_0 fragment
//         order (lane (g, t): 8 bytes, low nibbles k = 4t.., high nibbles
//         k = 16 + 4t.., rows g and g + 8), then per lane group g the float4
//         (D_g, M_g, D_g+8, M_g+8), D = d * sc and M = dmin * m of the
//         row's sub-block (GGML's get_scale_min_k4), each rounded as the
//         reference rounds them;
//   Q6_K  640 B: the quants q - 32 in [-32, 31] as int8 in the Q8_0
//         fragment order (16 bytes per lane), then per g the float4
//         (D_g,lo, D_g,hi, D_g+8,lo, D_g+8,hi), D = d * scale of the
//         block's two 16-element halves.
// A tile's block columns are contiguous ([tiles][K/32][bytes]).
//
// The x side is the prep records of prep.cuh (24-bit limb split, exact
// integer block sums).  Per block the epilogue adds
//   Q4_K  s * (D * sum(q * limb) - M * sum(limb))
//   Q6_K  s * (D_lo * sum_lo(q * limb) + D_hi * sum_hi(q * limb))
// per limb column, and the limbs meet at the end: the reference's per
// element products d * sc * q - dmin * m (Q4_K) and d * scale * q (Q6_K)
// summed in another order.
#pragma once

#include "brew_common.cuh"

namespace brew {

__host__ __device__ constexpr int kq_tile_bytes(int type) { return type == BREW_TYPE_Q4_K ? 384 : 640; }
// Bytes of the repacked copy of an N x K matrix (N rounded up to 16 rows).
inline size_t kq_packed_bytes(int type, int64_t N, int64_t K) {
    return (size_t)((N + 15) / 16) * (size_t)(K / 32) * (size_t)kq_tile_bytes(type);
}
// GGUF rows [N][K/256 super-blocks] -> fragment-ordered tiles (rows past N
// in the last tile are zero).
int kq_pack_launch(int type, const uint8_t* w, int64_t N, int K, uint8_t* out, cudaStream_t stream);
// y[b][i] = W x_b for the nv <= 16 vectors whose prep records (rec_bytes =
// prep_rec_bytes(nv)) are `prep`, over the packed tiles of rows [0, N).
int kq_mma_launch(int type, const uint8_t* packed, int64_t N, int K, const uint8_t* prep, int nv, float* y, int ldy,
                  cudaStream_t stream);

}  // namespace brew
