// gemm.cuh — the prefill GEMM: Y[t][n] = sum_k W[n][k] x[t][k] for many
// tokens t at once, on the 5th-generation tensor cores (tcgen05, int8, TMEM
// accumulators).
//
// The weights are a GEMM-layout copy of a Q8_0 matrix: quants [N][K] int8
// (row-major, so any 16-byte piece of a row is contiguous) and block scales
// [N][K/32] fp16.  The activations are split per 32-element block into three
// int8 limbs (24-bit block fixed point, prep.cuh) laid out per block as
// [K/32][3T][32]: limb-column n = 3t + l of token t.  One tcgen05.mma per
// block column multiplies a 128-row weight tile by 3 x 32 token columns in
// exact int32; the epilogue reads the tile from tensor memory and adds
// d_row * s_token * (lo + mid * 2^8 + hi * 2^16) to fp32 accumulators.
#pragma once

#include "brew_common.cuh"

namespace brew {

constexpr int GEMM_TM = 128;   // weight rows per CTA (tcgen05 M)
constexpr int GEMM_TT = 32;    // tokens per CTA (tcgen05 N = 3 * 32 = 96)

// Q8_0 GGUF rows [N][K/32 blocks of 34 B] -> quants [N][K] + scales [N][K/32].
int gemm_pack_q8_launch(const uint8_t* w, int N, int K, int8_t* wq, uint16_t* wd, cudaStream_t stream);
// x [T][ldx] fp32 (first K columns) -> limbs [K/32][3Tp][32] int8 + block
// scales [K/32][Tp] fp32 (the records' arithmetic of prep.cuh, one token per
// row); tokens T .. Tp-1 are zero.
int gemm_limbs_launch(const float* x, int ldx, int T, int Tp, int K, int8_t* limbs, float* scales,
                      cudaStream_t stream);
// y [T][N] = W x (T a multiple of GEMM_TT, N of GEMM_TM, K of 32).
int gemm_q8_launch(const int8_t* wq, const uint16_t* wd, const int8_t* limbs, const float* scales, int N, int K, int T,
                   float* y, unsigned int* err, cudaStream_t stream);

}  // namespace brew
