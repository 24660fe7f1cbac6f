// gemm.cuh — the prefill GEMM: Y[t][n] = sum_k W[n][k] x[t][k] for many
// tokens t at once, on the 5th-generation tensor cores (tcgen05, int8, TMEM
// accumulators).
//
// The weights are a GEMM-layout copy of a Q8_0 (or Q4_0, its quants as
// q - 8) matrix: for every 128-row
// tile and 32-element block column, the 4096 quant bytes in the K-major
// core-matrix layout the MMA reads from shared memory (8-row groups of 256 B,
// the two 16-byte halves of a row's block 128 B apart), tiles [N/128][K/32];
// block scales [K/32][N] fp16.  The activations are split per 32-element
// block into three int8 limbs (24-bit block fixed point, prep.cuh), stored
// the same way per block column and 32-token tile ([K/32][T/32][3072 B]),
// limb column 6 (t/2) + 2 l + (t%2) of token t in the tile.  One
// tcgen05.mma per block column multiplies a 128-row weight tile by the 96
// limb columns in exact int32; the epilogue reads the tile from tensor
// memory and adds d_row * s_token * (lo + mid * 2^8 + hi * 2^16) to fp32
// accumulators.
#pragma once

#include "brew_common.cuh"

namespace brew {

constexpr int GEMM_TM = 128;   // weight rows per CTA (tcgen05 M)
constexpr int GEMM_TT = 32;    // tokens per CTA (tcgen05 N = 3 * 32 = 96)

// `rows` Q8_0 or Q4_0 GGUF rows [rows][K/32 blocks] -> rows row0 .. of an
// ldn-row matrix: quant tiles in wq (the matrix's [ldn/128][K/32][4096 B])
// and block scales wd[kb][row0 + row] of its [K/32][ldn] scale matrix
// (block-column major: a column's scales of consecutive rows are contiguous
// for the GEMM epilogue).
int gemm_pack_launch(int type, const uint8_t* w, int rows, int K, int8_t* wq, uint16_t* wd, int ldn, int row0,
                     cudaStream_t stream);
// x [T][ldx] fp32 (first K columns) -> limb tiles [K/32][Tp/32][3072 B]
// int8 + block scales [K/32][Tp] fp32 (the records' arithmetic of prep.cuh,
// one token per row); tokens T .. Tp-1 are zero.
int gemm_limbs_launch(const float* x, int ldx, int T, int Tp, int K, int8_t* limbs, float* scales,
                      cudaStream_t stream);
// y [Tvalid][N] = W x (T the padded token count, a multiple of GEMM_TT; N a
// multiple of GEMM_TM, K of 32; rows Tvalid .. T-1 are not written).
int gemm_q8_launch(const int8_t* wq, const uint16_t* wd, const int8_t* limbs, const float* scales, int N, int K, int T,
                   int Tvalid, float* y, unsigned int* err, cudaStream_t stream);

}  // namespace brew
