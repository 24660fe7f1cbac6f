// eltwise.cuh — the per-row vector steps of the forward pass as separate
// kernels, for layers whose matrices are not fused with them (the K-quant
// forward): RMSNorm, bias, residual, gated activation.
#pragma once

#include "brew_common.cuh"

namespace brew {

// out[b][i] = x[b][i] * scale_b * w[i], scale_b = inverseRootMeanSquare
// (Kernels.rmsNorm, transformer/math/Kernels.java:47-58,77-88).
int rmsnorm_launch(const float* x, int ldx, const float* w, float eps, int K, int B, float* out, int ldo,
                   cudaStream_t s);
// y[b][i] = y[b][i] + bias[i] for i < N (Kernels.addBias, Kernels.java:171-197).
int add_bias_launch(float* y, int ldy, const float* bias, int N, int B, cudaStream_t s);
// x[b][i] = x[b][i] + t[b][i] (Kernels.accum), or with norm_w (Gemma3's
// post-norm): x[b][i] = x[b][i] + rmsnorm(t[b], norm_w)[i].
int residual_launch(float* x, int ldx, const float* t, int ldt, const float* norm_w, float eps, int K, int B,
                    cudaStream_t s);
// hb[b][i] = (float)act((double)g[b][i]) * u[b][i] (FfnActivation.swiGlu /
// geGlu, transformer/ffn/FfnActivation.java:23-58); hb's row stride is ldo
// when given, else ld.
int glu_launch(float* hb, const float* g, const float* u, int ld, int N, int B, bool gelu, cudaStream_t s, int ldo = 0);

// The residual of the previous sub-layer, the RMSNorm of the next, and the
// next matvec's x records, in one kernel (one CTA of 1024 threads per
// vector): with t, x[b] += t[b] (or + rmsnorm(t[b], post_w) with post_w) as
// residual_launch; then out[b] = rmsnorm(x[b], w) as rmsnorm_launch (the
// same operations, the sums of squares split over 1024 threads); then, with
// rec, the records of out for a tcgen05 K-quant matvec (kqtc.cuh) of the B
// vectors.
int norm_prep_launch(float* x, int ldx, const float* t, int ldt, const float* post_w, const float* w, float eps, int K,
                     int B, float* out, int ldo, uint8_t* rec, cudaStream_t s);
// glu_launch, then (with rec) the records of hb for a tcgen05 K-quant matvec.
int glu_prep_launch(float* hb, const float* g, const float* u, int ld, int N, int B, bool gelu, uint8_t* rec,
                    cudaStream_t s);

}  // namespace brew
