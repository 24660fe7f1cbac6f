// tp.cuh — tensor parallelism across the GPUs of one box: row-sharded
// matrices and NCCL all-gathers of the projection outputs.
//
// Rank r of P owns rows [r·N/P, (r+1)·N/P) of every matrix (N divisible by
// P).  Each output row is computed exactly as on one GPU, and a gather only
// copies, so the sharded forward returns the one-GPU result bit for bit.
#pragma once

#include "brew_common.cuh"

struct brew_comm_s {
    void* nccl = nullptr;   // ncclComm_t
    int nranks = 1, rank = 0, device = -1;
};

namespace brew {

// All-gather of `count` floats per rank on `stream`: recv = [nranks][count].
int tp_allgather(brew_comm_s* c, const float* send, float* recv, size_t count, cudaStream_t stream);
// The same for 64-bit words.
int tp_allgather_u64(brew_comm_s* c, const unsigned long long* send, unsigned long long* recv, size_t count,
                     cudaStream_t stream);

// One segment of a gathered output: rank r's slice holds `n` values of it at
// offset `src_off` (within the rank's [B][slice] row); they go to
// dst[b][dst_off + r·n + i].
struct TpSeg {
    int n, src_off, dst_off;
};

// recv [P][B][slice] -> dst [B][ldd], per segment (up to 3).
int tp_unshard_launch(const float* recv, int P, int B, int slice, const TpSeg* segs, int nseg, float* dst, int ldd,
                      cudaStream_t stream);
// Per-row argmax keys of a logits slice whose first row is global row `row0`
// (orderable: larger value first, then smaller index).
int tp_argmax_keys_launch(const float* logits, int ld, int n, int B, int row0, unsigned long long* keys,
                          cudaStream_t stream);
// keys [P][B] -> ids [B] (Kernels.argMax: the first maximum).
int tp_argmax_reduce_launch(const unsigned long long* keys, int P, int B, int32_t* out, cudaStream_t stream);

}  // namespace brew
