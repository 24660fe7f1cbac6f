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

// The peer-store gather.  Every rank holds a tagged arena with one slot per
// gather site of a forward step ([B][ldd] words, (tag << 32) | float bits),
// mapped into every other rank's address space (CUDA IPC).  A gather is
// two launches: push writes this rank's slice into its place in every
// rank's slot (system-scope 8-byte stores over NVLink), pull polls this
// rank's own slot until every word carries the tag and writes the floats
// unsharded.  tag = step * 256 + site, `step` a device counter advanced once
// per forward on every rank, so no word of an earlier gather passes for this
// one, and no slot is rewritten before every rank has read it (a rank starts
// the next step only after the last gather of this one, which needs every
// rank's push, and a rank pushes only after its own earlier pulls).
constexpr int TP_MAX_RANKS = 8;
struct TpPeers {
    unsigned long long* p[TP_MAX_RANKS];   // every rank's arena (this rank's included)
};
// send [B][slice] -> the site's slot (word offset site_off) of every rank.
int tp_push_launch(const float* send, int B, int slice, const TpSeg* segs, int nseg, int ldd, const TpPeers& peers,
                   int P, int R, size_t site_off, const uint32_t* step, int site, cudaStream_t stream);
// this rank's slot -> dst [B][ldd]; bounded wait (2 s, or another wait's
// abort), then the error word records a timeout.
int tp_pull_launch(const unsigned long long* slot, int B, int ldd, float* dst, const uint32_t* step, int site,
                   int* abort, unsigned int* err, cudaStream_t stream);
// step += 1 (once per forward, before its gathers)
int tp_step_launch(uint32_t* step, cudaStream_t stream);
// Per-row argmax keys of a logits slice whose first row is global row `row0`
// (orderable: larger value first, then smaller index).
int tp_argmax_keys_launch(const float* logits, int ld, int n, int B, int row0, unsigned long long* keys,
                          cudaStream_t stream);
// keys [P][B] -> ids [B] (Kernels.argMax: the first maximum).
int tp_argmax_reduce_launch(const unsigned long long* keys, int P, int B, int32_t* out, cudaStream_t stream);

}  // namespace brew
