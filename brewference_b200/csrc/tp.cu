// tp.cu — NCCL communicator, row-shard plan and the gather helpers of the
// tensor-parallel forward.  NCCL is loaded with dlopen when a communicator
// is first created, so one-GPU use has no NCCL dependency.
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <cstring>
#include <mutex>

#include "brew_internal.cuh"
#include "mv_device.cuh"
#include "tp.cuh"

namespace brew {
namespace {

struct NcclApi {
    void* lib = nullptr;
    ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
    ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
    ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    const char* (*error_string)(ncclResult_t) = nullptr;
};

NcclApi g_nccl;
std::mutex g_nccl_mu;

int nccl_load() {
    std::lock_guard<std::mutex> lk(g_nccl_mu);
    if (g_nccl.lib) return BREW_OK;
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return set_error(BREW_ERR_NCCL, "cannot load libnccl.so.2: %s", dlerror());
    NcclApi a;
    a.lib = h;
    a.get_unique_id = reinterpret_cast<decltype(a.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
    a.comm_init_rank = reinterpret_cast<decltype(a.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
    a.comm_destroy = reinterpret_cast<decltype(a.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
    a.all_gather = reinterpret_cast<decltype(a.all_gather)>(dlsym(h, "ncclAllGather"));
    a.error_string = reinterpret_cast<decltype(a.error_string)>(dlsym(h, "ncclGetErrorString"));
    if (!a.get_unique_id || !a.comm_init_rank || !a.comm_destroy || !a.all_gather || !a.error_string)
        return set_error(BREW_ERR_NCCL, "libnccl.so.2 lacks an entry point this library uses");
    g_nccl = a;
    return BREW_OK;
}

int nccl_check(ncclResult_t r, const char* what) {
    if (r == ncclSuccess) return BREW_OK;
    return set_error(BREW_ERR_NCCL, "%s: %s", what, g_nccl.error_string ? g_nccl.error_string(r) : "nccl error");
}

__global__ void unshard_kernel(const float* recv, int P, int B, int slice, TpSeg s0, TpSeg s1, TpSeg s2, int nseg,
                               float* dst, int ldd) {
    // one thread per (segment value, rank, row)
    const TpSeg segs[3] = {s0, s1, s2};
    const int b = blockIdx.y, r = blockIdx.z;
    for (int k = 0; k < nseg; ++k) {
        const TpSeg s = segs[k];
        const float* src = recv + ((int64_t)r * B + b) * slice + s.src_off;
        float* d = dst + (int64_t)b * ldd + s.dst_off + (int64_t)r * s.n;
        for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < s.n; i += gridDim.x * blockDim.x) d[i] = src[i];
    }
}

// Peer-store gather, push: one thread per pair of this rank's slice values
// (segment lengths, offsets and ldd are even, so a pair never straddles a
// segment and lands 16-byte aligned); the pair goes to every rank's slot.
__global__ void tp_push_kernel(const float* send, int B, int slice, TpSeg s0, TpSeg s1, TpSeg s2, int nseg, int ldd,
                               TpPeers peers, int P, int R, size_t site_off, const uint32_t* step, int site) {
    const int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int half = slice >> 1;
    if (q >= (int64_t)B * half) return;
    const int b = (int)(q / half), j = 2 * (int)(q - (int64_t)b * half);
    const TpSeg segs[3] = {s0, s1, s2};
    int k = 0;
    while (k + 1 < nseg && j >= segs[k + 1].src_off) ++k;
    const TpSeg sg = segs[k];
    const int64_t pos = (int64_t)b * ldd + sg.dst_off + (int64_t)R * sg.n + (j - sg.src_off);
    const uint64_t tag = (uint64_t)(*step * 256u + (uint32_t)site) << 32;
    const float2 v = *reinterpret_cast<const float2*>(send + (int64_t)b * slice + j);
    const uint64_t w0 = tag | __float_as_uint(v.x), w1 = tag | __float_as_uint(v.y);
    for (int r = 0; r < P; ++r)
        asm volatile("st.relaxed.sys.global.v2.u64 [%0], {%1, %2};" ::"l"(peers.p[r] + site_off + pos), "l"(w0),
                     "l"(w1)
                     : "memory");
}

// Peer-store gather, pull: one thread per pair of the unsharded row; polls
// the pair in this rank's slot until both words carry the tag.  Bounded: 2 s,
// or as soon as another pull gave up (abort), then a timeout is recorded.
__global__ void tp_pull_kernel(const unsigned long long* slot, int B, int ldd, float* dst, const uint32_t* step,
                               int site, int* abort, unsigned int* err) {
    const int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (q >= (int64_t)B * (ldd >> 1)) return;
    const uint32_t tag = *step * 256u + (uint32_t)site;
    const unsigned long long* p = slot + 2 * q;
    unsigned long long w0, w1;
    const uint64_t t0 = global_ns();
    for (uint32_t it = 1;; ++it) {
        asm volatile("ld.relaxed.sys.global.v2.u64 {%0, %1}, [%2];" : "=l"(w0), "=l"(w1) : "l"(p) : "memory");
        if ((uint32_t)(w0 >> 32) == tag && (uint32_t)(w1 >> 32) == tag) break;
        if ((it & 63u) == 0u && (global_ns() - t0 > 2000000000ull || ld_volatile_int(abort))) {
            atomicOr(err, BREW_DEVERR_TIMEOUT_FULL);
            atomicExch(abort, 1);
            return;
        }
    }
    const int64_t b = q / (ldd >> 1), i = 2 * (q - b * (ldd >> 1));
    *reinterpret_cast<float2*>(dst + b * ldd + i) = make_float2(__uint_as_float((uint32_t)w0), __uint_as_float((uint32_t)w1));
}

__global__ void tp_step_kernel(uint32_t* step) { *step += 1u; }

__global__ void argmax_keys_kernel(const float* logits, int ld, int n, int row0, unsigned long long* keys) {
    const int b = blockIdx.x;
    const float* lr = logits + (int64_t)b * ld;
    unsigned long long best = 0ull;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const unsigned long long k = argmax_key(lr[i], row0 + i);
        best = k > best ? k : best;
    }
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long v = __shfl_xor_sync(0xffffffffu, best, o);
        best = v > best ? v : best;
    }
    __shared__ unsigned long long red[32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (lane == 0) red[warp] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned long long t = 0ull;
        for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t = red[w] > t ? red[w] : t;
        keys[b] = t;
    }
}

__global__ void argmax_reduce_kernel(const unsigned long long* keys, int P, int B, int32_t* out) {
    const int b = threadIdx.x;
    if (b >= B) return;
    unsigned long long t = 0ull;
    for (int r = 0; r < P; ++r) t = keys[(int64_t)r * B + b] > t ? keys[(int64_t)r * B + b] : t;
    out[b] = (int32_t)(0xFFFFFFFFu - (uint32_t)(t & 0xFFFFFFFFull));
}

}  // namespace

int tp_allgather(brew_comm_s* c, const float* send, float* recv, size_t count, cudaStream_t stream) {
    return nccl_check(g_nccl.all_gather(send, recv, count, ncclFloat32, static_cast<ncclComm_t>(c->nccl), stream),
                      "ncclAllGather");
}

int tp_allgather_u64(brew_comm_s* c, const unsigned long long* send, unsigned long long* recv, size_t count,
                     cudaStream_t stream) {
    return nccl_check(g_nccl.all_gather(send, recv, count, ncclUint64, static_cast<ncclComm_t>(c->nccl), stream),
                      "ncclAllGather");
}

int tp_unshard_launch(const float* recv, int P, int B, int slice, const TpSeg* segs, int nseg, float* dst, int ldd,
                      cudaStream_t stream) {
    BREW_CHECK(nseg >= 1 && nseg <= 3, BREW_ERR_INVALID_ARG, "unshard: %d segments", nseg);
    int nmax = 0;
    for (int k = 0; k < nseg; ++k) nmax = std::max(nmax, segs[k].n);
    const TpSeg z = {0, 0, 0};
    const dim3 grid(std::max(1, std::min(64, (nmax + 255) / 256)), B, P);
    unshard_kernel<<<grid, 256, 0, stream>>>(recv, P, B, slice, segs[0], nseg > 1 ? segs[1] : z,
                                             nseg > 2 ? segs[2] : z, nseg, dst, ldd);
    BREW_CUDA(cudaGetLastError());
    count_launch();
    return BREW_OK;
}

int tp_argmax_keys_launch(const float* logits, int ld, int n, int B, int row0, unsigned long long* keys,
                          cudaStream_t stream) {
    argmax_keys_kernel<<<B, 1024, 0, stream>>>(logits, ld, n, row0, keys);
    BREW_CUDA(cudaGetLastError());
    count_launch();
    return BREW_OK;
}

int tp_push_launch(const float* send, int B, int slice, const TpSeg* segs, int nseg, int ldd, const TpPeers& peers,
                   int P, int R, size_t site_off, const uint32_t* step, int site, cudaStream_t stream) {
    BREW_CHECK(nseg >= 1 && nseg <= 3 && P >= 1 && P <= TP_MAX_RANKS && slice % 2 == 0 && ldd % 2 == 0 &&
                   site_off % 2 == 0 && site >= 0 && site < 256,
               BREW_ERR_INVALID_ARG, "peer gather: %d segments, %d ranks, slice %d, ldd %d", nseg, P, slice, ldd);
    for (int k = 0; k < nseg; ++k)
        BREW_CHECK(segs[k].n % 2 == 0 && segs[k].src_off % 2 == 0 && segs[k].dst_off % 2 == 0, BREW_ERR_INVALID_ARG,
                   "peer gather: odd segment");
    const TpSeg z = {0, slice, 0};
    const int64_t pairs = (int64_t)B * (slice / 2);
    if (pairs == 0) return BREW_OK;
    tp_push_kernel<<<(unsigned)((pairs + 255) / 256), 256, 0, stream>>>(send, B, slice, segs[0], nseg > 1 ? segs[1] : z,
                                                                     nseg > 2 ? segs[2] : z, nseg, ldd, peers, P, R,
                                                                     site_off, step, site);
    BREW_CUDA(cudaGetLastError());
    count_launch();
    return BREW_OK;
}

int tp_pull_launch(const unsigned long long* slot, int B, int ldd, float* dst, const uint32_t* step, int site,
                   int* abort, unsigned int* err, cudaStream_t stream) {
    BREW_CHECK(ldd % 2 == 0 && site >= 0 && site < 256, BREW_ERR_INVALID_ARG, "peer gather: ldd %d", ldd);
    const int64_t pairs = (int64_t)B * (ldd / 2);
    if (pairs == 0) return BREW_OK;
    tp_pull_kernel<<<(unsigned)((pairs + 255) / 256), 256, 0, stream>>>(slot, B, ldd, dst, step, site, abort, err);
    BREW_CUDA(cudaGetLastError());
    count_launch();
    return BREW_OK;
}

int tp_step_launch(uint32_t* step, cudaStream_t stream) {
    tp_step_kernel<<<1, 1, 0, stream>>>(step);
    BREW_CUDA(cudaGetLastError());
    count_launch();
    return BREW_OK;
}

int tp_argmax_reduce_launch(const unsigned long long* keys, int P, int B, int32_t* out, cudaStream_t stream) {
    // one thread per sequence in a single warp
    BREW_CHECK(B >= 1 && B <= 32, BREW_ERR_INVALID_ARG, "sharded argmax: %d sequences (at most 32)", B);
    argmax_reduce_kernel<<<1, 32, 0, stream>>>(keys, P, B, out);
    BREW_CUDA(cudaGetLastError());
    count_launch();
    return BREW_OK;
}

}  // namespace brew

using namespace brew;

extern "C" {

int brew_tp_rows(int64_t rows, int32_t nranks, int32_t rank, int64_t* r0, int64_t* r1) {
    BREW_CHECK(r0 && r1, BREW_ERR_INVALID_ARG, "null argument");
    BREW_CHECK(nranks >= 1 && rank >= 0 && rank < nranks, BREW_ERR_INVALID_ARG, "rank %d of %d", rank, nranks);
    BREW_CHECK(rows >= 0 && rows % nranks == 0, BREW_ERR_UNSUPPORTED, "%lld rows do not split over %d ranks",
               (long long)rows, nranks);
    *r0 = rows / nranks * rank;
    *r1 = rows / nranks * (rank + 1);
    return BREW_OK;
}

int brew_comm_unique_id(uint8_t* out) {
    BREW_CHECK(out, BREW_ERR_INVALID_ARG, "null argument");
    int rc = nccl_load();
    if (rc) return rc;
    ncclUniqueId id;
    if ((rc = nccl_check(g_nccl.get_unique_id(&id), "ncclGetUniqueId"))) return rc;
    memcpy(out, id.internal, NCCL_UNIQUE_ID_BYTES);
    return BREW_OK;
}

int brew_comm_init(const uint8_t* id_bytes, int32_t nranks, int32_t rank, brew_comm* out) {
    BREW_CHECK(id_bytes && out, BREW_ERR_INVALID_ARG, "null argument");
    BREW_CHECK(nranks >= 1 && rank >= 0 && rank < nranks, BREW_ERR_INVALID_ARG, "rank %d of %d", rank, nranks);
    *out = nullptr;
    int rc = ensure_init();
    if (rc) return rc;
    if ((rc = nccl_load())) return rc;
    ncclUniqueId id;
    memcpy(id.internal, id_bytes, NCCL_UNIQUE_ID_BYTES);
    ncclComm_t comm = nullptr;
    if ((rc = nccl_check(g_nccl.comm_init_rank(&comm, nranks, id, rank), "ncclCommInitRank"))) return rc;
    brew_comm c = new brew_comm_s();
    c->nccl = comm;
    c->nranks = nranks;
    c->rank = rank;
    c->device = ctx().device;
    *out = c;
    return BREW_OK;
}

int brew_comm_free(brew_comm c) {
    if (!c) return BREW_OK;
    if (c->nccl && g_nccl.comm_destroy) g_nccl.comm_destroy(static_cast<ncclComm_t>(c->nccl));
    delete c;
    return BREW_OK;
}

}  // extern "C"
