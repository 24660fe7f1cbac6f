// matmul_static.cu — brew_matmul_dev_static: the device-pointer matvec of
// brew_matmul_dev with its scratch (the quantized-activation records of x)
// in a fixed array that is part of the loaded module, so the call itself
// allocates nothing.
//
// Who cannot allocate: a caller that is inside a JNI critical region (arrays
// pinned with GetPrimitiveArrayCritical) must not block, and cudaMalloc /
// cudaFree may wait for the whole device, holding back the JVM's garbage
// collector for as long; and a server that reserves its device memory for
// its own pools at start-up cannot let a library take more in the middle of
// a request, where a failed allocation would abort the request half done.
// brew_matmul_dev grows a per-context buffer on demand; this entry point
// never does, and it does not create the context either (brew_init first).
//
// Limit: the records of one batch chunk (up to MV_MAX_BATCH vectors) must fit
// in BREW_STATIC_SCRATCH_BYTES = 256 KiB, i.e. (K / 32) * record bytes of
// min(batch, 16) vectors: K <= 74880 at batch 1, K <= 4672 at batch 16.
// Larger requests fail with BREW_ERR_INVALID_ARG.  Q4_K / Q6_K weights use no
// scratch and run the same kernel as brew_matmul_dev.
//
// Set-up: brew_init looks up the array's device address on the device it
// makes current (cudaGetSymbolAddress, which also loads this file's module),
// so the array is in place before the first call.  A later brew_init of
// another device does the same there; a call on a device whose address is
// still unknown looks it up first.  The kernels the call launches are loaded
// by the CUDA runtime on their first launch (lazy module loading), so make
// one call before entering a region that must not allocate or block, and
// before any stream capture begins.
//
// Nothing in the array has to start at zero: every byte the matvec kernel
// reads is written by the prep kernel earlier in the same call.
//
// Concurrency: there is one array per device.  Calls whose device work can
// overlap (different streams without an ordering between them) race on it;
// issue such calls on one stream or order them with events.
#include <mutex>

#include "brew_internal.cuh"
#include "matvec.cuh"
#include "prep.cuh"

namespace brew {
namespace {

constexpr int BREW_STATIC_SCRATCH_BYTES = 256 * 1024;
constexpr int BREW_STATIC_MAX_DEVICES = 64;

static __device__ __align__(256) uint8_t g_static_scratch[BREW_STATIC_SCRATCH_BYTES];

std::mutex g_static_mu;
void* g_static_addr[BREW_STATIC_MAX_DEVICES] = {};

// Device address of the array on the current device (looked up once per device).
int static_scratch(uint8_t** out) {
    int dev = 0;
    BREW_CUDA(cudaGetDevice(&dev));
    BREW_CHECK(dev >= 0 && dev < BREW_STATIC_MAX_DEVICES, BREW_ERR_UNSUPPORTED, "device %d", dev);
    std::lock_guard<std::mutex> lk(g_static_mu);
    if (!g_static_addr[dev]) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_static_scratch);
        if (e != cudaSuccess) {
            cudaGetLastError();
            return set_error(BREW_ERR_CUDA, "cudaGetSymbolAddress(static scratch) on device %d: %s", dev,
                             cudaGetErrorString(e));
        }
        g_static_addr[dev] = p;
    }
    *out = static_cast<uint8_t*>(g_static_addr[dev]);
    return BREW_OK;
}

}  // namespace

// Called by brew_init with the new device current.
int static_scratch_setup() {
    uint8_t* p = nullptr;
    return static_scratch(&p);
}

}  // namespace brew

using namespace brew;

extern "C" int brew_matmul_dev_static(float* y, const float* x, brew_tensor w, int64_t off, int32_t K, int32_t N,
                                      int32_t batch, void* stream) {
    // argument checks of Linear.validateMatmulArguments (transformer/math/Linear.java:67-74)
    // and the scale-index bound (Linear.java:46-50), as in brew_matmul_dev
    BREW_CHECK(w, BREW_ERR_INVALID_ARG, "Weight block cannot be null");
    BREW_CHECK(w->d, BREW_ERR_INVALID_ARG, "Weight block scales and data must be initialized");
    BREW_CHECK(x && y, BREW_ERR_INVALID_ARG, "Input and output arrays cannot be null");
    TypeInfo ti;
    BREW_CHECK(type_info(w->type, &ti) && is_quant_matrix_type(w->type), BREW_ERR_UNSUPPORTED,
               "matmul on GGML type %d", w->type);
    BREW_CHECK(K > 0 && K % ti.block_elems == 0, BREW_ERR_INVALID_ARG,
               "inputSize %d is not a whole number of %d-element blocks", K, ti.block_elems);
    BREW_CHECK(N >= 0 && off >= 0 && off % ti.block_elems == 0, BREW_ERR_INVALID_ARG,
               "weightsOffset %lld is not at a block boundary", (long long)off);
    BREW_CHECK(off + (int64_t)N * K <= w->n, BREW_ERR_OUT_OF_BOUNDS,
               "matmul scale index out of bounds (wOffset=%lld, n=%d, d=%d)", (long long)off, K, N);
    BREW_CHECK(batch >= 1, BREW_ERR_INVALID_ARG, "batch %d", batch);
    const bool kquant = w->type == BREW_TYPE_Q4_K || w->type == BREW_TYPE_Q6_K;
    const size_t need = (size_t)(K / 32) * prep_rec_bytes(std::min(batch, MV_MAX_BATCH));
    BREW_CHECK(kquant || need <= (size_t)BREW_STATIC_SCRATCH_BYTES, BREW_ERR_INVALID_ARG,
               "brew_matmul_dev_static: K=%d at batch %d needs %zu bytes of records; the static scratch holds %d "
               "(use brew_matmul_dev)", K, batch, need, BREW_STATIC_SCRATCH_BYTES);
    if (N == 0) return BREW_OK;
    BREW_CHECK(ctx().initialized, BREW_ERR_INVALID_ARG,
               "brew_matmul_dev_static: call brew_init first (this entry point does not create the context)");
    int rc = ensure_init();   // the context exists: this only makes its device current
    if (rc) return rc;
    std::lock_guard<std::mutex> lk(api_mutex());
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int64_t row_bytes = (int64_t)K / ti.block_elems * ti.block_bytes;
    const uint8_t* wp = w->d + off / ti.block_elems * ti.block_bytes;
    if (kquant) return kquant_matvec_launch(w->type, wp, row_bytes, x, K, K, N, y, N, batch, s, false);
    uint8_t* scratch = nullptr;
    if ((rc = static_scratch(&scratch))) return rc;
    for (int b0 = 0; b0 < batch; b0 += MV_MAX_BATCH) {
        const int nb = std::min(MV_MAX_BATCH, batch - b0);
        rc = prep_launch(x + (int64_t)b0 * K, K, K, nb, nullptr, 0.0f, scratch, s, false);
        if (rc) return rc;
        rc = launch_prepared(w, wp, row_bytes, scratch, K, N, y + (int64_t)b0 * N, nb, s);
        if (rc) return rc;
    }
    return BREW_OK;
}
