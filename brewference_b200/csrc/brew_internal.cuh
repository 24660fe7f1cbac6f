// brew_internal.cuh — library-internal state shared by the host files.
#pragma once

#include <mutex>

#include "attention.cuh"
#include "brew_common.cuh"
#include "matvec.cuh"
#include "misc.cuh"
#include "prep.cuh"

struct brew_tensor_s {
    int type = 0;
    int64_t n = 0;       // elements
    int64_t bytes = 0;   // packed bytes
    uint8_t* d = nullptr;
    bool owned = true;   // false: a view into another tensor (tied embeddings)
};

namespace brew {

// A growable device buffer.
struct Scratch {
    void* ptr = nullptr;
    size_t bytes = 0;
    int reserve(size_t need_bytes);
};

struct Context {
    bool initialized = false;
    int device = -1;
    cudaStream_t stream = nullptr;
    unsigned int* err_word = nullptr;
    Scratch mv_scratch;   // prep records of brew_matmul / brew_matmul_dev
    Scratch io_scratch;   // staging of brew_matmul / brew_dequantize_row
};

Context& ctx();
std::mutex& api_mutex();
int ensure_init();

int run_matvec(brew_tensor t, int64_t weights_offset, const float* x_dev, int K, int N, float* y_dev, int batch,
               cudaStream_t stream);
int run_matvec_prepared(brew_tensor t, int64_t weights_offset, const uint8_t* prep, int K, int N, float* y, int batch,
                        cudaStream_t stream);
int launch_prepared(brew_tensor t, const uint8_t* w, int64_t row_bytes, const uint8_t* prep, int K, int N, float* y,
                    int nb, cudaStream_t stream);
// Makes a model created with brew_model_create own (and free) its tensors.
void model_adopt_tensors(brew_model m);
// Looks up the device address of brew_matmul_dev_static's module array on
// the current device (brew_init calls it).
int static_scratch_setup();
int kquant_matvec_launch(int type, const uint8_t* w, int64_t row_bytes, const float* x, int ldx, int K, int N, float* y,
                         int ldy, int batch, cudaStream_t stream, bool pdl);

}  // namespace brew
