// Host-side runtime shared by the C-ABI translation units.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include <string>

#include "dequantized_tensor.h"
#include "fl_cuda.h"

namespace fl {

// Records the message of the latest failure on this thread and returns code.
int set_error(int code, const std::string& msg);
int cuda_error(cudaError_t e, const char* what);

// Library stream of the current device (created on first use).
cudaStream_t device_stream();
int ensure_device();

// Device mirror of a dequantized_tensor_t (stored in its `dev` field).
struct DevTensor {
    int8_t* w;
    __half* sblk;      // block mode
    float* srow;       // per-row mode
    int rows, cols;
    int scale_block;
    int pairsat;       // per-row mode with max|w| > 64
    int device;
    int P;             // tiled-layout panel width (block mode), 0 = row-major
};

int upload_tensor(dequantized_tensor_t* t);
void release_tensor(dequantized_tensor_t* t);

}  // namespace fl

#define FL_CHECK_CUDA(expr)                                          \
    do {                                                             \
        cudaError_t fl_e_ = (expr);                                  \
        if (fl_e_ != cudaSuccess) return fl::cuda_error(fl_e_, #expr); \
    } while (0)

#define FL_CHECK(expr)               \
    do {                             \
        int fl_r_ = (expr);          \
        if (fl_r_ != 0) return fl_r_; \
    } while (0)
