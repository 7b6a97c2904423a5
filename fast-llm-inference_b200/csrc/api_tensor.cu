// dequantized_tensor.h: host conversions (reference dequantized_tensor.c:
// 27-93) and matmul_dequantized on the GPU with host A / C buffers.
#include <stdlib.h>
#include <string.h>

#include <vector>

#include "fl_common.cuh"
#include "fl_runtime.h"

using namespace fl;

namespace {

struct HostIo {
    float* a = nullptr;
    float* c = nullptr;
    size_t acap = 0, ccap = 0;
};
thread_local std::vector<HostIo> t_io;

int io_buffers(size_t abytes, size_t cbytes, float** a, float** c) {
    int dev = 0;
    cudaGetDevice(&dev);
    if ((int)t_io.size() <= dev) t_io.resize(dev + 1);
    HostIo& io = t_io[dev];
    if (io.acap < abytes) {
        cudaFree(io.a);
        io.a = nullptr;
        io.acap = 0;
        FL_CHECK_CUDA(cudaMalloc(&io.a, abytes));
        io.acap = abytes;
    }
    if (io.ccap < cbytes) {
        cudaFree(io.c);
        io.c = nullptr;
        io.ccap = 0;
        FL_CHECK_CUDA(cudaMalloc(&io.c, cbytes));
        io.ccap = cbytes;
    }
    *a = io.a;
    *c = io.c;
    return FL_OK;
}

dequantized_tensor_t* new_tensor(int rows, int cols, int bits) {
    dequantized_tensor_t* dt = (dequantized_tensor_t*)calloc(1, sizeof(dequantized_tensor_t));
    if (!dt) return nullptr;
    dt->weights = (int8_t*)malloc((size_t)rows * cols);
    dt->scales = (float*)malloc(sizeof(float) * (size_t)rows);
    if (!dt->weights || !dt->scales) {
        free(dt->weights);
        free(dt->scales);
        free(dt);
        return nullptr;
    }
    dt->rows = rows;
    dt->cols = cols;
    dt->original_bits = bits;
    return dt;
}

}  // namespace

// Reference dequantized_tensor.c:27-58 (host): nibble q of element c is
// bits 4*(c%2) of byte (c%32)/2 of its block; int8 = clamp((q-8)*16); the
// row scale is the scale of the row's first block.
FL_API dequantized_tensor_t* dequantized_from_q4(const quantized_tensor_t* q4) {
    if (!q4 || q4->bits != 4 || !q4->blocks || q4->rows <= 0 || q4->cols <= 0) return nullptr;
    const block_q4_t* blocks = (const block_q4_t*)q4->blocks;
    const int rows = q4->rows, cols = q4->cols;
    const int bpr = (cols + Q4_BLOCK_SIZE - 1) / Q4_BLOCK_SIZE;
    dequantized_tensor_t* dt = new_tensor(rows, cols, 4);
    if (!dt) return nullptr;
    for (int r = 0; r < rows; r++) {
        dt->scales[r] = blocks[(size_t)r * bpr].scale;
        for (int c = 0; c < cols; c++) {
            const block_q4_t& b = blocks[(size_t)r * bpr + c / Q4_BLOCK_SIZE];
            const int off = c % Q4_BLOCK_SIZE;
            const int q = (b.qs[off / 2] >> ((off % 2) * 4)) & 0xF;
            int v = (q - 8) * 16;
            v = v < -128 ? -128 : (v > 127 ? 127 : v);
            dt->weights[(size_t)r * cols + c] = (int8_t)v;
        }
    }
    return dt;
}

// Reference dequantized_tensor.c:60-84 (host).
FL_API dequantized_tensor_t* dequantized_from_q8(const quantized_tensor_t* q8) {
    if (!q8 || q8->bits != 8 || !q8->blocks || q8->rows <= 0 || q8->cols <= 0) return nullptr;
    const block_q8_t* blocks = (const block_q8_t*)q8->blocks;
    const int rows = q8->rows, cols = q8->cols;
    const int bpr = (cols + Q8_BLOCK_SIZE - 1) / Q8_BLOCK_SIZE;
    dequantized_tensor_t* dt = new_tensor(rows, cols, 8);
    if (!dt) return nullptr;
    for (int r = 0; r < rows; r++) {
        dt->scales[r] = blocks[(size_t)r * bpr].scale;
        for (int c = 0; c < cols; c++)
            dt->weights[(size_t)r * cols + c] = blocks[(size_t)r * bpr + c / Q8_BLOCK_SIZE].qs[c % Q8_BLOCK_SIZE];
    }
    return dt;
}

FL_API void dequantized_tensor_free(dequantized_tensor_t* t) {
    if (!t) return;
    release_tensor(t);
    free(t->weights);
    free(t->scales);
    free(t->scales_f16);
    if (t->f32_weights && t->original_bits != -1) free(t->f32_weights);
    free(t);
}

FL_API void matmul_dequantized(const float* A, const dequantized_tensor_t* B, float* C, int M, int N, int K) {
    if (!A || !B || !C) return;  // reference dequantized_tensor.c:206
    if (M <= 0 || N <= 0 || K <= 0) return;
    if (upload_tensor((dequantized_tensor_t*)B) != FL_OK) return;
    const DevTensor* d = (const DevTensor*)B->dev;
    if (cudaSetDevice(d->device) != cudaSuccess) {
        set_error(FL_E_CUDA, "matmul_dequantized: cudaSetDevice");
        return;
    }
    float* dA = nullptr;
    float* dC = nullptr;
    if (io_buffers(sizeof(float) * (size_t)M * K, sizeof(float) * (size_t)M * N, &dA, &dC) != FL_OK) return;
    cudaStream_t s = device_stream();
    if (cudaMemcpyAsync(dA, A, sizeof(float) * (size_t)M * K, cudaMemcpyHostToDevice, s) != cudaSuccess) {
        cuda_error(cudaGetLastError(), "matmul_dequantized: H2D");
        return;
    }
    if (fl_cuda_matmul_i8(dA, B, dC, M, N, K, s) != FL_OK) return;
    cudaError_t e = cudaMemcpyAsync(C, dC, sizeof(float) * (size_t)M * N, cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) cuda_error(e, "matmul_dequantized: D2H");
}

FL_API void matmul_dequantized_avx2(const float* A, const dequantized_tensor_t* B, float* C, int M, int N, int K) {
    matmul_dequantized(A, B, C, M, N, K);
}

FL_API void matmul_dequantized_asm_style(const float* A, const dequantized_tensor_t* B, float* C, int M, int N,
                                         int K) {
    matmul_dequantized(A, B, C, M, N, K);
}

FL_API void matmul_dequantized_prefetch(const float* A, const dequantized_tensor_t* B, float* C, int M, int N,
                                        int K) {
    matmul_dequantized(A, B, C, M, N, K);
}
