/*
 * Pre-dequantized INT8 weight tensor and the INT8 matmul, B200 edition.
 *
 * Drop-in for the reference's dequantized_tensor.h
 * (fast_llm/include/dequantized_tensor.h:27-70): the first six struct fields
 * and every function signature are unchanged, so inference.c, main.c and the
 * benches compile against this header as they are. Three fields are appended
 * after the reference's last one (original_bits):
 *
 *   scale_block  0  -> reference per-row mode: weights may span [-128, 127]
 *                      (dequantized_from_q4 produces (q-8)*16), one float scale
 *                      per row in `scales`. Arithmetic is exactly the
 *                      reference's matmul_dequantized (dequantized_tensor.c:
 *                      204-247): u8 activations, int16 pair-saturated dot,
 *                      C = (float)dot * scales[n] / (127 * 16).
 *                32 -> block mode: weights are Q4_0 nibbles minus 8, in
 *                      [-8, 7], one fp16 scale per 32 consecutive weights of a
 *                      row in `scales_f16` ([rows, cols/32]).
 *                      C = (sum over blocks b of (float)dot_b * d_b) / 127,
 *                      dot_b the int32 dot of block b.
 *   scales_f16   host pointer to the per-block fp16 scales (block mode).
 *   dev          device-side mirror, created by fl_cuda_upload_tensor and
 *                released by dequantized_tensor_free; NULL until uploaded.
 *
 * In both modes the activation row is quantized exactly as the reference
 * does it (dequantized_tensor.c:112-143): u8 = clamp(rne(x*127 + 128), 0, 255)
 * with one fused multiply-add, and the +128 bias is NOT subtracted from the
 * dot product afterwards (dequantized_tensor.c:235-243). Every call below runs
 * on the GPU; there is no CPU fallback. A function that cannot run (no CUDA
 * device, bad arguments) leaves C untouched and records the reason, readable
 * through fl_cuda_last_error() (fl_cuda.h).
 */
#ifndef FL_DEQUANTIZED_TENSOR_H
#define FL_DEQUANTIZED_TENSOR_H

#include <stdint.h>
#include <stddef.h>
#include "quant_types.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
    int8_t* weights;       /* [rows, cols] int8, row-major (host)          */
    float*  scales;        /* [rows] per-row scales (per-row mode)         */
    float*  f32_weights;   /* unused by the INT8 path; kept for layout     */
    int     rows;
    int     cols;
    int     original_bits;
    /* --- appended; absent from the reference struct --- */
    int       scale_block; /* 0 = per-row mode, 32 = per-32-block fp16 mode */
    uint16_t* scales_f16;  /* [rows, cols/32] fp16 bits (block mode)        */
    void*     dev;         /* device mirror (opaque), NULL until uploaded   */
} dequantized_tensor_t;

/* Reference dequantized_tensor.c:27-58: 4-bit blocks -> int8 (q-8)*16 with
 * the first block's scale as the per-row scale. Host-side; result is in
 * per-row mode (scale_block = 0). Returns NULL on bad input. */
dequantized_tensor_t* dequantized_from_q4(const quantized_tensor_t* q4_tensor);

/* Reference dequantized_tensor.c:60-84: 8-bit blocks -> int8 with the first
 * block's scale as the per-row scale. Per-row mode. NULL on bad input. */
dequantized_tensor_t* dequantized_from_q8(const quantized_tensor_t* q8_tensor);

/* Frees host arrays and the device mirror. NULL is accepted. */
void dequantized_tensor_free(dequantized_tensor_t* tensor);

/* C[M, N] = A[M, K] @ B[N, K]^T with B pre-dequantized int8.
 * A and C are HOST pointers (reference contract, dequantized_tensor.h:50);
 * B is uploaded to the device on first use. Runs the sm_100a INT8 GEMV/GEMM.
 * Returns silently on NULL arguments, like the reference (:206). */
void matmul_dequantized(const float* A, const dequantized_tensor_t* B,
                        float* C, int M, int N, int K);

/* Legacy aliases (reference dequantized_tensor.h:54-70). All three run the
 * same GPU kernel as matmul_dequantized. The reference's asm-style kernel
 * overwrites instead of accumulating (matmul_asm_style.c:106-113); that
 * defect is not reproduced. */
void matmul_dequantized_avx2(const float* A, const dequantized_tensor_t* B,
                             float* C, int M, int N, int K);
void matmul_dequantized_asm_style(const float* A, const dequantized_tensor_t* B,
                                  float* C, int M, int N, int K);
void matmul_dequantized_prefetch(const float* A, const dequantized_tensor_t* B,
                                 float* C, int M, int N, int K);

#ifdef __cplusplus
}
#endif

#endif /* FL_DEQUANTIZED_TENSOR_H */
