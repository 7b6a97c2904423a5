/*
 * Quantized block and tensor types consumed by the INT8 upload path.
 *
 * Layout-compatible with the reference's quant_types.h
 * (fast_llm/include/quant_types.h:16-58) so that a caller's existing
 * quantized_tensor_t / block_q4_t / block_q8_t buffers can be handed to
 * dequantized_from_q4 / dequantized_from_q8 unchanged. Only the types are
 * declared here: the reference's generic Q2/Q4/Q8 quantizers (quant.c) are
 * not part of the speculative-decoding path.
 *
 * The GGUF Q4_0 block (18 bytes: fp16 d + 16 bytes of nibbles) is declared
 * separately as block_q4_0_gguf; it is the format the synthetic weight
 * generator produces before pre-dequantization to INT8 in [-8, 7].
 */
#ifndef FL_QUANT_TYPES_H
#define FL_QUANT_TYPES_H

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

#define Q2_BLOCK_SIZE 256
#define Q4_BLOCK_SIZE 32
#define Q8_BLOCK_SIZE 32

/* 2-bit block: 256 weights packed 4 per byte, float scale + zero point. */
typedef struct {
    uint8_t qs[64];
    float scale;
    float zero_point;
} block_q2_t;

/* 4-bit block: 32 weights, element 2i in the low nibble of qs[i],
 * element 2i+1 in the high nibble (reference dequantized_tensor.c:48-50). */
typedef struct {
    uint8_t qs[16];
    float scale;
    float zero_point;
} block_q4_t;

/* 8-bit block: 32 signed weights and one float scale. */
typedef struct {
    int8_t qs[32];
    float scale;
} block_q8_t;

/* A matrix of quantized blocks, blocks laid out row-major. */
typedef struct {
    void* blocks;
    int n_blocks;
    int rows;
    int cols;
    int bits;
} quantized_tensor_t;

/* GGUF Q4_0 block as stored on disk by ggml: fp16 scale d, then 16 bytes
 * where byte i holds element i (low nibble) and element i+16 (high nibble).
 * Value of element j = (nibble_j - 8) * d. */
typedef struct {
    uint16_t d;
    uint8_t qs[16];
} block_q4_0_gguf;

#ifdef __cplusplus
}
#endif

#endif /* FL_QUANT_TYPES_H */
