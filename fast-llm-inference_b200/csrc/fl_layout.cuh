// Device layout of INT8 weights for the TMA-ring GEMV ("tiled" layout).
//
// A [N, K] int8 matrix is cut along K into panels of width P (a divisor of
// K that is a multiple of 128: the widest up to FL_PANEL_MAX bytes for the
// TMA-ring GEMV, 128 for the tcgen05 step kernel). Panel p is stored as a row-major [N, P] block, so R consecutive rows
// of one panel are contiguous: one 1-D bulk copy moves a whole ring stage.
// Inside a row the 16-byte chunks of every 128-byte group are XOR-swizzled
// by (row & 7): chunk c of row n sits at chunk (c & ~7) | ((c & 7) ^ (n & 7)).
// Eight consecutive rows read at the same logical chunk therefore hit eight
// different shared-memory bank groups (ldmatrix / per-lane loads are
// conflict-free) while a warp sweeping one row still reads 32 distinct
// chunks. The fp16 block scales use the same panels, row-major [N, P/32],
// unswizzled.
#pragma once

#include <stddef.h>
#include <stdint.h>

namespace fl {

#ifndef FL_PANEL_MAX
#define FL_PANEL_MAX 4096
#endif
// Panel width of the tcgen05 step kernel: 128-byte rows are the SWIZZLE_128B
// K-major operand layout.
constexpr int kStepPanel = 128;

// Widest divisor of K that is a multiple of 128 and at most pmax.
__host__ __device__ inline int panel_width(int K, int pmax = FL_PANEL_MAX) {
    if (K <= 0 || K % 128) return 0;
    for (int n = 1; n <= K / 128; n++)
        if (K % n == 0 && (K / n) <= pmax && (K / n) % 128 == 0) return K / n;
    return 0;
}

// Byte offset of logical 16-byte chunk c (bytes [16c, 16c+16) of row n).
__host__ __device__ __forceinline__ size_t tiled_w_off(int N, int P, int n, int c) {
    const int cpp = P >> 4;
    const int p = c / cpp;
    const int cc = c - p * cpp;
    const int phys = (cc & ~7) | ((cc & 7) ^ (n & 7));
    return ((size_t)p * N + n) * (size_t)P + (size_t)phys * 16;
}

// Element offset of the fp16 scale of 32-element block b of row n.
__host__ __device__ __forceinline__ size_t tiled_s_off(int N, int P, int n, int b) {
    const int bpp = P >> 5;
    const int p = b / bpp;
    const int bb = b - p * bpp;
    return ((size_t)p * N + n) * (size_t)bpp + bb;
}

// 4-bit tiled layout (w4.cu): byte offset of the 16-byte chunk of 32-element
// block b of row n; panels of P columns are P / 2 bytes per row, chunks
// swizzled like the INT8 layout's.
__host__ __device__ __forceinline__ size_t tiled_w4_off(int N, int P, int n, int b) {
    const int bpp = P >> 5;
    const int p = b / bpp;
    const int bb = b - p * bpp;
    const int phys = (bb & ~7) | ((bb & 7) ^ (n & 7));
    return ((size_t)p * N + n) * (size_t)(P >> 1) + (size_t)phys * 16;
}

// Physical chunk of logical chunk cc (within a panel row) for row n.
__host__ __device__ __forceinline__ int swz_chunk(int cc, int n) { return (cc & ~7) | ((cc & 7) ^ (n & 7)); }

}  // namespace fl
