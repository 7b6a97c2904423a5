// Seeded synthetic weights: N(0, std) -> GGUF Q4_0 -> INT8 [-8, 7] + fp16
// block scales, and the GGUF Q4_0 -> INT8 load-time conversion. Host code.
//
// Normals come from Philox4x32-10 (Salmon, Moraes, Dror, Shaw, "Parallel
// random numbers: as easy as 1, 2, 3", SC'11) keyed by the seed, with the
// counter (element / 4, tensor id), turned into normals by Box-Muller in
// double precision. Every element is a pure function of (seed, tensor id,
// index), so the result does not depend on the thread count.
#include <cuda_fp16.h>
#include <math.h>
#include <stdint.h>
#include <string.h>

#include "fl_common.cuh"
#include "fl_cuda.h"

namespace {

inline void philox(const uint32_t ctr[4], const uint32_t key[2], uint32_t out[4]) {
    uint32_t c0 = ctr[0], c1 = ctr[1], c2 = ctr[2], c3 = ctr[3];
    uint32_t k0 = key[0], k1 = key[1];
    for (int r = 0; r < 10; r++) {
        const uint64_t p0 = (uint64_t)0xD2511F53u * c0;
        const uint64_t p1 = (uint64_t)0xCD9E8D57u * c2;
        const uint32_t hi0 = (uint32_t)(p0 >> 32), lo0 = (uint32_t)p0;
        const uint32_t hi1 = (uint32_t)(p1 >> 32), lo1 = (uint32_t)p1;
        c0 = hi1 ^ c1 ^ k0;
        c1 = lo1;
        c2 = hi0 ^ c3 ^ k1;
        c3 = lo0;
        k0 += 0x9E3779B9u;
        k1 += 0xBB67AE85u;
    }
    out[0] = c0; out[1] = c1; out[2] = c2; out[3] = c3;
}

inline double unit_open(uint32_t x) { return ((double)(x >> 8) + 0.5) * (1.0 / 16777216.0); }

// Four consecutive normals starting at element 4*g.
inline void normals4(uint64_t seed, uint32_t tid, uint64_t g, double z[4]) {
    const uint32_t ctr[4] = {(uint32_t)g, (uint32_t)(g >> 32), tid, 0x5EEDu};
    const uint32_t key[2] = {(uint32_t)seed, (uint32_t)(seed >> 32)};
    uint32_t o[4];
    philox(ctr, key, o);
    const double two_pi = 6.283185307179586476925;
    for (int h = 0; h < 2; h++) {
        const double r = sqrt(-2.0 * log(unit_open(o[2 * h])));
        const double t = two_pi * unit_open(o[2 * h + 1]);
        z[2 * h] = r * cos(t);
        z[2 * h + 1] = r * sin(t);
    }
}

inline void normal_row(uint64_t seed, uint32_t tid, uint64_t start, int n, float std, float* out) {
    // start is a multiple of 4 whenever cols % 32 == 0
    double z[4];
    uint64_t g = start >> 2;
    int off = (int)(start & 3);
    int i = 0;
    while (i < n) {
        normals4(seed, tid, g, z);
        for (int l = off; l < 4 && i < n; l++, i++) out[i] = (float)(z[l] * (double)std);
        off = 0;
        g++;
    }
}

inline uint16_t f32_to_f16_bits(float f) { return __half_as_ushort(__float2half_rn(f)); }
inline float f16_bits_to_f32(uint16_t h) { return __half2float(__ushort_as_half(h)); }

// ggml's quantize_row_q4_0_ref rule for one block of 32 values.
inline void q4_0_block(const float* x, int8_t* w, uint16_t* d) {
    float amax = 0.0f, vmax = 0.0f;
    for (int j = 0; j < 32; j++) {
        const float a = fabsf(x[j]);
        if (amax < a) { amax = a; vmax = x[j]; }
    }
    const float dd = vmax / -8.0f;
    const float id = dd != 0.0f ? 1.0f / dd : 0.0f;
    *d = f32_to_f16_bits(dd);
    for (int j = 0; j < 32; j++) {
        int q = (int)(int8_t)(x[j] * id + 8.5f);
        if (q > 15) q = 15;
        w[j] = (int8_t)(q - 8);
    }
}

}  // namespace

FL_API void fl_philox4x32_10(const uint32_t ctr[4], const uint32_t key[2], uint32_t out[4]) {
    philox(ctr, key, out);
}

FL_API int fl_synth_normal(uint64_t seed, uint32_t tensor_id, size_t count, float std, float* out) {
    if (!out) return FL_E_INVAL;
    const int64_t chunks = (int64_t)((count + 4095) / 4096);
#pragma omp parallel for schedule(static)
    for (int64_t c = 0; c < chunks; c++) {
        const uint64_t s = (uint64_t)c * 4096;
        const int n = (int)((count - s) < 4096 ? (count - s) : 4096);
        normal_row(seed, tensor_id, s, n, std, out + s);
    }
    return FL_OK;
}

FL_API int fl_synth_q4_0_i8(uint64_t seed, uint32_t tensor_id, int rows, int cols, float std, int8_t* w,
                            uint16_t* d) {
    if (!w || !d || rows <= 0 || cols <= 0 || cols % 32 != 0) return FL_E_INVAL;
#pragma omp parallel
    {
        float* buf = new float[cols];
#pragma omp for schedule(static)
        for (int r = 0; r < rows; r++) {
            normal_row(seed, tensor_id, (uint64_t)r * cols, cols, std, buf);
            for (int b = 0; b < cols / 32; b++)
                q4_0_block(buf + 32 * b, w + (size_t)r * cols + 32 * b, d + (size_t)r * (cols / 32) + b);
        }
        delete[] buf;
    }
    return FL_OK;
}

FL_API int fl_synth_q4_0_i8_block(uint64_t seed, uint32_t tensor_id, int rows, int cols, int r0, int nr, int c0, int nc,
                                  float std, int8_t* w, uint16_t* d) {
    if (!w || !d || rows <= 0 || cols <= 0 || cols % 32 != 0 || r0 < 0 || nr <= 0 || r0 + nr > rows || c0 < 0 ||
        nc <= 0 || c0 + nc > cols || c0 % 32 != 0 || nc % 32 != 0)
        return FL_E_INVAL;
#pragma omp parallel
    {
        float* buf = new float[nc];
#pragma omp for schedule(static)
        for (int r = 0; r < nr; r++) {
            normal_row(seed, tensor_id, (uint64_t)(r0 + r) * cols + c0, nc, std, buf);
            for (int b = 0; b < nc / 32; b++)
                q4_0_block(buf + 32 * b, w + (size_t)r * nc + 32 * b, d + (size_t)r * (nc / 32) + b);
        }
        delete[] buf;
    }
    return FL_OK;
}

FL_API int fl_synth_q4_0_f32(uint64_t seed, uint32_t tensor_id, int rows, int cols, float std, float* out) {
    if (!out || rows <= 0 || cols <= 0 || cols % 32 != 0) return FL_E_INVAL;
#pragma omp parallel
    {
        float* buf = new float[cols];
        int8_t* w = new int8_t[cols];
        uint16_t* d = new uint16_t[cols / 32];
#pragma omp for schedule(static)
        for (int r = 0; r < rows; r++) {
            normal_row(seed, tensor_id, (uint64_t)r * cols, cols, std, buf);
            for (int b = 0; b < cols / 32; b++) q4_0_block(buf + 32 * b, w + 32 * b, d + b);
            float* o = out + (size_t)r * cols;
            for (int i = 0; i < cols; i++) o[i] = (float)w[i] * f16_bits_to_f32(d[i / 32]);
        }
        delete[] buf;
        delete[] w;
        delete[] d;
    }
    return FL_OK;
}

FL_API int fl_q4_0_to_i8(const block_q4_0_gguf* blocks, int rows, int cols, int8_t* w, uint16_t* d) {
    if (!blocks || !w || !d || rows <= 0 || cols <= 0 || cols % 32 != 0) return FL_E_INVAL;
    const int nb = cols / 32;
#pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; r++) {
        for (int b = 0; b < nb; b++) {
            const block_q4_0_gguf& blk = blocks[(size_t)r * nb + b];
            int8_t* o = w + (size_t)r * cols + 32 * b;
            for (int i = 0; i < 16; i++) {
                o[i] = (int8_t)((blk.qs[i] & 0x0F) - 8);
                o[i + 16] = (int8_t)((blk.qs[i] >> 4) - 8);
            }
            d[(size_t)r * nb + b] = blk.d;
        }
    }
    return FL_OK;
}
