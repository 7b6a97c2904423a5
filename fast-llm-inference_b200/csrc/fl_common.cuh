// Shared device helpers of the sm_100a speculative-decoding kernels.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <string.h>

#define FL_API extern "C" __attribute__((visibility("default")))

namespace fl {

// ---------------------------------------------------------------------------
// Programmatic dependent launch (PDL). Every kernel calls pdl_trigger() early
// so the next kernel in the stream can be scheduled and start streaming its
// weights, and pdl_wait() before it reads anything an earlier kernel wrote or
// writes anything an earlier kernel reads.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void pdl_trigger() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}

// ---------------------------------------------------------------------------
// Activation quantization, dequantized_tensor.c:112-135: one fused
// multiply-add x*127+128, conversion rounding to nearest even with the x86
// cvtps2dq out-of-range rule (NaN or |v| >= 2^31 gives INT32_MIN), then
// saturation to int16 and to [0, 255] -- net effect: clamp to [0, 255] with
// out-of-range values mapping to 0.
// ---------------------------------------------------------------------------
// y / 127 rounded to nearest even, as the reference's epilogue divides
// (dequantized_tensor.c:204-247), without a division instruction sequence:
// q0 = RN(y * r) with r = RN(1 / 127), one fused residual correction
// (Markstein's method for division by a constant: e = y - q0 * 127 is exact,
// q = RN(q0 + e * r)) and y's sign on a zero result. Equal to the correctly
// rounded quotient for every finite float y (all 2^32 inputs checked on the
// host; tests/test_div127.py checks whole binades).
#ifndef FL_DIV127_FMA
#define FL_DIV127_FMA 1
#endif
__device__ __forceinline__ float div127(float y) {
#if FL_DIV127_FMA
    const float r = 1.0f / 127.0f;
    const float q0 = __fmul_rn(y, r);
    const float e = __fmaf_rn(-q0, 127.0f, y);
    return copysignf(__fmaf_rn(e, r, q0), y);
#else
    return __fdiv_rn(y, 127.0f);
#endif
}

__device__ __forceinline__ uint32_t quant_u8(float x) {
    float v = __fmaf_rn(x, 127.0f, 128.0f);
    if (!(v > -2147483648.0f && v < 2147483648.0f)) return 0u;
    int i = __float2int_rn(v);
    i = i < 0 ? 0 : i;
    i = i > 255 ? 255 : i;
    return (uint32_t)i;
}

__device__ __forceinline__ uint32_t quant_pack4(float a, float b, float c, float d) {
    return quant_u8(a) | (quant_u8(b) << 8) | (quant_u8(c) << 16) | (quant_u8(d) << 24);
}

// u8 x s8 4-way dot into int32 (plain, no saturation): dp4a with an
// unsigned first and a signed second operand.
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t w, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(w), "r"(c));
    return d;
}

// dot_product_u8_i8's pair rule (dequantized_tensor.c:168-176) on one 32-bit
// word: (a0*w0 + a1*w1) and (a2*w2 + a3*w3) each saturated to int16.
__device__ __forceinline__ int dp4_pairsat(uint32_t a, uint32_t w, int c) {
    uint32_t a01 = __byte_perm(a, 0u, 0x4140);  // a0, 0, a1, 0 -> two u16
    uint32_t a23 = __byte_perm(a, 0u, 0x4342);  // a2, 0, a3, 0
    int p0 = __dp2a_lo((int)a01, (int)w, 0);    // a0*w0 + a1*w1
    int p1 = __dp2a_hi((int)a23, (int)w, 0);    // a2*w2 + a3*w3
    p0 = max(-32768, min(32767, p0));
    p1 = max(-32768, min(32767, p1));
    return c + p0 + p1;
}

// Reference polynomial sigmoid (activations_avx2.c:33-63), written in the
// order of its source: clamp to [-10, 10], exp(-x) ~ 1 - x + x^2/2 - x^3/6
// + x^4/24, sigma = 1 / (1 + that). No FMA contraction.
__device__ __forceinline__ float poly_sigmoid(float x) {
    x = fmaxf(-10.0f, fminf(10.0f, x));
    float nx = __fsub_rn(0.0f, x);
    float x2 = __fmul_rn(x, x);
    float x3 = __fmul_rn(x2, x);
    float x4 = __fmul_rn(x2, x2);
    float t = __fadd_rn(__fmul_rn(x3, -0.166667f), __fmul_rn(x4, 0.041667f));
    t = __fadd_rn(__fmul_rn(x2, 0.5f), t);
    t = __fadd_rn(nx, t);
    float p = __fadd_rn(1.0f, t);
    return __fdiv_rn(1.0f, __fadd_rn(1.0f, p));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ int warp_sum_i(int v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Exact float of an int with |v| < 2^22 using full-rate integer and float
// adds (the int->float conversion instruction runs at a fraction of the FMA
// rate): 0x4B400000 is 1.5 * 2^23, whose ulp is 1.
// Two floats in one 64-bit register and the sm_100 packed f32x2 arithmetic:
// each lane is rounded exactly like the scalar fma.rn / add.rn.
__device__ __forceinline__ unsigned long long f2_pack(float lo, float hi) {
    return ((unsigned long long)__float_as_uint(hi) << 32) | __float_as_uint(lo);
}
__device__ __forceinline__ unsigned long long f2_fma(unsigned long long a, unsigned long long b,
                                                     unsigned long long c) {
    unsigned long long d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
__device__ __forceinline__ unsigned long long f2_add(unsigned long long a, unsigned long long b) {
    unsigned long long d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
// i2f_exact of two ints (|v| < 2^22) as a packed pair.
__device__ __forceinline__ unsigned long long i2f2_exact(int lo, int hi) {
    const unsigned long long b = ((unsigned long long)(uint32_t)(hi + 0x4B400000) << 32) | (uint32_t)(lo + 0x4B400000);
    return f2_add(b, f2_pack(-12582912.0f, -12582912.0f));
}
__device__ __forceinline__ float f2_lo(unsigned long long v) { return __uint_as_float((uint32_t)v); }
__device__ __forceinline__ float f2_hi(unsigned long long v) { return __uint_as_float((uint32_t)(v >> 32)); }

__device__ __forceinline__ float i2f_exact(int v) {
    return __fsub_rn(__int_as_float(v + 0x4B400000), 12582912.0f);
}

// GEMV activation prologue: rows of f32 x (row stride K) -> u8 codes in
// shared memory, optionally after RMSNorm with unit weights
// (activations_avx2.c:108-143 then dequantized_tensor.c:112-135). Warp w
// handles rows w, w + nwarps, ...; K % 128 == 0.
__device__ __forceinline__ void act_prologue(uint8_t* act, const float* x, int K, int rows, int norm, float eps,
                                             int warp, int lane, int nwarps) {
    for (int m = warp; m < rows; m += nwarps) {
        const float* xr = x + (size_t)m * K;
        float scale = 1.0f;
        if (norm) {
            float s = 0.0f;
#pragma unroll 4
            for (int i = lane * 4; i < K; i += 128) {
                const float4 v = __ldcg(reinterpret_cast<const float4*>(xr + i));
                s = __fmaf_rn(v.x, v.x, s);
                s = __fmaf_rn(v.y, v.y, s);
                s = __fmaf_rn(v.z, v.z, s);
                s = __fmaf_rn(v.w, v.w, s);
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
            scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(s, (float)K), eps)));
        }
#pragma unroll 4
        for (int i = lane * 4; i < K; i += 128) {
            const float4 v = __ldcg(reinterpret_cast<const float4*>(xr + i));
            *reinterpret_cast<uint32_t*>(act + (size_t)m * K + i) =
                quant_pack4(__fmul_rn(v.x, scale), __fmul_rn(v.y, scale), __fmul_rn(v.z, scale),
                            __fmul_rn(v.w, scale));
        }
    }
}

// RMS-norm (optional) + u8 quantisation of `rows` <= MR rows (row m of x at
// x + m * K, of act at act + m * ald) by all NT threads of the calling group:
// thread t handles float4 columns t, t + NT, t + 2 NT, ... of every row. The
// sum of squares of a row is the per-thread sums (column order), a butterfly
// per warp, then the NT / 32 warp sums added in warp order, so the result
// depends on NT only. With CACHE and K / 4 <= NT * CPT all loads of all rows
// are issued at once and the values stay in registers for the quantisation
// (one round trip); otherwise columns go in batches of CPT and are loaded
// again to quantise. `red` holds MR * NT / 32 floats; the barrier is named
// barrier `bar_id` over the NT threads. The caller synchronises before
// reading `act`. Per element the arithmetic is that of act_prologue
// (activations_avx2.c:108-143, dequantized_tensor.c:112-135). Layout of
// `act`: row-major with row stride `ald`, or with CM the tensor-core
// core-matrix layout of 8 rows (16-byte column chunk c of rows 0..7 is 128
// contiguous bytes at c * 128; `ald` unused).
__device__ __forceinline__ size_t act_off(bool cm, int m, int c4, int ald) {
    return cm ? ((size_t)(c4 >> 2) * 128 + (size_t)m * 16 + 4 * (c4 & 3)) : ((size_t)m * ald + 4 * (size_t)c4);
}

template <int NT, int MR, int CPT, bool CACHE, bool CM = false>
__device__ __forceinline__ void act_prologue_cta(uint8_t* act, int ald, const float* x, int K, int rows, int norm,
                                                 float eps, float* red, int tid, int bar_id) {
    constexpr int NW = NT / 32;
    const int K4 = K >> 2;
    const float4* x4 = reinterpret_cast<const float4*>(x);
    float scale[MR];
#pragma unroll
    for (int m = 0; m < MR; m++) scale[m] = 1.0f;
    if (CACHE && K4 <= NT * CPT) {
        float4 v[MR][CPT];
#pragma unroll
        for (int m = 0; m < MR; m++)
#pragma unroll
            for (int j = 0; j < CPT; j++) {
                const int c = tid + j * NT;
                v[m][j] = (m < rows && c < K4) ? __ldcg(x4 + (size_t)m * K4 + c) : make_float4(0.f, 0.f, 0.f, 0.f);
            }
        if (norm) {
#pragma unroll
            for (int m = 0; m < MR; m++) {
                float s = 0.0f;
#pragma unroll
                for (int j = 0; j < CPT; j++) {
                    if (tid + j * NT < K4) {
                        s = __fmaf_rn(v[m][j].x, v[m][j].x, s);
                        s = __fmaf_rn(v[m][j].y, v[m][j].y, s);
                        s = __fmaf_rn(v[m][j].z, v[m][j].z, s);
                        s = __fmaf_rn(v[m][j].w, v[m][j].w, s);
                    }
                }
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
                if (m < rows && (tid & 31) == 0) red[m * NW + (tid >> 5)] = s;
            }
            asm volatile("bar.sync %0, %1;" ::"r"(bar_id), "n"(NT) : "memory");
#pragma unroll
            for (int m = 0; m < MR; m++) {
                if (m < rows) {
                    float tot = red[m * NW];
                    for (int w = 1; w < NW; w++) tot += red[m * NW + w];
                    scale[m] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)K), eps)));
                }
            }
        }
#pragma unroll
        for (int m = 0; m < MR; m++)
#pragma unroll
            for (int j = 0; j < CPT; j++) {
                const int c = tid + j * NT;
                if (m < rows && c < K4)
                    *reinterpret_cast<uint32_t*>(act + act_off(CM, m, c, ald)) =
                        quant_pack4(__fmul_rn(v[m][j].x, scale[m]), __fmul_rn(v[m][j].y, scale[m]),
                                    __fmul_rn(v[m][j].z, scale[m]), __fmul_rn(v[m][j].w, scale[m]));
            }
        return;
    }
    if (norm) {
        float s[MR];
#pragma unroll
        for (int m = 0; m < MR; m++) s[m] = 0.0f;
        for (int c0 = tid; c0 < K4; c0 += NT * CPT) {
            // unrolled: the loads carry no dependence and are issued first
#pragma unroll
            for (int j = 0; j < CPT; j++)
#pragma unroll
                for (int m = 0; m < MR; m++)
                    if (m < rows && c0 + j * NT < K4) {
                        const float4 v = __ldcg(x4 + (size_t)m * K4 + c0 + j * NT);
                        s[m] = __fmaf_rn(v.x, v.x, s[m]);
                        s[m] = __fmaf_rn(v.y, v.y, s[m]);
                        s[m] = __fmaf_rn(v.z, v.z, s[m]);
                        s[m] = __fmaf_rn(v.w, v.w, s[m]);
                    }
        }
#pragma unroll
        for (int m = 0; m < MR; m++) {
            if (m < rows) {
                float t = s[m];
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
                if ((tid & 31) == 0) red[m * NW + (tid >> 5)] = t;
            }
        }
        asm volatile("bar.sync %0, %1;" ::"r"(bar_id), "n"(NT) : "memory");
#pragma unroll
        for (int m = 0; m < MR; m++) {
            if (m < rows) {
                float tot = red[m * NW];
                for (int w = 1; w < NW; w++) tot += red[m * NW + w];
                scale[m] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)K), eps)));
            }
        }
    }
    for (int c0 = tid; c0 < K4; c0 += NT * CPT) {
#pragma unroll
        for (int j = 0; j < CPT; j++)
#pragma unroll
            for (int m = 0; m < MR; m++)
                if (m < rows && c0 + j * NT < K4) {
                    const float4 v = __ldcg(x4 + (size_t)m * K4 + c0 + j * NT);
                    *reinterpret_cast<uint32_t*>(act + act_off(CM, m, c0 + j * NT, ald)) =
                        quant_pack4(__fmul_rn(v.x, scale[m]), __fmul_rn(v.y, scale[m]), __fmul_rn(v.z, scale[m]),
                                    __fmul_rn(v.w, scale[m]));
                }
    }
}

// act_prologue_cta with the row count rounded up to 1, 2, 4 or 8 (at most
// MMAX); CACHE keeps up to 24 float4 per thread in registers.
template <int NT, int MMAX, bool CACHE, bool CM = false>
__device__ __forceinline__ void act_prologue_rows(uint8_t* act, int ald, const float* x, int K, int rows, int norm,
                                                  float eps, float* red, int tid, int bar_id) {
    if (rows <= 1 || MMAX == 1)
        act_prologue_cta<NT, 1, (CACHE ? 12 : 8), CACHE, CM>(act, ald, x, K, rows, norm, eps, red, tid, bar_id);
    else if (rows <= 2 || MMAX == 2)
        act_prologue_cta<NT, 2, (CACHE ? 6 : 4), CACHE, CM>(act, ald, x, K, rows, norm, eps, red, tid, bar_id);
    else if (rows <= 4 || MMAX == 4)
        act_prologue_cta<NT, 4, (CACHE ? 3 : 2), CACHE, CM>(act, ald, x, K, rows, norm, eps, red, tid, bar_id);
    else
        act_prologue_cta<NT, (MMAX < 8 ? MMAX : 8), (CACHE ? 3 : 1), CACHE, CM>(act, ald, x, K, rows, norm, eps, red,
                                                                               tid, bar_id);
}

// Streaming 16-byte load that bypasses L1 allocation (weights are read once).
__device__ __forceinline__ uint4 ld_stream16(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

// Orderable 64-bit key for a deterministic argmax: larger value wins, ties go
// to the lower index (inference.c:104-111 keeps the first maximum).
__host__ __device__ __forceinline__ unsigned long long argmax_key(float v, int idx) {
#ifdef __CUDA_ARCH__
    uint32_t b = __float_as_uint(v);
#else
    uint32_t b;
    memcpy(&b, &v, sizeof(b));
#endif
    b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
    return ((unsigned long long)b << 32) | (uint32_t)(0x7fffffff - idx);
}
__host__ __device__ __forceinline__ int argmax_key_index(unsigned long long k) {
    return 0x7fffffff - (int)(uint32_t)(k & 0xffffffffu);
}
__device__ __forceinline__ float argmax_key_value(unsigned long long k) {
    uint32_t b = (uint32_t)(k >> 32);
    b = (b & 0x80000000u) ? (b & 0x7fffffffu) : ~b;
    return __uint_as_float(b);
}

}  // namespace fl
