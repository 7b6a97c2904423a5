/*
 * CPU oracle for the speculative-decoding hot path -- TEST INFRASTRUCTURE.
 * Used only by tests/, the smoke() check and the CPU-baseline leg of
 * bench.py, never by the product library. See oracle.h for the contract.
 *
 * Build: oracle/Makefile (-O2 -mavx2 -mfma -fopenmp -ffp-contract=off: every
 * float operation happens in the order written here; FMAs only where the
 * reference issues one explicitly).
 */
#include "oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#include <float.h>
#include <time.h>
#include <immintrin.h>

static double g_last_decode_s = 0.0;

static double now_s(void) {
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return ts.tv_sec + ts.tv_nsec * 1e-9;
}

double orc_last_decode_seconds(void) { return g_last_decode_s; }

/* ------------------------------------------------------------------ */
/* fp16 conversion (IEEE binary16)                                     */
/* ------------------------------------------------------------------ */

float orc_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1Fu;
    uint32_t man = h & 0x3FFu;
    uint32_t bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else { /* subnormal: renormalise */
            int e = -1;
            do { man <<= 1; e++; } while ((man & 0x400u) == 0);
            man &= 0x3FFu;
            bits = sign | ((uint32_t)(127 - 15 - e) << 23) | (man << 13);
        }
    } else if (exp == 31) {
        bits = sign | 0x7F800000u | (man << 13);
    } else {
        bits = sign | ((exp + 127 - 15) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

uint16_t orc_f32_to_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t absx = x & 0x7FFFFFFFu;
    if (absx >= 0x7F800000u) /* inf / nan */
        return (uint16_t)(sign | 0x7C00u | (absx > 0x7F800000u ? 0x200u : 0u));
    if (absx >= 0x477FF000u) /* rounds to >= 65520: inf */
        return (uint16_t)(sign | 0x7C00u);
    uint32_t e = absx >> 23;
    uint32_t m = (absx & 0x7FFFFFu) | 0x800000u;
    uint32_t shift, q;
    if (absx < 0x38800000u) {          /* half subnormal: q = |f| / 2^-24 */
        if (absx < 0x33000000u) return (uint16_t)sign;
        shift = 126u - e;              /* 14 .. 24 */
        q = m >> shift;
    } else {                           /* half normal */
        shift = 13u;
        q = ((e - 112u) << 10) | ((m & 0x7FFFFFu) >> 13);
    }
    uint32_t rem = m & ((1u << shift) - 1u);
    uint32_t half = 1u << (shift - 1u);
    if (rem > half || (rem == half && (q & 1u))) q++;
    return (uint16_t)(sign | q);
}

/* ------------------------------------------------------------------ */
/* activation quantization and dots                                    */
/* ------------------------------------------------------------------ */

/* cvtps2dq: round to nearest even; NaN or |v| >= 2^31 -> INT32_MIN. */
static inline int32_t cvt_rne_x86(float v) {
    if (!(v > -2147483648.0f && v < 2147483648.0f)) return INT32_MIN;
    return (int32_t)nearbyintf(v);
}

static inline uint8_t quant_one(float x) {
    int32_t i = cvt_rne_x86(fmaf(x, 127.0f, 128.0f));
    /* packs_epi32 saturates to int16, packus_epi16 to [0, 255]. */
    if (i < -32768) i = -32768;
    if (i > 32767) i = 32767;
    if (i < 0) i = 0;
    if (i > 255) i = 255;
    return (uint8_t)i;
}

void orc_quant_u8(const float* x, uint8_t* q, int n) {
    for (int i = 0; i < n; i++) q[i] = quant_one(x[i]);
}

int32_t orc_dot_pairsat(const uint8_t* a, const int8_t* w, int n) {
    int32_t s = 0;
    for (int j = 0; j < n; j += 2) {
        int32_t p = (int32_t)a[j] * w[j] + (int32_t)a[j + 1] * w[j + 1];
        if (p > 32767) p = 32767;
        if (p < -32768) p = -32768;
        s += p;
    }
    return s;
}

int32_t orc_dot_plain(const uint8_t* a, const int8_t* w, int n) {
    int32_t s = 0;
    for (int j = 0; j < n; j++) s += (int32_t)a[j] * w[j];
    return s;
}

/* AVX2 block dot (32 bytes): maddubs (pair-saturating) + madd + hsum. The
 * pair sums of [-8,7] weights never saturate, so this equals the plain dot. */
static inline int32_t block_dot32(const uint8_t* a, const int8_t* w) {
    __m256i va = _mm256_loadu_si256((const __m256i*)a);
    __m256i vw = _mm256_loadu_si256((const __m256i*)w);
    __m256i p16 = _mm256_maddubs_epi16(va, vw);
    __m256i p32 = _mm256_madd_epi16(p16, _mm256_set1_epi16(1));
    __m128i s = _mm_add_epi32(_mm256_castsi256_si128(p32), _mm256_extracti128_si256(p32, 1));
    s = _mm_hadd_epi32(s, s);
    s = _mm_hadd_epi32(s, s);
    return _mm_cvtsi128_si32(s);
}

void orc_matmul_rowscale(const float* A, const int8_t* W, const float* scales,
                         float* C, int M, int N, int K) {
    uint8_t* q = (uint8_t*)malloc((size_t)M * K);
    for (int m = 0; m < M; m++) orc_quant_u8(A + (size_t)m * K, q + (size_t)m * K, K);
#pragma omp parallel for schedule(static)
    for (int n = 0; n < N; n++) {
        const int8_t* wr = W + (size_t)n * K;
        for (int m = 0; m < M; m++) {
            int32_t dot = orc_dot_pairsat(q + (size_t)m * K, wr, K);
            /* the reference's `/ (127 * 16.0f)` compiled with -ffast-math is a
             * multiply by the rounded reciprocal (bit-exact with libref). */
            C[(size_t)m * N + n] = ((float)dot * scales[n]) * (1.0f / 2032.0f);
        }
    }
    free(q);
}

/* The block dots of eight weight rows (stride K) against one activation
 * block, lane r = row r: the maddubs + madd sums of block_dot32. */
static inline __m256i rows_dots8(const __m256i va, const __m256i* w) {
    const __m256i one = _mm256_set1_epi16(1);
    __m256i p[8];
    for (int r = 0; r < 8; r++) p[r] = _mm256_madd_epi16(_mm256_maddubs_epi16(va, w[r]), one);
    const __m256i s01 = _mm256_hadd_epi32(p[0], p[1]), s23 = _mm256_hadd_epi32(p[2], p[3]);
    const __m256i s45 = _mm256_hadd_epi32(p[4], p[5]), s67 = _mm256_hadd_epi32(p[6], p[7]);
    const __m256i s0123 = _mm256_hadd_epi32(s01, s23), s4567 = _mm256_hadd_epi32(s45, s67);
    return _mm256_add_epi32(_mm256_permute2x128_si256(s0123, s4567, 0x20),
                            _mm256_permute2x128_si256(s0123, s4567, 0x31));
}

/* Per block: t = (float)dot * scale (one rounding), acc = acc + t in block
 * order (matmul_dequantized's per-row accumulation, one scale per block),
 * C = acc / 127. Eight weight rows go through in the lanes of one vector and
 * up to four activation rows share each weight load; every lane still adds
 * its row's blocks one at a time in block order, so the result is that of
 * the one-block-at-a-time loop. Rows past the last multiple of 8 take that
 * loop directly. */
static void matmul_block_q(const uint8_t* q, const int8_t* W, const uint16_t* S,
                           float* C, int M, int N, int K) {
    const int nb = K / 32;
    const int N8 = N & ~7;
#pragma omp parallel
    {
        float* sf = (float*)malloc(sizeof(float) * (size_t)nb * 8);
#pragma omp for schedule(static)
        for (int n = 0; n < N8; n += 8) {
            for (int b = 0; b < nb; b++)
                for (int r = 0; r < 8; r++) sf[b * 8 + r] = orc_f16_to_f32(S[(size_t)(n + r) * nb + b]);
            const int8_t* wr = W + (size_t)n * K;
            for (int m0 = 0; m0 < M; m0 += 4) {
                const int mc = M - m0 < 4 ? M - m0 : 4;
                __m256 acc[4] = {_mm256_setzero_ps(), _mm256_setzero_ps(), _mm256_setzero_ps(),
                                 _mm256_setzero_ps()};
                for (int b = 0; b < nb; b++) {
                    __m256i w8[8];
                    for (int r = 0; r < 8; r++)
                        w8[r] = _mm256_loadu_si256((const __m256i*)(wr + (size_t)r * K + 32 * b));
                    const __m256 sc = _mm256_loadu_ps(sf + 8 * b);
                    for (int i = 0; i < mc; i++) {
                        const __m256i va = _mm256_loadu_si256((const __m256i*)(q + (size_t)(m0 + i) * K + 32 * b));
                        const __m256 t = _mm256_mul_ps(_mm256_cvtepi32_ps(rows_dots8(va, w8)), sc);
                        acc[i] = _mm256_add_ps(acc[i], t);
                    }
                }
                const __m256 d127 = _mm256_set1_ps(127.0f);
                for (int i = 0; i < mc; i++)
                    _mm256_storeu_ps(C + (size_t)(m0 + i) * N + n, _mm256_div_ps(acc[i], d127));
            }
        }
        free(sf);
    }
    for (int n = N8; n < N; n++) {
        const int8_t* wr = W + (size_t)n * K;
        const uint16_t* sr = S + (size_t)n * nb;
        for (int m = 0; m < M; m++) {
            const uint8_t* qa = q + (size_t)m * K;
            float acc = 0.0f;
            for (int b = 0; b < nb; b++) {
                const float t = (float)block_dot32(qa + 32 * b, wr + 32 * b) * orc_f16_to_f32(sr[b]);
                acc = acc + t;
            }
            C[(size_t)m * N + n] = acc / 127.0f;
        }
    }
}

/* The same rule over weights packed for 8-lane integer dots: rows in groups
 * of 8, and for each block of a group eight 32-byte chunks, chunk c holding
 * 4 consecutive weights of each of the 8 rows (byte 4r + j = row r, column
 * 32b + 4c + j). One maddubs of a chunk against 4 activation bytes repeated
 * 8 times gives, in int16 lanes 2r and 2r+1, row r's two pair sums; the
 * eight chunks of a block add up in int16 without overflow because every
 * weight is in [-8, 7] (16 products of at most 255 * 8 = 2040), and one madd
 * with ones then leaves row r's block dot in int32 lane r. Scales are packed
 * the same way as f32 ([group][block][8]). Only the order of the integer
 * adds differs from matmul_block_q, so every block dot, product and sum is
 * the same. */
int orc_pack_rows8(const int8_t* W, const uint16_t* S, int N, int K, int8_t* wp, float* sp) {
    if (N % 8 || K % 32) return -1;
    const int nb = K / 32;
    for (size_t i = 0; i < (size_t)N * K; i++)
        if (W[i] < -8 || W[i] > 7) return -1;
#pragma omp parallel for schedule(static)
    for (int g = 0; g < N / 8; g++)
        for (int b = 0; b < nb; b++) {
            int8_t* dst = wp + ((size_t)g * nb + b) * 256;
            for (int c = 0; c < 8; c++)
                for (int r = 0; r < 8; r++)
                    for (int j = 0; j < 4; j++)
                        dst[c * 32 + 4 * r + j] = W[(size_t)(8 * g + r) * K + 32 * b + 4 * c + j];
            for (int r = 0; r < 8; r++)
                sp[((size_t)g * nb + b) * 8 + r] = orc_f16_to_f32(S[(size_t)(8 * g + r) * nb + b]);
        }
    return 0;
}

static void matmul_packed_q(const uint8_t* q, const int8_t* wp, const float* sp, float* C, int M, int N, int K) {
    const int nb = K / 32;
    const __m256i one = _mm256_set1_epi16(1);
    const __m256 d127 = _mm256_set1_ps(127.0f);
#pragma omp parallel for schedule(static)
    for (int g = 0; g < N / 8; g++) {
        for (int m0 = 0; m0 < M; m0 += 4) {
            const int mc = M - m0 < 4 ? M - m0 : 4;
            __m256 acc[4] = {_mm256_setzero_ps(), _mm256_setzero_ps(), _mm256_setzero_ps(), _mm256_setzero_ps()};
            for (int b = 0; b < nb; b++) {
                const int8_t* wb = wp + ((size_t)g * nb + b) * 256;
                __m256i w8[8];
                for (int c = 0; c < 8; c++) w8[c] = _mm256_loadu_si256((const __m256i*)(wb + 32 * c));
                const __m256 sc = _mm256_loadu_ps(sp + ((size_t)g * nb + b) * 8);
                for (int i = 0; i < mc; i++) {
                    const uint8_t* qa = q + (size_t)(m0 + i) * K + 32 * b;
                    __m256i s16 = _mm256_setzero_si256();
                    for (int c = 0; c < 8; c++) {
                        int32_t a4;
                        memcpy(&a4, qa + 4 * c, 4);
                        s16 = _mm256_add_epi16(s16, _mm256_maddubs_epi16(_mm256_set1_epi32(a4), w8[c]));
                    }
                    const __m256 t = _mm256_mul_ps(_mm256_cvtepi32_ps(_mm256_madd_epi16(s16, one)), sc);
                    acc[i] = _mm256_add_ps(acc[i], t);
                }
            }
            for (int i = 0; i < mc; i++)
                _mm256_storeu_ps(C + (size_t)(m0 + i) * N + 8 * g, _mm256_div_ps(acc[i], d127));
        }
    }
}

void orc_matmul_packed(const float* A, const int8_t* wp, const float* sp, float* C, int M, int N, int K) {
    uint8_t* q = (uint8_t*)malloc((size_t)M * K);
    for (int m = 0; m < M; m++) orc_quant_u8(A + (size_t)m * K, q + (size_t)m * K, K);
    matmul_packed_q(q, wp, sp, C, M, N, K);
    free(q);
}

void orc_matmul_block(const float* A, const int8_t* W, const uint16_t* scales,
                      float* C, int M, int N, int K) {
    uint8_t* q = (uint8_t*)malloc((size_t)M * K);
    for (int m = 0; m < M; m++) orc_quant_u8(A + (size_t)m * K, q + (size_t)m * K, K);
    matmul_block_q(q, W, scales, C, M, N, K);
    free(q);
}

void orc_block_dots(const float* A, const int8_t* W, int32_t* D, int M, int N, int K) {
    const int nb = K / 32;
    uint8_t* q = (uint8_t*)malloc((size_t)M * K);
    for (int m = 0; m < M; m++) orc_quant_u8(A + (size_t)m * K, q + (size_t)m * K, K);
    for (int m = 0; m < M; m++)
        for (int n = 0; n < N; n++)
            for (int b = 0; b < nb; b++)
                D[((size_t)m * N + n) * nb + b] =
                    orc_dot_pairsat(q + (size_t)m * K + 32 * b, W + (size_t)n * K + 32 * b, 32);
    free(q);
}

/* ------------------------------------------------------------------ */
/* norm / activations / rope                                           */
/* ------------------------------------------------------------------ */

void orc_rmsnorm(const float* x, float* out, int n, float eps) {
    float lane[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    int i = 0;
    for (; i <= n - 8; i += 8)
        for (int j = 0; j < 8; j++) lane[j] = fmaf(x[i + j], x[i + j], lane[j]);
    /* Horizontal sum in the order the reference build reduces the vector
     * (high/low 128-bit halves, then pairs). The reference binary computes
     * 1/sqrtf with rsqrtss plus one Newton step under -ffast-math, which is
     * CPU-model dependent; the exact expression of the source is used here
     * and the two agree within a few ulp. */
    float s = ((lane[0] + lane[4]) + (lane[2] + lane[6])) + ((lane[1] + lane[5]) + (lane[3] + lane[7]));
    for (; i < n; i++) s += x[i] * x[i];
    float scale = 1.0f / sqrtf(s / (float)n + eps);
    for (i = 0; i < n; i++) out[i] = x[i] * scale;
}

float orc_fast_sigmoid(float x) {
    x = fmaxf(-10.0f, fminf(10.0f, x));
    float nx = 0.0f - x;
    float x2 = x * x;
    float x3 = x2 * x;
    float x4 = x2 * x2;
    float p = 1.0f + (nx + (x2 * 0.5f + (x3 * -0.166667f + x4 * 0.041667f)));
    return 1.0f / (1.0f + p);
}

void orc_swiglu(const float* g, const float* u, float* out, int n) {
    for (int i = 0; i < n; i++) {
        float s = orc_fast_sigmoid(g[i]);
        out[i] = (g[i] * s) * u[i];
    }
}

void orc_silu(const float* x, float* out, int n) {
    for (int i = 0; i < n; i++) out[i] = x[i] * orc_fast_sigmoid(x[i]);
}

void orc_rope_vec(float* v, int heads, int head_dim, int pos, float theta) {
    for (int h = 0; h < heads; h++) {
        float* p = v + (size_t)h * head_dim;
        for (int i = 0; i < head_dim; i += 2) {
            float freq = 1.0f / powf(theta, (float)i / (float)head_dim);
            float ang = (float)pos * freq;
            float c = cosf(ang), s = sinf(ang);
            float a = p[i], b = p[i + 1];
            p[i] = a * c - b * s;
            p[i + 1] = a * s + b * c;
        }
    }
}

/* ------------------------------------------------------------------ */
/* Q4_0 and Philox                                                     */
/* ------------------------------------------------------------------ */

void orc_q4_0_quantize_i8(const float* x, int n, int8_t* w, uint16_t* d) {
    for (int b = 0; b < n / 32; b++) {
        const float* xb = x + 32 * b;
        float amax = 0.0f, vmax = 0.0f;
        for (int j = 0; j < 32; j++) {
            float a = fabsf(xb[j]);
            if (amax < a) { amax = a; vmax = xb[j]; }
        }
        float dd = vmax / -8.0f;
        float id = dd != 0.0f ? 1.0f / dd : 0.0f;
        d[b] = orc_f32_to_f16(dd);
        for (int j = 0; j < 32; j++) {
            int q = (int)(int8_t)(xb[j] * id + 8.5f);
            if (q > 15) q = 15;
            w[32 * b + j] = (int8_t)(q - 8);
        }
    }
}

static inline void mulhilo32(uint32_t a, uint32_t b, uint32_t* hi, uint32_t* lo) {
    uint64_t p = (uint64_t)a * b;
    *hi = (uint32_t)(p >> 32);
    *lo = (uint32_t)p;
}

void orc_philox4x32_10(const uint32_t ctr[4], const uint32_t key[2], uint32_t out[4]) {
    uint32_t c0 = ctr[0], c1 = ctr[1], c2 = ctr[2], c3 = ctr[3];
    uint32_t k0 = key[0], k1 = key[1];
    for (int r = 0; r < 10; r++) {
        uint32_t hi0, lo0, hi1, lo1;
        mulhilo32(0xD2511F53u, c0, &hi0, &lo0);
        mulhilo32(0xCD9E8D57u, c2, &hi1, &lo1);
        uint32_t n0 = hi1 ^ c1 ^ k0, n1 = lo1, n2 = hi0 ^ c3 ^ k1, n3 = lo0;
        c0 = n0; c1 = n1; c2 = n2; c3 = n3;
        k0 += 0x9E3779B9u;
        k1 += 0xBB67AE85u;
    }
    out[0] = c0; out[1] = c1; out[2] = c2; out[3] = c3;
}

/* ------------------------------------------------------------------ */
/* seeded synthetic weights (the library's generator, restated)        */
/* ------------------------------------------------------------------ */

static double unit_open(uint32_t x) { return ((double)(x >> 8) + 0.5) * (1.0 / 16777216.0); }

/* Values [start, start + n) of a tensor's normal sequence (start % 4 == 0
 * whenever cols % 32 == 0). */
static void synth_normals(uint64_t seed, uint32_t tid, uint64_t start, int n, float std, float* out) {
    const uint32_t key[2] = {(uint32_t)seed, (uint32_t)(seed >> 32)};
    uint64_t g = start >> 2;
    int off = (int)(start & 3), i = 0;
    const double two_pi = 6.283185307179586476925;
    while (i < n) {
        const uint32_t ctr[4] = {(uint32_t)g, (uint32_t)(g >> 32), tid, 0x5EEDu};
        uint32_t o[4];
        orc_philox4x32_10(ctr, key, o);
        double z[4];
        for (int h = 0; h < 2; h++) {
            const double r = sqrt(-2.0 * log(unit_open(o[2 * h])));
            const double t = two_pi * unit_open(o[2 * h + 1]);
            z[2 * h] = r * cos(t);
            z[2 * h + 1] = r * sin(t);
        }
        for (int l = off; l < 4 && i < n; l++, i++) out[i] = (float)(z[l] * (double)std);
        off = 0;
        g++;
    }
}

int orc_synth_q4_0_i8(uint64_t seed, uint32_t tensor_id, int rows, int cols, float std, int8_t* w, uint16_t* d) {
    if (!w || !d || rows <= 0 || cols <= 0 || cols % 32 != 0) return -1;
#pragma omp parallel
    {
        float* buf = (float*)malloc(sizeof(float) * (size_t)cols);
#pragma omp for schedule(static)
        for (int r = 0; r < rows; r++) {
            synth_normals(seed, tensor_id, (uint64_t)r * cols, cols, std, buf);
            orc_q4_0_quantize_i8(buf, cols, w + (size_t)r * cols, d + (size_t)r * (cols / 32));
        }
        free(buf);
    }
    return 0;
}

int orc_synth_q4_0_f32(uint64_t seed, uint32_t tensor_id, int rows, int cols, float std, float* out) {
    if (!out || rows <= 0 || cols <= 0 || cols % 32 != 0) return -1;
#pragma omp parallel
    {
        float* buf = (float*)malloc(sizeof(float) * (size_t)cols);
        int8_t* w = (int8_t*)malloc((size_t)cols);
        uint16_t* d = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)(cols / 32));
#pragma omp for schedule(static)
        for (int r = 0; r < rows; r++) {
            synth_normals(seed, tensor_id, (uint64_t)r * cols, cols, std, buf);
            orc_q4_0_quantize_i8(buf, cols, w, d);
            for (int j = 0; j < cols; j++) out[(size_t)r * cols + j] = (float)w[j] * orc_f16_to_f32(d[j / 32]);
        }
        free(buf);
        free(w);
        free(d);
    }
    return 0;
}

/* ------------------------------------------------------------------ */
/* model                                                               */
/* ------------------------------------------------------------------ */

int orc_kv_init(orc_kv_t* kv, int layers, int cap, int kv_heads, int head_dim) {
    size_t n = (size_t)layers * cap * kv_heads * head_dim;
    kv->k = (float*)calloc(n, sizeof(float));
    kv->v = (float*)calloc(n, sizeof(float));
    kv->layers = layers; kv->cap = cap; kv->kv_heads = kv_heads; kv->head_dim = head_dim;
    return (kv->k && kv->v) ? 0 : -1;
}

void orc_kv_free(orc_kv_t* kv) {
    free(kv->k); free(kv->v);
    kv->k = kv->v = NULL;
}

static void lin(const orc_lin_t* L, const float* x, float* y, int M) {
    if (L->wp) {
        orc_matmul_packed(x, L->wp, L->sp, y, M, L->N, L->K);
        return;
    }
    if (L->f32) { /* inference.c:131-141 */
        for (int m = 0; m < M; m++)
            for (int o = 0; o < L->N; o++) {
                const float* row = L->f32 + (size_t)o * L->K;
                const float* in = x + (size_t)m * L->K;
                float s = 0.0f;
                for (int i = 0; i < L->K; i++) s += in[i] * row[i];
                y[(size_t)m * L->N + o] = s;
            }
        return;
    }
    orc_matmul_block(x, L->w, L->s, y, M, L->N, L->K);
}

/* inference.c:193-247 for one query row against the visible cache slots. */
static void attend_row(const float* q, const float* Kc, const float* Vc, int kvh, int hd,
                       int stride, const int* slots, int ns, float* out, float* sc) {
    float scale = 1.0f / sqrtf((float)hd);
    for (int t = 0; t < ns; t++) {
        const float* kk = Kc + (size_t)slots[t] * stride + (size_t)kvh * hd;
        float dot = 0.0f;
        for (int e = 0; e < hd; e++) dot += q[e] * kk[e];
        sc[t] = dot * scale;
    }
    float mx = sc[0];
    for (int t = 1; t < ns; t++) if (sc[t] > mx) mx = sc[t];
    float sum = 0.0f;
    for (int t = 0; t < ns; t++) { sc[t] = expf(sc[t] - mx); sum += sc[t]; }
    for (int t = 0; t < ns; t++) sc[t] /= sum;
    for (int e = 0; e < hd; e++) {
        float acc = 0.0f;
        for (int t = 0; t < ns; t++)
            acc += sc[t] * Vc[(size_t)slots[t] * stride + (size_t)kvh * hd + e];
        out[e] = acc;
    }
}

void orc_stack_forward(const orc_model_t* mdl, const orc_layer_t* layers, int n_layers,
                       orc_kv_t* kv, float* x, int M, int base, const int* pos,
                       const uint8_t* mask) {
    const orc_dims_t* D = &mdl->dims;
    const int d = D->d, H = D->heads, Hk = D->kv_heads, hd = D->head_dim, F = D->ffn;
    const int qd = H * hd, kd = Hk * hd, grp = H / Hk;
    float* nrm = (float*)malloc(sizeof(float) * (size_t)M * d);
    float* q = (float*)malloc(sizeof(float) * (size_t)M * qd);
    float* k = (float*)malloc(sizeof(float) * (size_t)M * kd);
    float* v = (float*)malloc(sizeof(float) * (size_t)M * kd);
    float* att = (float*)malloc(sizeof(float) * (size_t)M * qd);
    float* o = (float*)malloc(sizeof(float) * (size_t)M * d);
    float* g = (float*)malloc(sizeof(float) * (size_t)M * F);
    float* u = (float*)malloc(sizeof(float) * (size_t)M * F);
    int* slots_all = (int*)malloc(sizeof(int) * (size_t)M * (base + M));
    int* nslots = (int*)malloc(sizeof(int) * M);
    for (int m = 0; m < M; m++) {
        int* s = slots_all + (size_t)m * (base + M);
        int c = 0;
        for (int t = 0; t < base; t++) s[c++] = t;
        for (int j = 0; j < M; j++) {
            int vis = mask ? mask[(size_t)m * M + j] != 0 : (j <= m);
            if (vis) s[c++] = base + j;
        }
        nslots[m] = c;
    }
    const int stride = kd;
    for (int l = 0; l < n_layers; l++) {
        const orc_layer_t* L = &layers[l];
        float* Kc = kv->k + (size_t)l * kv->cap * kd;
        float* Vc = kv->v + (size_t)l * kv->cap * kd;
        for (int m = 0; m < M; m++) orc_rmsnorm(x + (size_t)m * d, nrm + (size_t)m * d, d, D->eps);
        lin(&L->q, nrm, q, M);
        lin(&L->k, nrm, k, M);
        lin(&L->v, nrm, v, M);
        for (int m = 0; m < M; m++) {
            orc_rope_vec(q + (size_t)m * qd, H, hd, pos[m], D->theta);
            orc_rope_vec(k + (size_t)m * kd, Hk, hd, pos[m], D->theta);
            memcpy(Kc + (size_t)(base + m) * kd, k + (size_t)m * kd, sizeof(float) * kd);
            memcpy(Vc + (size_t)(base + m) * kd, v + (size_t)m * kd, sizeof(float) * kd);
        }
#pragma omp parallel
        {
            float* sc = (float*)malloc(sizeof(float) * (size_t)(base + M));
#pragma omp for collapse(2) schedule(static)
            for (int m = 0; m < M; m++)
                for (int h = 0; h < H; h++)
                    attend_row(q + (size_t)m * qd + (size_t)h * hd, Kc, Vc, h / grp, hd, stride,
                               slots_all + (size_t)m * (base + M), nslots[m],
                               att + (size_t)m * qd + (size_t)h * hd, sc);
            free(sc);
        }
        lin(&L->o, att, o, M);
        for (size_t i = 0; i < (size_t)M * d; i++) x[i] = x[i] + o[i];
        for (int m = 0; m < M; m++) orc_rmsnorm(x + (size_t)m * d, nrm + (size_t)m * d, d, D->eps);
        lin(&L->gate, nrm, g, M);
        lin(&L->up, nrm, u, M);
        for (int m = 0; m < M; m++) orc_swiglu(g + (size_t)m * F, u + (size_t)m * F, g + (size_t)m * F, F);
        lin(&L->down, g, o, M);
        for (size_t i = 0; i < (size_t)M * d; i++) x[i] = x[i] + o[i];
    }
    free(nrm); free(q); free(k); free(v); free(att); free(o); free(g); free(u);
    free(slots_all); free(nslots);
}

void orc_lm_logits(const orc_model_t* mdl, const float* x, float* logits, int M) {
    const int d = mdl->dims.d;
    float* nrm = (float*)malloc(sizeof(float) * (size_t)M * d);
    for (int m = 0; m < M; m++) orc_rmsnorm(x + (size_t)m * d, nrm + (size_t)m * d, d, mdl->dims.eps);
    lin(&mdl->lm, nrm, logits, M);
    free(nrm);
}

/* inference.c:421-422: ids at or above the vocabulary read row 0. */
static inline int tok_or_zero(int t, int vocab) { return (t < 0 || t >= vocab) ? 0 : t; }

int orc_argmax(const float* v, int n) {
    int bi = 0;
    float bv = v[0];
    for (int i = 1; i < n; i++)
        if (v[i] > bv) { bv = v[i]; bi = i; }
    return bi;
}

/* (top1 - top2) / |top1|: the relative margin of the greedy choice. */
static float top2_margin(const float* v, int n) {
    float a = -FLT_MAX, b = -FLT_MAX;
    for (int i = 0; i < n; i++) {
        if (v[i] > a) { b = a; a = v[i]; }
        else if (v[i] > b) b = v[i];
    }
    float s = fabsf(a) > 1e-30f ? fabsf(a) : 1e-30f;
    return (a - b) / s;
}

void orc_greedy_generate(const orc_model_t* mdl, const int* prompt, int P, int n_new,
                         int* out, float* margins) {
    const orc_dims_t* D = &mdl->dims;
    const int d = D->d, V = D->vocab;
    orc_kv_t kv;
    orc_kv_init(&kv, D->layers, P + n_new + 1, D->kv_heads, D->head_dim);
    float* x = (float*)malloc(sizeof(float) * (size_t)P * d);
    float* lg = (float*)malloc(sizeof(float) * V);
    int* pos = (int*)malloc(sizeof(int) * P);
    for (int i = 0; i < P; i++) {
        memcpy(x + (size_t)i * d, mdl->embed + (size_t)tok_or_zero(prompt[i], V) * d, sizeof(float) * d);
        pos[i] = i;
    }
    orc_stack_forward(mdl, mdl->base, D->layers, &kv, x, P, 0, pos, NULL);
    orc_lm_logits(mdl, x + (size_t)(P - 1) * d, lg, 1);
    int cur = orc_argmax(lg, V);
    out[0] = cur;
    if (margins) margins[0] = top2_margin(lg, V);
    for (int i = 1; i < n_new; i++) {
        int p = P + i - 1;
        memcpy(x, mdl->embed + (size_t)cur * d, sizeof(float) * d);
        orc_stack_forward(mdl, mdl->base, D->layers, &kv, x, 1, p, &p, NULL);
        orc_lm_logits(mdl, x, lg, 1);
        cur = orc_argmax(lg, V);
        out[i] = cur;
        if (margins) margins[i] = top2_margin(lg, V);
    }
    free(x); free(lg); free(pos);
    orc_kv_free(&kv);
}

int orc_spec_generate(const orc_model_t* mdl, const int* prompt, int P, int K,
                      int max_acc, int n_new, int* out, int* acc_hist, float* margins) {
    const orc_dims_t* D = &mdl->dims;
    const int d = D->d, V = D->vocab;
    const int cap = P + n_new + K + 2;
    orc_kv_t kvb, kvd;
    orc_kv_init(&kvb, D->layers, cap, D->kv_heads, D->head_dim);
    orc_kv_init(&kvd, mdl->draft_layers, cap, D->kv_heads, D->head_dim);
    int* seq = (int*)malloc(sizeof(int) * (size_t)(cap + 1));
    const int rows_max = (P + 1 > K + 1) ? P + 1 : K + 1;
    float* x = (float*)malloc(sizeof(float) * (size_t)rows_max * d);
    float* feat = (float*)malloc(sizeof(float) * (size_t)rows_max * d); /* F_{m-1}.. */
    float* lg = (float*)malloc(sizeof(float) * (size_t)(K + 1) * V);
    int* pos = (int*)malloc(sizeof(int) * rows_max);
    int* drafted = (int*)malloc(sizeof(int) * (K + 1));

    for (int i = 0; i < P; i++) seq[i] = tok_or_zero(prompt[i], V);
    /* prefill */
    for (int i = 0; i < P; i++) {
        memcpy(x + (size_t)i * d, mdl->embed + (size_t)seq[i] * d, sizeof(float) * d);
        pos[i] = i;
    }
    orc_stack_forward(mdl, mdl->base, D->layers, &kvb, x, P, 0, pos, NULL);
    /* features F_{-1}=0, F_0..F_{P-1} for draft rows 0..P */
    memset(feat, 0, sizeof(float) * d);
    memcpy(feat + d, x, sizeof(float) * (size_t)(P - 1) * d);  /* F_0..F_{P-2} */
    float* last_f = (float*)malloc(sizeof(float) * d);
    memcpy(last_f, x + (size_t)(P - 1) * d, sizeof(float) * d);
    orc_lm_logits(mdl, last_f, lg, 1);
    int n = P;                 /* seq[n] is the last token, not in base KV */
    seq[n] = orc_argmax(lg, V);
    int produced = 0;
    out[produced] = seq[n];
    if (margins) margins[produced] = top2_margin(lg, V);
    produced++;
    /* feat rows for draft catch-up: positions m..n use F_{m-1}..F_{n-1} */
    memcpy(feat + (size_t)P * d, last_f, sizeof(float) * d); /* F_{P-1} */
    int m = 0;                 /* draft KV clean length */
    int steps = 0;
    const double t0 = now_s();
    while (produced < n_new) {
        /* --- draft catch-up pass: rows m..n --- */
        int R = n - m + 1;
        for (int r = 0; r < R; r++) {
            const float* e = mdl->embed + (size_t)seq[m + r] * d;
            for (int i = 0; i < d; i++) x[(size_t)r * d + i] = feat[(size_t)r * d + i] + e[i];
            pos[r] = m + r;
        }
        orc_stack_forward(mdl, mdl->draft, mdl->draft_layers, &kvd, x, R, m, pos, NULL);
        float* g = (float*)malloc(sizeof(float) * d);
        memcpy(g, x + (size_t)(R - 1) * d, sizeof(float) * d);
        orc_lm_logits(mdl, g, lg, 1);
        drafted[0] = orc_argmax(lg, V);
        for (int j = 1; j < K; j++) {
            int p = n + j;
            const float* e = mdl->embed + (size_t)drafted[j - 1] * d;
            for (int i = 0; i < d; i++) x[i] = g[i] + e[i];
            orc_stack_forward(mdl, mdl->draft, mdl->draft_layers, &kvd, x, 1, p, &p, NULL);
            memcpy(g, x, sizeof(float) * d);
            orc_lm_logits(mdl, g, lg, 1);
            drafted[j] = orc_argmax(lg, V);
        }
        free(g);
        m = n + 1;
        /* --- verify rows n..n+K --- */
        for (int r = 0; r <= K; r++) {
            int t = r == 0 ? seq[n] : drafted[r - 1];
            memcpy(x + (size_t)r * d, mdl->embed + (size_t)t * d, sizeof(float) * d);
            pos[r] = n + r;
        }
        orc_stack_forward(mdl, mdl->base, D->layers, &kvb, x, K + 1, n, pos, NULL);
        orc_lm_logits(mdl, x, lg, K + 1);
        int a = 0;
        while (a < K && a < max_acc && drafted[a] == orc_argmax(lg + (size_t)a * V, V)) a++;
        int bonus = orc_argmax(lg + (size_t)a * V, V);
        if (acc_hist) acc_hist[steps] = a;
        steps++;
        for (int j = 0; j <= a; j++) {
            int t = j < a ? drafted[j] : bonus;
            seq[n + 1 + j] = t;
            if (produced < n_new) {
                out[produced] = t;
                if (margins) margins[produced] = top2_margin(lg + (size_t)j * V, V);
                produced++;
            }
        }
        /* features for the next catch-up: F_n..F_{n+a} = verify rows 0..a */
        memcpy(feat, x, sizeof(float) * (size_t)(a + 1) * d);
        n = n + a + 1;
    }
    g_last_decode_s = now_s() - t0;
    free(seq); free(x); free(feat); free(lg); free(pos); free(drafted); free(last_f);
    orc_kv_free(&kvb);
    orc_kv_free(&kvd);
    return steps;
}

/* ------------------------------------------------------------------ */
/* Medusa (include/medusa.h rule; the reference declares the API at   */
/* medusa.h:84-229 without an implementation)                          */
/* ------------------------------------------------------------------ */

/* Top-k of one logits row (value desc, lower index first on ties) with
 * softmax probabilities p = exp(l - max) / sum_j exp(l_j - max), the sum in
 * index order. */
static void topk_probs(const float* lg, int V, int k, int* tok, float* prob) {
    float mx = lg[0];
    for (int i = 1; i < V; i++) if (lg[i] > mx) mx = lg[i];
    float sum = 0.0f;
    for (int i = 0; i < V; i++) sum += expf(lg[i] - mx);
    for (int j = 0; j < k; j++) {
        int bi = -1;
        for (int i = 0; i < V; i++) {
            int taken = 0;
            for (int q = 0; q < j; q++) if (tok[q] == i) { taken = 1; break; }
            if (taken) continue;
            if (bi < 0 || lg[i] > lg[bi]) bi = i;
        }
        tok[j] = bi;
        prob[j] = expf(lg[bi] - mx) / sum;
    }
}

typedef struct {
    float score;
    int depth, gen, parent_gen, token;
} med_cand_t;

/* score desc, depth asc, generation order asc */
static int cand_cmp(const void* a, const void* b) {
    const med_cand_t* x = (const med_cand_t*)a;
    const med_cand_t* y = (const med_cand_t*)b;
    if (x->score != y->score) return x->score > y->score ? -1 : 1;
    if (x->depth != y->depth) return x->depth < y->depth ? -1 : 1;
    return x->gen < y->gen ? -1 : (x->gen > y->gen);
}

int orc_medusa_tree(int root_tok, int n_heads, const int* topk, const int* tok, const float* prob, int kmax,
                    int max_nodes, int* out_tok, int* out_parent, int* out_depth, float* out_score) {
    /* candidates in generation (breadth-first) order: level L+1 = head L's
     * top-k under every level-L candidate; the root is generation -1 */
    int total = 0, width = 1;
    for (int h = 0; h < n_heads; h++) { width *= topk[h]; total += width; }
    med_cand_t* c = (med_cand_t*)malloc(sizeof(med_cand_t) * (size_t)(total > 0 ? total : 1));
    int lvl_begin = 0, lvl_end = 0, n = 0;
    for (int h = 0; h < n_heads; h++) {
        const int pb = lvl_begin, pe = lvl_end;  /* parents: previous level ([0,0) = the root) */
        lvl_begin = n;
        if (h == 0) {
            for (int k = 0; k < topk[0]; k++, n++) {
                c[n].score = prob[k];
                c[n].depth = 1;
                c[n].gen = n;
                c[n].parent_gen = -1;
                c[n].token = tok[k];
            }
        } else {
            for (int pi = pb; pi < pe; pi++)
                for (int k = 0; k < topk[h]; k++, n++) {
                    c[n].score = c[pi].score * prob[h * kmax + k];
                    c[n].depth = h + 1;
                    c[n].gen = n;
                    c[n].parent_gen = pi;
                    c[n].token = tok[h * kmax + k];
                }
        }
        lvl_end = n;
    }
    med_cand_t* s = (med_cand_t*)malloc(sizeof(med_cand_t) * (size_t)(n > 0 ? n : 1));
    memcpy(s, c, sizeof(med_cand_t) * (size_t)n);
    qsort(s, (size_t)n, sizeof(med_cand_t), cand_cmp);
    int keep = max_nodes - 1 < n ? max_nodes - 1 : n;
    /* generation index -> output node index */
    int* where = (int*)malloc(sizeof(int) * (size_t)(n > 0 ? n : 1));
    for (int i = 0; i < n; i++) where[i] = -1;
    for (int i = 0; i < keep; i++) where[s[i].gen] = i + 1;
    out_tok[0] = root_tok;
    out_parent[0] = -1;
    out_depth[0] = 0;
    if (out_score) out_score[0] = 1.0f;
    for (int i = 0; i < keep; i++) {
        out_tok[i + 1] = s[i].token;
        out_parent[i + 1] = s[i].parent_gen < 0 ? 0 : where[s[i].parent_gen];
        out_depth[i + 1] = s[i].depth;
        if (out_score) out_score[i + 1] = s[i].score;
    }
    free(c); free(s); free(where);
    return keep + 1;
}

int orc_medusa_generate(const orc_model_t* mdl, const int* prompt, int P, const int* topk, int max_nodes,
                        int n_new, int* out, int* acc_hist, float* margins) {
    const orc_dims_t* D = &mdl->dims;
    const int d = D->d, V = D->vocab, H = mdl->n_medusa;
    int kmax = 1;
    for (int h = 0; h < H; h++) if (topk[h] > kmax) kmax = topk[h];
    const int cap = P + n_new + max_nodes + 2;
    orc_kv_t kv;
    orc_kv_init(&kv, D->layers, cap, D->kv_heads, D->head_dim);
    const int rows_max = P > max_nodes ? P : max_nodes;
    float* x = (float*)malloc(sizeof(float) * (size_t)rows_max * d);
    float* lg = (float*)malloc(sizeof(float) * (size_t)max_nodes * V);
    float* feat = (float*)malloc(sizeof(float) * d);
    float* h = (float*)malloc(sizeof(float) * d);
    float* y = (float*)malloc(sizeof(float) * d);
    float* z = (float*)malloc(sizeof(float) * d);
    float* hl = (float*)malloc(sizeof(float) * V);
    int* pos = (int*)malloc(sizeof(int) * rows_max);
    int* ttok = (int*)malloc(sizeof(int) * (size_t)(H > 0 ? H : 1) * kmax);
    float* tprob = (float*)malloc(sizeof(float) * (size_t)(H > 0 ? H : 1) * kmax);
    int* ntok = (int*)malloc(sizeof(int) * max_nodes);
    int* npar = (int*)malloc(sizeof(int) * max_nodes);
    int* ndep = (int*)malloc(sizeof(int) * max_nodes);
    int* target = (int*)malloc(sizeof(int) * max_nodes);
    int* path = (int*)malloc(sizeof(int) * max_nodes);
    uint8_t* mask = (uint8_t*)malloc((size_t)max_nodes * max_nodes);

    /* prefill: base KV 0..P-1, first token from the last prompt row */
    for (int i = 0; i < P; i++) {
        memcpy(x + (size_t)i * d, mdl->embed + (size_t)tok_or_zero(prompt[i], V) * d, sizeof(float) * d);
        pos[i] = i;
    }
    orc_stack_forward(mdl, mdl->base, D->layers, &kv, x, P, 0, pos, NULL);
    memcpy(feat, x + (size_t)(P - 1) * d, sizeof(float) * d);
    orc_lm_logits(mdl, feat, lg, 1);
    int n = P;                  /* the newest token (seq[n]) is not in the KV yet */
    int cur_tok = orc_argmax(lg, V);
    int produced = 0;
    out[produced] = cur_tok;
    if (margins) margins[produced] = top2_margin(lg, V);
    produced++;
    int steps = 0;
    const double t0 = now_s();
    while (produced < n_new) {
        /* heads on h = RMSNorm(F): z_i = h + SiLU(W_i h), logits_i = LM(z_i) */
        orc_rmsnorm(feat, h, d, D->eps);
        for (int i = 0; i < H; i++) {
            lin(&mdl->medusa[i], h, y, 1);
            orc_silu(y, z, d);
            for (int j = 0; j < d; j++) z[j] = h[j] + z[j];
            lin(&mdl->lm, z, hl, 1);
            topk_probs(hl, V, topk[i], ttok + (size_t)i * kmax, tprob + (size_t)i * kmax);
        }
        const int M = orc_medusa_tree(cur_tok, H, topk, ttok, tprob, kmax, max_nodes, ntok, npar, ndep, NULL);
        /* tree-masked verify: node i at slot n + i, position n + depth */
        for (int i = 0; i < M; i++) {
            memcpy(x + (size_t)i * d, mdl->embed + (size_t)tok_or_zero(ntok[i], V) * d, sizeof(float) * d);
            pos[i] = n + ndep[i];
            for (int j = 0; j < M; j++) mask[(size_t)i * M + j] = 0;
            for (int j = i; j >= 0; j = npar[j]) mask[(size_t)i * M + j] = 1;
        }
        orc_stack_forward(mdl, mdl->base, D->layers, &kv, x, M, n, pos, mask);
        orc_lm_logits(mdl, x, lg, M);
        for (int i = 0; i < M; i++) target[i] = orc_argmax(lg + (size_t)i * V, V);
        /* longest path whose tokens are the base model's greedy choices */
        int a = 0, cur = 0;
        path[0] = 0;
        for (;;) {
            int nxt = -1;
            for (int c2 = 1; c2 < M; c2++)
                if (npar[c2] == cur && ntok[c2] == target[cur]) { nxt = c2; break; }
            if (nxt < 0) break;
            path[++a] = nxt;
            cur = nxt;
        }
        if (acc_hist) acc_hist[steps] = a;
        steps++;
        /* emitted: the accepted children, then the base token after the last one */
        for (int j = 1; j <= a + 1 && produced < n_new; j++) {
            const int t = j <= a ? ntok[path[j]] : target[cur];
            out[produced] = t;
            if (margins) margins[produced] = top2_margin(lg + (size_t)path[j - 1] * V, V);
            produced++;
        }
        /* KV compaction: the accepted nodes move to slots n .. n + a (their
         * rotary positions were already n + depth) */
        for (int j = 1; j <= a; j++) {
            const int src = n + path[j], dst = n + j;
            if (src == dst) continue;
            for (int l = 0; l < kv.layers; l++) {
                const size_t row = (size_t)kv.kv_heads * kv.head_dim;
                float* kb = kv.k + (size_t)l * kv.cap * row;
                float* vb = kv.v + (size_t)l * kv.cap * row;
                memcpy(kb + (size_t)dst * row, kb + (size_t)src * row, sizeof(float) * row);
                memcpy(vb + (size_t)dst * row, vb + (size_t)src * row, sizeof(float) * row);
            }
        }
        memcpy(feat, x + (size_t)cur * d, sizeof(float) * d);
        cur_tok = target[cur];
        n += a + 1;
    }
    g_last_decode_s = now_s() - t0;
    free(x); free(lg); free(feat); free(h); free(y); free(z); free(hl); free(pos); free(ttok); free(tprob);
    free(ntok); free(npar); free(ndep); free(target); free(path); free(mask);
    orc_kv_free(&kv);
    return steps;
}

/* ------------------------------------------------------------------ */
/* Stochastic speculative decoding (include/speculative.h rule for     */
/* temperature > 0; the reference declares the contract without code)  */
/* ------------------------------------------------------------------ */

/* 24 bits of Philox4x32-10 (Salmon et al., SC'11) with key (seed, 0) at
 * counter (sequence, step, position, purpose): U in [0, 2^24), u = U / 2^24. */
uint32_t orc_philox_u24(uint32_t seed, uint32_t seq, uint32_t step, uint32_t pos, uint32_t purpose) {
    const uint32_t ctr[4] = {seq, step, pos, purpose};
    const uint32_t key[2] = {seed, 0u};
    uint32_t o[4];
    orc_philox4x32_10(ctr, key, o);
    return o[0] >> 8;
}

float orc_philox_uniform(uint32_t seed, uint32_t seq, uint32_t step, uint32_t pos, uint32_t purpose) {
    return (float)orc_philox_u24(seed, seq, step, pos, purpose) * (1.0f / 16777216.0f);
}

/* Integer sampling weight of x = (l - max) / T <= 0: E = trunc(e^x * 2^24),
 * 0 below x = -17. e^x by Cody-Waite range reduction x = k ln2 + r (ln2 split
 * into a 16-bit head and a float tail, |k| <= 25 so k * head is exact) and
 * the degree-7 Taylor polynomial of e^r on |r| <= ln2 / 2 in Horner form
 * (truncation error below 6e-9), every step one correctly rounded fma or
 * multiply, then the exact scale 2^(k + 24). The device evaluates the same
 * operations, so E is the same integer on both. */
uint32_t orc_sample_weight(float x) {
    if (!(x >= -17.0f)) return 0u;
    const float kf = rintf(x * 1.442695f);
    float r = fmaf(-kf, 0.693145751953125f, x);
    r = fmaf(-kf, 1.4286068e-06f, r);
    float p = 0.0001984127f;
    p = fmaf(p, r, 0.0013888889f);
    p = fmaf(p, r, 0.008333334f);
    p = fmaf(p, r, 0.041666668f);
    p = fmaf(p, r, 0.16666667f);
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    const float s = ldexpf(p, (int)kf + 24);
    const uint32_t E = (uint32_t)s;
    return E > (1u << 24) ? (1u << 24) : E;
}

/* Nucleus weights of logits l: E_i = weight((l_i - max) / T); the nucleus is
 * {i : E_i >= t*} with t* the largest integer whose kept mass
 * S(t) = sum_{E_i >= t} E_i satisfies S(t) * 2^24 >= P * z, z = S(1) and
 * P = max(1, trunc(top_p * 2^24)). Kept weights stay, the rest become 0;
 * returns the kept mass M. All sums are exact integers. */
uint64_t orc_sample_weights(const float* l, int V, float T, float top_p, uint32_t* E) {
    float mx = l[0];
    for (int i = 1; i < V; i++) if (l[i] > mx) mx = l[i];
    uint64_t z = 0;
    for (int i = 0; i < V; i++) {
        E[i] = orc_sample_weight((l[i] - mx) / T);
        z += E[i];
    }
    uint32_t P = (uint32_t)(top_p * 16777216.0f);
    if (P < 1u) P = 1u;
    const unsigned __int128 need = (unsigned __int128)P * z;
    uint32_t lo = 1u, hi = (1u << 24) + 1u; /* S(lo) meets the mass, S(hi) = 0 does not */
    while (hi - lo > 1u) {
        const uint32_t mid = lo + (hi - lo) / 2u;
        uint64_t s = 0;
        for (int i = 0; i < V; i++) if (E[i] >= mid) s += E[i];
        if (((unsigned __int128)s << 24) >= need) lo = mid; else hi = mid;
    }
    uint64_t M = 0;
    for (int i = 0; i < V; i++) {
        if (E[i] < lo) E[i] = 0u;
        M += E[i];
    }
    return M;
}

/* q_i = E_i / M as floats (for inspection). */
void orc_sample_dist(const float* l, int V, float T, float top_p, float* q) {
    uint32_t* E = (uint32_t*)malloc(sizeof(uint32_t) * (size_t)V);
    const uint64_t M = orc_sample_weights(l, V, T, top_p, E);
    for (int i = 0; i < V; i++) q[i] = (float)((double)E[i] / (double)M);
    free(E);
}

/* Inverse CDF in index order: the first i whose running sum of w exceeds
 * trunc(U * total / 2^24) (total = sum w > 0). w32 or w64 gives the weights. */
int orc_sample_pick(const uint32_t* w32, const uint64_t* w64, int V, uint64_t total, uint32_t U) {
    const uint64_t tgt = (uint64_t)(((unsigned __int128)U * total) >> 24);
    uint64_t c = 0;
    for (int i = 0; i < V; i++) {
        c += w32 ? w32[i] : w64[i];
        if (c > tgt) return i;
    }
    return V - 1;
}

/* Acceptance of drafted x: u < p(x) / q(x) with p = Ep / Mp, q = Eq / Mq,
 * i.e. U * Mp * Eq < 2^24 * Ep * Mq. */
int orc_sample_accept(uint32_t U, uint32_t Ep, uint64_t Mp, uint32_t Eq, uint64_t Mq) {
    return (unsigned __int128)U * Mp * Eq < (((unsigned __int128)Ep * Mq) << 24);
}

/* Residual weights R_i = max(0, Ep_i * Mq - Eq_i * Mp) / 2^24 (truncated),
 * proportional to max(0, p - q); returns their sum. */
uint64_t orc_sample_residual(const uint32_t* Ep, uint64_t Mp, const uint32_t* Eq, uint64_t Mq, int V,
                             uint64_t* R) {
    uint64_t s = 0;
    for (int i = 0; i < V; i++) {
        const unsigned __int128 a = (unsigned __int128)Ep[i] * Mq, b = (unsigned __int128)Eq[i] * Mp;
        R[i] = a > b ? (uint64_t)((a - b) >> 24) : 0u;
        s += R[i];
    }
    return s;
}

int orc_spec_generate_sampled(const orc_model_t* mdl, const int* prompt, int P, int K, int n_new, float T,
                              float top_p, uint32_t seed, uint32_t seq_id, int* out, int* acc_hist) {
    const orc_dims_t* D = &mdl->dims;
    const int d = D->d, V = D->vocab;
    const int cap = P + n_new + K + 2;
    orc_kv_t kvb, kvd;
    orc_kv_init(&kvb, D->layers, cap, D->kv_heads, D->head_dim);
    orc_kv_init(&kvd, mdl->draft_layers, cap, D->kv_heads, D->head_dim);
    int* seq = (int*)malloc(sizeof(int) * (size_t)(cap + 1));
    const int rows_max = (P + 1 > K + 1) ? P + 1 : K + 1;
    float* x = (float*)malloc(sizeof(float) * (size_t)rows_max * d);
    float* feat = (float*)malloc(sizeof(float) * (size_t)rows_max * d);
    float* lg = (float*)malloc(sizeof(float) * (size_t)(K + 1) * V);
    uint32_t* qd = (uint32_t*)malloc(sizeof(uint32_t) * (size_t)K * V);       /* draft weights */
    uint32_t* pt = (uint32_t*)malloc(sizeof(uint32_t) * (size_t)(K + 1) * V); /* target weights */
    uint64_t* qm = (uint64_t*)malloc(sizeof(uint64_t) * (size_t)(K + 1));
    uint64_t* pm = (uint64_t*)malloc(sizeof(uint64_t) * (size_t)(K + 1));
    uint64_t* r = (uint64_t*)malloc(sizeof(uint64_t) * V);
    int* pos = (int*)malloc(sizeof(int) * rows_max);
    int* drafted = (int*)malloc(sizeof(int) * (K + 1));
    float* g = (float*)malloc(sizeof(float) * d);

    for (int i = 0; i < P; i++) seq[i] = tok_or_zero(prompt[i], V);
    for (int i = 0; i < P; i++) {
        memcpy(x + (size_t)i * d, mdl->embed + (size_t)seq[i] * d, sizeof(float) * d);
        pos[i] = i;
    }
    orc_stack_forward(mdl, mdl->base, D->layers, &kvb, x, P, 0, pos, NULL);
    memset(feat, 0, sizeof(float) * d);
    memcpy(feat + d, x, sizeof(float) * (size_t)(P - 1) * d);
    memcpy(g, x + (size_t)(P - 1) * d, sizeof(float) * d);
    orc_lm_logits(mdl, g, lg, 1);
    int n = P;
    {
        const uint64_t M = orc_sample_weights(lg, V, T, top_p, pt);
        seq[n] = orc_sample_pick(pt, NULL, V, M, orc_philox_u24(seed, seq_id, 0xFFFFFFFFu, (uint32_t)n, 2u));
    }
    int produced = 0;
    out[produced++] = seq[n];
    memcpy(feat + (size_t)P * d, g, sizeof(float) * d);
    int m = 0, steps = 0;
    const double t0 = now_s();
    while (produced < n_new) {
        /* draft catch-up rows m..n, then K sampled draft tokens */
        int R = n - m + 1;
        for (int rr = 0; rr < R; rr++) {
            const float* e = mdl->embed + (size_t)seq[m + rr] * d;
            for (int i = 0; i < d; i++) x[(size_t)rr * d + i] = feat[(size_t)rr * d + i] + e[i];
            pos[rr] = m + rr;
        }
        orc_stack_forward(mdl, mdl->draft, mdl->draft_layers, &kvd, x, R, m, pos, NULL);
        memcpy(g, x + (size_t)(R - 1) * d, sizeof(float) * d);
        for (int j = 0; j < K; j++) {
            if (j > 0) {
                int p = n + j;
                const float* e = mdl->embed + (size_t)drafted[j - 1] * d;
                for (int i = 0; i < d; i++) x[i] = g[i] + e[i];
                orc_stack_forward(mdl, mdl->draft, mdl->draft_layers, &kvd, x, 1, p, &p, NULL);
                memcpy(g, x, sizeof(float) * d);
            }
            orc_lm_logits(mdl, g, lg, 1);
            uint32_t* qj = qd + (size_t)j * V;
            qm[j] = orc_sample_weights(lg, V, T, top_p, qj);
            drafted[j] = orc_sample_pick(qj, NULL, V, qm[j],
                                         orc_philox_u24(seed, seq_id, (uint32_t)steps, (uint32_t)(n + 1 + j), 0u));
        }
        m = n + 1;
        /* verify rows n..n+K */
        for (int rr = 0; rr <= K; rr++) {
            int t = rr == 0 ? seq[n] : drafted[rr - 1];
            memcpy(x + (size_t)rr * d, mdl->embed + (size_t)t * d, sizeof(float) * d);
            pos[rr] = n + rr;
        }
        orc_stack_forward(mdl, mdl->base, D->layers, &kvb, x, K + 1, n, pos, NULL);
        orc_lm_logits(mdl, x, lg, K + 1);
        for (int rr = 0; rr <= K; rr++)
            pm[rr] = orc_sample_weights(lg + (size_t)rr * V, V, T, top_p, pt + (size_t)rr * V);
        /* rejection sampling (accept with probability min(1, p / q)) */
        int a = 0, last;
        for (;;) {
            const uint32_t pos_a = (uint32_t)(n + 1 + a);
            if (a == K) {
                last = orc_sample_pick(pt + (size_t)K * V, NULL, V, pm[K],
                                       orc_philox_u24(seed, seq_id, (uint32_t)steps, pos_a, 2u));
                break;
            }
            const int xt = drafted[a];
            const uint32_t U = orc_philox_u24(seed, seq_id, (uint32_t)steps, pos_a, 1u);
            if (orc_sample_accept(U, pt[(size_t)a * V + xt], pm[a], qd[(size_t)a * V + xt], qm[a])) {
                a++;
                continue;
            }
            const uint64_t zr = orc_sample_residual(pt + (size_t)a * V, pm[a], qd + (size_t)a * V, qm[a], V, r);
            const uint32_t Ur = orc_philox_u24(seed, seq_id, (uint32_t)steps, pos_a, 2u);
            last = zr > 0 ? orc_sample_pick(NULL, r, V, zr, Ur) : orc_sample_pick(pt + (size_t)a * V, NULL, V, pm[a], Ur);
            break;
        }
        if (acc_hist) acc_hist[steps] = a;
        steps++;
        for (int j = 0; j <= a; j++) {
            int t = j < a ? drafted[j] : last;
            seq[n + 1 + j] = t;
            if (produced < n_new) out[produced++] = t;
        }
        memcpy(feat, x, sizeof(float) * (size_t)(a + 1) * d);
        n = n + a + 1;
    }
    g_last_decode_s = now_s() - t0;
    free(seq); free(x); free(feat); free(lg); free(qd); free(pt); free(qm); free(pm); free(r); free(pos);
    free(drafted); free(g);
    orc_kv_free(&kvb);
    orc_kv_free(&kvd);
    return steps;
}
