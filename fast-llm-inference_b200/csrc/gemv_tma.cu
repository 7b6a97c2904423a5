// Persistent INT8 GEMV / skinny GEMM (M <= 8 activation rows) streaming
// weights through a TMA bulk-copy ring (sm_100a).
//
// Contract and epilogues as matmul_dequantized (fast_llm/src/kernels/
// dequantized_tensor.c:204-247) with the fused layer epilogues of
// transformer_layer (fast_llm/src/inference.c:286-386). Built for bs1 decode,
// where one launch is only 9-100 MB of weights:
//
//   * one CTA per SM; CTA c owns a contiguous range of 8-row units;
//   * weights are in the tiled layout (fl_layout.cuh): a ring stage is 16
//     rows x one K-panel, moved by ONE 1-D cp.async.bulk (+ one for its fp16
//     block scales) issued by a producer warp -- the first stages before
//     griddepcontrol.wait, so the stream overlaps the previous kernel;
//   * M == 1: 8 consumer warps, a row pair each, u8 x s8 dp4a (the
//     instruction count per weight byte is low enough);
//   * M >= 2: dp4a would be instruction bound, so each consumer warp runs
//     mma.sync m16n8k32 s8 x u8 -> s32 on its share of the stage's
//     32-element blocks (A operand = the 16 weight rows of the tile via one
//     ldmatrix.x4, B operand = up to 8 activation rows), scales each block's
//     int32 by its fp16 scale and reduces across warps once per 16-row tile;
//   * every mbarrier wait is bounded (fl_tma.cuh).
#include <algorithm>

#include "fl_common.cuh"
#include "fl_epilogue.cuh"
#include "fl_kernels.h"
#include "fl_layout.cuh"
#include "fl_tma.cuh"

namespace fl {

namespace {

constexpr int kCWarps = 8;                   // consumer warps
constexpr int kThreads = (kCWarps + 1) * 32; // + producer warp
constexpr int kStageRows = 16;
constexpr int kMaxStages = 8;
#ifndef FL_TMA_SMEM_KB
#define FL_TMA_SMEM_KB 208
#endif
#ifndef FL_TMA_CTAS_PER_SM
#define FL_TMA_CTAS_PER_SM 1
#endif
// Dynamic shared memory budget per CTA (activation rows + ring), with the
// static reduction buffers and barriers (~8.7 KB) on top. 208 KB keeps every
// launch at or below 216 KB in all, which leaves a profiler room to run the
// kernel (the one-row down projection, 221 KB at a 216 KB budget, failed to
// launch under ncu); the decode step measured the same at 208 and 216 KB.
constexpr int kSmemLimit = FL_TMA_SMEM_KB * 1024;
constexpr int kCtasPerSm = FL_TMA_CTAS_PER_SM;

struct Geo {
    int P;         // panel width (weights of a stage row)
    int npan;      // K / P
    int S;         // ring stages
    int act_ld;    // activation row stride in shared memory (K + 16)
    int act_bytes; // shared bytes of the activation rows (and, 4-bit, their block sums)
    int asum_off;  // 4-bit: byte offset of the int block sums [rows][K / 32]
};

// Bytes of a stage row's weights: P int8, or P / 2 packed 4-bit.
__host__ __device__ inline int row_bytes(int P, bool w4) { return w4 ? P >> 1 : P; }
__host__ __device__ inline size_t slot_bytes(int P, bool w4 = false) {
    return (size_t)kStageRows * row_bytes(P, w4) + (size_t)kStageRows * (P / 16);
}

// P: the weights' panel width (0 = the default width for K).
inline bool make_geo(int K, int mrows, Geo& g, int P = 0, bool w4 = false) {
    g.P = P ? P : panel_width(K);
    if (!g.P || g.P % 128 || K % g.P || mrows < 1 || mrows > kMaxRows) return false;
    if (w4 && g.P % 256) return false;
    g.npan = K / g.P;
    g.act_ld = K + 16;
    g.asum_off = ((mrows * g.act_ld) + 127) & ~127;
    const int mmax = mrows <= 1 ? 1 : (mrows <= 2 ? 2 : (mrows <= 4 ? 4 : 8));  // the kernel's row template
    g.act_bytes = g.asum_off + (w4 ? ((mmax * (K / 32) * 4 + 127) & ~127) : 0);
    const long avail = (long)kSmemLimit - g.act_bytes - 256;
    const int S = (int)(avail / (long)slot_bytes(g.P, w4));
    if (S < 2) return false;
    g.S = S > kMaxStages ? kMaxStages : S;
    return true;
}

__device__ __forceinline__ int dot16(const uint4& a, const uint4& w) {
    int d = dp4a_us(a.x, w.x, 0);
    d = dp4a_us(a.y, w.y, d);
    d = dp4a_us(a.z, w.z, d);
    return dp4a_us(a.w, w.w, d);
}

__device__ __forceinline__ void ldmatrix_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}


// Epilogue of one weight-row pair, chosen at compile time (EPI >= 0) or at
// run time (EPI < 0: one kernel body serves every layer projection, so the
// launches of a layer share their instructions in the SM's caches).
template <int EPI>
__device__ __forceinline__ void pair_epi_any(int epi, const GemvParams& p, int r, int n0, bool has1, float y0,
                                             float y1, unsigned long long* best_s) {
    if constexpr (EPI >= 0) {
        pair_epilogue<EPI>(p, r, n0, has1, y0, y1, best_s);
    } else {
        switch (epi) {
            case EPI_STORE: pair_epilogue<EPI_STORE>(p, r, n0, has1, y0, y1, best_s); break;
            case EPI_RESID: pair_epilogue<EPI_RESID>(p, r, n0, has1, y0, y1, best_s); break;
            case EPI_QKV: pair_epilogue<EPI_QKV>(p, r, n0, has1, y0, y1, best_s); break;
            case EPI_SWIGLU: pair_epilogue<EPI_SWIGLU>(p, r, n0, has1, y0, y1, best_s); break;
            case EPI_LOGITS: pair_epilogue<EPI_LOGITS>(p, r, n0, has1, y0, y1, best_s); break;
            case EPI_TP_PUSH: pair_epilogue<EPI_TP_PUSH>(p, r, n0, has1, y0, y1, best_s); break;
            default: break;
        }
    }
}

// d = u8 . q over one block of packed 4-bit weights (a: 32 activation bytes,
// w: the block's 16 bytes; q[j] low nibbles, q[j + 16] high nibbles).
__device__ __forceinline__ int dot_w4(const uint4& a0, const uint4& a1, const uint4& w) {
    const uint32_t m = 0x0F0F0F0Fu;
    int d = (int)__dp4a(a0.x, w.x & m, 0u);
    d = (int)__dp4a(a0.y, w.y & m, (unsigned)d);
    d = (int)__dp4a(a0.z, w.z & m, (unsigned)d);
    d = (int)__dp4a(a0.w, w.w & m, (unsigned)d);
    d = (int)__dp4a(a1.x, (w.x >> 4) & m, (unsigned)d);
    d = (int)__dp4a(a1.y, (w.y >> 4) & m, (unsigned)d);
    d = (int)__dp4a(a1.z, (w.z >> 4) & m, (unsigned)d);
    return (int)__dp4a(a1.w, (w.w >> 4) & m, (unsigned)d);
}

// D(16x8, s32) = A(16x32, u8, row) x B(32x8, u8, col) (4-bit weights as q).
__device__ __forceinline__ void mma_u8u8(uint32_t a0, uint32_t a2, uint32_t b0, uint32_t b1, int& d0, int& d1) {
    int c2, c3;
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.u8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%11,%12,%13};"
        : "=r"(d0), "=r"(d1), "=r"(c2), "=r"(c3)
        : "r"(a0), "r"(0), "r"(a2), "r"(0), "r"(b0), "r"(b1), "r"(0), "r"(0), "r"(0), "r"(0));
}

// D(16x8, s32) = A(16x32, s8, row: 16 weight rows) x B(32x8, u8, col: 8
// activation rows): one instruction covers a 16-row tile for every row.
__device__ __forceinline__ void mma_s8u8(uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1, int& d0, int& d1, int& d2, int& d3) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.u8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%11,%12,%13};"
        : "=r"(d0), "=r"(d1), "=r"(d2), "=r"(d3)
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0), "r"(0), "r"(0), "r"(0));
}

template <int MMAX, int EPI, bool MMA, bool W4>
__global__ void __launch_bounds__(kThreads, kCtasPerSm) gemv_tma_kernel(const GemvParams p, const Geo geo,
                                                                         const int epi_rt) {
    const int epi = EPI >= 0 ? EPI : epi_rt;
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ __align__(8) uint64_t full_bar[kMaxStages];
    __shared__ __align__(8) uint64_t empty_bar[kMaxStages];
    __shared__ unsigned long long best_s[kMaxRows];
    __shared__ float red[2][kCWarps][32][4];
    __shared__ float nred[kMaxRows * kCWarps];

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int N = p.N, K = p.K, P = geo.P, npan = geo.npan, S = geo.S;
    const int nunits = N >> 3;
    const int u0 = (int)(((long long)nunits * blockIdx.x) / gridDim.x);
    const int u1 = (int)(((long long)nunits * (blockIdx.x + 1)) / gridDim.x);
    const int row0 = u0 * 8, row1 = u1 * 8;
    const int ntiles = (row1 - row0 + kStageRows - 1) / kStageRows;
    const int total = ntiles * npan;
    // INT8 tiles: weights as the MMA's A operand (16 rows per instruction;
    // 3 % faster per decode step than activations as A, measured on B200);
    // the 4-bit tiles keep activations as A (their B fragments come from
    // 32-bit shared loads of the packed bytes)
    constexpr bool kSwap = !W4;
    const size_t slot = slot_bytes(P, W4);
    const int wrb = row_bytes(P, W4);  // weight bytes of a stage row
    uint8_t* act = smem;
    int* asum = reinterpret_cast<int*>(smem + geo.asum_off);  // 4-bit: [MMAX][K / 32]
    uint8_t* ring = smem + geo.act_bytes;

    if (threadIdx.x == 0) {
        for (int i = 0; i < S; i++) {
            mbar_init(&full_bar[i], 1);
            mbar_init(&empty_bar[i], kCWarps);
        }
        mbar_fence_init();
    }
    if (threadIdx.x < kMaxRows) best_s[threadIdx.x] = 0ull;
    __syncthreads();
    pdl_trigger();

    if (warp == kCWarps) {
        // ---------------- producer ----------------
        if (lane != 0) return;
        const uint8_t* sbase = reinterpret_cast<const uint8_t*>(p.sblk);
        auto issue = [&](int i) {
            const int sl = i % S;
            const int tile = i / npan, pan = i - tile * npan;
            const int r = row0 + tile * kStageRows;
            const int rows = min(kStageRows, row1 - r);
            uint8_t* dw = ring + (size_t)sl * slot;
            uint8_t* ds = dw + (size_t)kStageRows * wrb;
            const uint8_t* wsrc = W4 ? p.w4 : reinterpret_cast<const uint8_t*>(p.w);
            mbar_arrive_expect_tx(&full_bar[sl], (uint32_t)(rows * wrb + rows * (P / 16)));
            bulk_g2s(dw, wsrc + ((size_t)pan * N + r) * wrb, (uint32_t)(rows * wrb), &full_bar[sl]);
            bulk_g2s(ds, sbase + ((size_t)pan * N + r) * (P / 16), (uint32_t)(rows * (P / 16)), &full_bar[sl]);
        };
        const int first = total < S ? total : S;
        for (int i = 0; i < first; i++) issue(i);  // weights need no dependency
        pdl_wait();
        if (p.done && *p.done) return;
        for (int i = first; i < total; i++) {
            if (!mbar_wait(&empty_bar[i % S], ((i / S) - 1) & 1)) return;
            issue(i);
        }
        return;
    }

    // ---------------- consumers ----------------
    pdl_wait();
    if (p.done && *p.done) {
        const int first = total < S ? total : S;
        for (int i = 0; i < first; i++) mbar_wait(&full_bar[i], 0);  // drain the prefetch
        return;
    }
    int rows_m = p.M;
    if (p.dyn_M) rows_m = min(*p.dyn_M - p.row0, p.M);
    rows_m = max(0, min(rows_m, MMAX));
    const int ald = geo.act_ld;
    if (p.x) {
        const int src0 = p.x_row_dyn ? *p.x_row_dyn : p.row0;
        act_prologue_rows<kCWarps * 32, MMAX, false>(act, ald, p.x + (size_t)src0 * K, K, rows_m, p.norm, p.eps, nred,
                                              threadIdx.x, 1);
    } else {
        const int K16 = K >> 4;
        const uint4* src = reinterpret_cast<const uint4*>(p.aq + (size_t)p.row0 * K);
        for (int i = threadIdx.x; i < rows_m * K16; i += kCWarps * 32) {
            const int m = i / K16, c = i - m * K16;
            *reinterpret_cast<uint4*>(act + (size_t)m * ald + (size_t)c * 16) = src[(size_t)m * K16 + c];
        }
    }
    asm volatile("bar.sync 1, %0;" ::"n"(kCWarps * 32) : "memory");
    if (W4) {
        // per (row, block) sum of the u8 activations: the 4-bit dots are over
        // q = w + 8, so each block's dot is d(q) - 8 * sum
        const int nbk = K >> 5;
        for (int i = threadIdx.x; i < MMAX * nbk; i += kCWarps * 32) {
            const int m = i / nbk, b = i - m * nbk;
            int t = 0;
            if (m < rows_m) {
                const uint4* a = reinterpret_cast<const uint4*>(act + (size_t)m * ald + (size_t)b * 32);
                const uint4 x0 = a[0], x1 = a[1];
                const uint32_t one = 0x01010101u;
                t = (int)__dp4a(x0.x, one, 0u);
                t = (int)__dp4a(x0.y, one, (unsigned)t);
                t = (int)__dp4a(x0.z, one, (unsigned)t);
                t = (int)__dp4a(x0.w, one, (unsigned)t);
                t = (int)__dp4a(x1.x, one, (unsigned)t);
                t = (int)__dp4a(x1.y, one, (unsigned)t);
                t = (int)__dp4a(x1.z, one, (unsigned)t);
                t = (int)__dp4a(x1.w, one, (unsigned)t);
            }
            asum[i] = t;
        }
        asm volatile("bar.sync 1, %0;" ::"n"(kCWarps * 32) : "memory");
    }

    const int bpp = P >> 5;   // 32-element blocks per panel row
    bool bad = false;
    if (!MMA) {
        // ---- dp4a path: warp = row pair (2w, 2w + 1) of each 16-row stage ----
        float f0 = 0.0f, f1 = 0.0f;
        const int lr = 2 * warp;
        const int cpp = P >> 4;  // 16-byte chunks per panel row
        for (int i = 0; i < total; i++) {
            const int sl = i % S;
            const int tile = i / npan, pan = i - tile * npan;
            const int r = row0 + tile * kStageRows;
            const int rows = min(kStageRows, row1 - r);
            // After a timed-out wait keep looping without waiting or computing,
            // so every warp still reaches the same barriers and the kernel ends.
            if (!bad && !mbar_wait(&full_bar[sl], (i / S) & 1)) bad = true;
            if (!bad && lr < rows && rows_m > 0) {
                const bool two = lr + 1 < rows;
                const uint8_t* dw = ring + (size_t)sl * slot;
                const __half* ds = reinterpret_cast<const __half*>(dw + (size_t)kStageRows * wrb);
                const int ra = lr, rb = two ? lr + 1 : lr;
                const uint8_t* wa = dw + (size_t)ra * wrb;
                const uint8_t* wb = dw + (size_t)rb * wrb;
                if (W4) {
                    for (int c = lane; c < bpp; c += 32) {  // one 16-byte chunk = one block
                        const uint4 w0 = *reinterpret_cast<const uint4*>(wa + swz_chunk(c, r + ra) * 16);
                        const uint4 w1 = *reinterpret_cast<const uint4*>(wb + swz_chunk(c, r + rb) * 16);
                        const uint4* ap = reinterpret_cast<const uint4*>(act + (size_t)pan * P + (size_t)c * 32);
                        const uint4 x0 = ap[0], x1 = ap[1];
                        const int bsum = 8 * asum[pan * bpp + c];
                        const int d0 = dot_w4(x0, x1, w0) - bsum, d1 = dot_w4(x0, x1, w1) - bsum;
                        if (epi == EPI_DOTS) {
                            const int nbk = K >> 5;
                            int32_t* dd = p.dots + (size_t)p.row0 * N * nbk;
                            dd[(size_t)(r + ra) * nbk + pan * bpp + c] = d0;
                            if (two) dd[(size_t)(r + rb) * nbk + pan * bpp + c] = d1;
                        } else {
                            f0 = __fmaf_rn(i2f_exact(d0), __half2float(ds[ra * bpp + c]), f0);
                            f1 = __fmaf_rn(i2f_exact(d1), __half2float(ds[rb * bpp + c]), f1);
                        }
                    }
                } else {
                for (int c = lane; c < cpp; c += 32) {  // logical chunk within the panel row
                    const uint4 w0 = *reinterpret_cast<const uint4*>(wa + swz_chunk(c, r + ra) * 16);
                    const uint4 w1 = *reinterpret_cast<const uint4*>(wb + swz_chunk(c, r + rb) * 16);
                    const float s0 = __half2float(ds[ra * bpp + (c >> 1)]);
                    const float s1 = __half2float(ds[rb * bpp + (c >> 1)]);
                    const uint4 a = *reinterpret_cast<const uint4*>(act + (size_t)pan * P + (size_t)c * 16);
                    f0 = __fmaf_rn(i2f_exact(dot16(a, w0)), s0, f0);
                    f1 = __fmaf_rn(i2f_exact(dot16(a, w1)), s1, f1);
                }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty_bar[sl]);
            if (pan == npan - 1) {
                const float t0 = div127(warp_sum(f0));
                const float t1 = div127(warp_sum(f1));
                f0 = f1 = 0.0f;
                if (lane == 0 && lr < rows && rows_m > 0)
                    pair_epi_any<EPI>(epi, p, p.row0, r + lr, lr + 1 < rows, t0, t1, best_s);
            }
        }
    } else {
        // ---- MMA path: warp = a slice of the stage's blocks, all 16 rows ----
        const int g = lane >> 2, t = lane & 3;
        const int kb0 = (warp * bpp) / kCWarps, kb1 = ((warp + 1) * bpp) / kCWarps;
        float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        unsigned long long acc01 = 0ull, acc23 = 0ull;  // weights as A: (row g, row g + 8) x (col 2t, 2t + 1)
        int buf = 0;
        // ldmatrix row address of this lane: matrix j = lane / 8, row q = lane % 8
        const int lj = lane >> 3, lq = lane & 7;
        const int lrow = lq + 8 * (lj >> 1);
        const bool arow = g < rows_m;
        // byte offsets of this lane's ldmatrix row chunk for the four blocks of
        // a 128-byte swizzle group (chunk 2j + (lj & 1), rows at r + lrow with
        // r a multiple of 16)
        uint32_t goff[4];
#pragma unroll
        for (int j = 0; j < 4; j++) goff[j] = (uint32_t)(((2 * j + (lj & 1)) ^ (lrow & 7)) << 4);
        for (int i = 0; i < total; i++) {
            const int sl = i % S;
            const int tile = i / npan, pan = i - tile * npan;
            const int r = row0 + tile * kStageRows;
            const int rows = min(kStageRows, row1 - r);
            if (!bad && !mbar_wait(&full_bar[sl], (i / S) & 1)) bad = true;
            const uint8_t* dw = ring + (size_t)sl * slot;
            const __half* ds = reinterpret_cast<const __half*>(dw + (size_t)kStageRows * wrb);
            const uint32_t wrow = smem_u32(dw + (size_t)lrow * P);
            const uint8_t* arow_p = act + (size_t)g * ald + (size_t)pan * P;
            if (kSwap && (bpp & 31) == 0) {
                // Panels of a multiple of 1024 weights: every warp's block range
                // is whole groups of four blocks, i.e. whole 128-byte swizzle
                // groups; the four chunk offsets of a group are fixed per lane
                // (tile rows start at multiples of 16, so row & 7 = lane's row
                // & 7) and the fp16 scales of a group are one 8-byte load per
                // weight row. Same blocks in the same order as the loop below.
                for (int kg = kb0; kg < (bad ? kb0 : kb1); kg += 4) {
                    const uint32_t gbase = wrow + (uint32_t)((kg >> 2) << 7);
                    const uint2 sgv = *reinterpret_cast<const uint2*>(ds + g * bpp + kg);
                    const uint2 sg8v = *reinterpret_cast<const uint2*>(ds + (8 + g) * bpp + kg);
                    const uint32_t sgw[4] = {sgv.x, sgv.x >> 16, sgv.y, sgv.y >> 16};
                    const uint32_t sg8w[4] = {sg8v.x, sg8v.x >> 16, sg8v.y, sg8v.y >> 16};
#pragma unroll
                    for (int j = 0; j < 4; j++) {
                        const int kb = kg + j;
                        uint32_t b00, b01, b10, b11;
                        ldmatrix_x4(gbase + goff[j], b00, b01, b10, b11);
                        uint32_t a0 = 0, a2 = 0;
                        if (arow) {
                            a0 = *reinterpret_cast<const uint32_t*>(arow_p + kb * 32 + 4 * t);
                            a2 = *reinterpret_cast<const uint32_t*>(arow_p + kb * 32 + 16 + 4 * t);
                        }
                        int d0, d1, d2, d3;
                        mma_s8u8(b00, b10, b01, b11, a0, a2, d0, d1, d2, d3);
                        const float sg = __half2float(__ushort_as_half((unsigned short)(sgw[j] & 0xFFFFu)));
                        const float sg8 = __half2float(__ushort_as_half((unsigned short)(sg8w[j] & 0xFFFFu)));
                        acc01 = f2_fma(i2f2_exact(d0, d1), f2_pack(sg, sg), acc01);
                        acc23 = f2_fma(i2f2_exact(d2, d3), f2_pack(sg8, sg8), acc23);
                    }
                }
            } else
            for (int kb = kb0; kb < (bad ? kb0 : kb1); kb++) {
                uint32_t b00, b01, b10, b11;
                if (W4) {
                    // rows g and 8 + g of the tile, bytes 4t .. 4t + 3 of the block:
                    // low nibbles are elements 4t .. 4t + 3, high ones 16 + 4t ..
                    const uint32_t wa = *reinterpret_cast<const uint32_t*>(
                        dw + (size_t)g * wrb + swz_chunk(kb, r + g) * 16 + 4 * t);
                    const uint32_t wb = *reinterpret_cast<const uint32_t*>(
                        dw + (size_t)(8 + g) * wrb + swz_chunk(kb, r + 8 + g) * 16 + 4 * t);
                    b00 = wa & 0x0F0F0F0Fu;
                    b01 = (wa >> 4) & 0x0F0F0F0Fu;
                    b10 = wb & 0x0F0F0F0Fu;
                    b11 = (wb >> 4) & 0x0F0F0F0Fu;
                } else {
                    const int chunk = 2 * kb + (lj & 1);
                    ldmatrix_x4(wrow + swz_chunk(chunk, r + lrow) * 16, b00, b01, b10, b11);
                }
                uint32_t a0 = 0, a2 = 0;
                if (arow) {
                    a0 = *reinterpret_cast<const uint32_t*>(arow_p + kb * 32 + 4 * t);
                    a2 = *reinterpret_cast<const uint32_t*>(arow_p + kb * 32 + 16 + 4 * t);
                }
                int d0, d1, d2, d3;
                if (W4) {
                    mma_u8u8(a0, a2, b00, b01, d0, d1);
                    mma_u8u8(a0, a2, b10, b11, d2, d3);
                    const int bsum = arow ? 8 * asum[g * (K >> 5) + pan * bpp + kb] : 0;
                    d0 -= bsum;
                    d1 -= bsum;
                    d2 -= bsum;
                    d3 -= bsum;
                    if (epi == EPI_DOTS) {
                        if (arow) {
                            const int nbk = K >> 5;
                            int32_t* dd = p.dots + ((size_t)(p.row0 + g) * N) * nbk + pan * bpp + kb;
                            const int n0 = 2 * t, n1 = 8 + 2 * t;
                            if (n0 < rows) dd[(size_t)(r + n0) * nbk] = d0;
                            if (n0 + 1 < rows) dd[(size_t)(r + n0 + 1) * nbk] = d1;
                            if (n1 < rows) dd[(size_t)(r + n1) * nbk] = d2;
                            if (n1 + 1 < rows) dd[(size_t)(r + n1 + 1) * nbk] = d3;
                        }
                        continue;
                    }
                } else if (kSwap) {
                    // weights as A (rows g and g + 8), activations as B
                    // (columns 2t, 2t + 1): d0, d1 = row g; d2, d3 = row g + 8
                    mma_s8u8(b00, b10, b01, b11, a0, a2, d0, d1, d2, d3);
                    const float sg = __half2float(ds[g * bpp + kb]);
                    const float sg8 = __half2float(ds[(8 + g) * bpp + kb]);
                    // the scalar fma(i2f_exact(d), s, acc) of each column, two at a time
                    acc01 = f2_fma(i2f2_exact(d0, d1), f2_pack(sg, sg), acc01);
                    acc23 = f2_fma(i2f2_exact(d2, d3), f2_pack(sg8, sg8), acc23);
                    continue;
                }
                const float s0 = __half2float(ds[(2 * t) * bpp + kb]);
                const float s1 = __half2float(ds[(2 * t + 1) * bpp + kb]);
                const float s2 = __half2float(ds[(8 + 2 * t) * bpp + kb]);
                const float s3 = __half2float(ds[(9 + 2 * t) * bpp + kb]);
                acc[0] = __fmaf_rn(i2f_exact(d0), s0, acc[0]);
                acc[1] = __fmaf_rn(i2f_exact(d1), s1, acc[1]);
                acc[2] = __fmaf_rn(i2f_exact(d2), s2, acc[2]);
                acc[3] = __fmaf_rn(i2f_exact(d3), s3, acc[3]);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty_bar[sl]);
            if (pan == npan - 1) {
                // reduce the warps' block slices of this 16-row tile, then epilogue
                if (kSwap) {
                    acc[0] = f2_lo(acc01);
                    acc[1] = f2_hi(acc01);
                    acc[2] = f2_lo(acc23);
                    acc[3] = f2_hi(acc23);
                    acc01 = acc23 = 0ull;
                }
#pragma unroll
                for (int q = 0; q < 4; q++) red[buf][warp][lane][q] = acc[q];
                acc[0] = acc[1] = acc[2] = acc[3] = 0.0f;
                asm volatile("bar.sync 1, %0;" ::"n"(kCWarps * 32) : "memory");
                const int tid = threadIdx.x;
                if (tid < 64) {
                    const int pr = tid & 7, m = tid >> 3;  // row pair pr of the tile, activation row m
                    if (m < rows_m && 2 * pr < rows) {
                        // (weight row n, activation row m) of the tile lives in lane
                        // 4m + (n % 8) / 2, slot 2 (n / 8) + n % 2 (activations as A),
                        // or in lane 4 (n % 8) + m / 2, slot 2 (n / 8) + m % 2 (weights as A)
                        const int n0 = 2 * pr, n1 = 2 * pr + 1;
                        const int l0 = kSwap ? 4 * (n0 & 7) + (m >> 1) : 4 * m + ((n0 & 7) >> 1);
                        const int l1 = kSwap ? 4 * (n1 & 7) + (m >> 1) : 4 * m + ((n1 & 7) >> 1);
                        const int q0 = kSwap ? 2 * (n0 >> 3) + (m & 1) : 2 * (n0 >> 3) + (n0 & 1);
                        const int q1 = kSwap ? 2 * (n1 >> 3) + (m & 1) : 2 * (n1 >> 3) + (n1 & 1);
                        float y0 = 0.0f, y1 = 0.0f;
#pragma unroll
                        for (int w = 0; w < kCWarps; w++) {
                            y0 += red[buf][w][l0][q0];
                            y1 += red[buf][w][l1][q1];
                        }
                        pair_epi_any<EPI>(epi, p, p.row0 + m, r + 2 * pr, 2 * pr + 1 < rows, div127(y0),
                                           div127(y1), best_s);
                    }
                }
                buf ^= 1;
            }
        }
    }

    if (epi == EPI_LOGITS) {
        asm volatile("bar.sync 1, %0;" ::"n"(kCWarps * 32) : "memory");
        if (threadIdx.x < (unsigned)rows_m)
            p.amax_part[(size_t)(p.row0 + threadIdx.x) * gridDim.x + blockIdx.x] = best_s[threadIdx.x];
    }
    if (epi == EPI_TP_PUSH) {
        // this CTA's rows are on every rank: publish (system-scope fence, then count)
        __threadfence_system();
        asm volatile("bar.sync 1, %0;" ::"n"(kCWarps * 32) : "memory");
        if (threadIdx.x == 0) {
            const int par = (int)(*p.tp_seq & 1ull);
            for (int q = 0; q < p.tp_size; q++) atomicAdd(p.tp_cnt[q] + par * p.tp_size + p.tp_rank, 1ull);
        }
    }
}

__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* a) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(a) : "memory");
    return v;
}

__global__ void __launch_bounds__(256) tp_reduce_kernel(const TpReduceParams p) {
    __shared__ int ok_s;
    pdl_trigger();
    pdl_wait();
    if (p.done && *p.done) return;  // every rank skips the same reductions
    const unsigned long long s = *p.seq;
    const int par = (int)(s & 1ull);
    const unsigned long long need = p.ctas_per_push * (s / 2 + 1);
    if (threadIdx.x == 0) ok_s = 1;
    __syncthreads();
    if (threadIdx.x < (unsigned)p.size) {
        const unsigned long long* c = p.cnt + par * p.size + threadIdx.x;
        if (ld_acquire_sys(c) < need) {
            const long long t0 = clock64();
            int spins = 0;
            while (ld_acquire_sys(c) < need) {
                __nanosleep(64);
                // a bound of about two seconds of cycles: peers that never push raise the error
                if (++spins % 1024 == 0 && clock64() - t0 > 4000000000ll) {
                    atomicOr(&g_fl_error, kErrMbarTimeout);
                    ok_s = 0;
                    break;
                }
            }
        }
    }
    __syncthreads();
    if (!ok_s) return;
    const int rows = p.dyn_rows ? min(*p.dyn_rows, p.rows) : p.rows;
    const size_t total = (size_t)rows * p.d;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const size_t m = i / p.d, n = i - m * p.d;
        float v = p.x[i];
        for (int q = 0; q < p.size; q++) v = __fadd_rn(v, p.recv[(((size_t)par * p.size + q) * p.cap + m) * p.d + n]);
        p.x[i] = v;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        if (atomicAdd(p.arrived, 1) == (int)gridDim.x - 1) {
            *p.arrived = 0;
            __threadfence();
            *p.seq = s + 1;
        }
    }
}

int g_sm_count[16] = {0};

int sm_count() {
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 16 && g_sm_count[dev]) return g_sm_count[dev];
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (dev < 16) g_sm_count[dev] = n;
    return n;
}

template <int MMAX, int EPI, bool MMA, bool W4>
cudaError_t launch_t(const GemvParams& p, const Geo& geo, cudaStream_t s, bool pdl, int epi) {
    auto kern = gemv_tma_kernel<MMAX, EPI, MMA, W4>;
    const size_t smem = (size_t)geo.act_bytes + (size_t)geo.S * slot_bytes(geo.P, W4);
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(sm_count() * kCtasPerSm);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, p, geo, epi);
}

template <int EPI>
cudaError_t launch_e(const GemvParams& p, const Geo& geo, cudaStream_t s, bool pdl, int epi) {
    if (p.w4) {
        if (p.M <= 1) return launch_t<1, EPI, false, true>(p, geo, s, pdl, epi);
        if (p.M <= 2) return launch_t<2, EPI, true, true>(p, geo, s, pdl, epi);
        if (p.M <= 4) return launch_t<4, EPI, true, true>(p, geo, s, pdl, epi);
        return launch_t<8, EPI, true, true>(p, geo, s, pdl, epi);
    }
    if (p.M <= 1) return launch_t<1, EPI, false, false>(p, geo, s, pdl, epi);
    if (p.M <= 2) return launch_t<2, EPI, true, false>(p, geo, s, pdl, epi);
    if (p.M <= 4) return launch_t<4, EPI, true, false>(p, geo, s, pdl, epi);
    return launch_t<8, EPI, true, false>(p, geo, s, pdl, epi);
}

}  // namespace

int tma_gemv_grid() { return sm_count() * kCtasPerSm; }

int take_device_error() {
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_fl_error, sizeof(int)) != cudaSuccess) return -1;
    if (v) {
        const int z = 0;
        cudaMemcpyToSymbol(g_fl_error, &z, sizeof(int));
    }
    const int w = take_gemm_error();
    return w < 0 ? w : (v | w);
}

bool tma_gemv_supported(int N, int K, int M) {
    Geo g;
    return N > 0 && N % 8 == 0 && make_geo(K, M, g);
}

// p.M: rows held in shared memory (a static count, or the upper bound of
// *p.dyn_M), 1..kMaxRows. Weights must be in the tiled layout (p.P != 0).
cudaError_t launch_gemv_tma(const GemvParams& p, int epi, cudaStream_t s, bool pdl) {
    if (p.M <= 0 || p.M > kMaxRows || p.N % 8 != 0 || p.P == 0) return cudaErrorInvalidValue;
    Geo geo;
    if (!make_geo(p.K, p.M, geo, p.P, p.w4 != nullptr)) return cudaErrorInvalidValue;
    if (p.x && p.K % 128 != 0) return cudaErrorInvalidValue;
    // integer block dots only from 4-bit weights (the INT8 ones go through gemv_i8.cu)
    if (epi < EPI_STORE || epi > EPI_TP_PUSH || (epi == EPI_DOTS && !p.w4)) return cudaErrorInvalidValue;
    // One kernel body per row count for every epilogue: the epilogue is
    // chosen at run time, so the launches of a layer run the same code and
    // find it in the SM's instruction caches (7 % faster per decode step than
    // one specialised kernel per epilogue, measured on B200).
    return launch_e<-1>(p, geo, s, pdl, epi);
}

cudaError_t launch_tp_reduce(const TpReduceParams& p, cudaStream_t s, bool pdl) {
    if (p.rows <= 0 || p.rows > p.cap || p.size < 1 || p.size > 256) return cudaErrorInvalidValue;
    const int blocks = std::min(32, (int)(((size_t)p.rows * p.d + 1023) / 1024));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(blocks);
    cfg.blockDim = dim3(256);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, tp_reduce_kernel, p);
}

cudaError_t launch_gemv_auto(const GemvParams& p, int epi, cudaStream_t s, bool pdl) {
    Geo geo;
    if (p.w4 && p.P != 0 && p.N % 8 == 0 && make_geo(p.K, p.M, geo, p.P, true)) return launch_gemv_tma(p, epi, s, pdl);
    GemvParams q = p;  // the INT8 copy serves every other case
    q.w4 = nullptr;
    if (epi != EPI_DOTS && q.P != 0 && q.N % 8 == 0 && make_geo(q.K, q.M, geo, q.P)) return launch_gemv_tma(q, epi, s, pdl);
    return launch_gemv(q, epi, false, false, s, pdl);
}

int gemv_auto_grid(int N, int K) { return tma_gemv_supported(N, K, kMaxRows) ? tma_gemv_grid() : gemv_grid(N); }

}  // namespace fl
