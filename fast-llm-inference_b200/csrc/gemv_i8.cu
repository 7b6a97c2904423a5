// INT8 weight GEMV / skinny GEMM for M <= 8 activation rows (sm_100a).
//
// Replaces matmul_dequantized (fast_llm/src/kernels/dequantized_tensor.c:
// 204-247) and the per-row matvec loops of transformer_layer
// (fast_llm/src/inference.c:286-386). HBM-bound: every weight byte is read
// once per launch with 16-byte streaming loads; activations (already
// quantized to u8) sit in shared memory and are reused across the M rows.
//
// Work split: one warp owns a pair of consecutive weight rows (n, n+1) for
// the whole K; lane l reads bytes [512c + 16l, +16) of both rows for chunk c.
// The two rows of a pair are what the fused epilogues need side by side: a
// RoPE (i, i+1) rotation pair, or an interleaved (gate_i, up_i) pair.
// Weight loads for the next chunk batch are in flight while the current
// batch is multiplied (register double buffering), and the first batch is
// issued before griddepcontrol.wait so it overlaps the previous kernel.
#include "fl_common.cuh"
#include "fl_kernels.h"
#include "fl_epilogue.cuh"
#include "fl_layout.cuh"

namespace fl {

namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kU = 2;  // 512-byte chunks per batch per row

struct Batch {
    uint4 w0[kU], w1[kU];
    float s0[kU], s1[kU];
};

template <bool ROWMODE>
__device__ __forceinline__ void load_batch(Batch& b, const GemvParams& p, const int8_t* w0,
                                           const int8_t* w1, int n0, int n1, int c0, int lane,
                                           int nchunk) {
#pragma unroll
    for (int u = 0; u < kU; u++) {
        const int c = c0 + u;
        const int k = c * 512 + lane * 16;
        const bool ok = (c < nchunk) && (k < p.K);
        if (ok) {
            if (p.P) {  // tiled layout (fl_layout.cuh)
                b.w0[u] = ld_stream16(p.w + tiled_w_off(p.N, p.P, n0, k >> 4));
                b.w1[u] = ld_stream16(p.w + tiled_w_off(p.N, p.P, n1, k >> 4));
                b.s0[u] = __half2float(p.sblk[tiled_s_off(p.N, p.P, n0, k >> 5)]);
                b.s1[u] = __half2float(p.sblk[tiled_s_off(p.N, p.P, n1, k >> 5)]);
                continue;
            }
            b.w0[u] = ld_stream16(w0 + k);
            b.w1[u] = ld_stream16(w1 + k);
            if (!ROWMODE) {
                const size_t kb = (size_t)(p.K >> 5);
                b.s0[u] = __half2float(p.sblk[(size_t)n0 * kb + (k >> 5)]);
                b.s1[u] = __half2float(p.sblk[(size_t)n1 * kb + (k >> 5)]);
            }
        } else {
            b.w0[u] = make_uint4(0, 0, 0, 0);
            b.w1[u] = make_uint4(0, 0, 0, 0);
            b.s0[u] = 0.0f;
            b.s1[u] = 0.0f;
        }
    }
}

template <bool PAIRSAT>
__device__ __forceinline__ int dot16(const uint4& a, const uint4& w) {
    if (PAIRSAT) {
        int d = dp4_pairsat(a.x, w.x, 0);
        d = dp4_pairsat(a.y, w.y, d);
        d = dp4_pairsat(a.z, w.z, d);
        return dp4_pairsat(a.w, w.w, d);
    } else {
        int d = dp4a_us(a.x, w.x, 0);
        d = dp4a_us(a.y, w.y, d);
        d = dp4a_us(a.z, w.z, d);
        return dp4a_us(a.w, w.w, d);
    }
}

template <int MMAX, bool ROWMODE, bool PAIRSAT, int EPI>
__device__ __forceinline__ void compute_batch(const Batch& b, const uint4* act, int K16, int rows,
                                              int c0, int lane, int nchunk, int K,
                                              float (&f0)[MMAX], float (&f1)[MMAX],
                                              int (&i0)[MMAX], int (&i1)[MMAX],
                                              const GemvParams& p, int n0, bool has1) {
#pragma unroll
    for (int u = 0; u < kU; u++) {
        const int c = c0 + u;
        const int k = c * 512 + lane * 16;
        const bool ok = (c < nchunk) && (k < K);
        if (EPI == EPI_DOTS) {
            if (c >= nchunk) continue;  // warp-uniform
#pragma unroll
            for (int m = 0; m < MMAX; m++) {
                if (m >= rows) break;
                uint4 a = ok ? act[m * K16 + c * 32 + lane] : make_uint4(0, 0, 0, 0);
                int d0 = dot16<PAIRSAT>(a, b.w0[u]);
                int d1 = dot16<PAIRSAT>(a, b.w1[u]);
                d0 += __shfl_xor_sync(0xffffffffu, d0, 1);
                d1 += __shfl_xor_sync(0xffffffffu, d1, 1);
                if (ok && (lane & 1) == 0) {
                    const int kb = K >> 5;
                    const int blk = k >> 5;
                    const int r = p.row0 + m;
                    p.dots[((size_t)r * p.N + n0) * kb + blk] = d0;
                    if (has1) p.dots[((size_t)r * p.N + n0 + 1) * kb + blk] = d1;
                }
            }
            continue;
        }
        if (!ok) continue;
#pragma unroll
        for (int m = 0; m < MMAX; m++) {
            if (m < rows) {
                const uint4 a = act[m * K16 + c * 32 + lane];
                const int d0 = dot16<PAIRSAT>(a, b.w0[u]);
                const int d1 = dot16<PAIRSAT>(a, b.w1[u]);
                if (ROWMODE) {
                    i0[m] += d0;
                    i1[m] += d1;
                } else {
                    f0[m] = __fmaf_rn(i2f_exact(d0), b.s0[u], f0[m]);
                    f1[m] = __fmaf_rn(i2f_exact(d1), b.s1[u], f1[m]);
                }
            }
        }
    }
}

// Epilogue for one (row m, weight row n) value owned by this lane.
template <int EPI>
__device__ __forceinline__ void store_one(const GemvParams& p, int r, int n, float y) {
    if (EPI == EPI_STORE || EPI == EPI_LOGITS) {
        p.out[(size_t)r * p.ldo + n] = y;
    } else if (EPI == EPI_RESID) {
        float* o = p.out + (size_t)r * p.ldo + n;
        *o = __fadd_rn(*o, y);
    }
}

template <int MMAX, bool ROWMODE, bool PAIRSAT, int EPI>
__global__ void __launch_bounds__(kThreads) gemv_i8_kernel(const GemvParams p) {
    extern __shared__ uint4 act_s[];
    __shared__ unsigned long long red_s[kWarps][kMaxRows];

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int pair = blockIdx.x * kWarps + warp;
    const int n0 = pair * 2;
    const bool active = n0 < p.N;
    const bool has1 = active && (n0 + 1 < p.N);
    const int n1 = has1 ? n0 + 1 : n0;
    const int K = p.K;
    const int nchunk = (K + 511) >> 9;
    const int8_t* w0 = p.w + (size_t)(active ? n0 : 0) * K;
    const int8_t* w1 = p.w + (size_t)(active ? n1 : 0) * K;

    pdl_trigger();

    // Weights never depend on earlier kernels: start streaming them now.
    Batch ba, bb;
    if (active) load_batch<ROWMODE>(ba, p, w0, w1, n0, n1, 0, lane, nchunk);

    pdl_wait();
    if (p.done && *p.done) return;
    int rows = p.M;
    if (p.dyn_M) rows = min(*p.dyn_M - p.row0, p.M);
    rows = min(rows, MMAX);
    if (rows <= 0) return;

    // Quantized activations of this launch's rows into shared memory.
    const int K16 = K >> 4;
    if (p.x) {
        const int src0 = p.x_row_dyn ? *p.x_row_dyn : p.row0;
        act_prologue(reinterpret_cast<uint8_t*>(act_s), p.x + (size_t)src0 * K, K, rows, p.norm, p.eps, warp, lane,
                     kWarps);
    } else {
        const uint4* src = reinterpret_cast<const uint4*>(p.aq + (size_t)p.row0 * K);
        const int total = rows * K16;
        for (int i = threadIdx.x; i < total; i += kThreads) act_s[i] = src[i];
    }
    __syncthreads();

    float f0[MMAX], f1[MMAX];
    int i0[MMAX], i1[MMAX];
#pragma unroll
    for (int m = 0; m < MMAX; m++) { f0[m] = f1[m] = 0.0f; i0[m] = i1[m] = 0; }

    if (active) {
        for (int c0 = 0; c0 < nchunk; c0 += 2 * kU) {
            if (c0 + kU < nchunk) load_batch<ROWMODE>(bb, p, w0, w1, n0, n1, c0 + kU, lane, nchunk);
            compute_batch<MMAX, ROWMODE, PAIRSAT, EPI>(ba, act_s, K16, rows, c0, lane, nchunk, K,
                                                       f0, f1, i0, i1, p, n0, has1);
            if (c0 + kU >= nchunk) break;
            if (c0 + 2 * kU < nchunk) load_batch<ROWMODE>(ba, p, w0, w1, n0, n1, c0 + 2 * kU, lane, nchunk);
            compute_batch<MMAX, ROWMODE, PAIRSAT, EPI>(bb, act_s, K16, rows, c0 + kU, lane, nchunk, K,
                                                       f0, f1, i0, i1, p, n0, has1);
        }
    }
    if (EPI == EPI_DOTS) return;

    // Reduce over lanes; lane j then owns value (m = j >> 1, row j & 1).
    float y_own = 0.0f;
    const int m_own = lane >> 1;
    const int sel = lane & 1;
    float ypair0 = 0.0f, ypair1 = 0.0f;  // (row n0, row n1) values of row m = lane
#pragma unroll
    for (int m = 0; m < MMAX; m++) {
        if (m < rows) {
            float t0, t1;
            if (ROWMODE) {
                const int s0 = warp_sum_i(i0[m]);
                const int s1 = warp_sum_i(i1[m]);
                // dequantized_tensor.c:243 as compiled: (dot * scale) * (1/2032)
                t0 = __fmul_rn(__fmul_rn((float)s0, p.srow[active ? n0 : 0]), 1.0f / 2032.0f);
                t1 = __fmul_rn(__fmul_rn((float)s1, p.srow[active ? n1 : 0]), 1.0f / 2032.0f);
            } else {
                t0 = div127(warp_sum(f0[m]));
                t1 = div127(warp_sum(f1[m]));
            }
            if (m == m_own) y_own = sel ? t1 : t0;
            if (m == lane) { ypair0 = t0; ypair1 = t1; }
        }
    }

    if (EPI == EPI_STORE || EPI == EPI_RESID) {
        if (active && m_own < rows && (sel == 0 || has1))
            store_one<EPI>(p, p.row0 + m_own, n0 + sel, y_own);
    } else if (EPI == EPI_LOGITS) {
        if (active && m_own < rows && (sel == 0 || has1))
            store_one<EPI>(p, p.row0 + m_own, n0 + sel, y_own);
        // Per-CTA argmax partial for each row.
        unsigned long long key = 0ull;
        if (active && lane < rows) {
            key = argmax_key(ypair0, n0);
            if (has1) {
                unsigned long long k1 = argmax_key(ypair1, n1);
                key = k1 > key ? k1 : key;
            }
        }
        if (lane < kMaxRows) red_s[warp][lane] = key;
        __syncthreads();
        if (threadIdx.x < (unsigned)rows) {
            unsigned long long best = 0ull;
            for (int w = 0; w < kWarps; w++) {
                unsigned long long k = red_s[w][threadIdx.x];
                best = k > best ? k : best;
            }
            p.amax_part[(size_t)(p.row0 + threadIdx.x) * gridDim.x + blockIdx.x] = best;
        }
    } else if (EPI == EPI_QKV) {
        // lane m handles row m: rotate (n0, n1) if in the q or k region.
        if (active && lane < rows) {
            const int r = p.row0 + lane;
            float v0 = ypair0, v1 = ypair1;
            const int qkd = p.q_dim + p.kv_dim;
            if (n0 < qkd) {
                const int i = (n0 < p.q_dim ? n0 : n0 - p.q_dim) % p.head_dim;
                // inference.c:165-173 (theta from the model configuration)
                const float freq = __fdiv_rn(1.0f, powf(p.theta, __fdiv_rn((float)i, (float)p.head_dim)));
                const float ang = __fmul_rn((float)row_pos(p, r), freq);
                float sn, cs;
                sincosf(ang, &sn, &cs);
                const float a = v0, b = v1;
                v0 = __fsub_rn(__fmul_rn(a, cs), __fmul_rn(b, sn));
                v1 = __fadd_rn(__fmul_rn(a, sn), __fmul_rn(b, cs));
            }
            if (n0 < p.q_dim) {
                p.q_out[(size_t)r * p.q_dim + n0] = v0;
                p.q_out[(size_t)r * p.q_dim + n0 + 1] = v1;
            } else {
                const bool is_k = n0 < qkd;
                const int c = n0 - (is_k ? p.q_dim : qkd);
                const int h = c / p.head_dim;
                const int dd = c - h * p.head_dim;
                const int slot = row_slot(p, r);
                const int page = p.block_table[slot / kPageSize];
                const size_t off = (((size_t)page * p.kv_heads + h) * kPageSize + (slot % kPageSize)) *
                                       p.head_dim + dd;
                __half2* dst = reinterpret_cast<__half2*>((is_k ? p.kv.k : p.kv.v) + off);
                *dst = __floats2half2_rn(v0, v1);
            }
        }
    } else if (EPI == EPI_SWIGLU) {
        // rows (n0, n1) = (gate_i, up_i): activations_avx2.c:86-105.
        if (active && lane < rows) {
            const int r = p.row0 + lane;
            const float g = ypair0, u = ypair1;
            const float h = __fmul_rn(__fmul_rn(g, poly_sigmoid(g)), u);
            p.hq[(size_t)r * p.F + (n0 >> 1)] = (uint8_t)quant_u8(h);
        }
    }
}

template <int MMAX, bool ROWMODE, bool PAIRSAT, int EPI>
cudaError_t launch_t(const GemvParams& p, cudaStream_t s, bool pdl) {
    auto kern = gemv_i8_kernel<MMAX, ROWMODE, PAIRSAT, EPI>;
    const size_t smem = (size_t)MMAX * p.K;
    if (smem > 200 * 1024) return cudaErrorInvalidValue;
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(gemv_grid(p.N));
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, p);
}

template <bool ROWMODE, bool PAIRSAT, int EPI>
cudaError_t launch_m(const GemvParams& p, cudaStream_t s, bool pdl) {
    const int m = p.M;
    if (m <= 1) return launch_t<1, ROWMODE, PAIRSAT, EPI>(p, s, pdl);
    if (m <= 2) return launch_t<2, ROWMODE, PAIRSAT, EPI>(p, s, pdl);
    if (m <= 4) return launch_t<4, ROWMODE, PAIRSAT, EPI>(p, s, pdl);
    return launch_t<8, ROWMODE, PAIRSAT, EPI>(p, s, pdl);
}

template <int EPI>
cudaError_t launch_e(const GemvParams& p, bool rowmode, bool pairsat, cudaStream_t s, bool pdl) {
    if (rowmode) {
        if (pairsat) return launch_m<true, true, EPI>(p, s, pdl);
        return launch_m<true, false, EPI>(p, s, pdl);
    }
    return launch_m<false, false, EPI>(p, s, pdl);
}

}  // namespace

int gemv_grid(int N) { return ((N + 1) / 2 + kWarps - 1) / kWarps; }

namespace {

__global__ void relayout_w_kernel(const int8_t* src, int rows, int K, int8_t* dst, int N, int P, int row0,
                                  int stride) {
    const int cpr = K >> 4;
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long long)rows * cpr) return;
    const int r = (int)(i / cpr), c = (int)(i - (long long)r * cpr);
    const int n = row0 + r * stride;
    *reinterpret_cast<uint4*>(dst + tiled_w_off(N, P, n, c)) =
        *reinterpret_cast<const uint4*>(src + (size_t)r * K + (size_t)c * 16);
}

__global__ void relayout_s_kernel(const __half* src, int rows, int K, __half* dst, int N, int P, int row0,
                                  int stride) {
    const int bpr = K >> 5;
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long long)rows * bpr) return;
    const int r = (int)(i / bpr), b = (int)(i - (long long)r * bpr);
    dst[tiled_s_off(N, P, row0 + r * stride, b)] = src[(size_t)r * bpr + b];
}

}  // namespace

cudaError_t upload_rows(int8_t* dst_w, __half* dst_s, int N, int K, int P, int dst_row0, int dst_stride,
                        const int8_t* host_w, const uint16_t* host_s, int rows, cudaStream_t s) {
    const size_t kb = (size_t)K / 32;
    if (P == 0) {
        cudaError_t e = cudaMemcpy2DAsync(dst_w + (size_t)dst_row0 * K, (size_t)dst_stride * K, host_w, K, K, rows,
                                          cudaMemcpyHostToDevice, s);
        if (e != cudaSuccess) return e;
        e = cudaMemcpy2DAsync(dst_s + (size_t)dst_row0 * kb, (size_t)dst_stride * kb * sizeof(__half), host_s,
                              kb * sizeof(__half), kb * sizeof(__half), rows, cudaMemcpyHostToDevice, s);
        if (e != cudaSuccess) return e;
        return cudaStreamSynchronize(s);
    }
    if (K % P != 0 || P % 128 != 0 || dst_row0 + (rows - 1) * dst_stride >= N) return cudaErrorInvalidValue;
    int8_t* tw = nullptr;
    __half* ts = nullptr;
    cudaError_t e = cudaMalloc(&tw, (size_t)rows * K);
    if (e == cudaSuccess) e = cudaMalloc(&ts, (size_t)rows * kb * sizeof(__half));
    if (e == cudaSuccess) e = cudaMemcpyAsync(tw, host_w, (size_t)rows * K, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(ts, host_s, (size_t)rows * kb * sizeof(__half), cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) {
        const long long nw = (long long)rows * (K / 16), ns = (long long)rows * (long long)kb;
        relayout_w_kernel<<<(unsigned)((nw + 255) / 256), 256, 0, s>>>(tw, rows, K, dst_w, N, P, dst_row0, dst_stride);
        relayout_s_kernel<<<(unsigned)((ns + 255) / 256), 256, 0, s>>>(ts, rows, K, dst_s, N, P, dst_row0,
                                                                        dst_stride);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    cudaFree(tw);
    cudaFree(ts);
    return e;
}

cudaError_t launch_gemv(const GemvParams& p, int epi, bool rowmode, bool pairsat, cudaStream_t s,
                        bool pdl) {
    if (p.K % 32 != 0 || p.N <= 0 || p.K <= 0) return cudaErrorInvalidValue;
    if (p.x && p.K % 128 != 0) return cudaErrorInvalidValue;
    if (p.M <= 0 || p.M > kMaxRows) return cudaErrorInvalidValue;
    switch (epi) {
        case EPI_STORE: return launch_e<EPI_STORE>(p, rowmode, pairsat, s, pdl);
        case EPI_RESID: return launch_e<EPI_RESID>(p, rowmode, pairsat, s, pdl);
        case EPI_DOTS: return launch_e<EPI_DOTS>(p, rowmode, pairsat, s, pdl);
        // the fused model epilogues only exist for block-mode weights
        case EPI_QKV: return launch_m<false, false, EPI_QKV>(p, s, pdl);
        case EPI_SWIGLU: return launch_m<false, false, EPI_SWIGLU>(p, s, pdl);
        case EPI_LOGITS: return launch_m<false, false, EPI_LOGITS>(p, s, pdl);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace fl
