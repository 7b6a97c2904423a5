// Persistent INT8 GEMV streaming weights through a TMA bulk-copy ring
// (sm_100a). Same contract and epilogues as gemv_i8.cu's block-mode kernel
// (matmul_dequantized, dequantized_tensor.c:204-247, with the fused layer
// epilogues of inference.c:286-386), built for bs1 decode where a launch is
// only 9-100 MB and must not be latency bound:
//
//   * one CTA per SM, each owning a contiguous range of weight-row pairs;
//   * a producer warp issues 1-D cp.async.bulk copies of whole row segments
//     (weights + their fp16 block scales) into an S-stage shared-memory ring
//     -- up to ~200 KB in flight per SM -- starting BEFORE
//     griddepcontrol.wait, so the stream overlaps the previous kernel's tail;
//   * 8 consumer warps each take one row pair of a 16-row stage, multiply
//     with dp4a against the u8 activations held in shared memory, and release
//     the slot through an mbarrier;
//   * every mbarrier wait is bounded (fl_tma.cuh).
#include "fl_common.cuh"
#include "fl_kernels.h"
#include "fl_tma.cuh"

namespace fl {

namespace {

constexpr int kCWarps = 16;                  // consumer warps
constexpr int kThreads = (kCWarps + 1) * 32; // + producer warp
constexpr int kRowsPerStage = 2 * kCWarps;   // one row pair per consumer warp
constexpr int kMaxStages = 8;
// Ring budget: ~half the SM's shared memory, so that the CTA of the next
// kernel in the stream (launched early by PDL) fits beside this one and
// starts its own weight stream while this kernel drains.
constexpr int kSmemLimit = 112 * 1024;
constexpr int kMaxSeg = 2048;

struct TmaShape {
    int seg;      // bytes of one row segment (K / nseg)
    int nseg;
    int stages;
    size_t smem;  // dynamic shared memory
    size_t act_bytes;
};

inline size_t stage_bytes(int seg) { return (size_t)kRowsPerStage * seg + (size_t)kRowsPerStage * (seg / 16); }

// Ring geometry for K and `mrows` activation rows held in shared memory:
// the largest row segment (a multiple of 512 bytes dividing K, at most
// kMaxSeg) that still leaves >= 3 stages, else >= 2.
inline bool tma_shape(int K, int mrows, TmaShape& s) {
    if (K % 256 != 0 || mrows < 1 || mrows > kMaxRows) return false;
    s.act_bytes = ((size_t)mrows * K + 127) & ~(size_t)127;
    if (s.act_bytes + 256 >= (size_t)kSmemLimit) return false;
    const size_t avail = kSmemLimit - s.act_bytes - 256;
    for (int want = 3; want >= 2; want--) {
        for (int n = 1; n <= 64; n++) {
            if (K % n || (K / n) > kMaxSeg || (K / n) % 512) continue;
            const int seg = K / n;
            const int st = (int)(avail / stage_bytes(seg));
            if (st >= want) {
                s.seg = seg;
                s.nseg = n;
                s.stages = st > kMaxStages ? kMaxStages : st;
                s.smem = s.act_bytes + (size_t)s.stages * stage_bytes(seg);
                return true;
            }
        }
    }
    return false;
}

template <bool PAIR_ROWS>
__device__ __forceinline__ int dot16(const uint4& a, const uint4& w) {
    int d = dp4a_us(a.x, w.x, 0);
    d = dp4a_us(a.y, w.y, d);
    d = dp4a_us(a.z, w.z, d);
    return dp4a_us(a.w, w.w, d);
}

template <int MMAX, int EPI>
__global__ void __launch_bounds__(kThreads, 1) gemv_tma_kernel(const GemvParams p, const int seg, const int nseg,
                                                               const int S, const int act_bytes) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ __align__(8) uint64_t full_bar[kMaxStages];
    __shared__ __align__(8) uint64_t empty_bar[kMaxStages];
    __shared__ unsigned long long red_s[kCWarps][kMaxRows];

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int K = p.K;
    const int npairs = (p.N + 1) >> 1;
    const int pr0 = (int)(((long long)npairs * blockIdx.x) / gridDim.x);
    const int pr1 = (int)(((long long)npairs * (blockIdx.x + 1)) / gridDim.x);
    const int row0 = 2 * pr0;
    const int row1 = min(2 * pr1, p.N);
    const int nrows = row1 - row0;
    const int nrounds = (nrows + kRowsPerStage - 1) / kRowsPerStage;
    const int total = nrounds * nseg;
    const int sw = kRowsPerStage * seg;           // weight bytes of a full stage
    const int ss = kRowsPerStage * (seg / 16);    // scale bytes of a full stage
    uint8_t* act = smem;
    uint8_t* ring = smem + act_bytes;

    if (threadIdx.x == 0) {
        for (int i = 0; i < S; i++) {
            mbar_init(&full_bar[i], 1);
            mbar_init(&empty_bar[i], kCWarps);
        }
        mbar_fence_init();
    }
    __syncthreads();
    pdl_trigger();

    const int8_t* wbase = p.w;
    const uint8_t* sbase = reinterpret_cast<const uint8_t*>(p.sblk);
    const size_t srow = (size_t)(K / 16);  // scale bytes per weight row

    if (warp == kCWarps) {
        // ---------------- producer ----------------
        if (lane != 0) return;
        const int first = total < S ? total : S;
        auto issue = [&](int i) {
            const int slot = i % S;
            const int round = i / nseg, sg = i - round * nseg;
            const int r = row0 + round * kRowsPerStage;
            const int rows = min(kRowsPerStage, row1 - r);
            uint8_t* dw = ring + (size_t)slot * (sw + ss);
            uint8_t* ds = dw + sw;
            mbar_arrive_expect_tx(&full_bar[slot], (uint32_t)(rows * (seg + seg / 16)));
            for (int j = 0; j < rows; j++) {
                bulk_g2s(dw + (size_t)j * seg, wbase + (size_t)(r + j) * K + (size_t)sg * seg, seg, &full_bar[slot]);
                bulk_g2s(ds + (size_t)j * (seg / 16), sbase + (size_t)(r + j) * srow + (size_t)sg * (seg / 16),
                         seg / 16, &full_bar[slot]);
            }
        };
        for (int i = 0; i < first; i++) issue(i);  // weights need no dependency
        pdl_wait();
        if (p.done && *p.done) return;
        for (int i = first; i < total; i++) {
            const int slot = i % S;
            if (!mbar_wait(&empty_bar[slot], ((i / S) - 1) & 1)) return;
            issue(i);
        }
        return;
    }

    // ---------------- consumers ----------------
    pdl_wait();
    if (p.done && *p.done) {
        // drain the prefetched stages before leaving
        const int first = total < S ? total : S;
        for (int i = 0; i < first; i++) mbar_wait(&full_bar[i], 0);
        return;
    }
    // p.M bounds the rows (shared memory holds p.M rows); dyn_M narrows it.
    int rows_m = p.M;
    if (p.dyn_M) rows_m = min(*p.dyn_M - p.row0, p.M);
    rows_m = min(rows_m, MMAX);
    if (p.x) {
        const int src0 = p.x_row_dyn ? *p.x_row_dyn : p.row0;
        act_prologue(act, p.x + (size_t)src0 * K, K, max(rows_m, 0), p.norm, p.eps, warp, lane, kCWarps);
    } else {
        const int K16 = K >> 4;
        const uint4* src = reinterpret_cast<const uint4*>(p.aq + (size_t)p.row0 * K);
        uint4* dst = reinterpret_cast<uint4*>(act);
        const int tot = max(rows_m, 0) * K16;
        for (int i = threadIdx.x; i < tot; i += kCWarps * 32) dst[i] = src[i];
    }
    asm volatile("bar.sync 1, %0;" ::"n"(kCWarps * 32) : "memory");

    float f0[MMAX], f1[MMAX];
#pragma unroll
    for (int m = 0; m < MMAX; m++) f0[m] = f1[m] = 0.0f;
    unsigned long long best = 0ull;  // EPI_LOGITS: lane m keeps row m's best key
    const uint4* act4 = reinterpret_cast<const uint4*>(act);
    const int K16 = K >> 4;
    const int nj = seg >> 9;  // 512-byte sweeps per segment

    for (int i = 0; i < total; i++) {
        const int slot = i % S;
        const int round = i / nseg, sg = i - round * nseg;
        const int r = row0 + round * kRowsPerStage;
        const int rows = min(kRowsPerStage, row1 - r);
        // On a timeout stop consuming but still reach the final barrier below.
        if (!mbar_wait(&full_bar[slot], (i / S) & 1)) break;
        const int lr = 2 * warp;  // local row of this warp's pair
        if (lr < rows && rows_m > 0) {
            const bool two = lr + 1 < rows;
            const uint8_t* dw = ring + (size_t)slot * (sw + ss);
            const __half* ds = reinterpret_cast<const __half*>(dw + sw);
            const uint4* w0p = reinterpret_cast<const uint4*>(dw + (size_t)lr * seg);
            const uint4* w1p = reinterpret_cast<const uint4*>(dw + (size_t)(two ? lr + 1 : lr) * seg);
            const __half* s0p = ds + (size_t)lr * (seg / 32);
            const __half* s1p = ds + (size_t)(two ? lr + 1 : lr) * (seg / 32);
            for (int j = 0; j < nj; j++) {
                const int kl = j * 512 + lane * 16;  // byte within the segment
                const uint4 w0 = w0p[kl >> 4];
                const uint4 w1 = w1p[kl >> 4];
                const float s0 = __half2float(s0p[kl >> 5]);
                const float s1 = __half2float(s1p[kl >> 5]);
                const int ka = (sg * seg + kl) >> 4;
#pragma unroll
                for (int m = 0; m < MMAX; m++) {
                    if (m < rows_m) {
                        const uint4 a = act4[m * K16 + ka];
                        f0[m] = __fmaf_rn(i2f_exact(dot16<true>(a, w0)), s0, f0[m]);
                        f1[m] = __fmaf_rn(i2f_exact(dot16<true>(a, w1)), s1, f1[m]);
                    }
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty_bar[slot]);

        if (sg == nseg - 1) {
            // the pair (r + lr, r + lr + 1) is complete: reduce and apply the epilogue
            const int n0 = r + lr;
            const bool active = lr < rows;
            const bool has1 = active && lr + 1 < rows;
            float y_own = 0.0f, yp0 = 0.0f, yp1 = 0.0f;
            const int m_own = lane >> 1, sel = lane & 1;
#pragma unroll
            for (int m = 0; m < MMAX; m++) {
                if (m < rows_m) {
                    const float t0 = __fdiv_rn(warp_sum(f0[m]), 127.0f);
                    const float t1 = __fdiv_rn(warp_sum(f1[m]), 127.0f);
                    if (m == m_own) y_own = sel ? t1 : t0;
                    if (m == lane) { yp0 = t0; yp1 = t1; }
                    f0[m] = f1[m] = 0.0f;
                }
            }
            if (active) {
                if (EPI == EPI_STORE || EPI == EPI_LOGITS) {
                    if (m_own < rows_m && (sel == 0 || has1))
                        p.out[(size_t)(p.row0 + m_own) * p.ldo + n0 + sel] = y_own;
                    if (EPI == EPI_LOGITS && lane < rows_m) {
                        unsigned long long k = argmax_key(yp0, n0);
                        if (has1) {
                            const unsigned long long k1 = argmax_key(yp1, n0 + 1);
                            k = k1 > k ? k1 : k;
                        }
                        best = k > best ? k : best;
                    }
                } else if (EPI == EPI_RESID) {
                    if (m_own < rows_m && (sel == 0 || has1)) {
                        float* o = p.out + (size_t)(p.row0 + m_own) * p.ldo + n0 + sel;
                        *o = __fadd_rn(*o, y_own);
                    }
                } else if (EPI == EPI_QKV) {
                    if (lane < rows_m) {
                        const int rr = p.row0 + lane;
                        float v0 = yp0, v1 = yp1;
                        const int qkd = p.q_dim + p.kv_dim;
                        if (n0 < qkd) {
                            const int ii = (n0 < p.q_dim ? n0 : n0 - p.q_dim) % p.head_dim;
                            const float freq =
                                __fdiv_rn(1.0f, powf(p.theta, __fdiv_rn((float)ii, (float)p.head_dim)));
                            const float ang = __fmul_rn((float)p.pos[rr], freq);
                            float sn, cs;
                            sincosf(ang, &sn, &cs);
                            const float a = v0, b = v1;
                            v0 = __fsub_rn(__fmul_rn(a, cs), __fmul_rn(b, sn));
                            v1 = __fadd_rn(__fmul_rn(a, sn), __fmul_rn(b, cs));
                        }
                        if (n0 < p.q_dim) {
                            p.q_out[(size_t)rr * p.q_dim + n0] = v0;
                            p.q_out[(size_t)rr * p.q_dim + n0 + 1] = v1;
                        } else {
                            const bool is_k = n0 < qkd;
                            const int c = n0 - (is_k ? p.q_dim : qkd);
                            const int h = c / p.head_dim;
                            const int dd = c - h * p.head_dim;
                            const int slotk = *p.slot_base + rr;
                            const int page = p.block_table[slotk / kPageSize];
                            const size_t off =
                                (((size_t)page * p.kv_heads + h) * kPageSize + (slotk % kPageSize)) * p.head_dim + dd;
                            *reinterpret_cast<__half2*>((is_k ? p.kv.k : p.kv.v) + off) = __floats2half2_rn(v0, v1);
                        }
                    }
                } else if (EPI == EPI_SWIGLU) {
                    if (lane < rows_m) {
                        const int rr = p.row0 + lane;
                        const float h = __fmul_rn(__fmul_rn(yp0, poly_sigmoid(yp0)), yp1);
                        p.hq[(size_t)rr * p.F + (n0 >> 1)] = (uint8_t)quant_u8(h);
                    }
                }
            }
        }
    }

    if (EPI == EPI_LOGITS) {
        if (lane < kMaxRows) red_s[warp][lane] = lane < rows_m ? best : 0ull;
        asm volatile("bar.sync 1, %0;" ::"n"(kCWarps * 32) : "memory");
        if (threadIdx.x < (unsigned)rows_m) {
            unsigned long long b = 0ull;
            for (int w = 0; w < kCWarps; w++) b = red_s[w][threadIdx.x] > b ? red_s[w][threadIdx.x] : b;
            p.amax_part[(size_t)(p.row0 + threadIdx.x) * gridDim.x + blockIdx.x] = b;
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

template <int MMAX, int EPI>
cudaError_t launch_t(const GemvParams& p, const TmaShape& sh, cudaStream_t s, bool pdl) {
    auto kern = gemv_tma_kernel<MMAX, EPI>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sh.smem);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(tma_gemv_grid());
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = sh.smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, p, sh.seg, sh.nseg, sh.stages, (int)sh.act_bytes);
}

template <int EPI>
cudaError_t launch_e(const GemvParams& p, int mmax, const TmaShape& sh, cudaStream_t s, bool pdl) {
    if (mmax <= 1) return launch_t<1, EPI>(p, sh, s, pdl);
    if (mmax <= 2) return launch_t<2, EPI>(p, sh, s, pdl);
    if (mmax <= 4) return launch_t<4, EPI>(p, sh, s, pdl);
    return launch_t<8, EPI>(p, sh, s, pdl);
}

}  // namespace

int tma_gemv_grid() { return sm_count(); }

int take_device_error() {
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_fl_error, sizeof(int)) != cudaSuccess) return -1;
    if (v) {
        const int z = 0;
        cudaMemcpyToSymbol(g_fl_error, &z, sizeof(int));
    }
    return v;
}

cudaError_t launch_gemv_auto(const GemvParams& p, int epi, cudaStream_t s, bool pdl) {
    if (epi != EPI_DOTS && tma_gemv_supported(p.K, p.M)) return launch_gemv_tma(p, epi, s, pdl);
    return launch_gemv(p, epi, false, false, s, pdl);
}

int gemv_auto_grid(int N, int K) { return tma_gemv_supported(K, kMaxRows) ? tma_gemv_grid() : gemv_grid(N); }

bool tma_gemv_supported(int K, int M) {
    TmaShape sh;
    return tma_shape(K, M, sh);
}

// p.M: rows held in shared memory (static count, or the upper bound of
// *p.dyn_M), 1..kMaxRows.
cudaError_t launch_gemv_tma(const GemvParams& p, int epi, cudaStream_t s, bool pdl) {
    if (p.M <= 0 || p.M > kMaxRows) return cudaErrorInvalidValue;
    const int mm = p.M <= 1 ? 1 : p.M <= 2 ? 2 : p.M <= 4 ? 4 : 8;
    TmaShape sh;
    if (!tma_shape(p.K, p.M, sh)) return cudaErrorInvalidValue;
    if (p.x && p.K % 128 != 0) return cudaErrorInvalidValue;
    switch (epi) {
        case EPI_STORE: return launch_e<EPI_STORE>(p, mm, sh, s, pdl);
        case EPI_RESID: return launch_e<EPI_RESID>(p, mm, sh, s, pdl);
        case EPI_QKV: return launch_e<EPI_QKV>(p, mm, sh, s, pdl);
        case EPI_SWIGLU: return launch_e<EPI_SWIGLU>(p, mm, sh, s, pdl);
        case EPI_LOGITS: return launch_e<EPI_LOGITS>(p, mm, sh, s, pdl);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace fl
