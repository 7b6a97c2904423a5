// One speculative step as ONE persistent cooperative kernel (sm_100a).
//
// A phase list (fl_step.h) describes, in order, every operation of a step:
// the k-1 single-row draft passes, the verify pass over k+1 rows, the LM
// heads, the decode attentions and the acceptance / draft-pick control
// (the same arithmetic as gemv_tma.cu, attention.cu and decode_ops.cu).
// Every CTA walks the list; phases are separated by grid-wide barriers among
// the consumer warps. The producer warp of each CTA does not take part in
// the barriers: it walks the same list and streams the weight stages of
// every GEMV phase through one shared-memory ring, so the HBM stream keeps
// running across layer and phase boundaries, attention and barriers
// included. All waits (ring mbarriers, grid barrier) are bounded: on a
// timeout the kernel records an error word, stops waiting and computing,
// still passes every barrier, and ends.
#include <float.h>

#include "fl_common.cuh"
#include "fl_layout.cuh"
#include "fl_step.h"

namespace fl {

namespace {

constexpr int kCW = 8;                    // consumer warps
constexpr int kCThreads = kCW * 32;
constexpr int kThr = kCThreads + 32;      // + producer warp
constexpr int kMaxSlots = 8;
constexpr int kSmemLimit = 216 * 1024;
constexpr unsigned long long kWaitNs = 2000000000ull;  // every wait gives up after ~2 s
constexpr int kErrRing = 1, kErrGrid = 2;

__device__ __forceinline__ unsigned long long gtime() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// ---------------------------------------------------------------- sync helpers
__device__ __forceinline__ uint32_t saddr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void cbar() { asm volatile("bar.sync 1, %0;" ::"n"(kCThreads) : "memory"); }
__device__ __forceinline__ void abar() { asm volatile("bar.sync 2, 128;" ::: "memory"); }  // warps 0-3

__device__ __forceinline__ void mb_init(uint64_t* b, uint32_t n) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(saddr(b)), "r"(n) : "memory");
}
__device__ __forceinline__ void mb_expect(uint64_t* b, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(saddr(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mb_arrive(uint64_t* b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(saddr(b)) : "memory");
}
__device__ __forceinline__ bool mb_try(uint64_t* b, uint32_t par) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(saddr(b)), "r"(par)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ bool mb_wait(uint64_t* b, uint32_t par, int* err) {
    if (mb_try(b, par)) return true;
    const unsigned long long t0 = gtime();
    while (!mb_try(b, par)) {
        if (gtime() - t0 > kWaitNs) {
            atomicOr(err, kErrRing);
            return false;
        }
    }
    return true;
}
__device__ __forceinline__ void bulk(void* dst, const void* src, uint32_t bytes, uint64_t* b) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     saddr(dst)),
                 "l"(src), "r"(bytes), "r"(saddr(b))
                 : "memory");
}

// Grid-wide barrier of the consumer threads of all CTAs (generation
// counter). A CTA that already failed a wait (bad) passes without arriving
// or waiting, so a failure ends the kernel within one wait limit per CTA.
__device__ bool grid_sync(unsigned* bar, int* err, int* ok_s, bool bad) {
    if (bad) return false;
    cbar();
    if (threadIdx.x == 0) {
        volatile unsigned* gen = bar + 1;
        const unsigned g = *gen;
        __threadfence();
        const unsigned a = atomicAdd(bar, 1u);
        int ok = 1;
        if (a == gridDim.x - 1) {
            atomicExch(bar, 0u);
            __threadfence();
            atomicAdd(bar + 1, 1u);
        } else {
            const unsigned long long t0 = gtime();
            while (*gen == g) {
                if (gtime() - t0 > kWaitNs) {
                    ok = 0;
                    atomicOr(err, kErrGrid);
                    break;
                }
                __nanosleep(32);
            }
        }
        __threadfence();
        *ok_s = ok;
    }
    cbar();
    return *ok_s != 0;
}

// ---------------------------------------------------------------- GEMV geometry
struct GGeo {
    int P, npan, R, row0, row1, ntiles, nstages;
};

__host__ __device__ inline int stage_rows(int P, int slot_bytes) {
    int R = slot_bytes / (P + P / 16);
    if (R > 16) R = 16;
    return R & ~1;
}

__host__ __device__ inline void gemv_geo(const GemvParams& g, int slot_bytes, int cta, int ncta, GGeo& o) {
    o.P = g.P;
    o.npan = g.K / g.P;
    o.R = stage_rows(g.P, slot_bytes);
    const int nunits = g.N >> 3;
    const int u0 = (int)(((long long)nunits * cta) / ncta);
    const int u1 = (int)(((long long)nunits * (cta + 1)) / ncta);
    o.row0 = u0 * 8;
    o.row1 = u1 * 8;
    o.ntiles = (o.row1 - o.row0 + o.R - 1) / o.R;
    o.nstages = o.ntiles * o.npan;
}

__device__ __forceinline__ int dot16(const uint4& a, const uint4& w) {
    int d = dp4a_us(a.x, w.x, 0);
    d = dp4a_us(a.y, w.y, d);
    d = dp4a_us(a.z, w.z, d);
    return dp4a_us(a.w, w.w, d);
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

__device__ __forceinline__ void mma_u8s8(uint32_t a0, uint32_t a2, uint32_t b0, uint32_t b1, int& d0, int& d1) {
    int c2, c3;
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%11,%12,%13};"
        : "=r"(d0), "=r"(d1), "=r"(c2), "=r"(c3)
        : "r"(a0), "r"(0), "r"(a2), "r"(0), "r"(b0), "r"(b1), "r"(0), "r"(0), "r"(0), "r"(0));
    (void)c2;
    (void)c3;
}

// Epilogue of weight-row pair (n0, n0 + 1) for activation row r (same
// arithmetic as gemv_tma.cu's pair_epilogue, epilogue chosen at run time).
__device__ void pair_epi(const GemvParams& p, int epi, int r, int n0, bool has1, float y0, float y1,
                         unsigned long long* best_s) {
    if (epi == EPI_STORE || epi == EPI_LOGITS) {
        p.out[(size_t)r * p.ldo + n0] = y0;
        if (has1) p.out[(size_t)r * p.ldo + n0 + 1] = y1;
        if (epi == EPI_LOGITS) {
            unsigned long long k = argmax_key(y0, n0);
            if (has1) {
                const unsigned long long k1 = argmax_key(y1, n0 + 1);
                k = k1 > k ? k1 : k;
            }
            atomicMax(&best_s[r - p.row0], k);
        }
    } else if (epi == EPI_RESID) {
        float* o = p.out + (size_t)r * p.ldo + n0;
        o[0] = __fadd_rn(__ldcg(o), y0);
        if (has1) o[1] = __fadd_rn(__ldcg(o + 1), y1);
    } else if (epi == EPI_QKV) {
        float v0 = y0, v1 = y1;
        const int qkd = p.q_dim + p.kv_dim;
        if (n0 < qkd) {
            const int ii = (n0 < p.q_dim ? n0 : n0 - p.q_dim) % p.head_dim;
            const float freq = __fdiv_rn(1.0f, powf(p.theta, __fdiv_rn((float)ii, (float)p.head_dim)));
            const float ang = __fmul_rn((float)__ldcg(p.pos + r), freq);
            float sn, cs;
            sincosf(ang, &sn, &cs);
            v0 = __fsub_rn(__fmul_rn(y0, cs), __fmul_rn(y1, sn));
            v1 = __fadd_rn(__fmul_rn(y0, sn), __fmul_rn(y1, cs));
        }
        if (n0 < p.q_dim) {
            p.q_out[(size_t)r * p.q_dim + n0] = v0;
            p.q_out[(size_t)r * p.q_dim + n0 + 1] = v1;
        } else {
            const bool is_k = n0 < qkd;
            const int c = n0 - (is_k ? p.q_dim : qkd);
            const int h = c / p.head_dim;
            const int dd = c - h * p.head_dim;
            const int slot = __ldcg(p.slot_base) + r;
            const int page = p.block_table[slot / kPageSize];
            const size_t off = (((size_t)page * p.kv_heads + h) * kPageSize + (slot % kPageSize)) * p.head_dim + dd;
            *reinterpret_cast<__half2*>((is_k ? p.kv.k : p.kv.v) + off) = __floats2half2_rn(v0, v1);
        }
    } else if (epi == EPI_SWIGLU) {
        const float h = __fmul_rn(__fmul_rn(y0, poly_sigmoid(y0)), y1);
        p.hq[(size_t)r * p.F + (n0 >> 1)] = (uint8_t)quant_u8(h);
    }
}

struct Ring {
    uint8_t* base;
    uint64_t* full;
    uint64_t* empty;
    int S, slot;
};

// Consumer side of one GEMV phase. `s` is the global stage counter.
__device__ void gemv_phase(const GemvParams& p, int epi, bool skip, const Ring& rg, int& s, bool& bad, int* err,
                           uint8_t* act, unsigned long long* best_s, float (*red)[kCW][32][4]) {
    GGeo geo;
    gemv_geo(p, rg.slot, blockIdx.x, gridDim.x, geo);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int rows_m = p.M;
    if (p.dyn_M) rows_m = min(__ldcg(p.dyn_M) - p.row0, p.M);
    rows_m = max(0, min(rows_m, kMaxRows));
    if (skip || rows_m == 0) {
        // keep the ring in step with the producer without computing
        for (int i = 0; i < geo.nstages; i++, s++) {
            if (!bad && !mb_wait(&rg.full[s % rg.S], (s / rg.S) & 1, err)) bad = true;
            __syncwarp();
            if (lane == 0) mb_arrive(&rg.empty[s % rg.S]);
        }
        return;
    }
    const int K = p.K, P = geo.P, R = geo.R, npan = geo.npan;
    const int ald = K + 16;
    if (threadIdx.x < kMaxRows) best_s[threadIdx.x] = 0ull;
    if (p.x) {
        const int src0 = p.x_row_dyn ? __ldcg(p.x_row_dyn) : p.row0;
        for (int m = warp; m < rows_m; m += kCW)
            act_prologue(act + (size_t)m * ald, p.x + (size_t)(src0 + m) * K, K, 1, p.norm, p.eps, 0, lane, 1);
    } else {
        const int K16 = K >> 4;
        const uint4* src = reinterpret_cast<const uint4*>(p.aq + (size_t)p.row0 * K);
        for (int i = threadIdx.x; i < rows_m * K16; i += kCThreads) {
            const int m = i / K16, c = i - m * K16;
            *reinterpret_cast<uint4*>(act + (size_t)m * ald + (size_t)c * 16) = __ldcg(src + (size_t)m * K16 + c);
        }
    }
    cbar();
    const int bpp = P >> 5;
    if (rows_m == 1) {
        // dp4a: warp = row pair (2w, 2w + 1) of the stage
        float f0 = 0.0f, f1 = 0.0f;
        const int lr = 2 * warp;
        const int cpp = P >> 4;
        for (int i = 0; i < geo.nstages; i++, s++) {
            const int sl = s % rg.S;
            const int tile = i / npan, pan = i - tile * npan;
            const int r = geo.row0 + tile * R;
            const int rows = min(R, geo.row1 - r);
            if (!bad && !mb_wait(&rg.full[sl], (s / rg.S) & 1, err)) bad = true;
            if (!bad && lr < rows) {
                const uint8_t* dw = rg.base + (size_t)sl * rg.slot;
                const __half* ds = reinterpret_cast<const __half*>(dw + (size_t)R * P);
                const int ra = lr, rb = (lr + 1 < rows) ? lr + 1 : lr;
                const uint8_t* wa = dw + (size_t)ra * P;
                const uint8_t* wb = dw + (size_t)rb * P;
                for (int c = lane; c < cpp; c += 32) {
                    const uint4 w0 = *reinterpret_cast<const uint4*>(wa + swz_chunk(c, r + ra) * 16);
                    const uint4 w1 = *reinterpret_cast<const uint4*>(wb + swz_chunk(c, r + rb) * 16);
                    const float s0 = __half2float(ds[ra * bpp + (c >> 1)]);
                    const float s1 = __half2float(ds[rb * bpp + (c >> 1)]);
                    const uint4 a = *reinterpret_cast<const uint4*>(act + (size_t)pan * P + (size_t)c * 16);
                    f0 = __fmaf_rn(i2f_exact(dot16(a, w0)), s0, f0);
                    f1 = __fmaf_rn(i2f_exact(dot16(a, w1)), s1, f1);
                }
            }
            __syncwarp();
            if (lane == 0) mb_arrive(&rg.empty[sl]);
            if (pan == npan - 1) {
                const float t0 = __fdiv_rn(warp_sum(f0), 127.0f);
                const float t1 = __fdiv_rn(warp_sum(f1), 127.0f);
                f0 = f1 = 0.0f;
                if (!bad && lane == 0 && lr < rows) pair_epi(p, epi, p.row0, r + lr, lr + 1 < rows, t0, t1, best_s);
            }
        }
    } else {
        // MMA: warp = a slice of the stage's blocks, all rows of the stage
        const int g = lane >> 2, t = lane & 3;
        const int kb0 = (warp * bpp) / kCW, kb1 = ((warp + 1) * bpp) / kCW;
        float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        int buf = 0;
        const int lj = lane >> 3, lq = lane & 7;
        const bool arow = g < rows_m;
        for (int i = 0; i < geo.nstages; i++, s++) {
            const int sl = s % rg.S;
            const int tile = i / npan, pan = i - tile * npan;
            const int r = geo.row0 + tile * R;
            const int rows = min(R, geo.row1 - r);
            if (!bad && !mb_wait(&rg.full[sl], (s / rg.S) & 1, err)) bad = true;
            const uint8_t* dw = rg.base + (size_t)sl * rg.slot;
            const __half* ds = reinterpret_cast<const __half*>(dw + (size_t)R * P);
            // rows past the stage read its last row (in-bounds, results ignored)
            const int lrow = min(lq + 8 * (lj >> 1), rows - 1);
            const uint32_t wrow = saddr(dw + (size_t)lrow * P);
            const uint8_t* arow_p = act + (size_t)g * ald + (size_t)pan * P;
            const int sr0 = min(2 * t, rows - 1), sr1 = min(2 * t + 1, rows - 1);
            const int sr2 = min(8 + 2 * t, rows - 1), sr3 = min(9 + 2 * t, rows - 1);
            for (int kb = kb0; kb < (bad ? kb0 : kb1); kb++) {
                uint32_t b00, b01, b10, b11;
                ldsm_x4(wrow + swz_chunk(2 * kb + (lj & 1), r + lrow) * 16, b00, b01, b10, b11);
                uint32_t a0 = 0, a2 = 0;
                if (arow) {
                    a0 = *reinterpret_cast<const uint32_t*>(arow_p + kb * 32 + 4 * t);
                    a2 = *reinterpret_cast<const uint32_t*>(arow_p + kb * 32 + 16 + 4 * t);
                }
                int d0, d1, d2, d3;
                mma_u8s8(a0, a2, b00, b01, d0, d1);
                mma_u8s8(a0, a2, b10, b11, d2, d3);
                acc[0] = __fmaf_rn(i2f_exact(d0), __half2float(ds[sr0 * bpp + kb]), acc[0]);
                acc[1] = __fmaf_rn(i2f_exact(d1), __half2float(ds[sr1 * bpp + kb]), acc[1]);
                acc[2] = __fmaf_rn(i2f_exact(d2), __half2float(ds[sr2 * bpp + kb]), acc[2]);
                acc[3] = __fmaf_rn(i2f_exact(d3), __half2float(ds[sr3 * bpp + kb]), acc[3]);
            }
            __syncwarp();
            if (lane == 0) mb_arrive(&rg.empty[sl]);
            if (pan == npan - 1) {
#pragma unroll
                for (int q = 0; q < 4; q++) red[buf][warp][lane][q] = acc[q];
                acc[0] = acc[1] = acc[2] = acc[3] = 0.0f;
                cbar();
                if (threadIdx.x < 64 && !bad) {
                    const int pr = threadIdx.x & 7, m = threadIdx.x >> 3;
                    if (m < rows_m && 2 * pr < rows) {
                        const int src_lane = 4 * m + (pr & 3);
                        const int q0 = (pr >> 2) * 2;
                        float y0 = 0.0f, y1 = 0.0f;
#pragma unroll
                        for (int w = 0; w < kCW; w++) {
                            y0 += red[buf][w][src_lane][q0];
                            y1 += red[buf][w][src_lane][q0 + 1];
                        }
                        pair_epi(p, epi, p.row0 + m, r + 2 * pr, 2 * pr + 1 < rows, __fdiv_rn(y0, 127.0f),
                                 __fdiv_rn(y1, 127.0f), best_s);
                    }
                }
                buf ^= 1;
            }
        }
    }
    if (epi == EPI_LOGITS) {
        cbar();
        if (threadIdx.x < (unsigned)rows_m)
            p.amax_part[(size_t)(p.row0 + threadIdx.x) * gridDim.x + blockIdx.x] = best_s[threadIdx.x];
    }
}

// ---------------------------------------------------------------- attention
constexpr int kSplit = 64;   // keys per unit (one KV page)
constexpr int kHdMax = 128;

struct AttnSmem {
    float q[kMaxRows][kHdMax];
    uint32_t K[kSplit][kHdMax / 2 + 1];
    uint32_t V[kSplit][kHdMax / 2];
    float sc[kMaxRows][kSplit];
    float ml[kMaxRows][2];
    int ticket;
};

// One (head, page) unit of split-K decode attention, warps 0-3. Same rule
// as attention.cu's attention_split_kernel (inference.c:193-247).
__device__ void attn_unit(const AttnParams& p, int h, int sp, int nsplit_max, AttnSmem& sm) {
    const int tid = threadIdx.x;  // 0..127
    const int warp = tid >> 5, lane = tid & 31;
    const int M = p.dyn_M ? __ldcg(p.dyn_M) : p.M;
    const int nr = min(M, kMaxRows);
    const int base = __ldcg(p.slot_base);
    const int ctx = base + M;
    const int nsplit = (ctx + kSplit - 1) / kSplit;
    if (sp >= nsplit || nr <= 0) return;  // uniform over warps 0-3
    const int hd = p.head_dim, hd2 = hd >> 1;
    const int kvh = h / (p.heads / p.kv_heads);
    const int qd = p.heads * hd;
    const int j0 = sp * kSplit;
    const int nt = min(kSplit, ctx - j0);
    for (int i = tid; i < nr * hd; i += 128) {
        const int rr = i / hd, dd = i - rr * hd;
        sm.q[rr][dd] = __ldcg(p.q + (size_t)rr * qd + (size_t)h * hd + dd);
    }
    {
        const int page = p.block_table[sp];
        const size_t off = (((size_t)page * p.kv_heads + kvh) * kPageSize) * hd2;
        const uint32_t* kg = reinterpret_cast<const uint32_t*>(p.kv.k) + off;
        const uint32_t* vg = reinterpret_cast<const uint32_t*>(p.kv.v) + off;
        for (int i = tid; i < nt * hd2; i += 128) {
            const int key = i / hd2, c = i - key * hd2;
            sm.K[key][c] = __ldcg(kg + i);
            sm.V[key][c] = __ldcg(vg + i);
        }
    }
    abar();
    const float scale = __fdiv_rn(1.0f, sqrtf((float)hd));
    {
        const int key = lane + 32 * (warp & 1);
        const int rb = warp >> 1;
        float acc[kMaxRows / 2];
#pragma unroll
        for (int i = 0; i < kMaxRows / 2; i++) acc[i] = 0.0f;
        if (key < nt) {
            for (int e = 0; e < hd2; e++) {
                const float2 kf = __half22float2(*reinterpret_cast<const __half2*>(&sm.K[key][e]));
#pragma unroll
                for (int i = 0; i < kMaxRows / 2; i++) {
                    const int rr = rb + 2 * i;
                    if (rr < nr) {
                        const float2 qf = *reinterpret_cast<const float2*>(&sm.q[rr][2 * e]);
                        acc[i] = __fmaf_rn(qf.x, kf.x, acc[i]);
                        acc[i] = __fmaf_rn(qf.y, kf.y, acc[i]);
                    }
                }
            }
        }
        const int j = j0 + key;
#pragma unroll
        for (int i = 0; i < kMaxRows / 2; i++) {
            const int rr = rb + 2 * i;
            if (rr < nr) {
                bool vis = key < nt;
                if (vis && j >= base) {
                    const int jj = j - base;
                    vis = p.mask ? (p.mask[(size_t)rr * M + jj] != 0) : (jj <= rr);
                }
                sm.sc[rr][key] = vis ? __fmul_rn(acc[i], scale) : -INFINITY;
            }
        }
    }
    abar();
    for (int rr = warp; rr < nr; rr += 4) {
        const float s0 = sm.sc[rr][lane], s1 = sm.sc[rr][lane + 32];
        const float mx = warp_max(fmaxf(s0, s1));
        float e0 = 0.0f, e1 = 0.0f;
        if (mx != -INFINITY) {
            e0 = s0 == -INFINITY ? 0.0f : expf(__fsub_rn(s0, mx));
            e1 = s1 == -INFINITY ? 0.0f : expf(__fsub_rn(s1, mx));
        }
        sm.sc[rr][lane] = e0;
        sm.sc[rr][lane + 32] = e1;
        const float sum = warp_sum(e0 + e1);
        if (lane == 0) {
            sm.ml[rr][0] = mx;
            sm.ml[rr][1] = sum;
        }
    }
    abar();
    const int pstride = hd + 2;
    float* part = p.part + (((size_t)h * nsplit_max + sp) * kMaxRows) * pstride;
    if (tid < 2 * hd2) {
        const int d2 = tid % hd2, rb = tid / hd2;
        float a0[kMaxRows / 2], a1[kMaxRows / 2];
#pragma unroll
        for (int i = 0; i < kMaxRows / 2; i++) a0[i] = a1[i] = 0.0f;
        for (int tt = 0; tt < nt; tt++) {
            const float2 v = __half22float2(*reinterpret_cast<const __half2*>(&sm.V[tt][d2]));
#pragma unroll
            for (int i = 0; i < kMaxRows / 2; i++) {
                const int rr = rb + 2 * i;
                if (rr < nr) {
                    const float w = sm.sc[rr][tt];
                    a0[i] = __fmaf_rn(w, v.x, a0[i]);
                    a1[i] = __fmaf_rn(w, v.y, a1[i]);
                }
            }
        }
#pragma unroll
        for (int i = 0; i < kMaxRows / 2; i++) {
            const int rr = rb + 2 * i;
            if (rr < nr) {
                part[(size_t)rr * pstride + 2 + 2 * d2] = a0[i];
                part[(size_t)rr * pstride + 3 + 2 * d2] = a1[i];
            }
        }
    }
    if (tid < nr) {
        part[(size_t)tid * pstride] = sm.ml[tid][0];
        part[(size_t)tid * pstride + 1] = sm.ml[tid][1];
    }
    __threadfence();
    abar();
    if (tid == 0) sm.ticket = atomicAdd(&p.counters[h], 1);
    abar();
    if (sm.ticket != nsplit - 1) return;
    __threadfence();
    const float* ph = p.part + ((size_t)h * nsplit_max * kMaxRows) * pstride;
    for (int i = tid; i < nr * hd; i += 128) {
        const int rr = i / hd, dd = i - rr * hd;
        float gm = -INFINITY;
        for (int s2 = 0; s2 < nsplit; s2++) gm = fmaxf(gm, __ldcg(ph + ((size_t)s2 * kMaxRows + rr) * pstride));
        float L = 0.0f, O = 0.0f;
        for (int s2 = 0; s2 < nsplit; s2++) {
            const float* q = ph + ((size_t)s2 * kMaxRows + rr) * pstride;
            const float m = __ldcg(q);
            if (m == -INFINITY) continue;
            const float wgt = expf(__fsub_rn(m, gm));
            L = __fmaf_rn(__ldcg(q + 1), wgt, L);
            O = __fmaf_rn(__ldcg(q + 2 + dd), wgt, O);
        }
        const float o = __fdiv_rn(O, L);
        const size_t idx = (size_t)rr * qd + (size_t)h * hd + dd;
        p.out_q[idx] = (uint8_t)quant_u8(o);
        if (p.out_f) p.out_f[idx] = o;
    }
    if (tid == 0) p.counters[h] = 0;
}

// ---------------------------------------------------------------- control (CTA 0, 256 threads)
__device__ unsigned long long best_of(const unsigned long long* part, int n, unsigned long long* red8) {
    unsigned long long b = 0ull;
    for (int i = threadIdx.x; i < n; i += kCThreads) {
        const unsigned long long k = __ldcg(part + i);
        b = k > b ? k : b;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long k = __shfl_xor_sync(0xffffffffu, b, o);
        b = k > b ? k : b;
    }
    if ((threadIdx.x & 31) == 0) red8[threadIdx.x >> 5] = b;
    cbar();
    b = 0ull;
    for (int w = 0; w < kCW; w++) b = red8[w] > b ? red8[w] : b;
    cbar();
    return b;
}

__device__ void control(int kind, int arg, const StepBuffers& b, int K, unsigned long long* red8, int* tgt) {
    SpecState* st = b.st;
    const int d = b.d;
    if (kind == PH_DRAFT_PICK) {
        const int j = arg;
        const int tok = argmax_key_index(best_of(b.amax_part, b.nparts, red8));
        const int n = __ldcg(&st->n);
        if (j + 1 < K) {
            const int g_row = (j == 0) ? __ldcg(&st->last_row) : 0;
            const float* g = b.x_d + (size_t)g_row * d;
            const float* e = b.embed + (size_t)tok * d;
            for (int i = threadIdx.x; i < d; i += kCThreads) b.x_d[i] = __fadd_rn(__ldcg(g + i), e[i]);
        }
        cbar();
        if (threadIdx.x == 0) {
            st->drafted[j] = tok;
            if (j + 1 < K) {
                st->draft_base = n + j + 1;
                st->draft_pos[0] = n + j + 1;
            }
        }
    } else if (kind == PH_VERIFY_PREP) {
        const int n = __ldcg(&st->n);
        for (int r = 0; r <= K; r++) {
            const int tok = r == 0 ? __ldcg(b.seq + n) : __ldcg(&st->drafted[r - 1]);
            const float* e = b.embed + (size_t)tok * d;
            for (int i = threadIdx.x; i < d; i += kCThreads) b.x_v[(size_t)r * d + i] = e[i];
        }
        if (threadIdx.x <= K) st->verify_pos[threadIdx.x] = n + threadIdx.x;
        if (threadIdx.x == 0) st->verify_base = n;
    } else if (kind == PH_ACCEPT) {
        for (int r = 0; r <= K; r++) {
            const unsigned long long bk = best_of(b.amax_part + (size_t)r * b.nparts, b.nparts, red8);
            if (threadIdx.x == 0) tgt[r] = argmax_key_index(bk);
        }
        cbar();
        if (threadIdx.x == 0) {
            volatile SpecState* vs = st;  // written earlier in this launch: bypass L1
            const int n = vs->n;
            int a = 0;
            while (a < K && a < vs->max_acc && vs->drafted[a] == tgt[a]) a++;
            for (int r = 0; r <= K; r++) st->target[r] = tgt[r];
            int produced = vs->produced;
            const int n_new = vs->n_new;
            for (int j = 0; j <= a; j++) {
                const int t = j < a ? vs->drafted[j] : tgt[a];
                b.seq[n + 1 + j] = t;
                if (produced < n_new) b.out[produced++] = t;
            }
            const int steps = vs->steps;
            b.acc_hist[steps] = a;
            st->steps = steps + 1;
            st->produced = produced;
            st->a_last = a;
            st->n = n + a + 1;
            st->rows = a + 1;
            st->last_row = a;
            st->draft_base = n + 1;
            for (int r = 0; r <= a; r++) st->draft_pos[r] = n + 1 + r;
            st->done = produced >= n_new ? 1 : 0;
        }
    } else if (kind == PH_CATCHUP_PREP) {
        const int rows = __ldcg(&st->rows);
        const int base = __ldcg(&st->draft_base);
        for (int r = 0; r < rows; r++) {
            const int tok = __ldcg(b.seq + base + r);
            const float* e = b.embed + (size_t)tok * d;
            for (int i = threadIdx.x; i < d; i += kCThreads)
                b.x_d[(size_t)r * d + i] = __fadd_rn(__ldcg(b.x_v + (size_t)r * d + i), e[i]);
        }
    }
}

// ---------------------------------------------------------------- the kernel
__global__ void __launch_bounds__(kThr, 1) step_kernel(const StepParams p, int* err) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ __align__(8) uint64_t full[kMaxSlots];
    __shared__ __align__(8) uint64_t empty[kMaxSlots];
    __shared__ unsigned long long best_s[kMaxRows];
    __shared__ unsigned long long red8[kCW];
    __shared__ float red[2][kCW][32][4];
    __shared__ int tgt[kMaxRows];
    __shared__ int ok_s, skip_s;

    if (__ldcg(p.done)) return;  // whole step already finished: uniform early exit
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    Ring rg;
    rg.base = smem + p.region_bytes;
    rg.full = full;
    rg.empty = empty;
    rg.S = p.S;
    rg.slot = p.slot_bytes;
    if (threadIdx.x == 0) {
        for (int i = 0; i < p.S; i++) {
            mb_init(&full[i], 1);
            mb_init(&empty[i], kCW);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    if (warp == kCW) {
        // ---------------- producer: every GEMV phase's stages, in order ----------------
        if (lane != 0) return;
        int s = 0;
        for (int ph = 0; ph < p.nphases; ph++) {
            const Phase* P = p.phases + ph;
            if (P->kind != PH_GEMV) continue;
            GGeo geo;
            gemv_geo(P->g, p.slot_bytes, blockIdx.x, gridDim.x, geo);
            const int N = P->g.N;
            const uint8_t* sb = reinterpret_cast<const uint8_t*>(P->g.sblk);
            for (int i = 0; i < geo.nstages; i++, s++) {
                const int sl = s % p.S;
                if (s >= p.S && !mb_wait(&empty[sl], ((s / p.S) - 1) & 1, err)) return;
                const int tile = i / geo.npan, pan = i - tile * geo.npan;
                const int r = geo.row0 + tile * geo.R;
                const int rows = min(geo.R, geo.row1 - r);
                uint8_t* dw = rg.base + (size_t)sl * p.slot_bytes;
                uint8_t* ds = dw + (size_t)geo.R * geo.P;
                mb_expect(&full[sl], (uint32_t)(rows * geo.P + rows * (geo.P / 16)));
                bulk(dw, P->g.w + ((size_t)pan * N + r) * geo.P, (uint32_t)(rows * geo.P), &full[sl]);
                bulk(ds, sb + ((size_t)pan * N + r) * (geo.P / 16), (uint32_t)(rows * (geo.P / 16)), &full[sl]);
            }
        }
        return;
    }

    // ---------------- consumers ----------------
    int s = 0;
    bool bad = false, skip = false;
    for (int ph = 0; ph < p.nphases; ph++) {
        const Phase& P = p.phases[ph];
        const int kind = P.kind;
        if (kind == PH_GEMV) {
            gemv_phase(P.g, P.epi, skip || bad, rg, s, bad, err, smem, best_s, red);
        } else if (kind == PH_ATTN) {
            if (!skip && !bad && warp < 4) {
                const AttnParams& a = P.a;
                const int nsm = (a.max_ctx + kSplit - 1) / kSplit;
                const int units = a.heads * nsm;
                for (int u = blockIdx.x; u < units; u += gridDim.x)
                    attn_unit(a, u / nsm, u % nsm, nsm, *reinterpret_cast<AttnSmem*>(smem));
            }
        } else if (!skip && !bad && blockIdx.x == 0) {
            control(kind, P.arg, p.sb, p.K, red8, tgt);
        }
        if (ph + 1 < p.nphases) {
            if (!grid_sync(p.bar, err, &ok_s, bad)) bad = true;
            if (threadIdx.x == 0) skip_s = __ldcg(p.done);
            cbar();
            skip = skip_s != 0;
        }
    }
}

int g_sms[16] = {0};

}  // namespace

int step_grid() {
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 16 && g_sms[dev]) return g_sms[dev];
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (dev < 16) g_sms[dev] = n;
    return n;
}

bool step_plan(const Phase* ph, int n, StepParams& sp, size_t* smem_bytes) {
    int region = (int)sizeof(AttnSmem);
    int pmax = 0;
    for (int i = 0; i < n; i++) {
        if (ph[i].kind != PH_GEMV) continue;
        const GemvParams& g = ph[i].g;
        if (g.P == 0 || g.N % 8 || g.K % g.P || g.M < 1 || g.M > kMaxRows) return false;
        region = region > g.M * (g.K + 16) ? region : g.M * (g.K + 16);
        pmax = pmax > g.P ? pmax : g.P;
    }
    region = (region + 127) & ~127;
    const int avail = kSmemLimit - region;
    // choose the slot count that keeps the most bytes in flight (>= 2 slots,
    // and a stage of at least 2 rows of the widest panel)
    int best_s = 0, best_slot = 0;
    long best_inflight = -1;
    for (int S = 2; S <= kMaxSlots; S++) {
        int slot = (avail / S) & ~127;
        if (stage_rows(pmax ? pmax : 128, slot) < 2) break;
        long used = 0;
        for (int i = 0; i < n; i++) {
            if (ph[i].kind != PH_GEMV) continue;
            const int R = stage_rows(ph[i].g.P, slot);
            const long u = (long)S * R * (ph[i].g.P + ph[i].g.P / 16);
            used = used == 0 ? u : (u < used ? u : used);  // worst phase decides
        }
        if (used > best_inflight) {
            best_inflight = used;
            best_s = S;
            best_slot = slot;
        }
    }
    if (!best_s) return false;
    sp.region_bytes = region;
    sp.S = best_s;
    sp.slot_bytes = best_slot;
    *smem_bytes = (size_t)region + (size_t)best_s * best_slot;
    return true;
}

cudaError_t launch_step(const StepParams& p, size_t smem, cudaStream_t s) {
    cudaError_t e = cudaFuncSetAttribute(step_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    int* err = reinterpret_cast<int*>(p.bar + 2);  // bar: [arrivals, generation, error word]
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(step_grid());
    cfg.blockDim = dim3(kThr);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, step_kernel, p, err);
}

}  // namespace fl
