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
// included. In a GEMV phase each consumer warp owns 16 weight rows of the
// stage tile and runs mma.sync u8 x s8 -> s32 per 32-element block over
// them for all activation rows, scaling and adding the blocks in order
// (matmul_dequantized's order, bit-exact with the oracle), then applies the
// layer epilogue to its own rows: no cross-warp reduction, no CTA barrier
// inside a phase. All waits (ring mbarriers, grid barrier) are bounded: on
// a timeout the kernel records an error word, stops waiting and computing,
// still passes every barrier, and ends.
#include <float.h>

#include "fl_common.cuh"
#include "fl_layout.cuh"
#include "fl_step.h"

namespace fl {

namespace {

constexpr int kCW = 8;                    // consumer warps (phase work, barriers)
constexpr int kCThreads = kCW * 32;
constexpr int kProdWarp = kCW;            // TMA producer
constexpr int kThr = (kCW + 1) * 32;
constexpr int kMaxSlots = 12;
constexpr int kSmemLimit = 222 * 1024;    // + static shared memory <= 227 KB
constexpr unsigned long long kWaitNs = 2000000000ull;  // every wait gives up after ~2 s
constexpr int kErrRing = 1, kErrGrid = 2;
constexpr int kTr = 6;  // trace words per phase (fl_step.h)

__device__ __forceinline__ unsigned long long gtime() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// ---------------------------------------------------------------- sync helpers
__device__ __forceinline__ uint32_t saddr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void cbar() { asm volatile("bar.sync 1, %0;" ::"n"(kCThreads) : "memory"); }
// Consumer barrier that also ORs a flag over the consumer threads.
__device__ __forceinline__ bool cbar_or(bool v) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\tbar.red.or.pred q, 1, %2, p;\n\tselp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)v), "n"(kCThreads)
        : "memory");
    return r != 0;
}

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
// Polls in rounds of 64 tries; the clock (a slow read) only between rounds.
__device__ __forceinline__ bool mb_wait(uint64_t* b, uint32_t par, int* err) {
    unsigned long long t0 = 0;
    for (;;) {
        for (int i = 0; i < 64; i++)
            if (mb_try(b, par)) return true;
        const unsigned long long t = gtime();
        if (t0 == 0) t0 = t;
        else if (t - t0 > kWaitNs) {
            atomicOr(err, kErrRing);
            return false;
        }
    }
}
__device__ __forceinline__ void bulk(void* dst, const void* src, uint32_t bytes, uint64_t* b) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     saddr(dst)),
                 "l"(src), "r"(bytes), "r"(saddr(b))
                 : "memory");
}

// Grid-wide barrier of the consumer threads of all CTAs: a 64-bit arrival
// counter, zeroed before every launch, that only grows. Barrier b of a
// launch is open once the counter reaches (b + 1) * grid: each CTA adds 1
// with release semantics (no return value to wait for) and polls with
// acquire loads. `bad` is first made uniform over the CTA's consumer warps;
// a CTA that failed a wait passes without arriving or waiting, so a failure
// ends the kernel within one wait limit per CTA (the host zeroes the
// counter again after an error).
__device__ __forceinline__ unsigned long long ld_acquire(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__device__ bool grid_sync(unsigned long long* ctr, unsigned long long target, int* err, int* ok_s, bool bad,
                          unsigned long long* tr) {
    if (cbar_or(bad)) return false;
    if (threadIdx.x == 0) {
        if (tr) {
            const unsigned long long t = gtime();
            if (blockIdx.x == 0) tr[1] = t;
            atomicMax(tr + 2, t);
        }
        asm volatile("red.release.gpu.global.add.u64 [%0], 1;" ::"l"(ctr) : "memory");
        int ok = 1;
        if (ld_acquire(ctr) < target) {
            const unsigned long long t0 = gtime();
            for (bool open = false; !open;) {
                for (int i = 0; i < 16 && !open; i++) open = ld_acquire(ctr) >= target;
                if (!open && gtime() - t0 > kWaitNs) {
                    ok = 0;
                    atomicOr(err, kErrGrid);
                    break;
                }
            }
        }
        *ok_s = ok;
    }
    cbar();
    return *ok_s != 0;
}

// ---------------------------------------------------------------- GEMV geometry
// Weights are in the tiled layout with 128-byte panels (fl_layout.cuh): a
// panel's rows are 128 contiguous bytes whose 16-byte chunks are XORed with
// (row & 7), so the eight rows of an ldmatrix read hit eight different bank
// groups. A ring stage is a tile of kTileRows weight rows x kPPS panels plus
// their fp16 block scales; consumer warp w takes tile rows 16w .. 16w + 15.
constexpr int kP = 128;                         // panel bytes per row
constexpr int kPPS = 2;                         // panels per stage
constexpr int kTileRows = 128;                  // 8 warps x 16 rows
constexpr int kKBS = kPPS * kP / 32;            // 32-element blocks per stage
constexpr int kSlot = kPPS * (kTileRows * kP + kTileRows * (kP / 16));  // 34 KB
static_assert(kSlot % 1024 == 0, "stage slots keep 1024-byte alignment");
static_assert(kTileRows == 16 * kCW, "one 16-row group per consumer warp");

struct GGeo {
    int nps, row0, row1, ntiles, nstages;  // nps: stages per tile
    int W;   // panels per stage
    int rs;  // row spacing of a panel in a slot: tile rows rounded up to 16
};

// A CTA's rows are a contiguous run of 8-row units; tiles of up to kTileRows
// rows. A stage holds W whole panels of the tile, W the widest divisor of
// K / kP with W * rs <= kTileRows * kPPS, so a narrow CTA share still moves
// about a slot's worth of bytes per stage.
__host__ __device__ inline void gemv_geo(const GemvParams& g, int cta, int ncta, GGeo& o) {
    const int nunits = g.N >> 3;
    const int u0 = (int)(((long long)nunits * cta) / ncta);
    const int u1 = (int)(((long long)nunits * (cta + 1)) / ncta);
    o.row0 = u0 * 8;
    o.row1 = u1 * 8;
    const int R = o.row1 - o.row0;
    const int tr = R < kTileRows ? R : kTileRows;
    o.rs = tr <= 16 ? 16 : (tr + 15) & ~15;
    const int npan = g.K / kP;
    o.W = kPPS;
    for (int w = (kTileRows * kPPS) / o.rs; w > kPPS; w--)
        if (npan % w == 0) {
            o.W = w;
            break;
        }
    o.nps = npan / o.W;
    o.ntiles = (R + kTileRows - 1) / kTileRows;
    o.nstages = o.ntiles * o.nps;
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

// D(16x8, s32) = A(16x32, u8, row) x B(32x8, s8, col); A rows 8-15 are zero,
// so only the first two accumulator registers carry results.
__device__ __forceinline__ void mma_u8s8(uint32_t a0, uint32_t a2, uint32_t b0, uint32_t b1, int& d0, int& d1) {
    int c2, c3;
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%11,%12,%13};"
        : "=r"(d0), "=r"(d1), "=r"(c2), "=r"(c3)
        : "r"(a0), "r"(0), "r"(a2), "r"(0), "r"(b0), "r"(b1), "r"(0), "r"(0), "r"(0), "r"(0));
    (void)c2;
    (void)c3;
}

// warp-uniform bounded wait: lane 0 waits, the result is broadcast
__device__ __forceinline__ bool warp_wait(uint64_t* b, uint32_t par, int* err) {
    bool ok = true;
    if ((threadIdx.x & 31) == 0) ok = mb_wait(b, par, err);
    return __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
}

// Per-phase epilogue inputs staged in shared memory at the start of a GEMV
// phase (so no epilogue waits on a global load): RoPE positions, KV page
// and in-page slot per activation row, the RoPE inverse frequencies, and
// the residual slice [rows_m, nr] of the CTA's output rows.
constexpr int kResFloats = 512;
struct EpiSmem {
    int pos[kMaxRows];
    int page[kMaxRows];
    int off[kMaxRows];
    float freq[64];
    float res[kResFloats];
};

// Epilogue of weight-row pair (n0, n0 + 1) for activation row r = p.row0 + m
// (same arithmetic as gemv_tma.cu's pair_epilogue, chosen at run time).
// rbase / nr: first output row and row count of this CTA (residual slice).
__device__ void pair_epi(const GemvParams& p, int epi, int m, int n0, bool has1, float y0, float y1,
                         unsigned long long* best_s, const EpiSmem& es, int rbase, int nr) {
    const int r = p.row0 + m;
    if (epi == EPI_STORE || epi == EPI_LOGITS) {
        p.out[(size_t)r * p.ldo + n0] = y0;
        if (has1) p.out[(size_t)r * p.ldo + n0 + 1] = y1;
        if (epi == EPI_LOGITS) {
            unsigned long long k = argmax_key(y0, n0);
            if (has1) {
                const unsigned long long k1 = argmax_key(y1, n0 + 1);
                k = k1 > k ? k1 : k;
            }
            atomicMax(&best_s[m], k);
        }
    } else if (epi == EPI_RESID) {
        float* o = p.out + (size_t)r * p.ldo + n0;
        const float* res = es.res + m * nr + (n0 - rbase);
        o[0] = __fadd_rn(res[0], y0);
        if (has1) o[1] = __fadd_rn(res[1], y1);
    } else if (epi == EPI_QKV) {
        float v0 = y0, v1 = y1;
        const int qkd = p.q_dim + p.kv_dim;
        if (n0 < qkd) {
            const int ii = (n0 < p.q_dim ? n0 : n0 - p.q_dim) % p.head_dim;
            const float ang = __fmul_rn((float)es.pos[m], es.freq[ii >> 1]);
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
            const size_t off = (((size_t)es.page[m] * p.kv_heads + h) * kPageSize + es.off[m]) * p.head_dim + dd;
            *reinterpret_cast<__half2*>((is_k ? p.kv.k : p.kv.v) + off) = __floats2half2_rn(v0, v1);
        }
    } else if (epi == EPI_SWIGLU) {
        const float h = __fmul_rn(__fmul_rn(y0, poly_sigmoid(y0)), y1);
        p.hq[(size_t)r * p.F + (n0 >> 1)] = (uint8_t)quant_u8(h);
    }
}

struct Ring {
    uint8_t* base;
    uint64_t* full;    // TMA bytes landed
    uint64_t* empty;   // slot free (all consumer warps)
    int S, slot;
};

// The activation prologue out of line: its batched loads want registers
// that the GEMV loops around it do not need at the same time.
#ifndef FL_STEP_PROLOGUE_CACHE
#define FL_STEP_PROLOGUE_CACHE 1
#endif
__device__ __noinline__ void step_prologue(uint8_t* act, int ald, const float* x, int K, int rows, int norm, float eps,
                                           float* red, int tid) {
    act_prologue_rows<kCThreads, kMaxRows, FL_STEP_PROLOGUE_CACHE != 0>(act, ald, x, K, rows, norm, eps, red, tid, 1);
}

// Consumer side of one GEMV phase. The tile's rows form nrg = rs / 16
// groups of 16; warp w takes group w % nrg and, of every stage, the 32-element
// blocks kb with kb % wpr == w / nrg (wpr = 8 / nrg warps per group). Per
// block one ldmatrix.x4 brings the group's 16 rows, two mma.sync form the
// s32 dots against the activation rows (row-major in shared memory, row
// stride ald), and each dot is turned into float exactly, scaled by its fp16
// block scale and added. Lane (g, t) holds activation row g against weight
// rows 2t, 2t + 1, 8 + 2t, 9 + 2t of its group. With one warp per group
// (wide phases) the blocks are added in matmul_dequantized's order; with
// several, their partial sums are added in warp order at the tile's end.
// `s` is the global stage counter. With `skip` the protocol runs but no
// output is written.
__device__ void gemv_consume(const GemvParams& p, int epi, bool skip, const Ring& rg, int s, bool& bad, int* err,
                             const GGeo& geo, int rows_m, const uint8_t* act, int ald, unsigned long long* best_s,
                             const EpiSmem& es, float (*red)[32][4], unsigned long long* tr) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    const int lj = lane >> 3, lq = lane & 7;
    const int nrg = geo.rs >> 4, wpr = kCW / nrg;
    const int grp = warp % nrg, ks = warp / nrg;
    const bool busy = ks < wpr;
    const int lrow = 16 * grp + lq + 8 * (lj >> 1);  // this lane's ldmatrix row in the tile
    const int nkb = geo.W * (kP / 32);               // blocks per stage
    const int nr = geo.row1 - geo.row0;
    const bool arow = g < rows_m;
    const uint8_t* arow_p = act + (size_t)g * ald;
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    for (int i = 0; i < geo.nstages; i++, s++) {
        const int sl = s % rg.S;
        const int tile = i / geo.nps, pp = i - tile * geo.nps;
        const int r = geo.row0 + tile * kTileRows;
        const int rows = min(kTileRows, geo.row1 - r);
        if (!bad && !warp_wait(&rg.full[sl], (s / rg.S) & 1, err)) bad = true;
        if (tr && threadIdx.x == 0 && i == 0) tr[5] = gtime();
        if (!bad && busy && 16 * grp < rows) {
            const uint8_t* st = rg.base + (size_t)sl * rg.slot;
            const uint8_t* dsc = st + geo.W * geo.rs * kP;
            const uint32_t sbase = saddr(st);
            const int rb = 16 * grp + 2 * t;
            auto block = [&](int kb) {
                const int j = kb >> 2, kk = kb & 3;
                const int chunk = 2 * kk + (lj & 1);
                uint32_t b00, b01, b10, b11;
                ldsm_x4(sbase + (uint32_t)(j * geo.rs * kP + lrow * kP + ((chunk ^ (lrow & 7)) << 4)), b00, b01, b10,
                        b11);
                uint32_t a0 = 0, a2 = 0;
                if (arow) {
                    const int kc = (pp * nkb + kb) * 32 + 4 * t;
                    a0 = *reinterpret_cast<const uint32_t*>(arow_p + kc);
                    a2 = *reinterpret_cast<const uint32_t*>(arow_p + kc + 16);
                }
                int d0, d1, d2, d3;
                mma_u8s8(a0, a2, b00, b01, d0, d1);
                mma_u8s8(a0, a2, b10, b11, d2, d3);
                const __half* sc = reinterpret_cast<const __half*>(dsc + j * geo.rs * (kP / 16));
                const float s0 = __half2float(sc[rb * 4 + kk]);
                const float s1 = __half2float(sc[(rb + 1) * 4 + kk]);
                const float s2 = __half2float(sc[(rb + 8) * 4 + kk]);
                const float s3 = __half2float(sc[(rb + 9) * 4 + kk]);
                acc[0] = __fadd_rn(acc[0], __fmul_rn(i2f_exact(d0), s0));
                acc[1] = __fadd_rn(acc[1], __fmul_rn(i2f_exact(d1), s1));
                acc[2] = __fadd_rn(acc[2], __fmul_rn(i2f_exact(d2), s2));
                acc[3] = __fadd_rn(acc[3], __fmul_rn(i2f_exact(d3), s3));
            };
            if (wpr == 1 && nkb == kPPS * (kP / 32)) {
#pragma unroll
                for (int kb = 0; kb < kPPS * (kP / 32); kb++) block(kb);
            } else {
#pragma unroll 4
                for (int kb = ks; kb < nkb; kb += wpr) block(kb);
            }
        }
        __syncwarp();
        if (lane == 0) mb_arrive(&rg.empty[sl]);
        if (pp == geo.nps - 1) {
            if (wpr > 1) {
                // partial sums of the group's warps, added in warp order
#pragma unroll
                for (int q = 0; q < 4; q++) red[warp][lane][q] = acc[q];
                cbar();
                if (ks == 0) {
                    for (int k2 = 1; k2 < wpr; k2++)
#pragma unroll
                        for (int q = 0; q < 4; q++) acc[q] = __fadd_rn(acc[q], red[grp + nrg * k2][lane][q]);
                }
            }
            if (!bad && !skip && arow && ks == 0) {
#pragma unroll
                for (int h = 0; h < 2; h++) {
                    const int lr = 16 * grp + 8 * h + 2 * t;  // even row of the pair within the tile
                    if (lr < rows)
                        pair_epi(p, epi, g, r + lr, lr + 1 < rows, div127(acc[2 * h]),
                                 div127(acc[2 * h + 1]), best_s, es, geo.row0, nr);
                }
            }
            if (wpr > 1) cbar();  // red is free again
            acc[0] = acc[1] = acc[2] = acc[3] = 0.0f;
        }
    }
}

__device__ void gemv_phase(const GemvParams& p, int epi, bool skip, const Ring& rg, int& s, bool& bad, int* err,
                           uint8_t* act, unsigned long long* best_s, float* nred, EpiSmem& es, float (*red)[32][4],
                           unsigned long long* tr) {
    // tr (CTA 0 only, may be null): [3] prologue done, [5] first stage read
    GGeo geo;
    gemv_geo(p, blockIdx.x, gridDim.x, geo);
    // The phase's scalar inputs in one round of loads, then the epilogue
    // inputs and the activations together; the QKV epilogue values ride in
    // registers through the activation prologue and are stored after it.
    const bool qkv = !skip && epi == EPI_QKV;
    int dynm = p.M, sbase = 0, src0 = p.row0;
    if (p.dyn_M) dynm = __ldcg(p.dyn_M);
    if (qkv) sbase = __ldcg(p.slot_base);
    if (p.x_row_dyn) src0 = __ldcg(p.x_row_dyn);
    const int rows_m = max(0, min(min(dynm - p.row0, p.M), kMaxRows));
    const int K = p.K;
    const int ald = K + 16;
    const int tid = threadIdx.x;
    const int nr = geo.row1 - geo.row0;
    if (tid < kMaxRows) best_s[tid] = 0ull;
    int e_pos = 0, e_page = 0, e_off = 0;
    if (qkv) {
        if (tid < rows_m) {
            const int r = p.row0 + tid;
            const int slot = sbase + r;
            e_pos = __ldcg(p.pos + r);
            e_page = p.block_table[slot / kPageSize];
            e_off = slot % kPageSize;
        }
        const int half = p.head_dim >> 1;
        if (tid >= 32 && tid < 32 + half) {
            const int i = tid - 32;
            es.freq[i] = __fdiv_rn(1.0f, powf(p.theta, __fdiv_rn((float)(2 * i), (float)p.head_dim)));
        }
    }
    // activation rows, row-major with stride K + 16 (rows >= rows_m are
    // never stored by the epilogue, so they need no clearing)
    if (!skip && p.x && rows_m > 0) {
        step_prologue(act, ald, p.x + (size_t)src0 * K, K, rows_m, p.norm, p.eps, nred, tid);
    } else if (!skip && rows_m > 0) {
        const int K16 = K >> 4;
        const uint4* src = reinterpret_cast<const uint4*>(p.aq + (size_t)p.row0 * K);
#pragma unroll 4
        for (int i = tid; i < rows_m * K16; i += kCThreads) {
            const int m = i / K16, c = i - m * K16;
            *reinterpret_cast<uint4*>(act + (size_t)m * ald + (size_t)c * 16) = __ldcg(src + (size_t)m * K16 + c);
        }
    }
    if (qkv && tid < rows_m) {
        es.pos[tid] = e_pos;
        es.page[tid] = e_page;
        es.off[tid] = e_off;
    }
    if (!skip && epi == EPI_RESID) {
        for (int i = tid; i < rows_m * nr; i += kCThreads) {
            const int m = i / nr, j = i - m * nr;
            es.res[i] = __ldcg(p.out + (size_t)(p.row0 + m) * p.ldo + geo.row0 + j);
        }
    }
    cbar();
    if (tr && tid == 0) tr[3] = gtime();
    gemv_consume(p, epi, skip || rows_m == 0, rg, s, bad, err, geo, rows_m, act, ald, best_s, es, red, tr);
    s += geo.nstages;
    if (epi == EPI_LOGITS) {
        cbar();
        if (!skip && threadIdx.x < (unsigned)rows_m)
            p.amax_part[(size_t)(p.row0 + threadIdx.x) * gridDim.x + blockIdx.x] = best_s[threadIdx.x];
    }
}

// ---------------------------------------------------------------- attention
constexpr int kHdMax = 128;
constexpr int kAChunk = 64;  // keys per shared-memory chunk

__device__ __forceinline__ void cp16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(saddr(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Shared memory of an attention phase (in the activation region): q rows,
// one chunk of scores, two chunk buffers of K (rows padded by 4 words: the
// 16-byte row reads of a warp hit distinct banks) and of V, running max /
// sum / rescale per row.
constexpr int kAKst = kHdMax / 2 + 4;
constexpr size_t kAttnQ = 0;
constexpr size_t kAttnSc = kAttnQ + sizeof(float) * kMaxRows * kHdMax;
constexpr size_t kAttnK = kAttnSc + sizeof(float) * kMaxRows * kAChunk;
constexpr size_t kAttnV = kAttnK + sizeof(uint32_t) * 2 * kAChunk * kAKst;
constexpr size_t kAttnML = kAttnV + sizeof(uint32_t) * 2 * kAChunk * (kHdMax / 2);
constexpr size_t kAttnBytes = kAttnML + sizeof(float) * 3 * kMaxRows;

// Decode attention of one head for the phase's rows, by one CTA's 8
// consumer warps: the keys [0, base + M) stream through shared memory in
// chunks of kAChunk (16-byte cp.async copies, the next chunk in flight while
// this one is used), an online softmax per row (running max and sum,
// rescaled per chunk), then the normalised P.V is quantized for the o
// projection. Same rule as attention.cu (inference.c:193-247): scores
// q.k / sqrt(hd), causal among the new rows (or the tree mask).
__device__ void attn_head(const AttnParams& p, int h, uint8_t* smem) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int M = p.dyn_M ? __ldcg(p.dyn_M) : p.M;
    const int nr = min(M, kMaxRows);
    if (nr <= 0) return;  // uniform over the CTA
    const int base = __ldcg(p.slot_base);
    const int ctx = base + M;
    const int hd = p.head_dim, hd2 = hd >> 1, hd8 = hd2 >> 2, kst = hd2 + 4;
    const int kvh = h / (p.heads / p.kv_heads);
    const int qd = p.heads * hd;
    float* q_s = reinterpret_cast<float*>(smem + kAttnQ);
    float* sc = reinterpret_cast<float*>(smem + kAttnSc);
    uint32_t* Ks = reinterpret_cast<uint32_t*>(smem + kAttnK);
    uint32_t* Vs = reinterpret_cast<uint32_t*>(smem + kAttnV);
    float* m_run = reinterpret_cast<float*>(smem + kAttnML);
    float* l_run = m_run + kMaxRows;
    float* alpha = l_run + kMaxRows;
    const uint32_t* kg = reinterpret_cast<const uint32_t*>(p.kv.k);
    const uint32_t* vg = reinterpret_cast<const uint32_t*>(p.kv.v);
    const int nchunks = (ctx + kAChunk - 1) / kAChunk;
    auto load = [&](int c) {
        const int k0 = c * kAChunk, nt = min(kAChunk, ctx - k0);
        uint32_t* Kb = Ks + (c & 1) * kAChunk * kAKst;
        uint32_t* Vb = Vs + (c & 1) * kAChunk * (kHdMax / 2);
        for (int i = tid; i < nt * hd8; i += kCThreads) {
            const int key = i / hd8, cc = (i - key * hd8) * 4;
            const int slot = k0 + key;
            const size_t off =
                (((size_t)p.block_table[slot / kPageSize] * p.kv_heads + kvh) * kPageSize + (slot % kPageSize)) * hd2 +
                cc;
            cp16(Kb + key * kst + cc, kg + off);
            cp16(Vb + key * hd2 + cc, vg + off);
        }
        cp_commit();
    };
    load(0);
    for (int i = tid; i < nr * hd; i += kCThreads) {
        const int rr = i / hd, dd = i - rr * hd;
        q_s[rr * kHdMax + dd] = __ldcg(p.q + (size_t)rr * qd + (size_t)h * hd + dd);
    }
    if (tid < kMaxRows) {
        m_run[tid] = -INFINITY;
        l_run[tid] = 0.0f;
    }
    const float scale = __fdiv_rn(1.0f, sqrtf((float)hd));
    // P.V: thread -> (dimension pair d2, row group g of G), rows g, g + G
    const int G = kCThreads / hd2;
    const int d2 = tid % hd2, g = tid / hd2;
    const bool pv = g < G;
    float a0[2] = {0.0f, 0.0f}, a1[2] = {0.0f, 0.0f};
    for (int c = 0; c < nchunks; c++) {
        if (c + 1 < nchunks) {
            load(c + 1);
            cp_wait<1>();
        } else {
            cp_wait<0>();
        }
        cbar();
        const int k0 = c * kAChunk, nt = min(kAChunk, ctx - k0);
        const uint32_t* Kb = Ks + (c & 1) * kAChunk * kAKst;
        const uint32_t* Vb = Vs + (c & 1) * kAChunk * (kHdMax / 2);
        {   // scores: thread -> key (tid % 64), rows rq, rq + 4
            const int key = tid & (kAChunk - 1), rq = tid / kAChunk;
            float acc[2] = {0.0f, 0.0f};
            if (key < nt) {
                const uint4* kr = reinterpret_cast<const uint4*>(Kb + key * kst);
                for (int e4 = 0; e4 < hd8; e4++) {
                    const uint4 kw = kr[e4];
                    const float2 f0 = __half22float2(*reinterpret_cast<const __half2*>(&kw.x));
                    const float2 f1 = __half22float2(*reinterpret_cast<const __half2*>(&kw.y));
                    const float2 f2 = __half22float2(*reinterpret_cast<const __half2*>(&kw.z));
                    const float2 f3 = __half22float2(*reinterpret_cast<const __half2*>(&kw.w));
#pragma unroll
                    for (int i = 0; i < 2; i++) {
                        const int rr = rq + 4 * i;
                        if (rr < nr) {
                            const float4 qa = *reinterpret_cast<const float4*>(&q_s[rr * kHdMax + 8 * e4]);
                            const float4 qb = *reinterpret_cast<const float4*>(&q_s[rr * kHdMax + 8 * e4 + 4]);
                            float v = acc[i];
                            v = __fmaf_rn(qa.x, f0.x, v);
                            v = __fmaf_rn(qa.y, f0.y, v);
                            v = __fmaf_rn(qa.z, f1.x, v);
                            v = __fmaf_rn(qa.w, f1.y, v);
                            v = __fmaf_rn(qb.x, f2.x, v);
                            v = __fmaf_rn(qb.y, f2.y, v);
                            v = __fmaf_rn(qb.z, f3.x, v);
                            v = __fmaf_rn(qb.w, f3.y, v);
                            acc[i] = v;
                        }
                    }
                }
            }
            const int j = k0 + key;
#pragma unroll
            for (int i = 0; i < 2; i++) {
                const int rr = rq + 4 * i;
                if (rr < nr) {
                    bool vis = key < nt;
                    if (vis && j >= base) {
                        const int jj = j - base;
                        vis = p.mask ? (p.mask[(size_t)rr * M + jj] != 0) : (jj <= rr);
                    }
                    sc[rr * kAChunk + key] = vis ? __fmul_rn(acc[i], scale) : -INFINITY;
                }
            }
        }
        cbar();
        // online softmax: warp w -> row w; lane -> keys lane, lane + 32
        if (warp < nr) {
            const float s0 = sc[warp * kAChunk + lane], s1 = sc[warp * kAChunk + lane + 32];
            const float mx = warp_max(fmaxf(s0, s1));
            const float m_old = m_run[warp];
            const float m_new = fmaxf(m_old, mx);
            const float e0 = s0 == -INFINITY ? 0.0f : expf(__fsub_rn(s0, m_new));
            const float e1 = s1 == -INFINITY ? 0.0f : expf(__fsub_rn(s1, m_new));
            sc[warp * kAChunk + lane] = e0;
            sc[warp * kAChunk + lane + 32] = e1;
            const float sum = warp_sum(e0 + e1);
            if (lane == 0) {
                const float al = m_old == -INFINITY ? 0.0f : expf(__fsub_rn(m_old, m_new));
                alpha[warp] = al;
                l_run[warp] = __fmaf_rn(l_run[warp], al, sum);
                m_run[warp] = m_new;
            }
        }
        cbar();
        if (pv) {
#pragma unroll
            for (int i = 0; i < 2; i++) {
                const int rr = g + G * i;
                if (rr < nr) {
                    a0[i] *= alpha[rr];
                    a1[i] *= alpha[rr];
                }
            }
            for (int tt = 0; tt < nt; tt++) {
                const float2 v = __half22float2(*reinterpret_cast<const __half2*>(&Vb[tt * hd2 + d2]));
#pragma unroll
                for (int i = 0; i < 2; i++) {
                    const int rr = g + G * i;
                    if (rr < nr) {
                        const float w = sc[rr * kAChunk + tt];
                        a0[i] = __fmaf_rn(w, v.x, a0[i]);
                        a1[i] = __fmaf_rn(w, v.y, a1[i]);
                    }
                }
            }
        }
        cbar();  // the chunk's buffers and scores are free again
    }
    if (pv) {
#pragma unroll
        for (int i = 0; i < 2; i++) {
            const int rr = g + G * i;
            if (rr < nr) {
                const float inv_l = l_run[rr];
                const float o0 = __fdiv_rn(a0[i], inv_l), o1 = __fdiv_rn(a1[i], inv_l);
                const size_t idx = (size_t)rr * qd + (size_t)h * hd + 2 * d2;
                p.out_q[idx] = (uint8_t)quant_u8(o0);
                p.out_q[idx + 1] = (uint8_t)quant_u8(o1);
                if (p.out_f) {
                    p.out_f[idx] = o0;
                    p.out_f[idx + 1] = o1;
                }
            }
        }
    }
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
    extern __shared__ __align__(1024) uint8_t smem[];
    __shared__ __align__(8) uint64_t full[kMaxSlots];
    __shared__ __align__(8) uint64_t empty[kMaxSlots];
    __shared__ unsigned long long best_s[kMaxRows];
    __shared__ unsigned long long red8[kCW];
    __shared__ int tgt[kMaxRows];
    __shared__ int ok_s, skip_s;
    __shared__ float nred[kMaxRows * kCW];
    __shared__ float red[kCW][32][4];  // per-warp partial sums of a tile (K split over warps)
    __shared__ EpiSmem es;
    // phase descriptors, double-buffered: phase ph + 1 is loaded into
    // registers at the start of phase ph and stored here at its end
    constexpr int kPW = (int)(sizeof(Phase) / sizeof(uint2));
    static_assert(sizeof(Phase) % sizeof(uint2) == 0, "Phase is copied in 8-byte words");
    __shared__ uint2 sph[2][kPW];

    // uniform early exits, before any barrier
    if (__ldcg(p.done)) return;  // the whole decode already finished
    if ((saddr(smem) + p.region_bytes) & 1023) {
        if (threadIdx.x == 0) atomicOr(err, kErrRing);  // the swizzled ring needs 1024-byte alignment
        return;
    }
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

    if (warp == kProdWarp) {
        // ---------------- producer: every GEMV phase's stages, in order ----------------
        if (lane == 0) {
            int s = 0;
            bool ok = true;
            for (int ph = 0; ph < p.nphases && ok; ph++) {
                const Phase* P = p.phases + ph;
                if (P->kind != PH_GEMV) continue;
                GGeo geo;
                gemv_geo(P->g, blockIdx.x, gridDim.x, geo);
                const int N = P->g.N;
                const uint8_t* sb = reinterpret_cast<const uint8_t*>(P->g.sblk);
                for (int i = 0; i < geo.nstages; i++, s++) {
                    const int sl = s % p.S;
                    if (s >= p.S && !mb_wait(&empty[sl], ((s / p.S) - 1) & 1, err)) {
                        ok = false;
                        break;
                    }
                    const int tile = i / geo.nps, pp = i - tile * geo.nps;
                    const int r = geo.row0 + tile * kTileRows;
                    const int rows = min(kTileRows, geo.row1 - r);
                    uint8_t* dw = rg.base + (size_t)sl * p.slot_bytes;
                    mb_expect(&full[sl], (uint32_t)(geo.W * rows * (kP + kP / 16)));
                    for (int j = 0; j < geo.W; j++) {
                        const size_t pan = (size_t)(pp * geo.W + j);
                        bulk(dw + j * geo.rs * kP, P->g.w + (pan * N + r) * kP, (uint32_t)(rows * kP), &full[sl]);
                        bulk(dw + geo.W * geo.rs * kP + j * geo.rs * (kP / 16), sb + (pan * N + r) * (kP / 16),
                             (uint32_t)(rows * (kP / 16)), &full[sl]);
                    }
                }
            }
            // the copies of the last S issued stages land before the CTA ends
            for (int t = s - p.S < 0 ? 0 : s - p.S; t < s; t++)
                if (!mb_wait(&full[t % p.S], (t / p.S) & 1, err)) break;
        }
    } else {
        // ---------------- consumers ----------------
        int s = 0;
        bool bad = false, skip = false;
        const uint2* gph = reinterpret_cast<const uint2*>(p.phases);
        if (threadIdx.x < kPW) sph[0][threadIdx.x] = __ldg(gph + threadIdx.x);
        cbar();
        for (int ph = 0; ph < p.nphases; ph++) {
            const bool more = ph + 1 < p.nphases;
            uint2 nxt = make_uint2(0u, 0u);
            if (more && threadIdx.x < kPW) nxt = __ldg(gph + (size_t)(ph + 1) * kPW + threadIdx.x);
            const Phase& P = *reinterpret_cast<const Phase*>(sph[ph & 1]);
            const int kind = P.kind;
            if (p.trace && blockIdx.x == 0 && threadIdx.x == 0) p.trace[kTr * ph] = gtime();
            if (kind == PH_GEMV) {
                gemv_phase(P.g, P.epi, skip || bad, rg, s, bad, err, smem, best_s, nred, es, red,
                           p.trace && blockIdx.x == 0 ? p.trace + kTr * ph : nullptr);
            } else if (kind == PH_ATTN) {
                if (!skip && !bad) {
                    const AttnParams& a = P.a;
                    for (int h = blockIdx.x; h < a.heads; h += gridDim.x) attn_head(a, h, smem);
                }
            } else if (!skip && !bad && blockIdx.x == 0) {
                control(kind, P.arg, p.sb, p.K, red8, tgt);
            }
            if (more) {
                if (threadIdx.x < kPW) sph[(ph + 1) & 1][threadIdx.x] = nxt;
                if (!grid_sync(reinterpret_cast<unsigned long long*>(p.bar), (unsigned long long)(ph + 1) * gridDim.x,
                               err, &ok_s, bad, p.trace ? p.trace + kTr * ph : nullptr))
                    bad = true;
                if (kind == PH_ACCEPT) {
                    // `done` changes only in the acceptance phase
                    if (threadIdx.x == 0) skip_s = __ldcg(p.done);
                    cbar();
                    skip = skip_s != 0;
                }
            }
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
    int region = (int)kAttnBytes;
    for (int i = 0; i < n; i++) {
        if (ph[i].kind != PH_GEMV) continue;
        const GemvParams& g = ph[i].g;
        if (g.P != kP || g.N % 8 || g.K % (kP * kPPS) || g.M < 1 || g.M > kMaxRows) return false;
        if (ph[i].epi == EPI_QKV && (g.head_dim > kHdMax || g.head_dim % 8)) return false;
        if (ph[i].epi == EPI_RESID) {
            const int grid = step_grid();
            const int rows_cta = ((g.N / 8 + grid - 1) / grid) * 8;
            if (rows_cta * g.M > kResFloats) return false;
        }
        region = region > kMaxRows * (g.K + 16) ? region : kMaxRows * (g.K + 16);  // row-major activations
    }
    region = (region + 1023) & ~1023;
    const int avail = kSmemLimit - region;
    int S = avail / kSlot;
    if (S > kMaxSlots) S = kMaxSlots;
    if (S < 2) return false;
    sp.region_bytes = region;
    sp.S = S;
    sp.slot_bytes = kSlot;
    *smem_bytes = (size_t)region + (size_t)S * kSlot;
    return true;
}

cudaError_t step_set_smem(size_t smem) {
    return cudaFuncSetAttribute(step_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
}

cudaError_t launch_step(const StepParams& p, size_t smem, cudaStream_t s) {
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
