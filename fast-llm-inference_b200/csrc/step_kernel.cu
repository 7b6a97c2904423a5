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

constexpr int kCW = 8;                    // consumer warps (phase work, barriers)
constexpr int kRW = 4;                    // of them, TMEM readout warps in GEMV phases
constexpr int kCThreads = kCW * 32;
constexpr int kProdWarp = kCW;            // TMA producer
constexpr int kMmaWarp = kCW + 1;         // tcgen05.mma issuer, TMEM owner
constexpr int kThr = (kCW + 2) * 32;
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
// (row & 7), i.e. the tcgen05 SWIZZLE_128B K-major layout when a group of
// 8 rows starts on a 1024-byte boundary. A ring stage is a tile of
// kTileRows weight rows x kPPS panels, plus their fp16 block scales; the
// MMA warp issues one tcgen05.mma kind::i8 (A = 128 weight rows s8,
// B = the 8 activation rows u8, K = 32) per 32-element block into its own
// group of 8 TMEM columns, and readout warp w takes TMEM lanes (rows)
// 32w .. 32w + 31: it scales each block's s32 products by the row's block
// scale and adds them in block order (matmul_dequantized's order).
constexpr int kP = 128;                         // panel bytes per row
constexpr int kPPS = 2;                         // panels per stage
constexpr int kTileRows = 128;                  // UMMA M
constexpr int kKBS = kPPS * kP / 32;            // 32-element blocks per stage
constexpr int kSlot = kPPS * (kTileRows * kP + kTileRows * (kP / 16));  // 34 KB
constexpr int kCB = kKBS * 8;                   // TMEM columns per stage
constexpr int kNB = 4;                          // TMEM stage buffers
constexpr int kTmemCols = kNB * kCB;            // 256
static_assert(kSlot % 1024 == 0, "stage slots keep the 1024-byte swizzle alignment");

struct GGeo {
    int nps, row0, row1, ntiles, nstages;  // nps: stages per tile
};

__host__ __device__ inline void gemv_geo(const GemvParams& g, int cta, int ncta, GGeo& o) {
    o.nps = g.K / (kP * kPPS);
    const int nunits = g.N >> 3;
    const int u0 = (int)(((long long)nunits * cta) / ncta);
    const int u1 = (int)(((long long)nunits * (cta + 1)) / ncta);
    o.row0 = u0 * 8;
    o.row1 = u1 * 8;
    o.ntiles = (o.row1 - o.row0 + kTileRows - 1) / kTileRows;
    o.nstages = o.ntiles * o.nps;
}

// Shared-memory matrix descriptor (tcgen05): start, leading / stride byte
// offsets, version 1, layout type (0 none, 2 128-byte swizzle).
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo, uint32_t layout) {
    uint64_t d = (uint64_t)((addr >> 4) & 0x3FFF);
    d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
    d |= (uint64_t)((sbo >> 4) & 0x3FFF) << 32;
    d |= (uint64_t)1 << 46;
    d |= (uint64_t)(layout & 7) << 61;
    return d;
}

// D (s32, TMEM) = A (s8, 128 x 32) x B (u8, 32 x 8), not accumulated.
__device__ __forceinline__ void umma_i8(uint32_t tmem_d, uint64_t da, uint64_t db) {
    // instruction descriptor: D s32, A s8, B u8, both K-major, N = 8, M = 128
    constexpr uint32_t idesc = (2u << 4) | (1u << 7) | (0u << 10) | (1u << 17) | (8u << 24);
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(da), "l"(db), "r"(idesc), "r"(0)
        : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t* b) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(saddr(b))
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

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
    uint64_t* empty;   // slot free (readout warps)
    uint64_t* mdone;   // [kNB] stage MMAs complete (tcgen05.commit)
    uint64_t* tfree;   // [kNB] stage TMEM read (readout warps)
    uint64_t* actrdy;  // activations of the phase written
    uint32_t tmem;
    int S, slot;
};

// The activation prologue out of line: its batched loads want registers
// that the GEMV loops around it do not need at the same time.
__device__ __noinline__ void step_prologue(uint8_t* act, const float* x, int K, int rows, int norm, float eps,
                                           float* red, int tid) {
    act_prologue_rows<kCThreads, kMaxRows, true, true>(act, 0, x, K, rows, norm, eps, red, tid, 1);
}

// Consumer side of one GEMV phase (all 8 consumer warps: prologue; warps
// 0..3: TMEM readout and epilogue). `s` is the global stage counter, `g`
// the GEMV phase counter. With `skip` the protocol runs but no output is
// written.
template <int MR>
__device__ void gemv_readout(const GemvParams& p, int epi, bool skip, const Ring& rg, int s, bool& bad, int* err,
                             const GGeo& geo, int rows_m, unsigned long long* best_s, const EpiSmem& es,
                             unsigned long long* tr, unsigned long long* str) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row = 32 * warp + lane;  // tile row = TMEM lane
    const int nr = geo.row1 - geo.row0;
    float acc[MR];
#pragma unroll
    for (int m = 0; m < MR; m++) acc[m] = 0.0f;
    for (int i = 0; i < geo.nstages; i++, s++) {
        const int sl = s % rg.S, buf = s % kNB;
        const int tile = i / geo.nps, pp = i - tile * geo.nps;
        const int r = geo.row0 + tile * kTileRows;
        const int rows = min(kTileRows, geo.row1 - r);
        if (bad) break;
        if (!warp_wait(&rg.mdone[buf], (s / kNB) & 1, err)) {
            bad = true;
            break;
        }
        if (tr && threadIdx.x == 0 && i == 0) tr[5] = gtime();
        if (str && i < 64 && threadIdx.x == 0) str[8 * i] = gtime();
        tc_fence_after();
        uint32_t v[kKBS * MR];
        const uint32_t ta = rg.tmem + ((uint32_t)(32 * warp) << 16) + (uint32_t)(buf * kCB);
#pragma unroll
        for (int kb = 0; kb < kKBS; kb++) {
            if (MR == 8) {
                asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                             : "=r"(v[kb * MR + 0]), "=r"(v[kb * MR + 1]), "=r"(v[kb * MR + 2]), "=r"(v[kb * MR + 3]),
                               "=r"(v[kb * MR + 4]), "=r"(v[kb * MR + 5]), "=r"(v[kb * MR + 6]), "=r"(v[kb * MR + 7])
                             : "r"(ta + kb * 8));
            } else {
                asm volatile("tcgen05.ld.sync.aligned.32x32b.x1.b32 {%0}, [%1];" : "=r"(v[kb * MR]) : "r"(ta + kb * 8));
            }
        }
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mb_arrive(&rg.tfree[buf]);
        // the row's block scales; the slot is released right after
        if (!warp_wait(&rg.full[sl], (s / rg.S) & 1, err)) {
            bad = true;
            break;
        }
        const uint8_t* dsc = rg.base + (size_t)sl * rg.slot + kPPS * kTileRows * kP;
        uint2 sc[kPPS];
#pragma unroll
        for (int j = 0; j < kPPS; j++) sc[j] = *reinterpret_cast<const uint2*>(dsc + j * kTileRows * (kP / 16) + row * 8);
        __syncwarp();
        if (lane == 0) mb_arrive(&rg.empty[sl]);
        if (str && i < 64 && threadIdx.x == 0) str[8 * i + 1] = gtime();
#pragma unroll
        for (int kb = 0; kb < kKBS; kb++) {
            const uint32_t hw = (kb & 2) ? sc[kb / 4].y : sc[kb / 4].x;
            const __half2 h2 = *reinterpret_cast<const __half2*>(&hw);
            const float sk = (kb & 1) ? __high2float(h2) : __low2float(h2);
#pragma unroll
            for (int m = 0; m < MR; m++) acc[m] = __fadd_rn(acc[m], __fmul_rn(i2f_exact((int)v[kb * MR + m]), sk));
        }
        if (pp == geo.nps - 1) {
            // weight-row pairs (row, row + 1) for even rows: the odd row's
            // values come from lane + 1
#pragma unroll
            for (int m = 0; m < MR; m++) {
                const float o = __shfl_down_sync(0xffffffffu, acc[m], 1);
                if (!skip && !(lane & 1) && row < rows && m < rows_m)
                    pair_epi(p, epi, m, r + row, true, __fdiv_rn(acc[m], 127.0f), __fdiv_rn(o, 127.0f), best_s, es,
                             geo.row0, nr);
                acc[m] = 0.0f;
            }
        }
    }
}

__device__ void gemv_phase(const GemvParams& p, int epi, bool skip, const Ring& rg, int& s, int& g, bool& bad,
                           int* err, uint8_t* act, unsigned long long* best_s, float* nred, EpiSmem& es,
                           unsigned long long* tr, unsigned long long* str) {
    // tr (CTA 0 only, may be null): [3] prologue done, [5] first stage read
    GGeo geo;
    gemv_geo(p, blockIdx.x, gridDim.x, geo);
    const int warp = threadIdx.x >> 5;
    int rows_m = p.M;
    if (p.dyn_M) rows_m = min(__ldcg(p.dyn_M) - p.row0, p.M);
    rows_m = max(0, min(rows_m, kMaxRows));
    const int K = p.K;
    const int tid = threadIdx.x;
    const int nr = geo.row1 - geo.row0;
    if (tid < kMaxRows) best_s[tid] = 0ull;
    // epilogue inputs, loaded in parallel before the activation prologue
    if (!skip && epi == EPI_QKV) {
        if (tid < rows_m) {
            const int r = p.row0 + tid;
            const int slot = __ldcg(p.slot_base) + r;
            es.pos[tid] = __ldcg(p.pos + r);
            es.page[tid] = p.block_table[slot / kPageSize];
            es.off[tid] = slot % kPageSize;
        }
        const int half = p.head_dim >> 1;
        if (tid >= 32 && tid < 32 + half) {
            const int i = tid - 32;
            es.freq[i] = __fdiv_rn(1.0f, powf(p.theta, __fdiv_rn((float)(2 * i), (float)p.head_dim)));
        }
    } else if (!skip && epi == EPI_RESID) {
        for (int i = tid; i < rows_m * nr; i += kCThreads) {
            const int m = i / nr, j = i - m * nr;
            es.res[i] = __ldcg(p.out + (size_t)(p.row0 + m) * p.ldo + geo.row0 + j);
        }
    }
    // activations in the core-matrix layout of 8 rows; rows >= rows_m zero
    if (!skip && p.x && rows_m > 0) {
        const int src0 = p.x_row_dyn ? __ldcg(p.x_row_dyn) : p.row0;
        step_prologue(act, p.x + (size_t)src0 * K, K, rows_m, p.norm, p.eps, nred, tid);
    } else if (!skip && rows_m > 0) {
        const int K16 = K >> 4;
        const uint4* src = reinterpret_cast<const uint4*>(p.aq + (size_t)p.row0 * K);
        for (int i = tid; i < rows_m * K16; i += kCThreads) {
            const int m = i / K16, c = i - m * K16;
            *reinterpret_cast<uint4*>(act + (size_t)c * 128 + m * 16) = __ldcg(src + (size_t)m * K16 + c);
        }
    }
    {
        const int K16 = K >> 4;
        const int zr = kMaxRows - rows_m;
        for (int i = tid; i < zr * K16; i += kCThreads) {
            const int m = rows_m + i / K16, c = i % K16;
            *reinterpret_cast<uint4*>(act + (size_t)c * 128 + m * 16) = make_uint4(0u, 0u, 0u, 0u);
        }
    }
    // generic-proxy writes -> visible to the tensor core's async proxy
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    cbar();
    if (tid == 0) {
        mb_arrive(rg.actrdy);
        if (tr) tr[3] = gtime();
    }
    g++;
    if (warp < kRW) {
        if (rows_m <= 1)
            gemv_readout<1>(p, epi, skip || rows_m == 0, rg, s, bad, err, geo, rows_m, best_s, es, tr, str);
        else
            gemv_readout<8>(p, epi, skip, rg, s, bad, err, geo, rows_m, best_s, es, tr, str);
    }
    s += geo.nstages;
    if (epi == EPI_LOGITS) {
        cbar();
        if (!skip && threadIdx.x < (unsigned)rows_m)
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
        // the page of this head is nt * hd contiguous halves: 16-byte loads
        const int page = p.block_table[sp];
        const size_t off = (((size_t)page * p.kv_heads + kvh) * kPageSize) * hd2;
        const uint4* kg = reinterpret_cast<const uint4*>(reinterpret_cast<const uint32_t*>(p.kv.k) + off);
        const uint4* vg = reinterpret_cast<const uint4*>(reinterpret_cast<const uint32_t*>(p.kv.v) + off);
        const int hd8 = hd2 >> 2;  // 16-byte chunks per key
#pragma unroll 4
        for (int i = tid; i < nt * hd8; i += 128) {
            const uint4 kv4 = __ldcg(kg + i);
            const uint4 vv4 = __ldcg(vg + i);
            const int key = i / hd8, c = (i - key * hd8) * 4;
            sm.K[key][c] = kv4.x;
            sm.K[key][c + 1] = kv4.y;
            sm.K[key][c + 2] = kv4.z;
            sm.K[key][c + 3] = kv4.w;
            *reinterpret_cast<uint4*>(&sm.V[key][c]) = vv4;
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
    extern __shared__ __align__(1024) uint8_t smem[];
    __shared__ __align__(8) uint64_t full[kMaxSlots];
    __shared__ __align__(8) uint64_t empty[kMaxSlots];
    __shared__ __align__(8) uint64_t mdone[kNB];
    __shared__ __align__(8) uint64_t tfree[kNB];
    __shared__ __align__(8) uint64_t actrdy;
    __shared__ uint32_t tmem_base;
    __shared__ unsigned long long best_s[kMaxRows];
    __shared__ unsigned long long red8[kCW];
    __shared__ int tgt[kMaxRows];
    __shared__ int ok_s, skip_s;
    __shared__ float nred[kMaxRows * kCW];
    __shared__ EpiSmem es;
    // phase descriptors, double-buffered: phase ph + 1 is loaded into
    // registers at the start of phase ph and stored here at its end
    constexpr int kPW = (int)(sizeof(Phase) / sizeof(uint2));
    static_assert(sizeof(Phase) % sizeof(uint2) == 0, "Phase is copied in 8-byte words");
    __shared__ uint2 sph[2][kPW];

    // uniform early exits, before any barrier or TMEM allocation
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
    rg.mdone = mdone;
    rg.tfree = tfree;
    rg.actrdy = &actrdy;
    rg.S = p.S;
    rg.slot = p.slot_bytes;
    if (threadIdx.x == 0) {
        for (int i = 0; i < p.S; i++) {
            mb_init(&full[i], 1);
            mb_init(&empty[i], kRW);
        }
        for (int i = 0; i < kNB; i++) {
            mb_init(&mdone[i], 1);
            mb_init(&tfree[i], kRW);
        }
        mb_init(&actrdy, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == kMmaWarp) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(saddr(&tmem_base)),
                     "n"(kTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    rg.tmem = tmem_base;

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
                    mb_expect(&full[sl], (uint32_t)(kPPS * rows * (kP + kP / 16)));
#pragma unroll
                    for (int j = 0; j < kPPS; j++) {
                        const size_t pan = (size_t)(pp * kPPS + j);
                        bulk(dw + j * kTileRows * kP, P->g.w + (pan * N + r) * kP, (uint32_t)(rows * kP), &full[sl]);
                        bulk(dw + kPPS * kTileRows * kP + j * kTileRows * (kP / 16), sb + (pan * N + r) * (kP / 16),
                             (uint32_t)(rows * (kP / 16)), &full[sl]);
                    }
                }
            }
            // the copies of the last S issued stages land before the CTA ends
            for (int t = s - p.S < 0 ? 0 : s - p.S; t < s; t++)
                if (!mb_wait(&full[t % p.S], (t / p.S) & 1, err)) break;
        }
    } else if (warp == kMmaWarp) {
        // ---------------- MMA issuer: every GEMV phase's stages, in order ----------------
        int s = 0, g = 0, issued = 0;
        bool ok = true;
        const uint32_t act_addr = saddr(smem);
        for (int ph = 0; ph < p.nphases && ok; ph++) {
            const Phase* P = p.phases + ph;
            if (P->kind != PH_GEMV) continue;
            GGeo geo;
            gemv_geo(P->g, blockIdx.x, gridDim.x, geo);
            unsigned long long* str =
                p.trace && blockIdx.x == 0 && ph == p.trace_phase ? p.trace + kTr * p.nphases : nullptr;
            if (!warp_wait(&actrdy, g & 1, err)) {
                ok = false;
                break;
            }
            g++;
            for (int i = 0; i < geo.nstages; i++, s++) {
                const int sl = s % p.S, buf = s % kNB;
                const int pp = i % geo.nps;
                if (!warp_wait(&full[sl], (s / p.S) & 1, err)) {
                    ok = false;
                    break;
                }
                if (s >= kNB && !warp_wait(&tfree[buf], ((s / kNB) - 1) & 1, err)) {
                    ok = false;
                    break;
                }
                if (str && i < 64 && lane == 0) str[8 * i + 4] = gtime();
                tc_fence_after();
                if (lane == 0) {
                    const uint32_t wbase = saddr(rg.base + (size_t)sl * p.slot_bytes);
#pragma unroll
                    for (int kb = 0; kb < kKBS; kb++) {
                        const int j = kb / (kP / 32), kk = kb % (kP / 32);
                        const uint64_t da = smem_desc(wbase + j * kTileRows * kP + kk * 32, 16, 1024, 2);
                        const uint64_t db = smem_desc(act_addr + (uint32_t)((pp * kKBS + kb) * 256), 128, 256, 0);
                        umma_i8(rg.tmem + (uint32_t)(buf * kCB + kb * 8), da, db);
                    }
                    umma_commit(&mdone[buf]);
                    if (str && i < 64) str[8 * i + 5] = gtime();
                }
                __syncwarp();
                issued = s + 1;
            }
        }
        // the MMAs in flight complete before TMEM is released
        for (int t = issued - kNB < 0 ? 0 : issued - kNB; t < issued; t++)
            if (!warp_wait(&mdone[t % kNB], (t / kNB) & 1, err)) break;
    } else {
        // ---------------- consumers ----------------
        int s = 0, g = 0;
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
                gemv_phase(P.g, P.epi, skip || bad, rg, s, g, bad, err, smem, best_s, nred, es,
                           p.trace && blockIdx.x == 0 ? p.trace + kTr * ph : nullptr,
                           p.trace && blockIdx.x == 0 && ph == p.trace_phase ? p.trace + kTr * p.nphases : nullptr);
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
    // TMEM is released by its owner once every warp is done with it
    tc_fence_before();
    __syncthreads();
    if (warp == kMmaWarp) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(rg.tmem), "n"(kTmemCols));
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
        region = region > kMaxRows * g.K ? region : kMaxRows * g.K;  // core-matrix activations
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
