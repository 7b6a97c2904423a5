// INT8 GEMM on the 5th-generation tensor cores (sm_100a) for the many-row
// passes of the path: prompt prefill, tree verification (Medusa: 65 rows) and
// the M >= 16 shapes of the matmul sweep. Same contract and result bits as
// matmul_dequantized in block mode (fast_llm/src/kernels/
// dequantized_tensor.c:204-247 with per-32-block fp16 scales):
//   C[m, n] = (sum over blocks b, in order, of (float)dot_b(m, n) * d[n, b]) / 127
// with dot_b the exact int32 dot of 32 u8 activations and 32 s8 weights.
//
// A tile is 128 weight rows x BN (16, 32 or 64) activation rows. The kernel is
// persistent: one CTA per SM walks the tiles blockIdx.x, + gridDim.x, ...
// (activation tiles fastest, so concurrent CTAs share weight tiles in L2),
// and its stage counters run on across tiles, so the next tile's copies and
// MMAs overlap this tile's readout and epilogue (per-tile CTAs spent about
// 6 us per tile on start-up and drain).
//  - warp 0: producer. One thread copies, per 128-byte K-group, the weight
//    tile (128 rows x 128 B; the tiled weight layout already stores each
//    128-byte group XOR-swizzled by row & 7, which is the 128-byte swizzle
//    pattern the MMA descriptor expects, so the bytes move verbatim) and the
//    activation tile (BN rows x 128 B, SWIZZLE_128B) by TMA into a ring of
//    stages; a stage's barrier completes on the copies' byte count, and its
//    slot is reused once the MMAs that read it have committed.
//  - warp 1: allocates all 512 TMEM columns, then issues one
//    tcgen05.mma.cta_group::1.kind::i8 (M = 128, N = BN, K = 32) per 32-element
//    block into its own BN TMEM columns, and one tcgen05.commit per stage
//    (four blocks): the commit both frees the stage's shared-memory slot and
//    hands its TMEM buffer (4 BN columns, one of 512 / (4 BN)) to the
//    readout. Commits are slow enough (about half a microsecond apiece here)
//    that one per block was the kernel's bottleneck.
//  - warps 2 ..: readout, BN / 16 per TMEM lane quadrant, each with 16
//    columns of its quadrant's 32 lanes (one 32x32b.x16 load per block: 3-8 %
//    faster than 8-column warps, while 32-column warps are slower). Per half
//    stage (two blocks) it loads the s32 dots, writes its columns of a
//    stage's TMEM buffer back to 0x4B400000 and releases the buffer once both
//    halves are in registers; the MMAs accumulate onto that value, so each
//    loaded word is already the float 12582912 + dot (exact: |dot| < 2^22).
//    One fma with d and -12582912 d (exact) then yields exactly the rounded
//    product (float)dot * d, which is added to the row's running sum in block
//    order: the sum is bit-identical to the sequential reference order. Pairs
//    of columns go through the packed f32x2 fma / add (per-lane rounding
//    identical to the scalar instructions).
//  - After the last block the readout warps divide by 127 and apply the layer
//    epilogue to (n, n + 1) pairs (lane shuffles).
// Every wait is bounded (2 s of %globaltimer): on expiry the CTA raises an
// error word, stops issuing, waits (bounded) for its own copies and MMAs,
// frees TMEM and exits.
#include <cuda.h>

#include "fl_common.cuh"
#include "fl_epilogue.cuh"
#include "fl_kernels.h"
#include "fl_layout.cuh"

namespace fl {

namespace {

__device__ int g_gemm_error = 0;

constexpr int kMma = 1, kRd0 = 2;  // warp 0 producer, warp 1 MMA, readout from warp 2
// readout warps per TMEM lane quadrant (8 columns each at least), threads
#ifndef FL_GEMM_COLS
#define FL_GEMM_COLS 16
#endif
__host__ __device__ constexpr int rd_per_quad(int bn) { return bn / FL_GEMM_COLS > 1 ? bn / FL_GEMM_COLS : 1; }
__host__ __device__ constexpr int gemm_threads(int bn) { return (kRd0 + 4 * rd_per_quad(bn)) * 32; }
constexpr int kMinStages = 4;
constexpr int kTileN = 128;                 // weight rows per tile (UMMA M)
constexpr int kGroup = 128;                 // K bytes per stage (four 32-element blocks)
constexpr int kABytes = kTileN * kGroup;    // 16 KB
constexpr int kMaxStagesG = 8;
constexpr int kMaxBuf = 32;
constexpr int kSmemBudget = 220 * 1024;
constexpr unsigned long long kWaitNsG = 2000000000ull;
#ifndef FL_GEMM_SUSPEND
#define FL_GEMM_SUSPEND 0
#endif
#if FL_GEMM_SUSPEND
constexpr uint32_t kSuspendNs = 1000000;  // try_wait suspend-time hint (a bound; completion wakes earlier)
#endif
constexpr uint32_t kMagicBits = 0x4B400000u;  // 12582912.0f
// FL_GEMM_BIAS: the readout writes the bias 0x4B400000 back into a TMEM stage
// buffer before releasing it and the MMAs accumulate onto it, so the dots
// leave TMEM already as the bits of 12582912 + dot (no integer add per value).
// 1-6 % less time per launch at 64 and 448 rows (B200), same results.
#ifndef FL_GEMM_BIAS
#define FL_GEMM_BIAS 1
#endif
constexpr float kMagic = 12582912.0f;

__device__ __forceinline__ uint32_t saddr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ unsigned long long gtime() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ void mb_init(uint64_t* b, uint32_t n) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(saddr(b)), "r"(n) : "memory");
}
__device__ __forceinline__ void mb_arrive(uint64_t* b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(saddr(b)) : "memory");
}
__device__ __forceinline__ void mb_expect(uint64_t* b, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(saddr(b)), "r"(bytes) : "memory");
}
// try_wait: with FL_GEMM_SUSPEND a suspend-time hint lets a thread whose
// phase has not completed sleep (woken when the phase completes) instead of
// polling; without it the instruction polls for its own short window.
__device__ __forceinline__ bool mb_try(uint64_t* b, uint32_t par) {
    uint32_t ok;
#if FL_GEMM_SUSPEND
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(saddr(b)), "r"(par), "r"(kSuspendNs)
        : "memory");
#else
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(saddr(b)), "r"(par)
        : "memory");
#endif
    return ok != 0;
}
// Bounded wait of one thread: the clock is read between suspended tries.
__device__ __forceinline__ bool mb_wait(uint64_t* b, uint32_t par) {
    if (mb_try(b, par)) return true;
    const unsigned long long t0 = gtime();
    while (!mb_try(b, par))
        if (gtime() - t0 > kWaitNsG) {
            atomicOr(&g_gemm_error, 1);
            return false;
        }
    return true;
}
// Warp-uniform bounded wait: lane 0 waits, the outcome is broadcast.
__device__ __forceinline__ bool warp_wait(uint64_t* b, uint32_t par) {
    int ok = 1;
    if ((threadIdx.x & 31) == 0) ok = mb_wait(b, par) ? 1 : 0;
    return __shfl_sync(0xffffffffu, ok, 0) != 0;
}


__device__ __forceinline__ void tma_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* b) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
        "[%4];" ::"r"(saddr(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(saddr(b))
        : "memory");
}

// Shared-memory operand descriptor: 128-byte swizzled K-major rows, 8-row
// groups 1024 bytes apart.
__device__ __forceinline__ uint64_t desc_sw128(uint32_t addr) {
    uint64_t d = (uint64_t)((addr >> 4) & 0x3FFF);
    d |= (uint64_t)(16 >> 4) << 16;
    d |= (uint64_t)(1024 >> 4) << 32;
    d |= (uint64_t)1 << 46;
    d |= (uint64_t)2 << 61;
    return d;
}

// D (s32, TMEM) = A (s8, 128 x 32, K-major) x B (u8, 32 x BN, K-major).
template <int BN>
__device__ __forceinline__ void umma_i8(uint32_t tmem_d, uint64_t da, uint64_t db) {
    constexpr uint32_t idesc = (2u << 4) | (1u << 7) | (0u << 10) | ((uint32_t)(BN >> 3) << 17) | (8u << 24);
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(da), "l"(db), "r"(idesc), "r"(FL_GEMM_BIAS ? 1 : 0)
        : "memory");
}
__device__ __forceinline__ void umma_commit(uint64_t* b) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(saddr(b))
                 : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld8(uint32_t ta, uint32_t* v) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
                 : "r"(ta));
}
__device__ __forceinline__ void tmem_ld16(uint32_t ta, uint32_t* v) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(ta));
}
__device__ __forceinline__ void tmem_ld32(uint32_t ta, uint32_t* v) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
          "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]),
          "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
        : "r"(ta));
}
// The readout's load of `n` consecutive columns (n = 8, 16 or 32).
template <int n>
__device__ __forceinline__ void tmem_ld(uint32_t ta, uint32_t* v) {
    if constexpr (n >= 32) {
        tmem_ld32(ta, v);
    } else if constexpr (n >= 16) {
        tmem_ld16(ta, v);
    } else {
        tmem_ld8(ta, v);
    }
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

struct GemmGeo {
    int N, K, M, P;
    int stages, nbuf;
    int mtiles, tiles;  // activation-row tiles; tiles = mtiles x weight-row tiles (m fastest)
};

// Two floats in one 64-bit register: sm_100 packed arithmetic (f32x2), each
// lane rounded exactly like the scalar instruction.
__device__ __forceinline__ unsigned long long pk2(uint32_t lo, uint32_t hi) {
    return ((unsigned long long)hi << 32) | lo;
}
__device__ __forceinline__ unsigned long long fma2(unsigned long long a, unsigned long long b, unsigned long long c) {
    unsigned long long d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
__device__ __forceinline__ unsigned long long add2(unsigned long long a, unsigned long long b) {
    unsigned long long d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}

template <int BN, int EPI>
__global__ void __launch_bounds__(gemm_threads(BN), 1)
    gemm_i8_tc_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_a,
                      const GemvParams g, const GemmGeo geo) {
    extern __shared__ uint8_t smem_raw[];
    // full: stage copied (producers); done: stage's MMAs complete (one
    // tcgen05.commit per stage: frees the smem slot and hands the TMEM buffer
    // to the readout); tempty: TMEM buffer read (readout warps)
    __shared__ __align__(8) uint64_t full[kMaxStagesG], done[kMaxStagesG], tempty[kMaxBuf];
    __shared__ uint32_t tmem_base_s;
    __shared__ int bad_s, issued_s, consumed_s, last_commit_s;

    constexpr int kBBytes = BN * kGroup;
    constexpr int kStage = kABytes + kBBytes;
    constexpr int kWQ = rd_per_quad(BN);
    constexpr int kNRd = 4 * kWQ;
    uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int N = geo.N, K = geo.K, S = geo.stages, NB = geo.nbuf;
    const int nkg = K / kGroup;
    // persistent: this CTA takes tiles blockIdx.x, + gridDim.x, ...; the
    // stage counters (smem slots, TMEM buffers, barrier phases) run on across
    // its tiles, so the next tile's copies and MMAs overlap this tile's
    // readout and epilogue
    auto tile_n0 = [&](int tl) { return (tl / geo.mtiles) * kTileN; };
    auto tile_m0 = [&](int tl) { return (tl % geo.mtiles) * BN; };

    if (threadIdx.x == 0) {
        for (int i = 0; i < S; i++) {
            mb_init(&full[i], 1);  // the producer's expect_tx arrival; completes on the copied bytes
            mb_init(&done[i], 1);
        }
        for (int i = 0; i < NB; i++) mb_init(&tempty[i], kNRd);
        bad_s = 0;
        issued_s = 0;
        consumed_s = 0;
        last_commit_s = -1;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == kMma) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(saddr(&tmem_base_s)));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base_s;

    if (warp == 0) {
        if (lane == 0) {
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tm_w)) : "memory");
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tm_a)) : "memory");
            int gk = 0;  // stages issued over this CTA's tiles
            bool stop = false;
            for (int tl = blockIdx.x; tl < geo.tiles && !stop; tl += gridDim.x) {
                const int n0 = tile_n0(tl), m0 = tile_m0(tl);
                for (int kg = 0; kg < nkg; kg++, gk++) {
                    const int s = gk % S;
                    // the slot's previous stage must have been consumed by its MMAs
                    if ((gk >= S && !mb_wait(&done[s], ((gk / S) - 1) & 1)) || *(volatile int*)&bad_s) {
                        atomicOr(&bad_s, 1);
                        stop = true;
                        break;
                    }
                    uint8_t* st = smem + (size_t)s * kStage;
                    const int kb = kg * kGroup;
                    const int pan = kb / geo.P;
                    mb_expect(&full[s], kBBytes + kABytes);
                    tma_2d(st, &tm_w, kb - pan * geo.P, pan * N + n0, &full[s]);
                    tma_2d(st + kABytes, &tm_a, kb, m0, &full[s]);
                }
            }
            issued_s = gk;
        }
    } else if (warp == kMma) {
        if (lane == 0) {
            const int my_tiles = blockIdx.x < geo.tiles ? (geo.tiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;
            const int total = my_tiles * nkg;
            int kg = 0;
            for (; kg < total; kg++) {
                const int s = kg % S;
                if (!mb_wait(&full[s], (kg / S) & 1)) {
                    atomicOr(&bad_s, 1);
                    break;
                }
                const int t = kg % NB;
                // with the bias, phase 0 of every buffer is the readout's initial fill
                if ((FL_GEMM_BIAS || kg >= NB) && !mb_wait(&tempty[t], ((kg / NB) - (FL_GEMM_BIAS ? 0 : 1)) & 1)) {
                    atomicOr(&bad_s, 1);
                    break;
                }
                tc_fence_after();
                const uint32_t a_addr = saddr(smem + (size_t)s * kStage);
#pragma unroll
                for (int j = 0; j < 4; j++)
                    umma_i8<BN>(tmem + (uint32_t)((t * 4 + j) * BN), desc_sw128(a_addr + 32 * j),
                                desc_sw128(a_addr + kABytes + 32 * j));
                umma_commit(&done[s]);
                last_commit_s = kg;
            }
            consumed_s = kg;
        }
    } else {
        // readout warps: TMEM lanes of quadrant (warp % 4), 1 / kWQ of the columns
        const int q = warp & 3, part = (warp - kRd0) >> 2;  // warps 2-9: quadrants 2, 3, 0, 1, 2, 3, 0, 1
        constexpr int kCols = BN / kWQ;
        static_assert(kCols % 8 == 0, "TMEM loads move 8 columns");
        const int c0 = part * kCols;
        const uint32_t tq = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)c0;
        unsigned long long acc2[kCols / 2];  // column pairs (2c, 2c + 1)
        int n = 0, g0 = 0;  // this tile's weight row; global stage of its first K-group
        bool live = false;
        // fp16 block scales of row n: four per K-group, prefetched one group ahead
        auto load_sc = [&](int kg) -> uint2 {
            if (!live || kg >= nkg) return make_uint2(0u, 0u);
            return __ldg(reinterpret_cast<const uint2*>(g.sblk + tiled_s_off(N, geo.P, n, kg * 4)));
        };
        constexpr int kV = 2 * kCols;  // registers per half stage (two blocks)
        constexpr int kLdW = kCols >= 32 ? 32 : (kCols >= 16 ? 16 : 8);  // columns per TMEM load
        uint32_t va[kV], vb[kV];
        // half stage h of the tile: blocks 2 (h & 1), 2 (h & 1) + 1 of its
        // stage h / 2 (global stage g0 + h / 2)
        auto ld_half = [&](int h, uint32_t* v) {
            const uint32_t base = tq + (uint32_t)(((g0 + (h >> 1)) % NB) * 4 * BN + (h & 1) * 2 * BN);
#pragma unroll
            for (int j = 0; j < 2; j++)
#pragma unroll
                for (int c = 0; c < kCols; c += kLdW) tmem_ld<kLdW>(base + (uint32_t)(j * BN + c), v + j * kCols + c);
        };
        auto scale_add = [&](const uint32_t* v, float d) {
            const float nmd = __fmul_rn(-kMagic, d);  // exact: 3 * 2^22 * d
            const unsigned long long d2 = pk2(__float_as_uint(d), __float_as_uint(d));
            const unsigned long long n2 = pk2(__float_as_uint(nmd), __float_as_uint(nmd));
#pragma unroll
            for (int c = 0; c < kCols / 2; c++)
                acc2[c] = add2(acc2[c], FL_GEMM_BIAS ? fma2(pk2(v[2 * c], v[2 * c + 1]), d2, n2)
                                                     : fma2(pk2(v[2 * c] + kMagicBits, v[2 * c + 1] + kMagicBits), d2, n2));
        };
#if FL_GEMM_BIAS
        // this warp's columns of a stage buffer back to the bias (four
        // columns per store keep the register footprint small)
        auto fill = [&](int buf) {
#pragma unroll
            for (int j = 0; j < 4; j++)
#pragma unroll
                for (int c = 0; c < kCols; c += 4)
                    asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1, %1, %1, %1};" ::"r"(
                                     tq + (uint32_t)(buf * 4 * BN + j * BN + c)),
                                 "r"(kMagicBits)
                                 : "memory");
        };
        for (int b = 0; b < NB; b++) fill(b);
        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
        tc_fence_before();
        __syncwarp();
        if (lane == 0)
            for (int b = 0; b < NB; b++) mb_arrive(&tempty[b]);
#endif
        const int nh = 2 * nkg;
        // one half stage: start the next half's load (waiting for its stage's
        // MMAs when it opens a stage), free a stage's TMEM buffer once both its
        // halves are in registers, scale and add two blocks, wait for the load
        auto step = [&](int h, const uint32_t* cur, uint32_t* nxt, uint32_t scw) -> bool {
            const bool more = h + 1 < nh;
            if (more) {
                if (((h + 1) & 1) == 0) {
                    const int gs = g0 + ((h + 1) >> 1);
                    if (!warp_wait(&done[gs % S], (gs / S) & 1)) return false;
                    tc_fence_after();
                }
                ld_half(h + 1, nxt);
            }
            if (h & 1) {
#if FL_GEMM_BIAS
                fill((g0 + (h >> 1)) % NB);
                asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
#endif
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mb_arrive(&tempty[(g0 + (h >> 1)) % NB]);
            }
            const __half2 hs = *reinterpret_cast<const __half2*>(&scw);
            scale_add(cur, __low2float(hs));
            scale_add(cur + kCols, __high2float(hs));
            if (more) tmem_wait_ld();
            return true;
        };
        bool bad = false;
        for (int tl = blockIdx.x; tl < geo.tiles && !bad; tl += gridDim.x, g0 += nkg) {
            const int m0 = tile_m0(tl);
            n = tile_n0(tl) + 32 * q + lane;
            live = n < N;
#pragma unroll
            for (int j = 0; j < kCols / 2; j++) acc2[j] = 0ull;
            bad = !warp_wait(&done[g0 % S], (g0 / S) & 1);
            if (!bad) {
                tc_fence_after();
                ld_half(0, va);
                tmem_wait_ld();
            }
            uint2 sc_next = load_sc(0);
            for (int kg = 0; kg < nkg && !bad; kg++) {
                const uint2 sc = sc_next;
                sc_next = load_sc(kg + 1);
                if (!step(2 * kg, va, vb, sc.x)) bad = true;
                else if (!step(2 * kg + 1, vb, va, sc.y)) bad = true;
            }
            if (bad) break;
#pragma unroll
            for (int c = 0; c < kCols; c++) {
                const uint32_t bits = (c & 1) ? (uint32_t)(acc2[c >> 1] >> 32) : (uint32_t)acc2[c >> 1];
                const float y = div127(__uint_as_float(bits));
                const float y1 = __shfl_xor_sync(0xffffffffu, y, 1);
                const int m = m0 + c0 + c;
                if ((lane & 1) == 0 && live && m < geo.M) pair_epilogue<EPI>(g, m, n, n + 1 < N, y, y1, nullptr);
            }
        }
        if (bad && lane == 0) atomicOr(&bad_s, 1);
    }
    __syncthreads();
    if (bad_s) {
        // drain: the MMAs of the last commit, then every stage copied but not
        // consumed (its TMA writes land in this CTA's shared memory)
        if (warp == kMma && lane == 0 && last_commit_s >= 0)
            (void)mb_wait(&done[last_commit_s % S], (last_commit_s / S) & 1);
        if (threadIdx.x == 0)
            for (int g2 = consumed_s; g2 < issued_s; g2++) (void)mb_wait(&full[g2 % S], (g2 / S) & 1);
        __syncthreads();
    }
    if (warp == kMma) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem));
    }
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no -lcuda).
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (EncodeTiledFn)p;
    }
    return fn;
}

// 2-D u8 map: inner extent `inner` bytes, `rows` rows `stride` bytes apart,
// box {128 bytes, box_rows}.
bool make_map(CUtensorMap* m, const void* base, uint64_t inner, uint64_t rows, uint64_t stride, uint32_t box_rows,
              bool swizzle) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[2] = {inner, rows};
    const cuuint64_t strides[1] = {stride};
    const cuuint32_t box[2] = {(cuuint32_t)kGroup, box_rows};
    const cuuint32_t es[2] = {1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, es,
              CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// SMs of the current device (the persistent grid).
int gemm_sms() {
    static int sms = 0;
    if (!sms) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (sms <= 0) sms = 148;
    }
    return sms;
}

template <int BN, int EPI>
cudaError_t launch_bn(const CUtensorMap& tw, const CUtensorMap& ta, const GemvParams& g, int M, cudaStream_t s) {
    constexpr int stage = kABytes + BN * kGroup;
    GemmGeo geo;
    geo.N = g.N;
    geo.K = g.K;
    geo.M = M;
    geo.P = g.P;
    geo.stages = std::min(kMaxStagesG, (kSmemBudget - 1024) / stage);
    if (geo.stages < kMinStages) return cudaErrorInvalidConfiguration;
    geo.nbuf = std::min(geo.stages, 512 / (4 * BN));  // TMEM stage buffers (no more than smem stages)
    geo.mtiles = (M + BN - 1) / BN;
    geo.tiles = geo.mtiles * ((g.N + kTileN - 1) / kTileN);
    const size_t smem = (size_t)geo.stages * stage + 1024;
    auto kern = gemm_i8_tc_kernel<BN, EPI>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    // one CTA per SM (all TMEM columns, most of shared memory), persistent
    const dim3 grid(std::min(geo.tiles, gemm_sms()));
    kern<<<grid, gemm_threads(BN), smem, s>>>(tw, ta, g, geo);
    return cudaGetLastError();
}

template <int EPI>
cudaError_t launch_epi(const CUtensorMap& tw, const CUtensorMap& ta, const GemvParams& g, int M, int BN,
                       cudaStream_t s) {
    switch (BN) {
        case 16: return launch_bn<16, EPI>(tw, ta, g, M, s);
        case 32: return launch_bn<32, EPI>(tw, ta, g, M, s);
        default: return launch_bn<64, EPI>(tw, ta, g, M, s);
    }
}

}  // namespace

bool gemm_tc_supported(const GemvParams& g, int epi) {
    if (epi != EPI_STORE && epi != EPI_RESID && epi != EPI_QKV && epi != EPI_SWIGLU) return false;
    if (g.P == 0 || g.K % kGroup || g.P % kGroup || g.N % 16 || g.row0 != 0 || g.dyn_M || g.x) return false;
    if (((uintptr_t)g.aq & 15) || ((uintptr_t)g.w & 15) || ((uintptr_t)g.sblk & 7)) return false;
    return encode_fn() != nullptr;
}

// Tile width: the candidate (16, 32 or 64 activation rows) with the least
// modelled time = waves x per-tile time. Measured per-tile times over
// K = 3072 on B200 are about 27.6, 33.2 and 44.4 us for 16-, 32- and 64-row
// tiles (22 + 0.35 BN): wider tiles read each weight tile once for more rows
// and give it more readout warps, narrower ones spread small-N layers (the o
// and down projections: 24 weight tiles) over more SMs.
#ifndef FL_GEMM_MAX_BN
#define FL_GEMM_MAX_BN 64
#endif
int pick_bn(int M, int N) {
    const int sms = gemm_sms();
    const int ntiles = (N + kTileN - 1) / kTileN;
    int best = 16;
    double best_t = 1e30;
    for (int bn = 16; bn <= FL_GEMM_MAX_BN; bn *= 2) {
        const int mt = (M + bn - 1) / bn;
        const int waves = (ntiles * mt + sms - 1) / sms;
        const double t = waves * (22.0 + 0.35 * bn);
        if (t < best_t - 1e-9) {
            best_t = t;
            best = bn;
        }
        if (bn >= M) break;
    }
    return best;
}

cudaError_t launch_gemm_tc(const GemvParams& g, int epi, int M, cudaStream_t s) {
    if (M <= 0) return cudaSuccess;
    const int BN = pick_bn(M, g.N);
    CUtensorMap tw, ta;
    const int npan = g.K / g.P;
    if (!make_map(&tw, g.w, (uint64_t)g.P, (uint64_t)g.N * npan, (uint64_t)g.P, kTileN, false) ||
        !make_map(&ta, g.aq, (uint64_t)g.K, (uint64_t)M, (uint64_t)g.K, (uint32_t)BN, true))
        return cudaErrorInvalidValue;
    switch (epi) {
        case EPI_STORE: return launch_epi<EPI_STORE>(tw, ta, g, M, BN, s);
        case EPI_RESID: return launch_epi<EPI_RESID>(tw, ta, g, M, BN, s);
        case EPI_QKV: return launch_epi<EPI_QKV>(tw, ta, g, M, BN, s);
        case EPI_SWIGLU: return launch_epi<EPI_SWIGLU>(tw, ta, g, M, BN, s);
        default: return cudaErrorInvalidValue;
    }
}

int take_gemm_error() {
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_gemm_error, sizeof(int)) != cudaSuccess) return -1;
    if (v) {
        const int z = 0;
        cudaMemcpyToSymbol(g_gemm_error, &z, sizeof(int));
    }
    return v;
}

}  // namespace fl
