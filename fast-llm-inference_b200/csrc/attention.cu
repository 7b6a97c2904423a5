// RMSNorm + activation quantization, and tree-masked attention over the
// paged fp16 KV cache (sm_100a).
#include <float.h>

#include "fl_common.cuh"
#include "fl_kernels.h"

namespace fl {

namespace {

__device__ __forceinline__ int kv_head_of(const AttnParams& p, int h) {
    return p.group > 0 ? (p.q_head0 + h) / p.group - p.kv_head0 : h / (p.heads / p.kv_heads);
}

constexpr int kQThreads = 256;

// One CTA per activation row: optional RMSNorm with unit weights
// (activations_avx2.c:108-143 + inference.c:275-283), then the reference's
// u8 quantization (dequantized_tensor.c:112-135).
__global__ void __launch_bounds__(kQThreads) act_quant_kernel(const ActQuantParams p) {
    pdl_trigger();
    pdl_wait();
    if (p.done && *p.done) return;
    const int r = p.row0 + blockIdx.x;
    if (p.dyn_M && r >= *p.dyn_M) return;
    const int src = p.dyn_src_row ? *p.dyn_src_row + (int)blockIdx.x : r;
    const float* x = p.x + (size_t)src * p.K;
    uint8_t* q = p.q + (size_t)r * p.K;
    float scale = 1.0f;
    if (p.norm) {
        __shared__ float red[kQThreads / 32];
        float s = 0.0f;
        for (int i = threadIdx.x * 4; i < p.K; i += kQThreads * 4) {
            const float4 v = *reinterpret_cast<const float4*>(x + i);
            s = __fmaf_rn(v.x, v.x, s);
            s = __fmaf_rn(v.y, v.y, s);
            s = __fmaf_rn(v.z, v.z, s);
            s = __fmaf_rn(v.w, v.w, s);
        }
        s = warp_sum(s);
        if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
        __syncthreads();
        float tot = 0.0f;
#pragma unroll
        for (int w = 0; w < kQThreads / 32; w++) tot += red[w];
        scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)p.K), p.eps)));
    }
    for (int i = threadIdx.x * 4; i < p.K; i += kQThreads * 4) {
        const float4 v = *reinterpret_cast<const float4*>(x + i);
        *reinterpret_cast<uint32_t*>(q + i) =
            quant_pack4(__fmul_rn(v.x, scale), __fmul_rn(v.y, scale), __fmul_rn(v.z, scale),
                        __fmul_rn(v.w, scale));
    }
}

constexpr int kAThreads = 256;
constexpr int kARows = 8;     // query rows per CTA
constexpr int kMaxHd = 128;
constexpr int kTile = 128;    // keys per shared-memory tile

// Attention of up to kARows query rows of one head over slots
// [0, base + M): prefix slots [0, base) are visible to every row, new slot
// base + j to new row i iff mask[i*M + j] (causal j <= i when mask is NULL).
// inference.c:193-247 restated for a paged KV cache: scores q.k / sqrt(hd),
// softmax, p-weighted sum of V. Keys stream through shared memory in tiles
// of kTile with coalesced loads; the softmax is accumulated online (running
// max and sum per row, rescaled per tile), which equals the reference's
// two-pass softmax up to float rounding.
__global__ void __launch_bounds__(kAThreads) attention_kernel(const AttnParams p) {
    extern __shared__ __align__(16) float sm[];
    pdl_trigger();
    pdl_wait();
    if (p.done && *p.done) return;
    const int M = p.dyn_M ? *p.dyn_M : p.M;
    const int h = blockIdx.x;
    const int r0 = blockIdx.y * kARows;
    if (r0 >= M) return;
    const int nr = min(kARows, M - r0);
    // batched sequences: this CTA's sequence, its rows and its cache region
    const int sb = blockIdx.z;
    const int base = p.slot_base[sb * p.seq_state];
    const int* btab = p.block_table + (sb * p.seq_slots) / kPageSize;
    const size_t qrow0 = (size_t)sb * M + r0;
    const int ctx = base + M;
    const int hd = p.head_dim;
    const int hd2 = hd >> 1;
    const int kvh = kv_head_of(p, h);
    const int qd = p.heads * hd;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int kstride = hd2 + 1;  // words per K row in smem (odd: conflict-free)

    float* q_s = sm;                                   // [kARows][hd]
    float* sc = q_s + kARows * kMaxHd;                 // [kARows][kTile]
    uint32_t* Ks = reinterpret_cast<uint32_t*>(sc + kARows * kTile);  // [kTile][kstride] half2
    uint32_t* Vs = Ks + kTile * (kMaxHd / 2 + 1);      // [kTile][hd2] half2
    float* red = reinterpret_cast<float*>(Vs + kTile * (kMaxHd / 2));  // [groups][kARows][hd]
    __shared__ float m_run[kARows], l_run[kARows], alpha_s[kARows];

    for (int i = threadIdx.x; i < nr * hd; i += kAThreads) {
        const int rr = i / hd, dd = i - rr * hd;
        q_s[rr * hd + dd] = p.q[(qrow0 + rr) * qd + (size_t)h * hd + dd];
    }
    if (threadIdx.x < kARows) {
        m_run[threadIdx.x] = -INFINITY;
        l_run[threadIdx.x] = 0.0f;
    }
    const float scale = __fdiv_rn(1.0f, sqrtf((float)hd));
    // P.V mapping: thread -> (dimension pair d2, key group g)
    const int G = kAThreads / hd2;
    const int d2 = threadIdx.x % hd2;
    const int g = threadIdx.x / hd2;
    const bool pv = g < G;
    float a0[kARows], a1[kARows];
#pragma unroll
    for (int rr = 0; rr < kARows; rr++) { a0[rr] = 0.0f; a1[rr] = 0.0f; }

    // causal (no mask): keys after this CTA's last row are hidden from all
    // its rows, so the loop stops there; a tree mask may expose any new slot
    const int kend = p.mask ? ctx : min(ctx, base + r0 + nr);
    for (int j0 = 0; j0 < kend; j0 += kTile) {
        const int nt = min(kTile, kend - j0);
        __syncthreads();  // previous tile fully consumed
        // K and V tile, consecutive threads -> consecutive words: 16-byte
        // loads (four half2 words), several in flight per thread, when a key
        // row is a whole number of them; else one word at a time
        if ((hd2 & 3) == 0) {
            const int hd8 = hd2 >> 2;
#pragma unroll 4
            for (int i = threadIdx.x; i < nt * hd8; i += kAThreads) {
                const int key = i / hd8, c = (i - key * hd8) * 4;
                const int slot = j0 + key;
                const int page = btab[slot / kPageSize];
                const size_t off = (((size_t)page * p.kv_heads + kvh) * kPageSize + (slot % kPageSize)) * hd2 + c;
                const uint4 k4 = *reinterpret_cast<const uint4*>(reinterpret_cast<const uint32_t*>(p.kv.k) + off);
                const uint4 v4 = *reinterpret_cast<const uint4*>(reinterpret_cast<const uint32_t*>(p.kv.v) + off);
                uint32_t* kd = Ks + key * kstride + c;
                kd[0] = k4.x;
                kd[1] = k4.y;
                kd[2] = k4.z;
                kd[3] = k4.w;
                *reinterpret_cast<uint4*>(Vs + key * hd2 + c) = v4;
            }
        } else {
            for (int i = threadIdx.x; i < nt * hd2; i += kAThreads) {
                const int key = i / hd2, c = i - key * hd2;
                const int slot = j0 + key;
                const int page = btab[slot / kPageSize];
                const size_t off = (((size_t)page * p.kv_heads + kvh) * kPageSize + (slot % kPageSize)) * hd2 + c;
                Ks[key * kstride + c] = reinterpret_cast<const uint32_t*>(p.kv.k)[off];
                Vs[key * hd2 + c] = reinterpret_cast<const uint32_t*>(p.kv.v)[off];
            }
        }
        __syncthreads();
        // scores: thread -> key (tid % kTile) and half of the rows (tid / kTile);
        // warps lie within one half, so the q reads are broadcasts
        static_assert(kAThreads == 2 * kTile && kARows % 2 == 0, "two threads per key");
        {
            constexpr int kHalf = kARows / 2;
            const int key = threadIdx.x & (kTile - 1);
            const int rh = (threadIdx.x / kTile) * kHalf;
            if (key < nt && rh < nr) {
                const int j = j0 + key;
                float acc[kHalf];
#pragma unroll
                for (int i = 0; i < kHalf; i++) acc[i] = 0.0f;
                const uint32_t* kr = Ks + key * kstride;
                for (int e = 0; e < hd2; e++) {
                    const float2 kf = __half22float2(*reinterpret_cast<const __half2*>(&kr[e]));
#pragma unroll
                    for (int i = 0; i < kHalf; i++) {
                        if (rh + i < nr) {
                            acc[i] = __fmaf_rn(q_s[(rh + i) * hd + 2 * e], kf.x, acc[i]);
                            acc[i] = __fmaf_rn(q_s[(rh + i) * hd + 2 * e + 1], kf.y, acc[i]);
                        }
                    }
                }
#pragma unroll
                for (int i = 0; i < kHalf; i++) {
                    const int rr = rh + i;
                    if (rr < nr) {
                        bool vis = true;
                        if (j >= base) {
                            const int jj = j - base, ii = r0 + rr;
                            vis = p.mask ? (p.mask[(size_t)ii * M + jj] != 0) : (jj <= ii);
                        }
                        sc[rr * kTile + key] = vis ? __fmul_rn(acc[i], scale) : -INFINITY;
                    }
                }
            }
        }
        __syncthreads();
        // online softmax update: warp rr owns row rr
        if (warp < nr) {
            float* s = sc + warp * kTile;
            float mx = -INFINITY;
            for (int t = lane; t < nt; t += 32) mx = fmaxf(mx, s[t]);
            mx = warp_max(mx);
            const float m_old = m_run[warp];
            const float m_new = fmaxf(m_old, mx);
            float sum = 0.0f;
            for (int t = lane; t < nt; t += 32) {
                const float e = (s[t] == -INFINITY) ? 0.0f : expf(__fsub_rn(s[t], m_new));
                s[t] = e;
                sum += e;
            }
            sum = warp_sum(sum);
            if (lane == 0) {
                const float al = (m_old == -INFINITY) ? 0.0f : expf(__fsub_rn(m_old, m_new));
                alpha_s[warp] = al;
                l_run[warp] = __fmaf_rn(l_run[warp], al, sum);
                m_run[warp] = m_new;
            }
        }
        __syncthreads();
        if (pv) {
#pragma unroll
            for (int rr = 0; rr < kARows; rr++) {
                if (rr < nr) {
                    a0[rr] *= alpha_s[rr];
                    a1[rr] *= alpha_s[rr];
                }
            }
            for (int t = g; t < nt; t += G) {
                const float2 v = __half22float2(*reinterpret_cast<const __half2*>(&Vs[t * hd2 + d2]));
#pragma unroll
                for (int rr = 0; rr < kARows; rr++) {
                    if (rr < nr) {
                        const float w = sc[rr * kTile + t];
                        a0[rr] = __fmaf_rn(w, v.x, a0[rr]);
                        a1[rr] = __fmaf_rn(w, v.y, a1[rr]);
                    }
                }
            }
        }
    }
    // reduce the key groups, normalise, quantize
    __syncthreads();
    if (pv) {
#pragma unroll
        for (int rr = 0; rr < kARows; rr++) {
            if (rr < nr) {
                red[(g * kARows + rr) * hd + 2 * d2] = a0[rr];
                red[(g * kARows + rr) * hd + 2 * d2 + 1] = a1[rr];
            }
        }
    }
    __syncthreads();
    for (int i = threadIdx.x; i < nr * hd; i += kAThreads) {
        const int rr = i / hd, dd = i - rr * hd;
        float o = 0.0f;
        for (int gg = 0; gg < G; gg++) o += red[(gg * kARows + rr) * hd + dd];
        o = __fdiv_rn(o, l_run[rr]);
        const size_t idx = (qrow0 + rr) * qd + (size_t)h * hd + dd;
        p.out_q[idx] = (uint8_t)quant_u8(o);
        if (p.out_f) p.out_f[idx] = o;
    }
}


constexpr int kSplit = 64;     // keys per split = one KV page
constexpr int kDThreads = 128;

// Decode attention (M <= 8 new rows), split-K over pages: CTA (h, sp) takes
// the 64 slots of page sp, computes each row's local max, sum of exp and
// unnormalised P.V, writes them to scratch; the last CTA of the head to
// arrive (device-scope counter) combines the splits in split order --
// deterministic -- normalises, quantizes, and re-arms the counter. Same
// arithmetic as inference.c:193-247 up to float rounding.
template <int MR>
__global__ void __launch_bounds__(kDThreads) attention_split_kernel(const AttnParams p) {
    __shared__ __align__(16) float q_s[MR][kMaxHd];
    __shared__ uint32_t Ks[kSplit][kMaxHd / 2 + 1];
    __shared__ __align__(16) uint32_t Vs[kSplit][kMaxHd / 2];
    __shared__ float sc[MR][kSplit];
    __shared__ float ml_s[MR][2];
    __shared__ int ticket_s;
    pdl_trigger();
    pdl_wait();
    if (p.done && *p.done) return;
    const int M = p.dyn_M ? *p.dyn_M : p.M;
    const int nr = min(M, MR);
    const int h = blockIdx.x, sp = blockIdx.y;
    const int sb = blockIdx.z;  // batched sequence
    const int base = p.slot_base[sb * p.seq_state];
    const size_t qrow0 = (size_t)sb * M;
    const int ctx = base + M;
    const int nsplit = (ctx + kSplit - 1) / kSplit;
    if (sp >= nsplit || nr <= 0) return;
    const int hd = p.head_dim, hd2 = hd >> 1;
    const int kvh = kv_head_of(p, h);
    const int qd = p.heads * hd;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int j0 = sp * kSplit;
    const int nt = min(kSplit, ctx - j0);

    for (int i = threadIdx.x; i < nr * hd; i += kDThreads) {
        const int rr = i / hd, dd = i - rr * hd;
        q_s[rr][dd] = p.q[(qrow0 + rr) * qd + (size_t)h * hd + dd];
    }
    {   // the split is one page: contiguous [64][hd] halves for this kv head
        const int page = p.block_table[(sb * p.seq_slots) / kPageSize + sp];
        const size_t base_off = (((size_t)page * p.kv_heads + kvh) * kPageSize) * hd2;
        const uint32_t* kg = reinterpret_cast<const uint32_t*>(p.kv.k) + base_off;
        const uint32_t* vg = reinterpret_cast<const uint32_t*>(p.kv.v) + base_off;
        if ((hd2 & 3) == 0) {
            // 16-byte loads, all issued before the shared-memory stores
            const uint4* kg4 = reinterpret_cast<const uint4*>(kg);
            const uint4* vg4 = reinterpret_cast<const uint4*>(vg);
            const int hd8 = hd2 >> 2;
#pragma unroll 4
            for (int i = threadIdx.x; i < nt * hd8; i += kDThreads) {
                const uint4 k4 = kg4[i];
                const uint4 v4 = vg4[i];
                const int key = i / hd8, c = (i - key * hd8) * 4;
                Ks[key][c] = k4.x;
                Ks[key][c + 1] = k4.y;
                Ks[key][c + 2] = k4.z;
                Ks[key][c + 3] = k4.w;
                *reinterpret_cast<uint4*>(&Vs[key][c]) = v4;
            }
        } else {
            for (int i = threadIdx.x; i < nt * hd2; i += kDThreads) {
                const int key = i / hd2, c = i - key * hd2;
                Ks[key][c] = kg[i];
                Vs[key][c] = vg[i];
            }
        }
    }
    __syncthreads();
    const float scale = __fdiv_rn(1.0f, sqrtf((float)hd));
    {   // scores: warp w -> keys lane + 32 (w & 1), rows (w >> 1) + 2i
        const int key = lane + 32 * (warp & 1);
        const int rb = warp >> 1;
        if (key < nt) {
            float acc[(MR + 1) / 2];
#pragma unroll
            for (int i = 0; i < (MR + 1) / 2; i++) acc[i] = 0.0f;
            for (int e = 0; e < hd2; e++) {
                const float2 kf = __half22float2(*reinterpret_cast<const __half2*>(&Ks[key][e]));
#pragma unroll
                for (int i = 0; i < (MR + 1) / 2; i++) {
                    const int rr = rb + 2 * i;
                    if (rr < nr) {
                        const float2 qf = *reinterpret_cast<const float2*>(&q_s[rr][2 * e]);
                        acc[i] = __fmaf_rn(qf.x, kf.x, acc[i]);
                        acc[i] = __fmaf_rn(qf.y, kf.y, acc[i]);
                    }
                }
            }
            const int j = j0 + key;
#pragma unroll
            for (int i = 0; i < (MR + 1) / 2; i++) {
                const int rr = rb + 2 * i;
                if (rr < nr) {
                    bool vis = true;
                    if (j >= base) {
                        const int jj = j - base;
                        vis = p.mask ? (p.mask[(size_t)rr * M + jj] != 0) : (jj <= rr);
                    }
                    sc[rr][key] = vis ? __fmul_rn(acc[i], scale) : -INFINITY;
                }
            }
        } else {
#pragma unroll
            for (int i = 0; i < (MR + 1) / 2; i++) {
                const int rr = rb + 2 * i;
                if (rr < nr && key < kSplit) sc[rr][key] = -INFINITY;
            }
        }
    }
    __syncthreads();
    // local softmax statistics: warp w -> rows w, w + 4
    for (int rr = warp; rr < nr; rr += 4) {
        const float s0 = sc[rr][lane], s1 = sc[rr][lane + 32];
        const float mx = warp_max(fmaxf(s0, s1));
        float e0 = 0.0f, e1 = 0.0f;
        if (mx != -INFINITY) {
            e0 = s0 == -INFINITY ? 0.0f : expf(__fsub_rn(s0, mx));
            e1 = s1 == -INFINITY ? 0.0f : expf(__fsub_rn(s1, mx));
        }
        sc[rr][lane] = e0;
        sc[rr][lane + 32] = e1;
        const float sum = warp_sum(e0 + e1);
        if (lane == 0) {
            ml_s[rr][0] = mx;
            ml_s[rr][1] = sum;
        }
    }
    __syncthreads();
    // unnormalised P.V: thread -> (dimension pair d2, row parity)
    const int pstride = hd + 2;  // per (h, split, row): [max, sum, o[hd]]
    const int hs = sb * p.heads + h;  // (sequence, head) scratch index
    float* part = p.part + (((size_t)hs * gridDim.y + sp) * MR) * pstride;
    if (threadIdx.x < 2 * hd2) {
        const int d2 = threadIdx.x % hd2, rb = threadIdx.x / hd2;
        float a0[(MR + 1) / 2], a1[(MR + 1) / 2];
#pragma unroll
        for (int i = 0; i < (MR + 1) / 2; i++) a0[i] = a1[i] = 0.0f;
        for (int t = 0; t < nt; t++) {
            const float2 v = __half22float2(*reinterpret_cast<const __half2*>(&Vs[t][d2]));
#pragma unroll
            for (int i = 0; i < (MR + 1) / 2; i++) {
                const int rr = rb + 2 * i;
                if (rr < nr) {
                    const float w = sc[rr][t];
                    a0[i] = __fmaf_rn(w, v.x, a0[i]);
                    a1[i] = __fmaf_rn(w, v.y, a1[i]);
                }
            }
        }
#pragma unroll
        for (int i = 0; i < (MR + 1) / 2; i++) {
            const int rr = rb + 2 * i;
            if (rr < nr) {
                part[(size_t)rr * pstride + 2 + 2 * d2] = a0[i];
                part[(size_t)rr * pstride + 2 + 2 * d2 + 1] = a1[i];
            }
        }
    }
    if (threadIdx.x < nr) {
        part[(size_t)threadIdx.x * pstride] = ml_s[threadIdx.x][0];
        part[(size_t)threadIdx.x * pstride + 1] = ml_s[threadIdx.x][1];
    }
    // last CTA of this head combines
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) ticket_s = atomicAdd(&p.counters[hs], 1);
    __syncthreads();
    if (ticket_s != nsplit - 1) return;
    __threadfence();
    const float* ph = p.part + ((size_t)hs * gridDim.y * MR) * pstride;
    for (int i = threadIdx.x; i < nr * hd; i += kDThreads) {
        const int rr = i / hd, dd = i - rr * hd;
        float gm = -INFINITY;
        for (int s = 0; s < nsplit; s++) gm = fmaxf(gm, __ldcg(ph + ((size_t)s * MR + rr) * pstride));
        float L = 0.0f, O = 0.0f;
        for (int s = 0; s < nsplit; s++) {
            const float* q = ph + ((size_t)s * MR + rr) * pstride;
            const float m = __ldcg(q);
            if (m == -INFINITY) continue;
            const float wgt = expf(__fsub_rn(m, gm));
            L = __fmaf_rn(__ldcg(q + 1), wgt, L);
            O = __fmaf_rn(__ldcg(q + 2 + dd), wgt, O);
        }
        const float o = __fdiv_rn(O, L);
        const size_t idx = (qrow0 + rr) * qd + (size_t)h * hd + dd;
        p.out_q[idx] = (uint8_t)quant_u8(o);
        if (p.out_f) p.out_f[idx] = o;
    }
    if (threadIdx.x == 0) p.counters[hs] = 0;  // re-arm for the next launch
}

// Decode attention (M <= 8 new rows) as one thread-block cluster of kCl
// CTAs per (head, sequence). The live context [0, base + M) is cut into kCl
// contiguous key ranges (read from the device at run time, so a graph
// captured once serves every context length); CTA r of the cluster streams
// its range in 32-key tiles (16-byte cp.async copies, two tiles in flight),
// keeps an online softmax per row, and leaves (max, sum, unnormalised P.V)
// in its shared memory. After a cluster barrier every CTA combines a slice
// of the (row, dimension) outputs from all kCl CTAs' shared memory in rank
// order (deterministic), normalises and quantizes. No global scratch, no
// arrival counter, no launch-size dependence on max_ctx. Same arithmetic as
// inference.c:193-247 up to float rounding.
#ifndef FL_ATTN_CL
#define FL_ATTN_CL 8
#endif
// Early K/V prefetch of the cluster attention (below): 0.5 us less per verify
// launch, 0.6 % more tokens per second per decode step on B200.
#ifndef FL_ATTN_PREFETCH
#define FL_ATTN_PREFETCH 1
#endif
constexpr int kCl = FL_ATTN_CL;  // CTAs per head (portable cluster size: at most 8)
constexpr int kCTile = 32;     // keys per tile
constexpr int kCThreads = 128;
// a tile's key is a lane, its rows w, w + 4 belong to warp w in both the
// score and the softmax phase
static_assert(kCTile == 32 && kCThreads == 128, "cluster attention: one key per lane, four warps");
constexpr int kCRes = kMaxHd + 4;  // per row: max, sum, o[hd] (keeps the tile buffers 16-byte aligned)

__device__ __forceinline__ void cp16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)),
                 "l"(src)
                 : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ uint32_t cl_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// Cluster-wide barrier (all threads of all CTAs), release / acquire.
__device__ __forceinline__ void cl_sync() {
    asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}
// Load a float from CTA `rank`'s shared memory at the address of `p` in this CTA.
__device__ __forceinline__ float ld_dsmem(const float* p, uint32_t rank) {
    uint32_t a = (uint32_t)__cvta_generic_to_shared(p), ra;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(a), "r"(rank));
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(ra));
    return v;
}

// Dynamic shared memory of attention_cluster_kernel<MR> for head_dim hd.
__host__ __device__ inline size_t cluster_smem(int MR, int hd) {
    const int hd2 = hd / 2;
    return sizeof(float) * ((size_t)MR * kMaxHd + (size_t)MR * kCTile + (size_t)MR * kCRes) +
           sizeof(uint32_t) * 2 * (size_t)kCTile * ((hd2 + 4) + hd2);
}

template <int MR>
__global__ void __launch_bounds__(kCThreads) attention_cluster_kernel(const AttnParams p) {
    extern __shared__ __align__(16) float csm[];
    __shared__ float m_run[MR], l_run[MR], alpha_s[MR];
    pdl_trigger();
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t rank = cl_rank();
    const int h = blockIdx.x / kCl;
    const int sb = blockIdx.z;  // batched sequence
    const int hd = p.head_dim, hd2 = hd >> 1, hd8 = hd2 >> 2, kst = hd2 + 4;
    const int kvh = kv_head_of(p, h);
    const int qd = p.heads * hd;
    const int* btab = p.block_table + (sb * p.seq_slots) / kPageSize;

    float* q_s = csm;                                 // [MR][kMaxHd]
    float* sc = q_s + MR * kMaxHd;                    // [MR][kCTile]
    float* res = sc + MR * kCTile;                    // [MR][kCRes]
    uint32_t* Ks = reinterpret_cast<uint32_t*>(res + MR * kCRes);  // [2][kCTile][kst] half2
    uint32_t* Vs = Ks + 2 * kCTile * kst;                          // [2][kCTile][hd2] half2
    const uint32_t* kg = reinterpret_cast<const uint32_t*>(p.kv.k);
    const uint32_t* vg = reinterpret_cast<const uint32_t*>(p.kv.v);
    // This CTA's key range [k0, k1) of a live context of ctx slots.
    auto key_range = [&](int ctx, int& k0, int& k1) {
        int chunk = (ctx + kCl - 1) / kCl;
        chunk = (chunk + 15) & ~15;
        k0 = (int)rank * chunk;
        k1 = min(ctx, k0 + chunk);
    };
    auto load_tile_of = [&](int t, int k0, int k1) {
        const int t0 = k0 + t * kCTile;
        const int nt = min(kCTile, k1 - t0);
        uint32_t* Kb = Ks + (t & 1) * kCTile * kst;
        uint32_t* Vb = Vs + (t & 1) * kCTile * hd2;
        for (int i = tid; i < nt * hd8; i += kCThreads) {
            const int key = i / hd8, c = (i - key * hd8) * 4;
            const int slot = t0 + key;
            const size_t off =
                (((size_t)btab[slot / kPageSize] * p.kv_heads + kvh) * kPageSize + (slot % kPageSize)) * hd2 + c;
            cp16(Kb + key * kst + c, kg + off);
            cp16(Vb + key * hd2 + c, vg + off);
        }
        cp_commit();
    };
    bool pre = false;
    int base_e = 0, M_e = 0;
#if FL_ATTN_PREFETCH
    // Before the wait the previous kernel (the QKV projection that writes
    // this pass's new keys) may still run. Keys below the base slot were
    // written by earlier passes, so a first tile made only of them is put in
    // flight now; base and row count are read again after the wait, and if
    // either differs the early tile is drained and loaded again.
    base_e = p.slot_base[sb * p.seq_state];
    M_e = p.dyn_M ? *p.dyn_M : p.M;
    if (M_e > 0 && base_e >= 0) {
        int e0, e1;
        key_range(base_e + M_e, e0, e1);
        if (e1 > e0 && e0 + min(kCTile, e1 - e0) <= base_e) {
            load_tile_of(0, e0, e1);
            pre = true;
        }
    }
#endif
    pdl_wait();
    // Both early exits are uniform over the grid, so no CTA of a cluster
    // is left waiting at the cluster barriers below.
    if (p.done && *p.done) {
        if (pre) cp_wait<0>();
        return;
    }
    // Read again through L2: the values read before the wait may sit in L1
    // from before the launch that wrote them finished.
    const int M = p.dyn_M ? __ldcg(p.dyn_M) : p.M;
    const int nr = min(M, MR);
    if (nr <= 0) {
        if (pre) cp_wait<0>();
        return;
    }
    const int base = __ldcg(p.slot_base + sb * p.seq_state);
    const size_t qrow0 = (size_t)sb * M;
    const int ctx = base + M;
    int k0, k1;
    key_range(ctx, k0, k1);
    const int ntiles = k1 > k0 ? (k1 - k0 + kCTile - 1) / kCTile : 0;
    auto load_tile = [&](int t) { load_tile_of(t, k0, k1); };
    if (pre && (base != base_e || M != M_e)) {
        cp_wait<0>();  // the early copies land before the buffer is written again
        pre = false;
    }
    if (!pre && ntiles > 0) load_tile(0);

    for (int i = tid; i < nr * hd; i += kCThreads) {
        const int rr = i / hd, dd = i - rr * hd;
        q_s[rr * kMaxHd + dd] = p.q[(qrow0 + rr) * qd + (size_t)h * hd + dd];
    }
    if (tid < MR) {
        m_run[tid] = -INFINITY;
        l_run[tid] = 0.0f;
    }
    const float scale = __fdiv_rn(1.0f, sqrtf((float)hd));
    // P.V mapping: thread -> (dimension pair d2, row group g of G)
    const int G = kCThreads / hd2;
    const int d2 = tid % hd2, g = tid / hd2;
    const bool pv = g < G;
    constexpr int kPR = (MR + 1) / 2;  // rows per P.V thread (G >= 2: head_dim <= 128)
    float a0[kPR], a1[kPR];
#pragma unroll
    for (int i = 0; i < kPR; i++) a0[i] = a1[i] = 0.0f;

    for (int t = 0; t < ntiles; t++) {
        if (t + 1 < ntiles) {
            load_tile(t + 1);
            cp_wait<1>();
        } else {
            cp_wait<0>();
        }
        __syncthreads();  // tile t (and, first time round, q_s / m_run) visible
        const int t0 = k0 + t * kCTile;
        const int nt = min(kCTile, k1 - t0);
        const uint32_t* Kb = Ks + (t & 1) * kCTile * kst;
        const uint32_t* Vb = Vs + (t & 1) * kCTile * hd2;
        {   // scores: thread -> key (tid % 32), rows rq, rq + 4, ...
            const int key = tid & (kCTile - 1), rq = tid / kCTile;
            constexpr int kRQ = (MR + 3) / 4;
            if (key < nt) {
                float acc[kRQ];
#pragma unroll
                for (int i = 0; i < kRQ; i++) acc[i] = 0.0f;
                const uint4* kr = reinterpret_cast<const uint4*>(Kb + key * kst);
                for (int e4 = 0; e4 < hd8; e4++) {
                    const uint4 kw = kr[e4];
                    const float2 f0 = __half22float2(*reinterpret_cast<const __half2*>(&kw.x));
                    const float2 f1 = __half22float2(*reinterpret_cast<const __half2*>(&kw.y));
                    const float2 f2 = __half22float2(*reinterpret_cast<const __half2*>(&kw.z));
                    const float2 f3 = __half22float2(*reinterpret_cast<const __half2*>(&kw.w));
#pragma unroll
                    for (int i = 0; i < kRQ; i++) {
                        const int rr = rq + 4 * i;
                        if (rr < nr) {
                            const float4 qa = *reinterpret_cast<const float4*>(&q_s[rr * kMaxHd + 8 * e4]);
                            const float4 qb = *reinterpret_cast<const float4*>(&q_s[rr * kMaxHd + 8 * e4 + 4]);
                            float s = acc[i];
                            s = __fmaf_rn(qa.x, f0.x, s);
                            s = __fmaf_rn(qa.y, f0.y, s);
                            s = __fmaf_rn(qa.z, f1.x, s);
                            s = __fmaf_rn(qa.w, f1.y, s);
                            s = __fmaf_rn(qb.x, f2.x, s);
                            s = __fmaf_rn(qb.y, f2.y, s);
                            s = __fmaf_rn(qb.z, f3.x, s);
                            s = __fmaf_rn(qb.w, f3.y, s);
                            acc[i] = s;
                        }
                    }
                }
                const int j = t0 + key;
#pragma unroll
                for (int i = 0; i < kRQ; i++) {
                    const int rr = rq + 4 * i;
                    if (rr < nr) {
                        bool vis = true;
                        if (j >= base) {
                            const int jj = j - base;
                            vis = p.mask ? (p.mask[(size_t)rr * M + jj] != 0) : (jj <= rr);
                        }
                        sc[rr * kCTile + key] = vis ? __fmul_rn(acc[i], scale) : -INFINITY;
                    }
                }
            } else {
#pragma unroll
                for (int i = 0; i < kRQ; i++) {
                    const int rr = rq + 4 * i;
                    if (rr < nr) sc[rr * kCTile + key] = -INFINITY;
                }
            }
        }
        // the scores of rows w, w + 4 were written by warp w's lanes (key =
        // lane), which are the ones that read them next
        __syncwarp();
        // online softmax: warp w -> rows w, w + 4; lane -> key
        for (int rr = warp; rr < nr; rr += 4) {
            const float s = sc[rr * kCTile + lane];
            const float mx = warp_max(s);
            const float m_old = m_run[rr];
            const float m_new = fmaxf(m_old, mx);
            const float e = (s == -INFINITY) ? 0.0f : expf(__fsub_rn(s, m_new));
            sc[rr * kCTile + lane] = e;
            const float sum = warp_sum(e);
            if (lane == 0) {
                const float al = (m_old == -INFINITY) ? 0.0f : expf(__fsub_rn(m_old, m_new));
                alpha_s[rr] = al;
                l_run[rr] = __fmaf_rn(l_run[rr], al, sum);
                m_run[rr] = m_new;
            }
        }
        __syncthreads();
        if (pv) {
#pragma unroll
            for (int i = 0; i < kPR; i++) {
                const int rr = g + G * i;
                if (rr < nr) {
                    a0[i] *= alpha_s[rr];
                    a1[i] *= alpha_s[rr];
                }
            }
            for (int tt = 0; tt < nt; tt++) {
                const float2 v = __half22float2(*reinterpret_cast<const __half2*>(&Vb[tt * hd2 + d2]));
#pragma unroll
                for (int i = 0; i < kPR; i++) {
                    const int rr = g + G * i;
                    if (rr < nr) {
                        const float w = sc[rr * kCTile + tt];
                        a0[i] = __fmaf_rn(w, v.x, a0[i]);
                        a1[i] = __fmaf_rn(w, v.y, a1[i]);
                    }
                }
            }
        }
        // this tile's buffers and scores are free again before the next tile;
        // after the last one the partials go to `res`, which nothing here reads
        if (t + 1 < ntiles) __syncthreads();
    }
    // this CTA's partial result
    if (pv) {
#pragma unroll
        for (int i = 0; i < kPR; i++) {
            const int rr = g + G * i;
            if (rr < nr) {
                res[rr * kCRes + 2 + 2 * d2] = a0[i];
                res[rr * kCRes + 3 + 2 * d2] = a1[i];
            }
        }
    }
    if (tid < nr) {
        res[tid * kCRes] = m_run[tid];
        res[tid * kCRes + 1] = l_run[tid];
    }
    cl_sync();
    // combine: element i of [nr][hd] is handled by CTA i / kCThreads % kCl
    for (int i = (int)rank * kCThreads + tid; i < nr * hd; i += kCl * kCThreads) {
        const int rr = i / hd, dd = i - rr * hd;
        // all remote loads issued before any is used: two round trips
        float mv[kCl], lv[kCl], ov[kCl];
#pragma unroll
        for (int c = 0; c < kCl; c++) {
            mv[c] = ld_dsmem(&res[rr * kCRes], (uint32_t)c);
            lv[c] = ld_dsmem(&res[rr * kCRes + 1], (uint32_t)c);
            ov[c] = ld_dsmem(&res[rr * kCRes + 2 + dd], (uint32_t)c);
        }
        float gm = -INFINITY;
#pragma unroll
        for (int c = 0; c < kCl; c++) gm = fmaxf(gm, mv[c]);
        float L = 0.0f, O = 0.0f;
#pragma unroll
        for (int c = 0; c < kCl; c++) {
            if (mv[c] == -INFINITY) continue;
            const float wgt = expf(__fsub_rn(mv[c], gm));
            L = __fmaf_rn(lv[c], wgt, L);
            O = __fmaf_rn(ov[c], wgt, O);
        }
        const float o = __fdiv_rn(O, L);
        const size_t idx = (qrow0 + rr) * qd + (size_t)h * hd + dd;
        p.out_q[idx] = (uint8_t)quant_u8(o);
        if (p.out_f) p.out_f[idx] = o;
    }
    cl_sync();  // no CTA leaves while another still reads its shared memory
}

size_t attention_smem() {
    const size_t f = (size_t)kARows * kMaxHd + (size_t)kARows * kTile;
    const size_t kv = (size_t)kTile * (kMaxHd / 2 + 1) + (size_t)kTile * (kMaxHd / 2);
    const size_t red = (size_t)(kAThreads / 32) * kARows * kMaxHd;  // G <= kAThreads / (hd/2), hd >= 64
    return sizeof(float) * (f + red) + sizeof(uint32_t) * kv;
}

}  // namespace

cudaError_t launch_act_quant(const ActQuantParams& p, cudaStream_t s, bool pdl) {
    if (p.K % 4 != 0 || p.M <= 0) return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.M);
    cfg.blockDim = dim3(kQThreads);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, act_quant_kernel, p);
}

size_t attention_scratch_floats(int heads, int head_dim, int max_ctx) {
    return (size_t)heads * ((max_ctx + kSplit - 1) / kSplit) * kMaxRows * (head_dim + 2);
}
size_t attention_scratch_counters(int heads) { return (size_t)heads; }

template <int MR>
cudaError_t launch_split(const AttnParams& p, cudaStream_t s, bool pdl) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.heads, (p.max_ctx + kSplit - 1) / kSplit, p.seqs > 1 ? p.seqs : 1);
    cfg.blockDim = dim3(kDThreads);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, attention_split_kernel<MR>, p);
}

template <int MR>
cudaError_t launch_cluster(const AttnParams& p, cudaStream_t s, bool pdl) {
    auto kern = attention_cluster_kernel<MR>;
    const size_t smem = cluster_smem(MR, p.head_dim);
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.heads * kCl, 1, p.seqs > 1 ? p.seqs : 1);
    cfg.blockDim = dim3(kCThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = kCl;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 2 : 1;
    return cudaLaunchKernelEx(&cfg, kern, p);
}

#ifndef FL_ATTN_CLUSTER
#define FL_ATTN_CLUSTER 1
#endif
// Contexts up to this many slots take the cluster kernel (each CTA streams
// at most a 256-key range); longer ones the page-split kernel.
constexpr int kClusterMaxCtx = 2048;

cudaError_t launch_attention(const AttnParams& p, cudaStream_t s, bool pdl) {
    if (p.head_dim > kMaxHd || p.head_dim < 64 || p.head_dim % 2 != 0 || (p.group <= 0 && p.heads % p.kv_heads != 0))
        return cudaErrorInvalidValue;
    // batched sequences: static rows, page-aligned regions, grid z <= 65535
    if (p.seqs > 1 && (p.dyn_M || p.seq_slots % kPageSize != 0 || p.seqs > 65535)) return cudaErrorInvalidValue;
    if (FL_ATTN_CLUSTER && p.M <= kMaxRows && p.head_dim % 8 == 0 && p.max_ctx <= kClusterMaxCtx) {
        if (p.M <= 1) return launch_cluster<1>(p, s, pdl);
        if (p.M <= 2) return launch_cluster<2>(p, s, pdl);
        if (p.M <= 4) return launch_cluster<4>(p, s, pdl);
        return launch_cluster<8>(p, s, pdl);
    }
    if (p.M <= kMaxRows && p.part && p.counters) {
        // grid.y covers every page the context can reach; the partial layout
        // indexes (head, split) with gridDim.y, so max_ctx must be the one the
        // scratch was sized for.
        if (p.M <= 1) return launch_split<1>(p, s, pdl);
        if (p.M <= 2) return launch_split<2>(p, s, pdl);
        if (p.M <= 4) return launch_split<4>(p, s, pdl);
        return launch_split<8>(p, s, pdl);
    }
    const size_t smem = attention_smem();
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)smem);
        if (e != cudaSuccess) return e;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.heads, (p.M + kARows - 1) / kARows, p.seqs > 1 ? p.seqs : 1);
    cfg.blockDim = dim3(kAThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, attention_kernel, p);
}

}  // namespace fl
