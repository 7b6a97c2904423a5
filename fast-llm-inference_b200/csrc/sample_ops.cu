// Stochastic speculative decoding kernels (sm_100a): nucleus weights,
// Philox-keyed inverse-CDF draws and rejection-sampling acceptance. The rule
// (temperature > 0) is stated in include/speculative.h; the reference declares
// the contract (fast_llm/include/speculative.h:121-185) without an algorithm.
//
// The rule works on integer weights so that every sum is exact and the result
// does not depend on the reduction order: E_i = trunc(e^x * 2^24) of
// x = (l_i - max) / T (0 below x = -17), e^x evaluated by a fixed sequence of
// correctly rounded operations (Cody-Waite reduction by ln 2, degree-7 Taylor
// polynomial in Horner form, exact scale by 2^(k + 24)). The nucleus keeps
// {E_i >= t*}, t* the largest integer with S(t) * 2^24 >= P * z
// (S(t) = sum_{E_i >= t} E_i, z = S(1), P = max(1, trunc(top_p * 2^24))).
// Draws pick the first index whose running weight sum exceeds
// trunc(U * total / 2^24), U = the top 24 bits of word 0 of Philox4x32-10
// (Salmon et al., SC'11) keyed by (seed, 0) at counter (sequence, step,
// position, purpose): purpose 0 = draft sample, 1 = acceptance test,
// 2 = resample / bonus. Acceptance: U * Mp * Eq(x) < 2^24 * Ep(x) * Mq.
// Residual weights: max(0, Ep_i * Mq - Eq_i * Mp) / 2^24, truncated.
//
// One CTA of 1024 threads per distribution row; for vocabularies up to 32768
// each thread keeps its weights in registers through the 24 bisection passes.
#include <float.h>
#include <limits.h>

#include "fl_common.cuh"
#include "fl_state.h"

namespace fl {

namespace {

typedef unsigned __int128 u128;

constexpr int kST = 1024;      // threads per row CTA
constexpr int kSW = kST / 32;  // warps
constexpr int kRegPT = 32;     // register-resident weights per thread
constexpr uint32_t kOne = 1u << 24;

__device__ uint32_t philox_u24(uint32_t seed, uint32_t seq, uint32_t step, uint32_t pos, uint32_t purpose) {
    uint32_t c0 = seq, c1 = step, c2 = pos, c3 = purpose;
    uint32_t k0 = seed, k1 = 0u;
#pragma unroll
    for (int r = 0; r < 10; r++) {
        const uint32_t hi0 = __umulhi(0xD2511F53u, c0), lo0 = 0xD2511F53u * c0;
        const uint32_t hi1 = __umulhi(0xCD9E8D57u, c2), lo1 = 0xCD9E8D57u * c2;
        c0 = hi1 ^ c1 ^ k0;
        c1 = lo1;
        c2 = hi0 ^ c3 ^ k1;
        c3 = lo0;
        k0 += 0x9E3779B9u;
        k1 += 0xBB67AE85u;
    }
    return c0 >> 8;
}

// E = trunc(e^x * 2^24) for x <= 0 (see the file comment).
__device__ __forceinline__ uint32_t sample_weight(float x) {
    if (!(x >= -17.0f)) return 0u;
    const float kf = rintf(__fmul_rn(x, 1.442695f));
    float r = __fmaf_rn(-kf, 0.693145751953125f, x);
    r = __fmaf_rn(-kf, 1.4286068e-06f, r);
    float p = 0.0001984127f;
    p = __fmaf_rn(p, r, 0.0013888889f);
    p = __fmaf_rn(p, r, 0.008333334f);
    p = __fmaf_rn(p, r, 0.041666668f);
    p = __fmaf_rn(p, r, 0.16666667f);
    p = __fmaf_rn(p, r, 0.5f);
    p = __fmaf_rn(p, r, 1.0f);
    p = __fmaf_rn(p, r, 1.0f);
    const int e = 127 + 24 + (int)kf;  // 2^(k + 24), k in [-25, 0]: a normal float
    const uint32_t E = __float2uint_rz(__fmul_rn(p, __int_as_float(e << 23)));
    return E > kOne ? kOne : E;
}

// Block-wide exact sum / float max; every thread gets the result.
__device__ __forceinline__ unsigned long long bsum64(unsigned long long v, unsigned long long* red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    unsigned long long t = red[threadIdx.x & 31];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    return t;
}
__device__ __forceinline__ float bmax(float v, unsigned long long* red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    __syncthreads();
    float* rf = reinterpret_cast<float*>(red);
    if ((threadIdx.x & 31) == 0) rf[threadIdx.x >> 5] = v;
    __syncthreads();
    float t = rf[threadIdx.x & 31];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t = fmaxf(t, __shfl_xor_sync(0xffffffffu, t, o));
    return t;
}

// Nucleus weights of logits row l into E (0 outside); returns the kept mass.
template <bool REG>
__device__ unsigned long long nucleus_impl(const float* __restrict__ l, int V, float T, float top_p,
                                           uint32_t* __restrict__ E, unsigned long long* red) {
    uint32_t w[REG ? kRegPT : 1];
    float mx = -FLT_MAX;
    if constexpr (REG) {
#pragma unroll
        for (int k = 0; k < kRegPT; k++) {
            const int i = threadIdx.x + k * kST;
            if (i < V) mx = fmaxf(mx, l[i]);
        }
    } else {
        for (int i = threadIdx.x; i < V; i += kST) mx = fmaxf(mx, l[i]);
    }
    mx = bmax(mx, red);
    unsigned long long s = 0;
    if constexpr (REG) {
#pragma unroll
        for (int k = 0; k < kRegPT; k++) {
            const int i = threadIdx.x + k * kST;
            w[k] = i < V ? sample_weight(__fdiv_rn(__fsub_rn(l[i], mx), T)) : 0u;
            s += w[k];
        }
    } else {
        for (int i = threadIdx.x; i < V; i += kST) {
            const uint32_t e = sample_weight(__fdiv_rn(__fsub_rn(l[i], mx), T));
            E[i] = e;
            s += e;
        }
    }
    const unsigned long long z = bsum64(s, red);
    uint32_t P = __float2uint_rz(__fmul_rn(top_p, 16777216.0f));
    if (P < 1u) P = 1u;
    const u128 need = (u128)P * z;
    uint32_t lo = 1u, hi = kOne + 1u;
    while (hi - lo > 1u) {
        const uint32_t mid = lo + (hi - lo) / 2u;
        unsigned long long m = 0;
        if constexpr (REG) {
#pragma unroll
            for (int k = 0; k < kRegPT; k++) m += w[k] >= mid ? w[k] : 0u;
        } else {
            for (int i = threadIdx.x; i < V; i += kST) {
                const uint32_t e = E[i];
                m += e >= mid ? e : 0u;
            }
        }
        if (((u128)bsum64(m, red) << 24) >= need) lo = mid; else hi = mid;
    }
    unsigned long long m = 0;
    if constexpr (REG) {
#pragma unroll
        for (int k = 0; k < kRegPT; k++) {
            const int i = threadIdx.x + k * kST;
            const uint32_t e = w[k] >= lo ? w[k] : 0u;
            if (i < V) E[i] = e;
            m += e;
        }
    } else {
        for (int i = threadIdx.x; i < V; i += kST) {
            const uint32_t e = E[i] >= lo ? E[i] : 0u;
            E[i] = e;
            m += e;
        }
    }
    const unsigned long long M = bsum64(m, red);
    __syncthreads();
    return M;
}

__device__ __noinline__ unsigned long long nucleus(const float* l, int V, float T, float top_p, uint32_t* E,
                                                   unsigned long long* red) {
    return V <= kST * kRegPT ? nucleus_impl<true>(l, V, T, top_p, E, red) : nucleus_impl<false>(l, V, T, top_p, E, red);
}

// Inverse CDF over integer weights w (token order) at U: the first index whose
// running sum exceeds trunc(U * total / 2^24); V - 1 if none. Thread t owns
// the contiguous chunk [t*C, t*C + C); exact chunk prefixes come from a block
// scan, each thread walks its chunk and the smallest crossing index wins.
template <typename W>
__device__ __noinline__ int draw(const W* __restrict__ w, int V, unsigned long long total, uint32_t U) {
    __shared__ unsigned long long wsum[kSW];
    __shared__ int pick_s;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int C = (V + kST - 1) / kST;
    const int b0 = min(V, (int)threadIdx.x * C), b1 = min(V, b0 + C);
    unsigned long long local = 0;
    for (int i = b0; i < b1; i++) local += w[i];
    unsigned long long inc = local;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const unsigned long long y = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += y;
    }
    __syncthreads();
    if (threadIdx.x == 0) pick_s = INT_MAX;
    if (lane == 31) wsum[warp] = inc;
    __syncthreads();
    unsigned long long wpre = wsum[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const unsigned long long y = __shfl_up_sync(0xffffffffu, wpre, o);
        if (lane >= o) wpre += y;
    }
    const unsigned long long wbase = __shfl_sync(0xffffffffu, wpre, (warp + 31) & 31);
    unsigned long long c = (warp == 0 ? 0ull : wbase) + (inc - local);
    const unsigned long long tgt = (unsigned long long)(((u128)U * total) >> 24);
    if (c + local > tgt) {
        for (int i = b0; i < b1; i++) {
            c += w[i];
            if (c > tgt) {
                atomicMin(&pick_s, i);
                break;
            }
        }
    }
    __syncthreads();
    const int p = pick_s == INT_MAX ? V - 1 : pick_s;
    __syncthreads();
    return p;
}

__device__ __forceinline__ void trace_row(const StepBuffers& b, int row, const float* l) {
    if (!b.trace) return;
    float* t = b.trace + (size_t)row * b.V;
    for (int i = threadIdx.x; i < b.V; i += kST) t[i] = l[i];
}

__global__ void __launch_bounds__(kST) sample_first_kernel(const StepBuffers b0, int P, int s0) {
    __shared__ unsigned long long red[kSW];
    const StepBuffers b = seq_view(b0, s0 + blockIdx.x);
    trace_row(b, 2 * kMaxRows - 1, b.logits_d);
    const unsigned long long M = nucleus(b.logits_d, b.V, b.temp, b.top_p, b.pt, red);
    const int t = draw(b.pt, b.V, M, philox_u24(b.key[0], b.key[1], 0xFFFFFFFFu, (uint32_t)P, 2u));
    if (threadIdx.x == 0) b.seq[P] = t;
}

// Sampled draft token j from the draft LM-head logits (row 0; batched: row
// s); its weights and mass are kept for the acceptance test. The rest as the
// greedy pick.
__global__ void __launch_bounds__(kST) sample_pick_kernel(const StepBuffers b0, int j) {
    __shared__ unsigned long long red[kSW];
    pdl_trigger();
    pdl_wait();
    const StepBuffers b = seq_view(b0, blockIdx.x);
    SpecState* st = b.st;
    if (st->done) return;
    const int n = st->n;
    uint32_t* q = b.qd + (size_t)j * b.V;
    trace_row(b, j, b.logits_d);
    const unsigned long long M = nucleus(b.logits_d, b.V, b.temp, b.top_p, q, red);
    const int tok = draw(q, b.V, M, philox_u24(b.key[0], b.key[1], (uint32_t)st->steps, (uint32_t)(n + 1 + j), 0u));
    if (j + 1 < st->K) {
        const int g_row = (j == 0 && !b.batch) ? st->last_row : 0;
        const float* g = b.x_d1 + (size_t)g_row * b.d;
        const float* e = b.embed + (size_t)tok * b.d;
        // g_row may be 0: element-wise in place is safe.
        for (int i = threadIdx.x; i < b.d; i += blockDim.x) b.x_d1[i] = __fadd_rn(g[i], e[i]);
    }
    if (threadIdx.x == 0) {
        b.qm[j] = M;
        st->drafted[j] = tok;
        if (j + 1 < st->K) {
            st->draft_base = n + j + 1;
            st->draft_pos[0] = n + j + 1;
        }
    }
}

// Target weights of the K + 1 verify rows (one CTA per row).
__global__ void __launch_bounds__(kST) target_dist_kernel(const StepBuffers b0) {
    __shared__ unsigned long long red[kSW];
    pdl_trigger();
    pdl_wait();
    const StepBuffers b = seq_view(b0, blockIdx.y);
    if (b.st->done) return;
    const int r = blockIdx.x;
    trace_row(b, kMaxDraft + r, b.logits + (size_t)r * b.V);
    const unsigned long long M =
        nucleus(b.logits + (size_t)r * b.V, b.V, b.temp, b.top_p, b.pt + (size_t)r * b.V, red);
    if (threadIdx.x == 0) b.pm[r] = M;
}

// Rejection sampling over the drafted tokens (accept x with probability
// min(1, p(x) / q(x)); on rejection draw from the residual max(0, p - q), or
// from p when it is empty; all accepted: bonus from p_K), then the same state
// update as the greedy acceptance.
__global__ void __launch_bounds__(kST) accept_sampled_kernel(const StepBuffers b0, int K) {
    __shared__ unsigned long long red[kSW];
    pdl_trigger();
    pdl_wait();
    const StepBuffers b = seq_view(b0, blockIdx.x);
    SpecState* st = b.st;
    if (st->done) return;
    const int n = st->n;
    const int cap = min(K, st->max_acc);
    const uint32_t step = (uint32_t)st->steps;
    int a = 0, last = 0;
    for (;;) {
        const uint32_t pos = (uint32_t)(n + 1 + a);
        const uint32_t* p = b.pt + (size_t)a * b.V;
        const unsigned long long Mp = b.pm[a];
        if (a == cap) {
            last = draw(p, b.V, Mp, philox_u24(b.key[0], b.key[1], step, pos, 2u));
            break;
        }
        const int x = st->drafted[a];
        const uint32_t* q = b.qd + (size_t)a * b.V;
        const unsigned long long Mq = b.qm[a];
        const uint32_t U = philox_u24(b.key[0], b.key[1], step, pos, 1u);
        if ((u128)U * Mp * q[x] < (((u128)p[x] * Mq) << 24)) {
            a++;
            continue;
        }
        unsigned long long s = 0;
        for (int i = threadIdx.x; i < b.V; i += kST) {
            const u128 hp = (u128)p[i] * Mq, hq = (u128)q[i] * Mp;
            const unsigned long long y = hp > hq ? (unsigned long long)((hp - hq) >> 24) : 0ull;
            b.resid[i] = y;
            s += y;
        }
        const unsigned long long zr = bsum64(s, red);
        const uint32_t Ur = philox_u24(b.key[0], b.key[1], step, pos, 2u);
        last = zr > 0 ? draw(b.resid, b.V, zr, Ur) : draw(p, b.V, Mp, Ur);
        break;
    }
    if (threadIdx.x != 0) return;
    int produced = st->produced;
    for (int j = 0; j <= a; j++) {
        const int t = j < a ? st->drafted[j] : last;
        b.seq[n + 1 + j] = t;
        if (produced < st->n_new) b.out[produced++] = t;
    }
    b.acc_hist[st->steps] = a;
    st->steps += 1;
    st->produced = produced;
    st->a_last = a;
    st->n = n + a + 1;
    st->rows = a + 1;
    st->last_row = a;
    st->draft_base = n + 1;
    for (int r = 0; r <= K; r++) st->draft_pos[r] = n + 1 + r;
    st->done = produced >= st->n_new ? 1 : 0;
    batch_retire(b, st->done);
}

template <typename... KArgs, typename... Args>
cudaError_t launch_rows(void (*kern)(KArgs...), dim3 grid, cudaStream_t s, bool pdl, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(kST);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, args...);
}

}  // namespace

cudaError_t launch_sample_first(const StepBuffers& b, int P, cudaStream_t s, int seq) {
    return launch_rows(sample_first_kernel, dim3(1), s, false, b, P, seq);
}
cudaError_t launch_sample_pick(const StepBuffers& b, int j, cudaStream_t s, bool pdl) {
    return launch_rows(sample_pick_kernel, dim3(step_seqs(b)), s, pdl, b, j);
}
cudaError_t launch_target_dist(const StepBuffers& b, int K, cudaStream_t s, bool pdl) {
    return launch_rows(target_dist_kernel, dim3(K + 1, step_seqs(b)), s, pdl, b);
}
cudaError_t launch_accept_sampled(const StepBuffers& b, int K, cudaStream_t s, bool pdl) {
    return launch_rows(accept_sampled_kernel, dim3(step_seqs(b)), s, pdl, b, K);
}

}  // namespace fl
