// Medusa kernels (sm_100a): the heads' residual block, per-head top-k with
// softmax probabilities, and in-place KV compaction of an accepted tree path.
// The rule is include/medusa.h's; the reference declares the API
// (fast_llm/include/medusa.h:84-229) without an implementation.
#include <float.h>

#include "fl_common.cuh"
#include "fl_kernels.h"
#include "fl_state.h"

namespace fl {

namespace {

constexpr int kNT = 256;

// Block sum of one value per thread: warp butterflies, then the warp sums in
// warp order (deterministic).
__device__ float block_sum(float v, float* red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float t = red[0];
    for (int w = 1; w < (int)(blockDim.x >> 5); w++) t += red[w];
    return t;
}

// h = RMSNorm(x) (unit weights, activations_avx2.c:108-143), z_i = h + SiLU(y_i)
// with the reference's polynomial sigmoid (activations_avx2.c:33-63), for the
// H head rows of y [H, d]. One CTA.
__global__ void medusa_z_kernel(const float* x, const float* y, float* h_out, float* z, int d, int H, float eps) {
    __shared__ float red[kNT / 32];
    float s = 0.0f;
    for (int i = threadIdx.x; i < d; i += blockDim.x) s = __fmaf_rn(x[i], x[i], s);
    const float tot = block_sum(s, red);
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)d), eps)));
    for (int i = threadIdx.x; i < d; i += blockDim.x) {
        const float h = __fmul_rn(x[i], scale);
        if (h_out) h_out[i] = h;
        for (int k = 0; k < H; k++) {
            const float v = y[(size_t)k * d + i];
            z[(size_t)k * d + i] = __fadd_rn(h, __fmul_rn(v, poly_sigmoid(v)));
        }
    }
}

// Top-k of each logits row (value desc, lower index first on ties) and its
// softmax probability exp(l - max) / sum_j exp(l_j - max). One CTA per row.
__global__ void topk_rows_kernel(const float* logits, int V, int ld, const int* kk, int kmax, int* tok, float* prob) {
    __shared__ float redf[kNT / 32];
    __shared__ unsigned long long redk[kNT / 32];
    __shared__ int taken[32];
    const int row = blockIdx.x;
    const float* lg = logits + (size_t)row * ld;
    const int k = kk[row] < kmax ? kk[row] : kmax;
    // max
    float mx = -FLT_MAX;
    for (int i = threadIdx.x; i < V; i += blockDim.x) mx = fmaxf(mx, lg[i]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if ((threadIdx.x & 31) == 0) redf[threadIdx.x >> 5] = mx;
    __syncthreads();
    mx = redf[0];
    for (int w = 1; w < (int)(blockDim.x >> 5); w++) mx = fmaxf(mx, redf[w]);
    __syncthreads();
    float s = 0.0f;
    for (int i = threadIdx.x; i < V; i += blockDim.x) s = __fadd_rn(s, expf(__fsub_rn(lg[i], mx)));
    const float sum = block_sum(s, redf);
    for (int j = 0; j < k; j++) {
        unsigned long long best = 0ull;
        for (int i = threadIdx.x; i < V; i += blockDim.x) {
            bool used = false;
            for (int q = 0; q < j; q++) used |= taken[q] == i;
            if (!used) {
                const unsigned long long key = argmax_key(lg[i], i);
                best = key > best ? key : best;
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const unsigned long long o2 = __shfl_xor_sync(0xffffffffu, best, o);
            best = o2 > best ? o2 : best;
        }
        __syncthreads();
        if ((threadIdx.x & 31) == 0) redk[threadIdx.x >> 5] = best;
        __syncthreads();
        if (threadIdx.x == 0) {
            unsigned long long b = redk[0];
            for (int w = 1; w < (int)(blockDim.x >> 5); w++) b = redk[w] > b ? redk[w] : b;
            const int id = argmax_key_index(b);
            taken[j] = id;
            tok[(size_t)row * kmax + j] = id;
            prob[(size_t)row * kmax + j] = __fdiv_rn(expf(__fsub_rn(lg[id], mx)), sum);
        }
        __syncthreads();
    }
}

// Top-w keys (value, global index v0 + i; argmax_key order: larger value
// first, lower index on ties) of rows logits[row * ld ..] of V entries; best
// first into out[row * w ..]. One CTA per row.
__global__ void topk_keys_kernel(const float* logits, int V, int ld, int v0, int w, unsigned long long* out) {
    __shared__ unsigned long long redk[kNT / 32];
    __shared__ int taken[32];
    const int row = blockIdx.x;
    const float* lg = logits + (size_t)row * ld;
    for (int j = 0; j < w; j++) {
        unsigned long long best = 0ull;
        for (int i = threadIdx.x; i < V; i += blockDim.x) {
            bool used = false;
            for (int q = 0; q < j; q++) used |= taken[q] == i;
            if (!used) {
                const unsigned long long key = argmax_key(lg[i], v0 + i);
                best = key > best ? key : best;
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const unsigned long long o2 = __shfl_xor_sync(0xffffffffu, best, o);
            best = o2 > best ? o2 : best;
        }
        __syncthreads();
        if ((threadIdx.x & 31) == 0) redk[threadIdx.x >> 5] = best;
        __syncthreads();
        if (threadIdx.x == 0) {
            unsigned long long b = redk[0];
            for (int q = 1; q < (int)(blockDim.x >> 5); q++) b = redk[q] > b ? redk[q] : b;
            taken[j] = argmax_key_index(b) - v0;
            out[(size_t)row * w + j] = b;
        }
        __syncthreads();
    }
}

// Accepted path compaction: for j = 1 .. a in order, slot base + j takes the
// K / V of slot base + src[j] (src[j] >= j, src increasing, so an earlier move
// never overwrites a later source). CTA = (layer, stack of kv heads).
__global__ void kv_compact_kernel(const KvLayer* layers, const int* block_table, int kv_heads, int head_dim,
                                  const int* base_p, const int* src, int a, const int* a_dev) {
    const KvLayer L = layers[blockIdx.x];
    const int base = *base_p;
    if (a_dev) a = *a_dev;
    const int hd2 = head_dim >> 1;
    for (int j = 1; j <= a; j++) {
        const int s_slot = base + src[j], d_slot = base + j;
        if (s_slot != d_slot) {
            const int sp = block_table[s_slot / kPageSize], so = s_slot % kPageSize;
            const int dp = block_table[d_slot / kPageSize], dof = d_slot % kPageSize;
            for (int i = threadIdx.x; i < kv_heads * hd2; i += blockDim.x) {
                const int h = i / hd2, c = i - h * hd2;
                const size_t si = (((size_t)sp * kv_heads + h) * kPageSize + so) * hd2 + c;
                const size_t di = (((size_t)dp * kv_heads + h) * kPageSize + dof) * hd2 + c;
                reinterpret_cast<uint32_t*>(L.k)[di] = reinterpret_cast<const uint32_t*>(L.k)[si];
                reinterpret_cast<uint32_t*>(L.v)[di] = reinterpret_cast<const uint32_t*>(L.v)[si];
            }
        }
        __syncthreads();
    }
}

constexpr int kTreeThreads = 1024;

// Candidate tree (the rule of engine.cu build_tree and of the oracle's
// orc_medusa_tree): one thread per candidate computes its path score in the
// same left-to-right product order, its rank under the total order (score
// desc, depth asc, generation asc) by counting the candidates before it, and
// the kept ones (rank < max_nodes - 1) become node rank + 1. A kept
// candidate's parent ranks before it (its score is at least the child's and
// its depth smaller), so it is kept too.
__global__ void __launch_bounds__(kTreeThreads) medusa_tree_kernel(const MedusaTreeParams p) {
    __shared__ float sc[kMaxTreeCand];
    __shared__ int dep[kMaxTreeCand], par[kMaxTreeCand], tk[kMaxTreeCand], rk[kMaxTreeCand];
    __shared__ int spar[256];
    __shared__ int lstart[kMaxRows + 1], ltopk[kMaxRows];
    __shared__ int total_s;
    const int t = threadIdx.x;
    if (t == 0) {
        int width = 1, tot = 0;
        for (int h = 0; h < p.H; h++) {
            ltopk[h] = min(max(p.topk[h], 0), p.kmax);
            lstart[h] = tot;
            width *= ltopk[h];
            if (tot + width > kMaxTreeCand) width = kMaxTreeCand - tot;  // bounded (the host checks the count)
            tot += width;
        }
        lstart[p.H] = tot;
        total_s = tot;
    }
    __syncthreads();
    const int C = total_s;
    for (int i = t; i < C; i += kTreeThreads) {
        int h = 0;
        while (i >= lstart[h + 1]) h++;
        // per-level choice indices of the path, from this level up
        int ks[kMaxRows];
        int j = i - lstart[h];
        for (int l = h; l >= 0; l--) {
            ks[l] = ltopk[l] > 0 ? j % ltopk[l] : 0;
            j = ltopk[l] > 0 ? j / ltopk[l] : 0;
        }
        float s = p.prob[ks[0]];
        for (int l = 1; l <= h; l++) s = __fmul_rn(s, p.prob[l * p.kmax + ks[l]]);
        sc[i] = s;
        dep[i] = h + 1;
        tk[i] = p.tok[h * p.kmax + ks[h]];
        par[i] = h == 0 ? -1 : lstart[h - 1] + (i - lstart[h]) / ltopk[h];
    }
    __syncthreads();
    for (int i = t; i < C; i += kTreeThreads) {
        const float si = sc[i];
        const int di = dep[i];
        int r = 0;
        for (int j = 0; j < C; j++) {
            const float sj = sc[j];
            r += (sj > si || (sj == si && (dep[j] < di || (dep[j] == di && j < i)))) ? 1 : 0;
        }
        rk[i] = r;
    }
    __syncthreads();
    const int keep = min(p.max_nodes - 1, C);
    const int M = keep + 1;
    if (t == 0) {
        p.ntok[0] = *p.root;
        p.npar[0] = -1;
        p.ndep[0] = 0;
        p.pos[0] = p.n;
        spar[0] = -1;
    }
    for (int i = t; i < C; i += kTreeThreads) {
        const int r = rk[i];
        if (r < keep) {
            const int node = r + 1;
            const int pn = par[i] < 0 ? 0 : rk[par[i]] + 1;
            p.ntok[node] = tk[i];
            p.npar[node] = pn;
            p.ndep[node] = dep[i];
            p.pos[node] = p.n + dep[i];
            spar[node] = pn;
        }
    }
    __syncthreads();
    for (int i = t; i < M; i += kTreeThreads) {
        uint8_t* row = p.mask + (size_t)i * M;
        for (int j = 0; j < M; j++) row[j] = 0;
        for (int j = i, g = 0; j >= 0 && g <= kMaxRows; j = spar[j], g++) row[j] = 1;
    }
}

// Accepted path of a verified tree; thread 0 walks, then the CTA copies the
// last node's feature row.
__global__ void medusa_walk_kernel(const MedusaWalkParams p) {
    __shared__ int last_s;
    if (threadIdx.x == 0) {
        int cur = 0, a = 0;
        p.path[0] = 0;
        for (;;) {
            int nxt = -1;
            for (int c = 1; c < p.M; c++)
                if (p.npar[c] == cur && p.ntok[c] == p.target[cur]) {
                    nxt = c;
                    break;
                }
            if (nxt < 0) break;
            p.path[++a] = nxt;
            p.rec[1 + a] = p.ntok[nxt];
            cur = nxt;
        }
        p.rec[0] = a;
        p.rec[1] = cur;
        p.rec[2 + a] = p.target[cur];
        *p.root = p.target[cur];
        last_s = cur;
    }
    __syncthreads();
    const float* src = p.x + (size_t)last_s * p.d;
    for (int i = threadIdx.x; i < p.d; i += blockDim.x) p.f[i] = src[i];
}

}  // namespace

cudaError_t launch_medusa_z(const float* x, const float* y, float* h, float* z, int d, int H, float eps,
                            cudaStream_t s) {
    medusa_z_kernel<<<1, kNT, 0, s>>>(x, y, h, z, d, H, eps);
    return cudaGetLastError();
}

cudaError_t launch_topk_rows(const float* logits, int rows, int V, int ld, const int* k, int kmax, int* tok,
                             float* prob, cudaStream_t s) {
    if (kmax > 32) return cudaErrorInvalidValue;
    topk_rows_kernel<<<rows, kNT, 0, s>>>(logits, V, ld, k, kmax, tok, prob);
    return cudaGetLastError();
}

cudaError_t launch_topk_keys(const float* logits, int rows, int V, int ld, int v0, int w, unsigned long long* out,
                             cudaStream_t s) {
    if (w < 1 || w > 32 || w > V) return cudaErrorInvalidValue;
    topk_keys_kernel<<<rows, kNT, 0, s>>>(logits, V, ld, v0, w, out);
    return cudaGetLastError();
}

cudaError_t launch_kv_compact(const KvLayer* layers, int n_layers, const int* block_table, int kv_heads, int head_dim,
                              const int* base, const int* src, int a, cudaStream_t s) {
    if (a <= 0) return cudaSuccess;
    kv_compact_kernel<<<n_layers, kNT, 0, s>>>(layers, block_table, kv_heads, head_dim, base, src, a, nullptr);
    return cudaGetLastError();
}

cudaError_t launch_kv_compact_dev(const KvLayer* layers, int n_layers, const int* block_table, int kv_heads,
                                  int head_dim, const int* base, const int* src, const int* a_dev, cudaStream_t s) {
    kv_compact_kernel<<<n_layers, kNT, 0, s>>>(layers, block_table, kv_heads, head_dim, base, src, 0, a_dev);
    return cudaGetLastError();
}

cudaError_t launch_medusa_tree(const MedusaTreeParams& p, cudaStream_t s) {
    if (p.H < 1 || p.H > kMaxRows || p.kmax < 1 || p.max_nodes < 1 || p.max_nodes > 256) return cudaErrorInvalidValue;
    medusa_tree_kernel<<<1, kTreeThreads, 0, s>>>(p);
    return cudaGetLastError();
}

cudaError_t launch_medusa_walk(const MedusaWalkParams& p, cudaStream_t s) {
    if (p.M < 1 || p.M > 256 || p.d < 1) return cudaErrorInvalidValue;
    medusa_walk_kernel<<<1, kNT, 0, s>>>(p);
    return cudaGetLastError();
}

}  // namespace fl
