// Control kernels of the speculative step: embedding gathers, greedy draft
// picks, verify-row preparation and acceptance (sm_100a). They move a few KB
// and exist so that a whole draft + verify step runs on the device without a
// host round trip.
#include <algorithm>

#include "fl_common.cuh"
#include "fl_epilogue.cuh"
#include "fl_state.h"

namespace fl {

namespace {

constexpr int kT = 256;

template <typename F, typename... Args>
cudaError_t launch_pdl(F kern, dim3 grid, int threads, cudaStream_t s, bool pdl, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(threads);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, args...);
}

// Block-wide argmax over the LM-head partial keys of one row.
__device__ unsigned long long block_best(const unsigned long long* part, int nparts) {
    __shared__ unsigned long long red[kT / 32];
    unsigned long long best = 0ull;
    for (int i = threadIdx.x; i < nparts; i += blockDim.x) {
        const unsigned long long k = part[i];
        best = k > best ? k : best;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long k = __shfl_xor_sync(0xffffffffu, best, o);
        best = k > best ? k : best;
    }
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = best;
    __syncthreads();
    best = 0ull;
    for (int w = 0; w < (int)(blockDim.x >> 5); w++) best = red[w] > best ? red[w] : best;
    __syncthreads();
    return best;
}

__global__ void embed_rows_kernel(const float* embed, int vocab, const int* tok, const float* feat, int shift,
                                  float* x, int d, int rows_static, const int* dyn_rows,
                                  const int* done) {
    pdl_trigger();
    pdl_wait();
    if (done && *done) return;
    const int r = blockIdx.x;
    const int rows = dyn_rows ? *dyn_rows : rows_static;
    if (r >= rows) return;
    int t = tok[r];
    if (t < 0 || t >= vocab) t = 0;  // inference.c:421-422: out-of-vocabulary ids read row 0
    const float* e = embed + (size_t)t * d;
    float* xr = x + (size_t)r * d;
    const float* f = (feat && r >= shift) ? feat + (size_t)(r - shift) * d : nullptr;
    for (int i = threadIdx.x; i < d; i += blockDim.x) xr[i] = f ? __fadd_rn(f[i], e[i]) : e[i];
}

__global__ void draft_pick_kernel(const StepBuffers b0, int j) {
    pdl_trigger();
    pdl_wait();
    const StepBuffers b = seq_view(b0, blockIdx.x);
    SpecState* st = b.st;
    if (st->done) return;
    const unsigned long long best = block_best(b.amax_d, b.nparts);
    const int tok = argmax_key_index(best);
    const int n = st->n;
    if (threadIdx.x == 0) {
        st->drafted[j] = tok;
        if (j + 1 < st->K) {
            st->draft_base = n + j + 1;
            st->draft_pos[0] = n + j + 1;
        }
    }
    if (j + 1 < st->K) {
        const int g_row = (j == 0 && !b.batch) ? st->last_row : 0;
        const float* g = b.x_d1 + (size_t)g_row * b.d;
        const float* e = b.embed + (size_t)tok * b.d;
        float* x0 = b.x_d1;
        // g_row may be 0: element-wise in place is safe.
        for (int i = threadIdx.x; i < b.d; i += blockDim.x) x0[i] = __fadd_rn(g[i], e[i]);
    }
}

__global__ void verify_prep_kernel(const StepBuffers b0) {
    pdl_trigger();
    pdl_wait();
    const StepBuffers b = seq_view(b0, blockIdx.y);
    SpecState* st = b.st;
    if (st->done) return;
    const int r = blockIdx.x;
    const int n = st->n;
    const int tok = r == 0 ? b.seq[n] : st->drafted[r - 1];
    if (threadIdx.x == 0) {
        st->verify_pos[r] = n + r;
        if (r == 0) st->verify_base = n;
    }
    const float* e = b.embed + (size_t)tok * b.d;
    float* xr = b.x_v + (size_t)r * b.d;
    for (int i = threadIdx.x; i < b.d; i += blockDim.x) xr[i] = e[i];
}

__global__ void accept_kernel(const StepBuffers b0, int K) {
    pdl_trigger();
    pdl_wait();
    const StepBuffers b = seq_view(b0, blockIdx.x);
    SpecState* st = b.st;
    if (st->done) return;
    __shared__ int tgt[kMaxRows];
    for (int r = 0; r <= K; r++) {
        const unsigned long long best = block_best(b.amax_part + (size_t)r * b.nparts, b.nparts);
        if (threadIdx.x == 0) tgt[r] = argmax_key_index(best);
    }
    __syncthreads();
    if (threadIdx.x != 0) return;
    const int n = st->n;
    int a = 0;
    while (a < K && a < st->max_acc && st->drafted[a] == tgt[a]) a++;
    for (int r = 0; r <= K; r++) st->target[r] = tgt[r];
    int produced = st->produced;
    for (int j = 0; j <= a; j++) {
        const int t = j < a ? st->drafted[j] : tgt[a];
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

__global__ void catchup_prep_kernel(const StepBuffers b0) {
    pdl_trigger();
    pdl_wait();
    const StepBuffers b = seq_view(b0, blockIdx.y);
    SpecState* st = b.st;
    if (st->done) return;
    const int r = blockIdx.x;
    if (r >= st->rows) {
        // batched catch-up passes run K + 1 rows for every sequence: rows past
        // this sequence's accepted ones are zero (their outputs are unused,
        // and the cache slots they write are rewritten before they are read)
        if (b.batch) {
            float* xr = b.x_d + (size_t)r * b.d;
            for (int i = threadIdx.x; i < b.d; i += blockDim.x) xr[i] = 0.0f;
        }
        return;
    }
    const int pos = st->draft_base + r;  // = n_old + 1 + r
    const int tok = b.seq[pos];
    const float* e = b.embed + (size_t)tok * b.d;
    const float* f = b.x_v + (size_t)r * b.d;
    float* xr = b.x_d + (size_t)r * b.d;
    for (int i = threadIdx.x; i < b.d; i += blockDim.x) xr[i] = __fadd_rn(f[i], e[i]);
}

// Batched: the catch-up's feature of each sequence's newest token.
__global__ void gather_last_kernel(const StepBuffers b0) {
    pdl_trigger();
    pdl_wait();
    const StepBuffers b = seq_view(b0, blockIdx.x);
    if (b.st->done) return;
    const float* src = b.x_d + (size_t)b.st->last_row * b.d;
    for (int i = threadIdx.x; i < b.d; i += blockDim.x) b.x_d1[i] = src[i];
}

__global__ void argmax_rows_kernel(const unsigned long long* part, int nparts, int* out_tok,
                                   float* out_val) {
    pdl_wait();
    const int r = blockIdx.x;
    const unsigned long long best = block_best(part + (size_t)r * nparts, nparts);
    if (threadIdx.x == 0) {
        out_tok[r] = argmax_key_index(best);
        if (out_val) out_val[r] = argmax_key_value(best);
    }
}

// Tensor parallelism: this rank's best LM-head key per row, re-keyed from the
// local row index to the global one (index + v0; the key stores
// 0x7fffffff - index in its low word), then the maximum over all ranks'
// gathered keys.
__global__ void tp_local_best_kernel(const unsigned long long* part, int nparts, int v0, unsigned long long* out) {
    const int r = blockIdx.x;
    const unsigned long long best = block_best(part + (size_t)r * nparts, nparts);
    if (threadIdx.x == 0) out[r] = best ? best - (unsigned long long)v0 : 0ull;
}

__global__ void tp_reduce_best_kernel(const unsigned long long* all, int size, int stride, int rows,
                                      unsigned long long* out) {
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= rows) return;
    unsigned long long m = 0ull;
    for (int s = 0; s < size; s++) m = all[(size_t)s * stride + r] > m ? all[(size_t)s * stride + r] : m;
    out[r] = m;
}

}  // namespace

cudaError_t launch_tp_local_best(const unsigned long long* part, int nparts, int rows, int v0, unsigned long long* out,
                                 cudaStream_t s) {
    tp_local_best_kernel<<<rows, kT, 0, s>>>(part, nparts, v0, out);
    return cudaGetLastError();
}

cudaError_t launch_tp_reduce_best(const unsigned long long* all, int size, int stride, int rows,
                                  unsigned long long* out, cudaStream_t s) {
    tp_reduce_best_kernel<<<(rows + 127) / 128, 128, 0, s>>>(all, size, stride, rows, out);
    return cudaGetLastError();
}

cudaError_t launch_embed_rows(const float* embed, int vocab, const int* tok, const float* feat, int shift,
                              float* x, int d, int rows_static, const int* dyn_rows,
                              const int* done, cudaStream_t s, bool pdl) {
    return launch_pdl(embed_rows_kernel, dim3(rows_static), kT, s, pdl, embed, vocab, tok, feat, shift, x,
                      d, rows_static, dyn_rows, done);
}

__global__ void rope_table_kernel(float2* tab, int rows, int head_dim, float theta) {
    const int h2 = head_dim >> 1;
    const size_t n = (size_t)rows * h2;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const int pos = (int)(i / h2), j = (int)(i - (size_t)pos * h2);
        float sn, cs;
        rope_angle(pos, 2 * j, head_dim, theta, &sn, &cs);
        tab[i] = make_float2(cs, sn);
    }
}

cudaError_t launch_rope_table(float2* tab, int rows, int head_dim, float theta, cudaStream_t s) {
    if (!tab || rows <= 0 || head_dim <= 0 || head_dim % 2) return cudaErrorInvalidValue;
    const size_t n = (size_t)rows * (head_dim / 2);
    const int blocks = (int)std::min<size_t>((n + 255) / 256, 4096);
    rope_table_kernel<<<blocks, 256, 0, s>>>(tab, rows, head_dim, theta);
    return cudaGetLastError();
}

cudaError_t launch_draft_pick(const StepBuffers& b, int j, cudaStream_t s, bool pdl) {
    return launch_pdl(draft_pick_kernel, dim3(step_seqs(b)), kT, s, pdl, b, j);
}

cudaError_t launch_verify_prep(const StepBuffers& b, int K, cudaStream_t s, bool pdl) {
    return launch_pdl(verify_prep_kernel, dim3(K + 1, step_seqs(b)), kT, s, pdl, b);
}

cudaError_t launch_accept(const StepBuffers& b, int K, cudaStream_t s, bool pdl) {
    return launch_pdl(accept_kernel, dim3(step_seqs(b)), kT, s, pdl, b, K);
}

cudaError_t launch_catchup_prep(const StepBuffers& b, int K, cudaStream_t s, bool pdl) {
    return launch_pdl(catchup_prep_kernel, dim3(K + 1, step_seqs(b)), kT, s, pdl, b);
}

cudaError_t launch_gather_last(const StepBuffers& b, cudaStream_t s, bool pdl) {
    return launch_pdl(gather_last_kernel, dim3(step_seqs(b)), kT, s, pdl, b);
}

cudaError_t launch_argmax_rows(const unsigned long long* part, int nparts, int rows, int* out_tok,
                               float* out_val, cudaStream_t s) {
    return launch_pdl(argmax_rows_kernel, dim3(rows), kT, s, false, part, nparts, out_tok, out_val);
}

}  // namespace fl
