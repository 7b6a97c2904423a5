// RMSNorm + activation quantization, and tree-masked attention over the
// paged fp16 KV cache (sm_100a).
#include <float.h>

#include "fl_common.cuh"
#include "fl_kernels.h"

namespace fl {

namespace {

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

constexpr int kAThreads = 128;
constexpr int kARows = 8;     // query rows per CTA
constexpr int kMaxHd = 128;

// Attention of up to kARows query rows of one head over slots
// [0, base + M): prefix slots [0, base) are visible to every row, new slot
// base + j to new row i iff mask[i*M + j] (causal j <= i when mask is NULL).
// inference.c:193-247 restated for a KV cache: scores = q.k * 1/sqrt(hd),
// softmax with max subtraction and expf, then the p-weighted sum of V.
__global__ void __launch_bounds__(kAThreads) attention_kernel(const AttnParams p) {
    extern __shared__ float sm[];
    pdl_trigger();
    pdl_wait();
    if (p.done && *p.done) return;
    const int M = p.dyn_M ? *p.dyn_M : p.M;
    const int h = blockIdx.x;
    const int r0 = blockIdx.y * kARows;
    if (r0 >= M) return;
    const int nr = min(kARows, M - r0);
    const int base = *p.slot_base;
    const int ctx = base + M;
    const int hd = p.head_dim;
    const int kvh = h / (p.heads / p.kv_heads);
    const int qd = p.heads * hd;

    float* q_s = sm;                         // [kARows][hd]
    float* sc = sm + kARows * kMaxHd;        // [kARows][ctx]
    __shared__ float red[kAThreads / 32];
    __shared__ float rowstat[kARows];

    for (int i = threadIdx.x; i < nr * hd; i += kAThreads) {
        const int rr = i / hd, dd = i - rr * hd;
        q_s[rr * hd + dd] = p.q[(size_t)(r0 + rr) * qd + (size_t)h * hd + dd];
    }
    __syncthreads();

    const float scale = __fdiv_rn(1.0f, sqrtf((float)hd));
    // scores: one key per thread, all rows of the CTA
    for (int j = threadIdx.x; j < ctx; j += kAThreads) {
        const int page = p.block_table[j / kPageSize];
        const __half2* kr = reinterpret_cast<const __half2*>(
            p.kv.k + (((size_t)page * p.kv_heads + kvh) * kPageSize + (j % kPageSize)) * hd);
        float acc[kARows];
#pragma unroll
        for (int rr = 0; rr < kARows; rr++) acc[rr] = 0.0f;
        for (int d2 = 0; d2 < hd / 2; d2++) {
            const float2 kv = __half22float2(kr[d2]);
#pragma unroll
            for (int rr = 0; rr < kARows; rr++) {
                if (rr < nr) {
                    acc[rr] = __fmaf_rn(q_s[rr * hd + 2 * d2], kv.x, acc[rr]);
                    acc[rr] = __fmaf_rn(q_s[rr * hd + 2 * d2 + 1], kv.y, acc[rr]);
                }
            }
        }
#pragma unroll
        for (int rr = 0; rr < kARows; rr++) {
            if (rr < nr) {
                bool vis = true;
                if (j >= base) {
                    const int jj = j - base, ii = r0 + rr;
                    vis = p.mask ? (p.mask[(size_t)ii * M + jj] != 0) : (jj <= ii);
                }
                sc[rr * ctx + j] = vis ? __fmul_rn(acc[rr], scale) : -FLT_MAX;
            }
        }
    }
    __syncthreads();

    // softmax per row (max, exp, sum, normalise)
    for (int rr = 0; rr < nr; rr++) {
        float* s = sc + rr * ctx;
        float mx = -FLT_MAX;
        for (int j = threadIdx.x; j < ctx; j += kAThreads) mx = fmaxf(mx, s[j]);
        mx = warp_max(mx);
        if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
        __syncthreads();
        if (threadIdx.x == 0) {
            float t = red[0];
            for (int w = 1; w < kAThreads / 32; w++) t = fmaxf(t, red[w]);
            rowstat[rr] = t;
        }
        __syncthreads();
        mx = rowstat[rr];
        float sum = 0.0f;
        for (int j = threadIdx.x; j < ctx; j += kAThreads) {
            const float e = s[j] == -FLT_MAX ? 0.0f : expf(__fsub_rn(s[j], mx));
            s[j] = e;
            sum += e;
        }
        sum = warp_sum(sum);
        __syncthreads();
        if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = sum;
        __syncthreads();
        if (threadIdx.x == 0) {
            float t = 0.0f;
            for (int w = 0; w < kAThreads / 32; w++) t += red[w];
            rowstat[rr] = t;
        }
        __syncthreads();
        const float tot = rowstat[rr];
        for (int j = threadIdx.x; j < ctx; j += kAThreads) s[j] = __fdiv_rn(s[j], tot);
        __syncthreads();
    }

    // out[rr][d] = sum_j p[rr][j] * v[j][d]; thread -> dimension pair
    for (int d2 = threadIdx.x; d2 < hd / 2; d2 += kAThreads) {
        float a0[kARows], a1[kARows];
#pragma unroll
        for (int rr = 0; rr < kARows; rr++) { a0[rr] = 0.0f; a1[rr] = 0.0f; }
        for (int j = 0; j < ctx; j++) {
            const int page = p.block_table[j / kPageSize];
            const __half2* vr = reinterpret_cast<const __half2*>(
                p.kv.v + (((size_t)page * p.kv_heads + kvh) * kPageSize + (j % kPageSize)) * hd);
            const float2 v = __half22float2(vr[d2]);
#pragma unroll
            for (int rr = 0; rr < kARows; rr++) {
                if (rr < nr) {
                    const float w = sc[rr * ctx + j];
                    a0[rr] = __fmaf_rn(w, v.x, a0[rr]);
                    a1[rr] = __fmaf_rn(w, v.y, a1[rr]);
                }
            }
        }
#pragma unroll
        for (int rr = 0; rr < kARows; rr++) {
            if (rr < nr) {
                const size_t o = (size_t)(r0 + rr) * qd + (size_t)h * hd + 2 * d2;
                p.out_q[o] = (uint8_t)quant_u8(a0[rr]);
                p.out_q[o + 1] = (uint8_t)quant_u8(a1[rr]);
                if (p.out_f) { p.out_f[o] = a0[rr]; p.out_f[o + 1] = a1[rr]; }
            }
        }
    }
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

cudaError_t launch_attention(const AttnParams& p, cudaStream_t s, bool pdl) {
    if (p.head_dim > kMaxHd || p.head_dim % 2 != 0 || p.heads % p.kv_heads != 0) return cudaErrorInvalidValue;
    const size_t smem = sizeof(float) * ((size_t)kARows * kMaxHd + (size_t)kARows * p.max_ctx);
    if (smem > 200 * 1024) return cudaErrorInvalidValue;
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)smem);
        if (e != cudaSuccess) return e;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.heads, (p.M + kARows - 1) / kARows);
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
