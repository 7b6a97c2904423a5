// fl_cuda runtime: errors, device streams, memory helpers, INT8 tensor upload
// and the INT8 matmul entry points (include/fl_cuda.h).
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <mutex>
#include <string>
#include <vector>

#include "fl_common.cuh"
#include "fl_kernels.h"
#include "fl_layout.cuh"
#include "fl_runtime.h"

namespace fl {

namespace {
thread_local std::string g_err;
std::mutex g_mu;
std::vector<cudaStream_t> g_streams;  // per device
}  // namespace

int set_error(int code, const std::string& msg) {
    g_err = msg;
    return code;
}

int cuda_error(cudaError_t e, const char* what) {
    std::string m = std::string(what) + ": " + cudaGetErrorString(e);
    cudaGetLastError();  // clear a sticky launch error where possible
    return set_error(e == cudaErrorMemoryAllocation ? FL_E_NOMEM
                     : e == cudaErrorNoDevice || e == cudaErrorInsufficientDriver ? FL_E_NODEV
                                                                                  : FL_E_CUDA,
                     m);
}

int ensure_device() {
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess || n == 0) {
        cudaGetLastError();
        return set_error(FL_E_NODEV, "no CUDA device available (the INT8 path has no CPU fallback)");
    }
    return FL_OK;
}

cudaStream_t device_stream() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
    std::lock_guard<std::mutex> lk(g_mu);
    if ((int)g_streams.size() <= dev) g_streams.resize(dev + 1, nullptr);
    if (!g_streams[dev]) {
        cudaStream_t s = nullptr;
        if (cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking) != cudaSuccess) return nullptr;
        g_streams[dev] = s;
    }
    return g_streams[dev];
}

// The library stream of the current device if it exists (never creates one).
cudaStream_t existing_device_stream() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
    std::lock_guard<std::mutex> lk(g_mu);
    return dev < (int)g_streams.size() ? g_streams[dev] : nullptr;
}

int upload_tensor(dequantized_tensor_t* t) {
    if (!t || !t->weights || t->rows <= 0 || t->cols <= 0)
        return set_error(FL_E_INVAL, "upload_tensor: tensor without int8 weights");
    if (t->dev) return FL_OK;
    FL_CHECK(ensure_device());
    const int blk = t->scale_block;
    if (blk != 0 && blk != 32) return set_error(FL_E_INVAL, "upload_tensor: scale_block must be 0 or 32");
    if (blk == 32 && (!t->scales_f16 || t->cols % 32 != 0))
        return set_error(FL_E_INVAL, "upload_tensor: block mode needs scales_f16 and cols % 32 == 0");
    if (blk == 0 && !t->scales) return set_error(FL_E_INVAL, "upload_tensor: per-row mode needs scales");
    DevTensor* d = (DevTensor*)calloc(1, sizeof(DevTensor));
    if (!d) return set_error(FL_E_NOMEM, "upload_tensor: host allocation");
    d->rows = t->rows;
    d->cols = t->cols;
    d->scale_block = blk;
    cudaGetDevice(&d->device);
    const size_t nw = (size_t)t->rows * t->cols;
    cudaError_t e = cudaMalloc(&d->w, nw);
    if (blk == 32) {
        // block mode: the TMA-ring GEMV's tiled layout whenever it can serve the shape
        d->P = tma_gemv_supported(t->rows, t->cols, 1) ? panel_width(t->cols) : 0;
        const size_t ns = (size_t)t->rows * (t->cols / 32) * sizeof(__half);
        if (e == cudaSuccess) e = cudaMalloc(&d->sblk, ns);
        if (e == cudaSuccess)
            e = upload_rows(d->w, d->sblk, t->rows, t->cols, d->P, 0, 1, t->weights, t->scales_f16, t->rows,
                            device_stream());
    } else if (e == cudaSuccess) {
        e = cudaMemcpy(d->w, t->weights, nw, cudaMemcpyHostToDevice);
    }
    if (e == cudaSuccess && blk == 0) {
        e = cudaMalloc(&d->srow, (size_t)t->rows * sizeof(float));
        if (e == cudaSuccess)
            e = cudaMemcpy(d->srow, t->scales, (size_t)t->rows * sizeof(float), cudaMemcpyHostToDevice);
        // The int16 pair saturation of dot_product_u8_i8 can only trigger when
        // some |w| > 64 (255 * 64 * 2 < 32768): pick the exact kernel variant.
        for (size_t i = 0; i < nw; i++) {
            const int v = t->weights[i];
            if (v > 64 || v < -64) { d->pairsat = 1; break; }
        }
    }
    if (e != cudaSuccess) {
        cudaFree(d->w);
        cudaFree(d->sblk);
        cudaFree(d->srow);
        free(d);
        return cuda_error(e, "upload_tensor");
    }
    t->dev = d;
    return FL_OK;
}

void release_tensor(dequantized_tensor_t* t) {
    if (!t || !t->dev) return;
    DevTensor* d = (DevTensor*)t->dev;
    int cur = 0;
    cudaGetDevice(&cur);
    cudaSetDevice(d->device);
    cudaFree(d->w);
    cudaFree(d->sblk);
    cudaFree(d->srow);
    cudaSetDevice(cur);
    free(d);
    t->dev = nullptr;
}

// Fills the operand part of GemvParams from an uploaded tensor.
static int tensor_params(const dequantized_tensor_t* B, int N, int K, GemvParams& p) {
    if (!B || !B->dev) return set_error(FL_E_STATE, "tensor not uploaded (fl_cuda_upload_tensor)");
    const DevTensor* d = (const DevTensor*)B->dev;
    if (d->rows != N || d->cols != K) return set_error(FL_E_INVAL, "matmul: N/K do not match the tensor");
    if (K % 32 != 0) return set_error(FL_E_INVAL, "matmul: K must be a multiple of 32");
    int cur = 0;
    cudaGetDevice(&cur);
    if (cur != d->device) return set_error(FL_E_STATE, "matmul: tensor lives on another device");
    p.w = d->w;
    p.P = d->P;
    p.sblk = d->sblk;
    p.srow = d->srow;
    p.N = N;
    p.K = K;
    return FL_OK;
}

static int scratch_q(size_t bytes, uint8_t** out);

static int run_gemv_chunks(const uint8_t* Aq, const dequantized_tensor_t* B, float* C, int32_t* D,
                           int M, int N, int K, cudaStream_t s, int epi, const float* X = nullptr) {
    GemvParams p = {};
    FL_CHECK(tensor_params(B, N, K, p));
    const DevTensor* d = (const DevTensor*)B->dev;
    p.aq = Aq;
    p.x = X;
    p.out = C;
    p.ldo = N;
    p.dots = D;
    if (M > 2 * kMaxRows && epi == EPI_STORE && d->scale_block == 32 && d->P != 0) {
        // many rows: quantize once, then the tcgen05 GEMM reads every weight once
        GemvParams h = p;
        h.x = nullptr;
        uint8_t* q = const_cast<uint8_t*>(Aq);
        if (!q) {
            FL_CHECK(scratch_q((size_t)M * K, &q));
            FL_CHECK(fl_cuda_act_quant(X, q, M, K, 0, 0.0f, s));
        }
        h.aq = q;
        h.row0 = 0;
        h.M = M;
        if (gemm_tc_supported(h, epi)) {
            FL_CHECK_CUDA(launch_gemm_tc(h, epi, M, s));
            return FL_OK;
        }
        p.aq = q;
        p.x = nullptr;
    }
    for (int r0 = 0; r0 < M; r0 += kMaxRows) {
        p.row0 = r0;
        p.M = M - r0 < kMaxRows ? M - r0 : kMaxRows;
        if (d->scale_block == 32)
            FL_CHECK_CUDA(launch_gemv_auto(p, epi, s, false));
        else
            FL_CHECK_CUDA(launch_gemv(p, epi, true, d->pairsat != 0, s, false));
    }
    return FL_OK;
}

// Scratch for quantized activations of the host-facing matmul entry points.
struct Scratch {
    uint8_t* q = nullptr;
    size_t cap = 0;
};
static thread_local std::vector<Scratch> t_scratch;

static int scratch_q(size_t bytes, uint8_t** out) {
    int dev = 0;
    cudaGetDevice(&dev);
    if ((int)t_scratch.size() <= dev) t_scratch.resize(dev + 1);
    Scratch& sc = t_scratch[dev];
    if (sc.cap < bytes) {
        if (sc.q) cudaFree(sc.q);
        sc.q = nullptr;
        sc.cap = 0;
        FL_CHECK_CUDA(cudaMalloc(&sc.q, bytes));
        sc.cap = bytes;
    }
    *out = sc.q;
    return FL_OK;
}

// Fixed scratch of fl_cuda_block_dots_i8_noalloc: the quantized activations
// of one call (M * K bytes), in the module's static device memory so that
// the call allocates nothing. Each byte a call reads is first written by
// the same call's quantization, so nothing needs to start at zero. One
// buffer per device: overlapping calls (other streams or threads) race.
static __device__ __align__(256) uint8_t g_noalloc_q[FL_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
static uint8_t* g_noalloc_ptr[kMaxDevices] = {};
static std::mutex g_noalloc_mu;

// Device address of g_noalloc_q on the current device, resolved once per
// device (the first resolution may load the module).
static int noalloc_scratch(uint8_t** out) {
    int dev = 0;
    FL_CHECK_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kMaxDevices) return set_error(FL_E_INVAL, "block_dots_noalloc: device index out of range");
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
        void* a = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&a, g_noalloc_q);
        if (e != cudaSuccess || !a) return cuda_error(e != cudaSuccess ? e : cudaErrorInvalidSymbol,
                                                      "block_dots_noalloc: cudaGetSymbolAddress of the static scratch");
        g_noalloc_ptr[dev] = static_cast<uint8_t*>(a);
    }
    *out = g_noalloc_ptr[dev];
    return FL_OK;
}

}  // namespace fl

using namespace fl;

FL_API const char* fl_cuda_last_error(void) { return g_err.c_str(); }

FL_API int fl_cuda_device_count(int* count) {
    if (!count) return set_error(FL_E_INVAL, "count is NULL");
    *count = 0;
    cudaError_t e = cudaGetDeviceCount(count);
    if (e != cudaSuccess) {
        *count = 0;
        cudaGetLastError();
    }
    return FL_OK;
}

FL_API int fl_cuda_init(int device) {
    FL_CHECK(ensure_device());
    FL_CHECK_CUDA(cudaSetDevice(device));
    if (!device_stream()) return set_error(FL_E_CUDA, "stream creation failed");
    return FL_OK;
}

FL_API int fl_cuda_sync(void) {
    cudaStream_t s = device_stream();
    if (!s) return set_error(FL_E_NODEV, "no device");
    FL_CHECK_CUDA(cudaStreamSynchronize(s));
    if (take_device_error() != 0) return set_error(FL_E_TIMEOUT, "a bounded device-side wait gave up");
    return FL_OK;
}

FL_API void* fl_cuda_stream(void) { return (void*)device_stream(); }

FL_API int fl_cuda_malloc(void** dptr, size_t bytes) {
    if (!dptr) return set_error(FL_E_INVAL, "dptr is NULL");
    FL_CHECK(ensure_device());
    FL_CHECK_CUDA(cudaMalloc(dptr, bytes));
    return FL_OK;
}

FL_API int fl_cuda_free(void* dptr) {
    FL_CHECK_CUDA(cudaFree(dptr));
    return FL_OK;
}

FL_API int fl_cuda_h2d(void* dst, const void* src, size_t bytes) {
    FL_CHECK_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, device_stream()));
    FL_CHECK_CUDA(cudaStreamSynchronize(device_stream()));
    return FL_OK;
}

FL_API int fl_cuda_d2h(void* dst, const void* src, size_t bytes) {
    FL_CHECK_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, device_stream()));
    FL_CHECK_CUDA(cudaStreamSynchronize(device_stream()));
    return FL_OK;
}

FL_API int fl_cuda_memset(void* dptr, int value, size_t bytes) {
    FL_CHECK_CUDA(cudaMemsetAsync(dptr, value, bytes, device_stream()));
    return FL_OK;
}

FL_API int fl_cuda_upload_tensor(dequantized_tensor_t* t) { return upload_tensor(t); }

FL_API int fl_cuda_act_quant(const float* x, uint8_t* q, int M, int K, int rmsnorm, float eps,
                             void* stream) {
    if (!x || !q || M <= 0 || K <= 0 || K % 4 != 0) return set_error(FL_E_INVAL, "act_quant: bad arguments");
    ActQuantParams p = {};
    p.x = x;
    p.q = q;
    p.K = K;
    p.M = M;
    p.norm = rmsnorm;
    p.eps = eps;
    cudaStream_t s = stream ? (cudaStream_t)stream : device_stream();
    FL_CHECK_CUDA(launch_act_quant(p, s, false));
    return FL_OK;
}

FL_API int fl_cuda_gemv_i8(const uint8_t* Aq, const dequantized_tensor_t* B, float* C, int M, int N,
                           int K, void* stream) {
    if (!Aq || !C || M <= 0) return set_error(FL_E_INVAL, "gemv: bad arguments");
    cudaStream_t s = stream ? (cudaStream_t)stream : device_stream();
    return run_gemv_chunks(Aq, B, C, nullptr, M, N, K, s, EPI_STORE);
}

FL_API int fl_cuda_matmul_i8(const float* A, const dequantized_tensor_t* B, float* C, int M, int N,
                             int K, void* stream) {
    if (!A || !C || M <= 0 || N <= 0 || K <= 0) return set_error(FL_E_INVAL, "matmul: bad arguments");
    if (K % 32 != 0) return set_error(FL_E_INVAL, "matmul: K must be a multiple of 32");
    cudaStream_t s = stream ? (cudaStream_t)stream : device_stream();
    if (B && B->dev && ((const DevTensor*)B->dev)->scale_block == 32 && K % 128 == 0)
        return run_gemv_chunks(nullptr, B, C, nullptr, M, N, K, s, EPI_STORE, A);  // fused quantization
    uint8_t* q = nullptr;
    FL_CHECK(scratch_q((size_t)M * K, &q));
    FL_CHECK(fl_cuda_act_quant(A, q, M, K, 0, 0.0f, s));
    return run_gemv_chunks(q, B, C, nullptr, M, N, K, s, EPI_STORE);
}

FL_API int fl_cuda_block_dots_i8_noalloc(const float* A, const dequantized_tensor_t* B, int32_t* D, int M, int N,
                                         int K, void* stream) {
    if (!A || !D || M <= 0 || N <= 0 || K <= 0) return set_error(FL_E_INVAL, "block_dots_noalloc: bad arguments");
    if (K % 32 != 0) return set_error(FL_E_INVAL, "block_dots_noalloc: K must be a multiple of 32");
    if ((size_t)M * (size_t)K > (size_t)FL_NOALLOC_SCRATCH_BYTES)
        return set_error(FL_E_INVAL, "block_dots_noalloc: M * K = " + std::to_string((size_t)M * (size_t)K) +
                                         " exceeds the static scratch of " +
                                         std::to_string((size_t)FL_NOALLOC_SCRATCH_BYTES) + " bytes");
    cudaStream_t s = stream ? (cudaStream_t)stream : existing_device_stream();
    if (!s) return set_error(FL_E_STATE, "block_dots_noalloc: pass a stream or call fl_cuda_init first");
    uint8_t* q = nullptr;
    FL_CHECK(noalloc_scratch(&q));
    FL_CHECK(fl_cuda_act_quant(A, q, M, K, 0, 0.0f, s));
    return run_gemv_chunks(q, B, nullptr, D, M, N, K, s, EPI_DOTS);
}

FL_API int fl_cuda_block_dots_i8(const float* A, const dequantized_tensor_t* B, int32_t* D, int M, int N,
                                 int K, void* stream) {
    if (!A || !D || M <= 0 || N <= 0 || K <= 0) return set_error(FL_E_INVAL, "block_dots: bad arguments");
    if (K % 32 != 0) return set_error(FL_E_INVAL, "block_dots: K must be a multiple of 32");
    cudaStream_t s = stream ? (cudaStream_t)stream : device_stream();
    uint8_t* q = nullptr;
    FL_CHECK(scratch_q((size_t)M * K, &q));
    FL_CHECK(fl_cuda_act_quant(A, q, M, K, 0, 0.0f, s));
    return run_gemv_chunks(q, B, nullptr, D, M, N, K, s, EPI_DOTS);
}

FL_API int fl_cuda_block_dots_w4(const float* A, const dequantized_tensor_t* B, int32_t* D, int M, int N, int K,
                                 void* stream) {
    if (!A || !D || M <= 0 || M > kMaxRows || N <= 0 || K <= 0 || K % 32 != 0)
        return set_error(FL_E_INVAL, "block_dots_w4: bad arguments (M <= 8)");
    cudaStream_t s = stream ? (cudaStream_t)stream : device_stream();
    GemvParams p = {};
    FL_CHECK(tensor_params(B, N, K, p));
    const DevTensor* d = (const DevTensor*)B->dev;
    if (d->scale_block != 32 || !w4_supported(N, K, d->P))
        return set_error(FL_E_INVAL, "block_dots_w4: needs a tiled block-mode tensor (cols a multiple of 256)");
    uint8_t* q = nullptr;
    FL_CHECK(scratch_q((size_t)M * K, &q));
    FL_CHECK(fl_cuda_act_quant(A, q, M, K, 0, 0.0f, s));
    uint8_t* w4 = nullptr;
    int* bad = nullptr;
    int hbad = 0, rc = FL_OK;
    cudaError_t ce = cudaMalloc(&w4, (size_t)N * K / 2);
    if (ce == cudaSuccess) ce = cudaMalloc(&bad, sizeof(int));
    if (ce == cudaSuccess) ce = cudaMemsetAsync(bad, 0, sizeof(int), s);
    if (ce == cudaSuccess) ce = launch_pack_w4(d->w, w4, N, K, d->P, bad, s);
    if (ce == cudaSuccess) {
        p.aq = q;
        p.w4 = w4;
        p.dots = D;
        p.row0 = 0;
        p.M = M;
        ce = launch_gemv_tma(p, EPI_DOTS, s, false);
    }
    if (ce == cudaSuccess) ce = cudaMemcpyAsync(&hbad, bad, sizeof(int), cudaMemcpyDeviceToHost, s);
    if (ce == cudaSuccess) ce = cudaStreamSynchronize(s);
    if (ce != cudaSuccess) rc = cuda_error(ce, "block_dots_w4");
    else if (hbad) rc = set_error(FL_E_INVAL, "block_dots_w4: a weight lies outside [-8, 7]");
    cudaFree(w4);
    cudaFree(bad);
    return rc;
}

FL_API int fl_cuda_medusa_tree(const int* tok, const float* prob, const int* topk, int H, int kmax, int max_nodes,
                               int root, int n, int* out_tok, int* out_parent, int* out_depth, int* out_pos,
                               uint8_t* out_mask) {
    if (!tok || !prob || !topk || !out_tok || !out_parent || !out_depth || !out_pos || !out_mask || H < 1 ||
        H > kMaxRows || kmax < 1 || kmax > 32 || max_nodes < 1 || max_nodes > 256)
        return set_error(FL_E_INVAL, "medusa_tree: bad arguments");
    long long cand = 0, width = 1;
    for (int h = 0; h < H; h++) {
        if (topk[h] < 1 || topk[h] > kmax) return set_error(FL_E_INVAL, "medusa_tree: top-k must be 1..kmax");
        width *= topk[h];
        cand += width;
        if (cand > kMaxTreeCand) return set_error(FL_E_INVAL, "medusa_tree: more than 1024 candidates");
    }
    const int M = 1 + std::min<int>(max_nodes - 1, (int)cand);
    cudaStream_t s = device_stream();
    int *dtok = nullptr, *dk = nullptr, *droot = nullptr, *dout = nullptr;
    float* dprob = nullptr;
    uint8_t* dmask = nullptr;
    int rc = FL_OK;
    auto cuda_ok = [&](cudaError_t e, const char* what) {
        if (e != cudaSuccess && rc == FL_OK) rc = cuda_error(e, what);
        return rc == FL_OK;
    };
    do {
        if (!cuda_ok(cudaMalloc(&dtok, sizeof(int) * (size_t)H * kmax), "medusa_tree: alloc") ||
            !cuda_ok(cudaMalloc(&dprob, sizeof(float) * (size_t)H * kmax), "medusa_tree: alloc") ||
            !cuda_ok(cudaMalloc(&dk, sizeof(int) * H), "medusa_tree: alloc") ||
            !cuda_ok(cudaMalloc(&droot, sizeof(int)), "medusa_tree: alloc") ||
            !cuda_ok(cudaMalloc(&dout, sizeof(int) * 4 * (size_t)max_nodes), "medusa_tree: alloc") ||
            !cuda_ok(cudaMalloc(&dmask, (size_t)M * M), "medusa_tree: alloc"))
            break;
        if (!cuda_ok(cudaMemcpyAsync(dtok, tok, sizeof(int) * (size_t)H * kmax, cudaMemcpyHostToDevice, s), "up") ||
            !cuda_ok(cudaMemcpyAsync(dprob, prob, sizeof(float) * (size_t)H * kmax, cudaMemcpyHostToDevice, s), "up") ||
            !cuda_ok(cudaMemcpyAsync(dk, topk, sizeof(int) * H, cudaMemcpyHostToDevice, s), "up") ||
            !cuda_ok(cudaMemcpyAsync(droot, &root, sizeof(int), cudaMemcpyHostToDevice, s), "up"))
            break;
        MedusaTreeParams p = {dtok, dprob, dk, H, kmax, max_nodes, n, droot,
                              dout, dout + max_nodes, dout + 2 * max_nodes, dout + 3 * max_nodes, dmask};
        if (!cuda_ok(launch_medusa_tree(p, s), "medusa_tree: launch")) break;
        int* outs[4] = {out_tok, out_parent, out_depth, out_pos};
        for (int i = 0; i < 4; i++)
            if (!cuda_ok(cudaMemcpyAsync(outs[i], dout + (size_t)i * max_nodes, sizeof(int) * M,
                                         cudaMemcpyDeviceToHost, s), "medusa_tree: read"))
                break;
        if (rc != FL_OK) break;
        if (!cuda_ok(cudaMemcpyAsync(out_mask, dmask, (size_t)M * M, cudaMemcpyDeviceToHost, s), "medusa_tree: read"))
            break;
        cuda_ok(cudaStreamSynchronize(s), "medusa_tree: sync");
    } while (0);
    void* bufs[] = {dtok, dprob, dk, droot, dout, dmask};
    for (void* b : bufs) cudaFree(b);
    return rc == FL_OK ? M : rc;
}
