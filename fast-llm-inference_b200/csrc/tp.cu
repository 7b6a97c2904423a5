// Tensor parallelism across the GPUs of one node: the shard layout of a model
// over tp ranks and the NCCL calls the engine makes (host code).
//
// Layout (Megatron-style): rank r of g holds
//  - Q heads [r H/g, (r+1) H/g) and the KV heads they read (GQA group
//    G = H / Hkv: [q0 / G, (q1 - 1) / G]), so a KV head that straddles two
//    ranks is held by both;
//  - FFN features [r F/g, (r+1) F/g) (interleaved gate/up rows, down columns);
//  - LM-head rows [r ceil(V/g), ...) (the last rank may hold fewer);
//  - the full embedding.
// Q/K/V and gate/up are column-parallel, o and down row-parallel: after each
// of o and down the ranks' partial outputs are summed by one NCCL all-reduce
// (rank 0's epilogue adds the residual first). The LM head's per-rank argmax
// keys (value, global index) are all-gathered and reduced on every rank.
//
// NCCL is loaded with dlopen on first use (libnccl.so.2, the process's copy if
// one is already loaded), so single-GPU use needs no NCCL.
#include <dlfcn.h>
#include <nccl.h>

#include <string.h>

#include <algorithm>
#include <mutex>

#include "fl_common.cuh"
#include "fl_kernels.h"
#include "fl_runtime.h"
#include "fl_tp.h"

namespace fl {

namespace {

struct NcclApi {
    ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
    ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                               cudaStream_t) = nullptr;
    ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
    const char* (*error_string)(ncclResult_t) = nullptr;
    bool ok = false;
};

NcclApi& nccl() {
    static NcclApi api;
    static std::once_flag once;
    std::call_once(once, [] {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        if (!h) return;
        api.get_unique_id = (decltype(api.get_unique_id))dlsym(h, "ncclGetUniqueId");
        api.comm_init_rank = (decltype(api.comm_init_rank))dlsym(h, "ncclCommInitRank");
        api.all_reduce = (decltype(api.all_reduce))dlsym(h, "ncclAllReduce");
        api.all_gather = (decltype(api.all_gather))dlsym(h, "ncclAllGather");
        api.comm_destroy = (decltype(api.comm_destroy))dlsym(h, "ncclCommDestroy");
        api.error_string = (decltype(api.error_string))dlsym(h, "ncclGetErrorString");
        api.ok = api.get_unique_id && api.comm_init_rank && api.all_reduce && api.all_gather && api.comm_destroy &&
                 api.error_string;
    });
    return api;
}

int nccl_error(ncclResult_t r, const char* what) {
    const char* s = nccl().error_string ? nccl().error_string(r) : "?";
    return set_error(FL_E_CUDA, std::string(what) + ": NCCL " + s);
}

}  // namespace

int tp_layout(int H, int Hkv, int F, int V, int rank, int size, TpLayout& o) {
    if (size < 1 || rank < 0 || rank >= size || H <= 0 || Hkv <= 0 || H % Hkv || H % size || F % size)
        return set_error(FL_E_INVAL, "tensor parallel: heads and FFN features must divide by the rank count "
                                     "(and heads by KV heads)");
    const int G = H / Hkv;
    o.nq = H / size;
    o.q0 = rank * o.nq;
    o.kv0 = o.q0 / G;
    o.nkv = (o.q0 + o.nq - 1) / G + 1 - o.kv0;
    o.nf = F / size;
    o.f0 = rank * o.nf;
    const int vc = (V + size - 1) / size;
    o.v0 = std::min(V, rank * vc);
    o.nv = std::min(V, o.v0 + vc) - o.v0;
    o.group = G;
    if (o.nv <= 0) return set_error(FL_E_INVAL, "tensor parallel: more ranks than vocabulary rows");
    return FL_OK;
}

int tp_comm_init(int rank, int size, const unsigned char id[128], void** comm) {
    if (!nccl().ok) return set_error(FL_E_UNSUPPORTED, "tensor parallel: libnccl.so.2 could not be loaded");
    ncclUniqueId uid;
    static_assert(sizeof(uid) == 128, "ncclUniqueId is 128 bytes");
    memcpy(&uid, id, sizeof(uid));
    ncclComm_t c = nullptr;
    const ncclResult_t r = nccl().comm_init_rank(&c, size, uid, rank);
    if (r != ncclSuccess) return nccl_error(r, "ncclCommInitRank");
    *comm = c;
    return FL_OK;
}

void tp_comm_free(void* comm) {
    if (comm && nccl().ok) nccl().comm_destroy((ncclComm_t)comm);
}

int tp_allreduce_sum_f32(void* comm, float* buf, size_t count, cudaStream_t s) {
    const ncclResult_t r = nccl().all_reduce(buf, buf, count, ncclFloat32, ncclSum, (ncclComm_t)comm, s);
    return r == ncclSuccess ? FL_OK : nccl_error(r, "ncclAllReduce");
}

int tp_allgather_u64(void* comm, const unsigned long long* send, unsigned long long* recv, size_t count,
                     cudaStream_t s) {
    const ncclResult_t r = nccl().all_gather(send, recv, count, ncclUint64, (ncclComm_t)comm, s);
    return r == ncclSuccess ? FL_OK : nccl_error(r, "ncclAllGather");
}

}  // namespace fl

FL_API int fl_tp_unique_id(unsigned char* id) {
    using namespace fl;
    if (!id) return set_error(FL_E_INVAL, "tp_unique_id: id is NULL");
    if (!nccl().ok) return set_error(FL_E_UNSUPPORTED, "tensor parallel: libnccl.so.2 could not be loaded");
    ncclUniqueId uid;
    const ncclResult_t r = nccl().get_unique_id(&uid);
    if (r != ncclSuccess) return nccl_error(r, "ncclGetUniqueId");
    memcpy(id, &uid, sizeof(uid));
    return FL_OK;
}

FL_API int fl_tp_layout(const fl_model_config_t* cfg, int rank, int size, int* out) {
    using namespace fl;
    if (!cfg || !out) return set_error(FL_E_INVAL, "tp_layout: NULL argument");
    TpLayout L;
    FL_CHECK(tp_layout(cfg->num_heads, cfg->num_kv_heads, cfg->intermediate_size, cfg->vocab_size, rank, size, L));
    const int v[9] = {L.q0, L.nq, L.kv0, L.nkv, L.f0, L.nf, L.v0, L.nv, L.group};
    memcpy(out, v, sizeof(v));
    return FL_OK;
}

// The failure path of the tensor-parallel reduction's bounded wait, on one
// GPU: tp_reduce_kernel waits for arrival counters of a two-rank group that
// no rank ever increments; after its limit (about two seconds of clock
// cycles) it records the error word and returns without touching the
// activations, and fl_cuda_sync reports FL_E_TIMEOUT. The context stays
// usable. For tests of failure detection; no fault is involved.
FL_API int fl_cuda_tp_wait_timeout_check(void) {
    using namespace fl;
    FL_CHECK(ensure_device());
    cudaStream_t s = device_stream();
    if (!s) return set_error(FL_E_NODEV, "no device");
    float* x = nullptr;
    unsigned long long* words = nullptr;  // [4] counters of two ranks (two parities), [1] sequence
    int* arrived = nullptr;
    FL_CHECK_CUDA(cudaMalloc(&x, sizeof(float) * 256));
    FL_CHECK_CUDA(cudaMalloc(&words, sizeof(unsigned long long) * 5));
    FL_CHECK_CUDA(cudaMalloc(&arrived, sizeof(int)));
    FL_CHECK_CUDA(cudaMemsetAsync(x, 0, sizeof(float) * 256, s));
    FL_CHECK_CUDA(cudaMemsetAsync(words, 0, sizeof(unsigned long long) * 5, s));
    FL_CHECK_CUDA(cudaMemsetAsync(arrived, 0, sizeof(int), s));
    TpReduceParams p = {};
    p.x = x;
    p.rows = 1;
    p.d = 256;
    p.recv = x;  // never read: the wait gives up first
    p.cnt = words;
    p.size = 2;
    p.cap = 1;
    p.seq = words + 4;
    p.ctas_per_push = 1;
    p.arrived = arrived;
    const cudaError_t le = launch_tp_reduce(p, s, false);
    const cudaError_t se = cudaStreamSynchronize(s);
    cudaFree(x);
    cudaFree(words);
    cudaFree(arrived);
    FL_CHECK_CUDA(le);
    FL_CHECK_CUDA(se);
    return FL_OK;
}
