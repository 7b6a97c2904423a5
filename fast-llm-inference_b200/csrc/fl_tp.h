// Tensor-parallel shard layout and NCCL calls (tp.cu).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>

namespace fl {

struct TpLayout {
    int q0, nq;    // Q heads [q0, q0 + nq)
    int kv0, nkv;  // KV heads [kv0, kv0 + nkv) read by them
    int f0, nf;    // FFN features
    int v0, nv;    // LM-head (vocabulary) rows
    int group;     // Q heads per KV head
};

int tp_layout(int H, int Hkv, int F, int V, int rank, int size, TpLayout& o);
int tp_comm_init(int rank, int size, const unsigned char id[128], void** comm);
void tp_comm_free(void* comm);
int tp_allreduce_sum_f32(void* comm, float* buf, size_t count, cudaStream_t s);
int tp_allgather_u64(void* comm, const unsigned long long* send, unsigned long long* recv, size_t count,
                     cudaStream_t s);

}  // namespace fl
