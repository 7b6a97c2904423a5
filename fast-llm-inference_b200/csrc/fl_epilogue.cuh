// Layer epilogues of the INT8 GEMV / GEMM kernels, applied to one weight-row
// pair (n0, n0 + 1) of one activation row once its outputs are final
// (matmul_dequantized, fast_llm/src/kernels/dequantized_tensor.c:204-247,
// followed by the fused layer steps of inference.c:250-399).
#pragma once

#include "fl_common.cuh"
#include "fl_kernels.h"

namespace fl {

// Rotary position and cache slot of activation row r (batched rows: the
// row's sequence record and KV region).
__device__ __forceinline__ int row_pos(const GemvParams& p, int r) {
    if (p.seq_rows <= 0) return p.pos[r];
    const int b = r / p.seq_rows;
    return p.pos[b * p.seq_state + (r - b * p.seq_rows)];
}
__device__ __forceinline__ int row_slot(const GemvParams& p, int r) {
    if (p.seq_rows <= 0) return *p.slot_base + r;
    const int b = r / p.seq_rows;
    return b * p.seq_slots + p.slot_base[b * p.seq_state] + (r - b * p.seq_rows);
}

// sin and cos of the rotary angle of position pos and even dimension ii:
// pos x theta^(-ii / head_dim) (inference.c:165-173).
__device__ __forceinline__ void rope_angle(int pos, int ii, int head_dim, float theta, float* sn, float* cs) {
    const float freq = __fdiv_rn(1.0f, powf(theta, __fdiv_rn((float)ii, (float)head_dim)));
    sincosf(__fmul_rn((float)pos, freq), sn, cs);
}

// Epilogue of one weight-row pair (n0, n0 + 1) for activation row r.
template <int EPI>
__device__ __forceinline__ void pair_epilogue(const GemvParams& p, int r, int n0, bool has1, float y0, float y1,
                                              unsigned long long* best_s) {
    if (EPI == EPI_STORE || EPI == EPI_LOGITS) {
        p.out[(size_t)r * p.ldo + n0] = y0;
        if (has1) p.out[(size_t)r * p.ldo + n0 + 1] = y1;
        if (EPI == EPI_LOGITS) {
            unsigned long long k = argmax_key(y0, n0);
            if (has1) {
                const unsigned long long k1 = argmax_key(y1, n0 + 1);
                k = k1 > k ? k1 : k;
            }
            atomicMax(&best_s[r - p.row0], k);
        }
    } else if (EPI == EPI_RESID) {
        float* o = p.out + (size_t)r * p.ldo + n0;
        o[0] = __fadd_rn(o[0], y0);
        if (has1) o[1] = __fadd_rn(o[1], y1);
    } else if (EPI == EPI_QKV) {
        float v0 = y0, v1 = y1;
        const int qkd = p.q_dim + p.kv_dim;
        if (n0 < qkd) {
            // inference.c:165-173 adjacent-pair rotation at position pos[r]
            const int ii = (n0 < p.q_dim ? n0 : n0 - p.q_dim) % p.head_dim;
            const int pos = row_pos(p, r);
            float sn, cs;
            if (p.rope && pos < p.rope_rows) {
                const float2 t = p.rope[(size_t)pos * (p.head_dim >> 1) + (ii >> 1)];
                cs = t.x;
                sn = t.y;
            } else {
                rope_angle(pos, ii, p.head_dim, p.theta, &sn, &cs);
            }
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
            const int slot = row_slot(p, r);
            const int page = p.block_table[slot / kPageSize];
            const size_t off = (((size_t)page * p.kv_heads + h) * kPageSize + (slot % kPageSize)) * p.head_dim + dd;
            *reinterpret_cast<__half2*>((is_k ? p.kv.k : p.kv.v) + off) = __floats2half2_rn(v0, v1);
        }
    } else if (EPI == EPI_TP_PUSH) {
        const size_t par = (size_t)(*p.tp_seq & 1ull);
        for (int q = 0; q < p.tp_size; q++) {
            float* dst = p.tp_recv[q] + ((par * p.tp_size + p.tp_rank) * p.tp_rows + r) * (size_t)p.ldo + n0;
            if (has1) *reinterpret_cast<float2*>(dst) = make_float2(y0, y1);
            else dst[0] = y0;
        }
    } else if (EPI == EPI_SWIGLU) {
        // rows (n0, n0 + 1) = (gate_i, up_i): activations_avx2.c:86-105
        const float h = __fmul_rn(__fmul_rn(y0, poly_sigmoid(y0)), y1);
        p.hq[(size_t)r * p.F + (n0 >> 1)] = (uint8_t)quant_u8(h);
    }
}

}  // namespace fl
