// fl_engine: the base model, draft and Medusa heads resident in HBM, paged
// fp16 KV caches, and the speculative decode loop (include/fl_cuda.h).
//
// Layer chain (per stack, per layer; inference.c:250-399 restated):
//   act_quant(RMSNorm(x))           -> xq      [rows, d]   u8
//   GEMV qkv  (EPI_QKV)             -> q f32 + K/V fp16 pages (RoPE fused)
//   attention (tree/causal mask)    -> aq      [rows, qd]  u8
//   GEMV o    (EPI_RESID)           -> x += o
//   act_quant(RMSNorm(x))           -> xq
//   GEMV gate/up interleaved (EPI_SWIGLU) -> hq [rows, F] u8
//   GEMV down (EPI_RESID)           -> x += down
// One speculative step is captured once as a CUDA graph whose kernels read
// positions from the device-resident SpecState, and replayed.
#include <stddef.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <climits>
#include <functional>
#include <string>
#include <vector>

#include "fl_common.cuh"
#include "fl_kernels.h"
#include "fl_layout.cuh"
#include "fl_runtime.h"
#include "fl_state.h"
#include "fl_step.h"
#include "fl_tp.h"

#include "fl_engine_impl.h"

namespace fl_eng {

int alloc_linear(Linear& l, int N, int K, unsigned need, bool step_layout) {
    l.N = N;
    l.K = K;
    l.need = need;
    l.have = 0;
    // The TMA-ring GEMV reads the tiled layout; shapes it cannot serve stay
    // row-major. The tcgen05 step kernel wants 128-byte panels (pairs of them
    // per ring stage); the TMA-ring GEMV reads those too.
    if (step_layout && N % 8 == 0 && K % (2 * kStepPanel) == 0)
        l.P = kStepPanel;
    else
        l.P = tma_gemv_supported(N, K, 1) ? panel_width(K) : 0;
    FL_CHECK_CUDA(cudaMalloc(&l.w, (size_t)N * K));
    FL_CHECK_CUDA(cudaMalloc(&l.s, (size_t)N * (K / 32) * sizeof(__half)));
    return FL_OK;
}

void free_linear(Linear& l) {
    cudaFree(l.w);
    cudaFree(l.s);
    cudaFree(l.w4);
    l.w = nullptr;
    l.s = nullptr;
    l.w4 = nullptr;
}

int alloc_stack(fl_engine* e, Stack& S, int nl) {
    S.nl = nl;
    S.L.resize(nl);
    S.kv.resize(nl);
    const int d = e->d, qd = e->qd, kd = e->kd, F = e->F;
    S.pages = (e->c.max_seq_len + kPageSize - 1) / kPageSize;
    for (int l = 0; l < nl; l++) {
        LayerW& W = S.L[l];
        FL_CHECK(alloc_linear(W.qkv, qd + 2 * kd, d, 0x7u, e->step_layout));
        FL_CHECK(alloc_linear(W.o, d, qd, 0x1u, e->step_layout));
        FL_CHECK(alloc_linear(W.gu, 2 * F, d, 0x3u, e->step_layout));
        FL_CHECK(alloc_linear(W.down, d, F, 0x1u, e->step_layout));
        const size_t kvb = (size_t)S.pages * e->Hkv * kPageSize * e->hd * sizeof(__half);
        FL_CHECK_CUDA(cudaMalloc(&S.kv[l].k, kvb));
        FL_CHECK_CUDA(cudaMalloc(&S.kv[l].v, kvb));
        FL_CHECK_CUDA(cudaMemset(S.kv[l].k, 0, kvb));
        FL_CHECK_CUDA(cudaMemset(S.kv[l].v, 0, kvb));
    }
    // One sequence: identity block table (pages are still addressed through it).
    std::vector<int> bt(S.pages);
    for (int i = 0; i < S.pages; i++) bt[i] = i;
    FL_CHECK_CUDA(cudaMalloc(&S.block_table, sizeof(int) * S.pages));
    FL_CHECK_CUDA(cudaMemcpy(S.block_table, bt.data(), sizeof(int) * S.pages, cudaMemcpyHostToDevice));
    return FL_OK;
}

void free_stack(Stack& S) {
    for (auto& W : S.L) {
        free_linear(W.qkv);
        free_linear(W.o);
        free_linear(W.gu);
        free_linear(W.down);
    }
    for (auto& kv : S.kv) {
        cudaFree(kv.k);
        cudaFree(kv.v);
    }
    cudaFree(S.block_table);
    S.L.clear();
    S.kv.clear();
}

// Copies `rows` rows of int8 weights / fp16 scales into a fused matrix at
// destination row dst_row0 with a destination row stride of dst_stride rows
// (stride 2 interleaves gate and up).
int put_rows(Linear& l, int dst_row0, int dst_stride, const int8_t* w, const uint16_t* sc, int rows,
             int cols, cudaStream_t s) {
    if (cols != l.K) return set_error(FL_E_INVAL, "load_linear: column count does not match the model");
    FL_CHECK_CUDA(upload_rows(l.w, l.s, l.N, l.K, l.P, dst_row0, dst_stride, w, sc, rows, s));
    return FL_OK;
}

bool linear_ready(const Linear& l) { return l.w && (l.have & l.need) == l.need; }

bool stack_ready(const Stack& S) {
    for (const auto& W : S.L)
        if (!linear_ready(W.qkv) || !linear_ready(W.o) || !linear_ready(W.gu) || !linear_ready(W.down))
            return false;
    return true;
}

GemvParams gemv_base(const Linear& l, const uint8_t* aq, const int* done) {
    GemvParams g = {};
    g.aq = aq;
    g.w = l.w;
    g.w4 = l.w4;
    g.P = l.P;
    g.sblk = l.s;
    g.N = l.N;
    g.K = l.K;
    g.done = done;
    return g;
}

#ifndef FL_ROPE_TABLE
#define FL_ROPE_TABLE 1
#endif

// Many static rows (more than two GEMV launches' worth) go through the
// tcgen05 GEMM (weights read once); the fused RMSNorm prologue then runs as
// its own quantization pass.
constexpr int kGemmMinRows = 2 * kMaxRows;
bool gemm_enabled() {
    static const bool on = [] {
        const char* v = getenv("FL_GEMM_TC");
        return !(v && v[0] == '0');
    }();
    return on;
}

int launch_chunks(GemvParams g, int epi, int M, const int* dyn_M, cudaStream_t s, bool pdl) {
    if (!dyn_M && M > kGemmMinRows && gemm_enabled() && g.P != 0 && g.row0 == 0) {
        GemvParams h = g;
        h.x = nullptr;
        h.x_row_dyn = nullptr;
        if (gemm_tc_supported(h, epi)) {
            if (g.x) {
                ActQuantParams a = {};
                a.x = g.x;
                a.q = const_cast<uint8_t*>(g.aq);
                a.K = g.K;
                a.M = M;
                a.norm = g.norm;
                a.eps = g.eps;
                a.done = g.done;
                FL_CHECK_CUDA(launch_act_quant(a, s, pdl));
            }
            FL_CHECK_CUDA(launch_gemm_tc(h, epi, M, s));
            return FL_OK;
        }
    }
    if (dyn_M) {  // M is the static upper bound of *dyn_M (<= kMaxRows)
        g.dyn_M = dyn_M;
        g.row0 = 0;
        g.M = std::min(M, kMaxRows);
        FL_CHECK_CUDA(launch_gemv_auto(g, epi, s, pdl));
        return FL_OK;
    }
    for (int r0 = 0; r0 < M; r0 += kMaxRows) {
        g.row0 = r0;
        g.M = std::min(kMaxRows, M - r0);
        FL_CHECK_CUDA(launch_gemv_auto(g, epi, s, pdl));
    }
    return FL_OK;
}

int act_quant(fl_engine* e, const float* x, uint8_t* q, int K, int M, const int* dyn_M, int norm,
              const int* done, bool pdl) {
    ActQuantParams a = {};
    a.x = x;
    a.q = q;
    a.K = K;
    a.M = M;
    a.dyn_M = dyn_M;
    a.norm = norm;
    a.eps = e->c.norm_eps;
    a.done = done;
    FL_CHECK_CUDA(launch_act_quant(a, e->s, pdl));
    return FL_OK;
}

// x += the o / down projection g of the layer. Under tensor parallelism the
// projection is row-parallel: decode-sized passes push partial rows to every
// rank over NVLink and sum them there (fused path); otherwise rank 0 adds the
// residual, the others store their partials and NCCL all-reduces x.
int residual_linear(fl_engine* e, GemvParams g, float* x, int M, const int* dyn_M, const int* done, bool pdl) {
    if (e->tp_size == 1) return launch_chunks(g, EPI_RESID, M, dyn_M, e->s, pdl);
    if (e->tp_fused && M <= kMaxRows && g.P != 0 && tma_gemv_supported(g.N, g.K, M)) {
        g.tp_recv = e->tp_recv_ptrs;
        g.tp_cnt = e->tp_cnt_ptrs;
        g.tp_seq = e->tp_seq;
        g.tp_rank = e->tp_rank;
        g.tp_size = e->tp_size;
        g.tp_rows = kMaxRows;
        FL_CHECK(launch_chunks(g, EPI_TP_PUSH, M, dyn_M, e->s, pdl));
        TpReduceParams r = {};
        r.x = x;
        r.rows = M;
        r.dyn_rows = dyn_M;
        r.d = e->d;
        r.recv = (const float*)e->tp_region;
        r.cnt = (const unsigned long long*)((const char*)e->tp_region + e->tp_recv_bytes + 256);
        r.size = e->tp_size;
        r.cap = kMaxRows;
        r.seq = e->tp_seq;
        r.ctas_per_push = (unsigned long long)tma_gemv_grid();
        r.arrived = e->tp_arrived;
        r.done = done;
        FL_CHECK_CUDA(launch_tp_reduce(r, e->s, pdl));
        return FL_OK;
    }
    FL_CHECK(launch_chunks(g, e->tp_rank == 0 ? EPI_RESID : EPI_STORE, M, dyn_M, e->s, pdl));
    return tp_allreduce_sum_f32(e->tp_comm, x, (size_t)M * e->d, e->s);
}

// Runs M rows (M <= R; dyn_M bounds the live rows when set, M <= kMaxRows)
// through a stack. slot_base / pos are device pointers.
int run_stack(fl_engine* e, Stack& S, float* x, int M, const int* dyn_M, const int* slot_base, const int* pos,
              const uint8_t* mask, const int* done, bool pdl, const KvView* view) {
    const int d = e->d, qd = e->qd, F = e->F;
    const bool batched = view && view->seqs > 1;
    // Fused RMSNorm + quantization prologues need K % 128 == 0; otherwise a
    // separate act_quant launch produces xq.
    const bool fuse = (d % 128) == 0;
    for (int l = 0; l < S.nl; l++) {
        LayerW& W = S.L[l];
        if (!fuse) FL_CHECK(act_quant(e, x, e->xq, d, M, dyn_M, 1, done, pdl));
        GemvParams g = gemv_base(W.qkv, e->xq, done);
        if (fuse) {
            g.x = x;
            g.norm = 1;
            g.eps = e->c.norm_eps;
        }
        g.q_out = e->q;
        g.kv = view ? view->kv[l] : S.kv[l];
        g.block_table = view ? view->block_table : S.block_table;
        g.slot_base = slot_base;
        g.pos = pos;
        if (batched) {
            g.seq_rows = view->seq_rows;
            g.seq_state = view->seq_state;
            g.seq_slots = view->seq_slots;
        }
        g.q_dim = qd;
        g.kv_dim = e->kd;
        g.head_dim = e->hd;
        g.kv_heads = e->Hkv;
        g.theta = e->c.rope_theta;
        g.rope = e->rope;
        g.rope_rows = e->rope_rows;
        FL_CHECK(launch_chunks(g, EPI_QKV, M, dyn_M, e->s, pdl));
        AttnParams at = {};
        at.q = e->q;
        at.kv = view ? view->kv[l] : S.kv[l];
        at.block_table = view ? view->block_table : S.block_table;
        at.slot_base = slot_base;
        at.M = batched ? view->seq_rows : M;
        if (batched) {
            at.seqs = view->seqs;
            at.seq_state = view->seq_state;
            at.seq_slots = view->seq_slots;
        }
        at.dyn_M = dyn_M;
        at.mask = mask;
        at.heads = e->H;
        at.kv_heads = e->Hkv;
        at.head_dim = e->hd;
        if (e->tp_size > 1) {
            at.q_head0 = e->tp.q0;
            at.kv_head0 = e->tp.kv0;
            at.group = e->tp.group;
        }
        at.max_ctx = view && view->max_ctx ? view->max_ctx : e->c.max_seq_len;
        at.out_q = e->aq;
        at.done = done;
        at.part = view && view->attn_part ? view->attn_part : e->attn_part;
        at.counters = view && view->attn_cnt ? view->attn_cnt : e->attn_cnt;
        FL_CHECK_CUDA(launch_attention(at, e->s, pdl));
        g = gemv_base(W.o, e->aq, done);
        g.out = x;
        g.ldo = d;
        FL_CHECK(residual_linear(e, g, x, M, dyn_M, done, pdl));
        if (!fuse) FL_CHECK(act_quant(e, x, e->xq, d, M, dyn_M, 1, done, pdl));
        g = gemv_base(W.gu, e->xq, done);
        if (fuse) {
            g.x = x;
            g.norm = 1;
            g.eps = e->c.norm_eps;
        }
        g.hq = e->hq;
        g.F = F;
        FL_CHECK(launch_chunks(g, EPI_SWIGLU, M, dyn_M, e->s, pdl));
        g = gemv_base(W.down, e->hq, done);
        g.out = x;
        g.ldo = d;
        FL_CHECK(residual_linear(e, g, x, M, dyn_M, done, pdl));
    }
    return FL_OK;
}

// LM head over rows of x (M <= kMaxRows): logits [M, V] and argmax partials.
// dyn_src_row (device) selects the first source row of x.
// Vocabulary-parallel LM head: every rank's best key per row (re-keyed to
// the global index), all-gathered and reduced into tp_best[0, M).
int tp_argmax(fl_engine* e, const unsigned long long* part, int M) {
    if (M > e->tp_rows) return set_error(FL_E_INVAL, "tensor parallel: more LM-head rows than the key buffers hold");
    FL_CHECK_CUDA(launch_tp_local_best(part, e->nparts, M, e->tp.v0, e->tp_keys, e->s));
    FL_CHECK(tp_allgather_u64(e->tp_comm, e->tp_keys, e->tp_all, e->tp_rows, e->s));
    FL_CHECK_CUDA(launch_tp_reduce_best(e->tp_all, e->tp_size, e->tp_rows, M, e->tp_best, e->s));
    return FL_OK;
}

int run_lm(fl_engine* e, const float* x, int M, const int* dyn_src_row, const int* done, bool pdl,
           float* logits, unsigned long long* amax) {
    if (M > kMaxRows || logits) {
        // rows in launches of up to kMaxRows (batched steps), into the given
        // logits [M, V] and argmax partials [M, nparts]; under tensor
        // parallelism the keys of the rows end in tp_best[0, M)
        if (dyn_src_row || !logits || !amax || (e->d % 128) != 0)
            return set_error(FL_E_UNSUPPORTED, "LM head: many-row passes need the fused RMSNorm prologue");
        GemvParams g = gemv_base(e->lm, e->xq, done);
        g.x = x;
        g.norm = 1;
        g.eps = e->c.norm_eps;
        g.out = logits;
        g.ldo = e->V;
        g.amax_part = amax;
        for (int r0 = 0; r0 < M; r0 += kMaxRows) {
            g.row0 = r0;
            g.M = std::min(kMaxRows, M - r0);
            FL_CHECK_CUDA(launch_gemv_auto(g, EPI_LOGITS, e->s, pdl));
        }
        if (e->tp_size > 1) FL_CHECK(tp_argmax(e, amax, M));
        return FL_OK;
    }
    GemvParams g = gemv_base(e->lm, e->xq, done);
    if ((e->d % 128) == 0) {
        g.x = x;
        g.norm = 1;
        g.eps = e->c.norm_eps;
        g.x_row_dyn = dyn_src_row;
    } else {
        ActQuantParams a = {};
        a.x = x;
        a.q = e->xq;
        a.K = e->d;
        a.M = M;
        a.norm = 1;
        a.eps = e->c.norm_eps;
        a.done = done;
        a.dyn_src_row = dyn_src_row;
        FL_CHECK_CUDA(launch_act_quant(a, e->s, pdl));
    }
    g.out = e->logits;
    g.ldo = e->V;
    g.amax_part = e->amax;
    g.M = M;
    g.row0 = 0;
    FL_CHECK_CUDA(launch_gemv_auto(g, EPI_LOGITS, e->s, pdl));
    if (e->tp_size > 1) {
        // vocabulary-parallel head: each rank's winner (global index), all-gathered, reduced
        FL_CHECK(tp_argmax(e, e->amax, M));
    }
    return FL_OK;
}

int ensure_mask(fl_engine* e, int M) {
    if (e->mask_cap >= M * M) return FL_OK;
    cudaFree(e->mask);
    e->mask = nullptr;
    FL_CHECK_CUDA(cudaMalloc(&e->mask, (size_t)M * M));
    e->mask_cap = M * M;
    return FL_OK;
}

int carve_work(fl_engine* e, void** const* ptrs, const size_t* sizes, int n) {
    size_t total = 0;
    for (int i = 0; i < n; i++) total += (sizes[i] + 255) & ~(size_t)255;
    if (e->work_arena_cap < total) {
        FL_CHECK_CUDA(cudaStreamSynchronize(e->s));
        cudaFree(e->work_arena);
        e->work_arena = nullptr;
        e->work_arena_cap = 0;
        FL_CHECK_CUDA(cudaMalloc(&e->work_arena, total));
        e->work_arena_cap = total;
    }
    size_t off = 0;
    for (int i = 0; i < n; i++) {
        *ptrs[i] = e->work_arena + off;
        off += (sizes[i] + 255) & ~(size_t)255;
    }
    return FL_OK;
}

// Argmax keys of the last LM-head pass: the GEMV's per-CTA partials, or under
// tensor parallelism the all-rank maximum (one key per row).
const unsigned long long* amax_keys(const fl_engine* e) { return e->tp_size > 1 ? e->tp_best : e->amax; }
int amax_nparts(const fl_engine* e) { return e->tp_size > 1 ? 1 : e->nparts; }

StepBuffers step_buffers(fl_engine* e) {
    StepBuffers b = {};
    b.st = e->st;
    b.seq = e->seq;
    b.out = e->out;
    b.acc_hist = e->acc;
    b.embed = e->embed;
    b.x_d = e->x_d;
    b.x_v = e->x_v;
    b.amax_part = amax_keys(e);
    b.nparts = amax_nparts(e);
    b.d = e->d;
    b.logits = e->logits;
    b.V = e->V;
    b.temp = e->samp_T;
    b.top_p = e->samp_top_p;
    b.key = e->samp_key;
    b.qd = e->samp_q;
    b.qm = e->samp_m;
    b.pt = e->samp_p;
    b.pm = e->samp_m ? e->samp_m + kMaxDraft : nullptr;
    b.resid = e->samp_r;
    b.trace = e->trace_on ? e->samp_trace : nullptr;
    return b;
}

int check_ready(fl_engine* e, bool need_draft) {
    if (!e) return set_error(FL_E_INVAL, "engine is NULL");
    if (!fl_engine_ready(e)) return set_error(FL_E_STATE, "engine weights not fully loaded");
    if (need_draft && e->c.draft_layers <= 0) return set_error(FL_E_STATE, "engine has no draft model");
    FL_CHECK_CUDA(cudaSetDevice(e->device));
    return FL_OK;
}

// Records one speculative step (include/speculative.h rule) on e->s.
int record_step(fl_engine* e, bool pdl) {
    const int K = e->spec_K;
    SpecState* st = e->st;
    const int* done = &st->done;
    StepBuffers b = step_buffers(e);
    // greedy: argmax picks and exact-match acceptance; sampling: nucleus
    // draws and rejection-sampling acceptance
    auto pick = [&](int j) {
        return e->samp ? launch_sample_pick(b, j, e->s, pdl) : launch_draft_pick(b, j, e->s, pdl);
    };
    for (int j = 1; j < K; j++) {
        FL_CHECK(run_stack(e, e->draft, e->x_d, 1, nullptr, &st->draft_base, st->draft_pos, nullptr, done, pdl));
        FL_CHECK(run_lm(e, e->x_d, 1, nullptr, done, pdl));
        FL_CHECK_CUDA(pick(j));
    }
    FL_CHECK_CUDA(launch_verify_prep(b, K, e->s, pdl));
    FL_CHECK(run_stack(e, e->base, e->x_v, K + 1, nullptr, &st->verify_base, st->verify_pos, nullptr, done, pdl));
    FL_CHECK(run_lm(e, e->x_v, K + 1, nullptr, done, pdl));
    if (e->samp) {
        FL_CHECK_CUDA(launch_target_dist(b, K, e->s, pdl));
        FL_CHECK_CUDA(launch_accept_sampled(b, K, e->s, pdl));
    } else {
        FL_CHECK_CUDA(launch_accept(b, K, e->s, pdl));
    }
    FL_CHECK_CUDA(launch_catchup_prep(b, K, e->s, pdl));
    FL_CHECK(run_stack(e, e->draft, e->x_d, K + 1, &st->rows, &st->draft_base, st->draft_pos, nullptr, done, pdl));
    FL_CHECK(run_lm(e, e->x_d, 1, &st->last_row, done, pdl));
    FL_CHECK_CUDA(pick(0));
    return FL_OK;
}

// ---- one-kernel step: the same sequence as record_step as a phase list ----
Phase gemv_phase_of(const GemvParams& g, int epi) {
    Phase ph;
    memset(&ph, 0, sizeof(ph));
    ph.kind = PH_GEMV;
    ph.epi = epi;
    ph.g = g;
    return ph;
}

bool stack_phases(fl_engine* e, Stack& S, float* x, int M, const int* dyn_M, const int* slot_base,
                  const int* pos, const int* done, std::vector<Phase>& out) {
    const int d = e->d;
    for (int l = 0; l < S.nl; l++) {
        LayerW& W = S.L[l];
        if (!W.qkv.P || !W.o.P || !W.gu.P || !W.down.P) return false;
        GemvParams g = gemv_base(W.qkv, e->xq, done);
        g.x = x;
        g.norm = 1;
        g.eps = e->c.norm_eps;
        g.M = M;
        g.dyn_M = dyn_M;
        g.q_out = e->q;
        g.kv = S.kv[l];
        g.block_table = S.block_table;
        g.slot_base = slot_base;
        g.pos = pos;
        g.q_dim = e->qd;
        g.kv_dim = e->kd;
        g.head_dim = e->hd;
        g.kv_heads = e->Hkv;
        g.theta = e->c.rope_theta;
        out.push_back(gemv_phase_of(g, EPI_QKV));
        Phase a;
        memset(&a, 0, sizeof(a));
        a.kind = PH_ATTN;
        a.a.q = e->q;
        a.a.kv = S.kv[l];
        a.a.block_table = S.block_table;
        a.a.slot_base = slot_base;
        a.a.M = M;
        a.a.dyn_M = dyn_M;
        a.a.heads = e->H;
        a.a.kv_heads = e->Hkv;
        a.a.head_dim = e->hd;
        a.a.max_ctx = e->c.max_seq_len;
        a.a.out_q = e->aq;
        a.a.done = done;
        a.a.part = e->attn_part;
        a.a.counters = e->attn_cnt;
        out.push_back(a);
        g = gemv_base(W.o, e->aq, done);
        g.M = M;
        g.dyn_M = dyn_M;
        g.out = x;
        g.ldo = d;
        out.push_back(gemv_phase_of(g, EPI_RESID));
        g = gemv_base(W.gu, e->xq, done);
        g.x = x;
        g.norm = 1;
        g.eps = e->c.norm_eps;
        g.M = M;
        g.dyn_M = dyn_M;
        g.hq = e->hq;
        g.F = e->F;
        out.push_back(gemv_phase_of(g, EPI_SWIGLU));
        g = gemv_base(W.down, e->hq, done);
        g.M = M;
        g.dyn_M = dyn_M;
        g.out = x;
        g.ldo = d;
        out.push_back(gemv_phase_of(g, EPI_RESID));
    }
    return true;
}

bool lm_phase(fl_engine* e, const float* x, int M, const int* dyn_src_row, const int* done, std::vector<Phase>& out) {
    if (!e->lm.P) return false;
    GemvParams g = gemv_base(e->lm, e->xq, done);
    g.x = x;
    g.norm = 1;
    g.eps = e->c.norm_eps;
    g.x_row_dyn = dyn_src_row;
    g.out = e->logits;
    g.ldo = e->V;
    g.amax_part = e->amax;
    g.M = M;
    out.push_back(gemv_phase_of(g, EPI_LOGITS));
    return true;
}

Phase control_phase(int kind, int arg) {
    Phase ph;
    memset(&ph, 0, sizeof(ph));
    ph.kind = kind;
    ph.arg = arg;
    return ph;
}

// The whole speculative step of record_step as one phase list.
bool step_phases(fl_engine* e, std::vector<Phase>& ph) {
    const int K = e->spec_K;
    SpecState* st = e->st;
    const int* done = &st->done;
    for (int j = 1; j < K; j++) {
        if (!stack_phases(e, e->draft, e->x_d, 1, nullptr, &st->draft_base, st->draft_pos, done, ph)) return false;
        if (!lm_phase(e, e->x_d, 1, nullptr, done, ph)) return false;
        ph.push_back(control_phase(PH_DRAFT_PICK, j));
    }
    ph.push_back(control_phase(PH_VERIFY_PREP, 0));
    if (!stack_phases(e, e->base, e->x_v, K + 1, nullptr, &st->verify_base, st->verify_pos, done, ph)) return false;
    if (!lm_phase(e, e->x_v, K + 1, nullptr, done, ph)) return false;
    ph.push_back(control_phase(PH_ACCEPT, 0));
    ph.push_back(control_phase(PH_CATCHUP_PREP, 0));
    if (!stack_phases(e, e->draft, e->x_d, K + 1, &st->rows, &st->draft_base, st->draft_pos, done, ph)) return false;
    if (!lm_phase(e, e->x_d, 1, &st->last_row, done, ph)) return false;
    ph.push_back(control_phase(PH_DRAFT_PICK, 0));
    return true;
}

// Builds and uploads the phase list of the one-kernel step (outside any
// capture); returns FL_E_UNSUPPORTED when some weight is not in the tiled
// layout or the LM partials are not laid out per SM (the caller then
// records the multi-kernel step).
int prepare_step_kernel(fl_engine* e, StepParams& sp, size_t& smem) {
    std::vector<Phase> ph;
    if (!step_phases(e, ph)) return FL_E_UNSUPPORTED;
    if (e->nparts != step_grid()) return FL_E_UNSUPPORTED;
    sp = StepParams{};
    smem = 0;
    if (!step_plan(ph.data(), (int)ph.size(), sp, &smem)) return FL_E_UNSUPPORTED;
    FL_CHECK_CUDA(step_set_smem(smem));
    if (e->d_phases && e->n_phases < (int)ph.size()) {
        cudaFree(e->d_phases);
        e->d_phases = nullptr;
    }
    if (!e->d_phases) FL_CHECK_CUDA(cudaMalloc(&e->d_phases, sizeof(Phase) * ph.size()));
    e->n_phases = (int)ph.size();
    FL_CHECK_CUDA(cudaMemcpy(e->d_phases, ph.data(), sizeof(Phase) * ph.size(), cudaMemcpyHostToDevice));
    e->phase_desc.clear();
    for (const Phase& q : ph) {
        const bool g = q.kind == PH_GEMV;
        e->phase_desc.insert(e->phase_desc.end(), {q.kind, g ? q.epi : q.arg, g ? q.g.N : 0, g ? q.g.K : 0});
    }
    const char* tr = getenv("FL_STEP_TRACE");
    if (tr && tr[0] == '1') {
        if (e->d_trace) cudaFree(e->d_trace);
        e->d_trace = nullptr;
        FL_CHECK_CUDA(cudaMalloc(&e->d_trace, sizeof(unsigned long long) * (6 * ph.size() + 512)));
        FL_CHECK_CUDA(cudaMemset(e->d_trace, 0, sizeof(unsigned long long) * (6 * ph.size() + 512)));
    }
    sp.trace = e->d_trace;
    const char* tp = getenv("FL_STEP_TRACE_PHASE");
    sp.trace_phase = tp ? atoi(tp) : -1;
    sp.phases = e->d_phases;
    sp.nphases = (int)ph.size();
    sp.sb = step_buffers(e);
    sp.K = e->spec_K;
    sp.bar = e->step_bar;
    sp.done = &e->st->done;
    return FL_OK;
}

int build_step_graph(fl_engine* e) {
    if (e->step_exec && e->graph_K == e->spec_K) return FL_OK;
    if (e->step_exec) {
        cudaGraphExecDestroy(e->step_exec);
        e->step_exec = nullptr;
    }
    const char* dis = getenv("FL_DISABLE_STEP_KERNEL");
    StepParams sp;
    size_t smem = 0;
    // the one-kernel step implements the greedy rule only
    int prc = ((dis && dis[0] == '1') || e->samp) ? FL_E_UNSUPPORTED : prepare_step_kernel(e, sp, smem);
    if (prc != FL_OK && prc != FL_E_UNSUPPORTED) return prc;
    cudaGraph_t g = nullptr;
    int rc = FL_E_UNSUPPORTED;
    cudaError_t ce = cudaSuccess;
    if (prc == FL_OK) {
        // one-kernel step; if the cooperative launch cannot be captured the
        // multi-kernel step is recorded instead
        FL_CHECK_CUDA(cudaStreamBeginCapture(e->s, cudaStreamCaptureModeThreadLocal));
        // the grid-barrier counter starts every launch at zero
        rc = cudaMemsetAsync(e->step_bar, 0, sizeof(unsigned long long), e->s) == cudaSuccess &&
                     launch_step(sp, smem, e->s) == cudaSuccess
                 ? FL_OK
                 : FL_E_UNSUPPORTED;
        ce = cudaStreamEndCapture(e->s, &g);
        if (rc != FL_OK || ce != cudaSuccess) {
            if (g) cudaGraphDestroy(g);
            g = nullptr;
            (void)cudaGetLastError();
            rc = FL_E_UNSUPPORTED;
        }
    }
    e->step_kernel = rc == FL_OK;
    if (rc == FL_E_UNSUPPORTED) {
        FL_CHECK_CUDA(cudaStreamBeginCapture(e->s, cudaStreamCaptureModeThreadLocal));
        rc = record_step(e, true);
        ce = cudaStreamEndCapture(e->s, &g);
        if (rc != FL_OK) {
            if (g) cudaGraphDestroy(g);
            return rc;
        }
        FL_CHECK_CUDA(ce);
    }
    size_t nn = 0;
    cudaGraphGetNodes(g, nullptr, &nn);
    std::vector<cudaGraphNode_t> nodes(nn);
    cudaGraphGetNodes(g, nodes.data(), &nn);
    int nk = 0;
    for (auto nd : nodes) {
        cudaGraphNodeType t;
        if (cudaGraphNodeGetType(nd, &t) == cudaSuccess && t == cudaGraphNodeTypeKernel) nk++;
    }
    e->graph_kernels = nk;
    ce = cudaGraphInstantiate(&e->step_exec, g, 0);
    cudaGraphDestroy(g);
    FL_CHECK_CUDA(ce);
    e->graph_K = e->spec_K;
    return FL_OK;
}

int prefill_base(fl_engine* e, const int* prompt, int P) {
    FL_CHECK_CUDA(cudaMemcpyAsync(e->seq, prompt, sizeof(int) * P, cudaMemcpyHostToDevice, e->s));
    FL_CHECK_CUDA(launch_embed_rows(e->embed, e->Vg, e->seq, nullptr, 0, e->x, e->d, P, nullptr, nullptr, e->s, false));
    FL_CHECK(run_stack(e, e->base, e->x, P, nullptr, e->iota, e->iota, nullptr, nullptr, false));
    // next token from the last row
    FL_CHECK_CUDA(cudaMemcpyAsync(e->x_v, e->x + (size_t)(P - 1) * e->d, sizeof(float) * e->d,
                                  cudaMemcpyDeviceToDevice, e->s));
    FL_CHECK(run_lm(e, e->x_v, 1, nullptr, nullptr, false));
    FL_CHECK_CUDA(launch_argmax_rows(amax_keys(e), amax_nparts(e), 1, e->seq + P, nullptr, e->s));
    return FL_OK;
}

}  // namespace fl_eng

// ---------------------------------------------------------------------------
// C ABI
// ---------------------------------------------------------------------------

// Maps every rank's receive region (CUDA IPC handles all-gathered over NCCL).
// Fused mode needs every rank to succeed; the decision is collective.
static int tp_fused_setup(fl_engine* e) {
    const int g = e->tp_size;
    e->tp_recv_bytes = (size_t)2 * g * kMaxRows * e->d * sizeof(float);
    const size_t bytes = e->tp_recv_bytes + 256 + (size_t)2 * g * sizeof(unsigned long long);
    int ok = 1;
    cudaIpcMemHandle_t h;
    if (cudaMalloc(&e->tp_region, bytes) != cudaSuccess || cudaMemset(e->tp_region, 0, bytes) != cudaSuccess ||
        cudaIpcGetMemHandle(&h, e->tp_region) != cudaSuccess) {
        ok = 0;
        (void)cudaGetLastError();
        memset(&h, 0, sizeof(h));
    }
    static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handles are 64 bytes");
    unsigned long long send[9];
    memcpy(send, &h, 64);
    send[8] = (unsigned long long)ok;
    unsigned long long *dsend = nullptr, *drecv = nullptr;
    FL_CHECK_CUDA(cudaMalloc(&dsend, sizeof(send)));
    FL_CHECK_CUDA(cudaMalloc(&drecv, sizeof(send) * g));
    std::vector<unsigned long long> all((size_t)9 * g);
    int rc = FL_OK;
    if (cudaMemcpy(dsend, send, sizeof(send), cudaMemcpyHostToDevice) != cudaSuccess ||
        tp_allgather_u64(e->tp_comm, dsend, drecv, 9, e->s) != FL_OK || cudaStreamSynchronize(e->s) != cudaSuccess ||
        cudaMemcpy(all.data(), drecv, sizeof(send) * g, cudaMemcpyDeviceToHost) != cudaSuccess)
        rc = set_error(FL_E_CUDA, "tensor parallel: IPC handle exchange");
    cudaFree(dsend);
    cudaFree(drecv);
    FL_CHECK(rc);
    for (int q = 0; q < g; q++) ok = ok && all[(size_t)9 * q + 8] == 1;
    if (!ok) return FL_OK;  // every rank stays on NCCL
    e->tp_peer.assign(g, nullptr);
    for (int q = 0; q < g; q++) {
        if (q == e->tp_rank) {
            e->tp_peer[q] = e->tp_region;
            continue;
        }
        cudaIpcMemHandle_t hq;
        memcpy(&hq, &all[(size_t)9 * q], 64);
        FL_CHECK_CUDA(cudaIpcOpenMemHandle(&e->tp_peer[q], hq, cudaIpcMemLazyEnablePeerAccess));
    }
    std::vector<float*> rp(g);
    std::vector<unsigned long long*> cp(g);
    for (int q = 0; q < g; q++) {
        rp[q] = (float*)e->tp_peer[q];
        cp[q] = (unsigned long long*)((char*)e->tp_peer[q] + e->tp_recv_bytes + 256);
    }
    FL_CHECK_CUDA(cudaMalloc(&e->tp_recv_ptrs, sizeof(float*) * g));
    FL_CHECK_CUDA(cudaMalloc(&e->tp_cnt_ptrs, sizeof(unsigned long long*) * g));
    FL_CHECK_CUDA(cudaMalloc(&e->tp_seq, sizeof(unsigned long long)));
    FL_CHECK_CUDA(cudaMalloc(&e->tp_arrived, sizeof(int)));
    FL_CHECK_CUDA(cudaMemcpy(e->tp_recv_ptrs, rp.data(), sizeof(float*) * g, cudaMemcpyHostToDevice));
    FL_CHECK_CUDA(cudaMemcpy(e->tp_cnt_ptrs, cp.data(), sizeof(unsigned long long*) * g, cudaMemcpyHostToDevice));
    FL_CHECK_CUDA(cudaMemset(e->tp_seq, 0, sizeof(unsigned long long)));
    FL_CHECK_CUDA(cudaMemset(e->tp_arrived, 0, sizeof(int)));
    // The fused NVLink push (EPI_TP_PUSH + tp_reduce_kernel) is opt-in: at
    // TP 2 NCCL's all-reduce measured faster per decode step (5.69 against
    // 5.90 ms at Phi-3-medium shapes on B200).
    const char* v = getenv("FL_TP_FUSED");
    e->tp_fused = v && v[0] == '1';
    return FL_OK;
}

static fl_engine_t* engine_create(const fl_model_config_t* cfg, int device, int tp_rank, int tp_size,
                                  const unsigned char* tp_id) {
    if (!cfg) { set_error(FL_E_INVAL, "config is NULL"); return nullptr; }
    const fl_model_config_t& c = *cfg;
    if (c.hidden_size <= 0 || c.num_heads <= 0 || c.num_kv_heads <= 0 || c.head_dim <= 0 ||
        c.num_heads % c.num_kv_heads != 0 || c.hidden_size % 32 != 0 || c.intermediate_size % 32 != 0 ||
        (c.num_heads * c.head_dim) % 32 != 0 || c.head_dim % 2 != 0 || c.head_dim > 128 ||
        c.vocab_size <= 0 || c.num_layers < 0 || c.max_seq_len < 16 || c.draft_layers < 0 || c.medusa_heads < 0 ||
        (c.num_layers == 0 && c.draft_layers == 0 && c.medusa_heads == 0)) {
        set_error(FL_E_INVAL, "fl_engine_create: unsupported model configuration");
        return nullptr;
    }
    if (ensure_device() != FL_OK) return nullptr;
    if (cudaSetDevice(device) != cudaSuccess) { set_error(FL_E_NODEV, "cudaSetDevice failed"); return nullptr; }
    fl_engine* e = new fl_engine();
    e->c = c;
    {
        // FL_STEP_KERNEL=1: 128-byte panels and one persistent tcgen05 kernel
        // per speculative step; otherwise the multi-kernel step graph
        const char* sk = getenv("FL_STEP_KERNEL");
        e->step_layout = sk && sk[0] == '1';
    }
    e->device = device;
    e->d = c.hidden_size;
    e->H = c.num_heads;
    e->Hkv = c.num_kv_heads;
    e->hd = c.head_dim;
    e->qd = c.num_heads * c.head_dim;
    e->kd = c.num_kv_heads * c.head_dim;
    e->F = c.intermediate_size;
    e->V = c.vocab_size;
    e->Vg = c.vocab_size;
    e->R = c.max_seq_len;
    auto fail = [&](int) -> fl_engine_t* { fl_engine_destroy(e); return nullptr; };
    if (tp_size > 1) {
        // this rank's slice: local head, KV-head, feature and vocabulary counts
        if (c.medusa_heads > 0) return fail(set_error(FL_E_UNSUPPORTED, "tensor parallel: Medusa heads are not sharded"));
        if (tp_layout(c.num_heads, c.num_kv_heads, c.intermediate_size, c.vocab_size, tp_rank, tp_size, e->tp) != FL_OK)
            return fail(0);
        if ((e->tp.q0 * c.head_dim) % 32 || e->tp.f0 % 32 || e->tp.nf % 32)
            return fail(set_error(FL_E_INVAL, "tensor parallel: shard boundaries must fall on 32-element blocks"));
        e->tp_rank = tp_rank;
        e->tp_size = tp_size;
        e->step_layout = false;
        e->H = e->tp.nq;
        e->Hkv = e->tp.nkv;
        e->qd = e->tp.nq * c.head_dim;
        e->kd = e->tp.nkv * c.head_dim;
        e->F = e->tp.nf;
        e->V = e->tp.nv;
    }
    if (cudaStreamCreateWithFlags(&e->s, cudaStreamNonBlocking) != cudaSuccess) return fail(set_error(FL_E_CUDA, "stream"));
    if (tp_size > 1) {
        if (tp_comm_init(tp_rank, tp_size, tp_id, &e->tp_comm) != FL_OK) return fail(0);
        e->tp_rows = kMaxRows;
        if (cudaMalloc(&e->tp_keys, sizeof(unsigned long long) * kMaxRows) != cudaSuccess ||
            cudaMalloc(&e->tp_all, sizeof(unsigned long long) * kMaxRows * tp_size) != cudaSuccess ||
            cudaMalloc(&e->tp_best, sizeof(unsigned long long) * kMaxRows) != cudaSuccess)
            return fail(set_error(FL_E_NOMEM, "tensor parallel: key buffers"));
        if (tp_fused_setup(e) != FL_OK) return fail(0);
    }
    for (auto& ev : e->ev)
        if (cudaEventCreate(&ev) != cudaSuccess) return fail(set_error(FL_E_CUDA, "event"));
    if (alloc_stack(e, e->base, c.num_layers) != FL_OK) return fail(0);
    if (c.draft_layers > 0 && alloc_stack(e, e->draft, c.draft_layers) != FL_OK) return fail(0);
    if (alloc_linear(e->lm, e->V, e->d, 0x1u, e->step_layout) != FL_OK) return fail(0);
    e->medusa.resize(c.medusa_heads);
    for (auto& m : e->medusa)
        if (alloc_linear(m, e->d, e->d, 0x1u, e->step_layout) != FL_OK) return fail(0);
    const size_t R = e->R, d = e->d;
    const size_t wq = std::max(e->d, e->qd);
    e->nparts = gemv_auto_grid(e->V, e->d);
    bool ok = cudaMalloc(&e->embed, sizeof(float) * (size_t)e->Vg * d) == cudaSuccess &&
              cudaMalloc(&e->x, sizeof(float) * R * d) == cudaSuccess &&
              cudaMalloc(&e->x2, sizeof(float) * R * d) == cudaSuccess &&
              cudaMalloc(&e->xq, R * wq) == cudaSuccess &&
              cudaMalloc(&e->q, sizeof(float) * R * e->qd) == cudaSuccess &&
              cudaMalloc(&e->aq, R * e->qd) == cudaSuccess &&
              cudaMalloc(&e->hq, R * e->F) == cudaSuccess &&
              cudaMalloc(&e->logits, sizeof(float) * kMaxRows * e->V) == cudaSuccess &&
              cudaMalloc(&e->amax, sizeof(unsigned long long) * kMaxRows * e->nparts) == cudaSuccess &&
              cudaMalloc(&e->x_v, sizeof(float) * kMaxRows * d) == cudaSuccess &&
              cudaMalloc(&e->x_d, sizeof(float) * kMaxRows * d) == cudaSuccess &&
              cudaMalloc(&e->iota, sizeof(int) * (R + 16)) == cudaSuccess &&
              cudaMalloc(&e->tok, sizeof(int) * R) == cudaSuccess &&
              cudaMalloc(&e->st, sizeof(SpecState)) == cudaSuccess &&
              cudaMalloc(&e->st_snap, sizeof(SpecState)) == cudaSuccess &&
              cudaMalloc(&e->xd0_snap, sizeof(float) * d) == cudaSuccess &&
              cudaMalloc(&e->seq, sizeof(int) * (R + 16)) == cudaSuccess &&
              cudaMalloc(&e->out, sizeof(int) * (R + 16)) == cudaSuccess &&
              cudaMalloc(&e->acc, sizeof(int) * (R + 16)) == cudaSuccess &&
              cudaMalloc(&e->last_feat, sizeof(float) * d) == cudaSuccess &&
              cudaMalloc(&e->attn_part, sizeof(float) * attention_scratch_floats(e->H, e->hd, c.max_seq_len)) ==
                  cudaSuccess &&
              cudaMalloc(&e->attn_cnt, sizeof(int) * attention_scratch_counters(e->H)) == cudaSuccess &&
              cudaMalloc(&e->step_bar, sizeof(unsigned) * 4) == cudaSuccess &&
              cudaMemset(e->step_bar, 0, sizeof(unsigned) * 4) == cudaSuccess &&
              cudaMemset(e->attn_cnt, 0, sizeof(int) * attention_scratch_counters(e->H)) == cudaSuccess;
    if (!ok) return fail(set_error(FL_E_NOMEM, "fl_engine_create: device allocation failed"));
#if FL_ROPE_TABLE
    // Rotary (cos, sin) per context position and frequency, read by the QKV
    // epilogues instead of a powf and a sincosf per output pair (same values).
    e->rope_rows = c.max_seq_len + kMaxTreeCand;
    if (cudaMalloc(&e->rope, sizeof(float2) * (size_t)e->rope_rows * (e->hd / 2)) != cudaSuccess)
        return fail(set_error(FL_E_NOMEM, "fl_engine_create: rotary table"));
    if (launch_rope_table(e->rope, e->rope_rows, e->hd, c.rope_theta, e->s) != cudaSuccess ||
        cudaStreamSynchronize(e->s) != cudaSuccess)
        return fail(set_error(FL_E_CUDA, "fl_engine_create: rotary table"));
#endif
    std::vector<int> io(R + 16);
    for (size_t i = 0; i < io.size(); i++) io[i] = (int)i;
    if (cudaMemcpy(e->iota, io.data(), sizeof(int) * io.size(), cudaMemcpyHostToDevice) != cudaSuccess)
        return fail(set_error(FL_E_CUDA, "iota upload"));
    return e;
}

FL_API fl_engine_t* fl_engine_create(const fl_model_config_t* cfg, int device) {
    return engine_create(cfg, device, 0, 1, nullptr);
}

FL_API fl_engine_t* fl_engine_create_tp(const fl_model_config_t* cfg, int device, int tp_rank, int tp_size,
                                        const unsigned char* nccl_id) {
    if (tp_size < 1 || tp_rank < 0 || tp_rank >= tp_size || (tp_size > 1 && !nccl_id)) {
        set_error(FL_E_INVAL, "fl_engine_create_tp: bad rank, size or NCCL id");
        return nullptr;
    }
    return engine_create(cfg, device, tp_rank, tp_size, nccl_id);
}

FL_API int fl_engine_tp(const fl_engine_t* e, int* rank, int* size) {
    if (!e) return set_error(FL_E_INVAL, "engine is NULL");
    if (rank) *rank = e->tp_rank;
    if (size) *size = e->tp_size;
    return FL_OK;
}

FL_API void fl_engine_destroy(fl_engine_t* e) {
    if (!e) return;
    cudaSetDevice(e->device);
    if (e->s) cudaStreamSynchronize(e->s);
    if (e->step_exec) cudaGraphExecDestroy(e->step_exec);
    batch_free(e);
    free_stack(e->base);
    free_stack(e->draft);
    free_linear(e->lm);
    for (auto& m : e->medusa) free_linear(m);
    void* bufs[] = {e->embed, e->x, e->x2, e->xq, e->q, e->aq, e->hq, e->logits, e->amax, e->x_v, e->x_d,
                    e->iota, e->tok, e->mask, e->work_arena, e->st, e->st_snap, e->xd0_snap, e->seq, e->out, e->acc,
                    e->last_feat, e->attn_part, e->attn_cnt, e->rope, e->step_bar, e->d_phases, e->d_trace,
                    e->samp_q, e->samp_p, e->samp_r, e->samp_trace, e->samp_snap, e->samp_m, e->samp_key,
                    e->tp_keys, e->tp_all, e->tp_best, e->tp_recv_ptrs, e->tp_cnt_ptrs, e->tp_seq, e->tp_arrived};
    for (void* p : bufs) cudaFree(p);
    for (int q = 0; q < (int)e->tp_peer.size(); q++)
        if (q != e->tp_rank && e->tp_peer[q]) cudaIpcCloseMemHandle(e->tp_peer[q]);
    cudaFree(e->tp_region);
    tp_comm_free(e->tp_comm);
    for (auto& ev : e->ev)
        if (ev) cudaEventDestroy(ev);
    if (e->s) cudaStreamDestroy(e->s);
    delete e;
}

static int load_linear_local(fl_engine_t* e, int stack, int layer, int proj, const int8_t* w, const uint16_t* d,
                             int rows, int cols) {
    if (stack == 3) {
        if (proj != 1 || rows != e->V) return set_error(FL_E_INVAL, "load_linear: shared stack takes the LM head (proj 1)");
        FL_CHECK(put_rows(e->lm, 0, 1, w, d, rows, cols, e->s));
        e->lm.have |= 1u;
        return FL_OK;
    }
    if (stack == 2) {
        if (layer < 0 || layer >= (int)e->medusa.size() || proj != 0 || rows != e->d)
            return set_error(FL_E_INVAL, "load_linear: bad Medusa head");
        FL_CHECK(put_rows(e->medusa[layer], 0, 1, w, d, rows, cols, e->s));
        e->medusa[layer].have |= 1u;
        return FL_OK;
    }
    if (stack != 0 && stack != 1) return set_error(FL_E_INVAL, "load_linear: bad stack");
    Stack& S = stack == 0 ? e->base : e->draft;
    if (layer < 0 || layer >= S.nl) return set_error(FL_E_INVAL, "load_linear: bad layer");
    LayerW& W = S.L[layer];
    switch (proj) {
        case 0:
            if (rows != e->qd) return set_error(FL_E_INVAL, "load_linear: q rows");
            FL_CHECK(put_rows(W.qkv, 0, 1, w, d, rows, cols, e->s));
            W.qkv.have |= 1u;
            return FL_OK;
        case 1:
        case 2:
            if (rows != e->kd) return set_error(FL_E_INVAL, "load_linear: k/v rows");
            FL_CHECK(put_rows(W.qkv, e->qd + (proj == 2 ? e->kd : 0), 1, w, d, rows, cols, e->s));
            W.qkv.have |= (proj == 1 ? 2u : 4u);
            return FL_OK;
        case 3:
            if (rows != e->d) return set_error(FL_E_INVAL, "load_linear: o rows");
            FL_CHECK(put_rows(W.o, 0, 1, w, d, rows, cols, e->s));
            W.o.have |= 1u;
            return FL_OK;
        case 4:
        case 5:
            if (rows != e->F) return set_error(FL_E_INVAL, "load_linear: gate/up rows");
            FL_CHECK(put_rows(W.gu, proj == 4 ? 0 : 1, 2, w, d, rows, cols, e->s));
            W.gu.have |= (proj == 4 ? 1u : 2u);
            return FL_OK;
        case 6:
            if (rows != e->d) return set_error(FL_E_INVAL, "load_linear: down rows");
            FL_CHECK(put_rows(W.down, 0, 1, w, d, rows, cols, e->s));
            W.down.have |= 1u;
            return FL_OK;
        default:
            return set_error(FL_E_INVAL, "load_linear: bad projection");
    }
}

// Under tensor parallelism the caller passes every tensor whole (as a loader
// reads it) and the rank keeps its slice: rows of Q, K, V, gate, up and the LM
// head, columns of o and down.
FL_API int fl_engine_load_linear(fl_engine_t* e, int stack, int layer, int proj, const int8_t* w,
                                 const uint16_t* d, int rows, int cols) {
    if (!e || !w || !d) return set_error(FL_E_INVAL, "load_linear: NULL argument");
    FL_CHECK_CUDA(cudaSetDevice(e->device));
    if (e->tp_size == 1 || cols % 32) return load_linear_local(e, stack, layer, proj, w, d, rows, cols);
    const TpLayout& L = e->tp;
    const int hd = e->hd;
    auto row_slice = [&](int full_rows, int r0, int nr) -> int {
        if (rows != full_rows) return set_error(FL_E_INVAL, "load_linear: pass the whole tensor to every rank");
        return load_linear_local(e, stack, layer, proj, w + (size_t)r0 * cols, d + (size_t)r0 * (cols / 32), nr, cols);
    };
    auto col_slice = [&](int full_cols, int c0, int nc) -> int {
        if (cols != full_cols || rows != e->d) return set_error(FL_E_INVAL, "load_linear: pass the whole tensor to every rank");
        std::vector<int8_t> ws((size_t)rows * nc);
        std::vector<uint16_t> ds((size_t)rows * (nc / 32));
        for (int r = 0; r < rows; r++) {
            memcpy(ws.data() + (size_t)r * nc, w + (size_t)r * cols + c0, (size_t)nc);
            memcpy(ds.data() + (size_t)r * (nc / 32), d + (size_t)r * (cols / 32) + c0 / 32, sizeof(uint16_t) * (nc / 32));
        }
        return load_linear_local(e, stack, layer, proj, ws.data(), ds.data(), rows, nc);
    };
    const int Hg = e->c.num_heads, Hkvg = e->c.num_kv_heads, Fg = e->c.intermediate_size;
    if (stack == 3) return row_slice(e->Vg, L.v0, L.nv);
    if (stack != 0 && stack != 1) return set_error(FL_E_INVAL, "load_linear: bad stack for a tensor-parallel engine");
    switch (proj) {
        case 0: return row_slice(Hg * hd, L.q0 * hd, L.nq * hd);
        case 1:
        case 2: return row_slice(Hkvg * hd, L.kv0 * hd, L.nkv * hd);
        case 3: return col_slice(Hg * hd, L.q0 * hd, L.nq * hd);
        case 4:
        case 5: return row_slice(Fg, L.f0, L.nf);
        case 6: return col_slice(Fg, L.f0, L.nf);
        default: return set_error(FL_E_INVAL, "load_linear: bad projection");
    }
}

FL_API int fl_engine_load_embedding(fl_engine_t* e, const float* table) {
    if (!e || !table) return set_error(FL_E_INVAL, "load_embedding: NULL argument");
    FL_CHECK_CUDA(cudaSetDevice(e->device));
    FL_CHECK_CUDA(cudaMemcpy(e->embed, table, sizeof(float) * (size_t)e->Vg * e->d, cudaMemcpyHostToDevice));
    e->embed_loaded = true;
    return FL_OK;
}

// Whole-model widths (hidden, q_dim, kv_dim, ffn), not a rank's slice.
FL_API int fl_engine_dims(const fl_engine_t* e, int* out) {
    if (!e || !out) return set_error(FL_E_INVAL, "engine_dims: NULL");
    out[0] = e->c.hidden_size;
    out[1] = e->c.num_heads * e->c.head_dim;
    out[2] = e->c.num_kv_heads * e->c.head_dim;
    out[3] = e->c.intermediate_size;
    return FL_OK;
}

FL_API int fl_engine_ready(const fl_engine_t* e) {
    if (!e || !e->embed_loaded || !linear_ready(e->lm)) return 0;
    if (!stack_ready(e->base) || !stack_ready(e->draft)) return 0;
    for (const auto& m : e->medusa)
        if (!linear_ready(m)) return 0;
    return 1;
}

// Tensor-parallel rank: generates only its slice of every tensor (each
// element is a pure function of the seed, the tensor id and its index).
static int synthesize_tp(fl_engine_t* e, uint64_t seed) {
    const TpLayout& L = e->tp;
    const int d = e->d, hd = e->hd, Hg = e->c.num_heads, Hkvg = e->c.num_kv_heads, Fg = e->c.intermediate_size;
    const float stdv = 0.02f;
    std::vector<int8_t> w;
    std::vector<uint16_t> sc;
    auto gen = [&](int stack, int layer, int proj, int rows, int cols, int r0, int nr, int c0, int nc) -> int {
        w.resize((size_t)nr * nc);
        sc.resize((size_t)nr * nc / 32);
        const int rc = fl_synth_q4_0_i8_block(seed, FL_TENSOR_ID(stack, layer, proj), rows, cols, r0, nr, c0, nc, stdv,
                                              w.data(), sc.data());
        if (rc != FL_OK) return set_error(rc, "synth failed");
        return load_linear_local(e, stack, layer, proj, w.data(), sc.data(), nr, nc);
    };
    for (int s = 0; s < 2; s++) {
        const Stack& S = s == 0 ? e->base : e->draft;
        for (int l = 0; l < S.nl; l++) {
            FL_CHECK(gen(s, l, 0, Hg * hd, d, L.q0 * hd, L.nq * hd, 0, d));
            FL_CHECK(gen(s, l, 1, Hkvg * hd, d, L.kv0 * hd, L.nkv * hd, 0, d));
            FL_CHECK(gen(s, l, 2, Hkvg * hd, d, L.kv0 * hd, L.nkv * hd, 0, d));
            FL_CHECK(gen(s, l, 3, d, Hg * hd, 0, d, L.q0 * hd, L.nq * hd));
            FL_CHECK(gen(s, l, 4, Fg, d, L.f0, L.nf, 0, d));
            FL_CHECK(gen(s, l, 5, Fg, d, L.f0, L.nf, 0, d));
            FL_CHECK(gen(s, l, 6, d, Fg, 0, d, L.f0, L.nf));
        }
    }
    FL_CHECK(gen(3, 0, 1, e->Vg, d, L.v0, L.nv, 0, d));
    std::vector<float> emb((size_t)e->Vg * d);
    FL_CHECK(fl_synth_q4_0_f32(seed, FL_TENSOR_ID(3, 0, 0), e->Vg, d, stdv, emb.data()));
    return fl_engine_load_embedding(e, emb.data());
}

FL_API int fl_engine_synthesize(fl_engine_t* e, uint64_t seed) {
    if (!e) return set_error(FL_E_INVAL, "engine is NULL");
    if (e->tp_size > 1) return synthesize_tp(e, seed);
    const int d = e->d, qd = e->qd, kd = e->kd, F = e->F, V = e->V;
    const size_t maxel = std::max({(size_t)V * d, (size_t)2 * F * d, (size_t)qd * d});
    std::vector<int8_t> w(maxel);
    std::vector<uint16_t> sc(maxel / 32);
    const float stdv = 0.02f;
    auto gen = [&](int stack, int layer, int proj, int rows, int cols) -> int {
        int rc = fl_synth_q4_0_i8(seed, FL_TENSOR_ID(stack, layer, proj), rows, cols, stdv, w.data(), sc.data());
        if (rc != FL_OK) return set_error(rc, "synth failed");
        return fl_engine_load_linear(e, stack, layer, proj, w.data(), sc.data(), rows, cols);
    };
    for (int s = 0; s < 2; s++) {
        const Stack& S = s == 0 ? e->base : e->draft;
        for (int l = 0; l < S.nl; l++) {
            FL_CHECK(gen(s, l, 0, qd, d));
            FL_CHECK(gen(s, l, 1, kd, d));
            FL_CHECK(gen(s, l, 2, kd, d));
            FL_CHECK(gen(s, l, 3, d, qd));
            FL_CHECK(gen(s, l, 4, F, d));
            FL_CHECK(gen(s, l, 5, F, d));
            FL_CHECK(gen(s, l, 6, d, F));
        }
    }
    for (int h = 0; h < (int)e->medusa.size(); h++) FL_CHECK(gen(2, h, 0, d, d));
    FL_CHECK(gen(3, 0, 1, V, d));
    std::vector<float> emb((size_t)V * d);
    FL_CHECK(fl_synth_q4_0_f32(seed, FL_TENSOR_ID(3, 0, 0), V, d, stdv, emb.data()));
    return fl_engine_load_embedding(e, emb.data());
}

FL_API int fl_engine_forward_rows(fl_engine_t* e, int stack, const float* x_in, int M, int base, const int* pos,
                                  const uint8_t* mask, float* x_out, float* logits) {
    FL_CHECK(check_ready(e, stack == 1));
    if (!x_in || !pos || M <= 0 || base < 0 || base + M > e->R) return set_error(FL_E_INVAL, "forward_rows: bad arguments");
    if (stack != 0 && stack != 1) return set_error(FL_E_INVAL, "forward_rows: stack must be 0 or 1");
    if (logits && e->tp_size > 1)
        return set_error(FL_E_UNSUPPORTED, "forward_rows: a tensor-parallel rank holds a slice of the logits");
    Stack& S = stack == 0 ? e->base : e->draft;
    const size_t xb = sizeof(float) * (size_t)M * e->d;
    FL_CHECK_CUDA(cudaMemcpyAsync(e->x, x_in, xb, cudaMemcpyHostToDevice, e->s));
    FL_CHECK_CUDA(cudaMemcpyAsync(e->tok, pos, sizeof(int) * M, cudaMemcpyHostToDevice, e->s));
    const uint8_t* dmask = nullptr;
    if (mask) {
        FL_CHECK(ensure_mask(e, M));
        FL_CHECK_CUDA(cudaMemcpyAsync(e->mask, mask, (size_t)M * M, cudaMemcpyHostToDevice, e->s));
        dmask = e->mask;
    }
    FL_CHECK(run_stack(e, S, e->x, M, nullptr, e->iota + base, e->tok, dmask, nullptr, false));
    if (x_out) FL_CHECK_CUDA(cudaMemcpyAsync(x_out, e->x, xb, cudaMemcpyDeviceToHost, e->s));
    if (logits) {
        for (int r0 = 0; r0 < M; r0 += kMaxRows) {
            const int m = std::min(kMaxRows, M - r0);
            FL_CHECK(run_lm(e, e->x + (size_t)r0 * e->d, m, nullptr, nullptr, false));
            FL_CHECK_CUDA(cudaMemcpyAsync(logits + (size_t)r0 * e->V, e->logits, sizeof(float) * (size_t)m * e->V,
                                          cudaMemcpyDeviceToHost, e->s));
        }
    }
    FL_CHECK_CUDA(cudaStreamSynchronize(e->s));
    return FL_OK;
}

FL_API int fl_engine_greedy_generate(fl_engine_t* e, const int* prompt, int P, int n_new, int* out) {
    FL_CHECK(check_ready(e, false));
    if (!prompt || !out || P <= 0 || n_new <= 0 || P + n_new + 1 > e->R)
        return set_error(FL_E_INVAL, "greedy_generate: bad arguments or context too long");
    FL_CHECK(prefill_base(e, prompt, P));
    for (int i = 1; i < n_new; i++) {
        const int n = P + i - 1;  // seq[n] is the newest token
        FL_CHECK_CUDA(launch_embed_rows(e->embed, e->Vg, e->seq + n, nullptr, 0, e->x_v, e->d, 1, nullptr, nullptr, e->s, false));
        FL_CHECK(run_stack(e, e->base, e->x_v, 1, nullptr, e->iota + n, e->iota + n, nullptr, nullptr, false));
        FL_CHECK(run_lm(e, e->x_v, 1, nullptr, nullptr, false));
        FL_CHECK_CUDA(launch_argmax_rows(amax_keys(e), amax_nparts(e), 1, e->seq + n + 1, nullptr, e->s));
    }
    FL_CHECK_CUDA(cudaMemcpyAsync(out, e->seq + P, sizeof(int) * n_new, cudaMemcpyDeviceToHost, e->s));
    FL_CHECK_CUDA(cudaStreamSynchronize(e->s));
    return FL_OK;
}

namespace {
// Saves (save) or restores the draft state of step 0 that the prefill leaves
// behind: kept mass, weights and, with the trace on, the logits row.
int sample_snapshot(fl_engine* e, bool save) {
    const size_t V = e->V;
    unsigned char* s = e->samp_snap;
    struct Part { void* live; unsigned char* snap; size_t bytes; } parts[3] = {
        {e->samp_m, s, 8}, {e->samp_q, s + 8, 4 * V}, {e->samp_trace, s + 8 + 4 * V, 4 * V}};
    for (int i = 0; i < (e->trace_on ? 3 : 2); i++) {
        void* dst = save ? (void*)parts[i].snap : parts[i].live;
        const void* src = save ? (const void*)parts[i].live : (const void*)parts[i].snap;
        FL_CHECK_CUDA(cudaMemcpyAsync(dst, src, parts[i].bytes, cudaMemcpyDeviceToDevice, e->s));
    }
    return FL_OK;
}

// The step graph holds the rule, its key and the trace pointer by value:
// drop it so that the next prefill records it again.
int drop_step_graph(fl_engine* e) {
    e->spec_ready = 0;
    if (e->step_exec) {
        FL_CHECK_CUDA(cudaStreamSynchronize(e->s));
        cudaGraphExecDestroy(e->step_exec);
        e->step_exec = nullptr;
    }
    e->graph_K = -1;
    return FL_OK;
}
}  // namespace

FL_API int fl_engine_set_weight_bits(fl_engine_t* e, int bits) {
    if (!e) return set_error(FL_E_INVAL, "engine is NULL");
    if (bits != 4 && bits != 8) return set_error(FL_E_INVAL, "set_weight_bits: 4 or 8");
    FL_CHECK(check_ready(e, false));
    FL_CHECK(drop_step_graph(e));
    if (e->bt.exec) {
        FL_CHECK_CUDA(cudaStreamSynchronize(e->s));
        cudaGraphExecDestroy(e->bt.exec);
        e->bt.exec = nullptr;
        e->bt.ready = false;
    }
    std::vector<Linear*> all;
    for (Stack* S : {&e->base, &e->draft})
        for (auto& W : S->L) all.insert(all.end(), {&W.qkv, &W.o, &W.gu, &W.down});
    all.push_back(&e->lm);
    for (auto& m : e->medusa) all.push_back(&m);
    FL_CHECK_CUDA(cudaStreamSynchronize(e->s));
    for (Linear* l : all) {
        cudaFree(l->w4);
        l->w4 = nullptr;
    }
    if (bits == 8) return FL_OK;
    int* bad = nullptr;
    FL_CHECK_CUDA(cudaMalloc(&bad, sizeof(int)));
    int rc = FL_OK;
    cudaError_t ce = cudaMemsetAsync(bad, 0, sizeof(int), e->s);
    for (Linear* l : all) {
        if (ce != cudaSuccess || !l->w || !w4_supported(l->N, l->K, l->P)) continue;
        ce = cudaMalloc(&l->w4, (size_t)l->N * l->K / 2);
        if (ce == cudaSuccess) ce = launch_pack_w4(l->w, l->w4, l->N, l->K, l->P, bad, e->s);
    }
    int hbad = 0;
    if (ce == cudaSuccess) ce = cudaMemcpyAsync(&hbad, bad, sizeof(int), cudaMemcpyDeviceToHost, e->s);
    if (ce == cudaSuccess) ce = cudaStreamSynchronize(e->s);
    cudaFree(bad);
    if (ce != cudaSuccess) rc = cuda_error(ce, "set_weight_bits");
    else if (hbad) rc = set_error(FL_E_INVAL, "set_weight_bits: a weight lies outside [-8, 7]");
    if (rc != FL_OK)
        for (Linear* l : all) {
            cudaFree(l->w4);
            l->w4 = nullptr;
        }
    return rc;
}

FL_API int fl_engine_spec_prefill(fl_engine_t* e, const int* prompt, int P, int K, int max_acc) {
    FL_CHECK(check_ready(e, true));
    if (!prompt || P <= 0 || K < 1 || K > kMaxDraft || P + 2 > e->R)
        return set_error(FL_E_INVAL, "spec_prefill: bad arguments (1 <= K <= 7)");
    e->spec_ready = 0;
    e->spec_K = K;
    e->spec_P = P;
    FL_CHECK(prefill_base(e, prompt, P));
    // sampling: the first token is drawn from the last prompt row's logits
    if (e->samp) FL_CHECK_CUDA(launch_sample_first(step_buffers(e), P, e->s));
    // Draft catch-up over positions 0..P: x_i = F_{i-1} + E[t_i], F_{-1} = 0.
    FL_CHECK_CUDA(launch_embed_rows(e->embed, e->Vg, e->seq, e->x, 1, e->x2, e->d, P + 1, nullptr, nullptr, e->s, false));
    FL_CHECK(run_stack(e, e->draft, e->x2, P + 1, nullptr, e->iota, e->iota, nullptr, nullptr, false));
    FL_CHECK_CUDA(cudaMemcpyAsync(e->x_d, e->x2 + (size_t)P * e->d, sizeof(float) * e->d, cudaMemcpyDeviceToDevice, e->s));
    SpecState h = {};
    h.n = P;
    h.produced = 1;
    h.n_new = 1;
    h.done = 0;
    h.K = K;
    h.max_acc = max_acc < 0 ? K : std::min(max_acc, K);
    h.one = 1;
    h.rows = 1;
    h.last_row = 0;
    FL_CHECK_CUDA(cudaMemcpyAsync(e->st, &h, sizeof(h), cudaMemcpyHostToDevice, e->s));
    FL_CHECK_CUDA(cudaMemcpyAsync(e->out, e->seq + P, sizeof(int), cudaMemcpyDeviceToDevice, e->s));
    FL_CHECK(run_lm(e, e->x_d, 1, nullptr, nullptr, false));
    if (e->samp)
        FL_CHECK_CUDA(launch_sample_pick(step_buffers(e), 0, e->s, false));
    else
        FL_CHECK_CUDA(launch_draft_pick(step_buffers(e), 0, e->s, false));
    FL_CHECK_CUDA(cudaMemcpyAsync(e->st_snap, e->st, sizeof(SpecState), cudaMemcpyDeviceToDevice, e->s));
    FL_CHECK_CUDA(cudaMemcpyAsync(e->xd0_snap, e->x_d, sizeof(float) * e->d, cudaMemcpyDeviceToDevice, e->s));
    if (e->samp) FL_CHECK(sample_snapshot(e, true));
    FL_CHECK_CUDA(cudaStreamSynchronize(e->s));
    FL_CHECK(build_step_graph(e));
    e->spec_ready = 1;
    return FL_OK;
}


FL_API int fl_engine_set_sampling(fl_engine_t* e, float temperature, float top_p, unsigned seed,
                                  unsigned seq_id) {
    if (!e) return set_error(FL_E_INVAL, "engine is NULL");
    if (!(temperature <= 0.0f) && !(top_p > 0.0f && top_p <= 1.0f))
        return set_error(FL_E_INVAL, "set_sampling: top_p must be in (0, 1]");
    if (!(temperature <= 0.0f) && !(temperature < INFINITY))
        return set_error(FL_E_INVAL, "set_sampling: temperature must be finite");
    FL_CHECK_CUDA(cudaSetDevice(e->device));
    const bool samp = temperature > 0.0f;
    if (samp && e->tp_size > 1)
        return set_error(FL_E_UNSUPPORTED, "set_sampling: a tensor-parallel engine decodes greedily (its logits are split)");
    if (samp == e->samp && (!samp || (temperature == e->samp_T && top_p == e->samp_top_p &&
                                      seed == e->samp_seed && seq_id == e->samp_seq)))
        return FL_OK;  // unchanged
    if (samp && e->samp && temperature == e->samp_T && top_p == e->samp_top_p) {
        // a new key only: the step graph reads it from device memory; the
        // post-prefill state was drawn with the old key, so prefill again
        const uint32_t key[2] = {seed, seq_id};
        FL_CHECK_CUDA(cudaMemcpyAsync(e->samp_key, key, sizeof(key), cudaMemcpyHostToDevice, e->s));
        FL_CHECK_CUDA(cudaStreamSynchronize(e->s));
        e->samp_seed = seed;
        e->samp_seq = seq_id;
        e->spec_ready = 0;
        return FL_OK;
    }
    if (samp && !e->samp_q) {
        FL_CHECK_CUDA(cudaMalloc(&e->samp_q, sizeof(uint32_t) * (size_t)kMaxDraft * e->V));
        FL_CHECK_CUDA(cudaMalloc(&e->samp_p, sizeof(uint32_t) * (size_t)kMaxRows * e->V));
        FL_CHECK_CUDA(cudaMalloc(&e->samp_m, sizeof(unsigned long long) * (kMaxDraft + kMaxRows)));
        FL_CHECK_CUDA(cudaMalloc(&e->samp_r, sizeof(unsigned long long) * (size_t)e->V));
        FL_CHECK_CUDA(cudaMalloc(&e->samp_snap, 8 + (size_t)8 * e->V));
        FL_CHECK_CUDA(cudaMalloc(&e->samp_key, sizeof(uint32_t) * 2));
    }
    e->samp = samp;
    e->samp_T = samp ? temperature : 0.0f;
    e->samp_top_p = samp ? top_p : 1.0f;
    e->samp_seed = seed;
    e->samp_seq = seq_id;
    if (samp) {
        const uint32_t key[2] = {seed, seq_id};
        FL_CHECK_CUDA(cudaMemcpy(e->samp_key, key, sizeof(key), cudaMemcpyHostToDevice));
    }
    return drop_step_graph(e);
}

FL_API int fl_engine_sample_trace_enable(fl_engine_t* e, int on) {
    if (!e) return set_error(FL_E_INVAL, "engine is NULL");
    if ((on != 0) == e->trace_on) return FL_OK;
    FL_CHECK_CUDA(cudaSetDevice(e->device));
    if (on && !e->samp_trace)
        FL_CHECK_CUDA(cudaMalloc(&e->samp_trace, sizeof(float) * (size_t)2 * kMaxRows * e->V));
    e->trace_on = on != 0;
    return drop_step_graph(e);
}

FL_API int fl_engine_sample_trace(const fl_engine_t* e, float* logits, unsigned* qd, unsigned long long* qm,
                                  unsigned* pt, unsigned long long* pm, int* drafted) {
    if (!e) return set_error(FL_E_INVAL, "engine is NULL");
    if (!e->trace_on || !e->samp_q) return set_error(FL_E_STATE, "sample_trace: enable the trace and sampling first");
    FL_CHECK_CUDA(cudaSetDevice(e->device));
    FL_CHECK_CUDA(cudaStreamSynchronize(e->s));
    const size_t V = e->V;
    if (logits) FL_CHECK_CUDA(cudaMemcpy(logits, e->samp_trace, sizeof(float) * 2 * kMaxRows * V, cudaMemcpyDeviceToHost));
    if (qd) FL_CHECK_CUDA(cudaMemcpy(qd, e->samp_q, sizeof(uint32_t) * kMaxDraft * V, cudaMemcpyDeviceToHost));
    if (pt) FL_CHECK_CUDA(cudaMemcpy(pt, e->samp_p, sizeof(uint32_t) * kMaxRows * V, cudaMemcpyDeviceToHost));
    if (qm) FL_CHECK_CUDA(cudaMemcpy(qm, e->samp_m, sizeof(unsigned long long) * kMaxDraft, cudaMemcpyDeviceToHost));
    if (pm)
        FL_CHECK_CUDA(cudaMemcpy(pm, e->samp_m + kMaxDraft, sizeof(unsigned long long) * kMaxRows, cudaMemcpyDeviceToHost));
    if (drafted) {
        SpecState h;
        FL_CHECK_CUDA(cudaMemcpy(&h, e->st, sizeof(h), cudaMemcpyDeviceToHost));
        memcpy(drafted, h.drafted, sizeof(int) * kMaxDraft);
    }
    return FL_OK;
}

FL_API int fl_engine_get_sampling(const fl_engine_t* e, float* temperature, float* top_p, unsigned* seed,
                                  unsigned* seq_id) {
    if (!e) return set_error(FL_E_INVAL, "engine is NULL");
    if (temperature) *temperature = e->samp_T;
    if (top_p) *top_p = e->samp_top_p;
    if (seed) *seed = e->samp_seed;
    if (seq_id) *seq_id = e->samp_seq;
    return FL_OK;
}

FL_API int fl_engine_spec_begin(fl_engine_t* e, int n_new) {
    FL_CHECK(check_ready(e, true));
    if (!e->spec_ready) return set_error(FL_E_STATE, "spec_decode: call fl_engine_spec_prefill first");
    if (n_new <= 0 || e->spec_P + n_new + e->spec_K + 2 > e->R)
        return set_error(FL_E_INVAL, "spec_decode: context too long");
    FL_CHECK_CUDA(cudaMemcpyAsync(e->st, e->st_snap, sizeof(SpecState), cudaMemcpyDeviceToDevice, e->s));
    FL_CHECK_CUDA(cudaMemcpyAsync(e->x_d, e->xd0_snap, sizeof(float) * e->d, cudaMemcpyDeviceToDevice, e->s));
    // the step-0 draft weights are part of the saved state
    if (e->samp) FL_CHECK(sample_snapshot(e, false));
    const int patch[2] = {n_new, n_new <= 1 ? 1 : 0};
    FL_CHECK_CUDA(cudaMemcpyAsync(&e->st->n_new, patch, sizeof(patch), cudaMemcpyHostToDevice, e->s));
    return FL_OK;
}

FL_API int fl_engine_spec_step(fl_engine_t* e, int* state) {
    FL_CHECK(check_ready(e, true));
    if (!e->spec_ready || !e->step_exec) return set_error(FL_E_STATE, "spec_step: call fl_engine_spec_begin first");
    FL_CHECK_CUDA(cudaGraphLaunch(e->step_exec, e->s));
    SpecState h;
    FL_CHECK_CUDA(cudaMemcpyAsync(&h, e->st, sizeof(h), cudaMemcpyDeviceToHost, e->s));
    FL_CHECK_CUDA(cudaStreamSynchronize(e->s));
    if (take_device_error() != 0) return set_error(FL_E_TIMEOUT, "spec_step: a bounded device wait gave up");
    if (state) {
        state[0] = h.n;
        state[1] = h.produced;
        state[2] = h.steps;
        state[3] = h.a_last;
        state[4] = h.done;
    }
    return FL_OK;
}

FL_API int fl_engine_spec_decode(fl_engine_t* e, int n_new, int* out, int* acc_hist, int* steps) {
    FL_CHECK(fl_engine_spec_begin(e, n_new));
    const int K = e->spec_K;
    FL_CHECK_CUDA(cudaEventRecord(e->ev[0], e->s));
    SpecState h = {};
    int produced = 1;
    long long launched = 0;
    while (produced < n_new) {
        const int batch = (n_new - produced + K) / (K + 1);
        for (int i = 0; i < batch; i++) FL_CHECK_CUDA(cudaGraphLaunch(e->step_exec, e->s));
        launched += batch;
        FL_CHECK_CUDA(cudaMemcpyAsync(&h, e->st, sizeof(h), cudaMemcpyDeviceToHost, e->s));
        FL_CHECK_CUDA(cudaStreamSynchronize(e->s));
        if (h.produced <= produced) {
            unsigned err = 0;
            if (e->step_kernel && cudaMemcpy(&err, e->step_bar + 2, sizeof(unsigned), cudaMemcpyDeviceToHost) == cudaSuccess &&
                err) {
                cudaMemset(e->step_bar, 0, sizeof(unsigned) * 4);
                return set_error(FL_E_TIMEOUT, "spec_decode: a bounded wait of the step kernel gave up");
            }
            return set_error(FL_E_STATE, "spec_decode: no progress");
        }
        produced = h.produced;
    }
    FL_CHECK_CUDA(cudaEventRecord(e->ev[1], e->s));
    FL_CHECK_CUDA(cudaEventSynchronize(e->ev[1]));
    if (take_device_error() != 0) return set_error(FL_E_TIMEOUT, "spec_decode: a bounded device wait gave up");
    if (e->step_kernel) {
        unsigned err = 0;
        FL_CHECK_CUDA(cudaMemcpy(&err, e->step_bar + 2, sizeof(unsigned), cudaMemcpyDeviceToHost));
        if (err) {
            cudaMemset(e->step_bar, 0, sizeof(unsigned) * 4);
            return set_error(FL_E_TIMEOUT, "spec_decode: a bounded wait of the step kernel gave up");
        }
    }
    float ms = 0.0f;
    cudaEventElapsedTime(&ms, e->ev[0], e->ev[1]);
    e->t_total_us = ms * 1000.0;
    e->last_launches = (long long)launched * e->graph_kernels;
    if (out) FL_CHECK_CUDA(cudaMemcpy(out, e->out, sizeof(int) * n_new, cudaMemcpyDeviceToHost));
    if (acc_hist) FL_CHECK_CUDA(cudaMemcpy(acc_hist, e->acc, sizeof(int) * h.steps, cudaMemcpyDeviceToHost));
    if (steps) *steps = h.steps;
    return FL_OK;
}

FL_API int fl_engine_spec_generate(fl_engine_t* e, const int* prompt, int P, int n_new, int K, int max_acc,
                                   int* out, int* acc_hist, int* steps) {
    FL_CHECK(fl_engine_spec_prefill(e, prompt, P, K, max_acc));
    return fl_engine_spec_decode(e, n_new, out, acc_hist, steps);
}

FL_API int fl_engine_last_timing(const fl_engine_t* e, double* draft_us, double* verify_us, double* total_us) {
    if (!e) return set_error(FL_E_INVAL, "engine is NULL");
    if (draft_us) *draft_us = e->t_draft_us;
    if (verify_us) *verify_us = e->t_verify_us;
    if (total_us) *total_us = e->t_total_us;
    return FL_OK;
}

FL_API void* fl_engine_stream(const fl_engine_t* e) { return e ? (void*)e->s : nullptr; }

FL_API long long fl_engine_last_launches(const fl_engine_t* e) { return e ? e->last_launches : -1; }

FL_API int fl_engine_step_kernel(const fl_engine_t* e) { return e && e->step_kernel ? 1 : 0; }

FL_API int fl_engine_step_trace_stages(const fl_engine_t* e, unsigned long long* t) {
    if (!e) return set_error(FL_E_INVAL, "engine is NULL");
    if (!e->step_kernel || !e->d_trace || !t) return 0;
    FL_CHECK_CUDA(cudaSetDevice(e->device));
    FL_CHECK_CUDA(cudaStreamSynchronize(e->s));
    FL_CHECK_CUDA(cudaMemcpy(t, e->d_trace + 6 * (size_t)e->n_phases, sizeof(unsigned long long) * 512,
                             cudaMemcpyDeviceToHost));
    return 64;
}

FL_API int fl_engine_step_trace(const fl_engine_t* e, unsigned long long* t, int* desc, int cap) {
    if (!e) return set_error(FL_E_INVAL, "engine is NULL");
    if (!e->step_kernel || !e->d_trace) return 0;
    const int n = e->n_phases < cap ? e->n_phases : cap;
    if (n <= 0) return 0;
    FL_CHECK_CUDA(cudaSetDevice(e->device));
    FL_CHECK_CUDA(cudaStreamSynchronize(e->s));
    if (t) FL_CHECK_CUDA(cudaMemcpy(t, e->d_trace, sizeof(unsigned long long) * 6 * n, cudaMemcpyDeviceToHost));
    if (desc) memcpy(desc, e->phase_desc.data(), sizeof(int) * 4 * n);
    return n;
}

FL_API int fl_engine_draft_bound(const fl_engine_t* e, const void* draft) { return e && e->bound_draft == draft; }
FL_API void fl_engine_note_draft(fl_engine_t* e, const void* draft) {
    if (e) e->bound_draft = draft;
}

// Times one projection of every layer of a stack (kind 0 qkv, 1 o, 2
// gate/up, 3 down) as captured back-to-back GEMV launches at M rows: the
// per-launch device time and the algorithmic bytes of one launch (int8
// weights + fp16 scales + activations in + outputs). The layers' weights
// together exceed L2 for the full-size model.
FL_API int fl_engine_bench_linear(fl_engine_t* e, int stack, int kind, int M, int reps, double* us_per_launch,
                                  double* bytes_per_launch) {
    FL_CHECK(check_ready(e, stack == 1));
    if (kind < 0 || kind > 3 || M < 1 || M > e->R || reps < 1) return set_error(FL_E_INVAL, "bench_linear: bad arguments");
    Stack& S = stack == 0 ? e->base : e->draft;
    size_t nmax = 0;
    for (int l = 0; l < S.nl; l++) {
        const Linear& L = kind == 0 ? S.L[l].qkv : kind == 1 ? S.L[l].o : kind == 2 ? S.L[l].gu : S.L[l].down;
        nmax = std::max(nmax, (size_t)L.N);
    }
    float* out = nullptr;
    FL_CHECK_CUDA(cudaMalloc(&out, sizeof(float) * nmax * M));
    struct FreeOnExit {
        float* p;
        ~FreeOnExit() { cudaFree(p); }
    } out_guard{out};
    cudaGraph_t g = nullptr;
    FL_CHECK_CUDA(cudaStreamBeginCapture(e->s, cudaStreamCaptureModeThreadLocal));
    int rc = FL_OK;
    const Linear* l0 = nullptr;
    for (int l = 0; l < S.nl && rc == FL_OK; l++) {
        const Linear& L = kind == 0 ? S.L[l].qkv : kind == 1 ? S.L[l].o : kind == 2 ? S.L[l].gu : S.L[l].down;
        l0 = &L;
        GemvParams gp = gemv_base(L, kind == 3 ? e->hq : e->xq, nullptr);
        gp.M = M;
        gp.out = out;
        gp.ldo = L.N;
        // up to 8 rows: one GEMV launch; more: the many-row path of the layers
        if (M <= kMaxRows ? launch_gemv_auto(gp, EPI_STORE, e->s, true) != cudaSuccess
                          : launch_chunks(gp, EPI_STORE, M, nullptr, e->s, false) != FL_OK)
            rc = set_error(FL_E_CUDA, "bench_linear launch");
    }
    cudaError_t ce = cudaStreamEndCapture(e->s, &g);
    if (rc != FL_OK) {
        if (g) cudaGraphDestroy(g);
        return rc;
    }
    FL_CHECK_CUDA(ce);
    cudaGraphExec_t ex = nullptr;
    ce = cudaGraphInstantiate(&ex, g, 0);
    cudaGraphDestroy(g);
    FL_CHECK_CUDA(ce);
    FL_CHECK_CUDA(cudaGraphLaunch(ex, e->s));  // warm-up
    FL_CHECK_CUDA(cudaEventRecord(e->ev[2], e->s));
    for (int r = 0; r < reps; r++) FL_CHECK_CUDA(cudaGraphLaunch(ex, e->s));
    FL_CHECK_CUDA(cudaEventRecord(e->ev[3], e->s));
    FL_CHECK_CUDA(cudaEventSynchronize(e->ev[3]));
    cudaGraphExecDestroy(ex);
    float ms = 0.0f;
    cudaEventElapsedTime(&ms, e->ev[2], e->ev[3]);
    if (us_per_launch) *us_per_launch = ms * 1000.0 / ((double)reps * S.nl);
    if (bytes_per_launch)
        *bytes_per_launch = (double)l0->N * l0->K * ((l0->w4 && M <= kGemmMinRows ? 0.5 : 1.0) + 1.0 / 16.0) +
                            (double)M * l0->K + 4.0 * M * l0->N;
    return FL_OK;
}

FL_API int fl_engine_bench_attention(fl_engine_t* e, int stack, int M, int ctx, int reps, double* us_per_launch) {
    FL_CHECK(check_ready(e, stack == 1));
    if (M < 1 || M > kMaxRows || ctx < M || ctx > e->c.max_seq_len || reps < 1)
        return set_error(FL_E_INVAL, "bench_attention: bad arguments");
    Stack& S = stack == 0 ? e->base : e->draft;
    cudaGraph_t g = nullptr;
    FL_CHECK_CUDA(cudaStreamBeginCapture(e->s, cudaStreamCaptureModeThreadLocal));
    int rc = FL_OK;
    for (int l = 0; l < S.nl && rc == FL_OK; l++) {
        AttnParams at = {};
        at.q = e->q;
        at.kv = S.kv[l];
        at.block_table = S.block_table;
        at.slot_base = e->iota + (ctx - M);
        at.M = M;
        at.heads = e->H;
        at.kv_heads = e->Hkv;
        at.head_dim = e->hd;
        at.max_ctx = e->c.max_seq_len;
        at.out_q = e->aq;
        at.part = e->attn_part;
        at.counters = e->attn_cnt;
        if (launch_attention(at, e->s, true) != cudaSuccess) rc = set_error(FL_E_CUDA, "bench_attention launch");
    }
    cudaError_t ce = cudaStreamEndCapture(e->s, &g);
    if (rc != FL_OK) {
        if (g) cudaGraphDestroy(g);
        return rc;
    }
    FL_CHECK_CUDA(ce);
    cudaGraphExec_t ex = nullptr;
    ce = cudaGraphInstantiate(&ex, g, 0);
    cudaGraphDestroy(g);
    FL_CHECK_CUDA(ce);
    FL_CHECK_CUDA(cudaGraphLaunch(ex, e->s));  // warm-up
    FL_CHECK_CUDA(cudaEventRecord(e->ev[2], e->s));
    for (int r = 0; r < reps; r++) FL_CHECK_CUDA(cudaGraphLaunch(ex, e->s));
    FL_CHECK_CUDA(cudaEventRecord(e->ev[3], e->s));
    FL_CHECK_CUDA(cudaEventSynchronize(e->ev[3]));
    cudaGraphExecDestroy(ex);
    float ms = 0.0f;
    cudaEventElapsedTime(&ms, e->ev[2], e->ev[3]);
    if (us_per_launch) *us_per_launch = ms * 1000.0 / ((double)reps * S.nl);
    return FL_OK;
}

// ---------------------------------------------------------------------------
// Callback-level API: the engine as the reference's target_forward /
// base_forward model, with an explicit base-cache position.
// ---------------------------------------------------------------------------

FL_API int fl_engine_position(const fl_engine_t* e) { return e ? e->cb_pos : -1; }

FL_API int fl_engine_set_position(fl_engine_t* e, int pos) {
    if (!e || pos < 0 || pos > e->R) return set_error(FL_E_INVAL, "set_position: out of range");
    e->cb_pos = pos;
    return FL_OK;
}

FL_API int fl_engine_last_feature(const fl_engine_t* e, float* out) {
    if (!e || !out) return set_error(FL_E_INVAL, "last_feature: NULL");
    FL_CHECK_CUDA(cudaSetDevice(e->device));
    FL_CHECK_CUDA(cudaMemcpy(out, e->last_feat, sizeof(float) * e->d, cudaMemcpyDeviceToHost));
    return FL_OK;
}

// Appends len tokens at the callback position through the base model.
static int base_append(fl_engine* e, const int* tokens, int len, float* logits_out) {
    FL_CHECK(check_ready(e, false));
    if (logits_out && e->tp_size > 1)
        return set_error(FL_E_UNSUPPORTED, "target_forward: a tensor-parallel rank holds a slice of the logits");
    if (len <= 0 || e->cb_pos + len > e->R) return set_error(FL_E_INVAL, "base forward: context full");
    FL_CHECK_CUDA(cudaMemcpyAsync(e->tok, tokens, sizeof(int) * len, cudaMemcpyHostToDevice, e->s));
    FL_CHECK_CUDA(launch_embed_rows(e->embed, e->Vg, e->tok, nullptr, 0, e->x, e->d, len, nullptr, nullptr, e->s, false));
    FL_CHECK(run_stack(e, e->base, e->x, len, nullptr, e->iota + e->cb_pos, e->iota + e->cb_pos, nullptr, nullptr,
                       false));
    FL_CHECK_CUDA(cudaMemcpyAsync(e->last_feat, e->x + (size_t)(len - 1) * e->d, sizeof(float) * e->d,
                                  cudaMemcpyDeviceToDevice, e->s));
    if (logits_out) {
        for (int r0 = 0; r0 < len; r0 += kMaxRows) {
            const int m = std::min(kMaxRows, len - r0);
            FL_CHECK(run_lm(e, e->x + (size_t)r0 * e->d, m, nullptr, nullptr, false));
            FL_CHECK_CUDA(cudaMemcpyAsync(logits_out + (size_t)r0 * e->V, e->logits, sizeof(float) * (size_t)m * e->V,
                                          cudaMemcpyDeviceToHost, e->s));
        }
    }
    FL_CHECK_CUDA(cudaStreamSynchronize(e->s));
    e->cb_pos += len;
    return FL_OK;
}

FL_API void fl_cuda_target_forward(void* model, const float* input, float* output, int len) {
    fl_engine* e = (fl_engine*)model;
    if (!e || !input || !output || len <= 0) {
        set_error(FL_E_INVAL, "target_forward: bad arguments");
        return;
    }
    std::vector<int> t(len);
    for (int i = 0; i < len; i++) t[i] = (int)input[i];
    base_append(e, t.data(), len, output);
}

FL_API void fl_cuda_base_forward(void* model, const int* tokens, int len, float* hidden, int hidden_size) {
    fl_engine* e = (fl_engine*)model;
    if (!e || !tokens || len <= 0) {
        set_error(FL_E_INVAL, "base_forward: bad arguments");
        return;
    }
    if (base_append(e, tokens, len, nullptr) != FL_OK) return;
    if (hidden && hidden_size == e->d) fl_engine_last_feature(e, hidden);
}

// Single-row draft chain: x = hidden + E[tok] at position pos, then K greedy
// draft tokens (each next input = draft output + E[previous draft]).
FL_API int fl_engine_draft_chain(fl_engine_t* e, const float* hidden, int tok, int pos, int K, int* out_tokens,
                                 float* out_probs) {
    FL_CHECK(check_ready(e, true));
    if (!hidden || !out_tokens || K <= 0 || pos < 0 || pos + K > e->R) return set_error(FL_E_INVAL, "draft_chain: bad arguments");
    if (e->tp_size > 1) return set_error(FL_E_UNSUPPORTED, "draft_chain: not available on a tensor-parallel engine");
    std::vector<float> lg(e->V);
    FL_CHECK_CUDA(cudaMemcpyAsync(e->x2, hidden, sizeof(float) * e->d, cudaMemcpyHostToDevice, e->s));
    FL_CHECK_CUDA(cudaMemcpyAsync(e->tok, &tok, sizeof(int), cudaMemcpyHostToDevice, e->s));
    FL_CHECK_CUDA(launch_embed_rows(e->embed, e->Vg, e->tok, e->x2, 0, e->x_d, e->d, 1, nullptr, nullptr, e->s, false));
    for (int j = 0; j < K; j++) {
        FL_CHECK(run_stack(e, e->draft, e->x_d, 1, nullptr, e->iota + pos + j, e->iota + pos + j, nullptr, nullptr, false));
        FL_CHECK(run_lm(e, e->x_d, 1, nullptr, nullptr, false));
        FL_CHECK_CUDA(launch_argmax_rows(amax_keys(e), amax_nparts(e), 1, e->tok, nullptr, e->s));
        FL_CHECK_CUDA(cudaMemcpyAsync(lg.data(), e->logits, sizeof(float) * e->V, cudaMemcpyDeviceToHost, e->s));
        FL_CHECK_CUDA(cudaMemcpyAsync(&out_tokens[j], e->tok, sizeof(int), cudaMemcpyDeviceToHost, e->s));
        FL_CHECK_CUDA(launch_embed_rows(e->embed, e->Vg, e->tok, e->x_d, 0, e->x_d, e->d, 1, nullptr, nullptr, e->s, false));
        FL_CHECK_CUDA(cudaStreamSynchronize(e->s));
        if (out_probs) {
            float mx = lg[0];
            for (float v : lg) mx = v > mx ? v : mx;
            double sum = 0.0;
            for (float v : lg) sum += exp((double)(v - mx));
            out_probs[j] = (float)(exp((double)(lg[out_tokens[j]] - mx)) / sum);
        }
    }
    return FL_OK;
}

// ---------------------------------------------------------------------------
// Medusa greedy decoding (include/medusa.h rule)
// ---------------------------------------------------------------------------
namespace {

// out[M, N] = L(quantise(x)) (optionally RMSNorm first), M <= kMaxRows.
int gemv_rows(fl_engine* e, const Linear& L, const float* x, int M, bool norm, float* out, int ldo) {
    GemvParams g = gemv_base(L, e->xq, nullptr);
    if ((L.K % 128) == 0) {
        g.x = x;
        g.norm = norm ? 1 : 0;
        g.eps = e->c.norm_eps;
    } else {
        ActQuantParams a = {};
        a.x = x;
        a.q = e->xq;
        a.K = L.K;
        a.M = M;
        a.norm = norm ? 1 : 0;
        a.eps = e->c.norm_eps;
        FL_CHECK_CUDA(launch_act_quant(a, e->s, false));
    }
    g.out = out;
    g.ldo = ldo;
    g.M = M;
    g.row0 = 0;
    FL_CHECK_CUDA(launch_gemv_auto(g, EPI_STORE, e->s, false));
    return FL_OK;
}

struct MedCand {
    float score;
    int depth, gen, parent_gen, token;
};

// Candidate tree from the heads' top-k lists: level L + 1 = head L's top-k
// under every level-L node (breadth-first generation order), score = product
// of the probabilities along the path; the best max_nodes - 1 candidates by
// (score desc, depth asc, generation asc) are kept, root first. A child never
// outscores its parent and loses ties to it, so the kept set is
// ancestor-closed and every parent precedes its children.
int build_tree(int root_tok, int H, const int* topk, const int* tok, const float* prob, int kmax, int max_nodes,
               std::vector<int>& ntok, std::vector<int>& npar, std::vector<int>& ndep,
               std::vector<float>* nscore = nullptr) {
    std::vector<MedCand> c;
    int pb = 0, pe = 0;
    for (int h = 0; h < H; h++) {
        const int lb = (int)c.size();
        if (h == 0) {
            for (int k = 0; k < topk[0]; k++)
                c.push_back({prob[k], 1, (int)c.size(), -1, tok[k]});
        } else {
            for (int pi = pb; pi < pe; pi++)
                for (int k = 0; k < topk[h]; k++)
                    c.push_back({c[pi].score * prob[h * kmax + k], h + 1, (int)c.size(), pi, tok[h * kmax + k]});
        }
        pb = lb;
        pe = (int)c.size();
    }
    std::vector<MedCand> s = c;
    std::sort(s.begin(), s.end(), [](const MedCand& x, const MedCand& y) {
        if (x.score != y.score) return x.score > y.score;
        if (x.depth != y.depth) return x.depth < y.depth;
        return x.gen < y.gen;
    });
    const int keep = std::min<int>(max_nodes - 1, (int)s.size());
    std::vector<int> where(c.size(), -1);
    for (int i = 0; i < keep; i++) where[s[i].gen] = i + 1;
    ntok.assign(1, root_tok);
    npar.assign(1, -1);
    ndep.assign(1, 0);
    if (nscore) nscore->assign(1, 1.0f);
    for (int i = 0; i < keep; i++) {
        ntok.push_back(s[i].token);
        npar.push_back(s[i].parent_gen < 0 ? 0 : where[s[i].parent_gen]);
        ndep.push_back(s[i].depth);
        if (nscore) nscore->push_back(s[i].score);
    }
    return keep + 1;
}

// Draft + Medusa candidate tree: the draft chain d_1 .. d_K as one branch
// under the root (always kept), then the Medusa tree's nodes in its own order
// (parents first), each merged with an existing node of the same token under
// the same parent or added while fewer than max_nodes nodes exist; a node
// whose parent was dropped is dropped. Returns the node count.
int merge_chain_tree(int root_tok, const int* chain, int K, const std::vector<int>& mtok, const std::vector<int>& mpar,
                     const std::vector<int>& mdep, int max_nodes, std::vector<int>& ntok, std::vector<int>& npar,
                     std::vector<int>& ndep) {
    ntok.assign(1, root_tok);
    npar.assign(1, -1);
    ndep.assign(1, 0);
    for (int j = 0; j < K && (int)ntok.size() < max_nodes; j++) {
        ntok.push_back(chain[j]);
        npar.push_back(j);
        ndep.push_back(j + 1);
    }
    std::vector<int> map(mtok.size(), -1);
    map[0] = 0;
    for (size_t i = 1; i < mtok.size(); i++) {
        const int pp = map[mpar[i]];
        if (pp < 0) continue;
        int found = -1;
        for (size_t k = 1; k < ntok.size(); k++)
            if (npar[k] == pp && ntok[k] == mtok[i]) {
                found = (int)k;
                break;
            }
        if (found < 0 && (int)ntok.size() < max_nodes) {
            found = (int)ntok.size();
            ntok.push_back(mtok[i]);
            npar.push_back(pp);
            ndep.push_back(mdep[i]);
        }
        map[i] = found;
    }
    return (int)ntok.size();
}

}  // namespace

FL_API int fl_engine_medusa_generate(fl_engine_t* e, const int* prompt, int P, int n_new, const int* topk, int H,
                                     int max_nodes, int* out, int* acc_hist, int* steps_out) {
    FL_CHECK(check_ready(e, false));
    if (!prompt || !out || !topk || P <= 0 || n_new <= 0 || H <= 0 || H > (int)e->medusa.size() || H > kMaxRows ||
        max_nodes < 2 || max_nodes > 256 || P + n_new + max_nodes + 2 > e->R)
        return set_error(FL_E_INVAL, "medusa_generate: bad arguments, missing heads or context too long");
    int kmax = 1;
    long long cand = 0, width = 1;
    for (int h = 0; h < H; h++) {
        if (topk[h] < 1 || topk[h] > 32) return set_error(FL_E_INVAL, "medusa_generate: top-k must be 1..32");
        kmax = std::max(kmax, topk[h]);
        width *= topk[h];
        cand += width;
        if (cand > kMaxTreeCand)
            return set_error(FL_E_INVAL, "medusa_generate: more than 1024 tree candidates (sum of top-k products)");
    }
    const int M = 1 + std::min<int>(max_nodes - 1, (int)cand);  // tree nodes of every step
    const int d = e->d, V = e->V;
    cudaStream_t s = e->s;
    // device work buffers: carved from the engine's work arena (allocated
    // once, grown only when a call needs more), so a call makes no cudaMalloc
    // or cudaFree of its own
    float *mf = nullptr, *my = nullptr, *mz = nullptr, *mprob = nullptr;
    int *mk = nullptr, *mtt = nullptr, *mtok = nullptr, *mpos = nullptr, *mtarget = nullptr, *mpath = nullptr;
    int *mpar = nullptr, *mdep = nullptr, *mrec = nullptr, *mroot = nullptr;
    KvLayer* dkv = nullptr;
    auto fail = [&](int rc) { return rc; };
#define FL_MED_CUDA(expr)                                                    \
    do {                                                                     \
        cudaError_t fl_e_ = (expr);                                          \
        if (fl_e_ != cudaSuccess) return fail(cuda_error(fl_e_, #expr));     \
    } while (0)
#define FL_MED(expr)                      \
    do {                                  \
        int fl_r_ = (expr);               \
        if (fl_r_ != FL_OK) return fail(fl_r_); \
    } while (0)
    {
        const size_t sizes[] = {sizeof(float) * d, sizeof(float) * (size_t)H * d, sizeof(float) * (size_t)H * d,
                                sizeof(float) * (size_t)H * kmax, sizeof(int) * H, sizeof(int) * (size_t)H * kmax,
                                sizeof(int) * max_nodes, sizeof(int) * max_nodes, sizeof(int) * max_nodes,
                                sizeof(int) * max_nodes, sizeof(int) * max_nodes, sizeof(int) * max_nodes,
                                sizeof(int) * (max_nodes + 2), sizeof(int), sizeof(KvLayer) * e->base.nl};
        void** ptrs[] = {(void**)&mf, (void**)&my, (void**)&mz, (void**)&mprob, (void**)&mk, (void**)&mtt,
                         (void**)&mtok, (void**)&mpos, (void**)&mtarget, (void**)&mpath, (void**)&mpar,
                         (void**)&mdep, (void**)&mrec, (void**)&mroot, (void**)&dkv};
        FL_MED(carve_work(e, ptrs, sizes, (int)(sizeof(sizes) / sizeof(sizes[0]))));
    }
    FL_MED_CUDA(cudaMemcpyAsync(dkv, e->base.kv.data(), sizeof(KvLayer) * e->base.nl, cudaMemcpyHostToDevice, s));
    FL_MED_CUDA(cudaMemcpyAsync(mk, topk, sizeof(int) * H, cudaMemcpyHostToDevice, s));
    FL_MED(ensure_mask(e, max_nodes));

    // prefill: base KV 0 .. P-1, first token from the last prompt row
    FL_MED(prefill_base(e, prompt, P));
    FL_MED_CUDA(cudaMemcpyAsync(mf, e->x + (size_t)(P - 1) * d, sizeof(float) * d, cudaMemcpyDeviceToDevice, s));
    int cur_tok = 0;
    FL_MED_CUDA(cudaMemcpyAsync(mroot, e->seq + P, sizeof(int), cudaMemcpyDeviceToDevice, s));
    FL_MED_CUDA(cudaMemcpyAsync(&cur_tok, e->seq + P, sizeof(int), cudaMemcpyDeviceToHost, s));
    FL_MED_CUDA(cudaStreamSynchronize(s));
    int produced = 0, steps = 0, n = P;
    out[produced++] = cur_tok;
    std::vector<int> rec(M + 2);
    FL_MED_CUDA(cudaEventRecord(e->ev[0], s));
    while (produced < n_new) {
        // heads: h = RMSNorm(F), y_i = W_i h, z_i = h + SiLU(y_i), logits_i = LM(z_i)
        FL_MED_CUDA(launch_medusa_z(mf, my, e->x2, mz, d, 0, e->c.norm_eps, s));  // h -> x2
        for (int h = 0; h < H; h++) FL_MED(gemv_rows(e, e->medusa[h], e->x2, 1, false, my + (size_t)h * d, d));
        FL_MED_CUDA(launch_medusa_z(mf, my, nullptr, mz, d, H, e->c.norm_eps, s));
        FL_MED(gemv_rows(e, e->lm, mz, H, false, e->logits, V));
        FL_MED_CUDA(launch_topk_rows(e->logits, H, V, V, mk, kmax, mtt, mprob, s));
        // candidate tree on the device: node i at slot n + i, rotary position n + depth
        MedusaTreeParams tp = {mtt, mprob, mk, H, kmax, max_nodes, n, mroot, mtok, mpar, mdep, mpos, e->mask};
        FL_MED_CUDA(launch_medusa_tree(tp, s));
        // tree-masked verify
        FL_MED_CUDA(launch_embed_rows(e->embed, V, mtok, nullptr, 0, e->x, d, M, nullptr, nullptr, s, false));
        FL_MED(run_stack(e, e->base, e->x, M, nullptr, e->iota + n, mpos, e->mask, nullptr, false));
        for (int r0 = 0; r0 < M; r0 += kMaxRows) {
            const int m = std::min(kMaxRows, M - r0);
            FL_MED(run_lm(e, e->x + (size_t)r0 * d, m, nullptr, nullptr, false));
            FL_MED_CUDA(launch_argmax_rows(e->amax, e->nparts, m, mtarget + r0, nullptr, s));
        }
        // longest path of the base model's greedy choices, its KV moved to
        // consecutive slots, the next root and feature; one read-back per step
        MedusaWalkParams wp = {mtok, mpar, mtarget, M, mpath, mrec, mroot, e->x, mf, d};
        FL_MED_CUDA(launch_medusa_walk(wp, s));
        FL_MED_CUDA(launch_kv_compact_dev(dkv, e->base.nl, e->base.block_table, e->Hkv, e->hd, e->iota + n, mpath,
                                          mrec, s));
        FL_MED_CUDA(cudaMemcpyAsync(rec.data(), mrec, sizeof(int) * (M + 2), cudaMemcpyDeviceToHost, s));
        FL_MED_CUDA(cudaStreamSynchronize(s));
        const int a = rec[0];
        if (a < 0 || a >= M) return fail(set_error(FL_E_CUDA, "medusa_generate: bad accepted path"));
        if (acc_hist) acc_hist[steps] = a;
        steps++;
        for (int j = 1; j <= a + 1 && produced < n_new; j++) out[produced++] = rec[1 + j];
        n += a + 1;
    }
    FL_MED_CUDA(cudaEventRecord(e->ev[1], s));
    FL_MED_CUDA(cudaEventSynchronize(e->ev[1]));
    float ms = 0.0f;
    cudaEventElapsedTime(&ms, e->ev[0], e->ev[1]);
    e->t_total_us = ms * 1000.0;
    if (steps_out) *steps_out = steps;
#undef FL_MED_CUDA
#undef FL_MED
    if (take_device_error() != 0) return set_error(FL_E_TIMEOUT, "medusa_generate: a bounded device wait gave up");
    return FL_OK;
}

// Draft + Medusa (medusa.h:210-229 speculative_medusa_generate; the reference
// declares it without code): each step the EAGLE-style draft drafts a chain of
// K tokens from its state at the newest position while the Medusa heads
// propose per-depth candidates from the base feature; the merged tree
// (merge_chain_tree) is verified in one tree-masked base pass, the longest
// path of the base model's greedy choices is accepted (plus the base token
// after it), the base KV of that path is compacted, and the draft catches up
// over the accepted positions from the base features of the path's tree rows
// (draft input at position p = F_{p-1} + E[t_p]). The output is the base
// model's greedy stream whatever the tree.
FL_API int fl_engine_spec_medusa_generate(fl_engine_t* e, const int* prompt, int P, int n_new, int K, const int* topk,
                                          int H, int max_nodes, int* out, int* acc_hist, int* steps_out) {
    FL_CHECK(check_ready(e, true));
    if (!prompt || !out || !topk || P <= 0 || n_new <= 0 || K < 1 || K > kMaxDraft || H <= 0 ||
        H > (int)e->medusa.size() || H > kMaxRows || max_nodes < K + 2 || max_nodes > 256 ||
        P + n_new + max_nodes + K + 2 > e->R)
        return set_error(FL_E_INVAL, "spec_medusa_generate: bad arguments, missing heads or context too long");
    if (e->tp_size > 1) return set_error(FL_E_UNSUPPORTED, "spec_medusa_generate: not on a tensor-parallel engine");
    int kmax = 1;
    for (int h = 0; h < H; h++) {
        if (topk[h] < 1 || topk[h] > 32) return set_error(FL_E_INVAL, "spec_medusa_generate: top-k must be 1..32");
        kmax = std::max(kmax, topk[h]);
    }
    const int d = e->d, V = e->V;
    cudaStream_t s = e->s;
    float *mf = nullptr, *my = nullptr, *mz = nullptr, *mprob = nullptr;
    int *mk = nullptr, *mtt = nullptr, *mtok = nullptr, *mpos = nullptr, *mtarget = nullptr, *mpath = nullptr,
        *mchain = nullptr, *mcat = nullptr;
    KvLayer* dkv = nullptr;
    auto cleanup = [&]() {
        void* bufs[] = {mf, my, mz, mprob, mk, mtt, mtok, mpos, mtarget, mpath, mchain, mcat, dkv};
        for (void* p : bufs) cudaFree(p);
    };
    auto fail = [&](int rc) {
        cleanup();
        return rc;
    };
#define FL_SM_CUDA(expr)                                                     \
    do {                                                                     \
        cudaError_t fl_e_ = (expr);                                          \
        if (fl_e_ != cudaSuccess) return fail(cuda_error(fl_e_, #expr));     \
    } while (0)
#define FL_SM(expr)                       \
    do {                                  \
        int fl_r_ = (expr);               \
        if (fl_r_ != FL_OK) return fail(fl_r_); \
    } while (0)
    FL_SM_CUDA(cudaMalloc(&mf, sizeof(float) * d));
    FL_SM_CUDA(cudaMalloc(&my, sizeof(float) * (size_t)H * d));
    FL_SM_CUDA(cudaMalloc(&mz, sizeof(float) * (size_t)H * d));
    FL_SM_CUDA(cudaMalloc(&mprob, sizeof(float) * (size_t)H * kmax));
    FL_SM_CUDA(cudaMalloc(&mk, sizeof(int) * H));
    FL_SM_CUDA(cudaMalloc(&mtt, sizeof(int) * (size_t)H * kmax));
    FL_SM_CUDA(cudaMalloc(&mtok, sizeof(int) * max_nodes));
    FL_SM_CUDA(cudaMalloc(&mpos, sizeof(int) * max_nodes));
    FL_SM_CUDA(cudaMalloc(&mtarget, sizeof(int) * max_nodes));
    FL_SM_CUDA(cudaMalloc(&mpath, sizeof(int) * max_nodes));
    FL_SM_CUDA(cudaMalloc(&mchain, sizeof(int) * kMaxRows));
    FL_SM_CUDA(cudaMalloc(&mcat, sizeof(int) * max_nodes));
    FL_SM_CUDA(cudaMalloc(&dkv, sizeof(KvLayer) * e->base.nl));
    FL_SM_CUDA(cudaMemcpyAsync(dkv, e->base.kv.data(), sizeof(KvLayer) * e->base.nl, cudaMemcpyHostToDevice, s));
    FL_SM_CUDA(cudaMemcpyAsync(mk, topk, sizeof(int) * H, cudaMemcpyHostToDevice, s));
    FL_SM(ensure_mask(e, max_nodes));

    // prefill: base KV 0 .. P-1 and the first token; draft catch-up over 0 .. P
    FL_SM(prefill_base(e, prompt, P));
    FL_SM_CUDA(cudaMemcpyAsync(mf, e->x + (size_t)(P - 1) * d, sizeof(float) * d, cudaMemcpyDeviceToDevice, s));
    FL_SM_CUDA(launch_embed_rows(e->embed, e->Vg, e->seq, e->x, 1, e->x2, d, P + 1, nullptr, nullptr, s, false));
    FL_SM(run_stack(e, e->draft, e->x2, P + 1, nullptr, e->iota, e->iota, nullptr, nullptr, false));
    FL_SM_CUDA(cudaMemcpyAsync(e->x_d, e->x2 + (size_t)P * d, sizeof(float) * d, cudaMemcpyDeviceToDevice, s));
    int cur_tok = 0;
    FL_SM_CUDA(cudaMemcpyAsync(&cur_tok, e->seq + P, sizeof(int), cudaMemcpyDeviceToHost, s));
    FL_SM_CUDA(cudaStreamSynchronize(s));
    int produced = 0, steps = 0, n = P;
    out[produced++] = cur_tok;
    std::vector<int> htok((size_t)H * kmax), target(max_nodes), chain(K), mtk, mpr, mdp, ntok, npar, ndep, path, cat;
    std::vector<float> hprob((size_t)H * kmax);
    std::vector<int> hpos(max_nodes);
    std::vector<uint8_t> mask((size_t)max_nodes * max_nodes);
    FL_SM_CUDA(cudaEventRecord(e->ev[0], s));
    while (produced < n_new) {
        // draft chain from the draft state at position n (x_d row 0)
        for (int j = 0; j < K; j++) {
            if (j > 0) {
                FL_SM_CUDA(launch_embed_rows(e->embed, e->Vg, mchain + j - 1, e->x_d, 0, e->x_d, d, 1, nullptr, nullptr, s,
                                             false));
                FL_SM(run_stack(e, e->draft, e->x_d, 1, nullptr, e->iota + n + j, e->iota + n + j, nullptr, nullptr,
                                false));
            }
            FL_SM(run_lm(e, e->x_d, 1, nullptr, nullptr, false));
            FL_SM_CUDA(launch_argmax_rows(amax_keys(e), amax_nparts(e), 1, mchain + j, nullptr, s));
        }
        // Medusa heads from the base feature of position n - 1
        FL_SM_CUDA(launch_medusa_z(mf, my, e->x2, mz, d, 0, e->c.norm_eps, s));
        for (int h = 0; h < H; h++) FL_SM(gemv_rows(e, e->medusa[h], e->x2, 1, false, my + (size_t)h * d, d));
        FL_SM_CUDA(launch_medusa_z(mf, my, nullptr, mz, d, H, e->c.norm_eps, s));
        FL_SM(gemv_rows(e, e->lm, mz, H, false, e->logits, V));
        FL_SM_CUDA(launch_topk_rows(e->logits, H, V, V, mk, kmax, mtt, mprob, s));
        FL_SM_CUDA(cudaMemcpyAsync(chain.data(), mchain, sizeof(int) * K, cudaMemcpyDeviceToHost, s));
        FL_SM_CUDA(cudaMemcpyAsync(htok.data(), mtt, sizeof(int) * htok.size(), cudaMemcpyDeviceToHost, s));
        FL_SM_CUDA(cudaMemcpyAsync(hprob.data(), mprob, sizeof(float) * hprob.size(), cudaMemcpyDeviceToHost, s));
        FL_SM_CUDA(cudaStreamSynchronize(s));
        build_tree(cur_tok, H, topk, htok.data(), hprob.data(), kmax, max_nodes, mtk, mpr, mdp);
        const int M = merge_chain_tree(cur_tok, chain.data(), K, mtk, mpr, mdp, max_nodes, ntok, npar, ndep);
        for (int i = 0; i < M; i++) {
            hpos[i] = n + ndep[i];
            for (int j = 0; j < M; j++) mask[(size_t)i * M + j] = 0;
            for (int j = i; j >= 0; j = npar[j]) mask[(size_t)i * M + j] = 1;
        }
        FL_SM_CUDA(cudaMemcpyAsync(mtok, ntok.data(), sizeof(int) * M, cudaMemcpyHostToDevice, s));
        FL_SM_CUDA(cudaMemcpyAsync(mpos, hpos.data(), sizeof(int) * M, cudaMemcpyHostToDevice, s));
        FL_SM_CUDA(cudaMemcpyAsync(e->mask, mask.data(), (size_t)M * M, cudaMemcpyHostToDevice, s));
        FL_SM_CUDA(launch_embed_rows(e->embed, e->Vg, mtok, nullptr, 0, e->x, d, M, nullptr, nullptr, s, false));
        FL_SM(run_stack(e, e->base, e->x, M, nullptr, e->iota + n, mpos, e->mask, nullptr, false));
        for (int r0 = 0; r0 < M; r0 += kMaxRows) {
            const int m = std::min(kMaxRows, M - r0);
            FL_SM(run_lm(e, e->x + (size_t)r0 * d, m, nullptr, nullptr, false));
            FL_SM_CUDA(launch_argmax_rows(amax_keys(e), amax_nparts(e), m, mtarget + r0, nullptr, s));
        }
        FL_SM_CUDA(cudaMemcpyAsync(target.data(), mtarget, sizeof(int) * M, cudaMemcpyDeviceToHost, s));
        FL_SM_CUDA(cudaStreamSynchronize(s));
        path.assign(1, 0);
        int cur = 0;
        for (;;) {
            int nxt = -1;
            for (int c2 = 1; c2 < M; c2++)
                if (npar[c2] == cur && ntok[c2] == target[cur]) {
                    nxt = c2;
                    break;
                }
            if (nxt < 0) break;
            path.push_back(nxt);
            cur = nxt;
        }
        const int a = (int)path.size() - 1;
        if (acc_hist) acc_hist[steps] = a;
        steps++;
        for (int j = 1; j <= a + 1 && produced < n_new; j++) out[produced++] = j <= a ? ntok[path[j]] : target[cur];
        // draft catch-up over positions n+1 .. n+a+1: F of the path's tree rows + E[token]
        cat.resize(a + 1);
        for (int j = 0; j <= a; j++) cat[j] = j < a ? ntok[path[j + 1]] : target[cur];
        FL_SM_CUDA(cudaMemcpyAsync(mcat, cat.data(), sizeof(int) * (a + 1), cudaMemcpyHostToDevice, s));
        for (int j = 0; j <= a; j++)
            FL_SM_CUDA(cudaMemcpyAsync(e->x2 + (size_t)j * d, e->x + (size_t)path[j] * d, sizeof(float) * d,
                                       cudaMemcpyDeviceToDevice, s));
        if (a > 0) {
            FL_SM_CUDA(cudaMemcpyAsync(mpath, path.data(), sizeof(int) * (a + 1), cudaMemcpyHostToDevice, s));
            FL_SM_CUDA(launch_kv_compact(dkv, e->base.nl, e->base.block_table, e->Hkv, e->hd, e->iota + n, mpath, a, s));
        }
        FL_SM_CUDA(cudaMemcpyAsync(mf, e->x + (size_t)cur * d, sizeof(float) * d, cudaMemcpyDeviceToDevice, s));
        FL_SM_CUDA(launch_embed_rows(e->embed, e->Vg, mcat, e->x2, 0, e->x2, d, a + 1, nullptr, nullptr, s, false));
        FL_SM(run_stack(e, e->draft, e->x2, a + 1, nullptr, e->iota + n + 1, e->iota + n + 1, nullptr, nullptr, false));
        FL_SM_CUDA(cudaMemcpyAsync(e->x_d, e->x2 + (size_t)a * d, sizeof(float) * d, cudaMemcpyDeviceToDevice, s));
        cur_tok = target[cur];
        n += a + 1;
    }
    FL_SM_CUDA(cudaEventRecord(e->ev[1], s));
    FL_SM_CUDA(cudaEventSynchronize(e->ev[1]));
    float ms = 0.0f;
    cudaEventElapsedTime(&ms, e->ev[0], e->ev[1]);
    e->t_total_us = ms * 1000.0;
    if (steps_out) *steps_out = steps;
#undef FL_SM_CUDA
#undef FL_SM
    cleanup();
    if (take_device_error() != 0) return set_error(FL_E_TIMEOUT, "spec_medusa_generate: a bounded device wait gave up");
    return FL_OK;
}

// Medusa candidate tree from a base feature F (host [d]): the heads' per-head
// top-k (h = RMSNorm(F), z_i = h + SiLU(W_i h), LM(z_i)) and the tree rule of
// include/medusa.h. root >= 0 is the root token; root < 0 takes the base LM
// head's argmax of F. Writes up to max_nodes nodes; returns the node count.
FL_API int fl_engine_medusa_tree(fl_engine_t* e, const float* F, int root, const int* topk, int H, int max_nodes,
                                 int* tok, int* parent, int* depth, float* score) {
    FL_CHECK(check_ready(e, false));
    if (!F || !topk || !tok || !parent || !depth || H <= 0 || H > (int)e->medusa.size() || H > kMaxRows ||
        max_nodes < 1 || max_nodes > 256)
        return set_error(FL_E_INVAL, "medusa_tree: bad arguments or missing heads");
    if (e->tp_size > 1) return set_error(FL_E_UNSUPPORTED, "medusa_tree: not on a tensor-parallel engine");
    int kmax = 1;
    for (int h = 0; h < H; h++) {
        if (topk[h] < 1 || topk[h] > 32) return set_error(FL_E_INVAL, "medusa_tree: top-k must be 1..32");
        kmax = std::max(kmax, topk[h]);
    }
    const int d = e->d, V = e->V;
    cudaStream_t s = e->s;
    float *mf = nullptr, *my = nullptr, *mz = nullptr, *mprob = nullptr;
    int *mk = nullptr, *mtt = nullptr, *mroot = nullptr;
    auto cleanup = [&]() {
        void* bufs[] = {mf, my, mz, mprob, mk, mtt, mroot};
        for (void* p : bufs) cudaFree(p);
    };
    int rc = FL_OK;
    std::vector<int> htok((size_t)H * kmax), ntok, npar, ndep;
    std::vector<float> hprob((size_t)H * kmax), nscore;
    do {
        if (cudaMalloc(&mf, sizeof(float) * d) || cudaMalloc(&my, sizeof(float) * (size_t)H * d) ||
            cudaMalloc(&mz, sizeof(float) * (size_t)H * d) || cudaMalloc(&mprob, sizeof(float) * (size_t)H * kmax) ||
            cudaMalloc(&mk, sizeof(int) * H) || cudaMalloc(&mtt, sizeof(int) * (size_t)H * kmax) ||
            cudaMalloc(&mroot, sizeof(int))) {
            rc = set_error(FL_E_NOMEM, "medusa_tree: device buffers");
            break;
        }
        if (cudaMemcpyAsync(mf, F, sizeof(float) * d, cudaMemcpyHostToDevice, s) != cudaSuccess ||
            cudaMemcpyAsync(mk, topk, sizeof(int) * H, cudaMemcpyHostToDevice, s) != cudaSuccess) {
            rc = set_error(FL_E_CUDA, "medusa_tree: upload");
            break;
        }
        if (root < 0) {
            if ((rc = run_lm(e, mf, 1, nullptr, nullptr, false)) != FL_OK) break;
            if (launch_argmax_rows(amax_keys(e), amax_nparts(e), 1, mroot, nullptr, s) != cudaSuccess ||
                cudaMemcpyAsync(&root, mroot, sizeof(int), cudaMemcpyDeviceToHost, s) != cudaSuccess) {
                rc = set_error(FL_E_CUDA, "medusa_tree: root");
                break;
            }
        }
        if (launch_medusa_z(mf, my, e->x2, mz, d, 0, e->c.norm_eps, s) != cudaSuccess) {
            rc = set_error(FL_E_CUDA, "medusa_tree: heads");
            break;
        }
        for (int h = 0; h < H && rc == FL_OK; h++) rc = gemv_rows(e, e->medusa[h], e->x2, 1, false, my + (size_t)h * d, d);
        if (rc != FL_OK) break;
        if (launch_medusa_z(mf, my, nullptr, mz, d, H, e->c.norm_eps, s) != cudaSuccess) {
            rc = set_error(FL_E_CUDA, "medusa_tree: heads");
            break;
        }
        if ((rc = gemv_rows(e, e->lm, mz, H, false, e->logits, V)) != FL_OK) break;
        if (launch_topk_rows(e->logits, H, V, V, mk, kmax, mtt, mprob, s) != cudaSuccess ||
            cudaMemcpyAsync(htok.data(), mtt, sizeof(int) * htok.size(), cudaMemcpyDeviceToHost, s) != cudaSuccess ||
            cudaMemcpyAsync(hprob.data(), mprob, sizeof(float) * hprob.size(), cudaMemcpyDeviceToHost, s) != cudaSuccess ||
            cudaStreamSynchronize(s) != cudaSuccess) {
            rc = set_error(FL_E_CUDA, "medusa_tree: top-k");
            break;
        }
    } while (0);
    cleanup();
    FL_CHECK(rc);
    const int M = build_tree(root, H, topk, htok.data(), hprob.data(), kmax, max_nodes, ntok, npar, ndep, &nscore);
    for (int i = 0; i < M; i++) {
        tok[i] = ntok[i];
        parent[i] = npar[i];
        depth[i] = ndep[i];
        if (score) score[i] = nscore[i];
    }
    return M;
}

// Tree verification at the callback position (fl_engine_position): node i is
// fed at cache slot pos + i with rotary position pos + depth[i], attending to
// its ancestors; the longest path of the base model's greedy choices is
// accepted, its KV moved to slots pos + 1 .. pos + a, and the position
// advances by a + 1 (root and accepted nodes). out_tokens receives the a
// accepted tokens and the base model's token after them (a + 1 entries);
// *accepted = a. The feature of the last accepted node becomes the last
// feature (fl_engine_last_feature).
FL_API int fl_engine_tree_verify(fl_engine_t* e, const int* tok, const int* parent, const int* depth, int M,
                                 int* out_tokens, int* accepted) {
    FL_CHECK(check_ready(e, false));
    if (!tok || !parent || !depth || !out_tokens || M < 1 || M > 256 || e->cb_pos < 1 || e->cb_pos + M > e->R)
        return set_error(FL_E_INVAL, "tree_verify: bad arguments or context full");
    if (parent[0] != -1 || depth[0] != 0) return set_error(FL_E_INVAL, "tree_verify: node 0 must be the root");
    for (int i = 1; i < M; i++)
        if (parent[i] < 0 || parent[i] >= i || depth[i] != depth[parent[i]] + 1)
            return set_error(FL_E_INVAL, "tree_verify: parents must precede children, depth = parent depth + 1");
    if (e->tp_size > 1) return set_error(FL_E_UNSUPPORTED, "tree_verify: not on a tensor-parallel engine");
    const int d = e->d, n = e->cb_pos;
    cudaStream_t s = e->s;
    FL_CHECK(ensure_mask(e, M));
    std::vector<int> pos(M), target(M), path;
    std::vector<uint8_t> mask((size_t)M * M, 0);
    for (int i = 0; i < M; i++) {
        pos[i] = n + depth[i];
        for (int j = i; j >= 0; j = parent[j]) mask[(size_t)i * M + j] = 1;
    }
    int *mtok = nullptr, *mpos = nullptr, *mtarget = nullptr, *mpath = nullptr;
    KvLayer* dkv = nullptr;
    auto cleanup = [&]() {
        void* bufs[] = {mtok, mpos, mtarget, mpath, dkv};
        for (void* p : bufs) cudaFree(p);
    };
    int rc = FL_OK;
    do {
        if (cudaMalloc(&mtok, sizeof(int) * M) || cudaMalloc(&mpos, sizeof(int) * M) ||
            cudaMalloc(&mtarget, sizeof(int) * M) || cudaMalloc(&mpath, sizeof(int) * M) ||
            cudaMalloc(&dkv, sizeof(KvLayer) * e->base.nl)) {
            rc = set_error(FL_E_NOMEM, "tree_verify: device buffers");
            break;
        }
        if (cudaMemcpyAsync(mtok, tok, sizeof(int) * M, cudaMemcpyHostToDevice, s) != cudaSuccess ||
            cudaMemcpyAsync(mpos, pos.data(), sizeof(int) * M, cudaMemcpyHostToDevice, s) != cudaSuccess ||
            cudaMemcpyAsync(e->mask, mask.data(), (size_t)M * M, cudaMemcpyHostToDevice, s) != cudaSuccess ||
            cudaMemcpyAsync(dkv, e->base.kv.data(), sizeof(KvLayer) * e->base.nl, cudaMemcpyHostToDevice, s) !=
                cudaSuccess ||
            launch_embed_rows(e->embed, e->Vg, mtok, nullptr, 0, e->x, d, M, nullptr, nullptr, s, false) != cudaSuccess) {
            rc = set_error(FL_E_CUDA, "tree_verify: inputs");
            break;
        }
        if ((rc = run_stack(e, e->base, e->x, M, nullptr, e->iota + n, mpos, e->mask, nullptr, false)) != FL_OK) break;
        for (int r0 = 0; r0 < M && rc == FL_OK; r0 += kMaxRows) {
            const int m = std::min(kMaxRows, M - r0);
            if ((rc = run_lm(e, e->x + (size_t)r0 * d, m, nullptr, nullptr, false)) != FL_OK) break;
            if (launch_argmax_rows(amax_keys(e), amax_nparts(e), m, mtarget + r0, nullptr, s) != cudaSuccess)
                rc = set_error(FL_E_CUDA, "tree_verify: argmax");
        }
        if (rc != FL_OK) break;
        if (cudaMemcpyAsync(target.data(), mtarget, sizeof(int) * M, cudaMemcpyDeviceToHost, s) != cudaSuccess ||
            cudaStreamSynchronize(s) != cudaSuccess) {
            rc = set_error(FL_E_CUDA, "tree_verify: targets");
            break;
        }
        path.assign(1, 0);
        int cur = 0;
        for (;;) {
            int nxt = -1;
            for (int c2 = 1; c2 < M; c2++)
                if (parent[c2] == cur && tok[c2] == target[cur]) {
                    nxt = c2;
                    break;
                }
            if (nxt < 0) break;
            path.push_back(nxt);
            cur = nxt;
        }
        const int a = (int)path.size() - 1;
        for (int j = 1; j <= a; j++) out_tokens[j - 1] = tok[path[j]];
        out_tokens[a] = target[cur];
        if (accepted) *accepted = a;
        if (a > 0 && (cudaMemcpyAsync(mpath, path.data(), sizeof(int) * (a + 1), cudaMemcpyHostToDevice, s) != cudaSuccess ||
                      launch_kv_compact(dkv, e->base.nl, e->base.block_table, e->Hkv, e->hd, e->iota + n, mpath, a, s) !=
                          cudaSuccess)) {
            rc = set_error(FL_E_CUDA, "tree_verify: compaction");
            break;
        }
        if (cudaMemcpyAsync(e->last_feat, e->x + (size_t)cur * d, sizeof(float) * d, cudaMemcpyDeviceToDevice, s) !=
                cudaSuccess ||
            cudaStreamSynchronize(s) != cudaSuccess) {
            rc = set_error(FL_E_CUDA, "tree_verify: feature");
            break;
        }
        e->cb_pos = n + a + 1;
    } while (0);
    cleanup();
    FL_CHECK(rc);
    if (take_device_error() != 0) return set_error(FL_E_TIMEOUT, "tree_verify: a bounded device wait gave up");
    return FL_OK;
}
