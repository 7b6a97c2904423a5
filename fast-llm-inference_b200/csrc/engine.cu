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

using namespace fl;

namespace {

struct Linear {
    int8_t* w = nullptr;
    __half* s = nullptr;
    int N = 0, K = 0;
    int P = 0;  // tiled-layout panel width (fl_layout.cuh), 0 = row-major
    unsigned need = 0, have = 0;  // bit masks of the source tensors loaded
};

struct LayerW {
    Linear qkv, o, gu, down;
};

struct Stack {
    int nl = 0;
    std::vector<LayerW> L;
    std::vector<KvLayer> kv;
    int* block_table = nullptr;
    int pages = 0;
};

// The KV cache a pass reads and writes: one sequence's region, or an in-GPU
// batch (rows of sequence b are rows [b seq_rows, (b + 1) seq_rows) of the
// pass, its slots [b seq_slots, (b + 1) seq_slots), and its slot base and
// positions in state records seq_state ints apart).
struct KvView {
    const KvLayer* kv = nullptr;  // [layers] (host array)
    const int* block_table = nullptr;
    int seqs = 1, seq_rows = 0, seq_state = 0, seq_slots = 0;
    int max_ctx = 0;              // slots per sequence (attention grid)
    float* attn_part = nullptr;   // split-K scratch for seqs sequences
    int* attn_cnt = nullptr;
};

}  // namespace

struct fl_engine {
    fl_model_config_t c;
    int device = 0;
    cudaStream_t s = nullptr;
    int d = 0, qd = 0, kd = 0, F = 0, V = 0, hd = 0, H = 0, Hkv = 0;
    float* embed = nullptr;
    bool embed_loaded = false;
    Linear lm;
    Stack base, draft;
    std::vector<Linear> medusa;
    // work buffers for up to R rows
    int R = 0;
    float* x = nullptr;      // [R, d]
    float* x2 = nullptr;     // [R, d]
    uint8_t* xq = nullptr;   // [R, max(d, qd)]
    float* q = nullptr;      // [R, qd]
    uint8_t* aq = nullptr;   // [R, qd]
    uint8_t* hq = nullptr;   // [R, F]
    float* logits = nullptr; // [kMaxRows, V]
    unsigned long long* amax = nullptr;  // [kMaxRows, nparts]
    int nparts = 0;
    float* x_v = nullptr;    // [kMaxRows, d]
    float* x_d = nullptr;    // [kMaxRows, d]
    int* iota = nullptr;     // [R + 16]: iota[i] = i (positions and slot scalars)
    int* tok = nullptr;      // [R]
    uint8_t* mask = nullptr; // [R * R] bounded by kMaxRows^2 for tests
    int mask_cap = 0;
    // speculative state
    SpecState* st = nullptr;
    SpecState* st_snap = nullptr;
    float* xd0_snap = nullptr;
    int* seq = nullptr;
    int* out = nullptr;
    int* acc = nullptr;
    int spec_K = 0, spec_P = 0, spec_ready = 0;
    cudaGraphExec_t step_exec = nullptr;
    int graph_K = -1;
    cudaEvent_t ev[4] = {nullptr, nullptr, nullptr, nullptr};
    double t_draft_us = 0, t_verify_us = 0, t_total_us = 0;
    int cb_pos = 0;               // callback API: base cache length
    float* last_feat = nullptr;   // [d] base feature of the last appended token
    unsigned* step_bar = nullptr;  // step kernel: grid barrier + error word
    Phase* d_phases = nullptr;     // step kernel phase list (device)
    int n_phases = 0;
    std::vector<int> phase_desc;   // per phase: kind, epilogue, N, K (host)
    unsigned long long* d_trace = nullptr;  // FL_STEP_TRACE=1: 3 words per phase
    bool step_kernel = false;      // last step graph uses the one-kernel step
    bool step_layout = false;      // weights in 128-byte panels for the tcgen05 step kernel
    float* attn_part = nullptr;   // decode attention split-K scratch
    int* attn_cnt = nullptr;      // per-head arrival counters (zero at rest)
    int graph_kernels = 0;        // kernel nodes in the step graph
    long long last_launches = 0;  // kernels launched by the last decode
    const void* bound_draft = nullptr;
    // stochastic speculative decoding (temperature > 0); set by
    // fl_engine_set_sampling, used by the next fl_engine_spec_prefill
    bool samp = false;
    float samp_T = 0.0f, samp_top_p = 1.0f;
    uint32_t samp_seed = 0, samp_seq = 0;
    uint32_t* samp_q = nullptr;            // [kMaxDraft, V] draft nucleus weights
    uint32_t* samp_p = nullptr;            // [kMaxRows, V] target nucleus weights
    unsigned long long* samp_m = nullptr;  // [kMaxDraft + kMaxRows] kept masses (draft, then target)
    unsigned long long* samp_r = nullptr;  // [V] rejection residual weights
    uint32_t* samp_key = nullptr;          // [2] Philox seed, sequence id
    // tensor parallelism (fl_engine_create_tp): this rank's slice of the model;
    // H, Hkv, qd, kd, F and V above are the rank's local counts
    int tp_rank = 0, tp_size = 1;
    void* tp_comm = nullptr;
    TpLayout tp = {};
    int Vg = 0;                                // embedding rows (the full vocabulary)
    int tp_rows = 0;                           // rows of the key buffers (kMaxRows; more for a batch)
    unsigned long long* tp_keys = nullptr;     // [tp_rows] this rank's best LM-head key per row
    unsigned long long* tp_all = nullptr;      // [tp_size][tp_rows] gathered
    unsigned long long* tp_best = nullptr;     // [tp_rows] the argmax keys the control kernels read
    // fused all-reduce over NVLink peer memory for decode-sized passes: the o
    // and down GEMVs store partial rows into every rank's receive slots, a
    // small kernel sums them (tp_reduce_kernel); larger passes use NCCL
    bool tp_fused = false;
    void* tp_region = nullptr;                 // this rank's receive slots + counters (peers write here)
    size_t tp_recv_bytes = 0;
    std::vector<void*> tp_peer;                // every rank's region as mapped here (IPC)
    float** tp_recv_ptrs = nullptr;            // device [size]
    unsigned long long** tp_cnt_ptrs = nullptr;  // device [size]
    unsigned long long* tp_seq = nullptr;      // this rank's fused all-reduce count
    int* tp_arrived = nullptr;
    // post-prefill draft state of step 0: its mass, weights and traced logits
    // (8 + 4V + 4V bytes)
    unsigned char* samp_snap = nullptr;
    float* samp_trace = nullptr;  // [2 * kMaxRows, V] logits behind each draw (trace on)
    bool trace_on = false;
    // In-GPU batch of independent sequences (fl_engine_batch_*): its own KV
    // regions (bslots slots per sequence), per-sequence state and rows, and
    // one step graph that advances every sequence
    struct Batch {
        int cap = 0, slots = 0;          // sequences held, KV slots per sequence
        int n = 0, K = 0, P = 0;         // sequences, drafts per step, prompt length of the prefill
        bool ready = false, samp = false, traced = false;
        std::vector<KvLayer> kv_base, kv_draft;
        int* block = nullptr;            // identity table over cap * slots / kPageSize pages
        float* attn_part = nullptr;
        int* attn_cnt = nullptr;
        SpecState* st = nullptr;         // [cap]
        SpecState* st_snap = nullptr;
        int* seq = nullptr;              // [cap][slots] committed tokens
        int* out = nullptr;              // [cap][slots] emitted tokens
        int* acc = nullptr;              // [cap][slots] accepted drafts per step
        BatchCtl* ctl = nullptr;
        float* x_v = nullptr;            // [cap * kMaxRows, d] verify rows
        float* x_dc = nullptr;           // [cap * kMaxRows, d] draft catch-up rows
        float* x_d1 = nullptr;           // [cap, d] single-row draft inputs
        float* x_d1_snap = nullptr;
        float* logits = nullptr;         // [cap * kMaxRows, V]
        unsigned long long* amax = nullptr;  // [cap * kMaxRows, nparts]
        uint32_t* key = nullptr;         // [cap][2] Philox seed, sequence id
        uint32_t* q = nullptr;           // [cap][kMaxDraft][V] (sampling)
        uint32_t* p = nullptr;           // [cap][kMaxRows][V]
        unsigned long long* m = nullptr; // [cap][kMaxDraft + kMaxRows]
        unsigned long long* r = nullptr; // [cap][V]
        uint32_t* q_snap = nullptr;      // [cap][V] draft weights of step 0
        unsigned long long* m_snap = nullptr;  // [cap]
        float* trace = nullptr;          // [cap][2 * kMaxRows][V] (trace on)
        float* trace_snap = nullptr;     // [cap][V]
        cudaGraphExec_t exec = nullptr;
        int graph_kernels = 0;
    } bt;
};

namespace {

void batch_free(fl_engine* e);

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
    l.w = nullptr;
    l.s = nullptr;
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
    g.P = l.P;
    g.sblk = l.s;
    g.N = l.N;
    g.K = l.K;
    g.done = done;
    return g;
}

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
              const uint8_t* mask, const int* done, bool pdl, const KvView* view = nullptr) {
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
           float* logits = nullptr, unsigned long long* amax = nullptr) {
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

}  // namespace

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
    const char* v = getenv("FL_TP_FUSED");
    e->tp_fused = !(v && v[0] == '0');
    return FL_OK;
}

static fl_engine_t* engine_create(const fl_model_config_t* cfg, int device, int tp_rank, int tp_size,
                                  const unsigned char* tp_id) {
    if (!cfg) { set_error(FL_E_INVAL, "config is NULL"); return nullptr; }
    const fl_model_config_t& c = *cfg;
    if (c.hidden_size <= 0 || c.num_heads <= 0 || c.num_kv_heads <= 0 || c.head_dim <= 0 ||
        c.num_heads % c.num_kv_heads != 0 || c.hidden_size % 32 != 0 || c.intermediate_size % 32 != 0 ||
        (c.num_heads * c.head_dim) % 32 != 0 || c.head_dim % 2 != 0 || c.head_dim > 128 ||
        c.vocab_size <= 0 || c.num_layers <= 0 || c.max_seq_len < 16 || c.draft_layers < 0 || c.medusa_heads < 0) {
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
                    e->iota, e->tok, e->mask, e->st, e->st_snap, e->xd0_snap, e->seq, e->out, e->acc,
                    e->last_feat, e->attn_part, e->attn_cnt, e->step_bar, e->d_phases, e->d_trace,
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

// ---------------------------------------------------------------------------
// In-GPU batch of independent sequences. Every step runs each draft pass
// over one row per sequence and the verify and draft catch-up passes over
// K + 1 rows per sequence, so the weights stream once per pass for the whole
// batch (the tcgen05 GEMM takes passes of more than 16 rows). Each sequence
// keeps its own KV region, state record, token arrays and Philox key
// (seed, sequence id); its decisions are those of the one-sequence step.
// ---------------------------------------------------------------------------
namespace {

void batch_free(fl_engine* e) {
    auto& B = e->bt;
    if (B.exec) cudaGraphExecDestroy(B.exec);
    for (auto* kv : {&B.kv_base, &B.kv_draft})
        for (auto& l : *kv) {
            cudaFree(l.k);
            cudaFree(l.v);
        }
    void* bufs[] = {B.block, B.attn_part, B.attn_cnt, B.st, B.st_snap, B.seq, B.out, B.acc, B.ctl, B.x_v,
                    B.x_dc, B.x_d1, B.x_d1_snap, B.logits, B.amax, B.key, B.q, B.p, B.m, B.r, B.q_snap,
                    B.m_snap, B.trace, B.trace_snap};
    for (void* p : bufs) cudaFree(p);
    B = fl_engine::Batch();
}

// Device bytes one sequence of a batch holds with `slots` KV slots.
size_t batch_bytes_per_seq(const fl_engine* e, int slots) {
    const size_t kv = (size_t)(e->base.nl + e->draft.nl) * 2 * e->Hkv * e->hd * sizeof(__half) * slots;
    const size_t rows = (size_t)kMaxRows * (3 * e->d + e->V + e->nparts * 2) * 4 + (size_t)e->d * 8;
    const size_t toks = (size_t)3 * slots * sizeof(int);
    const size_t attn = sizeof(float) * attention_scratch_floats(e->H, e->hd, slots);
    return kv + rows + toks + attn + 2 * sizeof(SpecState);
}

int batch_alloc(fl_engine* e, int cap, int slots) {
    batch_free(e);
    auto& B = e->bt;
    slots = (slots + kPageSize - 1) / kPageSize * kPageSize;
    const size_t pages = (size_t)cap * (slots / kPageSize);
    const size_t kvb = pages * e->Hkv * kPageSize * e->hd * sizeof(__half);
    for (auto pr : {std::make_pair(&B.kv_base, e->base.nl), std::make_pair(&B.kv_draft, e->draft.nl)}) {
        pr.first->assign(pr.second, KvLayer{nullptr, nullptr});
        for (auto& l : *pr.first) {
            FL_CHECK_CUDA(cudaMalloc(&l.k, kvb));
            FL_CHECK_CUDA(cudaMalloc(&l.v, kvb));
            FL_CHECK_CUDA(cudaMemsetAsync(l.k, 0, kvb, e->s));
            FL_CHECK_CUDA(cudaMemsetAsync(l.v, 0, kvb, e->s));
        }
    }
    const size_t d = e->d, V = e->V, rows = (size_t)cap * kMaxRows, cnt = attention_scratch_counters(e->H) * cap;
    FL_CHECK_CUDA(cudaMalloc(&B.block, sizeof(int) * pages));
    FL_CHECK_CUDA(cudaMalloc(&B.attn_part, sizeof(float) * attention_scratch_floats(e->H, e->hd, slots) * cap));
    FL_CHECK_CUDA(cudaMalloc(&B.attn_cnt, sizeof(int) * cnt));
    FL_CHECK_CUDA(cudaMemsetAsync(B.attn_cnt, 0, sizeof(int) * cnt, e->s));
    FL_CHECK_CUDA(cudaMalloc(&B.st, sizeof(SpecState) * cap));
    FL_CHECK_CUDA(cudaMalloc(&B.st_snap, sizeof(SpecState) * cap));
    FL_CHECK_CUDA(cudaMalloc(&B.seq, sizeof(int) * cap * (size_t)slots));
    FL_CHECK_CUDA(cudaMalloc(&B.out, sizeof(int) * cap * (size_t)slots));
    FL_CHECK_CUDA(cudaMalloc(&B.acc, sizeof(int) * cap * (size_t)slots));
    FL_CHECK_CUDA(cudaMalloc(&B.ctl, sizeof(BatchCtl)));
    FL_CHECK_CUDA(cudaMalloc(&B.x_v, sizeof(float) * rows * d));
    FL_CHECK_CUDA(cudaMalloc(&B.x_dc, sizeof(float) * rows * d));
    FL_CHECK_CUDA(cudaMalloc(&B.x_d1, sizeof(float) * cap * d));
    FL_CHECK_CUDA(cudaMalloc(&B.x_d1_snap, sizeof(float) * cap * d));
    FL_CHECK_CUDA(cudaMalloc(&B.logits, sizeof(float) * rows * V));
    FL_CHECK_CUDA(cudaMalloc(&B.amax, sizeof(unsigned long long) * rows * e->nparts));
    FL_CHECK_CUDA(cudaMalloc(&B.key, sizeof(uint32_t) * 2 * cap));
    std::vector<int> id(pages);
    for (size_t i = 0; i < pages; i++) id[i] = (int)i;
    FL_CHECK_CUDA(cudaMemcpy(B.block, id.data(), sizeof(int) * pages, cudaMemcpyHostToDevice));
    B.cap = cap;
    B.slots = slots;
    return FL_OK;
}

int batch_alloc_sampling(fl_engine* e) {
    auto& B = e->bt;
    const size_t V = e->V, cap = B.cap;
    if (!B.q) {
        FL_CHECK_CUDA(cudaMalloc(&B.q, sizeof(uint32_t) * cap * kMaxDraft * V));
        FL_CHECK_CUDA(cudaMalloc(&B.p, sizeof(uint32_t) * cap * kMaxRows * V));
        FL_CHECK_CUDA(cudaMalloc(&B.m, sizeof(unsigned long long) * cap * (kMaxDraft + kMaxRows)));
        FL_CHECK_CUDA(cudaMalloc(&B.r, sizeof(unsigned long long) * cap * V));
        FL_CHECK_CUDA(cudaMalloc(&B.q_snap, sizeof(uint32_t) * cap * V));
        FL_CHECK_CUDA(cudaMalloc(&B.m_snap, sizeof(unsigned long long) * cap));
    }
    if (B.traced && !B.trace_snap) {
        FL_CHECK_CUDA(cudaMalloc(&B.trace, sizeof(float) * cap * 2 * kMaxRows * V));
        FL_CHECK_CUDA(cudaMalloc(&B.trace_snap, sizeof(float) * cap * V));
    }
    return FL_OK;
}

StepBuffers batch_buffers(fl_engine* e) {
    auto& B = e->bt;
    StepBuffers b = {};
    b.st = B.st;
    b.seq = B.seq;
    b.out = B.out;
    b.acc_hist = B.acc;
    b.embed = e->embed;
    b.x_d = B.x_dc;
    b.x_v = B.x_v;
    b.amax_part = e->tp_size > 1 ? e->tp_best : B.amax;  // tensor parallel: the reduced keys
    b.nparts = amax_nparts(e);
    b.d = e->d;
    b.logits = B.logits;
    b.V = e->V;
    b.temp = e->samp_T;
    b.top_p = e->samp_top_p;
    b.key = B.key;
    if (B.samp) {
        b.qd = B.q;
        b.qm = B.m;
        b.pt = B.p;
        b.pm = B.m + kMaxDraft;
        b.resid = B.r;
        b.trace = B.traced ? B.trace : nullptr;
    }
    b.batch = B.n;
    b.rows_per = B.K + 1;
    b.seq_cap = B.slots;
    b.x_d1 = B.x_d1;
    b.logits_d = B.logits;
    b.amax_d = b.amax_part;
    b.ctl = B.ctl;
    return b;
}

// The batch's KV regions as seen by a pass of `rows` rows per sequence.
KvView batch_view(fl_engine* e, bool base, int rows) {
    auto& B = e->bt;
    KvView v;
    v.kv = base ? B.kv_base.data() : B.kv_draft.data();
    v.block_table = B.block;
    v.seqs = B.n;
    v.seq_rows = rows;
    v.seq_state = (int)(sizeof(SpecState) / sizeof(int));
    v.seq_slots = B.slots;
    v.max_ctx = B.slots;
    v.attn_part = B.attn_part;
    v.attn_cnt = B.attn_cnt;
    return v;
}

// One batched speculative step (the rule of record_step, every sequence at once).
int record_batch_step(fl_engine* e, bool pdl) {
    auto& B = e->bt;
    const int K = B.K, n = B.n;
    const StepBuffers b = batch_buffers(e);
    const int* done = &B.ctl->done;
    KvView vd = batch_view(e, false, 1);
    const KvView vb = batch_view(e, true, K + 1);
    auto pick = [&](int j) {
        return B.samp ? launch_sample_pick(b, j, e->s, pdl) : launch_draft_pick(b, j, e->s, pdl);
    };
    for (int j = 1; j < K; j++) {
        FL_CHECK(run_stack(e, e->draft, B.x_d1, n, nullptr, &B.st->draft_base, B.st->draft_pos, nullptr, done, pdl, &vd));
        FL_CHECK(run_lm(e, B.x_d1, n, nullptr, done, pdl, B.logits, B.amax));
        FL_CHECK_CUDA(pick(j));
    }
    FL_CHECK_CUDA(launch_verify_prep(b, K, e->s, pdl));
    FL_CHECK(run_stack(e, e->base, B.x_v, n * (K + 1), nullptr, &B.st->verify_base, B.st->verify_pos, nullptr, done,
                       pdl, &vb));
    FL_CHECK(run_lm(e, B.x_v, n * (K + 1), nullptr, done, pdl, B.logits, B.amax));
    if (B.samp) {
        FL_CHECK_CUDA(launch_target_dist(b, K, e->s, pdl));
        FL_CHECK_CUDA(launch_accept_sampled(b, K, e->s, pdl));
    } else {
        FL_CHECK_CUDA(launch_accept(b, K, e->s, pdl));
    }
    FL_CHECK_CUDA(launch_catchup_prep(b, K, e->s, pdl));
    vd.seq_rows = K + 1;
    FL_CHECK(run_stack(e, e->draft, B.x_dc, n * (K + 1), nullptr, &B.st->draft_base, B.st->draft_pos, nullptr, done,
                       pdl, &vd));
    FL_CHECK_CUDA(launch_gather_last(b, e->s, pdl));
    FL_CHECK(run_lm(e, B.x_d1, n, nullptr, done, pdl, B.logits, B.amax));
    FL_CHECK_CUDA(pick(0));
    return FL_OK;
}

int build_batch_graph(fl_engine* e) {
    auto& B = e->bt;
    if (B.exec) {
        FL_CHECK_CUDA(cudaStreamSynchronize(e->s));
        cudaGraphExecDestroy(B.exec);
        B.exec = nullptr;
    }
    cudaGraph_t g = nullptr;
    FL_CHECK_CUDA(cudaStreamBeginCapture(e->s, cudaStreamCaptureModeThreadLocal));
    const int rc = record_batch_step(e, true);
    const cudaError_t ce = cudaStreamEndCapture(e->s, &g);
    if (rc != FL_OK) {
        if (g) cudaGraphDestroy(g);
        return rc;
    }
    FL_CHECK_CUDA(ce);
    size_t nn = 0;
    cudaGraphGetNodes(g, nullptr, &nn);
    std::vector<cudaGraphNode_t> nodes(nn);
    cudaGraphGetNodes(g, nodes.data(), &nn);
    int nk = 0;
    for (auto nd : nodes) {
        cudaGraphNodeType t;
        if (cudaGraphNodeGetType(nd, &t) == cudaSuccess && t == cudaGraphNodeTypeKernel) nk++;
    }
    B.graph_kernels = nk;
    const cudaError_t ie = cudaGraphInstantiate(&B.exec, g, 0);
    cudaGraphDestroy(g);
    FL_CHECK_CUDA(ie);
    return FL_OK;
}

// Tensor parallelism: argmax key buffers for at least `rows` LM-head rows.
// Growing them drops the step graphs that hold the old buffers.
int tp_ensure_rows(fl_engine* e, int rows) {
    if (e->tp_size == 1 || e->tp_rows >= rows) return FL_OK;
    FL_CHECK_CUDA(cudaStreamSynchronize(e->s));
    cudaFree(e->tp_keys);
    cudaFree(e->tp_all);
    cudaFree(e->tp_best);
    e->tp_keys = e->tp_all = e->tp_best = nullptr;
    e->tp_rows = 0;
    e->spec_ready = 0;
    if (e->step_exec) {
        cudaGraphExecDestroy(e->step_exec);
        e->step_exec = nullptr;
    }
    e->graph_K = -1;
    if (e->bt.exec) {
        cudaGraphExecDestroy(e->bt.exec);
        e->bt.exec = nullptr;
    }
    e->bt.ready = false;
    if (cudaMalloc(&e->tp_keys, sizeof(unsigned long long) * rows) != cudaSuccess ||
        cudaMalloc(&e->tp_all, sizeof(unsigned long long) * rows * e->tp_size) != cudaSuccess ||
        cudaMalloc(&e->tp_best, sizeof(unsigned long long) * rows) != cudaSuccess)
        return set_error(FL_E_NOMEM, "tensor parallel: argmax key buffers");
    e->tp_rows = rows;
    return FL_OK;
}

// Strided copy of `rows` rows of `width` bytes (row pitches in bytes).
cudaError_t copy_rows(void* dst, size_t dpitch, const void* src, size_t spitch, size_t width, size_t rows,
                      cudaMemcpyKind kind, cudaStream_t s) {
    return cudaMemcpy2DAsync(dst, dpitch, src, spitch, width, rows, kind, s);
}

}  // namespace

FL_API int fl_engine_batch_reserve(fl_engine_t* e, int nseq, int max_ctx) {
    FL_CHECK(check_ready(e, true));
    if (nseq <= 0 || max_ctx < 16 || nseq > 65535) return set_error(FL_E_INVAL, "batch_reserve: bad arguments");
    FL_CHECK_CUDA(cudaStreamSynchronize(e->s));
    // vocabulary-parallel argmax keys for every LM-head row of a batched
    // pass (every rank reserves the same batch, so the gathers match)
    FL_CHECK(tp_ensure_rows(e, nseq * kMaxRows));
    const int rc = batch_alloc(e, nseq, max_ctx);
    if (rc != FL_OK) {
        batch_free(e);
        (void)cudaGetLastError();
        return set_error(FL_E_NOMEM, "batch_reserve: device allocation failed");
    }
    FL_CHECK_CUDA(cudaStreamSynchronize(e->s));
    return FL_OK;
}

FL_API int fl_engine_batch_capacity(const fl_engine_t* e, int* nseq, int* slots) {
    if (!e) return set_error(FL_E_INVAL, "engine is NULL");
    if (nseq) *nseq = e->bt.cap;
    if (slots) *slots = e->bt.slots;
    return FL_OK;
}

FL_API int fl_engine_batch_prefill(fl_engine_t* e, const int* prompts, int P, int nseq, const unsigned* seq_ids, int K) {
    FL_CHECK(check_ready(e, true));
    auto& B = e->bt;
    if (!prompts || P <= 0 || nseq <= 0 || K < 1 || K > kMaxDraft)
        return set_error(FL_E_INVAL, "batch_prefill: bad arguments (1 <= K <= 7)");
    if (nseq > B.cap) return set_error(FL_E_INVAL, "batch_prefill: more sequences than reserved");
    if (P + K + 3 > B.slots || P + 2 > e->R || nseq * (K + 1) > e->R)
        return set_error(FL_E_INVAL, "batch_prefill: prompt or batch too long for the reservation");
    if (e->d % 128 != 0) return set_error(FL_E_UNSUPPORTED, "batch: the hidden size must be a multiple of 128");
    B.ready = false;
    B.n = nseq;
    B.K = K;
    B.P = P;
    B.samp = e->samp;
    B.traced = e->samp && e->trace_on;
    if (B.samp) {
        FL_CHECK(batch_alloc_sampling(e));
        std::vector<uint32_t> key(2 * (size_t)nseq);
        for (int s = 0; s < nseq; s++) {
            key[2 * s] = e->samp_seed;
            key[2 * s + 1] = seq_ids ? seq_ids[s] : (unsigned)s;
        }
        FL_CHECK_CUDA(cudaMemcpyAsync(B.key, key.data(), sizeof(uint32_t) * key.size(), cudaMemcpyHostToDevice, e->s));
    }
    const StepBuffers b = batch_buffers(e);
    const size_t d = e->d, V = e->V;
    const size_t region = (size_t)(B.slots / kPageSize) * e->Hkv * kPageSize * e->hd;  // halves per sequence
    std::vector<KvLayer> rb(B.kv_base.size()), rd(B.kv_draft.size());
    for (int s = 0; s < nseq; s++) {
        // this sequence's KV region, addressed as a cache of its own
        for (size_t l = 0; l < rb.size(); l++) rb[l] = {B.kv_base[l].k + s * region, B.kv_base[l].v + s * region};
        for (size_t l = 0; l < rd.size(); l++) rd[l] = {B.kv_draft[l].k + s * region, B.kv_draft[l].v + s * region};
        KvView vb, vd;
        vb.kv = rb.data();
        vd.kv = rd.data();
        vb.block_table = vd.block_table = B.block;
        int* sq = B.seq + (size_t)s * B.slots;
        FL_CHECK_CUDA(cudaMemcpyAsync(sq, prompts + (size_t)s * P, sizeof(int) * P, cudaMemcpyHostToDevice, e->s));
        FL_CHECK_CUDA(launch_embed_rows(e->embed, e->Vg, sq, nullptr, 0, e->x, e->d, P, nullptr, nullptr, e->s, false));
        FL_CHECK(run_stack(e, e->base, e->x, P, nullptr, e->iota, e->iota, nullptr, nullptr, false, &vb));
        // first token from the last prompt row (LM-head row s)
        FL_CHECK(run_lm(e, e->x + (size_t)(P - 1) * d, 1, nullptr, nullptr, false, B.logits + s * V,
                        B.amax + (size_t)s * e->nparts));
        if (B.samp)
            FL_CHECK_CUDA(launch_sample_first(b, P, e->s, s));
        else if (e->tp_size > 1)
            FL_CHECK_CUDA(launch_argmax_rows(e->tp_best, 1, 1, sq + P, nullptr, e->s));
        else
            FL_CHECK_CUDA(launch_argmax_rows(B.amax + (size_t)s * e->nparts, e->nparts, 1, sq + P, nullptr, e->s));
        // draft catch-up over positions 0..P: x_i = F_{i-1} + E[t_i]
        FL_CHECK_CUDA(launch_embed_rows(e->embed, e->Vg, sq, e->x, 1, e->x2, e->d, P + 1, nullptr, nullptr, e->s, false));
        FL_CHECK(run_stack(e, e->draft, e->x2, P + 1, nullptr, e->iota, e->iota, nullptr, nullptr, false, &vd));
        FL_CHECK_CUDA(cudaMemcpyAsync(B.x_d1 + s * d, e->x2 + (size_t)P * d, sizeof(float) * d,
                                      cudaMemcpyDeviceToDevice, e->s));
        FL_CHECK_CUDA(cudaMemcpyAsync(B.out + (size_t)s * B.slots, sq + P, sizeof(int), cudaMemcpyDeviceToDevice, e->s));
    }
    std::vector<SpecState> h(nseq);
    for (auto& x : h) {
        x = SpecState{};
        x.n = P;
        x.produced = 1;
        x.n_new = 1;
        x.K = K;
        x.max_acc = K;
        x.one = 1;
        x.rows = 1;
    }
    FL_CHECK_CUDA(cudaMemcpyAsync(B.st, h.data(), sizeof(SpecState) * nseq, cudaMemcpyHostToDevice, e->s));
    const BatchCtl c0 = {nseq, 0};
    FL_CHECK_CUDA(cudaMemcpyAsync(B.ctl, &c0, sizeof(c0), cudaMemcpyHostToDevice, e->s));
    FL_CHECK(run_lm(e, B.x_d1, nseq, nullptr, nullptr, false, B.logits, B.amax));
    if (B.samp)
        FL_CHECK_CUDA(launch_sample_pick(b, 0, e->s, false));
    else
        FL_CHECK_CUDA(launch_draft_pick(b, 0, e->s, false));
    // post-prefill state of every sequence (decodes start from it)
    FL_CHECK_CUDA(cudaMemcpyAsync(B.st_snap, B.st, sizeof(SpecState) * nseq, cudaMemcpyDeviceToDevice, e->s));
    FL_CHECK_CUDA(cudaMemcpyAsync(B.x_d1_snap, B.x_d1, sizeof(float) * d * nseq, cudaMemcpyDeviceToDevice, e->s));
    if (B.samp) {
        FL_CHECK_CUDA(copy_rows(B.q_snap, 4 * V, B.q, 4 * V * kMaxDraft, 4 * V, nseq, cudaMemcpyDeviceToDevice, e->s));
        FL_CHECK_CUDA(copy_rows(B.m_snap, 8, B.m, 8 * (kMaxDraft + kMaxRows), 8, nseq, cudaMemcpyDeviceToDevice, e->s));
        if (B.traced)
            FL_CHECK_CUDA(copy_rows(B.trace_snap, 4 * V, B.trace, 4 * V * 2 * kMaxRows, 4 * V, nseq,
                                    cudaMemcpyDeviceToDevice, e->s));
    }
    FL_CHECK_CUDA(cudaStreamSynchronize(e->s));
    if (take_device_error() != 0) return set_error(FL_E_TIMEOUT, "batch_prefill: a bounded device wait gave up");
    FL_CHECK(build_batch_graph(e));
    B.ready = true;
    return FL_OK;
}

FL_API int fl_engine_batch_begin(fl_engine_t* e, int n_new) {
    FL_CHECK(check_ready(e, true));
    auto& B = e->bt;
    if (!B.ready || !B.exec) return set_error(FL_E_STATE, "batch_decode: call fl_engine_batch_prefill first");
    if (n_new <= 0 || B.P + n_new + B.K + 3 > B.slots) return set_error(FL_E_INVAL, "batch_decode: context too long");
    const size_t V = e->V, d = e->d;
    FL_CHECK_CUDA(cudaMemcpyAsync(B.st, B.st_snap, sizeof(SpecState) * B.n, cudaMemcpyDeviceToDevice, e->s));
    FL_CHECK_CUDA(cudaMemcpyAsync(B.x_d1, B.x_d1_snap, sizeof(float) * d * B.n, cudaMemcpyDeviceToDevice, e->s));
    if (B.samp) {
        FL_CHECK_CUDA(copy_rows(B.q, 4 * V * kMaxDraft, B.q_snap, 4 * V, 4 * V, B.n, cudaMemcpyDeviceToDevice, e->s));
        FL_CHECK_CUDA(copy_rows(B.m, 8 * (kMaxDraft + kMaxRows), B.m_snap, 8, 8, B.n, cudaMemcpyDeviceToDevice, e->s));
        if (B.traced)
            FL_CHECK_CUDA(copy_rows(B.trace, 4 * V * 2 * kMaxRows, B.trace_snap, 4 * V, 4 * V, B.n,
                                    cudaMemcpyDeviceToDevice, e->s));
    }
    // n_new and done of every record (adjacent ints)
    static_assert(offsetof(SpecState, done) == offsetof(SpecState, n_new) + sizeof(int), "n_new, done adjacent");
    std::vector<int> patch(2 * (size_t)B.n);
    for (int s = 0; s < B.n; s++) {
        patch[2 * s] = n_new;
        patch[2 * s + 1] = n_new <= 1 ? 1 : 0;
    }
    FL_CHECK_CUDA(copy_rows(&B.st->n_new, sizeof(SpecState), patch.data(), 2 * sizeof(int), 2 * sizeof(int), B.n,
                            cudaMemcpyHostToDevice, e->s));
    const BatchCtl c0 = {n_new <= 1 ? 0 : B.n, n_new <= 1 ? 1 : 0};
    FL_CHECK_CUDA(cudaMemcpyAsync(B.ctl, &c0, sizeof(c0), cudaMemcpyHostToDevice, e->s));
    FL_CHECK_CUDA(cudaStreamSynchronize(e->s));
    return FL_OK;
}

FL_API int fl_engine_batch_decode(fl_engine_t* e, int n_new, int* out, int* steps) {
    FL_CHECK(fl_engine_batch_begin(e, n_new));
    auto& B = e->bt;
    const int K = B.K;
    std::vector<SpecState> h(B.n);
    FL_CHECK_CUDA(cudaEventRecord(e->ev[0], e->s));
    long long launched = 0;
    // every step emits at least one token per unfinished sequence and at
    // most K + 1: launch the steps the slowest sequence needs at least, then
    // check again
    int chunk = (n_new - 1 + K) / (K + 1);
    while (chunk > 0) {
        for (int i = 0; i < chunk; i++) FL_CHECK_CUDA(cudaGraphLaunch(B.exec, e->s));
        launched += chunk;
        FL_CHECK_CUDA(cudaMemcpyAsync(h.data(), B.st, sizeof(SpecState) * B.n, cudaMemcpyDeviceToHost, e->s));
        FL_CHECK_CUDA(cudaStreamSynchronize(e->s));
        if (take_device_error() != 0) return set_error(FL_E_TIMEOUT, "batch_decode: a bounded device wait gave up");
        int rem = 0;
        for (const auto& x : h) rem = std::max(rem, x.done ? 0 : x.n_new - x.produced);
        if (rem > 0 && launched > n_new + 1) return set_error(FL_E_STATE, "batch_decode: no progress");
        chunk = (rem + K) / (K + 1);
    }
    FL_CHECK_CUDA(cudaEventRecord(e->ev[1], e->s));
    FL_CHECK_CUDA(cudaEventSynchronize(e->ev[1]));
    float ms = 0.0f;
    cudaEventElapsedTime(&ms, e->ev[0], e->ev[1]);
    e->t_total_us = ms * 1000.0;
    e->last_launches = launched * B.graph_kernels;
    if (out)
        FL_CHECK_CUDA(cudaMemcpy2D(out, sizeof(int) * n_new, B.out, sizeof(int) * B.slots, sizeof(int) * n_new, B.n,
                                   cudaMemcpyDeviceToHost));
    long long total = 0;
    for (int s = 0; s < B.n; s++) {
        if (steps) steps[s] = h[s].steps;
        total += h[s].steps;
    }
    return (int)std::min<long long>(total, INT_MAX);
}

FL_API int fl_engine_batch_trace(const fl_engine_t* e, int seq, float* logits, unsigned* qd, unsigned long long* qm,
                                 unsigned* pt, unsigned long long* pm, int* drafted) {
    if (!e) return set_error(FL_E_INVAL, "engine is NULL");
    const auto& B = e->bt;
    if (!B.ready || !B.traced) return set_error(FL_E_STATE, "batch_trace: prefill a sampled batch with the trace on");
    if (seq < 0 || seq >= B.n) return set_error(FL_E_INVAL, "batch_trace: no such sequence");
    FL_CHECK_CUDA(cudaSetDevice(e->device));
    FL_CHECK_CUDA(cudaStreamSynchronize(e->s));
    const size_t V = e->V, s = seq;
    if (logits)
        FL_CHECK_CUDA(cudaMemcpy(logits, B.trace + s * 2 * kMaxRows * V, sizeof(float) * 2 * kMaxRows * V,
                                 cudaMemcpyDeviceToHost));
    if (qd) FL_CHECK_CUDA(cudaMemcpy(qd, B.q + s * kMaxDraft * V, sizeof(uint32_t) * kMaxDraft * V, cudaMemcpyDeviceToHost));
    if (pt) FL_CHECK_CUDA(cudaMemcpy(pt, B.p + s * kMaxRows * V, sizeof(uint32_t) * kMaxRows * V, cudaMemcpyDeviceToHost));
    const unsigned long long* m = B.m + s * (kMaxDraft + kMaxRows);
    if (qm) FL_CHECK_CUDA(cudaMemcpy(qm, m, sizeof(unsigned long long) * kMaxDraft, cudaMemcpyDeviceToHost));
    if (pm) FL_CHECK_CUDA(cudaMemcpy(pm, m + kMaxDraft, sizeof(unsigned long long) * kMaxRows, cudaMemcpyDeviceToHost));
    if (drafted) {
        SpecState h;
        FL_CHECK_CUDA(cudaMemcpy(&h, B.st + s, sizeof(h), cudaMemcpyDeviceToHost));
        memcpy(drafted, h.drafted, sizeof(int) * kMaxDraft);
    }
    return FL_OK;
}

// One step of the prefilled batch (after fl_engine_batch_begin); state[s] =
// (n, produced, steps, a_last, done) of sequence s.
FL_API int fl_engine_batch_step(fl_engine_t* e, int* state) {
    FL_CHECK(check_ready(e, true));
    auto& B = e->bt;
    if (!B.ready || !B.exec) return set_error(FL_E_STATE, "batch_step: call fl_engine_batch_prefill first");
    FL_CHECK_CUDA(cudaGraphLaunch(B.exec, e->s));
    std::vector<SpecState> h(B.n);
    FL_CHECK_CUDA(cudaMemcpyAsync(h.data(), B.st, sizeof(SpecState) * B.n, cudaMemcpyDeviceToHost, e->s));
    FL_CHECK_CUDA(cudaStreamSynchronize(e->s));
    if (take_device_error() != 0) return set_error(FL_E_TIMEOUT, "batch_step: a bounded device wait gave up");
    if (state)
        for (int s = 0; s < B.n; s++) {
            int* o = state + 5 * s;
            o[0] = h[s].n;
            o[1] = h[s].produced;
            o[2] = h[s].steps;
            o[3] = h[s].a_last;
            o[4] = h[s].done;
        }
    return FL_OK;
}

FL_API int fl_engine_spec_generate_batch(fl_engine_t* e, const int* prompts, int P, int nseq, const unsigned* seq_ids,
                                         int n_new, int K, int* out, int* steps) {
    FL_CHECK(check_ready(e, true));
    if (!prompts || !out || nseq <= 0 || P <= 0 || n_new <= 0 || K < 1 || K > kMaxDraft)
        return set_error(FL_E_INVAL, "spec_generate_batch: bad arguments");
    const int slots = P + n_new + K + 3;
    auto& B = e->bt;
    const int rows_cap = std::min(nseq, e->R / (K + 1));
    if (e->tp_size > 1 && (B.cap < 1 || B.slots < slots))
        // every rank must run the same batches: no memory-dependent choice
        return set_error(FL_E_STATE, "spec_generate_batch: reserve the batch (fl_engine_batch_reserve) on every rank first");
    if (e->tp_size == 1 && (B.cap < rows_cap || B.slots < slots)) {
        // as many sequences per batch as rows and (80 % of) free memory allow
        // (an existing reservation that holds them all is kept)
        size_t fr = 0, tot = 0;
        FL_CHECK_CUDA(cudaMemGetInfo(&fr, &tot));
        size_t free_now = fr;
        if (B.cap) free_now += batch_bytes_per_seq(e, B.slots) * B.cap;
        const int need_slots = std::max(slots, B.slots);
        const long long by_mem = (long long)(free_now * 0.8 / batch_bytes_per_seq(e, need_slots));
        const int cap = (int)std::min<long long>((long long)rows_cap, by_mem);
        if (cap < 1) return set_error(FL_E_NOMEM, "spec_generate_batch: no room for one sequence");
        if (cap > B.cap || B.slots < slots) FL_CHECK(fl_engine_batch_reserve(e, cap, need_slots));
    }
    cudaEvent_t t0 = nullptr, t1 = nullptr;
    FL_CHECK_CUDA(cudaEventCreate(&t0));
    FL_CHECK_CUDA(cudaEventCreate(&t1));
    struct Ev {
        cudaEvent_t a, b;
        ~Ev() { cudaEventDestroy(a); cudaEventDestroy(b); }
    } ev_guard{t0, t1};
    FL_CHECK_CUDA(cudaEventRecord(t0, e->s));
    long long total = 0;
    std::vector<unsigned> ids(nseq);
    for (int i = 0; i < nseq; i++) ids[i] = seq_ids ? seq_ids[i] : (unsigned)i;
    std::vector<int> st(nseq);
    double decode_us = 0.0;
    for (int s0 = 0; s0 < nseq; s0 += B.cap) {
        const int n = std::min(B.cap, nseq - s0);
        FL_CHECK(fl_engine_batch_prefill(e, prompts + (size_t)s0 * P, P, n, ids.data() + s0, K));
        const int rc = fl_engine_batch_decode(e, n_new, out + (size_t)s0 * n_new, st.data() + s0);
        if (rc < 0) return rc;
        decode_us += e->t_total_us;
    }
    for (int i = 0; i < nseq; i++) {
        if (steps) steps[i] = st[i];
        total += st[i];
    }
    FL_CHECK_CUDA(cudaEventRecord(t1, e->s));
    FL_CHECK_CUDA(cudaEventSynchronize(t1));
    float ms = 0.0f;
    cudaEventElapsedTime(&ms, t0, t1);
    e->t_total_us = ms * 1000.0;
    e->t_verify_us = decode_us;  // the decode loops alone (prefills excluded)
    e->t_draft_us = 0.0;
    return (int)std::min<long long>(total, INT_MAX);
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
        *bytes_per_launch = (double)l0->N * l0->K * (1.0 + 1.0 / 16.0) + (double)M * l0->K + 4.0 * M * l0->N;
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
    for (int h = 0; h < H; h++) {
        if (topk[h] < 1 || topk[h] > 32) return set_error(FL_E_INVAL, "medusa_generate: top-k must be 1..32");
        kmax = std::max(kmax, topk[h]);
    }
    const int d = e->d, V = e->V;
    cudaStream_t s = e->s;
    // device work buffers for this call
    float *mf = nullptr, *my = nullptr, *mz = nullptr, *mprob = nullptr;
    int *mk = nullptr, *mtt = nullptr, *mtok = nullptr, *mpos = nullptr, *mtarget = nullptr, *mpath = nullptr;
    KvLayer* dkv = nullptr;
    auto cleanup = [&]() {
        void* bufs[] = {mf, my, mz, mprob, mk, mtt, mtok, mpos, mtarget, mpath, dkv};
        for (void* p : bufs) cudaFree(p);
    };
    auto fail = [&](int rc) {
        cleanup();
        return rc;
    };
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
    FL_MED_CUDA(cudaMalloc(&mf, sizeof(float) * d));
    FL_MED_CUDA(cudaMalloc(&my, sizeof(float) * (size_t)H * d));
    FL_MED_CUDA(cudaMalloc(&mz, sizeof(float) * (size_t)H * d));
    FL_MED_CUDA(cudaMalloc(&mprob, sizeof(float) * (size_t)H * kmax));
    FL_MED_CUDA(cudaMalloc(&mk, sizeof(int) * H));
    FL_MED_CUDA(cudaMalloc(&mtt, sizeof(int) * (size_t)H * kmax));
    FL_MED_CUDA(cudaMalloc(&mtok, sizeof(int) * max_nodes));
    FL_MED_CUDA(cudaMalloc(&mpos, sizeof(int) * max_nodes));
    FL_MED_CUDA(cudaMalloc(&mtarget, sizeof(int) * max_nodes));
    FL_MED_CUDA(cudaMalloc(&mpath, sizeof(int) * max_nodes));
    FL_MED_CUDA(cudaMalloc(&dkv, sizeof(KvLayer) * e->base.nl));
    FL_MED_CUDA(cudaMemcpyAsync(dkv, e->base.kv.data(), sizeof(KvLayer) * e->base.nl, cudaMemcpyHostToDevice, s));
    FL_MED_CUDA(cudaMemcpyAsync(mk, topk, sizeof(int) * H, cudaMemcpyHostToDevice, s));
    FL_MED(ensure_mask(e, max_nodes));

    // prefill: base KV 0 .. P-1, first token from the last prompt row
    FL_MED(prefill_base(e, prompt, P));
    FL_MED_CUDA(cudaMemcpyAsync(mf, e->x + (size_t)(P - 1) * d, sizeof(float) * d, cudaMemcpyDeviceToDevice, s));
    int cur_tok = 0;
    FL_MED_CUDA(cudaMemcpyAsync(&cur_tok, e->seq + P, sizeof(int), cudaMemcpyDeviceToHost, s));
    FL_MED_CUDA(cudaStreamSynchronize(s));
    int produced = 0, steps = 0, n = P;
    out[produced++] = cur_tok;
    std::vector<int> htok((size_t)H * kmax), target(max_nodes), ntok, npar, ndep, path;
    std::vector<float> hprob((size_t)H * kmax);
    std::vector<int> hpos(max_nodes);
    std::vector<uint8_t> mask((size_t)max_nodes * max_nodes);
    FL_MED_CUDA(cudaEventRecord(e->ev[0], s));
    while (produced < n_new) {
        // heads: h = RMSNorm(F), y_i = W_i h, z_i = h + SiLU(y_i), logits_i = LM(z_i)
        FL_MED_CUDA(launch_medusa_z(mf, my, e->x2, mz, d, 0, e->c.norm_eps, s));  // h -> x2
        for (int h = 0; h < H; h++) FL_MED(gemv_rows(e, e->medusa[h], e->x2, 1, false, my + (size_t)h * d, d));
        FL_MED_CUDA(launch_medusa_z(mf, my, nullptr, mz, d, H, e->c.norm_eps, s));
        FL_MED(gemv_rows(e, e->lm, mz, H, false, e->logits, V));
        FL_MED_CUDA(launch_topk_rows(e->logits, H, V, V, mk, kmax, mtt, mprob, s));
        FL_MED_CUDA(cudaMemcpyAsync(htok.data(), mtt, sizeof(int) * htok.size(), cudaMemcpyDeviceToHost, s));
        FL_MED_CUDA(cudaMemcpyAsync(hprob.data(), mprob, sizeof(float) * hprob.size(), cudaMemcpyDeviceToHost, s));
        FL_MED_CUDA(cudaStreamSynchronize(s));
        const int M = build_tree(cur_tok, H, topk, htok.data(), hprob.data(), kmax, max_nodes, ntok, npar, ndep);
        for (int i = 0; i < M; i++) {
            hpos[i] = n + ndep[i];
            for (int j = 0; j < M; j++) mask[(size_t)i * M + j] = 0;
            for (int j = i; j >= 0; j = npar[j]) mask[(size_t)i * M + j] = 1;
        }
        FL_MED_CUDA(cudaMemcpyAsync(mtok, ntok.data(), sizeof(int) * M, cudaMemcpyHostToDevice, s));
        FL_MED_CUDA(cudaMemcpyAsync(mpos, hpos.data(), sizeof(int) * M, cudaMemcpyHostToDevice, s));
        FL_MED_CUDA(cudaMemcpyAsync(e->mask, mask.data(), (size_t)M * M, cudaMemcpyHostToDevice, s));
        // tree-masked verify: node i at slot n + i, rotary position n + depth
        FL_MED_CUDA(launch_embed_rows(e->embed, V, mtok, nullptr, 0, e->x, d, M, nullptr, nullptr, s, false));
        FL_MED(run_stack(e, e->base, e->x, M, nullptr, e->iota + n, mpos, e->mask, nullptr, false));
        for (int r0 = 0; r0 < M; r0 += kMaxRows) {
            const int m = std::min(kMaxRows, M - r0);
            FL_MED(run_lm(e, e->x + (size_t)r0 * d, m, nullptr, nullptr, false));
            FL_MED_CUDA(launch_argmax_rows(e->amax, e->nparts, m, mtarget + r0, nullptr, s));
        }
        FL_MED_CUDA(cudaMemcpyAsync(target.data(), mtarget, sizeof(int) * M, cudaMemcpyDeviceToHost, s));
        FL_MED_CUDA(cudaStreamSynchronize(s));
        // longest path of the base model's greedy choices
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
        if (a > 0) {
            FL_MED_CUDA(cudaMemcpyAsync(mpath, path.data(), sizeof(int) * (a + 1), cudaMemcpyHostToDevice, s));
            FL_MED_CUDA(launch_kv_compact(dkv, e->base.nl, e->base.block_table, e->Hkv, e->hd, e->iota + n, mpath, a, s));
        }
        FL_MED_CUDA(cudaMemcpyAsync(mf, e->x + (size_t)cur * d, sizeof(float) * d, cudaMemcpyDeviceToDevice, s));
        cur_tok = target[cur];
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
    cleanup();
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

namespace {

// Static draft-tree shape: node 0 is the root, then per depth j = 1 .. K the
// chain node (first) and width - 1 siblings, all children of the chain node
// of depth j - 1. mask[i * Mt + j] = 1 where node j is node i or one of its
// ancestors.
void draft_tree_shape(int K, int width, std::vector<int>& par, std::vector<int>& dep, std::vector<uint8_t>& mask) {
    const int Mt = 1 + K * width;
    par.assign(Mt, -1);
    dep.assign(Mt, 0);
    for (int j = 1; j <= K; j++)
        for (int c2 = 0; c2 < width; c2++) {
            const int i = 1 + (j - 1) * width + c2;
            par[i] = j == 1 ? 0 : 1 + (j - 2) * width;
            dep[i] = j;
        }
    mask.assign((size_t)Mt * Mt, 0);
    for (int i = 0; i < Mt; i++)
        for (int j = i; j >= 0; j = par[j]) mask[(size_t)i * Mt + j] = 1;
}

// Greedy tree acceptance: from the root, follow the child whose token is the
// base model's choice at its parent (target[parent]) while there is one.
// path[0] = 0 (the root); returns the accepted nodes (path length - 1).
int accept_path(const int* tok, const int* par, const int* target, int M, std::vector<int>& path) {
    path.assign(1, 0);
    int cur = 0;
    for (;;) {
        int nxt = -1;
        for (int c2 = 1; c2 < M; c2++)
            if (par[c2] == cur && tok[c2] == target[cur]) {
                nxt = c2;
                break;
            }
        if (nxt < 0) break;
        path.push_back(nxt);
        cur = nxt;
    }
    return (int)path.size() - 1;
}

// The width best candidates of one depth from every rank's top-width keys
// (value, global index; larger first): their token ids, best first.
void merge_topw(const unsigned long long* keys, int ranks, size_t rank_stride, int width, int* tok) {
    std::vector<unsigned long long> cand;
    for (int r = 0; r < ranks; r++)
        for (int c2 = 0; c2 < width; c2++) cand.push_back(keys[(size_t)r * rank_stride + c2]);
    std::sort(cand.begin(), cand.end(), std::greater<unsigned long long>());
    for (int c2 = 0; c2 < width; c2++) tok[c2] = 0x7fffffff - (int)(uint32_t)(cand[c2] & 0xffffffffu);
}

}  // namespace

// Static draft tree (EAGLE-style): the draft chain c_1..c_K plus, at every
// depth j, the draft's next w - 1 candidates after c_j, all children of
// c_{j-1} (c_0 = the newest committed token). Nodes in depth order: root,
// then per depth [c_j, siblings]; 1 + K w nodes. One tree-masked verify pass,
// greedy acceptance of the longest path whose tokens match the base argmax at
// their parents (a sibling ends the path), KV compaction of the path and the
// draft catch-up over it, as in fl_engine_spec_medusa_generate. Under tensor
// parallelism each rank's top-w keys (value, global index) are all-gathered
// and merged, so every rank builds the same tree.
FL_API int fl_engine_spec_tree_generate(fl_engine_t* e, const int* prompt, int P, int n_new, int K, int width,
                                        int* out, int* acc_hist, int* steps_out) {
    FL_CHECK(check_ready(e, true));
    const int Mt = 1 + K * width;
    if (!prompt || !out || P <= 0 || n_new <= 0 || K < 1 || K > kMaxDraft || width < 1 || width > 32 ||
        Mt > 256 || P + n_new + Mt + K + 2 > e->R)
        return set_error(FL_E_INVAL, "spec_tree_generate: bad arguments or context too long");
    const int d = e->d, G = e->tp_size;
    cudaStream_t s = e->s;
    int *mtok = nullptr, *mpos = nullptr, *mtarget = nullptr, *mpath = nullptr, *mchain = nullptr, *mcat = nullptr;
    unsigned long long *mkeys = nullptr, *mall = nullptr;
    KvLayer* dkv = nullptr;
    auto cleanup = [&]() {
        void* bufs[] = {mtok, mpos, mtarget, mpath, mchain, mcat, mkeys, mall, dkv};
        for (void* p : bufs) cudaFree(p);
    };
    auto fail = [&](int rc) {
        cleanup();
        return rc;
    };
#define FL_ST_CUDA(expr)                                                     \
    do {                                                                     \
        cudaError_t fl_e_ = (expr);                                          \
        if (fl_e_ != cudaSuccess) return fail(cuda_error(fl_e_, #expr));     \
    } while (0)
#define FL_ST(expr)                       \
    do {                                  \
        int fl_r_ = (expr);               \
        if (fl_r_ != FL_OK) return fail(fl_r_); \
    } while (0)
    FL_ST_CUDA(cudaMalloc(&mtok, sizeof(int) * Mt));
    FL_ST_CUDA(cudaMalloc(&mpos, sizeof(int) * Mt));
    FL_ST_CUDA(cudaMalloc(&mtarget, sizeof(int) * Mt));
    FL_ST_CUDA(cudaMalloc(&mpath, sizeof(int) * Mt));
    FL_ST_CUDA(cudaMalloc(&mchain, sizeof(int) * kMaxRows));
    FL_ST_CUDA(cudaMalloc(&mcat, sizeof(int) * Mt));
    FL_ST_CUDA(cudaMalloc(&mkeys, sizeof(unsigned long long) * K * width));
    FL_ST_CUDA(cudaMalloc(&mall, sizeof(unsigned long long) * K * width * G));
    FL_ST_CUDA(cudaMalloc(&dkv, sizeof(KvLayer) * e->base.nl));
    FL_ST_CUDA(cudaMemcpyAsync(dkv, e->base.kv.data(), sizeof(KvLayer) * e->base.nl, cudaMemcpyHostToDevice, s));
    FL_ST(ensure_mask(e, Mt));

    // prefill: base KV 0 .. P-1 and the first token; draft catch-up over 0 .. P
    FL_ST(prefill_base(e, prompt, P));
    FL_ST_CUDA(launch_embed_rows(e->embed, e->Vg, e->seq, e->x, 1, e->x2, d, P + 1, nullptr, nullptr, s, false));
    FL_ST(run_stack(e, e->draft, e->x2, P + 1, nullptr, e->iota, e->iota, nullptr, nullptr, false));
    FL_ST_CUDA(cudaMemcpyAsync(e->x_d, e->x2 + (size_t)P * d, sizeof(float) * d, cudaMemcpyDeviceToDevice, s));
    int cur_tok = 0;
    FL_ST_CUDA(cudaMemcpyAsync(&cur_tok, e->seq + P, sizeof(int), cudaMemcpyDeviceToHost, s));
    FL_ST_CUDA(cudaStreamSynchronize(s));
    int produced = 0, steps = 0, n = P;
    out[produced++] = cur_tok;
    std::vector<unsigned long long> keys((size_t)K * width * G);
    std::vector<int> ntok(Mt), npar, ndep, hpos(Mt), target(Mt), path, cat;
    std::vector<uint8_t> mask;
    draft_tree_shape(K, width, npar, ndep, mask);
    FL_ST_CUDA(cudaMemcpyAsync(e->mask, mask.data(), (size_t)Mt * Mt, cudaMemcpyHostToDevice, s));
    FL_ST_CUDA(cudaEventRecord(e->ev[0], s));
    while (produced < n_new) {
        // draft chain from the draft state at position n (x_d row 0); each
        // depth's top-w keys
        for (int j = 0; j < K; j++) {
            if (j > 0) {
                FL_ST_CUDA(launch_embed_rows(e->embed, e->Vg, mchain + j - 1, e->x_d, 0, e->x_d, d, 1, nullptr, nullptr, s,
                                             false));
                FL_ST(run_stack(e, e->draft, e->x_d, 1, nullptr, e->iota + n + j, e->iota + n + j, nullptr, nullptr,
                                false));
            }
            FL_ST(run_lm(e, e->x_d, 1, nullptr, nullptr, false));
            FL_ST_CUDA(launch_argmax_rows(amax_keys(e), amax_nparts(e), 1, mchain + j, nullptr, s));
            FL_ST_CUDA(launch_topk_keys(e->logits, 1, e->V, e->V, G > 1 ? e->tp.v0 : 0, width,
                                        mkeys + (size_t)j * width, s));
        }
        if (G > 1) FL_ST(tp_allgather_u64(e->tp_comm, mkeys, mall, (size_t)K * width, s));
        FL_ST_CUDA(cudaMemcpyAsync(keys.data(), G > 1 ? mall : mkeys, sizeof(unsigned long long) * keys.size(),
                                   cudaMemcpyDeviceToHost, s));
        FL_ST_CUDA(cudaStreamSynchronize(s));
        ntok[0] = cur_tok;
        for (int j = 0; j < K; j++)  // depth j + 1: the ranks' candidates merged
            merge_topw(keys.data() + (size_t)j * width, G, (size_t)K * width, width, ntok.data() + 1 + j * width);
        for (int i = 0; i < Mt; i++) hpos[i] = n + ndep[i];
        FL_ST_CUDA(cudaMemcpyAsync(mtok, ntok.data(), sizeof(int) * Mt, cudaMemcpyHostToDevice, s));
        FL_ST_CUDA(cudaMemcpyAsync(mpos, hpos.data(), sizeof(int) * Mt, cudaMemcpyHostToDevice, s));
        FL_ST_CUDA(launch_embed_rows(e->embed, e->Vg, mtok, nullptr, 0, e->x, d, Mt, nullptr, nullptr, s, false));
        FL_ST(run_stack(e, e->base, e->x, Mt, nullptr, e->iota + n, mpos, e->mask, nullptr, false));
        for (int r0 = 0; r0 < Mt; r0 += kMaxRows) {
            const int m = std::min(kMaxRows, Mt - r0);
            FL_ST(run_lm(e, e->x + (size_t)r0 * d, m, nullptr, nullptr, false));
            FL_ST_CUDA(launch_argmax_rows(amax_keys(e), amax_nparts(e), m, mtarget + r0, nullptr, s));
        }
        FL_ST_CUDA(cudaMemcpyAsync(target.data(), mtarget, sizeof(int) * Mt, cudaMemcpyDeviceToHost, s));
        FL_ST_CUDA(cudaStreamSynchronize(s));
        const int a = accept_path(ntok.data(), npar.data(), target.data(), Mt, path);
        const int cur = path[a];
        if (acc_hist) acc_hist[steps] = a;
        steps++;
        for (int j = 1; j <= a + 1 && produced < n_new; j++) out[produced++] = j <= a ? ntok[path[j]] : target[cur];
        // draft catch-up over positions n+1 .. n+a+1: F of the path's tree rows + E[token]
        cat.resize(a + 1);
        for (int j = 0; j <= a; j++) cat[j] = j < a ? ntok[path[j + 1]] : target[cur];
        FL_ST_CUDA(cudaMemcpyAsync(mcat, cat.data(), sizeof(int) * (a + 1), cudaMemcpyHostToDevice, s));
        for (int j = 0; j <= a; j++)
            FL_ST_CUDA(cudaMemcpyAsync(e->x2 + (size_t)j * d, e->x + (size_t)path[j] * d, sizeof(float) * d,
                                       cudaMemcpyDeviceToDevice, s));
        if (a > 0) {
            FL_ST_CUDA(cudaMemcpyAsync(mpath, path.data(), sizeof(int) * (a + 1), cudaMemcpyHostToDevice, s));
            FL_ST_CUDA(launch_kv_compact(dkv, e->base.nl, e->base.block_table, e->Hkv, e->hd, e->iota + n, mpath, a, s));
        }
        FL_ST_CUDA(launch_embed_rows(e->embed, e->Vg, mcat, e->x2, 0, e->x2, d, a + 1, nullptr, nullptr, s, false));
        FL_ST(run_stack(e, e->draft, e->x2, a + 1, nullptr, e->iota + n + 1, e->iota + n + 1, nullptr, nullptr, false));
        FL_ST_CUDA(cudaMemcpyAsync(e->x_d, e->x2 + (size_t)a * d, sizeof(float) * d, cudaMemcpyDeviceToDevice, s));
        cur_tok = target[cur];
        n += a + 1;
    }
    FL_ST_CUDA(cudaEventRecord(e->ev[1], s));
    FL_ST_CUDA(cudaEventSynchronize(e->ev[1]));
    float ms = 0.0f;
    cudaEventElapsedTime(&ms, e->ev[0], e->ev[1]);
    e->t_total_us = ms * 1000.0;
    if (steps_out) *steps_out = steps;
#undef FL_ST_CUDA
#undef FL_ST
    cleanup();
    if (take_device_error() != 0) return set_error(FL_E_TIMEOUT, "spec_tree_generate: a bounded device wait gave up");
    return FL_OK;
}

// Static draft tree for an in-GPU batch (greedy): every step each sequence's
// draft chain runs as one batched row per sequence, each depth's top-width
// candidates form that sequence's tree (the shape of
// fl_engine_spec_tree_generate, shared by all sequences), and the trees of
// all sequences are verified in one tree-masked pass of nseq x (1 + k width)
// rows over the sequences' own KV regions; then per sequence the accepted
// path, its KV compaction, and one batched draft catch-up over k + 1 rows per
// sequence (rows past its path zeroed and unused). On a tensor-parallel
// engine the ranks' candidates are gathered and merged as in the
// one-sequence tree. Needs fl_engine_batch_reserve(nseq, >= prompt_len + n_new
// + 1 + k width + k + 3) on every rank.
FL_API int fl_engine_batch_tree_generate(fl_engine_t* e, const int* prompts, int P, int nseq, int n_new, int K,
                                         int width, int* out, int* steps_out) {
    FL_CHECK(check_ready(e, true));
    auto& B = e->bt;
    const int Mt = 1 + K * width;
    if (!prompts || !out || P <= 0 || nseq <= 0 || n_new <= 0 || K < 1 || K > kMaxDraft || width < 1 || width > 32 ||
        Mt > 256)
        return set_error(FL_E_INVAL, "batch_tree_generate: bad arguments");
    if (nseq > B.cap || P + n_new + Mt + K + 3 > B.slots || nseq * Mt > e->R)
        return set_error(FL_E_INVAL, "batch_tree_generate: batch or context larger than the reservation");
    if (e->samp) return set_error(FL_E_UNSUPPORTED, "batch_tree_generate: the tree decode is greedy");
    if (e->d % 128 != 0) return set_error(FL_E_UNSUPPORTED, "batch: the hidden size must be a multiple of 128");
    const int d = e->d, G = e->tp_size, V = e->V, rows = nseq * Mt, cw = K * width;
    const size_t npart = (size_t)e->nparts;
    cudaStream_t s = e->s;
    FL_CHECK(tp_ensure_rows(e, rows));
    float* lg = nullptr;
    unsigned long long *am = nullptr, *mkeys = nullptr, *mall = nullptr;
    int *mtok = nullptr, *mvst = nullptr, *mdst = nullptr, *mcst = nullptr, *mtarget = nullptr, *mchain = nullptr,
        *mpath = nullptr, *mbase = nullptr, *mcat = nullptr;
    KvLayer* dkv = nullptr;
    auto cleanup = [&]() {
        void* bufs[] = {lg, am, mkeys, mall, mtok, mvst, mdst, mcst, mtarget, mchain, mpath, mbase, mcat, dkv};
        for (void* p : bufs) cudaFree(p);
    };
    auto fail = [&](int rc) {
        cleanup();
        return rc;
    };
#define FL_BT_CUDA(expr)                                                     \
    do {                                                                     \
        cudaError_t fl_e_ = (expr);                                          \
        if (fl_e_ != cudaSuccess) return fail(cuda_error(fl_e_, #expr));     \
    } while (0)
#define FL_BT(expr)                       \
    do {                                  \
        int fl_r_ = (expr);               \
        if (fl_r_ != FL_OK) return fail(fl_r_); \
    } while (0)
    const int nlb = e->base.nl;
    FL_BT_CUDA(cudaMalloc(&lg, sizeof(float) * (size_t)rows * V));
    FL_BT_CUDA(cudaMalloc(&am, sizeof(unsigned long long) * (size_t)rows * npart));
    FL_BT_CUDA(cudaMalloc(&mkeys, sizeof(unsigned long long) * (size_t)nseq * cw));
    FL_BT_CUDA(cudaMalloc(&mall, sizeof(unsigned long long) * (size_t)nseq * cw * G));
    FL_BT_CUDA(cudaMalloc(&mtok, sizeof(int) * rows));
    FL_BT_CUDA(cudaMalloc(&mvst, sizeof(int) * (size_t)nseq * (Mt + 1)));
    FL_BT_CUDA(cudaMalloc(&mdst, sizeof(int) * (size_t)K * nseq * 2));
    FL_BT_CUDA(cudaMalloc(&mcst, sizeof(int) * (size_t)nseq * (K + 2)));
    FL_BT_CUDA(cudaMalloc(&mtarget, sizeof(int) * rows));
    FL_BT_CUDA(cudaMalloc(&mchain, sizeof(int) * (size_t)K * nseq));
    FL_BT_CUDA(cudaMalloc(&mpath, sizeof(int) * rows));
    FL_BT_CUDA(cudaMalloc(&mbase, sizeof(int) * nseq));
    FL_BT_CUDA(cudaMalloc(&mcat, sizeof(int) * (size_t)nseq * (K + 1)));
    FL_BT_CUDA(cudaMalloc(&dkv, sizeof(KvLayer) * (size_t)nseq * nlb));
    // each sequence's base KV region as its own cache (compaction)
    const size_t region = (size_t)(B.slots / kPageSize) * e->Hkv * kPageSize * e->hd;
    std::vector<KvLayer> hkv((size_t)nseq * nlb);
    for (int q = 0; q < nseq; q++)
        for (int l = 0; l < nlb; l++)
            hkv[(size_t)q * nlb + l] = {B.kv_base[l].k + q * region, B.kv_base[l].v + q * region};
    FL_BT_CUDA(cudaMemcpyAsync(dkv, hkv.data(), sizeof(KvLayer) * hkv.size(), cudaMemcpyHostToDevice, s));
    FL_BT(ensure_mask(e, Mt));
    const unsigned long long* keys_lm = G > 1 ? e->tp_best : am;
    const int np_lm = G > 1 ? 1 : e->nparts;
    // prefill per sequence into its regions: base KV 0 .. P-1, the first
    // (greedy) token, the draft catch-up over 0 .. P; x_d1[q] = the draft
    // feature at position P
    {
        std::vector<KvLayer> rb(nlb), rd(e->draft.nl);
        for (int q = 0; q < nseq; q++) {
            for (int l = 0; l < nlb; l++) rb[l] = hkv[(size_t)q * nlb + l];
            for (size_t l = 0; l < rd.size(); l++) rd[l] = {B.kv_draft[l].k + q * region, B.kv_draft[l].v + q * region};
            KvView vb, vd;
            vb.kv = rb.data();
            vd.kv = rd.data();
            vb.block_table = vd.block_table = B.block;
            int* sq = B.seq + (size_t)q * B.slots;
            FL_BT_CUDA(cudaMemcpyAsync(sq, prompts + (size_t)q * P, sizeof(int) * P, cudaMemcpyHostToDevice, s));
            FL_BT_CUDA(launch_embed_rows(e->embed, e->Vg, sq, nullptr, 0, e->x, d, P, nullptr, nullptr, s, false));
            FL_BT(run_stack(e, e->base, e->x, P, nullptr, e->iota, e->iota, nullptr, nullptr, false, &vb));
            FL_BT(run_lm(e, e->x + (size_t)(P - 1) * d, 1, nullptr, nullptr, false, lg, am));
            FL_BT_CUDA(launch_argmax_rows(keys_lm, np_lm, 1, sq + P, nullptr, s));
            FL_BT_CUDA(launch_embed_rows(e->embed, e->Vg, sq, e->x, 1, e->x2, d, P + 1, nullptr, nullptr, s, false));
            FL_BT(run_stack(e, e->draft, e->x2, P + 1, nullptr, e->iota, e->iota, nullptr, nullptr, false, &vd));
            FL_BT_CUDA(cudaMemcpyAsync(B.x_d1 + (size_t)q * d, e->x2 + (size_t)P * d, sizeof(float) * d,
                                       cudaMemcpyDeviceToDevice, s));
        }
    }
    // static tree shape (as fl_engine_spec_tree_generate) and its mask
    std::vector<int> npar, ndep;
    std::vector<uint8_t> mask;
    draft_tree_shape(K, width, npar, ndep, mask);
    FL_BT_CUDA(cudaMemcpyAsync(e->mask, mask.data(), (size_t)Mt * Mt, cudaMemcpyHostToDevice, s));
    // views of the batch's KV regions for the three kinds of pass
    auto view = [&](bool base, int seq_rows, int state) {
        KvView v;
        v.kv = base ? B.kv_base.data() : B.kv_draft.data();
        v.block_table = B.block;
        v.seqs = nseq;
        v.seq_rows = seq_rows;
        v.seq_state = state;
        v.seq_slots = B.slots;
        v.max_ctx = B.slots;
        v.attn_part = B.attn_part;
        v.attn_cnt = B.attn_cnt;
        return v;
    };
    const KvView vdraft = view(false, 1, 2), vverify = view(true, Mt, Mt + 1), vcatch = view(false, K + 1, K + 2);
    std::vector<int> n(nseq, P), produced(nseq, 1), steps(nseq, 0), cur_tok(nseq), target(rows), ntok(rows);
    std::vector<int> hd_state((size_t)K * nseq * 2), hv_state((size_t)nseq * (Mt + 1)), hc_state((size_t)nseq * (K + 2));
    std::vector<int> hpath(rows), hcat((size_t)nseq * (K + 1)), acc(nseq), last_row(nseq), live(nseq), pathv;
    std::vector<unsigned long long> keys((size_t)nseq * cw * G);
    FL_BT_CUDA(cudaMemcpy2DAsync(cur_tok.data(), sizeof(int), B.seq + P, sizeof(int) * B.slots, sizeof(int), nseq,
                                 cudaMemcpyDeviceToHost, s));
    FL_BT_CUDA(cudaStreamSynchronize(s));
    for (int q = 0; q < nseq; q++) out[(size_t)q * n_new] = cur_tok[q];
    FL_BT_CUDA(cudaEventRecord(e->ev[0], s));
    auto active = [&]() {
        for (int q = 0; q < nseq; q++)
            if (produced[q] < n_new) return true;
        return false;
    };
    while (active()) {
        // draft chains: depth j of every sequence in one single-row pass
        for (int j = 0; j < K; j++)
            for (int q = 0; q < nseq; q++) {
                hd_state[((size_t)j * nseq + q) * 2] = n[q] + j;
                hd_state[((size_t)j * nseq + q) * 2 + 1] = n[q] + j;
            }
        FL_BT_CUDA(cudaMemcpyAsync(mdst, hd_state.data(), sizeof(int) * hd_state.size(), cudaMemcpyHostToDevice, s));
        for (int j = 0; j < K; j++) {
            if (j > 0) {
                FL_BT_CUDA(launch_embed_rows(e->embed, e->Vg, mchain + (size_t)(j - 1) * nseq, B.x_d1, 0, B.x_d1, d,
                                             nseq, nullptr, nullptr, s, false));
                const int* st = mdst + (size_t)j * nseq * 2;
                FL_BT(run_stack(e, e->draft, B.x_d1, nseq, nullptr, st, st + 1, nullptr, nullptr, false, &vdraft));
            }
            FL_BT(run_lm(e, B.x_d1, nseq, nullptr, nullptr, false, lg, am));
            FL_BT_CUDA(launch_argmax_rows(keys_lm, np_lm, nseq, mchain + (size_t)j * nseq, nullptr, s));
            FL_BT_CUDA(launch_topk_keys(lg, nseq, V, V, G > 1 ? e->tp.v0 : 0, width, mkeys + (size_t)j * nseq * width, s));
        }
        if (G > 1) FL_BT(tp_allgather_u64(e->tp_comm, mkeys, mall, (size_t)nseq * cw, s));
        FL_BT_CUDA(cudaMemcpyAsync(keys.data(), G > 1 ? mall : mkeys, sizeof(unsigned long long) * keys.size(),
                                   cudaMemcpyDeviceToHost, s));
        FL_BT_CUDA(cudaStreamSynchronize(s));
        // per sequence: merge the ranks' candidates of each depth into its tree
        for (int q = 0; q < nseq; q++) {
            int* tk = ntok.data() + (size_t)q * Mt;
            tk[0] = cur_tok[q];
            for (int j = 0; j < K; j++)
                merge_topw(keys.data() + ((size_t)j * nseq + q) * width, G, (size_t)K * nseq * width, width,
                           tk + 1 + j * width);
            hv_state[(size_t)q * (Mt + 1)] = n[q];
            for (int i = 0; i < Mt; i++) hv_state[(size_t)q * (Mt + 1) + 1 + i] = n[q] + ndep[i];
        }
        FL_BT_CUDA(cudaMemcpyAsync(mtok, ntok.data(), sizeof(int) * rows, cudaMemcpyHostToDevice, s));
        FL_BT_CUDA(cudaMemcpyAsync(mvst, hv_state.data(), sizeof(int) * hv_state.size(), cudaMemcpyHostToDevice, s));
        FL_BT_CUDA(launch_embed_rows(e->embed, e->Vg, mtok, nullptr, 0, e->x, d, rows, nullptr, nullptr, s, false));
        FL_BT(run_stack(e, e->base, e->x, rows, nullptr, mvst, mvst + 1, e->mask, nullptr, false, &vverify));
        FL_BT(run_lm(e, e->x, rows, nullptr, nullptr, false, lg, am));
        FL_BT_CUDA(launch_argmax_rows(keys_lm, np_lm, rows, mtarget, nullptr, s));
        FL_BT_CUDA(cudaMemcpyAsync(target.data(), mtarget, sizeof(int) * rows, cudaMemcpyDeviceToHost, s));
        FL_BT_CUDA(cudaStreamSynchronize(s));
        // per sequence: accepted path, emitted tokens, compaction, catch-up rows
        FL_BT_CUDA(cudaMemsetAsync(B.x_dc, 0, sizeof(float) * (size_t)nseq * (K + 1) * d, s));
        for (int q = 0; q < nseq; q++) {
            const int* tk = ntok.data() + (size_t)q * Mt;
            const int* tg = target.data() + (size_t)q * Mt;
            int* path = hpath.data() + (size_t)q * Mt;
            const int a = accept_path(tk, npar.data(), tg, Mt, pathv);
            const int cur = pathv[a];
            std::copy(pathv.begin(), pathv.end(), path);
            live[q] = produced[q] < n_new;  // finished sequences stay where they are
            acc[q] = live[q] ? a : 0;
            last_row[q] = a;
            int* cat = hcat.data() + (size_t)q * (K + 1);
            for (int j = 0; j <= K; j++) cat[j] = j < a ? tk[path[j + 1]] : (j == a ? tg[cur] : 0);
            hc_state[(size_t)q * (K + 2)] = n[q] + 1;
            for (int j = 0; j <= K; j++) hc_state[(size_t)q * (K + 2) + 1 + j] = n[q] + 1 + j;
            if (live[q]) {
                for (int j = 1; j <= a + 1 && produced[q] < n_new; j++)
                    out[(size_t)q * n_new + produced[q]++] = j <= a ? tk[path[j]] : tg[cur];
                steps[q]++;
            }
            for (int j = 0; j <= a; j++)
                FL_BT_CUDA(cudaMemcpyAsync(B.x_dc + ((size_t)q * (K + 1) + j) * d, e->x + ((size_t)q * Mt + path[j]) * d,
                                           sizeof(float) * d, cudaMemcpyDeviceToDevice, s));
            cur_tok[q] = tg[cur];
        }
        std::vector<int> hbase(nseq);
        for (int q = 0; q < nseq; q++) hbase[q] = n[q];
        FL_BT_CUDA(cudaMemcpyAsync(mbase, hbase.data(), sizeof(int) * nseq, cudaMemcpyHostToDevice, s));
        FL_BT_CUDA(cudaMemcpyAsync(mpath, hpath.data(), sizeof(int) * rows, cudaMemcpyHostToDevice, s));
        for (int q = 0; q < nseq; q++)
            if (acc[q] > 0)
                FL_BT_CUDA(launch_kv_compact(dkv + (size_t)q * nlb, nlb, B.block, e->Hkv, e->hd, mbase + q,
                                             mpath + (size_t)q * Mt, acc[q], s));
        FL_BT_CUDA(cudaMemcpyAsync(mcat, hcat.data(), sizeof(int) * hcat.size(), cudaMemcpyHostToDevice, s));
        FL_BT_CUDA(cudaMemcpyAsync(mcst, hc_state.data(), sizeof(int) * hc_state.size(), cudaMemcpyHostToDevice, s));
        FL_BT_CUDA(launch_embed_rows(e->embed, e->Vg, mcat, B.x_dc, 0, B.x_dc, d, nseq * (K + 1), nullptr, nullptr, s,
                                     false));
        FL_BT(run_stack(e, e->draft, B.x_dc, nseq * (K + 1), nullptr, mcst, mcst + 1, nullptr, nullptr, false, &vcatch));
        for (int q = 0; q < nseq; q++) {
            FL_BT_CUDA(cudaMemcpyAsync(B.x_d1 + (size_t)q * d, B.x_dc + ((size_t)q * (K + 1) + last_row[q]) * d,
                                       sizeof(float) * d, cudaMemcpyDeviceToDevice, s));
            if (live[q]) n[q] += acc[q] + 1;
        }
    }
    FL_BT_CUDA(cudaEventRecord(e->ev[1], s));
    FL_BT_CUDA(cudaEventSynchronize(e->ev[1]));
    float ms = 0.0f;
    cudaEventElapsedTime(&ms, e->ev[0], e->ev[1]);
    e->t_total_us = ms * 1000.0;
    long long total = 0;
    for (int q = 0; q < nseq; q++) {
        if (steps_out) steps_out[q] = steps[q];
        total += steps[q];
    }
#undef FL_BT_CUDA
#undef FL_BT
    cleanup();
    if (take_device_error() != 0) return set_error(FL_E_TIMEOUT, "batch_tree_generate: a bounded device wait gave up");
    return (int)std::min<long long>(total, INT_MAX);
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
