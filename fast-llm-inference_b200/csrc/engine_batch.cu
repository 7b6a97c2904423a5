// In-GPU batches of independent sequences and static draft trees for the
// device engine (fl_engine_batch_*, fl_engine_spec_tree_generate,
// fl_engine_batch_tree_generate; include/fl_cuda.h).
#include <stddef.h>
#include <string.h>

#include <algorithm>
#include <climits>
#include <functional>
#include <vector>

#include "fl_engine_impl.h"

// ---------------------------------------------------------------------------
// In-GPU batch of independent sequences. Every step runs each draft pass
// over one row per sequence and the verify and draft catch-up passes over
// K + 1 rows per sequence, so the weights stream once per pass for the whole
// batch (the tcgen05 GEMM takes passes of more than 16 rows). Each sequence
// keeps its own KV region, state record, token arrays and Philox key
// (seed, sequence id); its decisions are those of the one-sequence step.
// ---------------------------------------------------------------------------
namespace fl_eng {

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

}  // namespace fl_eng

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

// Host entry points of the tensor-parallel candidate merge (for tests of the
// control flow without a GPU): a logit's orderable argmax key, and the merge
// of the ranks' top-width keys into the width best tokens.
FL_API unsigned long long fl_argmax_key(float v, int index) { return argmax_key(v, index); }

FL_API int fl_tp_merge_topw(const unsigned long long* keys, int ranks, size_t rank_stride, int width, int* tok) {
    if (!keys || !tok || ranks < 1 || width < 1 || rank_stride < (size_t)width)
        return set_error(FL_E_INVAL, "tp_merge_topw: bad arguments");
    merge_topw(keys, ranks, rank_stride, width, tok);
    return FL_OK;
}

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
    auto cleanup = [&]() {};  // the work buffers belong to the engine's arena
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
    {
        const size_t sizes[] = {sizeof(int) * Mt, sizeof(int) * Mt, sizeof(int) * Mt, sizeof(int) * Mt,
                                sizeof(int) * kMaxRows, sizeof(int) * Mt, sizeof(unsigned long long) * K * width,
                                sizeof(unsigned long long) * K * width * G, sizeof(KvLayer) * e->base.nl};
        void** ptrs[] = {(void**)&mtok, (void**)&mpos, (void**)&mtarget, (void**)&mpath, (void**)&mchain,
                         (void**)&mcat, (void**)&mkeys, (void**)&mall, (void**)&dkv};
        FL_ST(carve_work(e, ptrs, sizes, 9));
    }
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
    // the per-sequence prefill embeds P + 1 rows into the engine's R-row
    // activation buffers, so the prompt is bounded by R as well as the slots
    if (nseq > B.cap || P + n_new + Mt + K + 3 > B.slots || nseq * Mt > e->R || P + 2 > e->R)
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
    auto cleanup = [&]() {};  // the work buffers belong to the engine's arena
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
    {
        const size_t sizes[] = {sizeof(float) * (size_t)rows * V, sizeof(unsigned long long) * (size_t)rows * npart,
                                sizeof(unsigned long long) * (size_t)nseq * cw,
                                sizeof(unsigned long long) * (size_t)nseq * cw * G, sizeof(int) * rows,
                                sizeof(int) * (size_t)nseq * (Mt + 1), sizeof(int) * (size_t)K * nseq * 2,
                                sizeof(int) * (size_t)nseq * (K + 2), sizeof(int) * rows, sizeof(int) * (size_t)K * nseq,
                                sizeof(int) * rows, sizeof(int) * nseq, sizeof(int) * (size_t)nseq * (K + 1),
                                sizeof(KvLayer) * (size_t)nseq * nlb};
        void** ptrs[] = {(void**)&lg, (void**)&am, (void**)&mkeys, (void**)&mall, (void**)&mtok, (void**)&mvst,
                         (void**)&mdst, (void**)&mcst, (void**)&mtarget, (void**)&mchain, (void**)&mpath,
                         (void**)&mbase, (void**)&mcat, (void**)&dkv};
        FL_BT(carve_work(e, ptrs, sizes, 14));
    }
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

