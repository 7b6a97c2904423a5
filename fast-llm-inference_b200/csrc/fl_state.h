// Device-resident state of one speculative decode and the kernels that
// advance it between the draft and verify passes.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "fl_kernels.h"

namespace fl {

constexpr int kMaxDraft = kMaxRows - 1;  // K <= 7 so that K + 1 rows fit a launch

// Lives in HBM; every step kernel reads positions from here so one captured
// step graph replays unchanged. Index convention: seq[n] is the newest
// committed token, not yet in the base KV cache (base holds slots [0, n)).
struct SpecState {
    int n;                  // newest committed token index
    int produced;           // tokens emitted so far
    int n_new;              // tokens requested
    int done;               // 1 once produced >= n_new: later kernels exit
    int steps;
    int K;                  // drafted tokens per step
    int max_acc;            // cap on accepted drafts
    int one;                // constant 1 (row count of single-row passes)
    int rows;               // rows of the current draft catch-up pass
    int last_row;           // rows - 1
    int draft_base;         // cache slot of row 0 of the current draft pass
    int verify_base;        // cache slot of verify row 0 (= n)
    int a_last;             // drafts accepted by the last verify
    int draft_pos[kMaxRows];
    int verify_pos[kMaxRows];
    int drafted[kMaxRows];  // draft tokens d_1..d_K of the current step
    int target[kMaxRows];   // base-model argmax of the verify rows
};

// Shared state of an in-GPU batch: sequences still decoding, and the flag
// every kernel of a batched step tests (set once all sequences are done).
struct BatchCtl {
    int active;
    int done;
};

struct StepBuffers {
    SpecState* st;
    int* seq;               // committed tokens
    int* out;               // emitted tokens [n_new]
    int* acc_hist;          // accepted drafts per step
    const float* embed;     // [vocab, d]
    float* x_d;             // draft rows [kMaxRows, d]
    float* x_v;             // verify rows [kMaxRows, d]
    const unsigned long long* amax_part;  // [rows][nparts]
    int nparts;             // partials per row (LM-head GEMV grid)
    int d;
    // stochastic mode (temp > 0): LM-head logits rows, integer nucleus
    // weights of the draft / target rows and their kept masses, Philox key
    const float* logits;    // [kMaxRows, V]
    int V;
    float temp, top_p;
    const uint32_t* key;    // device [2]: Philox seed, sequence id (set without re-recording)
    uint32_t* qd;           // [kMaxDraft, V] draft weights
    unsigned long long* qm; // [kMaxDraft]
    uint32_t* pt;           // [kMaxRows, V] target weights
    unsigned long long* pm; // [kMaxRows]
    unsigned long long* resid;  // [V] residual weights of a rejection
    // optional trace (null unless enabled): logits rows behind each draw,
    // [2 * kMaxRows, V]: draft j at row j, verify row r at kMaxDraft + r,
    // the first token after the prefill at 2 * kMaxRows - 1
    float* trace;
    // In-GPU batch of `batch` sequences (0: one sequence): the buffers above
    // hold every sequence, and the control kernels take sequence s's slice
    // (seq_view). Verify and
    // catch-up rows (x_v, x_d, logits, amax_part) are rows_per per sequence;
    // the single-row draft passes use x_d1 [sequences, d] and the LM-head
    // rows s of logits_d / amax_d.
    int batch;
    int rows_per;
    int seq_cap;            // ints per sequence in seq / out / acc_hist
    float* x_d1;
    const float* logits_d;
    const unsigned long long* amax_d;
    BatchCtl* ctl;
};

#ifdef __CUDACC__
// Sequence s's view of a batched step's buffers (unchanged for one sequence).
__device__ __forceinline__ StepBuffers seq_view(const StepBuffers& b0, int s) {
    StepBuffers b = b0;
    if (!b0.batch) {
        b.x_d1 = b0.x_d;
        b.logits_d = b0.logits;
        b.amax_d = b0.amax_part;
        return b;
    }
    const size_t rows = (size_t)s * b0.rows_per;
    b.st = b0.st + s;
    b.seq = b0.seq + (size_t)s * b0.seq_cap;
    b.out = b0.out + (size_t)s * b0.seq_cap;
    b.acc_hist = b0.acc_hist + (size_t)s * b0.seq_cap;
    b.x_d = b0.x_d + rows * b0.d;
    b.x_v = b0.x_v + rows * b0.d;
    b.x_d1 = b0.x_d1 + (size_t)s * b0.d;
    b.amax_part = b0.amax_part + rows * b0.nparts;
    b.amax_d = b0.amax_d + (size_t)s * b0.nparts;
    b.logits = b0.logits + rows * b0.V;
    b.logits_d = b0.logits_d + (size_t)s * b0.V;
    b.key = b0.key + 2 * s;
    if (b0.qd) {
        b.qd = b0.qd + (size_t)s * kMaxDraft * b0.V;
        b.qm = b0.qm + (size_t)s * (kMaxDraft + kMaxRows);
        b.pt = b0.pt + (size_t)s * kMaxRows * b0.V;
        b.pm = b0.pm + (size_t)s * (kMaxDraft + kMaxRows);
        b.resid = b0.resid + (size_t)s * b0.V;
    }
    if (b0.trace) b.trace = b0.trace + (size_t)s * 2 * kMaxRows * b0.V;
    return b;
}

// Called once by the acceptance of a sequence that has just finished: the
// last sequence of a batch to finish raises the batch's done flag.
__device__ __forceinline__ void batch_retire(const StepBuffers& b, int finished) {
    if (b.batch && finished && atomicSub(&b.ctl->active, 1) == 1) atomicExch(&b.ctl->done, 1);
}
#endif

// x[r] = E[tok[r]] + (r >= shift ? feat[r - shift] : 0) for r < rows,
// rows = dyn_rows ? *dyn_rows : rows_static; ids outside [0, vocab) read row 0.
cudaError_t launch_embed_rows(const float* embed, int vocab, const int* tok, const float* feat, int shift,
                              float* x, int d, int rows_static, const int* dyn_rows,
                              const int* done, cudaStream_t s, bool pdl);

// Greedy pick of draft token j from the LM-head partials of row 0; writes
// drafted[j] and, when j + 1 < K, the next single-row draft input
// x_d[0] = g + E[drafted[j]] with g = x_d[g_row] (g_row = last_row when
// j == 0, else 0) at slot/position n + j + 1. Batched: one CTA per sequence,
// draft row s of the LM head, g = x_d1[s] (the catch-up's last feature is
// gathered there first, launch_gather_last).
cudaError_t launch_draft_pick(const StepBuffers& b, int j, cudaStream_t s, bool pdl);

// Verify rows: x_v[r] = E[tok_r], tok_0 = seq[n], tok_r = drafted[r - 1],
// positions n + r.
cudaError_t launch_verify_prep(const StepBuffers& b, int K, cudaStream_t s, bool pdl);

// Base argmax per verify row, longest accepted prefix, commit tokens,
// advance the state (include/speculative.h rule).
cudaError_t launch_accept(const StepBuffers& b, int K, cudaStream_t s, bool pdl);

// Next draft catch-up rows: x_d[r] = x_v[r] + E[seq[n_old + 1 + r]] for
// r <= a_last, positions n_old + 1 + r.
cudaError_t launch_catchup_prep(const StepBuffers& b, int K, cudaStream_t s, bool pdl);

// out_tok[r] = argmax over the LM partials of row r, r < rows.
// Stochastic mode (sample_ops.cu): first token after the prefill from logits
// row 0; sampled draft pick j; nucleus distributions of the K + 1 verify rows;
// rejection-sampling acceptance with the same state update as launch_accept.
cudaError_t launch_sample_first(const StepBuffers& b, int P, cudaStream_t s, int seq = 0);
cudaError_t launch_sample_pick(const StepBuffers& b, int j, cudaStream_t s, bool pdl);
cudaError_t launch_target_dist(const StepBuffers& b, int K, cudaStream_t s, bool pdl);
cudaError_t launch_accept_sampled(const StepBuffers& b, int K, cudaStream_t s, bool pdl);

// Tensor parallelism (decode_ops.cu): per-row best key of this rank's LM-head
// partials with global indices; per-row maximum of the gathered keys
// [size][stride].
cudaError_t launch_tp_local_best(const unsigned long long* part, int nparts, int rows, int v0, unsigned long long* out,
                                 cudaStream_t s);
cudaError_t launch_tp_reduce_best(const unsigned long long* all, int size, int stride, int rows,
                                  unsigned long long* out, cudaStream_t s);

// Sequences of a step: launches take one CTA (or one row of CTAs) each.
inline int step_seqs(const StepBuffers& b) { return b.batch > 0 ? b.batch : 1; }

// Batched: x_d1[s] = x_d[s * rows_per + last_row_s] (the draft catch-up's
// feature of each sequence's newest token).
cudaError_t launch_gather_last(const StepBuffers& b, cudaStream_t s, bool pdl);

cudaError_t launch_argmax_rows(const unsigned long long* part, int nparts, int rows, int* out_tok,
                               float* out_val, cudaStream_t s);

}  // namespace fl
