// Private to the engine sources (engine.cu, engine_batch.cu): the device
// engine's state and the layer-pass helpers both files use.
#pragma once

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

namespace fl_eng {

struct Linear {
    int8_t* w = nullptr;
    __half* s = nullptr;
    uint8_t* w4 = nullptr;  // packed 4-bit copy (w4.cu) read by the GEMV when the engine runs 4-bit weights
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


}  // namespace fl_eng

using namespace fl_eng;

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
    // per-call work buffers of the Medusa and draft-tree loops, carved from
    // one arena kept across calls (grown when a call needs more, freed with
    // the engine; carve_work)
    uint8_t* work_arena = nullptr;
    size_t work_arena_cap = 0;
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
    float2* rope = nullptr;       // rotary (cos, sin) table [rope_rows][hd / 2]
    int rope_rows = 0;
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

namespace fl_eng {

int check_ready(fl_engine* e, bool need_draft);
// Points ptrs[i] at sizes[i] bytes (256-byte aligned) of the engine's work
// arena, growing it after a stream synchronisation when the call needs more.
// One user at a time: the buffers stay valid until the next carve_work.
int carve_work(fl_engine* e, void** const* ptrs, const size_t* sizes, int n);
// Runs M rows through a stack (the layer chain of engine.cu); view: the KV
// regions of an in-GPU batch, or of one sequence of it.
int run_stack(fl_engine* e, Stack& S, float* x, int M, const int* dyn_M, const int* slot_base, const int* pos,
              const uint8_t* mask, const int* done, bool pdl, const KvView* view = nullptr);
// LM head over rows of x; with logits / amax given, any number of rows into them.
int run_lm(fl_engine* e, const float* x, int M, const int* dyn_src_row, const int* done, bool pdl,
           float* logits = nullptr, unsigned long long* amax = nullptr);
int ensure_mask(fl_engine* e, int M);
const unsigned long long* amax_keys(const fl_engine* e);
int amax_nparts(const fl_engine* e);
int prefill_base(fl_engine* e, const int* prompt, int P);
void batch_free(fl_engine* e);

}  // namespace fl_eng
