// Launch-side declarations of the sm_100a kernels (host code includes this).
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>

namespace fl {

constexpr int kMaxRows = 8;      // rows of activations per GEMV launch
constexpr int kPageSize = 64;    // KV positions per page

enum Epilogue : int {
    EPI_STORE = 0,   // out[m, n] = y
    EPI_RESID = 1,   // out[m, n] += y  (residual add)
    EPI_QKV = 2,     // RoPE on q/k pairs, q -> f32 buffer, k/v -> fp16 KV pages
    EPI_SWIGLU = 3,  // interleaved gate/up rows -> quantized SwiGLU output
    EPI_LOGITS = 4,  // out[m, n] = y and per-CTA argmax partials
    EPI_DOTS = 5,    // per-(m, n, block) int32 dots (test path)
    EPI_TP_PUSH = 6, // tensor parallelism: partial rows stored into every rank's receive slot
};

// One paged KV pool of one layer: [pages][kv_heads][kPageSize][head_dim].
struct KvLayer {
    __half* k;
    __half* v;
};

struct GemvParams {
    const uint8_t* aq;        // [rows, K] quantized activations
    const int8_t* w;          // [N, K]: row-major (P == 0) or tiled (fl_layout.cuh)
    const uint8_t* w4;        // if set: the same weights packed 4-bit (w4.cu); the TMA-ring GEMV reads these
    int P;                    // tiled-layout panel width; 0 = plain row-major
    const __half* sblk;       // [N, K/32] block scales (block mode)
    const float* srow;        // [N] per-row scales (per-row mode)
    int M;                    // rows in this launch (<= kMaxRows)
    const int* dyn_M;         // if set, rows = min(*dyn_M - row0, kMaxRows)
    int row0;                 // first activation row of this launch
    int N, K;
    const int* done;          // if set and *done, the kernel exits
    // Fused activation prologue: when x is set the kernel quantizes rows of
    // x (f32, row stride K; RMSNorm first when norm) itself instead of
    // reading aq. Source row of activation row 0: *x_row_dyn if set, else row0.
    const float* x;
    int norm;
    float eps;
    const int* x_row_dyn;
    // EPI_STORE / EPI_RESID / EPI_LOGITS
    float* out;
    int ldo;
    // EPI_QKV
    float* q_out;             // [rows, q_dim]
    KvLayer kv;
    const int* block_table;   // slot / kPageSize -> page
    const int* slot_base;     // device scalar: cache slot of activation row 0
    const int* pos;           // [rows] rotary positions
    // Batched rows (seq_rows > 0): row r belongs to sequence b = r / seq_rows
    // as its row i = r % seq_rows; its slot is b * seq_slots +
    // slot_base[b * seq_state] + i and its position pos[b * seq_state + i]
    // (seq_state = ints between the sequences' state records)
    int seq_rows, seq_state, seq_slots;
    int q_dim, kv_dim, head_dim, kv_heads;
    float theta;
    // Optional rotary table [rope_rows][head_dim / 2] of (cos, sin) of
    // position x frequency (launch_rope_table; the values the epilogue would
    // compute); rows at or past rope_rows are computed in the epilogue.
    const float2* rope;
    int rope_rows;
    // EPI_SWIGLU
    uint8_t* hq;              // [rows, F]
    int F;
    // EPI_LOGITS: partial argmax keys [rows][gridDim.x]
    unsigned long long* amax_part;
    // EPI_DOTS
    int32_t* dots;            // [rows, N, K/32]
    // EPI_TP_PUSH: output row r goes to every rank q's receive slot
    // tp_recv[q][((parity * tp_size + tp_rank) * tp_rows + r) * ldo + n]
    // (parity = *tp_seq & 1); when a CTA is done it adds 1 to every rank's
    // counter tp_cnt[q][parity * tp_size + tp_rank] (TMA GEMV only)
    float* const* tp_recv;
    unsigned long long* const* tp_cnt;
    const unsigned long long* tp_seq;
    int tp_rank, tp_size, tp_rows;
};

// Chooses the kernel variant; `rowmode` selects per-row scales and
// `pairsat` the int16 pair-saturating dot. `pdl` enables programmatic
// dependent launch.
cudaError_t launch_gemv(const GemvParams& p, int epi, bool rowmode, bool pairsat,
                        cudaStream_t s, bool pdl);
int gemv_grid(int N);

// Persistent TMA-ring variant for block-mode weights (gemv_tma.cu): one CTA
// per SM. Supported when K % 256 == 0 and the ring fits (tma_gemv_supported).
cudaError_t launch_gemv_tma(const GemvParams& p, int epi, cudaStream_t s, bool pdl);
bool tma_gemv_supported(int N, int K, int M);

// Copies `rows` host rows (int8 [rows, K], fp16 scales [rows, K/32]) into a
// device matrix of N rows at rows dst_row0 + i * dst_stride, in the tiled
// layout when P != 0 (a device relayout kernel) or row-major when P == 0.
cudaError_t upload_rows(int8_t* dst_w, __half* dst_s, int N, int K, int P, int dst_row0, int dst_stride,
                        const int8_t* host_w, const uint16_t* host_s, int rows, cudaStream_t s);
int tma_gemv_grid();
// Block-mode GEMV through the TMA kernel when the shape allows it, else the
// register-streamed kernel; gemv_auto_grid is the grid it uses for up to
// kMaxRows rows (the number of argmax partials per row for EPI_LOGITS).
cudaError_t launch_gemv_auto(const GemvParams& p, int epi, cudaStream_t s, bool pdl);
int gemv_auto_grid(int N, int K);
// Returns and clears the device error word (bounded waits that gave up).
int take_device_error();

// Tensor-parallel sum after EPI_TP_PUSH GEMVs (gemv_tma.cu): waits (bounded)
// until every rank's counter for this parity reaches ctas_per_push x
// (pushes of this parity so far + 1), then x[r] += sum over ranks q in order
// of recv[parity][q][r] for r < rows (*dyn_rows when set); the last CTA
// advances *seq. Every rank computes the same bits.
struct TpReduceParams {
    float* x;
    int rows;
    const int* dyn_rows;
    int d;
    const float* recv;                // this rank's receive slots [2][size][cap][d]
    const unsigned long long* cnt;    // this rank's counters [2][size]
    int size, cap;
    unsigned long long* seq;          // this rank's all-reduce sequence number
    unsigned long long ctas_per_push;
    int* arrived;                     // CTA arrival counter (zero at rest)
    const int* done;
};
cudaError_t launch_tp_reduce(const TpReduceParams& p, cudaStream_t s, bool pdl);

// tcgen05 INT8 GEMM for many activation rows (gemm_tc.cu): block-mode tiled
// weights (P != 0), K a multiple of 128, N of 16, activations already
// quantized in g.aq (rows 0 .. M-1, row stride K), epilogues STORE, RESID,
// QKV and SWIGLU. Same result bits as the block-mode GEMV.
bool gemm_tc_supported(const GemvParams& g, int epi);
cudaError_t launch_gemm_tc(const GemvParams& g, int epi, int M, cudaStream_t s);
int take_gemm_error();

struct ActQuantParams {
    const float* x;           // [rows, K]
    uint8_t* q;               // [rows, K]
    int K;
    int M;                    // rows (grid size)
    const int* dyn_M;         // optional device row count (<= M)
    int row0;                 // first row handled
    int norm;                 // 1 = RMSNorm (unit weights) before quantization
    float eps;
    const int* done;
    const int* dyn_src_row;   // if set: source row *dyn_src_row + blockIdx.x,
                              // written to output row row0 + blockIdx.x
};
cudaError_t launch_act_quant(const ActQuantParams& p, cudaStream_t s, bool pdl);

struct AttnParams {
    const float* q;           // [rows, heads*head_dim], rotated
    KvLayer kv;
    const int* block_table;
    const int* slot_base;     // device scalar: slot of new row 0 (= prefix length)
    int M;                    // new rows (per sequence when seqs > 1)
    const int* dyn_M;
    // Batched sequences (grid z): sequence b owns rows [b M, (b + 1) M) of q
    // and out, cache slots [b seq_slots, (b + 1) seq_slots) (seq_slots a
    // multiple of the page size) and its prefix length slot_base[b * seq_state]
    int seqs, seq_state, seq_slots;
    const uint8_t* mask;      // [M*M] visibility among new rows, NULL = causal
    int heads, kv_heads, head_dim;
    // KV head of local query head h: (q_head0 + h) / group - kv_head0; group 0
    // means heads / kv_heads with zero offsets (a tensor-parallel rank holds
    // a slice of the heads that need not align with the GQA groups)
    int q_head0, kv_head0, group;
    int max_ctx;              // upper bound of slot_base + M (smem sizing)
    uint8_t* out_q;           // [rows, heads*head_dim] quantized output
    float* out_f;             // optional f32 output
    const int* done;
    // Decode split-K scratch (M <= kMaxRows): per (sequence, head, split,
    // row) partial max / sum / unnormalised output, and one arrival counter
    // per (sequence, head) (zero between launches). Sizes per sequence from
    // attention_scratch_*.
    float* part;
    int* counters;
};
cudaError_t launch_attention(const AttnParams& p, cudaStream_t s, bool pdl);
// Fills tab[pos][i] = (cos, sin) of pos x theta^(-2i / head_dim) for pos <
// rows, i < head_dim / 2, with the epilogue's own arithmetic (decode_ops.cu).
cudaError_t launch_rope_table(float2* tab, int rows, int head_dim, float theta, cudaStream_t s);
size_t attention_scratch_floats(int heads, int head_dim, int max_ctx);
size_t attention_scratch_counters(int heads);

// Medusa (medusa_ops.cu): h = RMSNorm(x), z_i = h + SiLU(y_i) for H rows of
// y (h written when h != nullptr); per-row top-k (k[row] <= kmax <= 32)
// with softmax probabilities; in-place compaction of an accepted tree path
// (slot base + j <- slot base + src[j], j = 1 .. a) over every layer.
cudaError_t launch_medusa_z(const float* x, const float* y, float* h, float* z, int d, int H, float eps,
                            cudaStream_t s);
cudaError_t launch_topk_rows(const float* logits, int rows, int V, int ld, const int* k, int kmax, int* tok,
                             float* prob, cudaStream_t s);
// Top-w argmax keys of each row with global indices v0 + i (w <= 32).
cudaError_t launch_topk_keys(const float* logits, int rows, int V, int ld, int v0, int w, unsigned long long* out,
                             cudaStream_t s);
cudaError_t launch_kv_compact(const KvLayer* layers, int n_layers, const int* block_table, int kv_heads, int head_dim,
                              const int* base, const int* src, int a, cudaStream_t s);
// The same compaction with the path length read on the device (*a_dev, at
// most a_max).
// Packed 4-bit copy (w4.cu) of tiled INT8 block-mode weights in [-8, 7]:
// w4 gets N * K / 2 bytes; *bad (device) is set if a weight is out of range.
bool w4_supported(int N, int K, int P);
cudaError_t launch_pack_w4(const int8_t* w, uint8_t* w4, int N, int K, int P, int* bad, cudaStream_t s);

cudaError_t launch_kv_compact_dev(const KvLayer* layers, int n_layers, const int* block_table, int kv_heads,
                                  int head_dim, const int* base, const int* src, const int* a_dev, cudaStream_t s);

// Medusa candidate tree on the device (one CTA): candidates in generation
// order (head h's top-k under every depth-h candidate), score = product of
// the path's probabilities from the first head on, kept by (score desc,
// depth asc, generation asc) up to max_nodes - 1 below the root; node i's
// token, parent, depth, rotary position n + depth and its ancestor mask row.
struct MedusaTreeParams {
    const int* tok;     // [H][kmax] per-head top-k tokens
    const float* prob;  // [H][kmax] their probabilities
    const int* topk;    // [H] (device)
    int H, kmax, max_nodes, n;
    const int* root;    // [1] root token (device)
    int* ntok;          // [max_nodes]
    int* npar;
    int* ndep;
    int* pos;
    uint8_t* mask;      // [M][M], M = 1 + min(max_nodes - 1, candidates)
};
constexpr int kMaxTreeCand = 1024;
cudaError_t launch_medusa_tree(const MedusaTreeParams& p, cudaStream_t s);

// Longest path of the base model's greedy choices through a verified tree
// (node c follows node cur when npar[c] == cur and ntok[c] == target[cur],
// first such c): path[0 .. a] (node indices), rec = {a, last node, the a
// accepted tokens, the base token after them}, *root = that token, and the
// last node's feature row x[last] copied to f (d floats).
struct MedusaWalkParams {
    const int* ntok;
    const int* npar;
    const int* target;  // [M] base argmax per node
    int M;
    int* path;
    int* rec;           // [M + 2]
    int* root;
    const float* x;     // [M][d] last-layer features of the tree rows
    float* f;
    int d;
};
cudaError_t launch_medusa_walk(const MedusaWalkParams& p, cudaStream_t s);

}  // namespace fl
