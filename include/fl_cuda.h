/*
 * fl_cuda -- the thin C ABI between the C host code of the speculative-
 * decoding path and its sm_100a kernels.
 *
 * The reference calls its AVX2 kernels directly from C (inference.c:131-156
 * matvec, dequantized_tensor.c:204 matmul_dequantized). This header is the
 * replacement seam: plain pointers, sizes and int status codes, no C++ or
 * framework types. Every call is ordered on the library's CUDA stream of the
 * current device unless a stream (a cudaStream_t passed as void*) is given.
 *
 * Status: 0 on success, a negative FL_E_* code otherwise; the message of the
 * last failure on the calling thread is returned by fl_cuda_last_error().
 * No function aborts or exits the process.
 */
#ifndef FL_CUDA_H
#define FL_CUDA_H

#include <stdint.h>
#include <stddef.h>
#include "dequantized_tensor.h"
#include "medusa.h"
#include "quant_types.h"
#include "speculative.h"

#ifdef __cplusplus
extern "C" {
#endif

#define FL_OK             0
#define FL_E_INVAL       -1   /* bad argument / unsupported shape          */
#define FL_E_CUDA        -2   /* CUDA runtime or launch failure            */
#define FL_E_NOMEM       -3   /* host or device allocation failed          */
#define FL_E_UNSUPPORTED -4   /* valid request this build does not serve   */
#define FL_E_TIMEOUT     -5   /* a bounded device-side wait gave up        */
#define FL_E_NODEV       -6   /* no CUDA device                            */
#define FL_E_STATE       -7   /* call out of order (e.g. not uploaded)     */

/* ------------------------------------------------------------------ */
/* runtime                                                             */
/* ------------------------------------------------------------------ */

const char* fl_cuda_last_error(void);
int fl_cuda_init(int device);                 /* select device, create stream */
int fl_cuda_device_count(int* count);
int fl_cuda_sync(void);                       /* drain the library stream     */
void* fl_cuda_stream(void);                   /* cudaStream_t of the device   */

int fl_cuda_malloc(void** dptr, size_t bytes);
int fl_cuda_free(void* dptr);
int fl_cuda_h2d(void* dst, const void* src, size_t bytes);
int fl_cuda_d2h(void* dst, const void* src, size_t bytes);
int fl_cuda_memset(void* dptr, int value, size_t bytes);

/* ------------------------------------------------------------------ */
/* INT8 tensors and the GEMV / skinny GEMM                             */
/* ------------------------------------------------------------------ */

/* Uploads t->weights (and t->scales or t->scales_f16) to HBM once and sets
 * t->dev. Block mode needs cols % 32 == 0. Replaces the host-side use of
 * the tensor in matmul_dequantized (dequantized_tensor.c:229-243). */
int fl_cuda_upload_tensor(dequantized_tensor_t* t);

/* Activation quantization of the reference (dequantized_tensor.c:112-135),
 * optionally preceded by RMSNorm with unit weights (activations_avx2.c:
 * 108-143): q[M, K] u8 from x[M, K] f32, device pointers. */
int fl_cuda_act_quant(const float* x, uint8_t* q, int M, int K, int rmsnorm,
                      float eps, void* stream);

/* C[M, N] = A[M, K] @ B^T on device pointers: activation quantization, INT8
 * dot products and the scale epilogue of matmul_dequantized
 * (dequantized_tensor.c:204-247; block mode per dequantized_tensor.h).
 * B must be uploaded. K % 32 == 0. Any M >= 1. */
int fl_cuda_matmul_i8(const float* A, const dequantized_tensor_t* B, float* C,
                      int M, int N, int K, void* stream);

/* Same product from already-quantized activations Aq[M, K] (u8). */
int fl_cuda_gemv_i8(const uint8_t* Aq, const dequantized_tensor_t* B, float* C,
                    int M, int N, int K, void* stream);

/* Per-(m, n, block) INT32 dot products of the quantized A row and the
 * weight row over each 32-element block, D[M, N, K/32], computed by the same
 * kernel as fl_cuda_matmul_i8 with its epilogue replaced by a store of the
 * integers. Per-row-mode tensors use the pair-saturated reduction of
 * dot_product_u8_i8 (dequantized_tensor.c:149-196) inside each block. */
int fl_cuda_block_dots_i8(const float* A, const dequantized_tensor_t* B, int32_t* D,
                          int M, int N, int K, void* stream);

/* fl_cuda_block_dots_i8 through the packed 4-bit GEMV (no counterpart in
 * the reference): B must be an uploaded block-mode tensor (scale_block 32)
 * whose weights lie in [-8, 7], in the tiled layout (cols a multiple of 256).
 * The weights are packed on the device for this call; D[M, N, K/32] gets the
 * int32 block dots, which must equal fl_cuda_block_dots_i8's. M <= 8. */
int fl_cuda_block_dots_w4(const float* A, const dequantized_tensor_t* B, int32_t* D, int M, int N, int K,
                          void* stream);

/* The Medusa candidate tree of one step, built on the device by the kernel
 * fl_engine_medusa_generate uses (host buffers in and out; no counterpart in
 * the reference, whose medusa_build_tree is declared at medusa.h:126-131
 * without code). tok / prob: [H][kmax] per-head top-k tokens and
 * probabilities (the first topk[h] of row h are used); root: the root token;
 * n: the slot and rotary position of the root. Writes M = 1 + min(max_nodes -
 * 1, candidates) nodes: tok, parent (-1 for the root), depth, pos = n +
 * depth, and mask[M][M] (1 where column j is row i or one of its ancestors).
 * Candidates (sum over h of topk[0] * ... * topk[h]) must be at most 1024.
 * Returns M, or a negative FL_E_* code. */
int fl_cuda_medusa_tree(const int* tok, const float* prob, const int* topk, int H, int kmax, int max_nodes,
                        int root, int n, int* out_tok, int* out_parent, int* out_depth, int* out_pos,
                        uint8_t* out_mask);

/* Failure detection, no counterpart in the reference: runs the
 * tensor-parallel reduction kernel on the library stream against the arrival
 * counters of a two-rank group that nobody increments. Its bounded wait gives
 * up after about two seconds, records the device error word and returns; the
 * following fl_cuda_sync() returns FL_E_TIMEOUT and clears the word, and the
 * device stays usable. Returns FL_OK once the kernel has finished. */
int fl_cuda_tp_wait_timeout_check(void);

/* fl_cuda_block_dots_i8 without any allocation: no counterpart in the
 * reference. The quantized activations go to a fixed device scratch of
 * FL_NOALLOC_SCRATCH_BYTES in the library's static device memory (one per
 * device) instead of a buffer cudaMalloc'd and grown on demand; calls with
 * M * K above that size fail with FL_E_INVAL. For callers that must not
 * allocate or free device memory: cudaFree synchronises the whole device
 * and cudaMalloc can fail once a serving process has reserved the rest of
 * HBM (KV page pools sized to the free memory). `stream` may be NULL only
 * after fl_cuda_init() created the library stream of the device. The first
 * call on a device resolves the scratch address (cudaGetSymbolAddress,
 * which may load the module); make it before any stream capture. The
 * address is kept for the life of the process: after cudaDeviceReset of a
 * device the kept address is stale, so this entry point must not be used on
 * that device again. Calls that overlap in time (other streams or threads on
 * the same device) race on the one scratch; calls on one stream are
 * ordered. */
#define FL_NOALLOC_SCRATCH_BYTES (1 << 20)
int fl_cuda_block_dots_i8_noalloc(const float* A, const dequantized_tensor_t* B, int32_t* D,
                                  int M, int N, int K, void* stream);

/* ------------------------------------------------------------------ */
/* seeded synthetic weights (the loader side; host code)               */
/* ------------------------------------------------------------------ */

/* Tensor ids name a weight of the model: stack 0 base, 1 draft, 2 Medusa
 * heads, 3 shared; proj 0..6 = q, k, v, o, gate, up, down; shared proj 0 =
 * embedding, 1 = LM head. */
#define FL_TENSOR_ID(stack, layer, proj) \
    ((uint32_t)(((stack) << 24) | ((layer) << 8) | (proj)))

/* rows x cols values N(0, std) from Philox4x32-10 (key = seed, counter =
 * (element/4, tensor_id)) and Box-Muller, quantized to GGUF Q4_0 blocks
 * (ggml quantize_row_q4_0_ref rule), pre-dequantized to int8 q-8 in [-8, 7]
 * plus one fp16 scale per 32 values. cols % 32 == 0. Multithreaded and
 * deterministic. */
int fl_synth_q4_0_i8(uint64_t seed, uint32_t tensor_id, int rows, int cols,
                     float std, int8_t* w, uint16_t* d);
/* Rows [r0, r0 + nr) x columns [c0, c0 + nc) of the same [rows, cols] tensor
 * (c0, nc multiples of 32): identical to that block of fl_synth_q4_0_i8's
 * output. w [nr, nc], d [nr, nc / 32]. */
int fl_synth_q4_0_i8_block(uint64_t seed, uint32_t tensor_id, int rows, int cols, int r0, int nr, int c0, int nc,
                           float std, int8_t* w, uint16_t* d);

/* Same values as fl_synth_q4_0_i8 dequantized to f32 ((q-8)*d), the
 * form the reference loader keeps embeddings in (gguf_loader.c:147-161). */
int fl_synth_q4_0_f32(uint64_t seed, uint32_t tensor_id, int rows, int cols,
                      float std, float* out);

/* Raw N(0, std) values of a tensor (before quantization). */
int fl_synth_normal(uint64_t seed, uint32_t tensor_id, size_t count, float std,
                    float* out);

/* GGUF Q4_0 (18-byte blocks) -> int8 q-8 plus fp16 scales: the load-time
 * pre-dequantization. Nibble order of gguf_loader.c:147-161. */
int fl_q4_0_to_i8(const block_q4_0_gguf* blocks, int rows, int cols, int8_t* w,
                  uint16_t* d);

/* Philox4x32-10 block (Salmon et al. 2011), host copy of the device one. */
void fl_philox4x32_10(const uint32_t ctr[4], const uint32_t key[2], uint32_t out[4]);

/* ------------------------------------------------------------------ */
/* engine: base model + draft + Medusa heads resident in HBM           */
/* ------------------------------------------------------------------ */

typedef struct fl_engine fl_engine_t;

typedef struct {
    int vocab_size;          /* 32064 for Phi-3-mini                     */
    int hidden_size;         /* d                                        */
    int intermediate_size;   /* SwiGLU width                             */
    int num_layers;          /* base decoder layers (0: an engine holding only
                                a draft stack or Medusa heads, with the
                                embedding and LM head, for host targets) */
    int num_heads;           /* query heads                              */
    int num_kv_heads;        /* key/value heads (GQA when < num_heads)   */
    int head_dim;
    int draft_layers;        /* 0 = no draft                             */
    int medusa_heads;        /* 0 = no Medusa heads                      */
    int max_seq_len;         /* KV capacity per sequence (positions)     */
    float rope_theta;
    float norm_eps;
} fl_model_config_t;

fl_engine_t* fl_engine_create(const fl_model_config_t* cfg, int device);

/* Tensor parallelism over tp_size GPUs of one node (one process or thread per
 * rank, each on its own device). Rank r holds Q heads [r H/g, (r+1) H/g)
 * with the KV heads they read (a KV head spanning two ranks is held by both),
 * FFN features [r F/g, (r+1) F/g) and LM-head rows [r ceil(V/g), ...), plus
 * the whole embedding; Q/K/V and gate/up are column-parallel, o and down
 * row-parallel with an NCCL all-reduce of the hidden rows after each, and the
 * LM head's argmax is all-gathered. Every rank passes whole tensors to
 * fl_engine_load_linear (or calls fl_engine_synthesize) and makes the same
 * calls in the same order. nccl_id: 128 bytes from fl_tp_unique_id on one
 * rank, shared by the caller. H and F must divide by tp_size; greedy
 * decoding only. libnccl.so.2 is loaded on first use. */
fl_engine_t* fl_engine_create_tp(const fl_model_config_t* cfg, int device, int tp_rank, int tp_size,
                                 const unsigned char* nccl_id);
int fl_engine_tp(const fl_engine_t* e, int* rank, int* size);
int fl_tp_unique_id(unsigned char* id);
/* This rank's slice: out[9] = {first Q head, Q heads, first KV head, KV
 * heads, first FFN feature, features, first vocabulary row, rows, Q heads per
 * KV head}. */
int fl_tp_layout(const fl_model_config_t* cfg, int rank, int size, int* out);
/* The orderable 64-bit key of a logit v at vocabulary index `index`
 * (larger value wins, ties to the lower index: inference.c:104-111), as the
 * LM-head epilogue builds it; the tensor-parallel argmax of a row is the
 * largest key over the ranks' local best keys (global indices). */
unsigned long long fl_argmax_key(float v, int index);
/* Tensor-parallel draft-tree candidates: the `width` best tokens of one
 * depth from every rank's top-width keys (keys[r * rank_stride + c], c <
 * width, global indices), best first. Host code. */
int fl_tp_merge_topw(const unsigned long long* keys, int ranks, size_t rank_stride, int width, int* tok);
void fl_engine_destroy(fl_engine_t* e);

/* Loads one INT8 linear from host arrays: stack/layer/proj as in
 * FL_TENSOR_ID (stack 3 proj 1 = LM head; stack 2 layer h proj 0 = Medusa
 * head h). w [rows, cols] int8 in [-8, 7], d [rows, cols/32] fp16 bits. */
int fl_engine_load_linear(fl_engine_t* e, int stack, int layer, int proj,
                          const int8_t* w, const uint16_t* d, int rows, int cols);
/* Token embedding table [vocab, d] f32. */
int fl_engine_load_embedding(fl_engine_t* e, const float* table);
/* Whole-model widths of the engine's configuration: out[0] hidden, [1] q_dim
 * (heads x head_dim), [2] kv_dim, [3] ffn. */
int fl_engine_dims(const fl_engine_t* e, int* out);
/* Loads a GGUF file with Q4_0 weights (18-byte blocks, fp16 d; the nibble
 * order of gguf_loader.c:147-161): blk.<l>.* weights into stack `stack`
 * (0 base, 1 draft), output.weight as the LM head, token_embd as the
 * embedding (Q4_0, F16 or F32). Each Q4_0 tensor is pre-dequantized once to
 * INT8 q-8 plus its fp16 block scales and uploaded. Names as the reference
 * loader (gguf_loader.c:307-342), fused attn_qkv and Phi-3's gate+up ffn_up
 * split; norm weights are not applied (unit RMSNorm weights). */
int fl_engine_load_gguf(fl_engine_t* e, int stack, const char* path);
/* Weight format read by the engine's GEMV passes (up to 16 rows: the decode
 * chain, its draft passes and the LM head), no counterpart in the reference.
 * bits = 4: every loaded block-mode tensor is packed once more, on the
 * device, two weights per byte (its values are Q4_0 nibbles minus 8, so the
 * packing is lossless) and those passes stream the packed copy: about half
 * the weight bytes per decode step; every int32 block dot is the same as
 * with INT8 weights (the 4-bit dot is taken over q = w + 8 and 8 x the
 * block's activation sum is subtracted). Passes of more than 16 rows (the
 * tcgen05 GEMM) keep reading the INT8 copy. bits = 8 frees the packed copy.
 * Needs every tensor loaded; drops the captured step and batch graphs (the
 * next prefill records them again). FL_E_INVAL if a weight lies outside
 * [-8, 7]. */
int fl_engine_set_weight_bits(fl_engine_t* e, int bits);
/* Generates and loads every tensor with fl_synth_* (std 0.02). */
int fl_engine_synthesize(fl_engine_t* e, uint64_t seed);
/* 1 when every tensor the configuration needs has been loaded. */
int fl_engine_ready(const fl_engine_t* e);

/* Runs M rows through a stack (0 base, 1 draft) at cache slots
 * [base, base+M) with rotary positions pos[M] and visibility mask[M*M]
 * (NULL = causal) over the new rows; slots [0, base) are visible to all.
 * Host buffers: x_in/x_out [M, d]; logits [M, vocab] (NULL to skip). */
int fl_engine_forward_rows(fl_engine_t* e, int stack, const float* x_in, int M,
                           int base, const int* pos, const uint8_t* mask,
                           float* x_out, float* logits);

/* Greedy base-model decoding: prefill the prompt, emit n_new tokens. */
int fl_engine_greedy_generate(fl_engine_t* e, const int* prompt, int prompt_len,
                              int n_new, int* out);

/* Greedy chain speculative decoding (include/speculative.h rule), k drafted
 * tokens per step. out[n_new] tokens; acc_hist[steps] accepted counts (may
 * be NULL; size >= n_new); *steps the number of steps (may be NULL). */
int fl_engine_spec_generate(fl_engine_t* e, const int* prompt, int prompt_len,
                            int n_new, int k, int max_accepted, int* out,
                            int* acc_hist, int* steps);

/* Independent sequences on one engine (one rank's share of a batch): for each
 * i < nseq, prompts[i * prompt_len ..] is decoded for n_new tokens with draft
 * length k into out[i * n_new ..], under the rule of fl_engine_set_sampling
 * with sequence id seq_ids[i] (i when seq_ids is NULL). The sequences are
 * decoded together in in-GPU batches (fl_engine_batch_*) as large as the
 * engine's rows (max_seq_len / (k + 1)) and 80 % of free device memory allow;
 * a larger existing reservation is reused. Every decision of a sequence
 * follows the rule with its own Philox key, whatever else shares its batch;
 * batches of different sizes may run other kernels (GEMV chunks or the
 * tcgen05 GEMM), whose logits differ in the last bits. steps[i] (may be
 * NULL) receives the speculative steps of sequence i. Returns the total
 * number of steps or a negative FL_E_* code; fl_engine_last_timing's
 * total_us is the device time of the whole call, prefills included, and
 * verify_us the decode loops alone. */
int fl_engine_spec_generate_batch(fl_engine_t* e, const int* prompts, int prompt_len, int nseq,
                                  const unsigned* seq_ids, int n_new, int k, int* out, int* steps);

/* In-GPU batch of independent sequences (one GPU; not tensor-parallel).
 * Each sequence has its own KV region of max_ctx positions (rounded up to a
 * page), state, tokens and Philox key; a step runs the k - 1 draft passes
 * over one row per sequence, one verify pass over nseq x (k + 1) rows, the
 * acceptance of every sequence, and the draft catch-up over nseq x (k + 1)
 * rows (rows past a sequence's accepted ones are zero and unused), all in
 * one CUDA graph. Passes of more than 16 rows run through the tcgen05 GEMM.
 *
 * reserve: allocates the regions and buffers for nseq sequences (frees a
 * previous reservation). capacity: the reserved sequences and slots.
 * prefill: prefills prompts[i * prompt_len ..] of sequence i < nseq
 * (nseq <= reserved, nseq * (k + 1) <= max_seq_len) under the current
 * rule with ids seq_ids (NULL: 0..nseq-1), draws every first token and the
 * first draft, and records the step graph. begin: restores the
 * post-prefill state for a decode of n_new tokens. decode: begin, then
 * steps until every sequence has n_new tokens; out[i * n_new ..], steps[i];
 * returns the total steps. step: one step after begin; state[5 i ..] =
 * (n, produced, steps, accepted, done) of sequence i. trace: the
 * fl_engine_sample_trace arrays of sequence seq (sampled prefill with the
 * trace enabled). */
int fl_engine_batch_reserve(fl_engine_t* e, int nseq, int max_ctx);
int fl_engine_batch_capacity(const fl_engine_t* e, int* nseq, int* slots);
int fl_engine_batch_prefill(fl_engine_t* e, const int* prompts, int prompt_len, int nseq,
                            const unsigned* seq_ids, int k);
int fl_engine_batch_begin(fl_engine_t* e, int n_new);
int fl_engine_batch_decode(fl_engine_t* e, int n_new, int* out, int* steps);
int fl_engine_batch_step(fl_engine_t* e, int* state);
int fl_engine_batch_trace(const fl_engine_t* e, int seq, float* logits, unsigned* qd, unsigned long long* qm,
                          unsigned* pt, unsigned long long* pm, int* drafted);

/* Decoding rule of the next fl_engine_spec_prefill / spec_generate.
 * temperature <= 0: greedy (argmax drafts, exact-match acceptance; the
 * default). temperature > 0: stochastic speculative decoding
 * (speculative.h:121-185 speculative_config_t.temperature): drafts are drawn
 * from the top-p nucleus q of softmax(l / temperature), each accepted with
 * probability min(1, p(x) / q(x)) against the target's nucleus p, the first
 * rejection resampled from max(0, p - q) (p when that is empty) and, when all
 * are accepted, a bonus token drawn from the last target row. Uniforms come
 * from Philox4x32-10 keyed by (seed, 0) at counter (seq_id, step, position,
 * purpose); the stream is a pure function of (weights, prompt, k,
 * temperature, top_p, seed, seq_id). top_p in (0, 1]. Distributions are
 * integer weights trunc(e^((l - max) / T) * 2^24) with exact sums, so the
 * draws do not depend on any reduction order (speculative.h states the rule). */
int fl_engine_set_sampling(fl_engine_t* e, float temperature, float top_p, unsigned seed,
                           unsigned seq_id);
/* The rule set last: temperature 0 for greedy; top_p 1, seed 0 and seq_id 0
 * until set. speculative_generate with config->temperature > 0 keeps this
 * top_p, seed and seq_id. */
int fl_engine_get_sampling(const fl_engine_t* e, float* temperature, float* top_p, unsigned* seed,
                           unsigned* seq_id);

/* Sampling trace, for checking the sampling rule against the oracle: when on
 * (before the next fl_engine_spec_prefill), the step records the logits
 * behind every draw. fl_engine_sample_trace copies (any may be NULL):
 * logits [2 * 8, V] (draft j at row j, verify row r at row 7 + r, the first
 * token after the prefill at row 15), the integer nucleus weights of the
 * drafts qd [7, V] with their kept masses qm [7], those of the verify rows
 * pt [8, V] with pm [8], and the drafted tokens [7]. Row 0 of qd / logits,
 * qm[0] and drafted[0] already belong to the next step once a step ends. */
int fl_engine_sample_trace_enable(fl_engine_t* e, int on);
int fl_engine_sample_trace(const fl_engine_t* e, float* logits, unsigned* qd, unsigned long long* qm,
                           unsigned* pt, unsigned long long* pm, int* drafted);

/* Step-wise decoding: fl_engine_spec_begin restores the post-prefill state
 * for n_new tokens (as fl_engine_spec_decode does); each fl_engine_spec_step
 * runs one speculative step and returns state[5] = {n (sequence length),
 * produced, steps, accepted drafts of this step, done}. */
int fl_engine_spec_begin(fl_engine_t* e, int n_new);
int fl_engine_spec_step(fl_engine_t* e, int* state);

/* Split form for timing: prefill once, then decode from the saved
 * post-prefill state as often as wanted (each decode restarts there). */
int fl_engine_spec_prefill(fl_engine_t* e, const int* prompt, int prompt_len, int k,
                           int max_accepted);
int fl_engine_spec_decode(fl_engine_t* e, int n_new, int* out, int* acc_hist,
                          int* steps);
/* Per-stage device times of the last fl_engine_spec_decode (microseconds,
 * summed over its steps): draft passes, verify passes, total. */
int fl_engine_last_timing(const fl_engine_t* e, double* draft_us, double* verify_us,
                          double* total_us);
/* cudaStream_t (as void*) the engine launches on. */
void* fl_engine_stream(const fl_engine_t* e);
/* Number of kernels the last fl_engine_spec_decode launched. */
long long fl_engine_last_launches(const fl_engine_t* e);
/* 1 when speculative steps run as one persistent kernel per step (all
 * weights in the tiled layout), 0 when they run as one kernel per op. */
int fl_engine_step_kernel(const fl_engine_t* e);
/* Phase trace of the last step-kernel launch, recorded only when the
 * environment has FL_STEP_TRACE=1 when the step graph is built. For each of
 * the first min(cap, phases) phases: t[6i] start on CTA 0, t[6i+1] end of
 * CTA 0's work, t[6i+2] latest end over all CTAs (%globaltimer ns; the last
 * phase has no end stamps), for GEMV phases on CTA 0 t[6i+3] activation
 * prologue done, t[6i+4] ns spent waiting for weight stages, t[6i+5] first
 * stage ready; and desc[4i..4i+3] = kind (0 GEMV, 1 attention,
 * 2 draft pick, 3 verify prep, 4 accept, 5 catch-up prep), epilogue (GEMV)
 * or argument, N, K. Returns the phase count written, 0 when not tracing. */
int fl_engine_step_trace(const fl_engine_t* e, unsigned long long* t, int* desc, int cap);
/* Stage trace of the phase named by FL_STEP_TRACE_PHASE (with FL_STEP_TRACE=1)
 * in the last launch, CTA 0: t[8s..8s+5] = warp 0 stage s ready, warp 0
 * done, last consumer warp ready, done, producer starts waiting for the
 * slot, producer issues the copy (%globaltimer ns), 64 stages; 512 words.
 * Returns 64, or 0 when not tracing. */
int fl_engine_step_trace_stages(const fl_engine_t* e, unsigned long long* t);

/* Medusa greedy decoding on the device (include/medusa.h rule): prefill P
 * prompt ids, then steps of: heads (residual block + shared LM head) on the
 * last hidden state, per-head top-k (topk[h] <= 32 for h < H <= 8 heads),
 * candidate tree of at most max_nodes nodes (<= 256), one tree-masked base
 * pass, longest accepted path, KV compaction. Writes n_new tokens (the first
 * from the prefill) and the accepted count of each step. The engine needs
 * H <= medusa_heads loaded heads and P + n_new + max_nodes + 2 <= max_seq_len. */
int fl_engine_medusa_generate(fl_engine_t* e, const int* prompt, int P, int n_new, const int* topk, int H,
                              int max_nodes, int* out, int* acc_hist, int* steps);

/* Draft + Medusa (speculative_medusa_generate): each step the draft drafts a
 * chain of k tokens and the Medusa heads propose per-depth top-k candidates;
 * the chain (always kept) and the heads' tree (merged, then added in score
 * order up to max_nodes nodes) are verified in one tree-masked base pass;
 * the longest path of the base model's greedy choices is accepted, its base
 * KV compacted, and the draft catches up over the accepted positions from
 * the base features of the path's tree rows. The output is the base model's
 * greedy stream. Needs a draft stack and Medusa heads. */
int fl_engine_spec_medusa_generate(fl_engine_t* e, const int* prompt, int prompt_len, int n_new, int k,
                                   const int* topk, int n_heads, int max_nodes, int* out, int* acc_hist,
                                   int* steps);

/* Static draft tree (EAGLE-style), greedy: each step the draft drafts a
 * chain of k tokens and, at every depth j, its next width - 1 candidates
 * after the chain token (children of the chain token of depth j - 1); the
 * 1 + k * width nodes are verified in one tree-masked base pass (passes of
 * more than 16 rows through the tcgen05 GEMM), the longest path of the base
 * model's greedy choices is accepted, its base KV compacted and the draft
 * catches up over it. On a tensor-parallel engine every rank's top-width
 * candidates (value, global index) are gathered and merged, so all ranks
 * build the same tree; the output is the base model's greedy stream.
 * Needs 1 + k * width <= 256 and prompt_len + n_new + 1 + k * width + k + 2
 * <= max_seq_len. out[n_new]; acc_hist[steps] accepted per step (may be
 * NULL); *steps (may be NULL). */
int fl_engine_spec_tree_generate(fl_engine_t* e, const int* prompt, int prompt_len, int n_new, int k, int width,
                                 int* out, int* acc_hist, int* steps);

/* The static draft tree for an in-GPU batch (greedy): nseq sequences
 * (prompts[i * prompt_len ..]) each get the tree of fl_engine_spec_tree_generate
 * every step; the draft chains run as batched single-row passes, the trees of
 * all sequences are verified in one tree-masked pass of nseq * (1 + k * width)
 * rows over their own KV regions, and the draft catch-up is batched too. On
 * one GPU or tensor-parallel. Needs fl_engine_batch_reserve(e, >= nseq,
 * >= prompt_len + n_new + 1 + k * width + k + 3) first (on every rank) and
 * nseq * (1 + k * width) <= max_seq_len. out[i * n_new ..]; steps[i] (may be
 * NULL). Returns the total steps or a negative FL_E_* code. */
int fl_engine_batch_tree_generate(fl_engine_t* e, const int* prompts, int prompt_len, int nseq, int n_new, int k,
                                  int width, int* out, int* steps);

/* Step-level Medusa pieces (medusa_predict / medusa_build_tree /
 * medusa_verify_tree / medusa_decode_step run on these).
 * fl_engine_medusa_tree: the heads' candidate tree from a base feature F
 * (host [d]); root >= 0 is the root token, root < 0 takes the LM head's
 * argmax of F; writes at most max_nodes nodes (tok, parent (-1 for the root),
 * depth, score = product of the softmax probabilities; score may be NULL) and
 * returns the node count.
 * fl_engine_tree_verify: feeds the tree at the callback position (node i at
 * slot pos + i, rotary position pos + depth[i], attending to its ancestors),
 * accepts the longest path of the base model's greedy choices, moves its KV
 * to slots pos + 1 .. pos + a, advances the position by a + 1 and makes the
 * last accepted node's feature the last feature; out_tokens gets the a
 * accepted tokens then the base model's next token. Parents must precede
 * their children. */
int fl_engine_medusa_tree(fl_engine_t* e, const float* F, int root, const int* topk, int n_heads, int max_nodes,
                          int* tok, int* parent, int* depth, float* score);
int fl_engine_tree_verify(fl_engine_t* e, const int* tok, const int* parent, const int* depth, int n_nodes,
                          int* out_tokens, int* accepted);
/* Loads a medusa_model_t's heads (medusa_model: a medusa_model_t*) into the
 * engine, as medusa_generate does on its first call, so that medusa_predict /
 * medusa_build_tree find the engine. */
int fl_engine_bind_medusa(fl_engine_t* e, void* medusa_model);
/* 1 when `draft` (a draft_model_t*) is the draft whose weights the engine
 * holds; fl_engine_note_draft records it after a load. */
int fl_engine_draft_bound(const fl_engine_t* e, const void* draft);
void fl_engine_note_draft(fl_engine_t* e, const void* draft);
/* Device time per launch of one projection kind (0 qkv, 1 o, 2 gate/up,
 * 3 down) over all layers of a stack at M rows, captured back to back and
 * replayed reps times, and the algorithmic bytes of one launch. */
int fl_engine_bench_linear(fl_engine_t* e, int stack, int kind, int M, int reps,
                           double* us_per_launch, double* bytes_per_launch);
/* Device time per launch of the decode attention of every layer of a stack:
 * M new rows over a context of ctx slots (the cache's current contents),
 * captured back to back and replayed reps times. */
int fl_engine_bench_attention(fl_engine_t* e, int stack, int M, int ctx, int reps, double* us_per_launch);

/* Host-target support (no counterpart in the reference): passes for an
 * engine created with num_layers = 0, which holds only a draft stack or
 * Medusa heads with the embedding and LM head, for callers whose target or
 * base model is their own host function.
 * fl_engine_draft_lm: the draft as a plain language model over token
 * embeddings (input at position i is E[t_i]): the nrows tokens rows_tok at
 * positions pos0 .. pos0 + nrows - 1 (not yet in the draft cache) in one
 * pass, drafts[0] = the last row's LM-head argmax, then each draft token fed
 * back at the next position; K tokens in drafts. The draft cache then holds
 * the positions below pos0 + nrows + K - 1.
 * fl_engine_lm_argmax / fl_engine_lm_logits: the LM head (final RMSNorm
 * included) over one host feature row F [hidden]: its argmax (ties to the
 * lowest index) or its logits [vocab] on the host. */
int fl_engine_draft_lm(fl_engine_t* e, const int* rows_tok, int nrows, int pos0, int K, int* drafts);
int fl_engine_lm_argmax(fl_engine_t* e, const float* F, int* tok);
int fl_engine_lm_logits(fl_engine_t* e, const float* F, float* logits);

/* Callback-level position of the base cache: tokens appended through
 * fl_cuda_target_forward / fl_cuda_base_forward land at this position.
 * Setting it lower discards (rolls back) the later cache entries. */
int fl_engine_position(const fl_engine_t* e);
int fl_engine_set_position(fl_engine_t* e, int pos);
/* Base feature F (last-layer output before the final norm) of the last
 * token appended through the callbacks, [hidden_size] host floats. */
int fl_engine_last_feature(const fl_engine_t* e, float* out);

/* Single-row greedy draft chain: input hidden + E[tok] at draft position
 * pos, K tokens out, each with its draft softmax probability. */
int fl_engine_draft_chain(fl_engine_t* e, const float* hidden, int tok, int pos, int K,
                          int* out_tokens, float* out_probs);

/* Loads a draft_model_t's host tensors (block mode) into the engine's draft
 * stack and binds it, so draft_tokens can run it. */
int fl_engine_bind_draft(fl_engine_t* e, draft_model_t* draft);

/* Vocabulary of the logits rows verify_tokens reads for this tree. */
int fl_draft_tree_set_vocab(draft_tree_t* tree, int vocab);

/* Callback of the reference's target_forward type (speculative.h:153)
 * served by an fl_engine_t: input = len token ids as floats appended at the
 * engine's next positions, output = logits [len, vocab]. */
void fl_cuda_target_forward(void* model, const float* input, float* output, int len);

/* Callback of the reference's base_forward type (medusa.h:143): tokens[len]
 * appended, hidden = base feature F of the last token [hidden_size]. */
void fl_cuda_base_forward(void* model, const int* tokens, int len, float* hidden,
                          int hidden_size);

#ifdef __cplusplus
}
#endif

#endif /* FL_CUDA_H */
