/*
 * CPU oracle for the speculative-decoding hot path.
 *
 * TEST INFRASTRUCTURE ONLY. This is the checker: tests/, the smoke() entry and
 * the CPU-baseline leg of bench.py call it to produce expected results and
 * CPU timings. Nothing in the product library links or calls it.
 *
 * Every function restates the reference's arithmetic in plain C. Citations
 * are file:line inside the reference project (fast_llm/...). Where the
 * reference has no implementation (draft / verify / accept / Medusa / KV
 * compaction are declared in speculative.h and medusa.h but never defined)
 * the rule implemented here is this project's specification, shared with the
 * GPU path; the header comments of include/speculative.h and include/medusa.h
 * state it.
 *
 * Pinning: the integer and FP primitives are checked against the
 * reference's own functions compiled from its sources into oracle/_ref
 * (tests/test_oracle_pin.py) and against committed golden vectors
 * (tests/golden/). The layer composition is checked against the reference's
 * model_forward in its f32-weight mode.
 */
#ifndef FL_ORACLE_H
#define FL_ORACLE_H

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------- primitives ---------------- */

/* dequantized_tensor.c:112-135: u8 = sat_u8(sat_i16(cvtps(fma(x,127,128)))),
 * cvtps rounding to nearest-even, out-of-range and NaN -> INT32_MIN. */
void orc_quant_u8(const float* x, uint8_t* q, int n);

/* dequantized_tensor.c:149-180: sum over pairs j of sat_i16(a[2j]*w[2j] +
 * a[2j+1]*w[2j+1]); n % 32 == 0. */
int32_t orc_dot_pairsat(const uint8_t* a, const int8_t* w, int n);

/* Plain int32 dot (equal to the pair-saturated one when max|w| <= 64). */
int32_t orc_dot_plain(const uint8_t* a, const int8_t* w, int n);

/* Per-row mode, dequantized_tensor.c:204-247:
 * C[m,n] = ((float)dot(m,n) * scales[n]) * (1.0f / 2032.0f). */
void orc_matmul_rowscale(const float* A, const int8_t* W, const float* scales,
                         float* C, int M, int N, int K);

/* Block mode (weights [-8,7], fp16 scale per 32-block):
 * C[m,n] = (sum_b (float)dot_b * d_b, summed in block order) / 127.0f. */
/* Packs [N, K] block-mode weights (all in [-8, 7], N % 8 == 0) and their
 * fp16 scales for orc_matmul_packed: wp N*K bytes, sp N*K/32 floats.
 * Returns -1 (nothing written past the check) when a condition fails. */
int orc_pack_rows8(const int8_t* W, const uint16_t* S, int N, int K, int8_t* wp, float* sp);
/* orc_matmul_block on packed weights; identical results. */
void orc_matmul_packed(const float* A, const int8_t* wp, const float* sp, float* C, int M, int N, int K);
void orc_matmul_block(const float* A, const int8_t* W, const uint16_t* scales,
                      float* C, int M, int N, int K);

/* Per-(m, n, b) int32 block dots, [M, N, K/32]. */
void orc_block_dots(const float* A, const int8_t* W, int32_t* D, int M, int N, int K);

/* activations_avx2.c:108-143: 8-lane FMA sum of squares, lanes reduced
 * ((0+4)+(2+6))+((1+5)+(3+7)), scale = 1/sqrtf(sum/n + eps),
 * out = x * scale. */
void orc_rmsnorm(const float* x, float* out, int n, float eps);

/* activations_avx2.c:33-63 polynomial sigmoid. */
float orc_fast_sigmoid(float x);
/* activations_avx2.c:86-105 (vector path): g * sigma~(g) * u. */
void orc_swiglu(const float* g, const float* u, float* out, int n);
/* activations_avx2.c:66-83 (vector path): x * sigma~(x). */
void orc_silu(const float* x, float* out, int n);

/* inference.c:159-190 adjacent-pair rotation, freq = 1/powf(theta, i/hd),
 * applied to one vector of `heads` heads at absolute position pos. */
void orc_rope_vec(float* v, int heads, int head_dim, int pos, float theta);

/* fp16 <-> f32 (IEEE binary16, round to nearest even on narrowing). */
float orc_f16_to_f32(uint16_t h);
uint16_t orc_f32_to_f16(float f);

/* ggml Q4_0 quantizer (published llama.cpp ggml-quants.c
 * quantize_row_q4_0_ref): d = max/-8 with max the signed value of largest
 * magnitude, id = 1/d, q = min(15, (int8)(x*id + 8.5)), fp16 d; nibble order of
 * gguf_loader.c:147-161 (element i low nibble of byte i, i+16 high).
 * Writes int8 q-8 and fp16 d per block directly. */
void orc_q4_0_quantize_i8(const float* x, int n, int8_t* w, uint16_t* d);

/* Philox4x32-10 (Salmon et al., SC'11). */
void orc_philox4x32_10(const uint32_t ctr[4], const uint32_t key[2], uint32_t out[4]);

/* The library's seeded synthetic weights (fl_synth_q4_0_i8 / _f32 of
 * include/fl_cuda.h), restated so that CPU-only runs need no product code:
 * N(0, std) from Philox4x32-10 (key = seed, counter = (element / 4, tensor
 * id, 0x5EED)) and Box-Muller in double precision, quantized to Q4_0 blocks
 * (orc_q4_0_quantize_i8), int8 q-8 plus fp16 scales; _f32 dequantizes. */
int orc_synth_q4_0_i8(uint64_t seed, uint32_t tensor_id, int rows, int cols, float std, int8_t* w, uint16_t* d);
int orc_synth_q4_0_f32(uint64_t seed, uint32_t tensor_id, int rows, int cols, float std, float* out);

/* ---------------- model ---------------- */

typedef struct {
    int vocab, d, ffn, layers, heads, kv_heads, head_dim;
    float theta, eps;
} orc_dims_t;

typedef struct {
    const int8_t* w;      /* [N, K] */
    const uint16_t* s;    /* [N, K/32] fp16 */
    int N, K;
    /* When non-NULL the layer uses these f32 weights [N, K] with the
     * reference's f32 matvec (inference.c:131-141) instead of INT8; used to
     * pin the layer composition against the reference's model_forward. */
    const float* f32;
    /* When non-NULL: `w` and `s` packed by orc_pack_rows8 (wp, sp); the
     * layer then runs orc_matmul_packed, with results identical to the
     * block matmul on w and s. */
    const int8_t* wp;
    const float* sp;
} orc_lin_t;

typedef struct {
    orc_lin_t q, k, v, o, gate, up, down;
} orc_layer_t;

typedef struct {
    orc_dims_t dims;
    const float* embed;       /* [vocab, d] */
    const orc_layer_t* base;  /* [dims.layers] */
    int draft_layers;
    const orc_layer_t* draft; /* [draft_layers] */
    orc_lin_t lm;             /* [vocab, d] */
    int n_medusa;
    const orc_lin_t* medusa;  /* [n_medusa] residual-block linears [d, d] */
} orc_model_t;

/* Per-stack KV cache, f32 [layers][cap][kv_heads][head_dim]. */
typedef struct {
    float* k;
    float* v;
    int layers, cap, kv_heads, head_dim;
} orc_kv_t;

int orc_kv_init(orc_kv_t* kv, int layers, int cap, int kv_heads, int head_dim);
void orc_kv_free(orc_kv_t* kv);

/* Runs M rows through a layer stack. Row m sits at cache slot base+m and
 * rotary position pos[m]; it attends to slots [0, base) and to slot base+j
 * iff mask[m*M + j] != 0 (mask NULL = causal). x: [M, d] in/out. */
void orc_stack_forward(const orc_model_t* mdl, const orc_layer_t* layers, int n_layers,
                       orc_kv_t* kv, float* x, int M, int base, const int* pos,
                       const uint8_t* mask);

/* logits[M, vocab] = LM(rmsnorm(x)). */
void orc_lm_logits(const orc_model_t* mdl, const float* x, float* logits, int M);

/* First index of the maximum (inference.c:104-111 ties rule). */
int orc_argmax(const float* v, int n);

/* Greedy chain speculative decoding (include/speculative.h rule).
 * Writes n_new tokens to out, per-step accepted counts to acc_hist (may be
 * NULL, length >= n_new), returns the number of steps. margins [n_new] (NULL
 * allowed): relative top-2 margin (top1 - top2) / |top1| of the base-model
 * logits row that chose out[i]. Prompt ids outside [0, vocab) read row 0. */
int orc_spec_generate(const orc_model_t* mdl, const int* prompt, int prompt_len,
                      int k_draft, int max_accepted, int n_new, int* out,
                      int* acc_hist, float* margins);

/* Wall time of the decode loop (after prefill and the first token) of the
 * last orc_spec_generate call, seconds. */
double orc_last_decode_seconds(void);

/* Plain greedy decoding with the base model only. */
void orc_greedy_generate(const orc_model_t* mdl, const int* prompt, int prompt_len,
                         int n_new, int* out, float* margins);

/* Medusa greedy decoding (include/medusa.h rule). topk[n_medusa], tree of at
 * most max_nodes nodes (root included). Returns steps. */
int orc_medusa_generate(const orc_model_t* mdl, const int* prompt, int prompt_len,
                        const int* topk, int max_nodes, int n_new, int* out,
                        int* acc_hist, float* margins);

/* Builds the Medusa candidate tree from per-head top-k lists.
 * tok[h][k], prob[h][k] for h < n_heads, k < topk[h]; writes tokens, parents,
 * depth, score of the kept nodes (root = node 0, token root_tok). Returns the
 * node count. */
int orc_medusa_tree(int root_tok, int n_heads, const int* topk, const int* tok,
                    const float* prob, int kmax, int max_nodes, int* out_tok,
                    int* out_parent, int* out_depth, float* out_score);

/* Stochastic speculative decoding (temperature T > 0, top-p nucleus):
 * Philox4x32-10 uniforms keyed by (seed, 0), counter (sequence, step,
 * position, purpose: 0 draft sample, 1 acceptance test, 2 resample / bonus;
 * the first token after the prefill uses step 0xFFFFFFFF). */
float orc_philox_uniform(uint32_t seed, uint32_t seq, uint32_t step, uint32_t pos, uint32_t purpose);
uint32_t orc_philox_u24(uint32_t seed, uint32_t seq, uint32_t step, uint32_t pos, uint32_t purpose);
/* Integer sampling rule (exact sums, so any summation order gives the same
 * result; see oracle.c): weight E = trunc(e^x * 2^24) of x = (l - max) / T;
 * nucleus weights (0 outside) and their mass; inverse-CDF pick at U / 2^24;
 * acceptance test u < p(x) / q(x); residual weights of max(0, p - q). */
uint32_t orc_sample_weight(float x);
uint64_t orc_sample_weights(const float* l, int V, float T, float top_p, uint32_t* E);
void orc_sample_dist(const float* l, int V, float T, float top_p, float* q);
int orc_sample_pick(const uint32_t* w32, const uint64_t* w64, int V, uint64_t total, uint32_t U);
int orc_sample_accept(uint32_t U, uint32_t Ep, uint64_t Mp, uint32_t Eq, uint64_t Mq);
uint64_t orc_sample_residual(const uint32_t* Ep, uint64_t Mp, const uint32_t* Eq, uint64_t Mq, int V,
                             uint64_t* R);
/* Draft tokens sampled from the draft distribution, accepted with
 * probability min(1, p / q), rejection resampled from norm(max(0, p - q)),
 * bonus from p when all K are accepted. Returns steps. */
int orc_spec_generate_sampled(const orc_model_t* mdl, const int* prompt, int prompt_len, int K, int n_new,
                              float T, float top_p, uint32_t seed, uint32_t seq_id, int* out, int* acc_hist);

#ifdef __cplusplus
}
#endif

#endif /* FL_ORACLE_H */
