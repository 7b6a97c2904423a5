/*
 * Reference shim -- TEST INFRASTRUCTURE.
 *
 * Compiles the reference project's own C sources (read in place from the
 * reference checkout, never copied) into oracle/_ref/libref.so and exports
 * their static helpers through plain-pointer wrappers, so tests can pin the
 * oracle's restatement against the reference's actual code. Built by
 * oracle/Makefile with the reference's flags (fast_llm/Makefile:5-6:
 * -O3 -fopenmp -ffast-math -mavx2 -mfma).
 *
 * Included translation units (paths relative to fast_llm/):
 *   src/kernels/dequantized_tensor.c  quantize_to_uint8, dot_product_u8_i8,
 *                                     matmul_dequantized
 *   src/kernels/activations_avx2.c    rms_norm_avx2, swiglu_avx2, silu_avx2
 *   src/inference.c                   apply_rope, compute_attention,
 *                                     model_forward (f32-weight mode)
 */
#include "src/kernels/dequantized_tensor.c"
#include "src/kernels/activations_avx2.c"
#include "src/inference.c"

#define REF_API __attribute__((visibility("default")))

REF_API void ref_quantize_to_uint8(const float* src, uint8_t* dst, int n) {
    quantize_to_uint8(src, dst, n, 127.0f);
}

REF_API int32_t ref_dot_product_u8_i8(const uint8_t* a, const int8_t* b, int n) {
    return dot_product_u8_i8(a, b, n);
}

/* The reference's matmul_dequantized on a per-row-scale tensor. */
REF_API void ref_matmul_dequantized(const float* A, const int8_t* W, const float* scales,
                                    float* C, int M, int N, int K) {
    dequantized_tensor_t t;
    memset(&t, 0, sizeof(t));
    t.weights = (int8_t*)W;
    t.scales = (float*)scales;
    t.rows = N;
    t.cols = K;
    t.original_bits = 8;
    matmul_dequantized(A, &t, C, M, N, K);
}

REF_API void ref_rms_norm(const float* in, float* out, int n, float eps) {
    rms_norm_avx2(in, out, n, eps);
}

REF_API void ref_swiglu(const float* g, const float* u, float* out, int n) {
    swiglu_avx2(g, u, out, n);
}

REF_API void ref_silu(const float* x, float* out, int n) {
    silu_avx2(x, out, n);
}

REF_API void ref_apply_rope(float* q, float* k, int seq_len, int heads, int kv_heads,
                            int head_dim, float theta) {
    apply_rope(q, k, seq_len, heads, kv_heads, head_dim, theta);
}

/* RoPE (theta 500000, inference.c:196) + causal softmax attention. */
REF_API void ref_compute_attention(float* Q, float* K, const float* V, float* out,
                                   int seq_len, int heads, int kv_heads, int head_dim) {
    compute_attention(Q, K, V, out, seq_len, heads, kv_heads, head_dim);
}

static dequantized_tensor_t* f32_tensor(const float* w, int rows, int cols) {
    dequantized_tensor_t* t = (dequantized_tensor_t*)calloc(1, sizeof(*t));
    t->f32_weights = (float*)w;
    t->rows = rows;
    t->cols = cols;
    t->original_bits = -1; /* borrowed pointer: do not free */
    return t;
}

/* Builds a transformer_model_t around caller-owned f32 weights and runs the
 * reference's model_forward (full recompute, LM head on the last row).
 * w holds 7 pointers per layer: q, k, v, o, gate, up, down ([out, in]).
 * Norm weights are all 1.0. Returns the reference's greedy token. */
REF_API int ref_model_forward_f32(int vocab, int d, int ffn, int layers, int heads,
                                  int kv_heads, int head_dim, const float* embed,
                                  const float* const* w, const float* lm,
                                  const int* tokens, int seq_len, float* logits) {
    transformer_model_t m;
    memset(&m, 0, sizeof(m));
    m.config.vocab_size = vocab;
    m.config.hidden_size = d;
    m.config.intermediate_size = ffn;
    m.config.num_layers = layers;
    m.config.num_heads = heads;
    m.config.num_kv_heads = kv_heads;
    m.config.head_dim = head_dim;
    m.config.max_seq_len = 4096;
    m.token_embeddings = (float*)embed;
    const int qd = heads * head_dim, kd = kv_heads * head_dim;
    m.q_proj = calloc(layers, sizeof(void*));
    m.k_proj = calloc(layers, sizeof(void*));
    m.v_proj = calloc(layers, sizeof(void*));
    m.o_proj = calloc(layers, sizeof(void*));
    m.gate_proj = calloc(layers, sizeof(void*));
    m.up_proj = calloc(layers, sizeof(void*));
    m.down_proj = calloc(layers, sizeof(void*));
    m.input_layernorm = calloc(layers, sizeof(float*));
    m.post_attn_layernorm = calloc(layers, sizeof(float*));
    float* ones = malloc(sizeof(float) * d);
    for (int i = 0; i < d; i++) ones[i] = 1.0f;
    for (int l = 0; l < layers; l++) {
        const float* const* lw = w + 7 * l;
        m.q_proj[l] = f32_tensor(lw[0], qd, d);
        m.k_proj[l] = f32_tensor(lw[1], kd, d);
        m.v_proj[l] = f32_tensor(lw[2], kd, d);
        m.o_proj[l] = f32_tensor(lw[3], d, qd);
        m.gate_proj[l] = f32_tensor(lw[4], ffn, d);
        m.up_proj[l] = f32_tensor(lw[5], ffn, d);
        m.down_proj[l] = f32_tensor(lw[6], d, ffn);
        m.input_layernorm[l] = ones;
        m.post_attn_layernorm[l] = ones;
    }
    m.output_norm = ones;
    m.lm_head = f32_tensor(lm, vocab, d);
    int tok = -1;
    model_forward(&m, tokens, seq_len, logits, &tok);
    for (int l = 0; l < layers; l++) {
        free(m.q_proj[l]); free(m.k_proj[l]); free(m.v_proj[l]); free(m.o_proj[l]);
        free(m.gate_proj[l]); free(m.up_proj[l]); free(m.down_proj[l]);
    }
    free(m.q_proj); free(m.k_proj); free(m.v_proj); free(m.o_proj);
    free(m.gate_proj); free(m.up_proj); free(m.down_proj);
    free(m.input_layernorm); free(m.post_attn_layernorm);
    free(m.lm_head);
    free(ones);
    return tok;
}
