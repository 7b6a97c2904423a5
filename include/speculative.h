/*
 * EAGLE-style speculative decoding on B200.
 *
 * Same types, defaults and function signatures as the reference's
 * speculative.h (fast_llm/include/speculative.h:25-185), so callers written
 * against it compile unchanged. The reference declares this API but ships no
 * implementation; the behaviour below is this library's, and the CPU oracle
 * (oracle/oracle.h) restates exactly the same rules.
 *
 * Decoding rule (greedy chain, temperature <= 0 or config->temperature used
 * only for sampling when > 0):
 *   - The draft is a stack of `num_layers` decoder layers with the base
 *     model's dimensions. It shares the base embedding E and LM head.
 *   - Draft input at position i is  x_i = F_{i-1} + E[t_i], where F_{i-1} is
 *     the base model's last-layer output (before the final RMSNorm) at
 *     position i-1 (F_{-1} = 0). For positions drafted in the same step the
 *     draft's own last-layer output stands in for F.
 *   - One step: draft K tokens d_1..d_K (K = num_draft_tokens), verify the K+1
 *     rows [t_n, d_1..d_K] with the base model in one pass, accept the longest
 *     prefix with d_j == argmax(base logits at row j-1), then append the base
 *     model's token at the first mismatch (or after d_K): 1..K+1 new tokens.
 *   - temperature > 0 (speculative_generate through the device engine):
 *     distributions are integer nucleus weights. E_i = trunc(e^x * 2^24) of
 *     x = (l_i - max l) / temperature (0 below x = -17; e^x by Cody-Waite
 *     reduction by ln 2 and the degree-7 Taylor polynomial in Horner form,
 *     each step a correctly rounded fma or multiply). The nucleus keeps
 *     E_i >= t*, t* the largest integer whose kept mass S(t) reaches
 *     trunc(top_p * 2^24) / 2^24 of the total; M is the kept mass. A draw at
 *     U (24 bits of Philox4x32-10 keyed by (seed, 0) at counter (seq_id,
 *     step, position, purpose), purpose 0 draft, 1 acceptance, 2 resample or
 *     bonus; the first token after the prefill at step 0xFFFFFFFF) picks the
 *     first token whose running weight sum exceeds trunc(U * M / 2^24).
 *     d_j is drawn from the draft's weights q_j and accepted iff
 *     U * Mp * q_j(d_j) < 2^24 * p_j(d_j) * Mq (u < p / q); the first
 *     rejection draws from the residual max(0, p_j * Mq - q_j * Mp) / 2^24
 *     (from p_j when it is empty); when all K are accepted a bonus token is
 *     drawn from p_{K+1}. All sums are exact integers. top_p, seed and
 *     seq_id come from fl_engine_set_sampling (default 1.0, 0, 0).
 *
 * Host/device split: every weight, KV page and activation lives in HBM; the
 * structs below are host handles. The seven projection pointers of
 * draft_model_t each point to an array of `num_layers` tensors (the
 * reference struct holds one set; a multi-layer draft needs one per layer).
 * w_lm_head points to the shared LM head.
 *
 * Targets. target_forward(model, input, output, len) appends the `len`
 * token ids in `input` (floats, exact below 2^24) to the target's context
 * and writes `len` rows of next-token logits [len, vocab] to `output`.
 * fl_cuda_target_forward (fl_cuda.h) is that function for the device engine
 * (model = fl_engine_t*); the library then verifies all K+1 rows of a step
 * in one pass and rolls the engine's cache back to the accepted prefix.
 * Any other target_forward is the caller's own host function with the same
 * contract (model may be NULL); the library then
 *   - runs the draft on a device engine of its own (no base layers: the
 *     draft stack, the embedding and LM head from the draft's synthetic seed,
 *     seed 0 weights if the draft never loaded any) as a plain language
 *     model over token embeddings (no base features exist on the host),
 *   - feeds the target only tokens that are already part of the output, one
 *     per call during verification (the current token, then each accepted
 *     draft), so a target that keeps per-position state never rolls back;
 *     a step costs the target a+1 calls instead of one,
 *   - decides with the rule above from the target's logits, drafts greedy:
 *     greedy acceptance, or (temperature > 0) draft d kept with probability
 *     p(d) (U * Mp < 2^24 * E_p(d)) and otherwise a draw from p without d,
 *     at top-p 1 with Philox key (seed 0, sequence 0).
 *
 * Prompts. prompt_hidden holds prompt_len token ids as floats (not hidden
 * vectors, which the reference's header implies): a device target must
 * prefill its KV cache from tokens, and a host target receives the same ids.
 * Ids outside [0, vocab) are read as 0 (inference.c:420-426).
 */
#ifndef FL_SPECULATIVE_H
#define FL_SPECULATIVE_H

#include <stdint.h>
#include <stdbool.h>
#include "dequantized_tensor.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
    int num_draft_tokens;      /* K: tokens drafted per step              */
    float temperature;         /* <= 0: greedy; > 0: rejection sampling   */
    int max_accepted;          /* cap on accepted draft tokens per step   */
} speculative_config_t;

typedef struct {
    dequantized_tensor_t* w_q_proj;   /* [num_layers] each [H*hd, d]     */
    dequantized_tensor_t* w_k_proj;   /* [num_layers] each [Hkv*hd, d]   */
    dequantized_tensor_t* w_v_proj;   /* [num_layers] each [Hkv*hd, d]   */
    dequantized_tensor_t* w_o_proj;   /* [num_layers] each [d, H*hd]     */
    dequantized_tensor_t* w_gate;     /* [num_layers] each [ffn, d]      */
    dequantized_tensor_t* w_up;       /* [num_layers] each [ffn, d]      */
    dequantized_tensor_t* w_down;     /* [num_layers] each [d, ffn]      */
    dequantized_tensor_t* w_lm_head;  /* shared LM head [vocab, d]       */
    int num_layers;
    int hidden_size;
    int intermediate_size;
    int vocab_size;
} draft_model_t;

/* Draft KV cache handle. The cache itself is fp16 pages in HBM owned by the
 * handle; k_cache / v_cache stay NULL (no host copy is kept). */
typedef struct {
    float* k_cache;
    float* v_cache;
    int cache_len;
    int max_len;
} draft_kv_cache_t;

/* Drafted tokens of one step and the draft probability of each. */
typedef struct {
    int* tokens;
    float* probs;
    int num_tokens;
    int max_tokens;
} draft_tree_t;

static inline speculative_config_t speculative_default_config(void) {
    speculative_config_t cfg;
    cfg.num_draft_tokens = 4;
    cfg.temperature = 0.8f;
    cfg.max_accepted = 4;
    return cfg;
}

/* Allocates a draft of `num_layers` layers with empty weights
 * (reference speculative.h:78). Heads: hidden_size / 96 when divisible,
 * else hidden_size / 128 (head_dim is fixed by the base model at upload). */
draft_model_t* draft_model_create(int num_layers, int hidden_size,
                                  int intermediate_size, int vocab_size);

/* Fills the draft's weights (reference speculative.h:82). Supported path:
 * "synthetic:<seed>" -> seeded N(0, 0.02) -> Q4_0 -> INT8 [-8,7] with fp16
 * block scales, the same generator the base model uses. Returns 0 on
 * success, -1 on failure. */
int draft_model_load(draft_model_t* model, const char* path);

void draft_model_free(draft_model_t* model);

draft_kv_cache_t* draft_kv_cache_create(int max_len, int num_heads, int head_dim);
void draft_kv_cache_reset(draft_kv_cache_t* cache);
void draft_kv_cache_free(draft_kv_cache_t* cache);

draft_tree_t* draft_tree_create(int max_tokens);
void draft_tree_free(draft_tree_t* tree);

/* Drafts config->num_draft_tokens tokens after `current_token`, the draft
 * input of the first one being hidden_state + E[current_token]
 * (hidden_state: host [hidden_size], the base feature F of the previous
 * position). The draft must be bound to a base model by a previous
 * speculative_generate / fl_engine_bind_draft call (it needs E and the LM
 * head). Appends to `cache`. Returns the number of tokens drafted, or -1. */
int draft_tokens(draft_model_t* model, draft_kv_cache_t* cache,
                 const float* hidden_state, int current_token,
                 draft_tree_t* tree, const speculative_config_t* config);

/* Acceptance (reference speculative.h:121). `target_hidden` holds the base
 * model's logits for the K+1 verify rows, [(K+1), vocab] host floats, with
 * K = tree->num_tokens and vocab the one recorded in the tree by
 * draft_tokens. Greedy: accepted_tokens gets the accepted drafts followed by
 * the base model's next token -- up to K+1 entries, one more than the
 * reference's "0 to K", so size it K+1; *num_accepted = number of accepted
 * drafts. Returns *num_accepted, or -1 on bad arguments. */
int verify_tokens(const float* target_hidden, const draft_tree_t* tree,
                  int* accepted_tokens, int* num_accepted,
                  const speculative_config_t* config);

/* One draft + verify + accept step (reference speculative.h:146).
 * current_token is the newest output token (not yet given to the target).
 * With fl_cuda_target_forward, target_model is the fl_engine_t* and
 * current_hidden the base feature of the position before current_token (as
 * in draft_tokens). With a host target_forward, current_hidden is unused
 * and the draft's own cache holds the positions before
 * draft_cache->cache_len, where current_token goes; cache_len advances past
 * the emitted tokens. Writes 1..K+1 tokens to output_tokens, sets
 * *num_output and returns it; -1 on error. */
int speculative_decode_step(draft_model_t* draft, draft_kv_cache_t* draft_cache,
                            void* target_model,
                            void (*target_forward)(void* model, const float* input,
                                                   float* output, int len),
                            const float* current_hidden, int current_token,
                            int* output_tokens, int* num_output,
                            const speculative_config_t* config);

/* Full loop (reference speculative.h:173). prompt_hidden holds the prompt's
 * prompt_len token ids as floats. The target (an fl_engine_t* with
 * fl_cuda_target_forward, or the caller's host function, see "Targets")
 * takes the prompt, then speculative steps run until num_tokens new tokens
 * exist. Returns the number written (num_tokens on success), -1 on error. */
int speculative_generate(draft_model_t* draft, void* target_model,
                         void (*target_forward)(void*, const float*, float*, int),
                         const float* prompt_hidden, int prompt_len,
                         int* output_tokens, int num_tokens,
                         const speculative_config_t* config);

#ifdef __cplusplus
}
#endif

#endif /* FL_SPECULATIVE_H */
