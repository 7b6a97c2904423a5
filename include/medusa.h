/*
 * Medusa multi-token prediction on B200.
 *
 * Same types, defaults and function signatures as the reference's medusa.h
 * (fast_llm/include/medusa.h:32-229). The reference declares this API but
 * ships no implementation; the behaviour below is this library's and the CPU
 * oracle restates the same rules.
 *
 * Head i (0-based) predicts the token at offset i+2 from the last verified
 * position (the base LM head itself predicts offset 1). A head is a residual
 * block on the normalised base hidden state h = RMSNorm(F):
 *     z_i = h + SiLU(W_i h),   logits_i = LM_head(z_i)
 * with W_i an INT8 [hidden, hidden] tensor in medusa_head_t.weights and the
 * base model's INT8 LM head shared by every head. SiLU uses the reference's
 * polynomial sigmoid (activations_avx2.c:33-63). medusa_head_t.bias, when
 * non-NULL, is added to W_i h before SiLU.
 *
 * Candidate tree: the root is the base model's next token; level L+1 holds
 * the children proposed by head L for every level-L node. Each head keeps its
 * top-k tokens (k per level from fl_medusa_set_tree, default config->top_k),
 * a node's score is the product of its ancestors' softmax probabilities, and
 * the tree is pruned to the max_candidates highest-scoring nodes (ties:
 * shallower first, then lower head rank); a child never outscores its
 * parent, so the kept set is ancestor-closed. Verification runs every node
 * through the base model in one pass with a tree attention mask; the longest
 * root-to-leaf path whose every token equals the base model's greedy choice
 * at its parent is accepted, plus the base model's token after it.
 *
 * Bases. base_forward(model, tokens, len, hidden, hidden_size) appends the
 * `len` tokens to the base's context and writes the last one's last-layer
 * feature F [hidden_size]. fl_cuda_base_forward is that function for the
 * device engine (model = fl_engine_t*), which verifies a whole tree in one
 * tree-masked pass. Any other base_forward is the caller's own host function
 * (model may be NULL): the heads and an LM head (the Medusa model's, from
 * its synthetic seed; seed 0 heads if it never loaded any) run on a device
 * engine of the Medusa model's own, and the tree is walked on the host --
 * the current node's token is fed, the base's next token g (LM-head argmax
 * of the returned F, or a draw at temperature > 0: top-p 1, Philox key
 * (0, 0)) is emitted, and the walk goes on while g is a child of the node.
 * The base is given only tokens that are part of the output, so it never
 * rolls back; each emitted token costs one base_forward call.
 * medusa_verify_tree needs the device engine (a tree carries no context).
 */
#ifndef FL_MEDUSA_H
#define FL_MEDUSA_H

#include <stdint.h>
#include <stdbool.h>
#include "dequantized_tensor.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
    int num_heads;             /* number of Medusa heads                 */
    int top_k;                 /* candidates kept per head (default k)   */
    float temperature;         /* <= 0 greedy acceptance                 */
} medusa_config_t;

typedef struct {
    dequantized_tensor_t* weights;   /* residual-block linear [hidden, hidden] */
    float* bias;                     /* optional [hidden]                      */
    int head_id;                     /* predicts offset head_id + 2            */
    int hidden_size;
    int vocab_size;
} medusa_head_t;

typedef struct {
    medusa_head_t* heads;
    int num_heads;
    int hidden_size;
    int vocab_size;
} medusa_model_t;

/* Candidate tree. Node 0 is the root; parent_indices[0] = -1. positions[i]
 * is the node's depth (root 0); its sequence position is prefix + depth. */
typedef struct {
    int* tokens;
    float* probs;
    int* parent_indices;
    int* positions;
    int num_candidates;
    int max_candidates;
} medusa_tree_t;

static inline medusa_config_t medusa_default_config(void) {
    medusa_config_t cfg;
    cfg.num_heads = 3;
    cfg.top_k = 8;
    cfg.temperature = 0.8f;
    return cfg;
}

medusa_model_t* medusa_model_create(int num_heads, int hidden_size, int vocab_size);

/* "synthetic:<seed>" fills every head with the seeded Q4_0 -> INT8 generator.
 * Returns 0 on success, -1 otherwise. */
int medusa_model_load(medusa_model_t* model, const char* path);
void medusa_model_free(medusa_model_t* model);

medusa_tree_t* medusa_tree_create(int max_candidates);
void medusa_tree_free(medusa_tree_t* tree);

/* Step-level entry points (greedy). The heads must be bound to an engine
 * (medusa_generate, medusa_decode_step or fl_engine_bind_medusa).
 * medusa_predict: candidate tree with current_token as the root, from the
 * base feature hidden_state (the feature of the position before
 * current_token); tree->probs holds node scores. medusa_build_tree: the same
 * with the base LM head's argmax of hidden_state as the root.
 * medusa_verify_tree: one tree-masked base pass at the engine's callback
 * position (fl_engine_position): accepted_tokens gets the accepted path and
 * then the base model's next token, *num_accepted the path length; the path's
 * KV is compacted and the position advances past root and path.
 * medusa_decode_step: predict + verify; output_tokens gets the accepted tokens
 * and the next token (*num_output = accepted + 1); the next current_hidden is
 * fl_engine_last_feature and the next current_token the last output. */
int medusa_predict(medusa_model_t* model, const float* hidden_state,
                   int current_token, medusa_tree_t* tree,
                   const medusa_config_t* config);
int medusa_build_tree(medusa_model_t* model, const float* hidden_state,
                      medusa_tree_t* tree, const medusa_config_t* config);
int medusa_verify_tree(void* base_model,
                       void (*base_forward)(void*, const int*, int, float*, int),
                       const medusa_tree_t* tree, int* accepted_tokens,
                       int* num_accepted, const medusa_config_t* config);
int medusa_decode_step(void* base_model,
                       void (*base_forward)(void*, const int*, int, float*, int),
                       medusa_model_t* medusa, const float* current_hidden,
                       int current_token, int* output_tokens, int* num_output,
                       const medusa_config_t* config);

/* base_model: an fl_engine_t* created with medusa_heads >= the heads used
 * and base_forward fl_cuda_base_forward (greedy acceptance only,
 * temperature <= 0; the heads' weights are loaded into the engine on the
 * first call), or the caller's own host base_forward (see "Bases";
 * temperature > 0 draws). prompt_hidden holds prompt_len token ids as
 * floats. Medusa steps run until num_tokens new tokens exist. Returns the
 * count written or -1. */
int medusa_generate(void* base_model,
                    void (*base_forward)(void*, const int*, int, float*, int),
                    medusa_model_t* medusa, const float* prompt_hidden,
                    int prompt_len, int* output_tokens, int num_tokens,
                    const medusa_config_t* config);

/* This library: per-model tree settings used by medusa_generate (no
 * counterpart in the reference): top-k of head h = topk[h] (h < n; default
 * config->top_k), at most max_nodes tree nodes (default 64). */
int fl_medusa_set_tree(medusa_model_t* model, const int* topk, int n, int max_nodes);

/* Draft + Medusa combination (reference medusa.h:210; the reference ships no
 * implementation). draft_model: a draft_model_t loaded for the engine;
 * draft_forward: fl_cuda_target_forward or NULL (the draft runs inside the
 * engine); target_model: the engine, target_forward fl_cuda_base_forward.
 * Each step the draft chain (config->num_heads tokens, at most 7) and the
 * Medusa heads' candidate tree (fl_medusa_set_tree settings) are verified
 * together in one tree pass; greedy acceptance of the longest matching path.
 * Returns num_tokens or -1. */
int speculative_medusa_generate(void* draft_model,
                                void (*draft_forward)(void*, const float*, float*, int),
                                medusa_model_t* medusa, void* target_model,
                                void (*target_forward)(void*, const int*, int, float*, int),
                                const float* prompt_hidden, int prompt_len,
                                int* output_tokens, int num_tokens,
                                const medusa_config_t* config);

#ifdef __cplusplus
}
#endif

#endif /* FL_MEDUSA_H */
