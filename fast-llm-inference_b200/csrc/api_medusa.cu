// medusa.h decode functions over the fl_engine.
#include "fl_common.cuh"
#include "fl_runtime.h"
#include "medusa.h"

#include <algorithm>
#include <vector>

using namespace fl;

// api_spec.cu: per-model tree settings and weight binding.
int medusa_tree_settings(const medusa_model_t* m, const medusa_config_t* cfg, std::vector<int>& topk, int* max_nodes);
int medusa_bind(fl_engine_t* e, medusa_model_t* m);
fl_engine_t* medusa_engine(const medusa_model_t* m);

namespace {

// Fills a medusa_tree_t from the heads (root >= 0: that token; < 0: the base
// LM head's argmax of the feature).
int predict_tree(medusa_model_t* model, const float* hidden, int root, medusa_tree_t* tree,
                 const medusa_config_t* config) {
    if (!model || !hidden || !tree || !config) return -1;
    fl_engine_t* e = medusa_engine(model);
    if (!e) {
        set_error(FL_E_STATE, "medusa: heads not bound to an engine (medusa_generate, medusa_decode_step or "
                              "fl_engine_bind_medusa)");
        return -1;
    }
    std::vector<int> topk;
    int max_nodes = 64;
    const int H = medusa_tree_settings(model, config, topk, &max_nodes);
    if (H <= 0) return -1;
    max_nodes = std::min(max_nodes, tree->max_candidates);
    const int M = fl_engine_medusa_tree(e, hidden, root, topk.data(), H, max_nodes, tree->tokens,
                                        tree->parent_indices, tree->positions, tree->probs);
    if (M < 0) return -1;
    tree->num_candidates = M;
    return M;
}

}  // namespace

// Candidate tree with current_token as the root (include/medusa.h rule).
FL_API int medusa_predict(medusa_model_t* model, const float* hidden_state, int current_token, medusa_tree_t* tree,
                          const medusa_config_t* config) {
    if (current_token < 0) return -1;
    return predict_tree(model, hidden_state, current_token, tree, config);
}

// Candidate tree whose root is the base model's next token (LM-head argmax of
// the feature).
FL_API int medusa_build_tree(medusa_model_t* model, const float* hidden_state, medusa_tree_t* tree,
                             const medusa_config_t* config) {
    return predict_tree(model, hidden_state, -1, tree, config);
}

// Verifies a tree at the engine's callback position: accepted_tokens gets the
// accepted path's tokens and, after them, the base model's next token;
// *num_accepted (and the return value) is the path length without that token.
FL_API int medusa_verify_tree(void* base_model, void (*base_forward)(void*, const int*, int, float*, int),
                              const medusa_tree_t* tree, int* accepted_tokens, int* num_accepted,
                              const medusa_config_t* config) {
    if (!base_model || !tree || !accepted_tokens || !num_accepted || !config || tree->num_candidates < 1) return -1;
    if (base_forward != fl_cuda_base_forward) {
        set_error(FL_E_UNSUPPORTED, "medusa_verify_tree: base_forward must be fl_cuda_base_forward");
        return -1;
    }
    if (config->temperature > 0.0f) {
        set_error(FL_E_UNSUPPORTED, "medusa_verify_tree: only greedy acceptance (temperature <= 0)");
        return -1;
    }
    int a = 0;
    if (fl_engine_tree_verify((fl_engine_t*)base_model, tree->tokens, tree->parent_indices, tree->positions,
                              tree->num_candidates, accepted_tokens, &a) != FL_OK)
        return -1;
    *num_accepted = a;
    return a;
}

// One Medusa step at the engine's callback position: current_token is the
// base model's latest token (not yet in the cache), current_hidden the base
// feature of the position before it. output_tokens receives the accepted
// tokens and the base model's next token (*num_output of them).
FL_API int medusa_decode_step(void* base_model, void (*base_forward)(void*, const int*, int, float*, int),
                              medusa_model_t* medusa, const float* current_hidden, int current_token,
                              int* output_tokens, int* num_output, const medusa_config_t* config) {
    if (!base_model || !medusa || !current_hidden || !output_tokens || !num_output || !config || current_token < 0)
        return -1;
    if (base_forward != fl_cuda_base_forward) {
        set_error(FL_E_UNSUPPORTED, "medusa_decode_step: base_forward must be fl_cuda_base_forward");
        return -1;
    }
    fl_engine_t* e = (fl_engine_t*)base_model;
    if (medusa_bind(e, medusa) != FL_OK) return -1;
    std::vector<int> topk;
    int max_nodes = 64;
    const int H = medusa_tree_settings(medusa, config, topk, &max_nodes);
    if (H <= 0) return -1;
    std::vector<int> tok(max_nodes), par(max_nodes), dep(max_nodes);
    const int M = fl_engine_medusa_tree(e, current_hidden, current_token, topk.data(), H, max_nodes, tok.data(),
                                        par.data(), dep.data(), nullptr);
    if (M < 0) return -1;
    int a = 0;
    if (fl_engine_tree_verify(e, tok.data(), par.data(), dep.data(), M, output_tokens, &a) != FL_OK) return -1;
    *num_output = a + 1;
    return a + 1;
}

// Greedy Medusa decoding over the device engine: base_model is an
// fl_engine_t* created with medusa_heads >= the model's heads, base_forward
// fl_cuda_base_forward, prompt_hidden the prompt ids as floats.
FL_API int medusa_generate(void* base_model, void (*base_forward)(void*, const int*, int, float*, int),
                           medusa_model_t* medusa, const float* prompt_hidden, int prompt_len, int* output_tokens,
                           int num_tokens, const medusa_config_t* config) {
    if (!base_model || !medusa || !prompt_hidden || prompt_len <= 0 || !output_tokens || num_tokens <= 0 || !config)
        return -1;
    if (base_forward != fl_cuda_base_forward) {
        set_error(FL_E_UNSUPPORTED, "medusa_generate: base_forward must be fl_cuda_base_forward");
        return -1;
    }
    if (config->temperature > 0.0f) {
        set_error(FL_E_UNSUPPORTED, "medusa_generate: only greedy acceptance (temperature <= 0)");
        return -1;
    }
    fl_engine_t* e = (fl_engine_t*)base_model;
    if (medusa_bind(e, medusa) != FL_OK) return -1;
    std::vector<int> topk;
    int max_nodes = 64;
    const int H = medusa_tree_settings(medusa, config, topk, &max_nodes);
    if (H <= 0) return -1;
    std::vector<int> prompt(prompt_len);
    for (int i = 0; i < prompt_len; i++) prompt[i] = (int)prompt_hidden[i];
    if (fl_engine_medusa_generate(e, prompt.data(), prompt_len, num_tokens, topk.data(), H, max_nodes, output_tokens,
                                  nullptr, nullptr) != FL_OK)
        return -1;
    return num_tokens;
}
