// medusa.h decode functions over the fl_engine.
#include "fl_common.cuh"
#include "fl_runtime.h"
#include "medusa.h"

#include <vector>

using namespace fl;

FL_API int medusa_predict(medusa_model_t*, const float*, int, medusa_tree_t*, const medusa_config_t*) {
    return set_error(FL_E_UNSUPPORTED, "medusa_predict: not available in this build"), -1;
}
FL_API int medusa_build_tree(medusa_model_t*, const float*, medusa_tree_t*, const medusa_config_t*) {
    return set_error(FL_E_UNSUPPORTED, "medusa_build_tree: not available in this build"), -1;
}
FL_API int medusa_verify_tree(void*, void (*)(void*, const int*, int, float*, int), const medusa_tree_t*, int*, int*,
                              const medusa_config_t*) {
    return set_error(FL_E_UNSUPPORTED, "medusa_verify_tree: not available in this build"), -1;
}
FL_API int medusa_decode_step(void*, void (*)(void*, const int*, int, float*, int), medusa_model_t*, const float*, int,
                              int*, int*, const medusa_config_t*) {
    return set_error(FL_E_UNSUPPORTED, "medusa_decode_step: not available in this build"), -1;
}
// api_spec.cu: per-model tree settings and weight binding.
int medusa_tree_settings(const medusa_model_t* m, const medusa_config_t* cfg, std::vector<int>& topk, int* max_nodes);
int medusa_bind(fl_engine_t* e, medusa_model_t* m);

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
