// medusa.h decode functions over the fl_engine.
#include "fl_common.cuh"
#include "fl_host_sample.h"
#include "fl_runtime.h"
#include "medusa.h"

#include <algorithm>
#include <map>
#include <mutex>
#include <vector>

using namespace fl;

// api_spec.cu: per-model tree settings and weight binding.
int medusa_tree_settings(const medusa_model_t* m, const medusa_config_t* cfg, std::vector<int>& topk, int* max_nodes);
int medusa_bind(fl_engine_t* e, medusa_model_t* m);
fl_engine_t* medusa_engine(const medusa_model_t* m);
fl_engine_t* host_medusa_engine(medusa_model_t* m);

namespace {

// ---- host bases (a caller's own base_forward, not fl_cuda_base_forward) ----
// The contract is fl_cuda_base_forward's: the call appends the `len` tokens
// to the model's context and writes the last one's last-layer feature
// [hidden_size]. The heads and the LM head run on the Medusa model's own
// device engine; the base is given only tokens that are already part of the
// output, so a base that keeps per-position state never rolls back.
struct HostBase {
    void* model;
    void (*fwd)(void*, const int*, int, float*, int);
    int d;
};

std::mutex g_step_mu;
std::map<const void*, uint32_t> g_steps;  // medusa_decode_step calls per model (Philox step counter)

// The base model's token after feature F: LM-head argmax, or a draw at
// temperature T (top-p 1, Philox key (0, 0), purpose 2) at (step, pos).
int host_next(fl_engine_t* e, const float* F, float T, int V, uint32_t step, int pos, std::vector<float>& lg) {
    if (!(T > 0.0f)) {
        int t = -1;
        return fl_engine_lm_argmax(e, F, &t) == FL_OK ? t : -1;
    }
    lg.resize(V);
    if (fl_engine_lm_logits(e, F, lg.data()) != FL_OK) return -1;
    std::vector<uint32_t> E;
    const uint64_t M = fl_host::weights(lg.data(), V, T, 1.0f, E);
    return fl_host::pick(E, M, fl_host::u24(0u, 0u, step, (uint32_t)pos, 2u));
}

// One step: the heads' tree under `root` (the newest output token, not yet
// given to the base) from F, the base feature of the position before it.
// Walking down from the root, the current node's token is fed, the base's
// token g after it is decided and emitted; while g is a child of the
// current node the walk continues from that child, otherwise g ends the step
// (it is the next root). F ends as the feature of the last token fed.
int host_medusa_step(fl_engine_t* e, const HostBase& b, const std::vector<int>& topk, int H, int max_nodes, float T,
                     int V, int root, int pos, std::vector<float>& F, uint32_t step, int room, std::vector<int>& emit) {
    std::vector<int> tok(max_nodes), par(max_nodes), dep(max_nodes);
    const int M = fl_engine_medusa_tree(e, F.data(), root, topk.data(), H, max_nodes, tok.data(), par.data(),
                                        dep.data(), nullptr);
    if (M < 1) return -1;
    std::vector<float> lg;
    int cur = 0, p = pos;  // node being fed and its position
    while ((int)emit.size() < room) {
        b.fwd(b.model, &tok[cur], 1, F.data(), b.d);
        const int g = host_next(e, F.data(), T, V, step, p + 1, lg);
        if (g < 0) return -1;
        emit.push_back(g);
        int child = -1;
        for (int i = cur + 1; i < M; i++)
            if (par[i] == cur && tok[i] == g) {
                child = i;
                break;
            }
        if (child < 0) break;
        cur = child;
        p++;
    }
    return (int)emit.size();
}

int host_medusa_generate(void* bm, void (*bf)(void*, const int*, int, float*, int), medusa_model_t* m,
                         const float* prompt_hidden, int P, int* out, int n, const medusa_config_t* cfg) {
    fl_engine_t* e = host_medusa_engine(m);
    if (!e) return -1;
    std::vector<int> topk;
    int max_nodes = 64;
    const int H = medusa_tree_settings(m, cfg, topk, &max_nodes);
    if (H <= 0) return -1;
    const int V = m->vocab_size;
    const HostBase b{bm, bf, m->hidden_size};
    std::vector<int> seq(P);
    for (int i = 0; i < P; i++) {
        const int t = (int)prompt_hidden[i];
        seq[i] = t >= 0 && t < V ? t : 0;  // inference.c:420-426: ids outside the vocabulary embed as 0
    }
    std::vector<float> F(m->hidden_size), lg;
    bf(bm, seq.data(), P, F.data(), m->hidden_size);
    int root = host_next(e, F.data(), cfg->temperature, V, 0xFFFFFFFFu, P, lg);
    if (root < 0) return -1;
    int produced = 0, pos = P;
    out[produced++] = root;
    std::vector<int> emit;
    for (uint32_t step = 0; produced < n; step++) {
        emit.clear();
        if (host_medusa_step(e, b, topk, H, max_nodes, cfg->temperature, V, root, pos, F, step, n - produced, emit) <
            0)
            return -1;
        for (int t : emit) out[produced++] = t;
        pos += (int)emit.size();
        root = emit.back();
    }
    return produced;
}


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
    if (!base_forward || !medusa || !current_hidden || !output_tokens || !num_output || !config || current_token < 0)
        return -1;
    if (base_forward != fl_cuda_base_forward) {
        fl_engine_t* he = host_medusa_engine(medusa);
        if (!he || current_token >= medusa->vocab_size) return -1;
        std::vector<int> topk;
        int max_nodes = 64;
        const int H = medusa_tree_settings(medusa, config, topk, &max_nodes);
        if (H <= 0) return -1;
        uint32_t step;
        {
            std::lock_guard<std::mutex> lk(g_step_mu);
            step = g_steps[medusa]++;
        }
        std::vector<float> F(current_hidden, current_hidden + medusa->hidden_size);
        std::vector<int> emit;
        const HostBase b{base_model, base_forward, medusa->hidden_size};
        if (host_medusa_step(he, b, topk, H, max_nodes, config->temperature, medusa->vocab_size, current_token, 0, F,
                             step, max_nodes + 1, emit) < 0)
            return -1;
        for (size_t i = 0; i < emit.size(); i++) output_tokens[i] = emit[i];
        *num_output = (int)emit.size();
        return *num_output;
    }
    if (!base_model) return -1;
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
    if (!base_forward || !medusa || !prompt_hidden || prompt_len <= 0 || !output_tokens || num_tokens <= 0 || !config)
        return -1;
    if (base_forward != fl_cuda_base_forward)
        return host_medusa_generate(base_model, base_forward, medusa, prompt_hidden, prompt_len, output_tokens,
                                    num_tokens, config);
    if (!base_model) return -1;
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
