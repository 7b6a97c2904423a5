// speculative.h and medusa.h over the fl_engine (include/speculative.h,
// include/medusa.h state the rules; the reference declares the functions in
// fast_llm/include/speculative.h:78-185 and medusa.h:84-229 without
// defining them).
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <map>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "fl_common.cuh"
#include "fl_host_sample.h"
#include "fl_runtime.h"
#include "medusa.h"
#include "speculative.h"

using namespace fl;

// api_gguf.cu
int gguf_load_draft(draft_model_t* m, const char* path);
int gguf_load_medusa(medusa_model_t* m, const char* path);
int gguf_load_embedding(const char* path, int vocab, int hidden, std::vector<float>& out);

namespace {

// Hidden extension of draft_tree_t: the vocabulary size recorded by
// draft_tokens so verify_tokens can walk [(K+1), vocab] logits.
struct TreeImpl {
    draft_tree_t pub;
    int vocab;
};

struct CacheImpl {
    draft_kv_cache_t pub;
    int num_heads, head_dim;
    int steps;  // speculative_decode_step calls with a host target (Philox step counter)
};

std::mutex g_bind_mu;
std::map<const void*, fl_engine_t*> g_bind;  // draft / Medusa model -> engine

void bind(const void* m, fl_engine_t* e) {
    std::lock_guard<std::mutex> lk(g_bind_mu);
    g_bind[m] = e;
}
fl_engine_t* bound(const void* m) {
    std::lock_guard<std::mutex> lk(g_bind_mu);
    auto it = g_bind.find(m);
    return it == g_bind.end() ? nullptr : it->second;
}
void unbind(const void* m) {
    std::lock_guard<std::mutex> lk(g_bind_mu);
    g_bind.erase(m);
}

bool parse_synthetic(const char* path, uint64_t* seed) {
    if (!path || strncmp(path, "synthetic:", 10) != 0) return false;
    char* end = nullptr;
    unsigned long long v = strtoull(path + 10, &end, 10);
    if (!end || *end != '\0' || end == path + 10) return false;
    *seed = v;
    return true;
}

// Seed of each draft / Medusa model's synthetic weights (0 when the model
// never loaded any: its weights are then generated from seed 0 on first
// use), and the device engines that run a draft or Medusa heads for host
// targets (a caller's own target_forward / base_forward).
std::map<const void*, uint64_t> g_seed;
std::map<const void*, std::string> g_gguf;  // model -> GGUF file it was loaded from
std::map<const void*, fl_engine_t*> g_host_eng;

uint64_t synth_seed(const void* m) {
    std::lock_guard<std::mutex> lk(g_bind_mu);
    auto it = g_seed.find(m);
    return it == g_seed.end() ? 0 : it->second;
}

// True (with the seed) when the model's weights came from "synthetic:<seed>".
bool synth_seed_of(const void* m, uint64_t* seed) {
    std::lock_guard<std::mutex> lk(g_bind_mu);
    auto it = g_seed.find(m);
    if (it == g_seed.end()) return false;
    *seed = it->second;
    return true;
}

// Head size of a draft / Medusa model given only its hidden size: 96 when it
// divides (the Phi-3 shapes), else 128, else 64.
int head_dim_for(int d) { return d % 96 == 0 ? 96 : d % 128 == 0 ? 128 : d % 64 == 0 ? 64 : 0; }

void free_tensor_array(dequantized_tensor_t* arr, int n) {
    if (!arr) return;
    for (int i = 0; i < n; i++) {
        release_tensor(&arr[i]);
        free(arr[i].weights);
        free(arr[i].scales);
        free(arr[i].scales_f16);
    }
    free(arr);
}

int synth_tensor(dequantized_tensor_t* t, uint64_t seed, uint32_t id, int rows, int cols) {
    release_tensor(t);
    free(t->weights);
    free(t->scales);
    free(t->scales_f16);
    t->weights = (int8_t*)malloc((size_t)rows * cols);
    t->scales_f16 = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)rows * (cols / 32));
    t->scales = nullptr;
    if (!t->weights || !t->scales_f16) return set_error(FL_E_NOMEM, "synthetic tensor: host allocation");
    t->rows = rows;
    t->cols = cols;
    t->original_bits = 4;
    t->scale_block = 32;
    return fl_synth_q4_0_i8(seed, id, rows, cols, 0.02f, t->weights, t->scales_f16);
}

// Pushes a draft model's host tensors into the engine's draft stack. The
// draft's layers share the engine's head layout, so a synthetic draft
// (whose host q/k/v/o tensors have the speculative.h shapes [d, d]) bound
// to an engine with grouped-query heads or q_dim != d gets those four
// projections generated again from the same seed and tensor ids at the
// engine's shapes: q [q_dim, d], k and v [kv_dim, d], o [d, q_dim]. Loaded
// (GGUF or caller-filled) tensors go in as they are, and a shape the engine
// does not take is an error from fl_engine_load_linear.
int load_draft_into(fl_engine_t* e, const draft_model_t* dm) {
    const dequantized_tensor_t* arrs[7] = {dm->w_q_proj, dm->w_k_proj, dm->w_v_proj, dm->w_o_proj,
                                           dm->w_gate, dm->w_up, dm->w_down};
    int dims[4];
    FL_CHECK(fl_engine_dims(e, dims));
    const int want[4][2] = {{dims[1], dims[0]}, {dims[2], dims[0]}, {dims[2], dims[0]}, {dims[0], dims[1]}};
    uint64_t seed = 0;
    const bool synth = synth_seed_of(dm, &seed);
    for (int l = 0; l < dm->num_layers; l++)
        for (int p = 0; p < 7; p++) {
            const dequantized_tensor_t* t = arrs[p] ? &arrs[p][l] : nullptr;
            if (!t || !t->weights) continue;  // keep what the engine holds
            if (t->scale_block != 32 || !t->scales_f16)
                return set_error(FL_E_UNSUPPORTED, "draft tensors must be in block mode (scale_block 32)");
            if (synth && p < 4 && (t->rows != want[p][0] || t->cols != want[p][1])) {
                dequantized_tensor_t r = {};
                int rc = synth_tensor(&r, seed, FL_TENSOR_ID(1, l, p), want[p][0], want[p][1]);
                if (rc == FL_OK) rc = fl_engine_load_linear(e, 1, l, p, r.weights, r.scales_f16, r.rows, r.cols);
                free(r.weights);
                free(r.scales_f16);
                FL_CHECK(rc);
                continue;
            }
            FL_CHECK(fl_engine_load_linear(e, 1, l, p, t->weights, t->scales_f16, t->rows, t->cols));
        }
    const dequantized_tensor_t* lm = dm->w_lm_head;
    if (lm && lm->weights) {
        if (lm->scale_block != 32 || !lm->scales_f16)
            return set_error(FL_E_UNSUPPORTED, "LM head must be in block mode (scale_block 32)");
        FL_CHECK(fl_engine_load_linear(e, 3, 0, 1, lm->weights, lm->scales_f16, lm->rows, lm->cols));
    }
    return FL_OK;
}

// Medusa tree settings per model (medusa_model_t has no room for them):
// per-head top-k and the node budget.
struct MedusaTree {
    std::vector<int> topk;
    int max_nodes = 64;
};
std::unordered_map<const void*, MedusaTree> g_med_tree;

}  // namespace

int medusa_tree_settings(const medusa_model_t* m, const medusa_config_t* cfg, std::vector<int>& topk,
                         int* max_nodes) {
    std::lock_guard<std::mutex> lk(g_bind_mu);
    const int H = m->num_heads < cfg->num_heads ? m->num_heads : cfg->num_heads;
    auto it = g_med_tree.find(m);
    topk.assign(H, cfg->top_k);
    *max_nodes = 64;
    if (it != g_med_tree.end()) {
        for (int h = 0; h < H && h < (int)it->second.topk.size(); h++) topk[h] = it->second.topk[h];
        *max_nodes = it->second.max_nodes;
    }
    return H;
}

int medusa_bind(fl_engine_t* e, medusa_model_t* m);
fl_engine_t* medusa_engine(const medusa_model_t* m) { return bound(m); }

// ------------------------------------------------------------------ host targets
// Device engines for models whose target / base is a caller's host function:
// no base layers, only the draft stack (or the Medusa heads) with the
// embedding and the LM head, generated from the model's synthetic seed
// (the LM head a loaded draft carries is used as it is). One engine per
// model, on the current device, released with the model.

void host_engine_release(const void* m) {
    fl_engine_t* e = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_bind_mu);
        auto it = g_host_eng.find(m);
        if (it != g_host_eng.end()) {
            e = it->second;
            g_host_eng.erase(it);
        }
        g_seed.erase(m);
        g_gguf.erase(m);
    }
    if (e) fl_engine_destroy(e);
}

static std::string gguf_of(const void* m) {
    std::lock_guard<std::mutex> lk(g_bind_mu);
    auto it = g_gguf.find(m);
    return it == g_gguf.end() ? std::string() : it->second;
}

static fl_engine_t* host_engine_get(const void* m) {
    std::lock_guard<std::mutex> lk(g_bind_mu);
    auto it = g_host_eng.find(m);
    return it == g_host_eng.end() ? nullptr : it->second;
}

// Context capacity of the host-target engines (draft cache positions).
constexpr int kHostCtx = 4096;

static fl_engine_t* host_engine_new(int vocab, int d, int ffn, int draft_layers, int medusa_heads, uint64_t seed,
                                    const std::string& gguf) {
    const int hd = head_dim_for(d);
    if (hd == 0) {
        set_error(FL_E_UNSUPPORTED, "host target: hidden size must be a multiple of 64");
        return nullptr;
    }
    fl_model_config_t c = {};
    c.vocab_size = vocab;
    c.hidden_size = d;
    c.intermediate_size = ffn;
    c.num_layers = 0;
    c.num_heads = d / hd;
    c.num_kv_heads = d / hd;
    c.head_dim = hd;
    c.draft_layers = draft_layers;
    c.medusa_heads = medusa_heads;
    c.max_seq_len = kHostCtx;
    c.rope_theta = 10000.0f;
    c.norm_eps = 1e-5f;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) dev = 0;
    fl_engine_t* e = fl_engine_create(&c, dev);
    if (!e) return nullptr;
    std::vector<float> emb((size_t)vocab * d);
    const int erc = gguf.empty() ? fl_synth_q4_0_f32(seed, FL_TENSOR_ID(3, 0, 0), vocab, d, 0.02f, emb.data())
                                 : gguf_load_embedding(gguf.c_str(), vocab, d, emb);
    if (erc != FL_OK || fl_engine_load_embedding(e, emb.data()) != FL_OK) {
        fl_engine_destroy(e);
        return nullptr;
    }
    return e;
}

// The draft's own engine (draft weights generated from seed 0 if the draft
// never loaded any).
static fl_engine_t* host_draft_engine(draft_model_t* dm) {
    if (fl_engine_t* e = host_engine_get(dm)) return e;
    if (!dm->w_q_proj[0].weights && draft_model_load(dm, "synthetic:0") != 0) return nullptr;
    fl_engine_t* e = host_engine_new(dm->vocab_size, dm->hidden_size, dm->intermediate_size, dm->num_layers, 0,
                                     synth_seed(dm), gguf_of(dm));
    if (!e) return nullptr;
    if (load_draft_into(e, dm) != FL_OK || !fl_engine_ready(e)) {
        fl_engine_destroy(e);
        set_error(FL_E_STATE, "host target: draft weights incomplete");
        return nullptr;
    }
    std::lock_guard<std::mutex> lk(g_bind_mu);
    g_host_eng[dm] = e;
    return e;
}

// The Medusa heads' own engine (heads generated from seed 0 if never
// loaded; LM head from the heads' seed).
fl_engine_t* host_medusa_engine(medusa_model_t* m) {
    if (fl_engine_t* e = host_engine_get(m)) return e;
    if ((!m->heads[0].weights || !m->heads[0].weights->weights) && medusa_model_load(m, "synthetic:0") != 0)
        return nullptr;
    const uint64_t seed = synth_seed(m);
    fl_engine_t* e = host_engine_new(m->vocab_size, m->hidden_size, 32, 0, m->num_heads, seed, gguf_of(m));
    if (!e) return nullptr;
    dequantized_tensor_t lm = {};
    unbind(m);
    if (synth_tensor(&lm, seed, FL_TENSOR_ID(3, 0, 1), m->vocab_size, m->hidden_size) != FL_OK ||
        fl_engine_load_linear(e, 3, 0, 1, lm.weights, lm.scales_f16, lm.rows, lm.cols) != FL_OK ||
        medusa_bind(e, m) != FL_OK || !fl_engine_ready(e)) {
        free(lm.weights);
        free(lm.scales_f16);
        fl_engine_destroy(e);
        return nullptr;
    }
    free(lm.weights);
    free(lm.scales_f16);
    std::lock_guard<std::mutex> lk(g_bind_mu);
    g_host_eng[m] = e;
    return e;
}

// Sampling rule of a host-target decode (include/speculative.h): greedy
// when temperature <= 0, else the library's integer rule at top-p 1 with
// Philox key (seed 0, sequence 0).
struct HostRule {
    float T;
    bool greedy() const { return !(T > 0.0f); }
};

// The token at position `pos` from target logits `row`: greedy argmax, or a
// draw (purpose 2) at Philox step `step`.
static int host_pick(const HostRule& r, const float* row, int V, uint32_t step, int pos) {
    if (r.greedy()) return fl_host::argmax(row, V);
    std::vector<uint32_t> E;
    const uint64_t M = fl_host::weights(row, V, r.T, 1.0f, E);
    return fl_host::pick(E, M, fl_host::u24(0u, 0u, step, (uint32_t)pos, 2u));
}

// Sequential verification of drafts d[0..K) against a host target whose
// context ends just before `cur` (not yet fed): feeds cur, compares the
// target's token at the next position with d[0], feeds d[0] if accepted,
// and so on; a rejected draft is replaced by the target's token there, and
// after K accepted drafts the target's next token follows (rejection
// sampling with a greedy draft when sampling: d is kept with probability
// p(d), otherwise the token is drawn from p without d). Only tokens that end
// up in the output are ever fed. Appends the accepted drafts and the final
// token to `emit` (at most `room`); returns the number of accepted drafts.
static int host_verify(void* tm, void (*tf)(void*, const float*, float*, int), const HostRule& rule, int V, int cur,
                       int pos, const int* d, int K, uint32_t step, int room, std::vector<int>& emit) {
    std::vector<float> row(V);
    std::vector<uint32_t> E;
    int a = 0;
    for (int j = 0; j <= K && (int)emit.size() < room; j++) {
        const float f = (float)(j == 0 ? cur : d[j - 1]);
        tf(tm, &f, row.data(), 1);
        const int p = pos + 1 + j;  // position of the token being decided
        if (j == K) {
            emit.push_back(host_pick(rule, row.data(), V, step, p));
            break;
        }
        int next;
        bool keep;
        if (rule.greedy()) {
            next = fl_host::argmax(row.data(), V);
            keep = next == d[j];
        } else {
            const uint64_t M = fl_host::weights(row.data(), V, rule.T, 1.0f, E);
            const uint32_t U = fl_host::u24(0u, 0u, step, (uint32_t)p, 1u);
            keep = (unsigned __int128)U * M < ((unsigned __int128)E[d[j]] << 24);
            next = d[j];
            if (!keep) {
                const uint64_t rest = M - E[d[j]];
                const uint32_t U2 = fl_host::u24(0u, 0u, step, (uint32_t)p, 2u);
                next = rest > 0 ? fl_host::pick(E, rest, U2, d[j]) : fl_host::pick(E, M, U2);
            }
        }
        emit.push_back(next);
        if (!keep) break;
        a++;
    }
    return a;
}

// speculative_generate with a host target_forward (see include/speculative.h).
static int host_spec_generate(draft_model_t* dm, void* tm, void (*tf)(void*, const float*, float*, int),
                              const float* prompt_hidden, int P, int* out, int n, const speculative_config_t* cfg) {
    const int V = dm->vocab_size;
    const int K = std::min(std::max(cfg->num_draft_tokens, 1), 7);
    if (P + n + K + 2 > kHostCtx) {
        set_error(FL_E_INVAL, "speculative_generate: prompt plus output longer than the host-target context");
        return -1;
    }
    fl_engine_t* e = host_draft_engine(dm);
    if (!e) return -1;
    const HostRule rule{cfg->temperature};
    std::vector<int> seq(P);
    std::vector<float> in(P);
    for (int i = 0; i < P; i++) {
        const int t = (int)prompt_hidden[i];
        seq[i] = t >= 0 && t < V ? t : 0;  // inference.c:420-426: ids outside the vocabulary embed as 0
        in[i] = (float)seq[i];
    }
    std::vector<float> lg((size_t)P * V);
    tf(tm, in.data(), lg.data(), P);
    int produced = 0;
    out[produced++] = seq.emplace_back(host_pick(rule, lg.data() + (size_t)(P - 1) * V, V, 0xFFFFFFFFu, P));
    std::vector<int> d(K), emit;
    int draft_len = 0;
    for (uint32_t step = 0; produced < n; step++) {
        const int L = (int)seq.size();
        if (fl_engine_draft_lm(e, seq.data() + draft_len, L - draft_len, draft_len, K, d.data()) != FL_OK) return -1;
        emit.clear();
        const int a = host_verify(tm, tf, rule, V, seq.back(), L - 1, d.data(), K, step, n - produced, emit);
        for (int t : emit) out[produced++] = seq.emplace_back(t);
        draft_len = L + std::min(a, K - 1);
    }
    return produced;
}

// speculative_decode_step with a host target_forward: the draft's cache
// holds the positions before `cache->cache_len`, where current_token goes.
static int host_spec_step(draft_model_t* dm, draft_kv_cache_t* cache, void* tm,
                          void (*tf)(void*, const float*, float*, int), int cur, int* out, int* num_out,
                          const speculative_config_t* cfg) {
    const int V = dm->vocab_size;
    const int K = std::min(std::max(cfg->num_draft_tokens, 1), 7);
    const int pos = cache->cache_len;
    if (cur < 0 || cur >= V || pos + K + 2 > kHostCtx) return -1;
    fl_engine_t* e = host_draft_engine(dm);
    if (!e) return -1;
    std::vector<int> d(K), emit;
    if (fl_engine_draft_lm(e, &cur, 1, pos, K, d.data()) != FL_OK) return -1;
    CacheImpl* ci = (CacheImpl*)cache;
    const int a = host_verify(tm, tf, HostRule{cfg->temperature}, V, cur, pos, d.data(), K, (uint32_t)ci->steps,
                              K + 1, emit);
    ci->steps++;
    int dummy = 0;
    // keep the draft cache contiguous up to the last accepted draft
    if (a == K && fl_engine_draft_lm(e, &d[K - 1], 1, pos + K, 1, &dummy) != FL_OK) return -1;
    cache->cache_len = pos + a + 1;
    for (size_t i = 0; i < emit.size(); i++) out[i] = emit[i];
    *num_out = (int)emit.size();
    return *num_out;
}

FL_API int fl_engine_bind_medusa(fl_engine_t* e, void* m) {
    if (!e || !m) return set_error(FL_E_INVAL, "bind_medusa: NULL");
    return medusa_bind(e, (medusa_model_t*)m);
}

int medusa_bind(fl_engine_t* e, medusa_model_t* m) {
    if (bound(m) == e) return FL_OK;
    for (int h = 0; h < m->num_heads; h++) {
        const dequantized_tensor_t* t = m->heads[h].weights;
        if (!t || !t->weights) return set_error(FL_E_STATE, "medusa head without weights");
        if (t->scale_block != 32 || !t->scales_f16)
            return set_error(FL_E_UNSUPPORTED, "medusa heads must be in block mode (scale_block 32)");
        if (m->heads[h].bias) return set_error(FL_E_UNSUPPORTED, "medusa head bias is not supported");
        FL_CHECK(fl_engine_load_linear(e, 2, h, 0, t->weights, t->scales_f16, t->rows, t->cols));
    }
    bind(m, e);
    return FL_OK;
}

FL_API int fl_medusa_set_tree(medusa_model_t* m, const int* topk, int n, int max_nodes) {
    if (!m || !topk || n <= 0 || max_nodes < 2) return set_error(FL_E_INVAL, "fl_medusa_set_tree: bad arguments");
    std::lock_guard<std::mutex> lk(g_bind_mu);
    MedusaTree& t = g_med_tree[m];
    t.topk.assign(topk, topk + n);
    t.max_nodes = max_nodes;
    return FL_OK;
}

// ------------------------------------------------------------------ speculative.h

FL_API draft_model_t* draft_model_create(int num_layers, int hidden_size, int intermediate_size, int vocab_size) {
    if (num_layers <= 0 || hidden_size <= 0 || intermediate_size <= 0 || vocab_size <= 0) return nullptr;
    draft_model_t* m = (draft_model_t*)calloc(1, sizeof(draft_model_t));
    if (!m) return nullptr;
    m->num_layers = num_layers;
    m->hidden_size = hidden_size;
    m->intermediate_size = intermediate_size;
    m->vocab_size = vocab_size;
    dequantized_tensor_t** arrs[7] = {&m->w_q_proj, &m->w_k_proj, &m->w_v_proj, &m->w_o_proj,
                                      &m->w_gate, &m->w_up, &m->w_down};
    for (auto a : arrs) {
        *a = (dequantized_tensor_t*)calloc(num_layers, sizeof(dequantized_tensor_t));
        if (!*a) { draft_model_free(m); return nullptr; }
    }
    m->w_lm_head = (dequantized_tensor_t*)calloc(1, sizeof(dequantized_tensor_t));
    if (!m->w_lm_head) { draft_model_free(m); return nullptr; }
    return m;
}

FL_API int draft_model_load(draft_model_t* m, const char* path) {
    uint64_t seed = 0;
    if (!m || !path) return -1;
    if (!parse_synthetic(path, &seed)) {
        if (gguf_load_draft(m, path) != FL_OK) return -1;
        std::lock_guard<std::mutex> lk(g_bind_mu);
        g_gguf[m] = path;
        return 0;
    }
    const int d = m->hidden_size, F = m->intermediate_size;
    const int shapes[7][2] = {{d, d}, {d, d}, {d, d}, {d, d}, {F, d}, {F, d}, {d, F}};
    dequantized_tensor_t* arrs[7] = {m->w_q_proj, m->w_k_proj, m->w_v_proj, m->w_o_proj, m->w_gate, m->w_up, m->w_down};
    for (int l = 0; l < m->num_layers; l++)
        for (int p = 0; p < 7; p++)
            if (synth_tensor(&arrs[p][l], seed, FL_TENSOR_ID(1, l, p), shapes[p][0], shapes[p][1]) != FL_OK) return -1;
    if (synth_tensor(m->w_lm_head, seed, FL_TENSOR_ID(3, 0, 1), m->vocab_size, d) != FL_OK) return -1;
    std::lock_guard<std::mutex> lk(g_bind_mu);
    g_seed[m] = seed;
    return 0;
}

FL_API void draft_model_free(draft_model_t* m) {
    if (!m) return;
    unbind(m);
    host_engine_release(m);
    free_tensor_array(m->w_q_proj, m->num_layers);
    free_tensor_array(m->w_k_proj, m->num_layers);
    free_tensor_array(m->w_v_proj, m->num_layers);
    free_tensor_array(m->w_o_proj, m->num_layers);
    free_tensor_array(m->w_gate, m->num_layers);
    free_tensor_array(m->w_up, m->num_layers);
    free_tensor_array(m->w_down, m->num_layers);
    free_tensor_array(m->w_lm_head, 1);
    free(m);
}

FL_API draft_kv_cache_t* draft_kv_cache_create(int max_len, int num_heads, int head_dim) {
    if (max_len <= 0 || num_heads <= 0 || head_dim <= 0) return nullptr;
    CacheImpl* c = (CacheImpl*)calloc(1, sizeof(CacheImpl));
    if (!c) return nullptr;
    c->pub.max_len = max_len;
    c->num_heads = num_heads;
    c->head_dim = head_dim;
    return &c->pub;
}

FL_API void draft_kv_cache_reset(draft_kv_cache_t* c) {
    if (c) c->cache_len = 0;
}

FL_API void draft_kv_cache_free(draft_kv_cache_t* c) { free(c); }

FL_API draft_tree_t* draft_tree_create(int max_tokens) {
    if (max_tokens <= 0) return nullptr;
    TreeImpl* t = (TreeImpl*)calloc(1, sizeof(TreeImpl));
    if (!t) return nullptr;
    t->pub.tokens = (int*)calloc(max_tokens, sizeof(int));
    t->pub.probs = (float*)calloc(max_tokens, sizeof(float));
    t->pub.max_tokens = max_tokens;
    if (!t->pub.tokens || !t->pub.probs) {
        free(t->pub.tokens);
        free(t->pub.probs);
        free(t);
        return nullptr;
    }
    return &t->pub;
}

FL_API void draft_tree_free(draft_tree_t* t) {
    if (!t) return;
    free(t->tokens);
    free(t->probs);
    free(t);
}

// Sets the vocabulary a tree's logits rows use (trees from draft_tree_create).
FL_API int fl_draft_tree_set_vocab(draft_tree_t* t, int vocab) {
    if (!t || vocab <= 0) return set_error(FL_E_INVAL, "tree/vocab");
    ((TreeImpl*)t)->vocab = vocab;
    return FL_OK;
}

FL_API int verify_tokens(const float* target_hidden, const draft_tree_t* tree, int* accepted_tokens,
                         int* num_accepted, const speculative_config_t* config) {
    if (!target_hidden || !tree || !accepted_tokens || !num_accepted || !config) return -1;
    const int V = ((const TreeImpl*)tree)->vocab;
    if (V <= 0) {
        set_error(FL_E_STATE, "verify_tokens: tree vocabulary unknown (draft_tokens or fl_draft_tree_set_vocab)");
        return -1;
    }
    if (config->temperature > 0.0f) {
        set_error(FL_E_UNSUPPORTED, "verify_tokens: host rejection sampling needs the draft distributions; "
                                    "use speculative_generate (or fl_engine_set_sampling)");
        return -1;
    }
    const int K = tree->num_tokens;
    const int cap = config->max_accepted < 0 ? K : (config->max_accepted < K ? config->max_accepted : K);
    auto argmax = [&](int r) {
        const float* l = target_hidden + (size_t)r * V;
        int bi = 0;
        for (int i = 1; i < V; i++)
            if (l[i] > l[bi]) bi = i;
        return bi;
    };
    int a = 0;
    while (a < cap && tree->tokens[a] == argmax(a)) {
        accepted_tokens[a] = tree->tokens[a];
        a++;
    }
    accepted_tokens[a] = argmax(a);
    *num_accepted = a;
    return a;
}

FL_API int draft_tokens(draft_model_t* model, draft_kv_cache_t* cache, const float* hidden_state, int current_token,
                        draft_tree_t* tree, const speculative_config_t* config) {
    if (!model || !cache || !hidden_state || !tree || !config) return -1;
    fl_engine_t* e = bound(model);
    if (!e) {
        set_error(FL_E_STATE, "draft_tokens: draft not bound to an engine (speculative_generate or fl_engine_bind_draft)");
        return -1;
    }
    const int K = config->num_draft_tokens < tree->max_tokens ? config->num_draft_tokens : tree->max_tokens;
    if (K <= 0) return -1;
    if (fl_engine_draft_chain(e, hidden_state, current_token, cache->cache_len, K, tree->tokens, tree->probs) != FL_OK)
        return -1;
    tree->num_tokens = K;
    ((TreeImpl*)tree)->vocab = model->vocab_size;
    cache->cache_len += 1;
    return K;
}

FL_API int fl_engine_bind_draft(fl_engine_t* e, draft_model_t* dm) {
    if (!e || !dm) return set_error(FL_E_INVAL, "bind_draft: NULL");
    // Weights go to HBM once per (engine, draft) pair; later calls reuse them.
    if (bound(dm) == e && fl_engine_draft_bound(e, dm)) return FL_OK;
    FL_CHECK(load_draft_into(e, dm));
    bind(dm, e);
    fl_engine_note_draft(e, dm);
    return FL_OK;
}

FL_API int speculative_decode_step(draft_model_t* draft, draft_kv_cache_t* draft_cache, void* target_model,
                                   void (*target_forward)(void*, const float*, float*, int),
                                   const float* current_hidden, int current_token, int* output_tokens,
                                   int* num_output, const speculative_config_t* config) {
    if (!draft || !draft_cache || !target_forward || !output_tokens || !num_output || !config) return -1;
    if (target_forward != fl_cuda_target_forward)
        return host_spec_step(draft, draft_cache, target_model, target_forward, current_token, output_tokens,
                              num_output, config);
    if (!target_model || !current_hidden) return -1;
    fl_engine_t* e = (fl_engine_t*)target_model;
    if (!bound(draft) && fl_engine_bind_draft(e, draft) != FL_OK) return -1;
    const int K = config->num_draft_tokens;
    if (K <= 0 || K > 7) return -1;
    draft_tree_t* tree = draft_tree_create(K);
    if (!tree) return -1;
    const int pos0 = fl_engine_position(e);
    int rc = draft_tokens(draft, draft_cache, current_hidden, current_token, tree, config);
    if (rc < 0) { draft_tree_free(tree); return -1; }
    std::vector<float> in(K + 1), logits((size_t)(K + 1) * draft->vocab_size);
    in[0] = (float)current_token;
    for (int i = 0; i < K; i++) in[i + 1] = (float)tree->tokens[i];
    target_forward(target_model, in.data(), logits.data(), K + 1);
    if (fl_engine_position(e) != pos0 + K + 1) { draft_tree_free(tree); return -1; }
    speculative_config_t greedy = *config;
    greedy.temperature = 0.0f;
    int a = 0;
    rc = verify_tokens(logits.data(), tree, output_tokens, &a, &greedy);
    draft_tree_free(tree);
    if (rc < 0) return -1;
    // keep the verified prefix in the base cache; the bonus token is next
    if (fl_engine_set_position(e, pos0 + a + 1) != FL_OK) return -1;
    draft_cache->cache_len = pos0 + a + 1;
    *num_output = a + 1;
    return a + 1;
}

FL_API int speculative_generate(draft_model_t* draft, void* target_model,
                                void (*target_forward)(void*, const float*, float*, int), const float* prompt_hidden,
                                int prompt_len, int* output_tokens, int num_tokens, const speculative_config_t* config) {
    if (!draft || !target_forward || !prompt_hidden || !output_tokens || !config || prompt_len <= 0 || num_tokens <= 0)
        return -1;
    if (target_forward != fl_cuda_target_forward)
        return host_spec_generate(draft, target_model, target_forward, prompt_hidden, prompt_len, output_tokens,
                                  num_tokens, config);
    if (!target_model) return -1;
    fl_engine_t* e = (fl_engine_t*)target_model;
    if (fl_engine_bind_draft(e, draft) != FL_OK) return -1;
    // temperature > 0: rejection sampling with the engine's top_p and Philox
    // key (fl_engine_set_sampling); otherwise greedy
    float t0 = 0.0f, top_p = 1.0f;
    unsigned seed = 0, seq_id = 0;
    if (fl_engine_get_sampling(e, &t0, &top_p, &seed, &seq_id) != FL_OK ||
        fl_engine_set_sampling(e, config->temperature > 0.0f ? config->temperature : 0.0f, top_p, seed, seq_id) !=
            FL_OK)
        return -1;
    std::vector<int> prompt(prompt_len);
    for (int i = 0; i < prompt_len; i++) prompt[i] = (int)prompt_hidden[i];
    const int K = config->num_draft_tokens;
    if (fl_engine_spec_generate(e, prompt.data(), prompt_len, num_tokens, K, config->max_accepted, output_tokens,
                                nullptr, nullptr) != FL_OK)
        return -1;
    return num_tokens;
}

// ------------------------------------------------------------------ medusa.h

FL_API medusa_model_t* medusa_model_create(int num_heads, int hidden_size, int vocab_size) {
    if (num_heads <= 0 || hidden_size <= 0 || vocab_size <= 0) return nullptr;
    medusa_model_t* m = (medusa_model_t*)calloc(1, sizeof(medusa_model_t));
    if (!m) return nullptr;
    m->heads = (medusa_head_t*)calloc(num_heads, sizeof(medusa_head_t));
    if (!m->heads) { free(m); return nullptr; }
    m->num_heads = num_heads;
    m->hidden_size = hidden_size;
    m->vocab_size = vocab_size;
    for (int h = 0; h < num_heads; h++) {
        m->heads[h].head_id = h;
        m->heads[h].hidden_size = hidden_size;
        m->heads[h].vocab_size = vocab_size;
        m->heads[h].weights = (dequantized_tensor_t*)calloc(1, sizeof(dequantized_tensor_t));
    }
    return m;
}

FL_API int medusa_model_load(medusa_model_t* m, const char* path) {
    uint64_t seed = 0;
    if (!m || !path) return -1;
    if (!parse_synthetic(path, &seed)) {
        if (gguf_load_medusa(m, path) != FL_OK) return -1;
        std::lock_guard<std::mutex> lk(g_bind_mu);
        g_gguf[m] = path;
        return 0;
    }
    for (int h = 0; h < m->num_heads; h++)
        if (!m->heads[h].weights ||
            synth_tensor(m->heads[h].weights, seed, FL_TENSOR_ID(2, h, 0), m->hidden_size, m->hidden_size) != FL_OK)
            return -1;
    std::lock_guard<std::mutex> lk(g_bind_mu);
    g_seed[m] = seed;
    return 0;
}

FL_API void medusa_model_free(medusa_model_t* m) {
    if (!m) return;
    unbind(m);
    host_engine_release(m);
    {
        std::lock_guard<std::mutex> lk(g_bind_mu);
        g_med_tree.erase(m);
    }
    for (int h = 0; h < m->num_heads; h++) {
        free_tensor_array(m->heads[h].weights, 1);
        free(m->heads[h].bias);
    }
    free(m->heads);
    free(m);
}

FL_API medusa_tree_t* medusa_tree_create(int max_candidates) {
    if (max_candidates <= 0) return nullptr;
    medusa_tree_t* t = (medusa_tree_t*)calloc(1, sizeof(medusa_tree_t));
    if (!t) return nullptr;
    t->tokens = (int*)calloc(max_candidates, sizeof(int));
    t->probs = (float*)calloc(max_candidates, sizeof(float));
    t->parent_indices = (int*)calloc(max_candidates, sizeof(int));
    t->positions = (int*)calloc(max_candidates, sizeof(int));
    t->max_candidates = max_candidates;
    if (!t->tokens || !t->probs || !t->parent_indices || !t->positions) {
        medusa_tree_free(t);
        return nullptr;
    }
    return t;
}

FL_API void medusa_tree_free(medusa_tree_t* t) {
    if (!t) return;
    free(t->tokens);
    free(t->probs);
    free(t->parent_indices);
    free(t->positions);
    free(t);
}

// Draft + Medusa (reference medusa.h:210-229): draft_model is a draft_model_t
// bound to the engine, draft_forward fl_cuda_target_forward (the draft runs
// inside the engine) or NULL, target_model the engine with its base_forward
// fl_cuda_base_forward; the draft chain length is config->num_heads (at most
// 7), the Medusa heads and tree settings as for medusa_generate. Greedy only.
FL_API int speculative_medusa_generate(void* draft_model, void (*draft_forward)(void*, const float*, float*, int),
                                       medusa_model_t* medusa, void* target_model,
                                       void (*target_forward)(void*, const int*, int, float*, int),
                                       const float* prompt_hidden, int prompt_len, int* output_tokens, int num_tokens,
                                       const medusa_config_t* config) {
    if (!draft_model || !medusa || !target_model || !prompt_hidden || prompt_len <= 0 || !output_tokens ||
        num_tokens <= 0 || !config)
        return -1;
    if (target_forward != fl_cuda_base_forward || (draft_forward && draft_forward != fl_cuda_target_forward)) {
        set_error(FL_E_UNSUPPORTED, "speculative_medusa_generate: the forwards must be fl_cuda_base_forward "
                                    "(target) and fl_cuda_target_forward or NULL (draft)");
        return -1;
    }
    if (config->temperature > 0.0f) {
        set_error(FL_E_UNSUPPORTED, "speculative_medusa_generate: only greedy acceptance (temperature <= 0)");
        return -1;
    }
    fl_engine_t* e = (fl_engine_t*)target_model;
    if (fl_engine_bind_draft(e, (draft_model_t*)draft_model) != FL_OK || medusa_bind(e, medusa) != FL_OK) return -1;
    std::vector<int> topk;
    int max_nodes = 64;
    const int H = medusa_tree_settings(medusa, config, topk, &max_nodes);
    if (H <= 0) return -1;
    const int K = std::min(std::max(config->num_heads, 1), 7);
    std::vector<int> prompt(prompt_len);
    for (int i = 0; i < prompt_len; i++) prompt[i] = (int)prompt_hidden[i];
    if (fl_engine_spec_medusa_generate(e, prompt.data(), prompt_len, num_tokens, K, topk.data(), H,
                                       std::max(max_nodes, K + 2), output_tokens, nullptr, nullptr) != FL_OK)
        return -1;
    return num_tokens;
}
