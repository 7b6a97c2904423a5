// GGUF files with Q4_0 weights (gguf_loader.c:147-161, 574-671 restated with
// the real 18-byte Q4_0 block: fp16 d + 16 bytes of nibbles, low nibbles =
// elements 0..15, high nibbles = 16..31): each tensor is pre-dequantized
// once to INT8 q-8 in [-8, 7] plus its fp16 block scales (fl_q4_0_to_i8) and
// uploaded to HBM. Host code.
//
// Names follow the reference loader (gguf_loader.c:307-342): token_embd,
// output (LM head), blk.<l>.attn_q / attn_k / attn_v / attn_output (or a fused
// attn_qkv of q_dim + 2 kv_dim rows), ffn_gate / ffn_up / ffn_down (or an
// ffn_up of 2 ffn rows, gate rows first, as Phi-3 stores gate_up_proj).
// Norm weights are not applied (the engine's RMSNorm has unit weights, as
// in the configurations served); tensors other than Q4_0 / F32 / F16 and
// unknown names are skipped.
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <string>
#include <vector>

#include "fl_common.cuh"
#include "fl_runtime.h"
#include "medusa.h"
#include "speculative.h"

using namespace fl;

namespace {

constexpr uint32_t kGgufMagic = 0x46554747u;  // "GGUF"
constexpr uint32_t kTypeF32 = 0, kTypeF16 = 1, kTypeQ4_0 = 2;

struct GTensor {
    std::string name;
    std::vector<uint64_t> dims;  // ne0 (innermost, columns) first
    uint32_t type = 0;
    uint64_t offset = 0;
};

struct GFile {
    std::vector<uint8_t> buf;
    std::vector<GTensor> tensors;
    size_t data = 0;  // start of the tensor data

    const uint8_t* at(const GTensor& t) const { return buf.data() + data + t.offset; }
};

struct Reader {
    const std::vector<uint8_t>& b;
    size_t p = 0;
    bool ok = true;
    template <typename T>
    T get() {
        T v{};
        if (p + sizeof(T) > b.size()) {
            ok = false;
            return v;
        }
        memcpy(&v, b.data() + p, sizeof(T));
        p += sizeof(T);
        return v;
    }
    std::string str() {
        const uint64_t n = get<uint64_t>();
        if (!ok || n > b.size() - p) {
            ok = false;
            return {};
        }
        std::string s((const char*)b.data() + p, n);
        p += n;
        return s;
    }
    // Skips one metadata value of GGUF type t (reading general.alignment on the way).
    void skip(uint32_t t, uint64_t* as_u64) {
        static const int sz[13] = {1, 1, 2, 2, 4, 4, 4, 1, 0, 0, 8, 8, 8};
        if (t == 8) {
            str();
        } else if (t == 9) {
            const uint32_t et = get<uint32_t>();
            const uint64_t n = get<uint64_t>();
            for (uint64_t i = 0; i < n && ok; i++) skip(et, nullptr);
        } else if (t < 13) {
            uint64_t v = 0;
            if (p + sz[t] > b.size()) {
                ok = false;
                return;
            }
            memcpy(&v, b.data() + p, sz[t]);
            p += sz[t];
            if (as_u64) *as_u64 = v;
        } else {
            ok = false;
        }
    }
};

int read_gguf(const char* path, GFile& f) {
    FILE* fp = fopen(path, "rb");
    if (!fp) return set_error(FL_E_INVAL, std::string("gguf: cannot open ") + path);
    fseek(fp, 0, SEEK_END);
    const long n = ftell(fp);
    fseek(fp, 0, SEEK_SET);
    f.buf.resize(n > 0 ? (size_t)n : 0);
    const size_t got = n > 0 ? fread(f.buf.data(), 1, (size_t)n, fp) : 0;
    fclose(fp);
    if (got != f.buf.size()) return set_error(FL_E_INVAL, "gguf: short read");
    Reader r{f.buf};
    if (r.get<uint32_t>() != kGgufMagic) return set_error(FL_E_INVAL, "gguf: bad magic");
    const uint32_t version = r.get<uint32_t>();
    if (version < 2 || version > 3) return set_error(FL_E_UNSUPPORTED, "gguf: version must be 2 or 3");
    const uint64_t nt = r.get<uint64_t>(), nkv = r.get<uint64_t>();
    uint64_t align = 32;
    for (uint64_t i = 0; i < nkv && r.ok; i++) {
        const std::string key = r.str();
        const uint32_t t = r.get<uint32_t>();
        uint64_t v = 0;
        r.skip(t, &v);
        if (key == "general.alignment" && v > 0) align = v;
    }
    for (uint64_t i = 0; i < nt && r.ok; i++) {
        GTensor g;
        g.name = r.str();
        const uint32_t nd = r.get<uint32_t>();
        if (nd == 0 || nd > 4) r.ok = false;
        for (uint32_t k = 0; k < nd && r.ok; k++) g.dims.push_back(r.get<uint64_t>());
        g.type = r.get<uint32_t>();
        g.offset = r.get<uint64_t>();
        f.tensors.push_back(g);
    }
    if (!r.ok) return set_error(FL_E_INVAL, "gguf: truncated header");
    f.data = (r.p + align - 1) / align * align;
    for (const GTensor& g : f.tensors) {
        uint64_t elems = 1;
        for (uint64_t d : g.dims) elems *= d;
        const uint64_t bytes = g.type == kTypeQ4_0 ? elems / 32 * 18 : g.type == kTypeF16 ? elems * 2 : elems * 4;
        if (f.data + g.offset + bytes > f.buf.size()) return set_error(FL_E_INVAL, "gguf: tensor data past the end");
    }
    return FL_OK;
}

// Rows x cols of a 2-D Q4_0 tensor as INT8 q-8 + fp16 scales.
int q4_rows(const GFile& f, const GTensor& g, std::vector<int8_t>& w, std::vector<uint16_t>& d, int* rows,
            int* cols) {
    if (g.type != kTypeQ4_0 || g.dims.size() != 2 || g.dims[0] % 32)
        return set_error(FL_E_UNSUPPORTED, "gguf: " + g.name + " is not a 2-D Q4_0 tensor");
    *cols = (int)g.dims[0];
    *rows = (int)g.dims[1];
    w.resize((size_t)*rows * *cols);
    d.resize((size_t)*rows * (*cols / 32));
    return fl_q4_0_to_i8(reinterpret_cast<const block_q4_0_gguf*>(f.at(g)), *rows, *cols, w.data(), d.data());
}

// Layer index and projection (0..6 = q k v o gate up down; 7 fused qkv;
// -2 embedding; -3 LM head) of a tensor name, -1 if unused. A fused gate+up
// arrives as ffn_up (5) with twice the ffn rows.
int classify(const std::string& n, int* layer) {
    *layer = -1;
    auto has = [&](const char* s) { return n.find(s) != std::string::npos; };
    if (has(".bias") || has("norm")) return -1;
    if (has("token_embd") || has("tok_embeddings")) return -2;
    const size_t b = n.find("blk.");
    if (b == std::string::npos) return (has("output.weight") || has("lm_head")) ? -3 : -1;
    *layer = atoi(n.c_str() + b + 4);
    if (has("attn_qkv")) return 7;
    if (has("attn_q.") || has("q_proj")) return 0;
    if (has("attn_k.") || has("k_proj")) return 1;
    if (has("attn_v.") || has("v_proj")) return 2;
    if (has("attn_output") || has("o_proj")) return 3;
    if (has("ffn_gate") || has("gate_proj")) return 4;
    if (has("ffn_up") || has("up_proj")) return 5;
    if (has("ffn_down") || has("down_proj")) return 6;
    return -1;
}

// Calls put(layer, proj, w, d, rows, cols) for every 2-D Q4_0 weight of the
// file (fused tensors split into their parts) and emb(table, vocab, d) for the
// embedding. q_dim / kv_dim / ffn split fused tensors.
template <typename Put, typename Emb>
int walk(const GFile& f, int q_dim, int kv_dim, int ffn, Put put, Emb emb) {
    std::vector<int8_t> w;
    std::vector<uint16_t> d;
    for (const GTensor& g : f.tensors) {
        int layer = -1;
        const int k = classify(g.name, &layer);
        if (k == -1) continue;
        if (k == -2) {
            if (g.dims.size() != 2) return set_error(FL_E_UNSUPPORTED, "gguf: embedding must be 2-D");
            const int cols = (int)g.dims[0], rows = (int)g.dims[1];
            std::vector<float> tab((size_t)rows * cols);
            if (g.type == kTypeF32) {
                memcpy(tab.data(), f.at(g), tab.size() * 4);
            } else if (g.type == kTypeF16) {
                const uint16_t* h = reinterpret_cast<const uint16_t*>(f.at(g));
                for (size_t i = 0; i < tab.size(); i++) tab[i] = __half2float(__ushort_as_half(h[i]));
            } else if (g.type == kTypeQ4_0) {
                int r = 0, c = 0;
                FL_CHECK(q4_rows(f, g, w, d, &r, &c));
                for (size_t i = 0; i < tab.size(); i++)
                    tab[i] = (float)w[i] * __half2float(__ushort_as_half(d[i / 32]));  // (q-8)*d, gguf_loader.c:147-161
            } else {
                return set_error(FL_E_UNSUPPORTED, "gguf: embedding type");
            }
            FL_CHECK(emb(tab.data(), rows, cols));
            continue;
        }
        if (g.type != kTypeQ4_0) continue;
        int rows = 0, cols = 0;
        FL_CHECK(q4_rows(f, g, w, d, &rows, &cols));
        const size_t nb = cols / 32;
        if (k == -3) {
            FL_CHECK(put(-1, -3, w.data(), d.data(), rows, cols));
        } else if (k == 7) {
            if (rows != q_dim + 2 * kv_dim) return set_error(FL_E_INVAL, "gguf: " + g.name + " rows != q + 2 kv");
            const int off[3] = {0, q_dim, q_dim + kv_dim}, cnt[3] = {q_dim, kv_dim, kv_dim};
            for (int p = 0; p < 3; p++)
                FL_CHECK(put(layer, p, w.data() + (size_t)off[p] * cols, d.data() + (size_t)off[p] * nb, cnt[p], cols));
        } else if (k == 5 && rows == 2 * ffn) {
            FL_CHECK(put(layer, 4, w.data(), d.data(), ffn, cols));
            FL_CHECK(put(layer, 5, w.data() + (size_t)ffn * cols, d.data() + (size_t)ffn * nb, ffn, cols));
        } else {
            FL_CHECK(put(layer, k, w.data(), d.data(), rows, cols));
        }
    }
    return FL_OK;
}

}  // namespace

// The base model (blk.* -> stack 0), LM head and embedding of a GGUF Q4_0
// file into an engine created with matching dimensions.
FL_API int fl_engine_load_gguf(fl_engine_t* e, int stack, const char* path) {
    if (!e || !path || (stack != 0 && stack != 1)) return set_error(FL_E_INVAL, "load_gguf: bad arguments");
    GFile f;
    FL_CHECK(read_gguf(path, f));
    int cfg[4];  // hidden, q_dim, kv_dim, ffn of the engine
    FL_CHECK(fl_engine_dims(e, cfg));
    return walk(
        f, cfg[1], cfg[2], cfg[3],
        [&](int layer, int proj, const int8_t* w, const uint16_t* d, int rows, int cols) {
            if (proj == -3) return fl_engine_load_linear(e, 3, 0, 1, w, d, rows, cols);
            return fl_engine_load_linear(e, stack, layer, proj, w, d, rows, cols);
        },
        [&](const float* tab, int rows, int cols) {
            if (cols != cfg[0]) return set_error(FL_E_INVAL, "gguf: embedding width != hidden size");
            return fl_engine_load_embedding(e, tab);
        });
}

// draft_model_load / medusa_model_load with a GGUF path: the tensors into
// the model's host dequantized_tensor_t arrays (block mode, uploaded when
// the model is bound to an engine).
int gguf_fill_tensor(dequantized_tensor_t* t, const int8_t* w, const uint16_t* d, int rows, int cols) {
    release_tensor(t);
    free(t->weights);
    free(t->scales);
    free(t->scales_f16);
    t->weights = (int8_t*)malloc((size_t)rows * cols);
    t->scales_f16 = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)rows * (cols / 32));
    t->scales = nullptr;
    if (!t->weights || !t->scales_f16) return set_error(FL_E_NOMEM, "gguf: host allocation");
    memcpy(t->weights, w, (size_t)rows * cols);
    memcpy(t->scales_f16, d, sizeof(uint16_t) * (size_t)rows * (cols / 32));
    t->rows = rows;
    t->cols = cols;
    t->original_bits = 4;
    t->scale_block = 32;
    return FL_OK;
}

int gguf_load_draft(draft_model_t* m, const char* path) {
    GFile f;
    FL_CHECK(read_gguf(path, f));
    dequantized_tensor_t* arrs[7] = {m->w_q_proj, m->w_k_proj, m->w_v_proj, m->w_o_proj, m->w_gate, m->w_up, m->w_down};
    int got = 0;
    // the draft's own attention widths come from its q / k / v tensors; a
    // fused qkv is split as multi-head (q = k = v = hidden)
    const int d = m->hidden_size;
    FL_CHECK(walk(
        f, d, d, m->intermediate_size,
        [&](int layer, int proj, const int8_t* w, const uint16_t* s, int rows, int cols) {
            if (proj == -3) return gguf_fill_tensor(m->w_lm_head, w, s, rows, cols);
            if (layer < 0 || layer >= m->num_layers) return set_error(FL_E_INVAL, "gguf: draft layer out of range");
            got++;
            return gguf_fill_tensor(&arrs[proj][layer], w, s, rows, cols);
        },
        [&](const float*, int, int) { return FL_OK; }));
    if (got != 7 * m->num_layers) return set_error(FL_E_INVAL, "gguf: the file does not hold every draft weight");
    return FL_OK;
}

int gguf_load_medusa(medusa_model_t* m, const char* path) {
    GFile f;
    FL_CHECK(read_gguf(path, f));
    // Medusa heads: "medusa.<h>.weight" (or "medusa_head.<h>...") [hidden, hidden]
    std::vector<int8_t> w;
    std::vector<uint16_t> d;
    int got = 0;
    for (const GTensor& g : f.tensors) {
        const size_t p = g.name.find("medusa");
        if (p == std::string::npos || g.name.find(".bias") != std::string::npos) continue;
        const size_t dot = g.name.find('.', p);
        if (dot == std::string::npos) continue;
        const int h = atoi(g.name.c_str() + dot + 1);
        if (h < 0 || h >= m->num_heads) continue;
        int rows = 0, cols = 0;
        FL_CHECK(q4_rows(f, g, w, d, &rows, &cols));
        if (rows != m->hidden_size || cols != m->hidden_size) return set_error(FL_E_INVAL, "gguf: medusa head shape");
        FL_CHECK(gguf_fill_tensor(m->heads[h].weights, w.data(), d.data(), rows, cols));
        got++;
    }
    if (got != m->num_heads) return set_error(FL_E_INVAL, "gguf: the file does not hold every Medusa head");
    return FL_OK;
}

// The embedding table of a GGUF file ([vocab, hidden] f32), for models loaded
// from one (the host-target engines of api_spec.cu).
int gguf_load_embedding(const char* path, int vocab, int hidden, std::vector<float>& out) {
    GFile f;
    FL_CHECK(read_gguf(path, f));
    bool found = false;
    FL_CHECK(walk(
        f, hidden, hidden, 1 << 30, [&](int, int, const int8_t*, const uint16_t*, int, int) { return FL_OK; },
        [&](const float* tab, int rows, int cols) {
            if (rows != vocab || cols != hidden) return set_error(FL_E_INVAL, "gguf: embedding shape");
            out.assign(tab, tab + (size_t)rows * cols);
            found = true;
            return FL_OK;
        }));
    return found ? FL_OK : set_error(FL_E_INVAL, "gguf: no token_embd tensor");
}
