// Device passes for callers whose target / base model is their own host
// function (speculative_generate with a target_forward other than
// fl_cuda_target_forward, medusa_generate with a base_forward other than
// fl_cuda_base_forward). The engine then holds no base layers, only the
// draft stack or the Medusa heads with the embedding and LM head; the host
// orchestration and the acceptance rule are in api_host.cu.
#include "fl_engine_impl.h"

using namespace fl_eng;

// Draft tokens of a draft that runs as a plain language model over token
// embeddings (draft input at position i is E[t_i]; no base features exist
// for a host target): the nrows tokens rows_tok at positions pos0 ..
// pos0 + nrows - 1, which the draft cache does not hold yet, go through the
// draft stack in one pass; the last row's LM-head argmax is drafts[0]; each
// next draft token is fed back at the next position (K - 1 single-row
// passes). Afterwards the draft cache holds positions < pos0 + nrows + K - 1.
FL_API int fl_engine_draft_lm(fl_engine_t* e, const int* rows_tok, int nrows, int pos0, int K, int* drafts) {
    FL_CHECK(check_ready(e, true));
    if (!rows_tok || !drafts || nrows <= 0 || K <= 0 || pos0 < 0 || pos0 + nrows + K > e->R)
        return set_error(FL_E_INVAL, "draft_lm: bad arguments or context full");
    if (e->tp_size > 1) return set_error(FL_E_UNSUPPORTED, "draft_lm: not available on a tensor-parallel engine");
    const size_t d = e->d;
    FL_CHECK_CUDA(cudaMemcpyAsync(e->tok, rows_tok, sizeof(int) * nrows, cudaMemcpyHostToDevice, e->s));
    FL_CHECK_CUDA(launch_embed_rows(e->embed, e->Vg, e->tok, nullptr, 0, e->x, e->d, nrows, nullptr, nullptr, e->s,
                                    false));
    FL_CHECK(run_stack(e, e->draft, e->x, nrows, nullptr, e->iota + pos0, e->iota + pos0, nullptr, nullptr, false));
    FL_CHECK(run_lm(e, e->x + (size_t)(nrows - 1) * d, 1, nullptr, nullptr, false));
    FL_CHECK_CUDA(launch_argmax_rows(amax_keys(e), amax_nparts(e), 1, e->tok, nullptr, e->s));
    for (int j = 1; j < K; j++) {
        const int pos = pos0 + nrows - 1 + j;
        FL_CHECK_CUDA(cudaMemcpyAsync(drafts + j - 1, e->tok, sizeof(int), cudaMemcpyDeviceToHost, e->s));
        FL_CHECK_CUDA(launch_embed_rows(e->embed, e->Vg, e->tok, nullptr, 0, e->x_d, e->d, 1, nullptr, nullptr, e->s,
                                        false));
        FL_CHECK(run_stack(e, e->draft, e->x_d, 1, nullptr, e->iota + pos, e->iota + pos, nullptr, nullptr, false));
        FL_CHECK(run_lm(e, e->x_d, 1, nullptr, nullptr, false));
        FL_CHECK_CUDA(launch_argmax_rows(amax_keys(e), amax_nparts(e), 1, e->tok, nullptr, e->s));
    }
    FL_CHECK_CUDA(cudaMemcpyAsync(drafts + K - 1, e->tok, sizeof(int), cudaMemcpyDeviceToHost, e->s));
    FL_CHECK_CUDA(cudaStreamSynchronize(e->s));
    if (take_device_error() != 0) return set_error(FL_E_TIMEOUT, "draft_lm: a bounded device wait gave up");
    return FL_OK;
}

// LM-head argmax of one host feature row F [hidden] (final RMSNorm
// included): the greedy next token of a base model whose last-layer output
// is F (ties to the lowest index).
FL_API int fl_engine_lm_argmax(fl_engine_t* e, const float* F, int* tok) {
    FL_CHECK(check_ready(e, false));
    if (!F || !tok) return set_error(FL_E_INVAL, "lm_argmax: NULL");
    if (e->tp_size > 1) return set_error(FL_E_UNSUPPORTED, "lm_argmax: not available on a tensor-parallel engine");
    FL_CHECK_CUDA(cudaMemcpyAsync(e->x_d, F, sizeof(float) * e->d, cudaMemcpyHostToDevice, e->s));
    FL_CHECK(run_lm(e, e->x_d, 1, nullptr, nullptr, false));
    FL_CHECK_CUDA(launch_argmax_rows(amax_keys(e), amax_nparts(e), 1, e->tok, nullptr, e->s));
    FL_CHECK_CUDA(cudaMemcpyAsync(tok, e->tok, sizeof(int), cudaMemcpyDeviceToHost, e->s));
    FL_CHECK_CUDA(cudaStreamSynchronize(e->s));
    return FL_OK;
}

FL_API int fl_engine_lm_logits(fl_engine_t* e, const float* F, float* logits) {
    FL_CHECK(check_ready(e, false));
    if (!F || !logits) return set_error(FL_E_INVAL, "lm_logits: NULL");
    if (e->tp_size > 1) return set_error(FL_E_UNSUPPORTED, "lm_logits: not available on a tensor-parallel engine");
    FL_CHECK_CUDA(cudaMemcpyAsync(e->x_d, F, sizeof(float) * e->d, cudaMemcpyHostToDevice, e->s));
    FL_CHECK(run_lm(e, e->x_d, 1, nullptr, nullptr, false));
    FL_CHECK_CUDA(cudaMemcpyAsync(logits, e->logits, sizeof(float) * e->V, cudaMemcpyDeviceToHost, e->s));
    FL_CHECK_CUDA(cudaStreamSynchronize(e->s));
    return FL_OK;
}
