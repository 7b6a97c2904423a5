"""The whole decode path on the GPU against the oracle, on seeded small
models (seconds of oracle time) and one full-size Phi-3-mini case.

Tolerances (BASELINE parity rules): logits within 1e-2 relative to the row's
largest |logit|; token streams identical except from a position where the
oracle's top-2 logit margin is below 1e-2 of its top logit (a near-tie).
"""
import numpy as np
import pytest

import flb200
from _model import SMALL, SMALL_GQA, SMALL_V1, engine_cfg, load_engine, make_weights, prompt

pytestmark = pytest.mark.gpu

LOGIT_RTOL = 1e-2


def oracle_model(orc, dims, w, embed, draft_layers=1, n_medusa=0):
    import bind
    return bind.OracleModel(orc, dims, embed, w, draft_layers=draft_layers, n_medusa=n_medusa)


@pytest.fixture(scope="module", params=["mha", "gqa", "v1"])
def small(request, gpu, orc):
    dims = {"mha": SMALL, "gqa": SMALL_GQA, "v1": SMALL_V1}[request.param]
    w, embed = make_weights(gpu, dims, seed=21)
    eng = flb200.Engine(gpu, engine_cfg(dims, draft_layers=1))
    load_engine(eng, w, embed)
    om = oracle_model(orc, dims, w, embed)
    yield dims, eng, om, embed
    eng.close()


def assert_logits_close(got, want):
    scale = np.abs(want).max(axis=-1, keepdims=True)
    err = np.abs(got - want) / scale
    assert err.max() < LOGIT_RTOL, f"logit error {err.max():.3g} of row max"


def assert_stream_matches(got, want, margins):
    """Identical, or diverging only where the oracle's relative top-2 margin
    (top1 - top2) / |top1| is below the logit tolerance (a near-tie)."""
    got, want = np.asarray(got), np.asarray(want)
    diff = np.nonzero(got != want)[0]
    if diff.size == 0:
        return
    i = int(diff[0])
    assert margins[i] < LOGIT_RTOL, \
        f"streams diverge at {i}: gpu {got[i]} vs oracle {want[i]} (oracle margin {margins[i]:.4g})"


def test_stack_forward_prefill_and_chain(small):
    dims, eng, om, embed = small
    toks = prompt(1, 20, dims["vocab"])
    x0 = embed[toks]
    for stack in (0, 1):
        kv = om.kv(dims["layers"] if stack == 0 else 1, 64)
        want = om.stack_forward(stack, kv, x0, 0, np.arange(20))
        got, lg = eng.forward_rows(stack, x0, 0, np.arange(20))
        np.testing.assert_allclose(got, want, rtol=0, atol=1e-2 * np.abs(want).max())
        assert_logits_close(lg, om.lm_logits(want))
        # 5 more rows on top of the 20-position cache (a verify pass)
        x1 = embed[prompt(2, 5, dims["vocab"])]
        want1 = om.stack_forward(stack, kv, x1, 20, np.arange(20, 25))
        got1, lg1 = eng.forward_rows(stack, x1, 20, np.arange(20, 25))
        assert_logits_close(lg1, om.lm_logits(want1))


def test_tree_mask_attention(small):
    """A 7-node tree: rows see the prefix and their ancestors only; rotary
    positions are prefix + depth."""
    dims, eng, om, embed = small
    parent = [-1, 0, 0, 1, 1, 2, 3]
    depth = [0, 1, 1, 2, 2, 2, 3]
    M = len(parent)
    mask = np.zeros((M, M), np.uint8)
    for i in range(M):
        j = i
        while j >= 0:
            mask[i, j] = 1
            j = parent[j]
    base = 12
    kv = om.kv(dims["layers"], 64)
    pre = embed[prompt(3, base, dims["vocab"])]
    om.stack_forward(0, kv, pre, 0, np.arange(base))
    eng.forward_rows(0, pre, 0, np.arange(base), logits=False)
    x = embed[prompt(4, M, dims["vocab"])]
    pos = base + np.array(depth)
    want = om.stack_forward(0, kv, x, base, pos, mask)
    got, lg = eng.forward_rows(0, x, base, pos, mask)
    assert_logits_close(lg, om.lm_logits(want))


def test_greedy_stream(small):
    dims, eng, om, embed = small
    p = prompt(5, 16, dims["vocab"])
    want, margins = om.greedy(p, 24)
    assert_stream_matches(eng.greedy(p, 24), want, margins)


@pytest.mark.parametrize("k", [1, 4, 7])
def test_spec_stream_matches_oracle_and_greedy(small, k):
    """Speculative output equals the oracle's, and (greedy rule) equals plain
    greedy decoding of the base model."""
    dims, eng, om, embed = small
    p = prompt(6, 16, dims["vocab"])
    want, acc_want, margins = om.spec(p, 40, k)
    got, acc = eng.spec_generate(p, 40, k)
    assert_stream_matches(got, want, margins)
    if np.array_equal(got, want):
        assert np.array_equal(acc, acc_want), "acceptance histogram differs"
    g_want, _ = om.greedy(p, 40)
    assert np.array_equal(want, g_want), "oracle spec != oracle greedy"
    assert_stream_matches(got, eng.greedy(p, 40), margins)


def test_spec_decode_repeatable(small):
    """Decoding restarts from the saved post-prefill state every call."""
    dims, eng, om, embed = small
    p = prompt(7, 16, dims["vocab"])
    eng.spec_prefill(p, 4)
    a, ha = eng.spec_decode(33)
    b, hb = eng.spec_decode(33)
    c, hc = eng.spec_decode(7)
    assert np.array_equal(a, b) and np.array_equal(ha, hb)
    assert np.array_equal(c, a[:7])


@pytest.mark.parametrize("k", [1, 4])
def test_step_kernel_and_multi_kernel_match_oracle(small, gpu, monkeypatch, k):
    """The multi-kernel step graph (default engine) and the one-kernel
    tcgen05 step (engine created with FL_STEP_KERNEL=1: 128-byte panels, one
    persistent cooperative kernel per step) each reproduce the oracle's
    stream over several steps."""
    dims, eng, om, embed = small
    p = prompt(12, 16, dims["vocab"])
    want, acc_want, margins = om.spec(p, 33, k)
    got, acc = eng.spec_generate(p, 33, k)
    assert not eng.step_kernel()
    assert_stream_matches(got, want, margins)
    if np.array_equal(got, want):
        assert np.array_equal(acc, acc_want)
    w, embed2 = make_weights(gpu, dims, seed=21)
    monkeypatch.setenv("FL_STEP_KERNEL", "1")
    sk = flb200.Engine(gpu, engine_cfg(dims, draft_layers=1))
    load_engine(sk, w, embed2)
    got_sk, acc_sk = sk.spec_generate(p, 33, k)
    on_step_kernel = sk.step_kernel()
    sk.close()
    assert on_step_kernel, "the FL_STEP_KERNEL=1 engine should take the one-kernel step"
    assert_stream_matches(got_sk, want, margins)
    if np.array_equal(got_sk, want):
        assert np.array_equal(acc_sk, acc_want)


def test_max_accepted_cap(small):
    dims, eng, om, embed = small
    p = prompt(8, 16, dims["vocab"])
    want, acc_want, margins = om.spec(p, 30, 4, max_acc=1)
    got, acc = eng.spec_generate(p, 30, 4, max_acc=1)
    assert acc.max() <= 1
    assert_stream_matches(got, want, margins)


def test_speculative_generate_reference_api(gpu, orc):
    """speculative_generate() through the reference signature: draft_model_t
    loaded with draft_model_load("synthetic:SEED"), target = the engine,
    prompt ids passed as floats."""
    import ctypes as C
    dims = SMALL
    seed = 31
    w, embed = make_weights(gpu, dims, seed=seed)
    eng = flb200.Engine(gpu, engine_cfg(dims, draft_layers=1))
    load_engine(eng, {k: v for k, v in w.items() if k[0] != 1}, embed)
    dm = gpu.draft_model_create(1, dims["d"], dims["ffn"], dims["vocab"])
    assert gpu.draft_model_load(dm, b"synthetic:31") == 0
    cfg = flb200.SpecConfig(4, 0.0, 4)
    p = prompt(9, 12, dims["vocab"])
    ph = p.astype(np.float32)
    out = np.empty(20, np.int32)
    n = gpu.speculative_generate(dm, eng.h, C.cast(gpu.so.fl_cuda_target_forward, C.c_void_p), flb200.ptr(ph),
                                 len(p), flb200.ptr(out), 20, C.byref(cfg))
    assert n == 20, gpu.err()
    want, _, margins = oracle_model(orc, dims, w, embed).spec(p, 20, 4)
    assert_stream_matches(out, want, margins)
    gpu.draft_model_free(dm)
    eng.close()


def test_phi3_mini_full_size_spec(gpu, orc):
    """Full Phi-3-mini-shaped base (32 layers) + 4-layer draft, k = 4: the
    first 16 tokens after a 128-token prompt against the oracle."""
    dims = dict(vocab=32064, d=3072, ffn=8192, layers=32, heads=32, kv_heads=32, head_dim=96, theta=10000.0,
                eps=1e-5)
    w, embed = make_weights(gpu, dims, seed=1, draft_layers=4)
    eng = flb200.Engine(gpu, engine_cfg(dims, draft_layers=4, max_seq_len=512))
    load_engine(eng, w, embed)
    p = prompt(2024, 128, dims["vocab"])
    got, acc = eng.spec_generate(p, 16, 4)
    om = oracle_model(orc, dims, w, embed, draft_layers=4)
    want, acc_want, margins = om.spec(p, 16, 4)
    assert_stream_matches(got, want, margins)
    eng.close()


MEDUSA_TOPK = [10, 5, 3, 2]


def test_medusa_stream_matches_oracle(gpu, orc):
    """Medusa on the device (heads, top-k, tree, tree-masked verify, path
    acceptance, KV compaction) against the oracle; 16-token vocabulary so
    that multi-node paths are accepted and compacted."""
    dims = dict(SMALL, vocab=16)
    w, embed = make_weights(gpu, dims, seed=3, draft_layers=0, medusa_heads=4)
    eng = flb200.Engine(gpu, engine_cfg(dims, draft_layers=0, medusa_heads=4, max_seq_len=256))
    load_engine(eng, w, embed)
    p = prompt(4, 12, dims["vocab"])
    got, acc = eng.medusa_generate(p, 48, MEDUSA_TOPK, 64)
    eng.close()
    om = oracle_model(orc, dims, w, embed, draft_layers=0, n_medusa=4)
    want, acc_want, margins = om.medusa(p, 48, MEDUSA_TOPK, 64)
    assert_stream_matches(got, want, margins)
    assert acc.max() >= 2, f"no multi-node path accepted: {acc.tolist()}"
    g_want, _ = om.greedy(p, 48)
    assert np.array_equal(want, g_want)


def test_medusa_phi3_mini_shapes(gpu, orc):
    """Config-2 shapes: Phi-3-mini base, 4 heads of 3072 x 3072, top-k
    10/5/3/2, 64-node tree; the first 8 tokens after a 64-token prompt."""
    dims = dict(vocab=32064, d=3072, ffn=8192, layers=32, heads=32, kv_heads=32, head_dim=96, theta=10000.0,
                eps=1e-5)
    w, embed = make_weights(gpu, dims, seed=1, draft_layers=0, medusa_heads=4)
    eng = flb200.Engine(gpu, engine_cfg(dims, draft_layers=0, medusa_heads=4, max_seq_len=256))
    load_engine(eng, w, embed)
    p = prompt(2025, 64, dims["vocab"])
    got, acc = eng.medusa_generate(p, 8, MEDUSA_TOPK, 64)
    eng.close()
    om = oracle_model(orc, dims, w, embed, draft_layers=0, n_medusa=4)
    want, _, margins = om.medusa(p, 8, MEDUSA_TOPK, 64)
    assert_stream_matches(got, want, margins)


def test_medusa_generate_reference_api(gpu, orc):
    """medusa_generate() through the reference signature: heads from
    medusa_model_load("synthetic:SEED"), base = the engine with
    fl_cuda_base_forward, per-head top-k from fl_medusa_set_tree."""
    import ctypes as C
    dims = dict(SMALL, vocab=16)
    w, embed = make_weights(gpu, dims, seed=3, draft_layers=0, medusa_heads=4)
    eng = flb200.Engine(gpu, engine_cfg(dims, draft_layers=0, medusa_heads=4, max_seq_len=256))
    load_engine(eng, {k: v for k, v in w.items() if k[0] != 2}, embed)
    mm = gpu.medusa_model_create(4, dims["d"], dims["vocab"])
    assert gpu.medusa_model_load(mm, b"synthetic:3") == 0
    tk = np.array(MEDUSA_TOPK, np.int32)
    assert gpu.fl_medusa_set_tree(mm, flb200.ptr(tk), 4, 64) == 0
    cfg = flb200.MedusaConfig(4, 10, 0.0)
    p = prompt(4, 12, dims["vocab"])
    ph = p.astype(np.float32)
    out = np.empty(48, np.int32)
    n = gpu.medusa_generate(eng.h, C.cast(gpu.so.fl_cuda_base_forward, C.c_void_p), mm, flb200.ptr(ph), len(p),
                            flb200.ptr(out), 48, C.byref(cfg))
    assert n == 48, gpu.err()
    gpu.medusa_model_free(mm)
    eng.close()
    want, _, margins = oracle_model(orc, dims, w, embed, draft_layers=0, n_medusa=4).medusa(p, 48, MEDUSA_TOPK, 64)
    assert_stream_matches(out, want, margins)
