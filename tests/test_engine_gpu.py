"""The whole decode path on the GPU against the oracle, on seeded small
models (seconds of oracle time) and one full-size Phi-3-mini case.

Tolerances (the parity rules of the path): logits within 1e-2 relative to the row's
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


@pytest.mark.parametrize("dims", [SMALL, SMALL_GQA], ids=["mha", "gqa"])
def test_speculative_generate_reference_api(gpu, orc, dims):
    """speculative_generate() through the reference signature: draft_model_t
    loaded with draft_model_load("synthetic:SEED"), target = the engine,
    prompt ids passed as floats. With grouped-query heads the synthetic
    draft's host k/v tensors are [d, d] while the engine's draft layers take
    [kv_dim, d]: binding generates them again at the engine's shapes."""
    import ctypes as C
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


def device_tree(lib, root, topk, tok, prob, max_nodes, n):
    """fl_cuda_medusa_tree: (tokens, parents, depths, positions, mask)."""
    tk = np.ascontiguousarray(topk, np.int32)
    t = np.ascontiguousarray(tok, np.int32)
    pr = np.ascontiguousarray(prob, np.float32)
    outs = [np.full(max_nodes, -7, np.int32) for _ in range(4)]
    mask = np.zeros(max_nodes * max_nodes, np.uint8)
    M = lib.fl_cuda_medusa_tree(flb200.ptr(t), flb200.ptr(pr), flb200.ptr(tk), len(tk), t.shape[1], max_nodes, root,
                                n, *[flb200.ptr(o) for o in outs], flb200.ptr(mask))
    assert M > 0, lib.err()
    return [o[:M] for o in outs] + [mask[:M * M].reshape(M, M)]


@pytest.mark.parametrize("topk,max_nodes,ties", [([10, 5, 3, 2], 64, False), ([10, 5, 3, 2], 64, True),
                                                 ([4, 4, 4, 4], 256, True), ([3, 2], 5, False),
                                                 ([8, 8, 8], 200, False)])
def test_device_tree_matches_oracle(gpu, topk, max_nodes, ties, orc):
    """The device tree builder (the one medusa_generate runs every step)
    against the oracle's, node for node: tokens, parents, depths, rotary
    positions and the ancestor mask, with equal scores (ties broken by depth,
    then generation order) when `ties`."""
    import bind
    rng = np.random.default_rng(sum(topk) + max_nodes)
    kmax = max(topk)
    tok = rng.integers(0, 32064, (len(topk), kmax)).astype(np.int32)
    prob = np.sort(rng.random((len(topk), kmax)).astype(np.float32), axis=1)[:, ::-1].copy()
    if ties:
        prob = np.round(prob * 4) / 4  # many equal probabilities and products
        prob[:, 0] = 1.0
    t, par, dep, pos, mask = device_tree(gpu, 77, topk, tok, prob, max_nodes, 300)
    wt, wpar, wdep, _ = bind.medusa_tree(orc, 77, topk, tok, prob, max_nodes)
    assert np.array_equal(t, wt) and np.array_equal(par, wpar) and np.array_equal(dep, wdep)
    assert np.array_equal(pos, 300 + wdep)
    want = np.zeros_like(mask)
    for i in range(len(wt)):
        j = i
        while j >= 0:
            want[i, j] = 1
            j = wpar[j]
    assert np.array_equal(mask, want)


def test_device_tree_rejects_too_many_candidates(gpu):
    tok = np.zeros((3, 32), np.int32)
    prob = np.ones((3, 32), np.float32)
    t = np.zeros(64, np.int32)
    m = np.zeros(64 * 64, np.uint8)
    rc = gpu.fl_cuda_medusa_tree(flb200.ptr(tok), flb200.ptr(prob), flb200.ptr(np.array([32, 32, 2], np.int32)), 3,
                                 32, 64, 0, 0, *[flb200.ptr(t)] * 4, flb200.ptr(m))
    assert rc < 0


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


# ---- stochastic speculative decoding (temperature > 0) ----
#
# The sampling rule works on integer weights with exact sums, so given the
# same logits the device and the oracle make bit-identical decisions. Device
# and oracle logits agree within the logit tolerance but not bit for bit
# (activation-quantization rounding can flip on reordered float sums), and a
# draw moves with logit changes far below that tolerance; so the rule is
# checked by replay: every draw, acceptance test and emitted token of a device
# decode is recomputed by the oracle from the logits the device drew from,
# with the same Philox counters, and must be identical.

SAMPLE_T, SAMPLE_TOP_P, SAMPLE_SEED = 0.8, 0.95, 1234
FIRST_ROW, TARGET_ROW0 = 15, 7


def check_weights(orc, E_dev, M_dev, logits, T, top_p, what):
    E, M = orc.sample_weights(logits, T, top_p)
    assert np.array_equal(E_dev, E), f"{what}: nucleus weights differ at {np.nonzero(E_dev != E)[0][:5]}"
    assert int(M_dev) == M, f"{what}: kept mass"
    return E, M


def check_sampled_step(orc, u24, k, n_new, T, top_p, pre, t, before, after, out, acc_hist=None):
    """Replays one sampled step of one sequence: `pre` = (logits, weights,
    mass, token) of draft 0 (drawn by the previous step), `t` the trace after
    the step, `before` / `after` its state; the emitted tokens are in `out`."""
    n, s, produced = before["n"], before["steps"], before["produced"]
    d_lg = [pre[0]] + [t["logits"][j] for j in range(1, k)]
    d_q = [pre[1]] + [t["qd"][j] for j in range(1, k)]
    d_m = [pre[2]] + [int(t["qm"][j]) for j in range(1, k)]
    drafted = [pre[3]] + [int(t["drafted"][j]) for j in range(1, k)]
    for j in range(k):
        check_weights(orc, d_q[j], d_m[j], d_lg[j], T, top_p, f"step {s} draft {j}")
        assert drafted[j] == orc.sample_pick(d_q[j], d_m[j], u24(s, n + 1 + j, 0)), f"step {s}: draft draw {j}"
    pt, pm = t["pt"], [int(v) for v in t["pm"]]
    for r in range(k + 1):
        check_weights(orc, pt[r], pm[r], t["logits"][TARGET_ROW0 + r], T, top_p, f"step {s} target {r}")
    a = 0
    while True:
        pos = n + 1 + a
        if a == k:
            last = orc.sample_pick(pt[k], pm[k], u24(s, pos, 2))
            break
        x = drafted[a]
        if orc.sample_accept(u24(s, pos, 1), pt[a][x], pm[a], d_q[a][x], d_m[a]):
            a += 1
            continue
        R, zr = orc.sample_residual(pt[a], pm[a], d_q[a], d_m[a])
        last = orc.sample_pick(R, zr, u24(s, pos, 2)) if zr > 0 else orc.sample_pick(pt[a], pm[a], u24(s, pos, 2))
        break
    assert after["accepted"] == a, f"step {s}: accepted {after['accepted']} vs {a}"
    if acc_hist is not None:
        assert acc_hist[s] == a, f"step {s}: histogram"
    assert after["n"] == n + a + 1
    want = (drafted[:a] + [last])[: n_new - produced]
    assert out[produced: produced + len(want)].tolist() == want, f"step {s}: emitted tokens"


def replay_sampled(eng, orc, p, k, n_new, T, top_p, seed, seq_id=0):
    """Steps the device decode and replays every sampling decision; returns
    (tokens, accepted per step)."""
    P = len(p)
    u24 = lambda step, pos, purpose: orc.philox_u24(seed, seq_id, step, pos, purpose)
    eng.set_sampling(T, top_p, seed, seq_id)
    eng.sample_trace_enable(True)
    eng.spec_prefill(p, k)
    out, acc_hist = eng.spec_decode(n_new)  # the stream; the steps below repeat it
    t = eng.sample_trace()
    E, M = orc.sample_weights(t["logits"][FIRST_ROW], T, top_p)
    assert out[0] == orc.sample_pick(E, M, u24(0xFFFFFFFF, P, 2)), "first token"
    eng.spec_begin(n_new)
    t = eng.sample_trace()
    state = dict(n=P, produced=1, steps=0, done=0)
    while not state["done"]:
        pre = (t["logits"][0].copy(), t["qd"][0].copy(), int(t["qm"][0]), int(t["drafted"][0]))
        after = eng.spec_step()
        t = eng.sample_trace()
        check_sampled_step(orc, u24, k, n_new, T, top_p, pre, t, state, after, out, acc_hist)
        state = after
    assert state["produced"] == n_new and state["steps"] == len(acc_hist)
    eng.sample_trace_enable(False)
    eng.set_sampling(0.0)
    return out, acc_hist


def replay_sampled_batch(eng, orc, prompts, k, n_new, T, top_p, seed, ids):
    """replay_sampled for an in-GPU batch: every sequence's decisions, step
    by step, with its own Philox key (seed, id)."""
    nseq, P = prompts.shape
    eng.set_sampling(T, top_p, seed)
    eng.sample_trace_enable(True)
    try:
        eng.batch_prefill(prompts, k, ids)
        out, steps, _ = eng.batch_decode(n_new)
        u24s = [(lambda sid: (lambda st, pos, pu: orc.philox_u24(seed, sid, st, pos, pu)))(int(i)) for i in ids]
        traces = [eng.batch_trace(s) for s in range(nseq)]
        for s in range(nseq):
            E, M = orc.sample_weights(traces[s]["logits"][FIRST_ROW], T, top_p)
            assert out[s][0] == orc.sample_pick(E, M, u24s[s](0xFFFFFFFF, P, 2)), f"sequence {s}: first token"
        eng.batch_begin(n_new)
        traces = [eng.batch_trace(s) for s in range(nseq)]
        states = [dict(n=P, produced=1, steps=0, done=0) for _ in range(nseq)]
        while not all(st["done"] for st in states):
            pres = [(t["logits"][0].copy(), t["qd"][0].copy(), int(t["qm"][0]), int(t["drafted"][0])) for t in traces]
            after = eng.batch_step()
            traces = [eng.batch_trace(s) for s in range(nseq)]
            for s in range(nseq):
                if states[s]["done"]:
                    assert after[s]["steps"] == states[s]["steps"], f"sequence {s} stepped after finishing"
                    continue
                check_sampled_step(orc, u24s[s], k, n_new, T, top_p, pres[s], traces[s], states[s], after[s], out[s])
            states = after
        assert [st["steps"] for st in states] == steps.tolist()
    finally:
        eng.sample_trace_enable(False)
        eng.set_sampling(0.0)
    return out, steps


@pytest.mark.parametrize("T,top_p", [(SAMPLE_T, SAMPLE_TOP_P), (1.5, 1.0), (0.3, 0.5)])
def test_sampled_decisions_replay_on_oracle(small, orc, T, top_p):
    """Every draft draw, target distribution, acceptance test, residual or
    bonus draw and the emitted tokens of a 40-token sampled decode (k = 4)
    follow the oracle's rule and counter layout."""
    dims, eng, om, embed = small
    p = prompt(12, 16, dims["vocab"])
    try:
        out, acc = replay_sampled(eng, orc, p, 4, 40, T, top_p, SAMPLE_SEED)
    finally:
        eng.sample_trace_enable(False)
        eng.set_sampling(0.0)
    assert acc.min() < 4, "no rejection exercised"


def test_sampled_stream_repeatable(small):
    """Same seed and counter layout, same stream (also after restarting from
    the saved state); another seed or sequence id, another stream."""
    dims, eng, om, embed = small
    p = prompt(12, 16, dims["vocab"])
    try:
        eng.set_sampling(SAMPLE_T, SAMPLE_TOP_P, SAMPLE_SEED)
        a, ha = eng.spec_generate(p, 40, 4)
        b, hb = eng.spec_decode(40)
        c, _ = eng.spec_generate(p, 40, 4)
        eng.set_sampling(SAMPLE_T, SAMPLE_TOP_P, SAMPLE_SEED + 1)
        d, _ = eng.spec_generate(p, 40, 4)
        eng.set_sampling(SAMPLE_T, SAMPLE_TOP_P, SAMPLE_SEED, 1)
        f, _ = eng.spec_generate(p, 40, 4)
    finally:
        eng.set_sampling(0.0)
    assert np.array_equal(a, b) and np.array_equal(ha, hb) and np.array_equal(a, c)
    assert not np.array_equal(a, d) and not np.array_equal(a, f)


def test_sampled_greedy_limit(small):
    """A vanishing temperature with a one-token nucleus is greedy decoding."""
    dims, eng, om, embed = small
    p = prompt(13, 16, dims["vocab"])
    want, margins = om.greedy(p, 32)
    try:
        eng.set_sampling(1e-4, 1e-6, 7)
        got, _ = eng.spec_generate(p, 32, 4)
    finally:
        eng.set_sampling(0.0)
    assert_stream_matches(got, want, margins)


def test_sampled_large_vocab(gpu, orc):
    """Vocabulary above the register-resident size (32768): the nucleus
    passes read the distribution from memory."""
    dims = dict(SMALL_V1, vocab=40000)
    w, embed = make_weights(gpu, dims, seed=5)
    eng = flb200.Engine(gpu, engine_cfg(dims, draft_layers=1))
    load_engine(eng, w, embed)
    p = prompt(14, 12, dims["vocab"])
    try:
        replay_sampled(eng, orc, p, 4, 24, 1.0, 0.9, 77, 3)
    finally:
        eng.close()


def test_speculative_generate_sampled_reference_api(gpu, orc):
    """speculative_generate() with config->temperature > 0 runs the sampled
    rule with the engine's top_p and Philox key: the same stream as the
    engine's own sampled decode."""
    import ctypes as C
    dims = SMALL
    w, embed = make_weights(gpu, dims, seed=31)
    eng = flb200.Engine(gpu, engine_cfg(dims, draft_layers=1))
    load_engine(eng, {k: v for k, v in w.items() if k[0] != 1}, embed)
    dm = gpu.draft_model_create(1, dims["d"], dims["ffn"], dims["vocab"])
    assert gpu.draft_model_load(dm, b"synthetic:31") == 0
    eng.set_sampling(0.5, SAMPLE_TOP_P, 99, 2)
    cfg = flb200.SpecConfig(4, 0.7, 4)  # the call's temperature wins
    p = prompt(9, 12, dims["vocab"])
    ph = p.astype(np.float32)
    out = np.empty(20, np.int32)
    n = gpu.speculative_generate(dm, eng.h, C.cast(gpu.so.fl_cuda_target_forward, C.c_void_p), flb200.ptr(ph),
                                 len(p), flb200.ptr(out), 20, C.byref(cfg))
    assert n == 20, gpu.err()
    assert eng.get_sampling() == pytest.approx((0.7, SAMPLE_TOP_P, 99, 2))
    want, _ = eng.spec_generate(p, 20, 4)
    assert np.array_equal(out, want)
    cfg = flb200.SpecConfig(4, 0.0, 4)
    n = gpu.speculative_generate(dm, eng.h, C.cast(gpu.so.fl_cuda_target_forward, C.c_void_p), flb200.ptr(ph),
                                 len(p), flb200.ptr(out), 20, C.byref(cfg))
    assert n == 20 and eng.get_sampling()[0] == 0.0
    g_want, _, margins = oracle_model(orc, dims, w, embed).spec(p, 20, 4)
    assert_stream_matches(out, g_want, margins)
    gpu.draft_model_free(dm)
    eng.close()


def test_sampled_batch_independent_of_sharding(small):
    """A sequence's sampled stream depends only on its prompt and id, not on
    its place in the batch or on the other sequences: reordered batches and
    equal-size shards give the same tokens. (Batches of different sizes may
    take other kernels for their passes -- GEMV chunks or the tcgen05 GEMM --
    whose logits differ in the last bits, so only the rule is exact there:
    test_sampled_batch_replays_on_oracle.)"""
    import shard
    dims, eng, om, embed = small
    ids = np.arange(4, dtype=np.uint32)
    prompts = shard.prompts_for(ids, 12, dims["vocab"], 77)
    try:
        eng.set_sampling(SAMPLE_T, SAMPLE_TOP_P, SAMPLE_SEED)
        all_toks, steps, secs = eng.spec_generate_batch(prompts, 20, 4, seq_ids=ids)
        rev, _, _ = eng.spec_generate_batch(prompts[::-1], 20, 4, seq_ids=ids[::-1])
        lo, _, _ = eng.spec_generate_batch(prompts[:2], 20, 4, seq_ids=ids[:2])
        hi, _, _ = eng.spec_generate_batch(prompts[2:][::-1], 20, 4, seq_ids=ids[2:][::-1])
        pair, _, _ = eng.spec_generate_batch(prompts[[1, 2]], 20, 4, seq_ids=ids[[1, 2]])
    finally:
        eng.set_sampling(0.0)
    assert np.array_equal(rev[::-1], all_toks)
    assert np.array_equal(lo[1], pair[0]) and np.array_equal(hi[1], pair[1])
    assert len({tuple(r) for r in all_toks.tolist()}) == 4 and secs > 0 and steps.min() >= 1


@pytest.mark.parametrize("nseq,k", [(3, 4), (5, 6)])
def test_sampled_batch_replays_on_oracle(small, orc, nseq, k):
    """Every decision of every sequence of a sampled in-GPU batch follows the
    oracle's rule with that sequence's Philox key (3 x 5 verify rows through
    GEMV chunks; 5 x 7 through the tcgen05 GEMM)."""
    dims, eng, om, embed = small
    ids = np.array([7, 3, 11, 0, 5][:nseq], np.uint32)
    prompts = np.stack([prompt(60 + i, 12, dims["vocab"]) for i in range(nseq)])
    eng.batch_reserve(nseq, 12 + 24 + k + 3)
    out, steps = replay_sampled_batch(eng, orc, prompts, k, 24, SAMPLE_T, SAMPLE_TOP_P, SAMPLE_SEED, ids)
    assert out.shape == (nseq, 24) and steps.min() >= 1


@pytest.mark.parametrize("nseq,k", [(3, 4), (4, 5), (20, 4)])
def test_batch_greedy_streams_match_oracle(small, nseq, k):
    """An in-GPU batch decodes every sequence to the oracle's greedy stream:
    3 x 5 verify rows (GEMV chunks), 4 x 6 and 20 x 5 (tcgen05 GEMM; 20
    single-row draft passes through it too)."""
    dims, eng, om, embed = small
    prompts = np.stack([prompt(30 + i, 16, dims["vocab"]) for i in range(nseq)])
    eng.batch_reserve(nseq, 16 + 40 + k + 3)
    eng.batch_prefill(prompts, k)
    toks, steps, secs = eng.batch_decode(40)
    for i in range(nseq):
        want, margins = om.greedy(prompts[i], 40)
        assert_stream_matches(toks[i], want, margins)
    assert steps.min() >= 1 and secs > 0
    # decoding restarts from the post-prefill state
    again, steps2, _ = eng.batch_decode(40)
    assert np.array_equal(again, toks) and np.array_equal(steps2, steps)
    short, _, _ = eng.batch_decode(9)
    assert np.array_equal(short, toks[:, :9])


def test_batch_step_api(small):
    """fl_engine_batch_step advances every unfinished sequence by one step
    and leaves finished ones alone."""
    dims, eng, om, embed = small
    prompts = np.stack([prompt(90 + i, 10, dims["vocab"]) for i in range(3)])
    eng.batch_reserve(3, 64)
    eng.batch_prefill(prompts, 3)
    toks, steps, _ = eng.batch_decode(12)
    eng.batch_begin(12)
    n_steps = 0
    while True:
        st = eng.batch_step()
        n_steps += 1
        assert all(s["produced"] <= 12 or s["done"] for s in st)
        if all(s["done"] for s in st):
            break
        assert n_steps <= 12
    assert [s["steps"] for s in st] == steps.tolist()
    assert n_steps == steps.max()


def test_spec_medusa_stream_is_greedy(gpu, orc):
    """Draft chain + Medusa heads in one tree: the output is the base model's
    greedy stream (oracle), with multi-token steps; the reference signature
    speculative_medusa_generate gives the same tokens."""
    import ctypes as C
    dims = dict(SMALL, vocab=16)
    w, embed = make_weights(gpu, dims, seed=3, draft_layers=1, medusa_heads=4)
    eng = flb200.Engine(gpu, engine_cfg(dims, draft_layers=1, medusa_heads=4, max_seq_len=256))
    load_engine(eng, w, embed)
    p = prompt(4, 12, dims["vocab"])
    got, acc = eng.spec_medusa_generate(p, 40, 3, MEDUSA_TOPK, 48)
    om = oracle_model(orc, dims, w, embed, draft_layers=1, n_medusa=4)
    want, margins = om.greedy(p, 40)
    assert_stream_matches(got, want, margins)
    assert acc.max() >= 2, f"no multi-node path accepted: {acc.tolist()}"
    eng.close()
    # the same through the reference API: draft and heads loaded from "synthetic:SEED"
    eng = flb200.Engine(gpu, engine_cfg(dims, draft_layers=1, medusa_heads=4, max_seq_len=256))
    load_engine(eng, {k: v for k, v in w.items() if k[0] == 0 or k[0] == 3}, embed)
    dm = gpu.draft_model_create(1, dims["d"], dims["ffn"], dims["vocab"])
    assert gpu.draft_model_load(dm, b"synthetic:3") == 0
    mm = gpu.medusa_model_create(4, dims["d"], dims["vocab"])
    assert gpu.medusa_model_load(mm, b"synthetic:3") == 0
    tk = np.array(MEDUSA_TOPK, np.int32)
    assert gpu.fl_medusa_set_tree(mm, flb200.ptr(tk), 4, 48) == 0
    cfg = flb200.MedusaConfig(3, 10, 0.0)
    ph = p.astype(np.float32)
    out = np.empty(40, np.int32)
    n = gpu.speculative_medusa_generate(dm, C.cast(gpu.so.fl_cuda_target_forward, C.c_void_p), mm, eng.h,
                                        C.cast(gpu.so.fl_cuda_base_forward, C.c_void_p), flb200.ptr(ph), len(p),
                                        flb200.ptr(out), 40, C.byref(cfg))
    assert n == 40, gpu.err()
    assert_stream_matches(out, want, margins)
    gpu.medusa_model_free(mm)
    gpu.draft_model_free(dm)
    eng.close()


@pytest.mark.parametrize("k,width", [(4, 8), (3, 4), (2, 1)])
def test_spec_tree_stream_is_greedy(gpu, orc, small, k, width):
    """Static draft tree (chain + top-width per depth; 33 nodes at k = 4,
    width = 8, verified through the tcgen05 GEMM): the output is the base
    model's greedy stream, on the small models and on a 16-token vocabulary
    where paths through siblings are accepted often (KV compaction)."""
    dims, eng, om, embed = small
    p = prompt(12, 16, dims["vocab"])
    got, acc = eng.spec_tree_generate(p, 40, k, width)
    want, margins = om.greedy(p, 40)
    assert_stream_matches(got, want, margins)
    dims16 = dict(SMALL, vocab=16)
    w, emb = make_weights(gpu, dims16, seed=5, draft_layers=1)
    e16 = flb200.Engine(gpu, engine_cfg(dims16, draft_layers=1, max_seq_len=256))
    load_engine(e16, w, emb)
    p16 = prompt(13, 12, 16)
    got, acc = e16.spec_tree_generate(p16, 60, k, width)
    om16 = oracle_model(orc, dims16, w, emb, draft_layers=1)
    want, margins = om16.greedy(p16, 60)
    assert_stream_matches(got, want, margins)
    chain, cacc = e16.spec_generate(p16, 60, k)
    assert_stream_matches(chain, want, margins)
    if width > 1:
        assert acc.max() >= 2, acc.tolist()
    e16.close()


@pytest.mark.parametrize("nseq,k,width", [(3, 3, 4), (4, 4, 8), (1, 2, 2)])
def test_batch_tree_streams_are_greedy(gpu, orc, small, nseq, k, width):
    """Draft trees for an in-GPU batch (4 x 33 nodes at k = 4, width = 8,
    132 verify rows): every sequence's output is the base model's greedy
    stream; on a 16-token vocabulary paths through siblings are accepted."""
    dims, eng, om, embed = small
    prompts = np.stack([prompt(110 + i, 14, dims["vocab"]) for i in range(nseq)])
    eng.batch_reserve(nseq, 14 + 32 + 1 + k * width + k + 3)
    got, steps, secs = eng.batch_tree_generate(prompts, 32, k, width)
    for i in range(nseq):
        want, margins = om.greedy(prompts[i], 32)
        assert_stream_matches(got[i], want, margins)
    assert steps.min() >= 1 and secs > 0
    dims16 = dict(SMALL, vocab=16)
    w, emb = make_weights(gpu, dims16, seed=5, draft_layers=1)
    e16 = flb200.Engine(gpu, engine_cfg(dims16, draft_layers=1, max_seq_len=256))
    load_engine(e16, w, emb)
    om16 = oracle_model(orc, dims16, w, emb, draft_layers=1)
    p16 = np.stack([prompt(120 + i, 12, 16) for i in range(nseq)])
    e16.batch_reserve(nseq, 12 + 48 + 1 + k * width + k + 3)
    got, steps, _ = e16.batch_tree_generate(p16, 48, k, width)
    for i in range(nseq):
        want, margins = om16.greedy(p16[i], 48)
        assert_stream_matches(got[i], want, margins)
        one, acc = e16.spec_tree_generate(p16[i], 48, k, width)
        assert_stream_matches(one, want, margins)
    assert steps.max() < 47, steps.tolist()  # multi-token steps
    e16.close()


def test_medusa_step_api_matches_generate(gpu, orc):
    """The reference's step-level Medusa API on the engine's callback position
    (prefill with fl_cuda_base_forward, then medusa_decode_step /
    medusa_build_tree + medusa_verify_tree) reproduces the greedy stream."""
    import ctypes as C
    dims = dict(SMALL, vocab=16)
    w, embed = make_weights(gpu, dims, seed=3, draft_layers=0, medusa_heads=4)
    eng = flb200.Engine(gpu, engine_cfg(dims, draft_layers=0, medusa_heads=4, max_seq_len=256))
    load_engine(eng, {k: v for k, v in w.items() if k[0] != 2}, embed)
    mm = gpu.medusa_model_create(4, dims["d"], dims["vocab"])
    assert gpu.medusa_model_load(mm, b"synthetic:3") == 0
    tk = np.array(MEDUSA_TOPK, np.int32)
    assert gpu.fl_medusa_set_tree(mm, flb200.ptr(tk), 4, 48) == 0
    cfg = flb200.MedusaConfig(4, 10, 0.0)
    base_fwd = C.cast(gpu.so.fl_cuda_base_forward, C.c_void_p)
    p = prompt(4, 12, dims["vocab"])
    om = oracle_model(orc, dims, w, embed, draft_layers=0, n_medusa=4)
    want, margins = om.greedy(p, 30)
    # heads into the engine, then the prompt through base_forward (the feature
    # of its last position comes back)
    assert gpu.fl_engine_bind_medusa(eng.h, mm) == 0, gpu.err()
    assert gpu.fl_engine_set_position(eng.h, 0) == 0
    F = np.empty(dims["d"], np.float32)
    gpu.fl_cuda_base_forward(eng.h, flb200.ptr(p), len(p), flb200.ptr(F), dims["d"])
    assert gpu.fl_engine_position(eng.h) == len(p), gpu.err()
    # first token: the root of a tree built from the prompt's last feature
    tree = gpu.medusa_tree_create(48)
    assert gpu.medusa_build_tree(mm, flb200.ptr(F), tree, C.byref(cfg)) > 0
    got = [tree.contents.tokens[0]]
    acc = []
    out = np.empty(48, np.int32)
    nout = C.c_int(0)
    while len(got) < 30:
        # alternate the two decompositions of a step
        if len(acc) % 2 == 0:
            r = gpu.medusa_decode_step(eng.h, base_fwd, mm, flb200.ptr(F), got[-1], flb200.ptr(out), C.byref(nout),
                                       C.byref(cfg))
            assert r == nout.value and r >= 1, gpu.err()
        else:
            assert gpu.medusa_predict(mm, flb200.ptr(F), got[-1], tree, C.byref(cfg)) > 0
            na = C.c_int(0)
            a = gpu.medusa_verify_tree(eng.h, base_fwd, tree, flb200.ptr(out), C.byref(na), C.byref(cfg))
            assert a == na.value and a >= 0, gpu.err()
            nout.value = a + 1
        acc.append(nout.value - 1)
        got.extend(out[:nout.value].tolist())
        assert gpu.fl_engine_last_feature(eng.h, flb200.ptr(F)) == 0
    got = np.array(got[:30])
    assert_stream_matches(got, want, margins)
    assert max(acc) >= 2, f"no multi-node path accepted: {acc}"
    gpu.medusa_tree_free(tree)
    gpu.medusa_model_free(mm)
    eng.close()
