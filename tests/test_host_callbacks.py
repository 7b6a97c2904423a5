"""The reference API with the caller's own host target / base functions
(speculative.h:146-185, medusa.h:161-198): the target here is the oracle's
base model behind a ctypes callback with fl_cuda_target_forward's contract
(append `len` tokens, write their next-token logits), the base the same
behind fl_cuda_base_forward's (append, write the last feature). The library
runs its draft / Medusa heads on the GPU and feeds the host function only
tokens that end up in the output, so the greedy output must be exactly the
oracle's greedy stream, whatever the draft proposes."""
import ctypes as C

import numpy as np
import pytest

import flb200
from _model import SMALL, make_weights, prompt

pytestmark = pytest.mark.gpu

TARGET_FN = C.CFUNCTYPE(None, C.c_void_p, C.POINTER(C.c_float), C.POINTER(C.c_float), C.c_int)
BASE_FN = C.CFUNCTYPE(None, C.c_void_p, C.POINTER(C.c_int), C.c_int, C.POINTER(C.c_float), C.c_int)


class HostModel:
    """The oracle's base stack as a stateful host model: every call appends
    tokens at the next positions of its own KV cache."""

    def __init__(self, orc, dims, w, embed, cap=256):
        import bind
        self.om = bind.OracleModel(orc, dims, embed, w, draft_layers=0)
        self.embed, self.dims = embed, dims
        self.kv = self.om.kv(dims["layers"], cap)
        self.pos = 0
        self.calls = 0
        self.fed = []

    def append(self, toks):
        toks = np.asarray(toks, np.int32)
        F = self.om.stack_forward(0, self.kv, self.embed[toks], self.pos, np.arange(self.pos, self.pos + len(toks)))
        self.pos += len(toks)
        self.calls += 1
        self.fed += toks.tolist()
        self.last_F = np.ascontiguousarray(F[-1])
        return F

    def target_fn(self):
        V = self.dims["vocab"]

        def fwd(model, inp, out, n):
            toks = [int(inp[i]) for i in range(n)]
            lg = self.om.lm_logits(self.append(toks))
            C.memmove(out, lg.ctypes.data, lg.nbytes)
            assert lg.shape == (n, V)
        return TARGET_FN(fwd)

    def base_fn(self):
        d = self.dims["d"]

        def fwd(model, toks, n, hidden, hs):
            F = self.append([toks[i] for i in range(n)])
            assert hs == d
            C.memmove(hidden, np.ascontiguousarray(F[-1]).ctypes.data, 4 * d)
        return BASE_FN(fwd)


@pytest.fixture(scope="module")
def target(gpu, orc):
    w, embed = make_weights(gpu, SMALL, seed=41, draft_layers=0)
    return w, embed


def oracle_greedy(orc, w, embed, p, n):
    import bind
    return bind.OracleModel(orc, SMALL, embed, w, draft_layers=0).greedy(p, n)[0]


def test_speculative_generate_host_target_greedy(gpu, orc, target):
    w, embed = target
    hm = HostModel(orc, SMALL, w, embed)
    fn = hm.target_fn()
    dm = gpu.draft_model_create(1, SMALL["d"], SMALL["ffn"], SMALL["vocab"])
    assert gpu.draft_model_load(dm, b"synthetic:7") == 0
    p = prompt(12, 20, SMALL["vocab"])
    out = np.empty(40, np.int32)
    cfg = flb200.SpecConfig(4, 0.0, 4)
    n = gpu.speculative_generate(dm, None, C.cast(fn, C.c_void_p), flb200.ptr(p.astype(np.float32)), len(p),
                                 flb200.ptr(out), 40, C.byref(cfg))
    assert n == 40, gpu.err()
    assert np.array_equal(out, oracle_greedy(orc, w, embed, p, 40))
    # the host target saw the prompt, then only output tokens, each once
    assert hm.fed == p.tolist() + out[:len(hm.fed) - len(p)].tolist()
    gpu.draft_model_free(dm)


def test_speculative_generate_host_target_sampled(gpu, orc, target):
    """temperature > 0: the same call twice gives the same stream; the first
    token replays on the oracle's rule from the target's prompt logits; a
    vanishing temperature is the greedy stream."""
    w, embed = target
    dm = gpu.draft_model_create(1, SMALL["d"], SMALL["ffn"], SMALL["vocab"])  # never loaded: seed 0 weights
    p = prompt(13, 16, SMALL["vocab"])
    outs = []
    for T in (0.8, 0.8, 1e-6):
        hm = HostModel(orc, SMALL, w, embed)
        fn = hm.target_fn()
        out = np.empty(24, np.int32)
        cfg = flb200.SpecConfig(3, T, 3)
        n = gpu.speculative_generate(dm, None, C.cast(fn, C.c_void_p), flb200.ptr(p.astype(np.float32)), len(p),
                                     flb200.ptr(out), 24, C.byref(cfg))
        assert n == 24, gpu.err()
        outs.append(out.copy())
    assert np.array_equal(outs[0], outs[1])
    assert np.array_equal(outs[2], oracle_greedy(orc, w, embed, p, 24))
    import bind
    om = bind.OracleModel(orc, SMALL, embed, w, draft_layers=0)
    lg = om.lm_logits(om.stack_forward(0, om.kv(SMALL["layers"], 64), embed[p], 0, np.arange(len(p))))[-1]
    E, M = orc.sample_weights(lg, 0.8, 1.0)
    assert outs[0][0] == orc.sample_pick(E, M, orc.philox_u24(0, 0, 0xFFFFFFFF, len(p), 2))
    gpu.draft_model_free(dm)


def test_speculative_decode_step_host_target(gpu, orc, target):
    """Step by step: the caller prefills its target, then chains
    speculative_decode_step on the last output token."""
    w, embed = target
    hm = HostModel(orc, SMALL, w, embed)
    fn = hm.target_fn()
    p = prompt(14, 12, SMALL["vocab"])
    first = int(hm.om.lm_logits(hm.append(p))[-1].argmax())
    dm = gpu.draft_model_create(1, SMALL["d"], SMALL["ffn"], SMALL["vocab"])
    assert gpu.draft_model_load(dm, b"synthetic:9") == 0
    cache = gpu.draft_kv_cache_create(256, SMALL["heads"], SMALL["head_dim"])
    cache.contents.cache_len = len(p)  # the draft's own cache starts at the first output position
    cfg = flb200.SpecConfig(4, 0.0, 4)
    stream, cur = [first], first
    hidden = np.zeros(SMALL["d"], np.float32)  # unused with a host target
    buf = np.empty(8, np.int32)
    nout = C.c_int()
    while len(stream) < 30:
        r = gpu.speculative_decode_step(dm, cache, None, C.cast(fn, C.c_void_p), flb200.ptr(hidden), cur,
                                        flb200.ptr(buf), C.byref(nout), C.byref(cfg))
        assert r == nout.value and 1 <= r <= 5, gpu.err()
        stream += buf[:r].tolist()
        cur = stream[-1]
    want = oracle_greedy(orc, w, embed, p, len(stream))
    assert np.array_equal(np.array(stream), want)
    gpu.draft_kv_cache_free(cache)
    gpu.draft_model_free(dm)


def with_lm_head(gpu, w, seed):
    """The base weights with the LM head a Medusa model generates from its
    seed: with a host base_forward (features only) the library applies the
    Medusa model's LM head to them."""
    w = dict(w)
    w[(3, 0, 1)] = gpu.synth_q4_0_i8(seed, flb200.tensor_id(3, 0, 1), SMALL["vocab"], SMALL["d"])
    return w


def test_medusa_generate_host_base(gpu, orc, target):
    w, embed = target
    w = with_lm_head(gpu, w, 11)
    hm = HostModel(orc, SMALL, w, embed)
    fn = hm.base_fn()
    med = gpu.medusa_model_create(4, SMALL["d"], SMALL["vocab"])
    assert gpu.medusa_model_load(med, b"synthetic:11") == 0
    p = prompt(15, 18, SMALL["vocab"])
    out = np.empty(36, np.int32)
    cfg = flb200.MedusaConfig(4, 4, 0.0)
    n = gpu.medusa_generate(None, C.cast(fn, C.c_void_p), med, flb200.ptr(p.astype(np.float32)), len(p),
                            flb200.ptr(out), 36, C.byref(cfg))
    assert n == 36, gpu.err()
    assert np.array_equal(out, oracle_greedy(orc, w, embed, p, 36))
    assert hm.fed == p.tolist() + out[:len(hm.fed) - len(p)].tolist()
    gpu.medusa_model_free(med)


def test_medusa_decode_step_host_base(gpu, orc, target):
    w, embed = target
    w = with_lm_head(gpu, w, 0)  # the heads are never loaded: seed 0
    hm = HostModel(orc, SMALL, w, embed)
    fn = hm.base_fn()
    med = gpu.medusa_model_create(3, SMALL["d"], SMALL["vocab"])  # never loaded: seed 0 heads
    p = prompt(16, 10, SMALL["vocab"])
    F = hm.append(p)[-1].copy()
    first = int(hm.om.lm_logits(F[None])[0].argmax())
    cfg = flb200.MedusaConfig(3, 4, 0.0)
    stream, cur = [first], first
    buf = np.empty(80, np.int32)
    nout = C.c_int()
    while len(stream) < 24:
        r = gpu.medusa_decode_step(None, C.cast(fn, C.c_void_p), med, flb200.ptr(F), cur, flb200.ptr(buf),
                                   C.byref(nout), C.byref(cfg))
        assert r == nout.value and r >= 1, gpu.err()
        stream += buf[:r].tolist()
        cur = stream[-1]
        F = hm.last_F.copy()  # the feature of the last token the base saw (the one before cur)
    want = oracle_greedy(orc, w, embed, p, len(stream))
    assert np.array_equal(np.array(stream), want)
    gpu.medusa_model_free(med)
