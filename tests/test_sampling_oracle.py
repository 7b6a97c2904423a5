"""The oracle's stochastic speculative decoding rule (temperature, top-p
nucleus, Philox-keyed draws, rejection sampling)."""
import numpy as np

import bind
from _model import SMALL, make_weights, prompt


def test_nucleus_distribution(orc):
    rng = np.random.default_rng(0)
    lg = (rng.standard_normal(4096) * 3).astype(np.float32)
    q = orc.sample_dist(lg, 0.8, 0.95)
    assert abs(q.sum() - 1.0) < 1e-4
    p = np.exp((lg - lg.max()) / 0.8)
    p /= p.sum()
    kept = q > 0
    assert p[kept].sum() >= 0.95 - 1e-4
    # ancestor of every kept token: every more likely token is kept too
    assert p[~kept].max() <= p[kept].min() + 1e-12
    # dropping the least likely kept token would fall below top_p
    assert p[kept].sum() - p[kept].min() < 0.95 + 1e-4


def test_inverse_cdf(orc):
    w = np.array([0, 100, 0, 600, 300], np.uint32)
    counts = np.zeros(5)
    for U in np.linspace(0, 1 << 24, 2000, endpoint=False).astype(np.int64):
        counts[orc.sample_pick(w, int(w.sum()), int(U))] += 1
    assert counts[0] == counts[2] == 0
    np.testing.assert_allclose(counts / counts.sum(), w / w.sum(), atol=2e-3)
    # 64-bit weights, and the first index whose running sum exceeds the target
    w64 = np.array([5, 0, 7], np.uint64)
    assert orc.sample_pick(w64, 12, 0) == 0
    assert orc.sample_pick(w64, 12, (5 << 24) // 12) == 0  # target 4
    assert orc.sample_pick(w64, 12, -(-(5 << 24) // 12)) == 2  # target 5
    assert orc.sample_pick(w64, 12, (1 << 24) - 1) == 2


def test_sampling_weight_is_exp(orc):
    """E = trunc(e^x * 2^24) within one unit (the polynomial exp is within a
    few float ulps of e^x on [-17, 0]); 0 below -17; 2^24 at 0."""
    xs = np.concatenate([np.linspace(-17, 0, 20001), -np.logspace(-8, 1, 500)]).astype(np.float32)
    got = np.array([orc.sample_weight(x) for x in xs], np.int64)
    want = np.floor(np.exp(xs.astype(np.float64)) * 2.0 ** 24).astype(np.int64)
    assert np.abs(got - want).max() <= 1
    assert orc.sample_weight(0.0) == 1 << 24
    assert orc.sample_weight(-17.5) == 0 and orc.sample_weight(float("nan")) == 0


def test_acceptance_and_residual(orc):
    """u < p(x)/q(x) in integers; the residual is proportional to max(0, p-q)."""
    rng = np.random.default_rng(3)
    Ep = rng.integers(0, 1 << 24, 64).astype(np.uint32)
    Eq = rng.integers(0, 1 << 24, 64).astype(np.uint32)
    Mp, Mq = int(Ep.sum()), int(Eq.sum())
    for x in range(64):
        if Eq[x] == 0:
            continue
        ratio = (int(Ep[x]) / Mp) / (int(Eq[x]) / Mq)
        for U in (0, 1 << 23, (1 << 24) - 1):
            if abs(U / 2 ** 24 - ratio) > 1e-9:
                assert orc.sample_accept(U, Ep[x], Mp, Eq[x], Mq) == (U / 2 ** 24 < ratio)
    R, s = orc.sample_residual(Ep, Mp, Eq, Mq)
    r = np.maximum(0.0, Ep / Mp - Eq / Mq)
    assert s == int(R.sum()) and s > 0
    np.testing.assert_allclose(R / s, r / r.sum(), atol=1e-9)
    R0, s0 = orc.sample_residual(Ep, Mp, Ep, Mp)
    assert s0 == 0


def test_sampled_streams_seeded_and_greedy_limit(lib, orc):
    dims = SMALL
    w, embed = make_weights(lib, dims, seed=11, draft_layers=1)
    om = bind.OracleModel(orc, dims, embed, w, draft_layers=1)
    p = prompt(5, 12, dims["vocab"])
    a, acc_a = om.spec_sampled(p, 24, 4, 0.8, 0.95, 1234)
    b, _ = om.spec_sampled(p, 24, 4, 0.8, 0.95, 1234)
    c, _ = om.spec_sampled(p, 24, 4, 0.8, 0.95, 99)
    assert np.array_equal(a, b), "same seed, same stream"
    assert not np.array_equal(a, c), "another seed, another stream"
    # a vanishing temperature with a tiny nucleus is greedy decoding
    g, _ = om.greedy(p, 24)
    t, _ = om.spec_sampled(p, 24, 4, 1e-4, 1e-6, 1234)
    assert np.array_equal(t, g)
