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
    w = np.array([0.0, 0.1, 0.0, 0.6, 0.3], np.float32)
    counts = np.zeros(5)
    for u in np.linspace(0, 1, 2000, endpoint=False, dtype=np.float32):
        counts[orc.sample_index(w, float(u))] += 1
    assert counts[0] == counts[2] == 0
    np.testing.assert_allclose(counts / counts.sum(), w, atol=2e-3)


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
