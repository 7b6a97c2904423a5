"""The oracle's Medusa rule (include/medusa.h): tree construction and greedy
tree verification. With greedy acceptance the produced stream is exactly the
base model's greedy stream whatever the heads propose; a 16-token vocabulary
makes the heads' top-k lists cover the greedy token often, so accepted paths
of several nodes (and the KV compaction after them) are exercised."""
import numpy as np

import bind
from _model import SMALL, make_weights, prompt

TOPK = [10, 5, 3, 2]


def test_tree_is_ancestor_closed_and_ordered(orc):
    rng = np.random.default_rng(0)
    kmax = max(TOPK)
    tok = rng.integers(0, 1000, (4, kmax)).astype(np.int32)
    prob = np.sort(rng.random((4, kmax)).astype(np.float32), axis=1)[:, ::-1].copy()
    prob[1, 0] = 1.0  # a child as likely as its parent: the parent must still come first
    t, par, dep, sc = bind.medusa_tree(orc, 7, TOPK, tok, prob, 64)
    assert len(t) == 64 and t[0] == 7 and par[0] == -1 and dep[0] == 0
    for i in range(1, len(t)):
        assert 0 <= par[i] < i, "parents precede children"
        assert dep[i] == dep[par[i]] + 1
        assert sc[i] <= sc[par[i]]
        assert t[i] == tok[dep[i] - 1][list(tok[dep[i] - 1]).index(t[i])]
    # the kept set is the 63 best candidates: nothing dropped scores above a kept node
    total = sum(int(np.prod(TOPK[:L + 1])) for L in range(4))
    assert total == 10 + 50 + 150 + 300
    s_kept = np.sort(sc[1:])
    assert s_kept[0] >= 0


def test_medusa_stream_is_the_greedy_stream(lib, orc):
    dims = dict(SMALL, vocab=16)
    w, embed = make_weights(lib, dims, seed=3, draft_layers=0, medusa_heads=4)
    om = bind.OracleModel(orc, dims, embed, w, draft_layers=0, n_medusa=4)
    p = prompt(4, 12, dims["vocab"])
    g, _ = om.greedy(p, 48)
    m, acc, _ = om.medusa(p, 48, TOPK, 64)
    assert np.array_equal(m, g)
    assert acc.max() >= 2, f"accepted paths too short to exercise compaction: {acc.tolist()}"
    assert acc.sum() + len(acc) + 1 >= 48
