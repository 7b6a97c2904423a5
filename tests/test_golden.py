"""The oracle against golden vectors of the reference's own functions
(tests/golden/ref_primitives.npz, made by tests/golden/make_golden.py from
the reference sources compiled into oracle/_ref/libref.so). Integer work is
bit-exact; float work agrees to a few ulp (the reference is built with
-ffast-math). This pin needs neither the reference sources nor a GPU."""
import os

import numpy as np
import pytest

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "ref_primitives.npz")


@pytest.fixture(scope="module")
def gold():
    return np.load(GOLDEN)


def test_quant_u8(orc, gold):
    assert np.array_equal(orc.quant_u8(gold["quant_x"]), gold["quant_q"])


def test_block_dots_pairsat(orc, gold):
    a, w, want = gold["dots_a"], gold["dots_w"], gold["dots"]
    for i in range(a.shape[0]):
        for b in range(96):
            got = orc.dot_pairsat(np.ascontiguousarray(a[i, 32 * b:32 * b + 32]),
                                  np.ascontiguousarray(w[i, 32 * b:32 * b + 32]))
            assert got == want[i, b], (i, b)


def test_matmul_rowscale(orc, gold):
    assert np.array_equal(orc.matmul_rowscale(gold["mm_A"], gold["mm_W"], gold["mm_s"]), gold["mm_C"])


def test_rmsnorm_swiglu_silu(orc, gold):
    np.testing.assert_allclose(orc.rmsnorm(gold["rms_x"]), gold["rms_y"], rtol=3e-6, atol=0)
    np.testing.assert_allclose(orc.swiglu(gold["swiglu_g"], gold["swiglu_u"]), gold["swiglu_y"], rtol=2e-5, atol=1e-6)
    np.testing.assert_allclose(orc.silu(gold["swiglu_g"]), gold["silu_y"], rtol=2e-5, atol=1e-6)


def test_rope(orc, gold):
    q, k = gold["rope_q"], gold["rope_k"]
    for p in range(q.shape[0]):
        np.testing.assert_allclose(orc.rope_vec(q[p], 4, 96, p, 10000.0), gold["rope_oq"][p], rtol=1e-5, atol=2e-6)
        np.testing.assert_allclose(orc.rope_vec(k[p], 2, 96, p, 10000.0), gold["rope_ok"][p], rtol=1e-5, atol=2e-6)


def test_attention_semantics(orc, gold):
    """compute_attention's rule (RoPE at theta 500000 applied to Q and K
    first, as inference.c:196-197 does; scale 1/sqrt(hd); causal; kv head
    h / (H / Hkv); max-subtracted softmax) restated in float64 after the
    oracle's RoPE: the rule every attention kernel of the product implements."""
    seq, H, Hk, hd = 7, 4, 2, 32
    Qr = np.stack([orc.rope_vec(gold["attn_Q"][p], H, hd, p, 500000.0) for p in range(seq)])
    Kr = np.stack([orc.rope_vec(gold["attn_K"][p], Hk, hd, p, 500000.0) for p in range(seq)])
    Q, K = Qr.astype(np.float64), Kr.astype(np.float64)
    V, O = gold["attn_V"].astype(np.float64), gold["attn_O"].astype(np.float64)
    want = np.empty_like(O)
    for h in range(H):
        kh = h // (H // Hk)
        q = Q[:, h * hd:(h + 1) * hd]
        k = K[:, kh * hd:(kh + 1) * hd]
        v = V[:, kh * hd:(kh + 1) * hd]
        s = q @ k.T / np.sqrt(hd)
        s[np.triu_indices(seq, 1)] = -np.inf
        p = np.exp(s - s.max(axis=1, keepdims=True))
        p /= p.sum(axis=1, keepdims=True)
        want[:, h * hd:(h + 1) * hd] = p @ v
    np.testing.assert_allclose(O, want, rtol=1e-4, atol=1e-5)
