"""The oracle restatement against the reference's own functions compiled from
its sources (oracle/_ref/libref.so). Integer work is bit-exact; float work
agrees to a few ulp (the reference is built with -ffast-math, which
reassociates sums and turns 1/sqrtf into rsqrtss + one Newton step)."""
import numpy as np
import pytest

from _model import SMALL


def test_quant_u8_bit_exact(orc, ref):
    rng = np.random.default_rng(0)
    x = (rng.standard_normal(1 << 16) * 2.0).astype(np.float32)
    # rounding ties, clamp edges, NaN and out-of-int32-range values
    special = np.array([0.5 / 127, -0.5 / 127, 1.5 / 127, 2.5 / 127, -128.5 / 127, 127.5 / 127, 1.0, -1.0,
                        np.nan, np.inf, -np.inf, 1e30, -1e30, 2.0e7, -2.0e7, 0.0, -0.0], np.float32)
    x[: special.size] = special
    assert np.array_equal(orc.quant_u8(x), ref.quant_u8(x))


@pytest.mark.parametrize("scale16", [False, True])
def test_dot_pairsat_bit_exact(orc, ref, scale16):
    """dot_product_u8_i8 for [-8,7] weights and the reference's (q-8)*16
    weights, where the int16 pair saturation fires."""
    rng = np.random.default_rng(1)
    for _ in range(200):
        a = rng.integers(0, 256, 3072, dtype=np.uint8)
        q = rng.integers(0, 16, 3072) - 8
        w = (np.clip(q * 16, -128, 127) if scale16 else q).astype(np.int8)
        assert orc.dot_pairsat(a, w) == ref.dot(a, w)


def test_matmul_rowscale_bit_exact(orc, ref):
    """Per-row mode equals the reference's matmul_dequantized float for float."""
    rng = np.random.default_rng(2)
    M, N, K = 3, 1100, 3072
    A = rng.standard_normal((M, K)).astype(np.float32)
    W = np.clip((rng.integers(0, 16, (N, K)) - 8) * 16, -128, 127).astype(np.int8)
    s = (rng.random(N) * 0.01).astype(np.float32)
    assert np.array_equal(orc.matmul_rowscale(A, W, s), ref.matmul_dequantized(A, W, s))


def test_block_dots_are_reference_block_dots(orc, ref):
    """Each per-(m, n, block) int32 of block mode is dot_product_u8_i8 over
    that 32-byte block (one iteration of the reference's AVX2 loop)."""
    rng = np.random.default_rng(3)
    M, N, K = 2, 16, 256
    A = rng.standard_normal((M, K)).astype(np.float32)
    W = (rng.integers(0, 16, (N, K)) - 8).astype(np.int8)
    D = orc.block_dots(A, W)
    for m in range(M):
        q = ref.quant_u8(A[m])
        for n in range(N):
            for b in range(K // 32):
                assert D[m, n, b] == ref.dot(np.ascontiguousarray(q[32 * b:32 * b + 32]),
                                             np.ascontiguousarray(W[n, 32 * b:32 * b + 32]))


@pytest.mark.parametrize("n", [3072, 8192, 5120, 17920])
def test_rmsnorm_close(orc, ref, n):
    rng = np.random.default_rng(n)
    for _ in range(10):
        x = (rng.standard_normal(n) * rng.random() * 20).astype(np.float32)
        np.testing.assert_allclose(orc.rmsnorm(x), ref.rms_norm(x), rtol=3e-6, atol=0)


def test_swiglu_silu_close(orc, ref):
    rng = np.random.default_rng(5)
    g = (rng.standard_normal(8192) * 3).astype(np.float32)
    u = rng.standard_normal(8192).astype(np.float32)
    np.testing.assert_allclose(orc.swiglu(g, u), ref.swiglu(g, u), rtol=2e-5, atol=1e-6)
    np.testing.assert_allclose(orc.silu(g), ref.silu(g), rtol=2e-5, atol=1e-6)


def test_fast_sigmoid_is_the_reference_polynomial(orc, ref):
    """The polynomial is far from a true sigmoid above ~1.5 (sigma(3) ~ 0.42):
    the oracle must reproduce that, not 1/(1+exp(-x))."""
    x = np.array([3.0] * 8, np.float32)
    s = ref.silu(x) / x
    assert abs(s[0] - 0.42) < 0.02
    assert abs(orc.so.orc_fast_sigmoid(3.0) - s[0]) < 1e-6


@pytest.mark.parametrize("theta", [500000.0, 10000.0])
def test_rope_close(orc, ref, theta):
    rng = np.random.default_rng(6)
    seq, H, Hk, hd = 9, 4, 2, 64
    q = rng.standard_normal((seq, H * hd)).astype(np.float32)
    k = rng.standard_normal((seq, Hk * hd)).astype(np.float32)
    rq, rk = ref.apply_rope(q, k, seq, H, Hk, hd, theta)
    for p in range(seq):
        np.testing.assert_allclose(orc.rope_vec(q[p], H, hd, p, theta), rq[p], rtol=1e-5, atol=2e-6)
        np.testing.assert_allclose(orc.rope_vec(k[p], Hk, hd, p, theta), rk[p], rtol=1e-5, atol=2e-6)


def test_layer_composition_matches_reference_model_forward(orc, ref, lib):
    """The oracle's layer stack with f32 weights (matvec mode) against the
    reference's model_forward: norm, RoPE (theta 500000 as hard-coded at
    inference.c:196), GQA attention, residuals, SwiGLU, final norm, LM head of
    the last row, greedy token."""
    import bind
    dims = dict(SMALL, theta=500000.0, kv_heads=2)
    rng = np.random.default_rng(7)
    d, F, qd, kd = dims["d"], dims["ffn"], dims["heads"] * dims["head_dim"], dims["kv_heads"] * dims["head_dim"]
    shapes = [(qd, d), (kd, d), (kd, d), (d, qd), (F, d), (F, d), (d, F)]
    f32 = {}
    for l in range(dims["layers"]):
        for p, (r, c) in enumerate(shapes):
            f32[(0, l, p)] = (rng.standard_normal((r, c)) * 0.05).astype(np.float32)
    f32[(3, 0, 1)] = (rng.standard_normal((dims["vocab"], d)) * 0.05).astype(np.float32)
    embed = (rng.standard_normal((dims["vocab"], d)) * 0.5).astype(np.float32)
    tokens = rng.integers(0, dims["vocab"], 13).astype(np.int32)

    om = bind.OracleModel(orc, dims, embed, {}, f32=f32)
    kv = om.kv(dims["layers"], 32)
    x = om.stack_forward(0, kv, embed[tokens], 0, np.arange(len(tokens)))
    lg = om.lm_logits(x[-1:])[0]

    layers_w = [tuple(f32[(0, l, p)] for p in range(7)) for l in range(dims["layers"])]
    rtok, rlg = ref.model_forward_f32(dims, embed, layers_w, f32[(3, 0, 1)], tokens)
    np.testing.assert_allclose(lg, rlg, rtol=1e-4, atol=1e-4 * np.abs(rlg).max())
    assert int(np.argmax(lg)) == rtok
