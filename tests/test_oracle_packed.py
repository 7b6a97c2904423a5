"""The oracle's packed block matmul (orc_pack_rows8 + orc_matmul_packed),
the kernel the CPU baseline decodes with, against the oracle's
one-block-at-a-time block matmul: every result bit-identical, for row counts
that fill and do not fill its four-row activation groups, and the packing's
refusals."""
import numpy as np
import pytest


@pytest.mark.parametrize("M,N,K", [(1, 8, 32), (3, 40, 96), (4, 64, 3072), (5, 1024, 3072), (9, 24, 256),
                                   (17, 3072 // 8, 8192)])
def test_packed_equals_block_matmul(orc, M, N, K):
    rng = np.random.default_rng(M * 1000 + N)
    A = (rng.standard_normal((M, K)) * 0.7).astype(np.float32)
    if K >= 128:
        A[0, 64:68] = [3.0, -3.0, 0.5 / 127, -np.inf]  # clamps and a rounding tie
    W = rng.integers(-8, 8, (N, K)).astype(np.int8)
    W[0, :64] = -8  # the largest int16 partial sums: 16 products of 255 x -8
    A[0, :64] = 2.0
    d = (rng.standard_normal((N, K // 32)) * 0.01).astype(np.float16).view(np.uint16)
    wp, sp = orc.pack_rows8(W, d)
    got = orc.matmul_packed(A, wp, sp)
    want = orc.matmul_block(A, W, d)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_packed_synthetic_weights(orc):
    """Q4_0-generated weights of the gate/up shape at the verify width."""
    w, d = orc.synth_q4_0_i8(1, 7, 2048, 3072)
    A = np.random.default_rng(3).standard_normal((5, 3072)).astype(np.float32)
    wp, sp = orc.pack_rows8(w, d)
    assert np.array_equal(orc.matmul_packed(A, wp, sp).view(np.uint32), orc.matmul_block(A, w, d).view(np.uint32))


def test_pack_refuses(orc):
    d = np.zeros((16, 2), np.uint16)
    assert orc.pack_rows8(np.zeros((12, 64), np.int8), np.zeros((12, 2), np.uint16)) is None  # rows % 8
    w = np.zeros((16, 64), np.int8)
    w[3, 5] = 8  # outside [-8, 7]: int16 sums could overflow
    assert orc.pack_rows8(w, d) is None
    w[3, 5] = -9
    assert orc.pack_rows8(w, d) is None
