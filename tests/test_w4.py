"""Packed 4-bit weights through the C ABI against the oracle.

The block-mode INT8 weights are Q4_0 nibbles minus 8, so the 4-bit copy is
lossless: fl_cuda_block_dots_w4 must give exactly the int32 block dots of the
oracle (the kernel dots q = w + 8 and subtracts 8 x the block's activation
sum), and an engine switched to 4-bit weights (fl_engine_set_weight_bits)
must give the INT8 engine's logits up to the order of the float additions
and the oracle's greedy stream."""
import ctypes as C

import numpy as np
import pytest

import flb200
from flb200 import block_tensor
from _model import SMALL, engine_cfg, load_engine, make_weights, prompt

pytestmark = pytest.mark.gpu


class Dev:
    def __init__(self, lib, nbytes):
        self.lib = lib
        self.p = C.c_void_p()
        lib.check(lib.fl_cuda_malloc(C.byref(self.p), max(nbytes, 16)), "malloc")

    def put(self, a):
        self.lib.check(self.lib.fl_cuda_h2d(self.p, flb200.ptr(a), a.nbytes), "h2d")
        return self

    def get(self, out):
        self.lib.check(self.lib.fl_cuda_sync(), "sync")
        self.lib.check(self.lib.fl_cuda_d2h(flb200.ptr(out), self.p, out.nbytes), "d2h")
        return out

    def __del__(self):
        try:
            self.lib.fl_cuda_free(self.p)
        except Exception:
            pass


def dots_w4(lib, A, t, N):
    M, K = A.shape
    dA = Dev(lib, A.nbytes).put(A)
    dD = Dev(lib, M * N * (K // 32) * 4)
    lib.check(lib.fl_cuda_upload_tensor(C.byref(t)), "upload")
    lib.check(lib.fl_cuda_block_dots_w4(dA.p, C.byref(t), dD.p, M, N, K, None), "dots_w4")
    return dD.get(np.empty((M, N, K // 32), np.int32))


@pytest.mark.parametrize("M,N,K", [(1, 9216, 3072), (5, 3072, 8192), (8, 16384, 3072), (3, 264, 256),
                                   (2, 32064, 3072), (4, 3072, 3072)])
def test_block_dots_w4_bit_exact(gpu, orc, M, N, K):
    w, d = gpu.synth_q4_0_i8(17, 4000 + N + K, N, K)
    A = np.random.default_rng(M * 11 + N).standard_normal((M, K)).astype(np.float32)
    A[0, :32] = 4.0   # quantizes to 255 (largest u8 sum of a block)
    A[-1, 32:64] = -4.0  # quantizes to 0
    w[0, :32] = -8    # every weight at its extremes
    w[1 % N, :32] = 7
    got = dots_w4(gpu, A, block_tensor(w, d), N)
    want = orc.block_dots(A, w)
    bad = np.argwhere(got != want)
    assert bad.size == 0, f"{len(bad)} dots differ, first {bad[:3].tolist()}"


def test_block_dots_w4_rejects_out_of_range(gpu):
    w, d = gpu.synth_q4_0_i8(17, 5000, 64, 256)
    w[3, 5] = 9
    A = np.ones((1, 256), np.float32)
    dA = Dev(gpu, A.nbytes).put(A)
    dD = Dev(gpu, 64 * 8 * 4)
    t = block_tensor(w, d)
    gpu.check(gpu.fl_cuda_upload_tensor(C.byref(t)), "upload")
    assert gpu.fl_cuda_block_dots_w4(dA.p, C.byref(t), dD.p, 1, 64, 256, None) != 0


def test_engine_w4_logits_and_stream(gpu, orc):
    import bind
    dims = SMALL
    w, embed = make_weights(gpu, dims, seed=31, draft_layers=1)
    eng = flb200.Engine(gpu, engine_cfg(dims, draft_layers=1))
    load_engine(eng, w, embed)
    toks = prompt(2, 8, dims["vocab"])
    x0 = embed[toks]
    _, lg8 = eng.forward_rows(0, x0, 0, np.arange(8))
    p = prompt(5, 16, dims["vocab"])
    s8, a8 = eng.spec_generate(p, 24, 4)
    eng.set_weight_bits(4)
    _, lg4 = eng.forward_rows(0, x0, 0, np.arange(8))
    s4, a4 = eng.spec_generate(p, 24, 4)
    eng.set_weight_bits(8)
    s8b, _ = eng.spec_generate(p, 24, 4)
    eng.close()
    err = np.abs(lg4 - lg8) / np.abs(lg8).max(axis=-1, keepdims=True)
    assert err.max() < 1e-5, f"4-bit logits differ from INT8 by {err.max():.3g} of the row max"
    om = bind.OracleModel(orc, dims, embed, w, draft_layers=1)
    want, _, margins = om.spec(p, 24, 4)
    for got in (s4, s8, s8b):
        diff = np.nonzero(np.asarray(got) != want)[0]
        assert diff.size == 0 or margins[int(diff[0])] < 1e-2, f"stream diverges at {diff[:3]}"
    assert np.array_equal(s8, s8b)
