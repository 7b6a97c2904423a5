"""fl_cuda_block_dots_i8_noalloc: the allocation-free variant of
fl_cuda_block_dots_i8 (fixed static device scratch of
FL_NOALLOC_SCRATCH_BYTES). Collected last (file name) so that it also runs
after every other test; it must pass alone as well.

- CPU: a call whose M * K exceeds the scratch fails with FL_E_INVAL before
  touching the device;
- GPU: two calls in a row on one stream give exactly the integers of the
  allocating entry point and of the oracle's pair-saturated block dots, in
  block and per-row tensor modes, up to a call that fills the whole scratch;
  the same on a caller-created stream passed explicitly.
"""
import ctypes as C

import numpy as np
import pytest

from flb200 import block_tensor, row_tensor

SCRATCH = 1 << 20  # FL_NOALLOC_SCRATCH_BYTES in include/fl_cuda.h
FL_E_INVAL = -1


def test_oversize_rejected_without_device(lib):
    dummy = C.c_void_p(256)  # never dereferenced: the size check comes first
    M, K = 33, 32768         # M * K = 1 081 344 > 1 MiB
    assert M * K > SCRATCH
    rc = lib.fl_cuda_block_dots_i8_noalloc(dummy, None, dummy, M, 64, K, None)
    assert rc == FL_E_INVAL
    assert "exceeds the static scratch" in lib.err()


@pytest.mark.gpu
@pytest.mark.parametrize("mode", ["block", "row"])
def test_noalloc_matches_allocating_entry_point(gpu, orc, mode):
    from test_gemv_gpu import Dev
    lib = gpu
    rng = np.random.default_rng(77)
    cases = [(5, 1100, 3072), (3, 333, 8192), (SCRATCH // 8192, 64, 8192)]  # the last fills the scratch
    tensors, inputs, host = [], [], []
    for M, N, K in cases:
        if mode == "block":
            W, d = lib.synth_q4_0_i8(17, 5000 + N + K, N, K)
            t = block_tensor(W, d)
        else:
            W = np.clip((rng.integers(0, 16, (N, K)) - 8) * 16, -128, 127).astype(np.int8)
            t = row_tensor(W, (rng.random(N) * 0.01 + 1e-4).astype(np.float32))
        lib.check(lib.fl_cuda_upload_tensor(C.byref(t)), "upload")
        A = rng.standard_normal((M, K)).astype(np.float32)
        tensors.append(t)
        inputs.append(Dev(lib, A.nbytes).put(A))
        host.append((A, W))
    for i in range(0, len(cases), 2):
        pair = cases[i:i + 2]
        outs = []
        # two calls in a row on the library stream, no synchronisation between
        for j, (M, N, K) in enumerate(pair):
            dD = Dev(lib, M * N * (K // 32) * 4)
            lib.check(lib.fl_cuda_block_dots_i8_noalloc(inputs[i + j].p, C.byref(tensors[i + j]), dD.p, M, N, K,
                                                        None), "noalloc")
            outs.append(dD)
        for j, (M, N, K) in enumerate(pair):
            got = outs[j].get(np.empty((M, N, K // 32), np.int32))
            dW = Dev(lib, M * N * (K // 32) * 4)
            lib.check(lib.fl_cuda_block_dots_i8(inputs[i + j].p, C.byref(tensors[i + j]), dW.p, M, N, K, None),
                      "dots")
            want = dW.get(np.empty((M, N, K // 32), np.int32))
            assert np.array_equal(got, want), f"case {pair[j]} differs"
            A, W = host[i + j]
            assert np.array_equal(got, orc.block_dots(A, W)), f"case {pair[j]} differs from the oracle"


@pytest.mark.gpu
def test_noalloc_on_caller_stream(gpu, orc):
    """The stream argument: two calls in a row on a stream the caller made,
    read back after synchronising that stream, equal the oracle's dots."""
    import torch
    from test_gemv_gpu import Dev
    lib = gpu
    rng = np.random.default_rng(78)
    s = torch.cuda.Stream()
    M, N, K = 4, 700, 3072
    W, d = lib.synth_q4_0_i8(19, 6000, N, K)
    t = block_tensor(W, d)
    lib.check(lib.fl_cuda_upload_tensor(C.byref(t)), "upload")
    lib.check(lib.fl_cuda_sync(), "sync")
    outs = []
    for call in range(2):
        A = rng.standard_normal((M, K)).astype(np.float32)
        dA = Dev(lib, A.nbytes).put(A)
        dD = Dev(lib, M * N * (K // 32) * 4)
        lib.check(lib.fl_cuda_block_dots_i8_noalloc(dA.p, C.byref(t), dD.p, M, N, K, C.c_void_p(s.cuda_stream)),
                  "noalloc on a caller stream")
        outs.append((A, dA, dD))
    s.synchronize()
    for A, _, dD in outs:
        got = dD.get(np.empty((M, N, K // 32), np.int32))
        assert np.array_equal(got, orc.block_dots(A, W))
