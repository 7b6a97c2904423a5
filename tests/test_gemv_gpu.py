"""INT8 GEMV / skinny GEMM on the GPU through the C ABI against the oracle.

- per-(m, n, block) INT32 dot products: bit-exact;
- per-row (reference) mode: float outputs bit-exact with the reference's own
  matmul_dequantized, including the int16 pair saturation of (q-8)*16 weights;
- block mode: within 1e-5 of the row's largest |value| (only the order of
  the float additions differs from the oracle).
"""
import ctypes as C

import numpy as np
import pytest

import flb200
from flb200 import block_tensor, ptr, row_tensor

pytestmark = pytest.mark.gpu

SHAPES = [(9216, 3072), (16384, 3072), (3072, 8192), (3072, 3072), (32064, 3072)]


class Dev:
    """Device buffer helper through the C ABI."""

    def __init__(self, lib, nbytes):
        self.lib = lib
        self.p = C.c_void_p()
        lib.check(lib.fl_cuda_malloc(C.byref(self.p), max(nbytes, 16)), "malloc")
        self.n = nbytes

    def put(self, a):
        self.lib.check(self.lib.fl_cuda_h2d(self.p, ptr(a), a.nbytes), "h2d")
        return self

    def get(self, a):
        self.lib.check(self.lib.fl_cuda_sync(), "sync")
        self.lib.check(self.lib.fl_cuda_d2h(ptr(a), self.p, a.nbytes), "d2h")
        return a

    def __del__(self):
        try:
            self.lib.fl_cuda_free(self.p)
        except Exception:
            pass


def gpu_matmul(lib, A, t, N):
    M, K = A.shape
    dA = Dev(lib, A.nbytes).put(A)
    dC = Dev(lib, M * N * 4)
    lib.check(lib.fl_cuda_upload_tensor(C.byref(t)), "upload")
    lib.check(lib.fl_cuda_matmul_i8(dA.p, C.byref(t), dC.p, M, N, K, None), "matmul")
    return dC.get(np.empty((M, N), np.float32))


def gpu_dots(lib, A, t, N):
    M, K = A.shape
    dA = Dev(lib, A.nbytes).put(A)
    dD = Dev(lib, M * N * (K // 32) * 4)
    lib.check(lib.fl_cuda_upload_tensor(C.byref(t)), "upload")
    lib.check(lib.fl_cuda_block_dots_i8(dA.p, C.byref(t), dD.p, M, N, K, None), "dots")
    return dD.get(np.empty((M, N, K // 32), np.int32))


def assert_block_close(got, want):
    scale = np.abs(want).max(axis=1, keepdims=True) + 1e-30
    err = np.abs(got - want) / scale
    assert err.max() < 1e-5, f"max row-relative error {err.max():.3g}"


@pytest.mark.parametrize("N,K", SHAPES)
@pytest.mark.parametrize("M", [1, 5])
def test_block_mode_config_shapes(gpu, orc, N, K, M):
    lib = gpu
    w, d = lib.synth_q4_0_i8(11, 1000 + N + K, N, K)
    A = np.random.default_rng(M * 7 + N).standard_normal((M, K)).astype(np.float32)
    t = block_tensor(w, d)
    got = gpu_matmul(lib, A, t, N)
    assert_block_close(got, orc.matmul_block(A, w, d))
    lib.fl_cuda_sync()


@pytest.mark.parametrize("N,K", [(3072, 3072), (32064, 3072)])
@pytest.mark.parametrize("M", [17, 64, 256])
def test_block_mode_larger_m(gpu, orc, N, K, M):
    lib = gpu
    w, d = lib.synth_q4_0_i8(12, 2000 + N, N, K)
    A = np.random.default_rng(M).standard_normal((M, K)).astype(np.float32)
    got = gpu_matmul(lib, A, block_tensor(w, d), N)
    assert_block_close(got, orc.matmul_block(A, w, d))


@pytest.mark.parametrize("N,K", SHAPES)
@pytest.mark.parametrize("M", [17, 24, 33, 65, 129, 256])
def test_tcgen05_gemm_bit_exact(gpu, orc, N, K, M):
    """More than 16 rows run through the tcgen05 INT8 GEMM: its block-scaled
    result is bit-identical to the oracle's sequential block order, on every
    config shape (two weight panels at K = 8192, a partial 128-row tile at
    N = 32064) and ragged row counts."""
    lib = gpu
    w, d = lib.synth_q4_0_i8(13, 3000 + N + K, N, K)
    A = np.random.default_rng(M * 3 + K).standard_normal((M, K)).astype(np.float32)
    got = gpu_matmul(lib, A, block_tensor(w, d), N)
    want = orc.matmul_block(A, w, d)
    bad = np.argwhere(got != want)
    assert bad.size == 0, f"{len(bad)} outputs differ, first {bad[:3].tolist()}: {got[tuple(bad[0])]} vs {want[tuple(bad[0])]}"


@pytest.mark.parametrize("M,N,K", [(1, 9216, 3072), (5, 3072, 8192), (3, 37, 96), (8, 1, 32), (9, 64, 64)])
def test_block_dots_bit_exact(gpu, orc, M, N, K):
    lib = gpu
    w, d = lib.synth_q4_0_i8(13, 3000 + N, N, K)
    A = np.random.default_rng(N + M).standard_normal((M, K)).astype(np.float32)
    assert np.array_equal(gpu_dots(lib, A, block_tensor(w, d), N), orc.block_dots(A, w))


@pytest.mark.parametrize("scale16", [True, False])
@pytest.mark.parametrize("M,N,K", [(1, 3072, 3072), (5, 1100, 3072), (2, 333, 8192)])
def test_row_mode_bit_exact_with_reference(gpu, ref, scale16, M, N, K):
    """Reference-format tensor ((q-8)*16, per-row scale): the GPU output is the
    reference's matmul_dequantized float for float."""
    lib = gpu
    rng = np.random.default_rng(N)
    q = rng.integers(0, 16, (N, K)) - 8
    W = (np.clip(q * 16, -128, 127) if scale16 else q).astype(np.int8)
    s = (rng.random(N) * 0.01 + 1e-4).astype(np.float32)
    A = rng.standard_normal((M, K)).astype(np.float32)
    got = gpu_matmul(lib, A, row_tensor(W, s), N)
    assert np.array_equal(got, ref.matmul_dequantized(A, W, s))


def test_matmul_dequantized_host_api(gpu, ref, orc):
    """The reference entry point itself (host A / C), both tensor modes."""
    lib = gpu
    rng = np.random.default_rng(5)
    M, N, K = 4, 2048, 3072
    A = rng.standard_normal((M, K)).astype(np.float32)
    W = np.clip((rng.integers(0, 16, (N, K)) - 8) * 16, -128, 127).astype(np.int8)
    s = (rng.random(N) * 0.01).astype(np.float32)
    t = row_tensor(W, s)
    Cg = np.empty((M, N), np.float32)
    lib.matmul_dequantized(ptr(A), C.byref(t), ptr(Cg), M, N, K)
    assert np.array_equal(Cg, ref.matmul_dequantized(A, W, s))
    w, d = lib.synth_q4_0_i8(3, 77, N, K)
    tb = block_tensor(w, d)
    lib.matmul_dequantized(ptr(A), C.byref(tb), ptr(Cg), M, N, K)
    assert_block_close(Cg, orc.matmul_block(A, w, d))


def test_activation_edge_values(gpu, orc):
    """NaN, +-inf, huge and tie values quantize like the reference's x86 path
    (out-of-range -> 0, not 255), visible in the block dots."""
    lib = gpu
    K = 64
    A = np.zeros((1, K), np.float32)
    A[0, :16] = [np.nan, np.inf, -np.inf, 1e30, -1e30, 2e7, -2e7, 0.5 / 127, 1.5 / 127, -0.5 / 127, 1.0, -1.0,
                 127.5 / 127, -128.5 / 127, 3.0, -3.0]
    w = np.ones((2, K), np.int8)
    d = np.full((2, K // 32), np.float16(1.0).view(np.uint16), np.uint16)
    assert np.array_equal(gpu_dots(lib, A, block_tensor(w, d), 2), orc.block_dots(A, w))


def test_act_quant_rmsnorm(gpu, orc):
    """RMSNorm + quantization kernel: u8 codes equal the oracle's except where
    the normalised value sits within float rounding of a code boundary."""
    lib = gpu
    M, K = 5, 3072
    X = (np.random.default_rng(9).standard_normal((M, K)) * 7).astype(np.float32)
    dX = Dev(lib, X.nbytes).put(X)
    dQ = Dev(lib, M * K)
    lib.check(lib.fl_cuda_act_quant(dX.p, dQ.p, M, K, 1, 1e-5, None), "act_quant")
    q = dQ.get(np.empty((M, K), np.uint8))
    want = np.stack([orc.quant_u8(orc.rmsnorm(X[m])) for m in range(M)])
    diff = np.abs(q.astype(int) - want.astype(int))
    assert diff.max() <= 1 and (diff != 0).mean() < 1e-3


def test_rejects_bad_shapes(gpu):
    lib = gpu
    w, d = lib.synth_q4_0_i8(1, 1, 8, 64)
    t = block_tensor(w, d)
    lib.check(lib.fl_cuda_upload_tensor(C.byref(t)), "upload")
    dA = Dev(lib, 4 * 64)
    dC = Dev(lib, 4 * 8)
    assert lib.fl_cuda_matmul_i8(dA.p, C.byref(t), dC.p, 1, 8, 48, None) != 0  # K % 32
    assert lib.fl_cuda_matmul_i8(dA.p, C.byref(t), dC.p, 1, 9, 64, None) != 0  # N mismatch
    assert "K" in lib.err() or "N" in lib.err()
