"""Host-side generator and loader logic (no GPU): Philox known answers, the
seeded N(0, std) -> Q4_0 -> INT8 path against the oracle's Q4_0 quantizer,
GGUF nibble order, and determinism."""
import numpy as np

from flb200 import tensor_id

# Philox4x32-10 known-answer vectors published with Random123 (kat_vectors):
# (counter, key) -> output.
PHILOX_KAT = [
    ((0, 0, 0, 0), (0, 0), (0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8)),
    ((0xFFFFFFFF,) * 4, (0xFFFFFFFF,) * 2, (0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD)),
    ((0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344), (0xA4093822, 0x299F31D0),
     (0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1)),
]


def test_philox_known_answers(lib, orc):
    for ctr, key, want in PHILOX_KAT:
        assert tuple(int(v) for v in lib.philox(ctr, key)) == want
        assert tuple(int(v) for v in orc.philox(ctr, key)) == want


def test_synth_q4_0_matches_oracle_quantizer(lib, orc):
    rows, cols = 37, 256
    seed, tid = 1234, tensor_id(0, 3, 4)
    w, d = lib.synth_q4_0_i8(seed, tid, rows, cols, 0.02)
    x = lib.synth_normal(seed, tid, rows * cols, 0.02)
    w2, d2 = orc.q4_0_i8(x)
    assert np.array_equal(w.reshape(-1), w2)
    assert np.array_equal(d.reshape(-1), d2)
    assert w.min() >= -8 and w.max() <= 7
    # each block holds its extreme value at -8 (d = max / -8)
    assert (w.reshape(-1, 32).min(axis=1) == -8).all()


def test_synth_statistics_and_determinism(lib):
    x = lib.synth_normal(7, 99, 1 << 18, 0.02)
    assert abs(x.mean()) < 2e-4 and abs(x.std() - 0.02) < 2e-4
    assert np.array_equal(x, lib.synth_normal(7, 99, 1 << 18, 0.02))
    assert not np.array_equal(x, lib.synth_normal(8, 99, 1 << 18, 0.02))
    f = lib.synth_q4_0_f32(7, 5, 16, 64)
    w, d = lib.synth_q4_0_i8(7, 5, 16, 64)
    dd = d.view(np.float16).astype(np.float32)
    assert np.array_equal(f, w.astype(np.float32) * np.repeat(dd, 32, axis=1))


def test_gguf_q4_0_nibble_order(lib):
    """gguf_loader.c:147-161: byte i holds element i (low) and i+16 (high)."""
    import ctypes
    blk = np.zeros(18, np.uint8)
    blk[0:2] = np.frombuffer(np.float16(0.5).tobytes(), np.uint8)
    blk[2:18] = [(i & 0xF) | (((15 - i) & 0xF) << 4) for i in range(16)]
    w = np.empty(32, np.int8)
    d = np.empty(1, np.uint16)
    lib.check(lib.fl_q4_0_to_i8(blk.ctypes.data, 1, 32, w.ctypes.data, d.ctypes.data), "q4_0_to_i8")
    assert list(w[:16]) == [i - 8 for i in range(16)]
    assert list(w[16:]) == [(15 - i) - 8 for i in range(16)]
    assert d[0] == np.float16(0.5).view(np.uint16)


def test_block_synthesis_is_a_slice(lib):
    """A tensor-parallel rank generates only its block; it must equal that
    block of the whole tensor."""
    import numpy as np
    from flb200 import ptr
    rows, cols = 96, 256
    w, d = lib.synth_q4_0_i8(9, 77, rows, cols)
    for r0, nr, c0, nc in [(0, 96, 0, 256), (32, 40, 0, 256), (0, 96, 64, 128), (17, 5, 224, 32)]:
        wb = np.empty((nr, nc), np.int8)
        db = np.empty((nr, nc // 32), np.uint16)
        assert lib.fl_synth_q4_0_i8_block(9, 77, rows, cols, r0, nr, c0, nc, 0.02, ptr(wb), ptr(db)) == 0
        assert np.array_equal(wb, w[r0:r0 + nr, c0:c0 + nc])
        assert np.array_equal(db, d[r0:r0 + nr, c0 // 32:(c0 + nc) // 32])
    wb = np.empty((4, 30), np.int8)
    assert lib.fl_synth_q4_0_i8_block(9, 77, rows, cols, 0, 4, 2, 30, 0.02, ptr(wb), ptr(wb)) != 0


def test_oracle_generator_equals_library(lib, orc):
    """The oracle's restatement of the seeded generator (used where no
    product code may run, e.g. the CPU baseline) gives the library's bits."""
    for seed, tid, rows, cols, std in ((1, tensor_id(0, 0, 0), 9, 3072, 0.02), (7, tensor_id(3, 0, 0), 5, 96, 50.0),
                                       (2 ** 40 + 3, tensor_id(1, 2, 6), 3, 8192, 0.02)):
        w, d = lib.synth_q4_0_i8(seed, tid, rows, cols, std)
        w2, d2 = orc.synth_q4_0_i8(seed, tid, rows, cols, std)
        assert np.array_equal(w, w2) and np.array_equal(d, d2)
        assert np.array_equal(lib.synth_q4_0_f32(seed, tid, rows, cols, std), orc.synth_q4_0_f32(seed, tid, rows, cols, std))
