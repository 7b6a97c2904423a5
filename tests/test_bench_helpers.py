"""Host-side helpers of bench.py (no GPU): the roofline traffic read from the
committed ncu summary, the algorithmic byte counts, the CPU/GPU stream
comparison and the OpenMP thread split under torchrun."""
import importlib
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
bench = importlib.import_module("bench")


def test_traffic_comes_from_the_committed_profile():
    t = bench.profiled_traffic("gemv_tma_gateup_16384x3072.md", 5)
    # dram read + write of one launch: the algorithmic 53.48 MB plus a few
    # hundred KB of activations and outputs, never less than the weights
    assert t is not None and 53.48e6 <= t <= 54.0e6
    assert bench.profiled_traffic("gemv_tma_gateup_16384x3072.md", 3) is None
    assert bench.profiled_traffic("no_such_summary.md", 5) is None


def test_step_bytes():
    full = bench.step_bytes(4, 192)
    half = bench.step_bytes(4, 192, 0.5)
    # 6.41 GB per config-0 step; packed 4-bit weights halve the weight bytes
    assert abs(full - 6.412e9) < 0.01e9
    assert 0.5 < half / full < 0.56
    # a Medusa tree step streams the base once and the LM head once per 8 rows
    assert bench.medusa_step_bytes(64, 4, 0) > bench.medusa_step_bytes(8, 4, 0)


def test_stream_check():
    cpu = np.array([5, 6, 7, 8])
    m = np.array([0.5, 0.4, 0.001, 0.3])
    same = bench.stream_check(cpu, m, np.array([5, 6, 7, 8]))
    assert same == {"tokens": 4, "identical_prefix": 4}
    part = bench.stream_check(cpu, m, np.array([5, 6, 9, 9]))
    assert part["identical_prefix"] == 2 and abs(part["margin_at_divergence"] - 0.001) < 1e-9


def test_thread_split(monkeypatch):
    cores = os.cpu_count() or 1
    monkeypatch.setenv("WORLD_SIZE", "4")
    monkeypatch.setenv("LOCAL_WORLD_SIZE", "4")
    monkeypatch.setenv("OMP_NUM_THREADS", "1")  # what torchrun exports
    bench.split_host_threads("b200")
    assert os.environ["OMP_NUM_THREADS"] == str(max(1, cores // 4))
    monkeypatch.setenv("OMP_NUM_THREADS", "1")
    bench.split_host_threads("reference")
    assert os.environ["OMP_NUM_THREADS"] == str(cores)
    monkeypatch.setenv("OMP_NUM_THREADS", "3")  # set by the user: kept
    bench.split_host_threads("b200")
    assert os.environ["OMP_NUM_THREADS"] == "3"
