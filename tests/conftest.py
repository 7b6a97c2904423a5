"""Shared fixtures. GPU tests carry @pytest.mark.gpu and call the product
through its C ABI (libfl_b200.so); CPU tests cover the oracle, the golden
vectors, the host logic and the library's exported symbols."""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "fast-llm-inference_b200")
for p in (PKG, os.path.join(ROOT, "oracle"), ROOT):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def lib():
    import flb200
    return flb200.Lib()


@pytest.fixture(scope="session")
def orc():
    import bind
    return bind.Oracle()


@pytest.fixture(scope="session")
def ref():
    import bind
    if not os.path.exists(bind.REF_SO):
        pytest.skip("oracle/_ref/libref.so not built (reference sources absent)")
    return bind.Ref()


@pytest.fixture(scope="session")
def gpu(lib):
    if lib.device_count() < 1:
        pytest.fail("GPU test without a CUDA device")
    lib.check(lib.fl_cuda_init(0), "fl_cuda_init")
    return lib
