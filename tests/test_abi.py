"""The C-ABI library loads without a GPU and exports every function that
include/*.h declares (no compute calls here)."""
import ctypes
import glob
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    names = set()
    for path in glob.glob(os.path.join(ROOT, "include", "*.h")):
        src = open(path).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        src = re.sub(r"//[^\n]*", "", src)
        src = re.sub(r"#[^\n]*(\\\n[^\n]*)*", "", src)          # preprocessor lines
        src = re.sub(r"static\s+inline[^{]*\{[^}]*\}", "", src)  # inline helpers
        for stmt in src.split(";"):
            m = re.search(r"\b([A-Za-z_]\w*)\s*\(", stmt)
            if not m or "typedef" in stmt:
                continue
            names.add(m.group(1))
    return sorted(names)


def test_headers_declare_the_reference_api():
    names = set(declared_functions())
    for required in ("matmul_dequantized", "dequantized_from_q4", "dequantized_from_q8", "dequantized_tensor_free",
                     "draft_model_create", "draft_tokens", "verify_tokens", "speculative_decode_step",
                     "speculative_generate", "medusa_model_create", "medusa_predict", "medusa_build_tree",
                     "medusa_verify_tree", "medusa_decode_step", "medusa_generate",
                     "speculative_medusa_generate"):
        assert required in names


@pytest.mark.parametrize("name", declared_functions())
def test_library_exports(lib, name):
    assert hasattr(lib.so, name), f"{name} is declared in include/ but not exported by {lib.path}"


def test_library_is_sm100a_only():
    """The shared object carries an sm_100a fatbin and nothing else is needed
    at load time (the GPU itself is only touched by compute calls)."""
    import flb200
    assert os.path.exists(flb200.LIB_PATH)
    ctypes.CDLL(flb200.LIB_PATH)
