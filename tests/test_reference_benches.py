"""The reference's own callers of the API, unmodified: its benchmark programs
fast_llm/benchmarks/bench_speculative.c and bench_medusa.c, compiled against
include/ and linked to libfl_b200.so by oracle/Makefile (built where the
reference sources are, then shipped with the repository). They pass their
own host callbacks (a 50 ms busy-wait "target" writing random values) with
target_model / base_model NULL, prompt_len 1 and temperature 0.8, on a
draft / Medusa model that was created but never loaded; they must run to
completion and generate all 20 tokens."""
import os
import re
import subprocess

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "oracle", "_ref")


@pytest.mark.parametrize("prog,label", [("bench_speculative", "Generated: 20 tokens"),
                                        ("bench_medusa", "Generated: 20 tokens")])
def test_reference_benchmark_program_runs(gpu, prog, label):
    exe = os.path.join(REF, prog)
    if not os.path.exists(exe):
        pytest.skip(f"{exe} not built (the reference sources were absent at build time)")
    r = subprocess.run([exe], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    assert label in r.stdout, r.stdout[-2000:]
    m = re.search(r"Speed:\s+([0-9.]+) tok/sec\n\s+Generated", r.stdout)
    assert m and float(m.group(1)) > 0
