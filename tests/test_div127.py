"""The division by 127 of the GEMV / GEMM epilogues (div127 in
fl_common.cuh: one multiply by RN(1/127), a fused residual correction and
the sign of y on a zero result) against the correctly rounded quotient,
modelled on the host in C with the same operations: every float of the
subnormal binade, the smallest normal binades, the binades of the epilogue's
values (about 2^-8 .. 2^8 and beyond) and the largest, both signs. The
device results are checked bit for bit against the oracle by the GEMV and
GEMM parity tests."""
import os
import shutil
import subprocess

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.mark.skipif(shutil.which("gcc") is None, reason="needs gcc")
def test_div127_matches_correct_rounding(tmp_path):
    exe = tmp_path / "div127_check"
    subprocess.run(["gcc", "-O2", "-ffp-contract=off", "-o", str(exe), os.path.join(HERE, "div127_check.c"), "-lm"],
                   check=True)
    r = subprocess.run([str(exe), "0", "2", "115", "140", "252", "254"], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "bad 0" in r.stdout
