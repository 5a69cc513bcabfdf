"""CPU: div_qscale, the epilogues' (float)dot / S (common.cuh), equals IEEE
round-to-nearest division for all 2^32 int32 dot products and both
quantisation divisors, so replacing the divide keeps every output bit."""
import os
import subprocess

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))


def test_reciprocal_correction_matches_ieee_division_exhaustively(tmp_path):
    exe = str(tmp_path / "divide_check")
    cc = subprocess.run(["gcc", "-O2", "-fopenmp", "-ffp-contract=off", "-mfma", "-o", exe,
                         os.path.join(HERE, "divide_check.c"), "-lm"], capture_output=True, text=True)
    if cc.returncode != 0:
        pytest.skip("no gcc with FMA here: " + cc.stderr[-200:])
    r = subprocess.run([exe], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr
    lines = [l for l in r.stdout.splitlines() if "mismatches" in l]
    assert len(lines) == 2, r.stdout
    for l in lines:
        assert l.rstrip().endswith(": 0"), l
    # the reciprocals hard-coded in common.cuh
    assert "r=0x1.020408p-7" in r.stdout and "r=0x1.24924ap-3" in r.stdout
