"""CPU: expf_ref (moe.cc_b200/csrc/expf_ref.h), the device kernels' expf,
equals the C library's expf (what the reference calls for the softmax and
SiLU, test_model_trace.c:233,485) on every one of the 2^32 float inputs, and
its table holds the doubles nearest 2^(j/32)."""
import os
import re
import subprocess
from decimal import Decimal, getcontext
from fractions import Fraction

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))


def test_expf_ref_equals_libc_expf_exhaustively(tmp_path):
    exe = str(tmp_path / "expf_check")
    cc = subprocess.run(["gcc", "-O2", "-fopenmp", "-ffp-contract=off", "-mfma", "-o", exe,
                         os.path.join(HERE, "expf_check.c"), "-lm"], capture_output=True, text=True)
    if cc.returncode != 0:
        pytest.skip("no gcc with FMA here: " + cc.stderr[-200:])
    r = subprocess.run([exe], capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stderr
    assert "expf_ref mismatches: 0" in r.stdout, r.stdout[:500]
    # the double-precision shortcut it replaces is not enough
    m = re.search(r"double exp rounded once, mismatches: (\d+)", r.stdout)
    assert m and int(m.group(1)) > 0
    # table: the double nearest 2^(j/32), from 60-digit decimal arithmetic
    getcontext().prec = 60
    for j in range(32):
        want = float(Fraction(Decimal(2) ** (Decimal(j) / Decimal(32))))
        got = float.fromhex(re.search(rf"^t{j}=(\S+)$", r.stdout, re.M).group(1))
        assert got == want, (j, got.hex(), want.hex())
