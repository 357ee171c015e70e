"""The bounds-checked build on the GPU (a memory checker that needs no
sanitizer): every value gather and value-gradient scatter of the kernels is
tested against its buffer, and tests/_checked_cases.py runs forward and
backward over dtypes, clamp modes, out-of-range locations, host/device
shapes, row shapes, the direct/accumulated value-gradient split and the fused
prologue.  No case may record a violation, and the fp32 cases must still
match the oracle."""

from __future__ import annotations

import json
import os
import subprocess
import sys

import pytest

from msda_triton_b200 import build as B

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_checked_build_records_no_violation():
    lib = B.CHECKED_LIB
    if not os.path.exists(lib):
        lib = B.build(checked=True)
    env = dict(os.environ, MSDA_B200_LIB=lib)
    res = subprocess.run([sys.executable, os.path.join(ROOT, "tests", "_checked_cases.py")],
                         env=env, capture_output=True, text=True, timeout=900)
    assert res.returncode == 0, res.stdout[-2000:] + res.stderr[-4000:]
    summary = json.loads(res.stdout.strip().splitlines()[-1])
    assert summary["cases"] >= 60
    assert summary["violations"] == [], summary["violations"]
    assert summary["parity_failures"] == [], summary["parity_failures"]
