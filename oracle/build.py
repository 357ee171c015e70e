"""Build recipe for the CPU oracle (test infrastructure only).

Compiles oracle/msda_oracle.c into oracle/_build/libmsda_oracle.so with
OpenMP.  -ffp-contract=off keeps every coordinate operation a separate float
rounding, as the restated algorithm is written.
"""

from __future__ import annotations

import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "msda_oracle.c")
OUT_DIR = os.path.join(HERE, "_build")
LIB = os.path.join(OUT_DIR, "libmsda_oracle.so")


def build(force: bool = False) -> str:
    """Compile the oracle if the library is missing or older than its source."""
    if (
        not force
        and os.path.exists(LIB)
        and os.path.getmtime(LIB) >= os.path.getmtime(SRC)
    ):
        return LIB
    os.makedirs(OUT_DIR, exist_ok=True)
    cmd = [
        "gcc", "-O2", "-fopenmp", "-ffp-contract=off", "-fno-fast-math",
        "-fPIC", "-shared", "-std=c11", "-Wall", "-Wextra",
        SRC, "-o", LIB + ".tmp", "-lm",
    ]
    subprocess.run(cmd, check=True)
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    print(build(force=True))
