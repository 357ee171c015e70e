"""CPU oracle for multi-scale deformable attention -- TEST INFRASTRUCTURE ONLY.

This package is the checker: tests/, __graft_entry__.smoke() and bench.py's
cpu_baseline / reference arm may import it.  The product package
(msda_triton_b200) never imports it and has no CPU fallback.

The oracle restates the reference's pure-PyTorch path
(src/msda_triton/pytorch/msda_2d.py:23-114 and
src/msda_triton/pytorch/msda_3d.py:23-118) in C (msda_oracle.c).  It is pinned
against golden vectors produced by that reference path (tests/golden/).
"""

from oracle.oracle import msda_bwd_oracle, msda_cell_oracle, msda_fwd_oracle

__all__ = ["msda_fwd_oracle", "msda_bwd_oracle", "msda_cell_oracle"]
