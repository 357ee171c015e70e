"""msda_triton_b200 -- B200-native (sm_100a) multi-scale deformable attention.

Drop-in replacement for the public API of mach9robotics/msda-triton
(src/msda_triton/__init__.py:16-26 and src/msda_triton/triton/__init__.py:10-22):

    from msda_triton_b200 import msda2d, msda2d_fwd, msda3d, msda3d_fwd
    from msda_triton_b200 import MSDA2DFn, MSDA3DFn
    from msda_triton_b200 import MSDA2D, MSDA3D   # the nn.Modules (msda_triton.pytorch)

The ops run in hand-written CUDA kernels (libmsda_b200.so, C ABI in
include/msda_b200.h).  There is no CPU fallback: CPU tensors raise
ValueError, and a missing library raises RuntimeError at the first call.
"""

from __future__ import annotations

__version__ = "0.1.0"

from msda_triton_b200.msda_2d import MSDA2DFn, msda2d, msda2d_fwd
from msda_triton_b200.msda_3d import MSDA3DFn, msda3d, msda3d_fwd
from msda_triton_b200.fused import msda2d_fused, msda3d_fused
from msda_triton_b200.modules import MSDA2D, MSDA3D

__all__ = [
    "__version__",
    "msda2d",
    "msda2d_fwd",
    "MSDA2DFn",
    "msda3d",
    "msda3d_fwd",
    "MSDA3DFn",
    "MSDA2D",
    "MSDA3D",
    "msda2d_fused",
    "msda3d_fused",
]
