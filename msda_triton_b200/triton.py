"""Import path of the reference's kernel backend, for a drop-in rename.

`from msda_triton.triton import MSDA3DFn` becomes
`from msda_triton_b200.triton import MSDA3DFn`: the same six names as
src/msda_triton/triton/__init__.py:10-22, bound to this package's CUDA ops
(nothing here uses the Triton compiler).
"""

from msda_triton_b200.msda_2d import MSDA2DFn, msda2d, msda2d_fwd
from msda_triton_b200.msda_3d import MSDA3DFn, msda3d, msda3d_fwd

__all__ = ["msda2d", "msda2d_fwd", "MSDA2DFn", "msda3d", "msda3d_fwd", "MSDA3DFn"]
