"""Import path of the reference's module backend, for a drop-in rename.

`from msda_triton.pytorch import MSDA3D` becomes
`from msda_triton_b200.pytorch import MSDA3D`: the nn.Modules of
src/msda_triton/pytorch/__init__.py:10-20, sampling in this package's CUDA
kernels.  The reference's grid_sample functions `msda2d_pytorch` /
`msda3d_pytorch` are its test oracle and are not part of this package.
"""

from msda_triton_b200.modules import MSDA2D, MSDA3D

__all__ = ["MSDA2D", "MSDA3D"]
