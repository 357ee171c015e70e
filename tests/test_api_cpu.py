"""The public import surface without a GPU: the reference's three import
paths (src/msda_triton/__init__.py:16-26, triton/__init__.py:10-22,
pytorch/__init__.py:10-20) exist under this package with the same names, and
CPU tensors get the reference's error instead of a silent fallback."""

from __future__ import annotations

import pytest
import torch

import msda_triton_b200 as top
from msda_triton_b200 import pytorch as pt_backend
from msda_triton_b200 import triton as kernel_backend

REFERENCE_TOP = ["msda2d", "msda2d_fwd", "msda3d", "msda3d_fwd"]
REFERENCE_TRITON = ["msda2d", "msda2d_fwd", "MSDA2DFn", "msda3d", "msda3d_fwd", "MSDA3DFn"]


def test_top_level_names():
    for name in REFERENCE_TOP:
        assert callable(getattr(top, name))


def test_kernel_backend_path():
    assert sorted(kernel_backend.__all__) == sorted(REFERENCE_TRITON)
    for name in REFERENCE_TRITON:
        assert getattr(kernel_backend, name) is getattr(top, name)


def test_module_backend_path():
    assert pt_backend.MSDA2D is top.MSDA2D and pt_backend.MSDA3D is top.MSDA3D
    # the reference's grid_sample oracle functions are test utilities, not product
    assert not hasattr(pt_backend, "msda3d_pytorch")


@pytest.mark.parametrize("fn", [top.msda2d, top.msda2d_fwd])
def test_cpu_tensors_raise_reference_error(fn):
    value = torch.zeros(1, 4, 2, 8)
    shapes = torch.tensor([[2, 2]])
    loc = torch.zeros(1, 3, 2, 1, 2, 2)
    attn = torch.zeros(1, 3, 2, 1, 2)
    with pytest.raises(ValueError, match="requires CUDA tensors"):
        fn(value, shapes, loc, attn)
