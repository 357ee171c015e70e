"""MSDA2D / MSDA3D modules without a GPU: the same parameters as the
reference's modules, the same init_weights() values from the same seed
(pinned by tests/golden/modules/*.npz, made by the reference itself), and the
reference's errors."""

from __future__ import annotations

import ast
import glob
import os

import numpy as np
import pytest
import torch

from msda_triton_b200.modules import MSDA2D, MSDA3D

GOLDEN = sorted(glob.glob(os.path.join(os.path.dirname(__file__), "golden", "modules", "*.npz")))


def _load(path):
    z = np.load(path)
    return {k: z[k] for k in z.files}


def _build(z):
    cls = MSDA3D if int(z["ndim"]) == 3 else MSDA2D
    return cls(**ast.literal_eval(str(z["module_kwargs"])))


def test_goldens_present():
    assert len(GOLDEN) >= 4


@pytest.mark.parametrize("path", GOLDEN, ids=[os.path.basename(p)[:-4] for p in GOLDEN])
def test_parameters_and_init_match_reference(path):
    z = _load(path)
    torch.manual_seed(int(z["init_seed"]))
    m = _build(z)
    m.init_weights()
    sd = m.state_dict()
    ref = {k[5:]: v for k, v in z.items() if k.startswith("init/")}
    assert set(sd) == set(ref)
    for k, v in ref.items():
        assert tuple(sd[k].shape) == v.shape, k
        np.testing.assert_allclose(sd[k].numpy(), v, rtol=0, atol=1e-7, err_msg=k)


@pytest.mark.parametrize("cls,d", [(MSDA2D, 2), (MSDA3D, 3)])
def test_errors(cls, d):
    with pytest.raises(ValueError, match="embed_dims must be divisible by num_heads"):
        cls(embed_dims=30, num_heads=4, num_levels=1, num_points=1)
    m = cls(embed_dims=16, num_heads=2, num_levels=1, num_points=2, batch_first=True)
    shapes = torch.tensor([[2] * d], dtype=torch.int64)
    K = 2 ** d
    q = torch.randn(1, 3, 16)
    with pytest.raises(ValueError, match=f"Last dim of reference_points must be {d}"):
        m(q, value=torch.randn(1, K, 16), reference_points=torch.rand(1, 3, 1, d + 1),
          spatial_shapes=shapes)
    with pytest.raises(AssertionError, match="doesn't match value size"):
        m(q, value=torch.randn(1, K + 1, 16), reference_points=torch.rand(1, 3, 1, d),
          spatial_shapes=shapes)
    # the sampling runs only in the CUDA kernels: CPU tensors are rejected
    with pytest.raises(ValueError, match="requires CUDA tensors"):
        m(q, value=torch.randn(1, K, 16), reference_points=torch.rand(1, 3, 1, d),
          spatial_shapes=shapes)
