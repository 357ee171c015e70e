"""The modules' value projection over many rows (modules._WideLinearFn):
F.linear forward, the bias gradient as a ones-vector GEMM.  Output and all
three gradients agree with nn.Linear within the suite's tolerances, and
_project routes only large inputs in the parameters' dtype through it."""

from __future__ import annotations

import pytest
import torch
from torch import nn

from msda_triton_b200 import modules
from tests._util import TOL_FWD_F32, TOL_GRAD_F32, TOL_HALF

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16], ids=["float32", "bfloat16"])
def test_wide_linear_matches_nn_linear(dt):
    torch.manual_seed(5)
    lin = nn.Linear(64, 96).to(DEV, dt)
    x = torch.randn(3, 5001, 64, device=DEV, dtype=dt)
    g = torch.randn(3, 5001, 96, device=DEV, dtype=dt)
    res = []
    for wide in (True, False):
        xx = x.detach().requires_grad_(True)
        out = (modules._WideLinearFn.apply(xx, lin.weight, lin.bias) if wide else lin(xx))
        grads = torch.autograd.grad(out, [xx, lin.weight, lin.bias], g)
        res.append([out, *grads])
    tf, tg = (TOL_FWD_F32, TOL_GRAD_F32) if dt == torch.float32 else (TOL_HALF, TOL_HALF)
    for i, (a, b) in enumerate(zip(*res)):
        tol = tf if i == 0 else tg
        scale = b.float().abs().max().clamp_min(1.0)
        torch.testing.assert_close(a.float() / scale, b.float() / scale, rtol=tol, atol=tol,
                                   msg=lambda m, i=i: f"tensor {i}: {m}")


def test_project_routes_large_inputs(monkeypatch):
    lin = nn.Linear(16, 16).to(DEV)
    x = torch.randn(2, 50, 16, device=DEV, requires_grad=True)
    assert "WideLinear" not in type(modules._project(lin, x).grad_fn).__name__
    monkeypatch.setattr(modules, "WIDE_LINEAR_MIN_ROWS", 100)
    assert "WideLinear" in type(modules._project(lin, x).grad_fn).__name__
    with torch.autocast("cuda", dtype=torch.bfloat16):
        assert "WideLinear" not in type(modules._project(lin, x).grad_fn).__name__
