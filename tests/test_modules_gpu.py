"""MSDA2D / MSDA3D modules on the GPU against the reference's own modules.

tests/golden/modules/*.npz hold the reference modules' parameters, inputs,
output and every gradient (tests/golden/make_module_golden.py, fp32 on the
CPU with grid_sample).  Ours load the same state_dict, run on cuda:0 in fp32
(TF32 off) and must match: the sampling kernels agree with grid_sample to
1e-5 / 1e-4 and the projections are the same Linear layers, so the bar is
rtol = atol = 1e-4 throughout.
"""

from __future__ import annotations

import ast
import glob
import os

import numpy as np
import pytest
import torch

from msda_triton_b200.modules import MSDA2D, MSDA3D

pytestmark = pytest.mark.gpu

GOLDEN = sorted(glob.glob(os.path.join(os.path.dirname(__file__), "golden", "modules", "*.npz")))
DEV = torch.device("cuda", 0)


@pytest.fixture(autouse=True)
def no_tf32():
    prev = (torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32)
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    yield
    torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32 = prev


def _load(path):
    z = np.load(path)
    return {k: z[k] for k in z.files}


def _module(z, fused=True):
    kw = ast.literal_eval(str(z["module_kwargs"]))
    m = (MSDA3D if int(z["ndim"]) == 3 else MSDA2D)(**kw, fused_prologue=fused)
    m.load_state_dict({k[6:]: torch.from_numpy(v) for k, v in z.items() if k.startswith("param/")})
    m.train(bool(kw.get("use_checkpoint")))   # the fixtures' chunked cases ran in training mode
    return m.to(DEV)


def _run(m, z, shapes_on_device):
    t = lambda k, grad=False: (torch.from_numpy(z[k]).to(DEV).requires_grad_(grad)
                               if k in z else None)
    query, ref = t("query", True), t("reference_points", True)
    value = t("value", True)
    mask = t("key_padding_mask")
    shapes = torch.from_numpy(z["shapes"])
    out = m(query, value=value, identity=t("identity"), query_pos=t("query_pos"),
            key_padding_mask=mask, reference_points=ref,
            spatial_shapes=shapes.to(DEV) if shapes_on_device else shapes)
    (out * t("grad_out")).sum().backward()
    res = {"out": out, "grad_query": query.grad, "grad_reference_points": ref.grad}
    if value is not None:
        res["grad_value"] = value.grad
    for k, p in m.named_parameters():
        res["grad/" + k] = p.grad
    return res


@pytest.mark.parametrize("fused", [True, False], ids=["fused", "unfused"])
@pytest.mark.parametrize("shapes_on_device", [True, False])
@pytest.mark.parametrize("path", GOLDEN, ids=[os.path.basename(p)[:-4] for p in GOLDEN])
def test_module_matches_reference(path, shapes_on_device, fused):
    z = _load(path)
    got = _run(_module(z, fused), z, shapes_on_device)
    for k, g in got.items():
        torch.testing.assert_close(g.detach().cpu(), torch.from_numpy(z[k]), rtol=1e-4, atol=1e-4,
                                   msg=lambda m, k=k: f"{os.path.basename(path)} {k}: {m}")


@pytest.mark.parametrize("fused", [True, False], ids=["fused", "unfused"])
@pytest.mark.parametrize("cls,d", [(MSDA2D, 2), (MSDA3D, 3)])
def test_module_bf16_autocast(cls, d, fused):
    """Mixed precision: under autocast the projections run in bf16, the
    locations and softmax weights stay fp32 -- the kernels take the mixed
    pair.  The result stays within the half-precision bar of fp32."""
    torch.manual_seed(0)
    m = cls(embed_dims=64, num_heads=4, num_levels=2, num_points=4, dropout=0.0,
            batch_first=True, fused_prologue=fused).to(DEV)
    m.init_weights()
    shapes = torch.tensor([[6] * d, [3] * d], dtype=torch.int64, device=DEV)
    K = 6 ** d + 3 ** d
    q = torch.randn(2, 50, 64, device=DEV)
    v = torch.randn(2, K, 64, device=DEV)
    ref = torch.rand(2, 50, 2, d, device=DEV) * 0.8 + 0.1
    want = m(q, value=v, reference_points=ref, spatial_shapes=shapes)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        got = m(q, value=v, reference_points=ref, spatial_shapes=shapes)
        got.float().square().sum().backward()
    torch.testing.assert_close(got.float(), want, rtol=3e-2, atol=3e-2)
    assert all(torch.isfinite(p.grad).all() for p in m.parameters())
