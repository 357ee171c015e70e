"""The torch.library registration without a GPU: the ops exist under
torch.ops.msda_b200 and their fake implementations give the shapes, dtypes
and devices torch.compile needs (fake CUDA tensors need no device)."""

from __future__ import annotations

import pytest
import torch
from torch._subclasses.fake_tensor import FakeTensorMode

import msda_triton_b200.ops  # noqa: F401  (registers the ops)


def test_ops_registered():
    for name in ("msda_forward", "msda_backward", "msda_fused_forward", "msda_fused_backward"):
        assert hasattr(torch.ops.msda_b200, name)


@pytest.mark.parametrize("ndim", [2, 3])
@pytest.mark.parametrize("vdt,sdt", [(torch.bfloat16, torch.bfloat16), (torch.float16, torch.float32),
                                     (torch.float32, torch.float32)])
def test_fake_shapes(ndim, vdt, sdt):
    B, K, H, C, Q, L, P = 2, 84, 4, 16, 37, 2, 3
    with FakeTensorMode():
        value = torch.empty(B, K, H, C, device="cuda", dtype=vdt)
        shapes = torch.empty(L, ndim, dtype=torch.int64)
        loc = torch.empty(B, Q, H, L, P, ndim, device="cuda", dtype=sdt)
        attn = torch.empty(B, Q, H, L, P, device="cuda", dtype=sdt)
        out = torch.ops.msda_b200.msda_forward(value, shapes, loc, attn, ndim, True, 1e-4)
        assert out.shape == (B, Q, H * C) and out.dtype == vdt and out.device.type == "cuda"
        go = torch.empty(B, Q, H * C, device="cuda", dtype=vdt)
        gv, gl, ga = torch.ops.msda_b200.msda_backward(go, value, shapes, loc, attn, ndim, True,
                                                       1e-4)
        for g, ref in ((gv, value), (gl, loc), (ga, attn)):
            assert g.shape == ref.shape and g.dtype == ref.dtype and g.is_contiguous()


@pytest.mark.parametrize("ndim", [2, 3])
def test_fused_fake_shapes(ndim):
    B, K, H, C, Q, L, P = 2, 84, 4, 16, 37, 2, 3
    with FakeTensorMode():
        value = torch.empty(B, K, H, C, device="cuda", dtype=torch.bfloat16)
        shapes = torch.empty(L, ndim, dtype=torch.int64)
        ref = torch.empty(B, Q, L, ndim, device="cuda", dtype=torch.float32)
        off = torch.empty(B, Q, H, L, P, ndim, device="cuda", dtype=torch.bfloat16)
        logits = torch.empty(B, Q, H, L * P, device="cuda", dtype=torch.bfloat16)
        out = torch.ops.msda_b200.msda_fused_forward(value, shapes, ref, off, logits, ndim, True,
                                                     1e-4)
        assert out.shape == (B, Q, H * C) and out.dtype == torch.bfloat16
        go = torch.empty(B, Q, H * C, device="cuda", dtype=torch.bfloat16)
        grads = torch.ops.msda_b200.msda_fused_backward(go, value, shapes, ref, off, logits, ndim,
                                                        True, 1e-4)
        for g, t in zip(grads, (value, ref, off, logits)):
            assert g.shape == t.shape and g.dtype == t.dtype
