"""Test helpers: seeded inputs in the reference's tensor contract, and the
tolerance check used throughout (|a - e| <= atol + rtol * |e|, elementwise)."""

from __future__ import annotations

import numpy as np
import torch

# Tolerances of the parity bar: fp32 forward 1e-5, fp32 gradients 1e-4,
# fp16/bf16 2e-2 against an fp32 reference (rtol = atol).
TOL_FWD_F32 = 1e-5
TOL_GRAD_F32 = 1e-4
TOL_HALF = 2e-2


def num_keys(shapes) -> int:
    return int(sum(int(np.prod(s)) for s in shapes))


def make_inputs(B, Q, H, C, P, shapes, *, seed=0, dtype=torch.float32, device="cpu",
                loc_range=(0.0, 1.0), gen_device="cpu"):
    """value ~ N(0,1); loc ~ U[lo,hi); weights = softmax over L*P of N(0,1)
    logits; grad_out ~ N(0,1) -- drawn in that order from one generator."""
    g = torch.Generator(device=gen_device).manual_seed(seed)
    d = len(shapes[0])
    L = len(shapes)
    K = num_keys(shapes)
    kw = dict(generator=g, device=gen_device)
    value = torch.randn(B, K, H, C, **kw)
    lo, hi = loc_range
    loc = torch.rand(B, Q, H, L, P, d, **kw) * (hi - lo) + lo
    attn = torch.randn(B, Q, H, L * P, **kw).softmax(-1).view(B, Q, H, L, P)
    grad_out = torch.randn(B, Q, H * C, **kw)
    shp = torch.tensor(shapes, dtype=torch.int64)
    cast = lambda t: t.to(device=device, dtype=dtype)
    return cast(value), shp, cast(loc), cast(attn), cast(grad_out)


def max_violation(actual, expected, rtol: float, atol: float) -> float:
    """max(|a-e| - (atol + rtol*|e|)); <= 0 means within tolerance."""
    a = torch.as_tensor(np.asarray(actual) if not torch.is_tensor(actual) else actual).double().cpu()
    e = torch.as_tensor(np.asarray(expected) if not torch.is_tensor(expected) else expected).double().cpu()
    if a.numel() == 0:
        return -1.0
    return float(((a - e).abs() - (atol + rtol * e.abs())).max())


def assert_close(actual, expected, tol: float, what: str = "") -> None:
    a = actual if torch.is_tensor(actual) else torch.as_tensor(np.asarray(actual))
    e = expected if torch.is_tensor(expected) else torch.as_tensor(np.asarray(expected))
    assert tuple(a.shape) == tuple(e.shape), f"{what}: shape {tuple(a.shape)} != {tuple(e.shape)}"
    v = max_violation(a, e, tol, tol)
    if v > 0:
        d = (a.double().cpu() - e.double().cpu()).abs()
        idx = int(d.argmax())
        raise AssertionError(
            f"{what}: exceeds rtol=atol={tol}: max|diff|={float(d.max()):.3e} at flat index "
            f"{idx} (actual {float(a.reshape(-1)[idx]):.6g}, expected {float(e.reshape(-1)[idx]):.6g})"
        )
