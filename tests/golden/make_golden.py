"""Generate the golden vectors in tests/golden/*.npz from the reference itself.

Run in a container where the reference package source is available:

    MSDA_REFERENCE_SRC=<reference checkout>/src python tests/golden/make_golden.py

It imports the reference's pure-PyTorch functions msda2d_pytorch /
msda3d_pytorch (src/msda_triton/pytorch/msda_2d.py:23-114,
src/msda_triton/pytorch/msda_3d.py:23-118), runs forward and backward in
float32 on the CPU on seeded inputs, and stores inputs and outputs.  The GPU
box does not have the reference; the tests only read the stored .npz files.

Input recipe (one CPU torch.Generator per case, drawn in this order):
value ~ N(0,1); sampling_locations ~ U[0,1) (then case-specific edits);
attention logits ~ N(0,1) -> softmax over L*P; grad_output ~ N(0,1).
"""

from __future__ import annotations

import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _reference():
    src = os.environ.get("MSDA_REFERENCE_SRC")
    if not src:
        raise SystemExit("set MSDA_REFERENCE_SRC to the reference's src/ directory")
    sys.path.insert(0, src)
    from msda_triton.pytorch.msda_2d import msda2d_pytorch
    from msda_triton.pytorch.msda_3d import msda3d_pytorch

    return msda2d_pytorch, msda3d_pytorch


def make_inputs(seed, B, Q, H, C, P, shapes, loc_lo=0.0, loc_hi=1.0):
    """Seeded inputs in the reference's tensor contract (float32, CPU)."""
    g = torch.Generator().manual_seed(seed)
    d = len(shapes[0])
    L = len(shapes)
    K = int(sum(int(np.prod(s)) for s in shapes))
    value = torch.randn(B, K, H, C, generator=g)
    loc = torch.rand(B, Q, H, L, P, d, generator=g) * (loc_hi - loc_lo) + loc_lo
    logits = torch.randn(B, Q, H, L * P, generator=g)
    attn = logits.softmax(-1).view(B, Q, H, L, P)
    grad_out = torch.randn(B, Q, H * C, generator=g)
    return value, torch.tensor(shapes, dtype=torch.int64), loc, attn, grad_out


# name: (seed, B, Q, H, C, P, shapes, clamp, eps, loc range, edit)
CASES = {
    # 2D, B1 Q300 H8 C32 L4 P4, K=1360, clamp on.
    "cfg0_2d": (0, 1, 300, 8, 32, 4, [(32, 32), (16, 16), (8, 8), (4, 4)], True, 1e-4, (0, 1), None),
    # Reference test shapes (tests/test_msda_3d.py:61, test_msda_2d.py:61).
    "basic_3d": (1, 2, 50, 8, 32, 4, [(4, 5, 5), (2, 3, 3)], True, 1e-4, (0, 1), None),
    "points8_2d": (2, 2, 25, 4, 32, 8, [(16, 16), (8, 8)], True, 1e-4, (0, 1), None),
    "heads16_3d": (3, 1, 40, 16, 16, 4, [(4, 5, 5), (2, 3, 3), (3, 4, 4), (2, 2, 2)], True, 1e-4, (0, 1), None),
    "c64_3d": (4, 1, 30, 4, 64, 4, [(4, 5, 5), (2, 3, 3), (3, 4, 4)], True, 1e-4, (0, 1), None),
    # Boundary and out-of-range locations (tests/test_msda_3d.py:252-285).
    "boundary_3d": (5, 1, 10, 8, 32, 4, [(4, 5, 5), (2, 3, 3)], True, 1e-4, (0, 1), "boundary"),
    "boundary_2d": (6, 1, 10, 4, 32, 4, [(12, 16), (6, 8)], True, 1e-4, (0, 1), "boundary"),
    "oob_clamp_3d": (7, 1, 10, 8, 32, 4, [(4, 5, 5), (2, 3, 3)], True, 1e-4, (0, 1), "oob"),
    "oob_clamp_2d": (8, 1, 10, 4, 32, 4, [(12, 16), (6, 8)], True, 1e-4, (0, 1), "oob"),
    # clamp_grid=False with locations spilling outside [0,1]: zero padding.
    "noclamp_3d": (9, 2, 30, 4, 32, 4, [(4, 5, 5), (2, 3, 3)], False, 1e-4, (-0.2, 1.2), None),
    "noclamp_2d": (10, 2, 30, 4, 32, 4, [(12, 16), (6, 8)], False, 1e-4, (-0.2, 1.2), None),
    # Wide clamp window so many points sit on the clamp and get zero loc-grad.
    "eps05_2d": (11, 1, 40, 4, 32, 4, [(8, 8), (4, 4)], True, 0.05, (-0.1, 1.1), None),
    "eps05_3d": (12, 1, 40, 4, 32, 4, [(4, 5, 5), (2, 3, 3)], True, 0.05, (-0.1, 1.1), None),
    # Single level (tests/test_msda_3d.py:343-374).
    "single_level_3d": (13, 2, 50, 8, 32, 4, [(4, 5, 5)], True, 1e-4, (0, 1), None),
    # Ragged: odd channel count and head count, non-square levels, size-1 axes.
    "ragged_2d": (14, 1, 7, 3, 5, 3, [(5, 7), (3, 4), (1, 2)], True, 1e-4, (0, 1), None),
    "ragged_3d": (15, 2, 9, 3, 6, 3, [(3, 5, 7), (1, 2, 3), (2, 1, 1)], True, 1e-4, (0, 1), None),
    "c8_2d": (16, 2, 33, 2, 8, 2, [(6, 9), (3, 5)], True, 1e-4, (0, 1), None),
    # Empty query set.
    "empty_q_2d": (17, 2, 0, 8, 32, 4, [(8, 8), (4, 4)], True, 1e-4, (0, 1), None),
}


def _edit(loc, kind):
    if kind == "boundary":
        loc[0, 0, 0, 0, 0, :] = 0.0
        loc[0, 1, 0, 0, 0, :] = 1.0
        mixed = [0.0, 1.0, 0.5][: loc.shape[-1]]
        loc[0, 2, 0, 0, 0, :] = torch.tensor(mixed)
        loc[0, 3, :, :, :, :] = 0.5
    elif kind == "oob":
        loc[0, 0, 0, 0, 0, :] = -0.1
        loc[0, 1, 0, 0, 0, :] = 1.1
        loc[0, 2, :, :, :, 0] = -0.3
        loc[0, 3, :, :, :, -1] = 1.4


def main() -> None:
    msda2d_pytorch, msda3d_pytorch = _reference()
    for name, (seed, B, Q, H, C, P, shapes, clamp, eps, rng, edit) in CASES.items():
        value, shp, loc, attn, go = make_inputs(seed, B, Q, H, C, P, shapes, *rng)
        if edit:
            _edit(loc, edit)
        fn = msda2d_pytorch if len(shapes[0]) == 2 else msda3d_pytorch
        v = value.clone().requires_grad_(True)
        lo = loc.clone().requires_grad_(True)
        a = attn.clone().requires_grad_(True)
        out = fn(v, shp, lo, a, clamp_grid=clamp, clamp_eps=eps)
        if out.numel():
            out.backward(go)
            gv, gl, ga = v.grad, lo.grad, a.grad
        else:
            gv, gl, ga = torch.zeros_like(v), torch.zeros_like(lo), torch.zeros_like(a)
        np.savez_compressed(
            os.path.join(HERE, f"{name}.npz"),
            value=value.numpy(), shapes=shp.numpy(), loc=loc.numpy(), attn=attn.numpy(),
            grad_out=go.numpy(), clamp=np.array(clamp), eps=np.array(eps),
            out=out.detach().numpy(), grad_value=gv.numpy(), grad_loc=gl.numpy(),
            grad_attn=ga.numpy(),
        )
        print(f"{name}: out {tuple(out.shape)}")


if __name__ == "__main__":
    main()
