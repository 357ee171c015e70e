"""Our kernels against the reference's own Triton kernels on the same GPU.

Runs only where the unmodified reference package is installed under
baseline/_ref (it is not part of the product).  The reference's Triton path
maps coordinates as x*W - 0.5 after a location-space clamp
(src/msda_triton/triton/msda_3d.py:164-169, :193) while both the oracle and
our kernels follow grid_sample's grid-space arithmetic, so near cell
boundaries the two pick different floor cells; the reference's own suite
bounds that against grid_sample (tests/test_msda_3d.py:130-233: out 1e-4,
grad_value 1e-5, grad_loc max 0.25 / mean 2e-5, grad_attn 3e-4).  Both
implementations sit within those bars of grid_sample, so they sit within
twice the bars of each other.
"""

from __future__ import annotations

import os
import sys

import pytest
import torch

from tests._util import make_inputs

pytestmark = pytest.mark.gpu

REF_DIR = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                       "baseline", "_ref")


@pytest.fixture(scope="module")
def ref():
    if not os.path.isdir(os.path.join(REF_DIR, "msda_triton")):
        pytest.skip("reference not installed under baseline/_ref")
    sys.path.insert(0, REF_DIR)
    try:
        import msda_triton
    except ImportError as e:  # triton missing or broken
        pytest.skip(f"reference package not importable: {e}")
    finally:
        sys.path.remove(REF_DIR)
    return msda_triton


def _both(ref, ndim, inp, dtype=torch.float32):
    import msda_triton_b200 as M

    dev = torch.device("cuda", 0)
    value, shp, loc, attn, go = inp
    res = []
    for fn in ((M.msda3d, ref.msda3d) if ndim == 3 else (M.msda2d, ref.msda2d)):
        v, lo, a = (t.to(dev, dtype).requires_grad_(True) for t in (value, loc, attn))
        out = fn(v, shp.to(dev), lo, a)
        g = torch.autograd.grad(out, (v, lo, a), go.to(dev, dtype))
        res.append([t.detach().float().cpu() for t in (out, *g)])
    return res


CASES = [
    (2, 2, 300, 8, 32, 4, [(32, 32), (16, 16), (8, 8), (4, 4)]),
    (2, 1, 500, 4, 64, 3, [(25, 38), (13, 19)]),
    (3, 2, 400, 8, 32, 4, [(16, 32, 32), (8, 16, 16), (4, 8, 8)]),
    (3, 1, 256, 4, 32, 2, [(8, 16, 16), (4, 8, 8)]),
]


@pytest.mark.parametrize("case", CASES, ids=[f"{c[0]}d-q{c[2]}" for c in CASES])
def test_fp32_matches_reference_triton(ref, case):
    ndim, B, Q, H, C, P, shapes = case
    inp = make_inputs(B, Q, H, C, P, shapes, seed=Q)
    ours, theirs = _both(ref, ndim, inp)
    d = [(o - t).abs() for o, t in zip(ours, theirs)]
    assert d[0].max() < 2e-4, f"out max diff {d[0].max()}"
    assert d[1].max() < 2e-5, f"grad_value max diff {d[1].max()}"
    assert d[2].max() < 0.5 and d[2].mean() < 4e-5, f"grad_loc diff {d[2].max()} / {d[2].mean()}"
    assert d[3].max() < 6e-4 and d[3].mean() < 2e-6, f"grad_attn diff {d[3].max()}"


@pytest.mark.parametrize("ndim", [2, 3])
def test_bf16_forward_matches_reference_triton(ref, ndim):
    case = CASES[0] if ndim == 2 else CASES[2]
    _, B, Q, H, C, P, shapes = case
    inp = make_inputs(B, Q, H, C, P, shapes, seed=3)
    ours, theirs = _both(ref, ndim, inp, torch.bfloat16)
    # both round the same fp32 accumulation to bf16: at most one bf16 ulp apart
    torch.testing.assert_close(ours[0], theirs[0], rtol=1e-2, atol=1e-2)
