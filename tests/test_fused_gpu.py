"""msda2d_fused / msda3d_fused against the unfused composition.

The fused ops form loc = ref + offsets / (W, H[, D]) and weights =
softmax(logits) inside the kernels.  The reference modules compute exactly
that composition with tensor ops and then sample
(pytorch/msda_3d.py:325-350), so the check is: the fused output and the
gradients of value, reference points, offsets and logits equal those of
msda{2,3}d on the composed tensors (whose kernels are pinned to the oracle
elsewhere) -- fp32 at 1e-5 / 1e-4, half precision at 2e-2 against fp32.
"""

from __future__ import annotations

import pytest
import torch

import msda_triton_b200 as M

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _inputs(ndim, B, Q, H, C, P, shapes, seed, ref_range=(0.0, 1.0), off_scale=1.5):
    g = torch.Generator().manual_seed(seed)
    L = len(shapes)
    K = sum(int(torch.tensor(s).prod()) for s in shapes)
    value = torch.randn(B, K, H, C, generator=g)
    lo, hi = ref_range
    ref = torch.rand(B, Q, L, ndim, generator=g) * (hi - lo) + lo
    off = torch.randn(B, Q, H, L, P, ndim, generator=g) * off_scale
    logits = torch.randn(B, Q, H, L, P, generator=g) * 2.0
    go = torch.randn(B, Q, H * C, generator=g)
    return value, torch.tensor(shapes, dtype=torch.int64), ref, off, logits, go


def _unfused(ndim, value, shapes, ref, off, logits, clamp, eps):
    B, Q, H, L, P, _ = off.shape
    norm = shapes.flip(-1).to(off.device)[None, None, None, :, None, :]
    loc = ref[:, :, None, :, None, :] + off / norm
    w = logits.reshape(B, Q, H, L * P).softmax(-1).view(B, Q, H, L, P)
    fn = M.msda3d if ndim == 3 else M.msda2d
    return fn(value, shapes, loc, w, clamp, eps)


def _run(fn, tensors, go):
    xs = [t.clone().requires_grad_(True) for t in tensors]
    out = fn(*xs)
    grads = torch.autograd.grad(out, xs, go)
    return [out.detach().float().cpu()] + [g.float().cpu() for g in grads]


CASES = [
    # ndim, B, Q, H, C, P, shapes, clamp, ref range
    (2, 2, 60, 4, 32, 4, [(20, 24), (10, 12), (5, 6)], True, (0.0, 1.0)),
    (2, 1, 45, 2, 64, 3, [(17, 9), (4, 5)], False, (-0.1, 1.1)),
    (3, 2, 50, 4, 32, 4, [(6, 8, 10), (3, 4, 5)], True, (0.0, 1.0)),
    (3, 1, 40, 8, 16, 2, [(5, 7, 9), (2, 3, 4), (1, 2, 2)], False, (-0.1, 1.1)),
    (3, 2, 30, 3, 6, 3, [(4, 4, 4), (2, 2, 2)], True, (0.0, 1.0)),   # narrow rows, odd H
]


@pytest.mark.parametrize("shapes_on_device", [False, True])
@pytest.mark.parametrize("case", CASES, ids=[f"{c[0]}d-h{c[3]}c{c[4]}-clamp{c[7]}" for c in CASES])
def test_fp32_matches_unfused(case, shapes_on_device):
    ndim, B, Q, H, C, P, shapes, clamp, rng = case
    value, shp, ref, off, logits, go = _inputs(ndim, B, Q, H, C, P, shapes, seed=Q + C,
                                               ref_range=rng)
    shp_k = shp.to(DEV) if shapes_on_device else shp
    fused = M.msda3d_fused if ndim == 3 else M.msda2d_fused
    t = [x.to(DEV) for x in (value, ref, off, logits)]
    got = _run(lambda v, r, o, lg: fused(v, shp_k, r, o, lg, clamp, 1e-4), t, go.to(DEV))
    want = _run(lambda v, r, o, lg: _unfused(ndim, v, shp_k, r, o, lg, clamp, 1e-4), t,
                go.to(DEV))
    for name, a, b, tol in zip(("out", "value", "ref", "offsets", "logits"), got, want,
                               (1e-5, 1e-4, 1e-4, 1e-4, 1e-4)):
        torch.testing.assert_close(a, b, rtol=tol, atol=tol, msg=lambda m, n=name: f"{n}: {m}")


@pytest.mark.parametrize("ndim", [2, 3])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_half_layouts(ndim, dtype):
    """Autocast layout (16-bit value/offsets/logits, fp32 reference points)
    and all-fp32 projections with a 16-bit value; against fp32 at the 2e-2 bar."""
    case = CASES[0] if ndim == 2 else CASES[2]
    _, B, Q, H, C, P, shapes, clamp, rng = case
    value, shp, ref, off, logits, go = _inputs(ndim, B, Q, H, C, P, shapes, seed=7)
    fused = M.msda3d_fused if ndim == 3 else M.msda2d_fused
    fn = lambda v, r, o, lg: fused(v, shp, r, o, lg, clamp, 1e-4)
    go16 = go.to(DEV, dtype)
    for sdt in (dtype, torch.float32):
        t = [value.to(DEV, dtype), ref.to(DEV), off.to(DEV, sdt), logits.to(DEV, sdt)]
        # the fp32 run sees the same (rounded) inputs and output gradient
        want = _run(fn, [x.float() for x in t], go16.float())
        got = _run(fn, t, go16)
        for name, a, b in zip(("out", "value", "ref", "offsets", "logits"), got, want):
            torch.testing.assert_close(a, b, rtol=2e-2, atol=2e-2,
                                       msg=lambda m, n=name: f"{n} ({sdt}): {m}")


def test_logits_shapes_and_views():
    """(B,Q,H,L*P) logits, non-contiguous head slices of every input."""
    ndim, B, Q, H, C, P, shapes, clamp, _ = CASES[2]
    value, shp, ref, off, logits, go = _inputs(ndim, B, Q, H, C, P, shapes, seed=3)
    v, r, o, lg = (x.to(DEV) for x in (value, ref, off, logits))
    a = M.msda3d_fused(v, shp, r, o, lg.flatten(3))
    b = M.msda3d_fused(v, shp, r, o, lg)
    assert torch.equal(a, b)
    h = slice(1, 3)
    sl = M.msda3d_fused(v[:, :, h], shp, r, o[:, :, h], lg[:, :, h])
    ct = M.msda3d_fused(v[:, :, h].contiguous(), shp, r, o[:, :, h].contiguous(),
                        lg[:, :, h].contiguous())
    assert torch.equal(sl, ct)


def test_errors():
    ndim, B, Q, H, C, P, shapes, clamp, _ = CASES[2]
    value, shp, ref, off, logits, go = _inputs(ndim, B, Q, H, C, P, shapes, seed=1)
    v, r, o, lg = (x.to(DEV) for x in (value, ref, off, logits))
    with pytest.raises(ValueError, match="reference_points must be"):
        M.msda3d_fused(v, shp, r[:, :, :1], o, lg)
    with pytest.raises(ValueError, match="requires CUDA tensors"):
        M.msda3d_fused(value, shp, ref, off, logits)
    with pytest.raises(NotImplementedError):
        M.msda3d_fused(v.double(), shp, r, o, lg)


@pytest.mark.parametrize("ndim", [2, 3])
def test_location_bit_exact(ndim):
    """One sample per row (L = P = 1): both paths weigh it exactly 1, so the
    output and the offset gradient are bitwise equal iff the fused location
    ref + offset / size rounds exactly like the separate tensor expression
    (level sizes that are not powers of two, offsets of several cells)."""
    shapes = [(37, 53)] if ndim == 2 else [(11, 19, 23)]
    B, Q, H, C, P = 2, 4000, 4, 16, 1
    value, shp, ref, off, logits, go = _inputs(ndim, B, Q, H, C, P, shapes, seed=11,
                                               off_scale=7.0)
    t = [x.to(DEV) for x in (value, ref, off, logits)]
    fused = M.msda3d_fused if ndim == 3 else M.msda2d_fused
    got = _run(lambda v, r, o, lg: fused(v, shp, r, o, lg, False, 1e-4), t, go.to(DEV))
    want = _run(lambda v, r, o, lg: _unfused(ndim, v, shp, r, o, lg, False, 1e-4), t,
                go.to(DEV))
    assert torch.equal(got[0], want[0]), "output"
    assert torch.equal(got[3], want[3]), "offset gradient"
    torch.testing.assert_close(got[2], want[2], rtol=1e-5, atol=1e-5)
