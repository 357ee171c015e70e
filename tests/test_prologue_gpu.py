"""The modules' sampling prologue as its own pass (msda_prologue_fwd /
msda_prologue_bwd through fused.sampling_prologue) against the reference's
tensor expressions (pytorch/msda_3d.py:336-350, pytorch/msda_2d.py:325-339):

    loc     = reference_points[:, :, None, :, None, :] + offsets / normalizer
    weights = softmax(logits over each row's L*P samples)

The locations and the offsets' gradient are bit-identical (the same
roundings in the sampling dtype); the weights and the logits' and reference
points' gradients agree within the suite's tolerances (summation order).
A module call above 2^20 samples, which takes this path, agrees with the
same module on the tensor ops (fused_prologue=False)."""

from __future__ import annotations

import pytest
import torch

from msda_triton_b200.fused import sampling_prologue
from msda_triton_b200.modules import MSDA2D, MSDA3D
from tests._util import TOL_FWD_F32, TOL_GRAD_F32, TOL_HALF

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)
DTYPES = [torch.float32, torch.bfloat16, torch.float16]


def _tol(dt):
    return (TOL_FWD_F32, TOL_GRAD_F32) if dt == torch.float32 else (TOL_HALF, TOL_HALF)


def _inputs(ndim, dt, seed, B=2, Q=300, H=4, P=4):
    shapes = [(6, 9, 7), (3, 300, 5)] if ndim == 3 else [(37, 301), (12, 20), (5, 7)]
    g = torch.Generator().manual_seed(seed)
    L = len(shapes)
    ref = torch.rand(B, Q, L, ndim, generator=g)
    off = torch.randn(B, Q, H, L, P, ndim, generator=g) * 4.0
    lg = torch.randn(B, Q, H, L, P, generator=g) * 3.0
    shp = torch.tensor(shapes, dtype=torch.int64)
    return shp, *(t.to(DEV, dt) for t in (ref, off, lg))


def _torch_prologue(shp, ref, off, lg):
    B, Q, H, L, P, _ = off.shape
    normalizer = shp.flip(-1).to(off.device)[None, None, None, :, None, :]
    w = lg.view(B, Q, H, L * P).softmax(-1).view(B, Q, H, L, P)
    loc = ref[:, :, None, :, None, :] + off / normalizer
    return loc, w


@pytest.mark.parametrize("dt", DTYPES, ids=lambda d: str(d)[6:])
@pytest.mark.parametrize("ndim", [2, 3])
def test_prologue_matches_tensor_ops(ndim, dt):
    shp, ref, off, lg = _inputs(ndim, dt, seed=ndim * 7 + DTYPES.index(dt))
    leaves = [t.detach().requires_grad_(True) for t in (ref, off, lg)]
    loc, w = sampling_prologue(ndim, shp, *leaves)
    leaves_t = [t.detach().requires_grad_(True) for t in (ref, off, lg)]
    loc_t, w_t = _torch_prologue(shp, *leaves_t)
    # sizes above 256 (301, 300) are not exact in bf16: the divisor rounds as in the tensor op
    assert torch.equal(loc, loc_t)
    tf, tg = _tol(dt)
    torch.testing.assert_close(w, w_t, rtol=tf, atol=tf)
    g = torch.Generator().manual_seed(99)
    gl = (torch.randn(loc.shape, generator=g) * 0.5).to(DEV, dt)
    gw = torch.randn(w.shape, generator=g).to(DEV, dt)
    got = torch.autograd.grad((loc, w), leaves, (gl, gw))
    want = torch.autograd.grad((loc_t, w_t), leaves_t, (gl, gw))
    assert torch.equal(got[1], want[1])  # offsets: grad / normalizer, the same rounding
    for name, a, b in zip(("reference_points", "logits"), (got[0], got[2]), (want[0], want[2])):
        torch.testing.assert_close(a.float(), b.float(), rtol=tg, atol=tg,
                                   msg=lambda m, n=name: f"{n}: {m}")


def _shifted(t):
    """The same values in a contiguous tensor whose data starts one element
    past an allocation's start: not 16-byte aligned."""
    buf = torch.empty(t.numel() + 1, dtype=t.dtype, device=t.device)
    out = buf[1:].view(t.shape)
    out.copy_(t)
    return out


@pytest.mark.parametrize("dt", DTYPES, ids=lambda d: str(d)[6:])
@pytest.mark.parametrize("ndim", [2, 3])
def test_prologue_unaligned_and_ragged(ndim, dt):
    """Rows whose count leaves a partial vector in the last tile (Q=301, H=3,
    P=3), through the 16-byte vector copies (aligned tensors) and the
    element copies (tensors one element off alignment): the same bits, and
    the tensor ops' locations and offset gradients."""
    shp, ref, off, lg = _inputs(ndim, dt, seed=40 + ndim, Q=301, H=3, P=3)
    g = torch.Generator().manual_seed(41)
    gl = (torch.randn(off.shape, generator=g) * 0.5).to(DEV, dt)
    gw = torch.randn(lg.shape, generator=g).to(DEV, dt)
    res = []
    for shift in (False, True):
        ins = [_shifted(t) if shift else t.clone() for t in (ref, off, lg)]
        assert all((t.data_ptr() % 16 != 0) == shift for t in ins[1:])
        leaves = [t.detach().requires_grad_(True) for t in ins]
        loc, w = sampling_prologue(ndim, shp, *leaves)
        gouts = (_shifted(gl), _shifted(gw)) if shift else (gl, gw)
        res.append([loc, w, *torch.autograd.grad((loc, w), leaves, gouts)])
    for i, (a, b) in enumerate(zip(*res)):
        assert torch.equal(a, b), f"tensor {i} differs between the vector and element copies"
    leaves_t = [t.detach().requires_grad_(True) for t in (ref, off, lg)]
    loc_t, w_t = _torch_prologue(shp, *leaves_t)
    want = torch.autograd.grad((loc_t, w_t), leaves_t, (gl, gw))
    assert torch.equal(res[0][0], loc_t)
    assert torch.equal(res[0][3], want[1])


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("cls,ndim", [(MSDA3D, 3), (MSDA2D, 2)])
def test_large_module_call_matches_tensor_ops(cls, ndim, dt):
    """Above 2^20 samples the module forms locations and weights with the
    prologue pass; fused_prologue=False keeps the tensor ops.  Output and
    every gradient agree (no dropout, whose masks would differ)."""
    shapes = [(4, 8, 8), (2, 4, 4)] if ndim == 3 else [(16, 16), (8, 8)]
    K = sum(int(torch.tensor(s).prod()) for s in shapes)
    B, Q, E, H, L, P = 2, 9000, 128, 8, len(shapes), 4
    assert B * Q * H * L * P >= 1 << 20
    torch.manual_seed(3)
    mods = []
    for fused in (True, False):
        torch.manual_seed(3)
        m = cls(embed_dims=E, num_heads=H, num_levels=L, num_points=P, batch_first=True,
                dropout=0.0, fused_prologue=fused).to(DEV, dt)
        mods.append(m)
    mods[1].load_state_dict(mods[0].state_dict())
    g = torch.Generator().manual_seed(4)
    query = torch.randn(B, Q, E, generator=g).to(DEV, dt)
    value = torch.randn(B, K, E, generator=g).to(DEV, dt)
    refp = torch.rand(B, Q, L, ndim, generator=g).to(DEV, dt)
    gout = torch.randn(B, Q, E, generator=g).to(DEV, dt)
    res = []
    for m in mods:
        q, v, r = (t.detach().requires_grad_(True) for t in (query, value, refp))
        out = m(q, value=v, reference_points=r, spatial_shapes=torch.tensor(shapes))
        grads = torch.autograd.grad(out, [q, v, r] + list(m.parameters()), gout)
        res.append([out] + list(grads))
    tf, tg = _tol(dt)
    for i, (a, b) in enumerate(zip(*res)):
        if i >= 4 and dt != torch.float32:
            # 16-bit parameter gradients sum thousands of rows of two equally
            # valid roundings (softmax in bf16): compared by relative norm
            err = ((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-30)).item()
            assert err < tg, f"tensor {i}: relative norm error {err:.3g}"
            continue
        tol = tf if i == 0 else tg
        torch.testing.assert_close(a.float(), b.float(), rtol=tol, atol=tol,
                                   msg=lambda m, i=i: f"tensor {i}: {m}")
