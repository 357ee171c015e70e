"""Head-major value: (B, H, K, C) in memory, handed to the ops as the
(B, K, H, C) view `v.permute(0, 2, 1, 3)` of a dense (B, H, K, C) tensor.

The kernels read that layout in place (MSDA_VALUE_HEAD_MAJOR in the C ABI)
and write grad_value in it.  Every backward plan -- the gather/scatter
kernel (fp32 accumulator, direct 16-bit levels, device shapes), the
cell-sorted pipeline (per-row gathered and per-cell aggregated levels, dot
products in query and in sorted order) and the fused prologue -- must give
the oracle's results, and the forward must equal the (B, K, H, C) run
bit for bit.
"""

from __future__ import annotations

import pytest
import torch

import msda_triton_b200 as M
from msda_triton_b200 import _core, _lib
from tests._util import TOL_FWD_F32, TOL_GRAD_F32, TOL_HALF, make_inputs
from tests.test_fused_gpu import _inputs as fused_inputs
from tests.test_fused_gpu import _run as fused_run
from tests.test_msda_gpu import FNS, check_all, oracle_all

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


def head_major(value: torch.Tensor) -> torch.Tensor:
    """The same (B, K, H, C) values, stored (B, H, K, C)."""
    return value.permute(0, 2, 1, 3).contiguous().permute(0, 2, 1, 3)


def _fwd_bwd(ndim, value, shp, loc, attn, go, clamp=True):
    v = value.detach().requires_grad_(True)
    lo = loc.detach().requires_grad_(True)
    a = attn.detach().requires_grad_(True)
    out = FNS[ndim][0](v, shp, lo, a, clamp, 1e-4)
    gv, gl, ga = torch.autograd.grad(out, (v, lo, a), go.to(out.dtype))
    torch.cuda.synchronize()
    f = lambda t: t.detach().float().cpu()
    return [f(out), f(gv), f(gl), f(ga)], gv


# (env, dtypes): each backward plan and value-gradient target
PLANS = {
    "scatter": {"MSDA_BWD_PATH": "scatter"},
    "scatter-direct16": {"MSDA_BWD_PATH": "scatter", "MSDA_BWD_DIRECT16": "1"},
    "sorted-voxel": {"MSDA_BWD_PATH": "sorted", "MSDA_VOXEL_DENSITY": "1e9"},
    "sorted-voxel-cc": {"MSDA_BWD_PATH": "sorted", "MSDA_VOXEL_DENSITY": "1e9",
                        "MSDA_VOXEL_MMA": "0"},
    "sorted-voxel-tc": {"MSDA_BWD_PATH": "sorted", "MSDA_VOXEL_DENSITY": "1e9",
                        "MSDA_VOXEL_MMA": "tc"},
    "sorted-cell-sdots": {"MSDA_BWD_PATH": "sorted", "MSDA_VOXEL_DENSITY": "0",
                          "MSDA_SORTED_DOTS_MB": "0"},
    "sorted-cell-mma": {"MSDA_BWD_PATH": "sorted", "MSDA_VOXEL_DENSITY": "0",
                        "MSDA_DENSE_MMA_DENSITY": "0"},
    "sorted-auto-sdots": {"MSDA_BWD_PATH": "sorted", "MSDA_SORTED_DOTS_MB": "0",
                          "MSDA_SORTED_CHUNK_B": "1"},
}
CASES = [
    # ndim, B, Q, H, C, P, shapes
    (2, 2, 600, 4, 32, 4, [(40, 60), (20, 30), (10, 15)]),
    (3, 2, 700, 8, 32, 4, [(16, 24, 24), (8, 12, 12), (4, 6, 6)]),
    (3, 1, 300, 3, 16, 3, [(6, 9, 7), (3, 4, 5)]),
]
DTYPES = [torch.float32, torch.bfloat16, torch.float16]


def _set_env(monkeypatch, plan):
    for k in ("MSDA_BWD_PATH", "MSDA_BWD_DIRECT16", "MSDA_VOXEL_DENSITY", "MSDA_SORTED_DOTS_MB",
              "MSDA_SORTED_CHUNK_B", "MSDA_DENSE_MMA_DENSITY", "MSDA_VOXEL_MMA"):
        monkeypatch.delenv(k, raising=False)
    for k, v in PLANS[plan].items():
        monkeypatch.setenv(k, v)


@pytest.mark.parametrize("plan", sorted(PLANS))
@pytest.mark.parametrize("dtype", DTYPES, ids=lambda d: str(d)[6:])
@pytest.mark.parametrize("case", CASES, ids=[f"{c[0]}d-h{c[3]}c{c[4]}" for c in CASES])
def test_head_major_matches_oracle(monkeypatch, case, dtype, plan):
    ndim, B, Q, H, C, P, shapes = case
    _set_env(monkeypatch, plan)
    value, shp, loc, attn, go = make_inputs(B, Q, H, C, P, shapes, seed=Q + H + ndim,
                                            loc_range=(-0.1, 1.1))
    inp = [t.to(DEV, dtype) for t in (value, loc, attn, go)]
    vhm = head_major(inp[0])
    assert _core.prepare_value(vhm) is vhm  # read in place, no copy
    assert _core.value_code(vhm) & _lib.VALUE_HEAD_MAJOR
    got, gv = _fwd_bwd(ndim, vhm, shp, inp[1], inp[2], inp[3])
    assert gv.stride() == vhm.stride()  # grad_value written head-major
    ref = oracle_all(*[t.float().cpu() for t in (inp[0], shp, inp[1], inp[2], inp[3])])
    tf, tg = (TOL_FWD_F32, TOL_GRAD_F32) if dtype == torch.float32 else (TOL_HALF, TOL_HALF)
    check_all(got, ref, tf, tg, f"head-major {plan} {dtype}")
    # the forward is the same arithmetic in either layout
    dense, _ = _fwd_bwd(ndim, inp[0], shp, inp[1], inp[2], inp[3])
    assert torch.equal(got[0], dense[0])


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("ndim", [2, 3])
def test_head_major_device_shapes(ndim, dtype):
    """Device-resident level shapes (the gather/scatter plan, full-size fp32
    accumulator for 16-bit values)."""
    shapes = [(30, 40), (15, 20)] if ndim == 2 else [(10, 12, 14), (5, 6, 7)]
    value, shp, loc, attn, go = make_inputs(2, 400, 4, 32, 4, shapes, seed=5 + ndim)
    inp = [t.to(DEV, dtype) for t in (value, loc, attn, go)]
    got, _ = _fwd_bwd(ndim, head_major(inp[0]), shp.to(DEV), inp[1], inp[2], inp[3])
    ref = oracle_all(*[t.float().cpu() for t in (inp[0], shp, inp[1], inp[2], inp[3])])
    tf, tg = (TOL_FWD_F32, TOL_GRAD_F32) if dtype == torch.float32 else (TOL_HALF, TOL_HALF)
    check_all(got, ref, tf, tg, f"head-major device shapes {dtype}")


@pytest.mark.parametrize("ndim", [2, 3])
def test_head_major_fused(ndim):
    """The fused prologue on a head-major value against the dense layout."""
    shapes = [(20, 24), (10, 12)] if ndim == 2 else [(6, 8, 10), (3, 4, 5)]
    value, shp, ref, off, logits, go = fused_inputs(ndim, 2, 50, 4, 32, 4, shapes, seed=9)
    fused = M.msda3d_fused if ndim == 3 else M.msda2d_fused
    t = [x.to(DEV) for x in (value, ref, off, logits)]
    fn = lambda v, r, o, lg: fused(v, shp, r, o, lg, True, 1e-4)
    want = fused_run(fn, t, go.to(DEV))
    got = fused_run(lambda v, r, o, lg: fn(head_major(v), r, o, lg), t, go.to(DEV))
    assert torch.equal(got[0], want[0])
    for name, a, b in zip(("value", "ref", "offsets", "logits"), got[1:], want[1:]):
        torch.testing.assert_close(a, b, rtol=1e-4, atol=1e-4, msg=lambda m, n=name: f"{n}: {m}")


def test_other_strides_are_copied():
    """A value view that is neither layout is made dense (B, K, H, C) first."""
    v = torch.randn(2, 10, 8, 32, device=DEV)[:, :, ::2]
    assert not _core.is_head_major(v)
    pv = _core.prepare_value(v)
    assert pv.is_contiguous() and torch.equal(pv, v)
