"""The binned backward (sample bins + shared-memory tiles) against the oracle.

The library picks the binned backward for large problems with host-resident
shapes.  These tests force it (MSDA_BWD_PATH=binned) on small problems and
use the tuning knobs to exercise every branch: tiny tiles (most samples
straddle several tiles, so secondary records dominate), levels reduced
through the fp32 accumulator, and work items split across CTAs.
"""

from __future__ import annotations

import pytest
import torch

from tests._util import TOL_FWD_F32, TOL_GRAD_F32, TOL_HALF, make_inputs
from tests.conftest import golden_names, load_golden
from tests.test_msda_gpu import check_all, cuda_fwd_bwd, oracle_all

pytestmark = pytest.mark.gpu


@pytest.fixture
def binned(monkeypatch):
    monkeypatch.setenv("MSDA_BWD_PATH", "binned")

    def knobs(tile=None, atomic_records=None, smax=None):
        for key, val in (("MSDA_BIN_TILE", tile), ("MSDA_BIN_ATOMIC_RECORDS", atomic_records),
                         ("MSDA_BIN_SMAX", smax)):
            if val is None:
                monkeypatch.delenv(key, raising=False)
            else:
                monkeypatch.setenv(key, str(val))

    return knobs


@pytest.mark.parametrize("name", golden_names())
def test_golden_parity_binned(binned, name):
    z = load_golden(name)
    t = {k: torch.from_numpy(z[k]) for k in ("value", "loc", "attn", "grad_out", "shapes")}
    ndim = t["shapes"].shape[1]
    clamp, eps = bool(z["clamp"]), float(z["eps"])
    got = cuda_fwd_bwd(ndim, t["value"], t["shapes"], t["loc"], t["attn"], t["grad_out"],
                       clamp, eps)
    ref = [torch.from_numpy(z[k]) for k in ("out", "grad_value", "grad_loc", "grad_attn")]
    check_all(got, ref, TOL_FWD_F32, TOL_GRAD_F32, f"{name} binned vs reference")


STRESS = [
    # ndim, B, Q, H, C, P, shapes, tile, atomic_records, smax
    (2, 2, 300, 4, 32, 4, [(20, 30), (10, 15), (5, 8)], "2,2", None, None),
    (2, 2, 300, 4, 32, 4, [(20, 30), (10, 15), (5, 8)], "4,2", 64, 32),
    (2, 1, 500, 2, 64, 3, [(33, 17), (9, 4)], "8,4", 100, 64),
    (3, 2, 200, 4, 32, 4, [(8, 10, 12), (4, 5, 6), (2, 3, 3)], "2,2,2", None, None),
    (3, 2, 200, 4, 32, 4, [(8, 10, 12), (4, 5, 6), (2, 3, 3)], "4,2,2", 50, 16),
    (3, 1, 400, 8, 16, 2, [(9, 7, 11), (3, 3, 3)], "4,4,4", 30, 8),
]


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("case", STRESS, ids=[f"{c[0]}d-tile{c[7]}-at{c[8]}" for c in STRESS])
def test_binned_stress(binned, case, dtype):
    ndim, B, Q, H, C, P, shapes, tile, atomic_records, smax = case
    binned(tile=tile, atomic_records=atomic_records, smax=smax)
    for clamp, rng in ((True, (0.0, 1.0)), (False, (-0.2, 1.2))):
        inp = make_inputs(B, Q, H, C, P, shapes, seed=Q + C, loc_range=rng)
        inp = [x.to(dtype) if x.is_floating_point() else x for x in inp]
        got = cuda_fwd_bwd(ndim, *inp, clamp=clamp)
        ref = oracle_all(*[x.float() if x.is_floating_point() else x for x in inp], clamp=clamp)
        half = dtype != torch.float32
        check_all(got, ref, TOL_HALF if half else TOL_FWD_F32, TOL_HALF if half else TOL_GRAD_F32,
                  f"{case} {dtype} clamp={clamp}")


@pytest.mark.parametrize("ndim", [2, 3])
def test_binned_tile_boundary_points(binned, ndim):
    """Lower corners exactly on the last column/row/slab of a tile: every such
    sample straddles into the next tile along that axis."""
    binned(tile="4,4" if ndim == 2 else "4,4,4")
    shapes = [(16, 16)] if ndim == 2 else [(8, 8, 8)]
    B, Q, H, C, P = 1, 64, 2, 32, 4
    value, shp, loc, attn, go = make_inputs(B, Q, H, C, P, shapes, seed=7)
    size = shapes[0][0]
    # ix = ((2*loc-1)+1)*size - 1)/2 = loc*size - 0.5; a lower corner of 3
    # (last column of tile 0 when T=4) needs loc*size in [3.5, 4.5).
    frac = torch.rand(B, Q, H, 1, P, ndim) * 0.98 + 0.01
    col = torch.randint(0, size // 4, (B, Q, H, 1, P, ndim)) * 4 + 3
    loc = ((col.float() + 0.5 + frac) / size).clamp(max=1.0)
    got = cuda_fwd_bwd(ndim, value, shp, loc, attn, go)
    check_all(got, oracle_all(value, shp, loc, attn, go), TOL_FWD_F32, TOL_GRAD_F32, "tile edge")


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("ndim", [2, 3])
def test_binned_matches_gather(monkeypatch, ndim, dtype):
    """Both backward implementations on one medium problem."""
    shapes = [(40, 60), (20, 30), (10, 15), (5, 8)] if ndim == 2 else \
        [(16, 24, 24), (8, 12, 12), (4, 6, 6)]
    inp = make_inputs(2, 3000, 8, 32, 4, shapes, seed=11)
    inp = [x.to(dtype) if x.is_floating_point() else x for x in inp]
    monkeypatch.setenv("MSDA_BWD_PATH", "gather")
    a = cuda_fwd_bwd(ndim, *inp)
    monkeypatch.setenv("MSDA_BWD_PATH", "binned")
    b = cuda_fwd_bwd(ndim, *inp)
    tol = 1e-5 if dtype == torch.float32 else 1e-2
    check_all(b, a, tol, tol, "binned vs gather")


@pytest.mark.parametrize("ndim", [2, 3])
def test_binned_mixed_dtype(binned, ndim):
    binned(tile="4,4" if ndim == 2 else "4,4,2", atomic_records=40, smax=16)
    shapes = [(12, 20), (6, 10)] if ndim == 2 else [(6, 8, 10), (3, 4, 5)]
    value, shp, loc, attn, go = make_inputs(2, 150, 4, 32, 4, shapes, seed=3)
    got = cuda_fwd_bwd(ndim, value.bfloat16(), shp, loc, attn, go.bfloat16())
    ref = oracle_all(value.bfloat16().float(), shp, loc, attn, go.bfloat16().float())
    check_all(got, ref, TOL_HALF, TOL_HALF, "binned bf16 value, fp32 sampling")
