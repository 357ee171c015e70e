"""The CPU oracle (oracle/msda_oracle.c) pinned against the reference.

The golden vectors in tests/golden/ were produced by the reference's own
msda2d_pytorch / msda3d_pytorch (grid_sample based) on seeded inputs by
tests/golden/make_golden.py.  Before the oracle is trusted as the checker of
the CUDA kernels it must reproduce every one of them within the parity bar.
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle import msda_bwd_oracle, msda_cell_oracle, msda_fwd_oracle
from tests._util import TOL_FWD_F32, TOL_GRAD_F32, assert_close, make_inputs
from tests.conftest import golden_names, load_golden


@pytest.mark.parametrize("name", golden_names())
def test_oracle_matches_reference_golden(name):
    z = load_golden(name)
    clamp, eps = bool(z["clamp"]), float(z["eps"])
    out = msda_fwd_oracle(z["value"], z["shapes"], z["loc"], z["attn"], clamp, eps)
    assert_close(out, z["out"], TOL_FWD_F32, f"{name} out")
    gv, gl, ga = msda_bwd_oracle(z["value"], z["shapes"], z["loc"], z["attn"], z["grad_out"],
                                 clamp, eps)
    assert_close(gv, z["grad_value"], TOL_GRAD_F32, f"{name} grad_value")
    assert_close(gl, z["grad_loc"], TOL_GRAD_F32, f"{name} grad_loc")
    assert_close(ga, z["grad_attn"], TOL_GRAD_F32, f"{name} grad_attn")


def test_golden_set_covers_reference_cases():
    names = set(golden_names())
    for required in ("cfg0_2d", "basic_3d", "boundary_2d", "boundary_3d", "oob_clamp_3d",
                     "noclamp_2d", "noclamp_3d", "single_level_3d", "ragged_2d", "empty_q_2d"):
        assert required in names


def test_cell_known_answers():
    # loc 0.5 on 4 cells: g = 0, ix = ((0+1)*4-1)/2 = 1.5 -> lower corner 1.
    assert msda_cell_oracle(0.5, 4) == 1
    # loc 0 with clamp: g = -1+1e-4, ix = -0.4998 -> corner -1 (zero padding).
    assert msda_cell_oracle(0.0, 4, True) == -1
    # loc 1 with clamp: g = 1-1e-4, ix = 3.4998 -> corner 3 (its +1 neighbour is padding).
    assert msda_cell_oracle(1.0, 4, True) == 3
    # Cell centres: loc = (i + 0.5)/size resolves exactly to cell i when every
    # step is exact in float (power-of-two sizes; other sizes may round to the
    # neighbouring cell, exactly as grid_sample does).
    for size in (2, 4, 64, 128):
        for i in range(size):
            assert msda_cell_oracle((i + 0.5) / size, size) == i


def test_constant_value_gives_weight_sum():
    # Constant value and interior locations: every sample reads the constant,
    # so out = const * sum of the weights of the row.
    B, Q, H, C, P = 2, 16, 3, 8, 4
    shapes = [(6, 7), (3, 4)]
    value, shp, loc, attn, _ = make_inputs(B, Q, H, C, P, shapes, seed=3, loc_range=(0.2, 0.8))
    value = np.full(value.shape, 1.75, dtype=np.float32)
    attn = attn.numpy() * 1.3  # weights need not sum to 1 (the reference does not require it)
    out = msda_fwd_oracle(value, shp, loc, attn)
    expect = 1.75 * attn.sum(axis=(3, 4))  # (B, Q, H)
    np.testing.assert_allclose(out.reshape(B, Q, H, C), np.repeat(expect[..., None], C, -1),
                               rtol=1e-6, atol=1e-6)


def test_voxel_centre_reads_exact_row():
    # A point at a voxel centre has fractional offset 0: it reads exactly that row.
    shapes = [(3, 4, 5)]
    B, Q, H, C, P = 1, 1, 2, 4, 1
    value, shp, loc, attn, _ = make_inputs(B, Q, H, C, P, shapes, seed=5)
    z, y, x = 2, 1, 3
    loc = loc.numpy()
    loc[0, 0, :, 0, 0, :] = [(x + 0.5) / 5, (y + 0.5) / 4, (z + 0.5) / 3]
    attn = np.ones((B, Q, H, 1, P), dtype=np.float32)
    out = msda_fwd_oracle(value, shp, loc, attn).reshape(H, C)
    key = (z * 4 + y) * 5 + x
    np.testing.assert_allclose(out, value.numpy()[0, key], rtol=0, atol=1e-6)


def test_corners_outside_volume_read_zero():
    # clamp_grid=False and a location far outside: every corner is padding.
    shapes = [(4, 4)]
    value, shp, loc, attn, go = make_inputs(1, 3, 1, 4, 1, shapes, seed=9)
    loc = loc.numpy()
    loc[0, :, 0, 0, 0, :] = [[-3.0, 0.5], [0.5, 4.0], [-1.0, -1.0]]
    out = msda_fwd_oracle(value, shp, loc, attn, clamp_grid=False)
    assert np.all(out == 0.0)
    gv, gl, ga = msda_bwd_oracle(value, shp, loc, attn, go, clamp_grid=False)
    assert np.all(gv == 0.0) and np.all(gl == 0.0) and np.all(ga == 0.0)


def test_oracle_thread_count_invariant():
    B, Q, H, C, P = 2, 40, 4, 16, 4
    shapes = [(4, 5, 6), (2, 3, 3)]
    value, shp, loc, attn, go = make_inputs(B, Q, H, C, P, shapes, seed=11)
    o1 = msda_fwd_oracle(value, shp, loc, attn, nthreads=1)
    o8 = msda_fwd_oracle(value, shp, loc, attn, nthreads=8)
    assert np.array_equal(o1, o8)
    g1 = msda_bwd_oracle(value, shp, loc, attn, go, nthreads=1)
    g8 = msda_bwd_oracle(value, shp, loc, attn, go, nthreads=8)
    for a, b in zip(g1, g8):
        assert np.array_equal(a, b)


def test_oracle_rejects_inconsistent_k():
    value, shp, loc, attn, _ = make_inputs(1, 2, 1, 4, 1, [(4, 4)], seed=1)
    with pytest.raises(ValueError):
        msda_fwd_oracle(value[:, :15], shp, loc, attn)


@pytest.mark.parametrize("ndim,shapes", [(2, [(6, 7), (3, 4)]), (3, [(4, 5, 6), (2, 3, 3)])])
def test_gradients_are_derivatives_of_the_forward(ndim, shapes):
    """Central differences of the oracle's forward against its backward, a
    check independent of the golden vectors: with S(x) = <grad_out, out(x)>,
    every gradient the backward returns must be dS/dx.  Locations sit at
    cell fractions in [0.25, 0.75] so each +-h step stays inside its cell,
    where the interpolation is linear along the stepped axis."""
    rng = np.random.default_rng(17)
    B, Q, H, C, P = 1, 4, 2, 3, 2
    L = len(shapes)
    K = int(sum(np.prod(s) for s in shapes))
    value = rng.standard_normal((B, K, H, C)).astype(np.float32)
    attn = rng.uniform(0.2, 1.0, (B, Q, H, L, P)).astype(np.float32)
    go = rng.standard_normal((B, Q, H * C)).astype(np.float32)
    loc = np.empty((B, Q, H, L, P, ndim), dtype=np.float32)
    for lvl, s in enumerate(shapes):
        for ax in range(ndim):
            n = s[ndim - 1 - ax]  # axis 0 is x (W-indexed), the last shapes entry
            cell = rng.integers(0, n - 1, (B, Q, H, P))
            frac = rng.uniform(0.25, 0.75, (B, Q, H, P))
            loc[:, :, :, lvl, :, ax] = (cell + frac + 0.5) / n  # ix = loc * n - 0.5
    shp = np.array(shapes, dtype=np.int64)
    gv, gl, ga = msda_bwd_oracle(value, shp, loc, attn, go)

    def score(v=value, lo=loc, a=attn):
        return float(np.dot(msda_fwd_oracle(v, shp, lo, a).ravel().astype(np.float64),
                            go.ravel().astype(np.float64)))

    def central(array, idx, h, **which):
        up, dn = array.copy(), array.copy()
        up[idx] += h
        dn[idx] -= h
        key = next(iter(which))
        return (score(**{key: up}) - score(**{key: dn})) / (2 * h)

    for _ in range(8):
        b, q, hh, lvl, p = (int(rng.integers(0, m)) for m in (B, Q, H, L, P))
        for ax in range(ndim):
            n = shapes[lvl][ndim - 1 - ax]
            idx = (b, q, hh, lvl, p, ax)
            fd = central(loc, idx, 0.1 / n, lo=loc)
            np.testing.assert_allclose(gl[idx], fd, rtol=2e-2, atol=2e-3)
        idx = (b, q, hh, lvl, p)
        np.testing.assert_allclose(ga[idx], central(attn, idx, 0.05, a=attn), rtol=1e-2, atol=1e-3)
        idx = (0, int(rng.integers(0, K)), hh, int(rng.integers(0, C)))
        np.testing.assert_allclose(gv[idx], central(value, idx, 0.05, v=value), rtol=1e-2,
                                   atol=1e-3)
