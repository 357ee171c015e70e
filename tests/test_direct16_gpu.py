"""Backward of 16-bit values with per-level value-gradient targets, the
opt-in mode of the gather/scatter backward (MSDA_BWD_DIRECT16=1).

Levels with at most 8 expected contributions per grad_value element reduce
with 16-bit vector reductions straight into grad_value (as the reference's
atomic_add into a grad_value of the input dtype does); busier levels keep
fp32 accumulation in a workspace that holds only their keys, rounded into
grad_value by a cast kernel.  Every case below mixes the two, on uniformly
spread locations (the assumption of the contribution bound), and is checked
against the oracle at the half-precision bar.  The default keeps every level
in fp32 (clustered locations: tests/test_sorted_gpu.py).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from msda_triton_b200 import _lib
from tests._util import TOL_HALF, make_inputs
from tests.test_msda_gpu import check_all, cuda_fwd_bwd, oracle_all

pytestmark = pytest.mark.gpu

HALF = [torch.bfloat16, torch.float16]


@pytest.fixture(autouse=True)
def direct16_scatter(monkeypatch):
    monkeypatch.setenv("MSDA_BWD_PATH", "scatter")
    monkeypatch.setenv("MSDA_BWD_DIRECT16", "1")


def _workspace(ndim, dtype, B, shapes, H, C, Q, P):
    shp = np.ascontiguousarray(np.array(shapes, dtype=np.int32))
    K = int(sum(np.prod(s) for s in shapes))
    code = _lib.BFLOAT16 if dtype == torch.bfloat16 else _lib.FLOAT16
    return _lib.lib().msda_bwd_workspace_bytes(ndim, code, B, K, H, C, shp.ctypes.data, 0,
                                               len(shapes), Q, P)


def _run(ndim, dtype, B, Q, H, C, P, shapes, seed, clamp=True, loc_range=(0.0, 1.0)):
    inp = make_inputs(B, Q, H, C, P, shapes, seed=seed, loc_range=loc_range)
    half = [x.to(dtype) if x.is_floating_point() else x for x in inp]
    got = cuda_fwd_bwd(ndim, *half, clamp=clamp)
    ref = oracle_all(*[x.float() if x.is_floating_point() else x for x in half], clamp=clamp)
    return got, ref


CASES = [
    # ndim, B, Q, H, C, P, shapes -- fine level direct, the others in fp32
    (2, 2, 500, 4, 32, 4, [(40, 60), (20, 30), (10, 15), (5, 8)]),
    (3, 2, 1000, 4, 32, 4, [(16, 24, 24), (8, 12, 12), (4, 6, 6)]),
    # a direct level between two accumulated ones (compacted key remap)
    (2, 2, 500, 4, 32, 4, [(5, 8), (40, 60), (10, 15)]),
    (3, 1, 600, 8, 16, 2, [(3, 4, 4), (12, 16, 20), (2, 3, 3)]),
    # every level direct: no workspace at all
    (3, 2, 20, 4, 32, 4, [(8, 10, 12), (4, 5, 6)]),
]


@pytest.mark.parametrize("dtype", HALF)
@pytest.mark.parametrize("case", CASES, ids=[f"{c[0]}d-{len(c[6])}lvl-q{c[2]}" for c in CASES])
def test_mixed_targets_match_oracle(case, dtype):
    ndim, B, Q, H, C, P, shapes = case
    K = int(sum(np.prod(s) for s in shapes))
    ws = _workspace(ndim, dtype, B, shapes, H, C, Q, P)
    assert ws < B * K * H * C * 4, "no level was planned as direct"
    for clamp, rng in ((True, (0.0, 1.0)), (False, (-0.1, 1.1))):
        got, ref = _run(ndim, dtype, B, Q, H, C, P, shapes, seed=Q + C, clamp=clamp,
                        loc_range=rng)
        check_all(got, ref, TOL_HALF, TOL_HALF, f"{case} {dtype} clamp={clamp}")


@pytest.mark.parametrize("dtype", HALF)
@pytest.mark.parametrize("ndim,C,H", [(2, 3, 2), (3, 6, 2), (2, 2, 3), (3, 20, 1)])
def test_narrow_rows(ndim, dtype, C, H):
    """Rows too narrow for 8-byte chunks: scalar and pair reductions, and the
    scalar cast of the compacted accumulator (H*C not a multiple of 4)."""
    shapes = [(30, 40), (6, 8)] if ndim == 2 else [(10, 12, 14), (3, 4, 4)]
    got, ref = _run(ndim, dtype, 2, 300, H, C, 4, shapes, seed=C * 7 + H)
    check_all(got, ref, TOL_HALF, TOL_HALF, f"C={C} H={H} {dtype}")


@pytest.mark.parametrize("ndim", [2, 3])
def test_direct_and_fp32_accumulation_agree(monkeypatch, ndim):
    """The same problem with the direct levels switched off: the per-sample
    gradients and the output are identical, grad_value agrees at the bar."""
    shapes = CASES[0][6] if ndim == 2 else CASES[1][6]
    B, Q, H, C, P = 2, 800, 4, 32, 4
    inp = make_inputs(B, Q, H, C, P, shapes, seed=5)
    inp = [x.to(torch.bfloat16) if x.is_floating_point() else x for x in inp]
    a = cuda_fwd_bwd(ndim, *inp)
    monkeypatch.setenv("MSDA_BWD_DIRECT16", "0")
    b = cuda_fwd_bwd(ndim, *inp)
    for i in (0, 2, 3):
        assert torch.equal(a[i], b[i])
    check_all(a, b, TOL_HALF, TOL_HALF, "direct vs fp32 accumulation")
