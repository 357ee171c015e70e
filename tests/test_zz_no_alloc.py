"""msda_bwd_static_scratch: the backward for callers that cannot allocate
device memory (for example an inference-engine plugin that may not call
cudaMalloc).  It must give the same gradients as msda{2,3}d_bwd with a
caller-allocated workspace, on consecutive calls (the shared static scratch
is re-cleared by every call), and reject problems larger than its 32 MiB
scratch.  This file is collected last on purpose."""

from __future__ import annotations

import pytest
import torch

from msda_triton_b200 import _core, _lib
from tests._util import TOL_GRAD_F32, TOL_HALF, assert_close, make_inputs

pytestmark = pytest.mark.gpu

SHAPES = {2: [(24, 32), (12, 16), (6, 8)], 3: [(8, 12, 12), (4, 6, 6), (2, 3, 3)]}


def _call_static(ndim, value, shapes, loc, attn, go):
    lib = _lib.lib()
    gv = torch.empty_like(value)
    gl = torch.empty_like(loc)
    ga = torch.empty_like(attn)
    with torch.cuda.device(value.device):
        rc = lib.msda_bwd_static_scratch(
            ndim, *_core._common_args(value, shapes, shapes.is_cuda, loc, attn), 1, 1e-4,
            go.data_ptr(), gv.data_ptr(), gl.data_ptr(), ga.data_ptr(),
            torch.cuda.current_stream(value.device).cuda_stream)
    return rc, gv, gl, ga


def _check_against_workspace_backward(ndim, dtype, dev, shapes, seed):
    value, _, loc, attn, go = make_inputs(2, 300, 4, 32, 4, SHAPES[ndim], seed=seed,
                                          dtype=dtype, device=dev)
    host_shapes = torch.tensor(SHAPES[ndim], dtype=torch.int32)
    with torch.cuda.device(dev):
        ref = _core.backward(ndim, value, host_shapes, False, loc, attn, True, 1e-4, go)
    rc, *got = _call_static(ndim, value, shapes, loc, attn, go)
    assert rc == _lib.SUCCESS, _lib.last_error()
    torch.cuda.synchronize(dev)
    tol = TOL_GRAD_F32 if dtype == torch.float32 else TOL_HALF
    for name, g, r in zip(("grad_value", "grad_loc", "grad_attn"), got, ref):
        assert_close(g.float().cpu(), r.float().cpu(), tol,
                     f"{ndim}D {dtype} {dev} shapes on {shapes.device} seed={seed} {name}")


@pytest.mark.parametrize("ndim", [2, 3])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_static_scratch_matches_workspace_backward(ndim, dtype):
    dev = torch.device("cuda", 0)
    shapes = torch.tensor(SHAPES[ndim], dtype=torch.int32)
    for seed in (1, 2):  # two calls in a row; the second must not see the first's sums
        _check_against_workspace_backward(ndim, dtype, dev, shapes, seed)


@pytest.mark.parametrize("ndim", [2, 3])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_static_scratch_device_resident_shapes(ndim, dtype):
    """spatial_shapes on the device: the scratch size is then planned from the
    problem's bounds (no host copy of the table), the kernels read the table
    from device memory."""
    dev = torch.device("cuda", 0)
    shapes = torch.tensor(SHAPES[ndim], dtype=torch.int32, device=dev)
    for seed in (3, 4):
        _check_against_workspace_backward(ndim, dtype, dev, shapes, seed)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two visible GPUs")
@pytest.mark.parametrize("ndim", [2, 3])
def test_static_scratch_second_device(ndim):
    """A call on device 1 uses device 1's copy of the array (its own slot of the
    address cache), then device 0 again still gets its own."""
    shapes = torch.tensor(SHAPES[ndim], dtype=torch.int32)
    for i, seed in ((1, 5), (0, 6), (1, 7)):
        _check_against_workspace_backward(ndim, torch.bfloat16, torch.device("cuda", i),
                                          shapes, seed)


def test_static_scratch_rejects_oversized_problem():
    # 4 corners * 25000 queries * 2 points on 20000 cells = 10 contributions per
    # element: the level is accumulated in fp32, 3 * 20000 * 8 * 32 * 4 bytes =
    # 61 MB > 32 MiB: rejected on the host before any launch.
    dev = torch.device("cuda", 0)
    shapes = torch.tensor([[100, 200]], dtype=torch.int32)
    value = torch.zeros(3, 20000, 8, 32, device=dev, dtype=torch.bfloat16)
    loc = torch.zeros(3, 25000, 8, 1, 2, 2, device=dev, dtype=torch.bfloat16)
    attn = torch.zeros(3, 25000, 8, 1, 2, device=dev, dtype=torch.bfloat16)
    go = torch.zeros(3, 25000, 256, device=dev, dtype=torch.bfloat16)
    rc, *_ = _call_static(2, value, shapes, loc, attn, go)
    assert rc == _lib.ERROR_WORKSPACE
    assert "static scratch holds" in _lib.last_error()
