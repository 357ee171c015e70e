"""The custom-op path on the GPU: torch.library.opcheck, torch.compile with
fullgraph=True (no graph break at the MSDA call), and CUDA-graph capture and
replay of the forward and backward -- each against the eager kernels."""

from __future__ import annotations

import pytest
import torch

import msda_triton_b200 as M
from msda_triton_b200 import ops
from tests._util import make_inputs

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)
SHAPES = {2: [(12, 16), (6, 8)], 3: [(6, 8, 8), (3, 4, 4)]}


def _inputs(ndim, dtype=torch.float32, sdtype=None, seed=0, device_shapes=False):
    value, shp, loc, attn, go = make_inputs(2, 50, 4, 16, 3, SHAPES[ndim], seed=seed)
    sdtype = sdtype or dtype
    value, go = value.to(DEV, dtype), go.to(DEV, dtype)
    loc, attn = loc.to(DEV, sdtype), attn.to(DEV, sdtype)
    return value, shp.to(DEV) if device_shapes else shp, loc, attn, go


@pytest.mark.parametrize("ndim", [2, 3])
@pytest.mark.parametrize("dtype,sdtype,dev_shapes", [(torch.float32, None, False),
                                                     (torch.bfloat16, None, True),
                                                     (torch.float16, torch.float32, False)])
def test_opcheck(monkeypatch, ndim, dtype, sdtype, dev_shapes):
    if dtype == torch.float16:
        # opcheck compares two runs of the backward at fp16's default rtol (1e-3);
        # fp16 reductions straight into grad_value round at every atomic add, so
        # their order moves results by 1-2 fp16 ulps between runs.  Accumulate
        # in fp32 here (one rounding at the end).
        monkeypatch.setenv("MSDA_BWD_DIRECT16", "0")
    value, shp, loc, attn, go = _inputs(ndim, dtype, sdtype, device_shapes=dev_shapes)
    value.requires_grad_(True)
    loc.requires_grad_(True)
    attn.requires_grad_(True)
    torch.library.opcheck(ops.msda_forward, (value, shp, loc, attn, ndim, True, 1e-4))
    torch.library.opcheck(ops.msda_backward,
                          (go, value.detach(), shp, loc.detach(), attn.detach(), ndim, True, 1e-4))


@pytest.mark.parametrize("ndim", [2, 3])
def test_compile_fullgraph_matches_eager(ndim):
    fn = M.msda3d if ndim == 3 else M.msda2d
    value, shp, loc, attn, go = _inputs(ndim, seed=3)

    def step(v, lo, a):
        out = fn(v, shp, lo, a)
        return (out * go).sum() + 0.5 * out.square().mean()

    def grads(f):
        v, lo, a = (t.clone().requires_grad_(True) for t in (value, loc, attn))
        loss = f(v, lo, a)
        return [loss.detach(), *torch.autograd.grad(loss, (v, lo, a))]

    eager = grads(step)
    compiled = grads(torch.compile(step, fullgraph=True, backend="aot_eager"))
    for e, c in zip(eager, compiled):
        torch.testing.assert_close(c, e, rtol=1e-6, atol=1e-6)

    fwd = M.msda3d_fwd if ndim == 3 else M.msda2d_fwd
    cfwd = torch.compile(lambda v, lo, a: fwd(v, shp, lo, a) * 2.0, fullgraph=True,
                         backend="aot_eager")
    assert torch.equal(cfwd(value, loc, attn), fwd(value, shp, loc, attn) * 2.0)


@pytest.mark.parametrize("ndim", [2, 3])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_cuda_graph_capture_and_replay(ndim, dtype):
    value, shp, loc, attn, go = _inputs(ndim, dtype, seed=5)
    fwd = M.msda3d_fwd if ndim == 3 else M.msda2d_fwd

    def run():
        out = fwd(value, shp, loc, attn)
        return (out, *ops.msda_backward(go, value, shp, loc, attn, ndim, True, 1e-4))

    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(2):
            run()
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        static = run()
    # new inputs in place, replay, compare with an eager run on the same data
    fresh = _inputs(ndim, dtype, seed=6)
    for dst, src in zip((value, loc, attn, go), (fresh[0], fresh[2], fresh[3], fresh[4])):
        dst.copy_(src)
    graph.replay()
    torch.cuda.synchronize()
    eager = run()
    # output, grad_loc and grad_attn have one writer per element: bitwise equal;
    # grad_value is summed by atomics, whose order may differ between runs
    for i in (0, 2, 3):
        assert torch.equal(static[i], eager[i])
    tol = 1e-5 if dtype == torch.float32 else 1e-2
    torch.testing.assert_close(static[1], eager[1], rtol=tol, atol=tol)


@pytest.mark.parametrize("ndim", [2, 3])
def test_fused_opcheck_and_compile(ndim):
    """The fused-prologue ops: opcheck, and a compiled module-like step with
    fullgraph=True against eager."""
    value, shp, loc, attn, go = _inputs(ndim, seed=9)
    B, Q, H, L, P, _ = loc.shape
    g = torch.Generator(device=DEV).manual_seed(1)
    ref = torch.rand(B, Q, L, ndim, generator=g, device=DEV)
    off = torch.randn(B, Q, H, L, P, ndim, generator=g, device=DEV)
    logits = torch.randn(B, Q, H, L * P, generator=g, device=DEV)
    args = [t.clone().requires_grad_(True) for t in (value, ref, off, logits)]
    torch.library.opcheck(ops.msda_fused_forward, (args[0], shp, *args[1:], ndim, True, 1e-4))
    fused = M.msda3d_fused if ndim == 3 else M.msda2d_fused

    def step(v, r, o, lg):
        return (fused(v, shp, r, o, lg) * go).sum()

    def grads(f):
        xs = [t.clone().requires_grad_(True) for t in (value, ref, off, logits)]
        loss = f(*xs)
        return [loss.detach(), *torch.autograd.grad(loss, xs)]

    eager = grads(step)
    compiled = grads(torch.compile(step, fullgraph=True, backend="aot_eager"))
    for e, c in zip(eager, compiled):
        torch.testing.assert_close(c, e, rtol=1e-5, atol=1e-5)
