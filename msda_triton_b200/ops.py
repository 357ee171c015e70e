"""torch.library registration of the MSDA ops.

The reference hides its kernels from torch.compile (`@torch.compiler.disable`,
src/msda_triton/triton/msda_3d.py:729,797), which costs a graph break at
every call.  Here the forward and backward are registered as custom ops with
fake (meta) implementations and an autograd formula, so torch.compile traces
through them (Dynamo sees an opaque op with known output shapes) and CUDA
graphs capture them like any other kernel launch:

    torch.ops.msda_b200.msda_forward(value, shapes, loc, attn, ndim, clamp, eps)
    torch.ops.msda_b200.msda_backward(grad_out, value, shapes, loc, attn, ndim, clamp, eps)

`msda2d`/`msda3d`/`msda2d_fwd`/`msda3d_fwd` route through these ops while
torch.compile is tracing, and call the autograd Functions directly in eager
mode (no dispatcher overhead).  Both paths run the same C ABI entry points.
"""

from __future__ import annotations

import torch
from torch import Tensor

from msda_triton_b200 import _core


@torch.library.custom_op("msda_b200::msda_forward", mutates_args=())
def msda_forward(value: Tensor, spatial_shapes: Tensor, sampling_locations: Tensor,
                 attention_weights: Tensor, ndim: int, clamp_grid: bool,
                 clamp_eps: float) -> Tensor:
    """(B, Q, H*C) output of MSDA in value's dtype (same checks and errors as msda2d/msda3d)."""
    return _core.fwd_entry(ndim, value, spatial_shapes, sampling_locations, attention_weights,
                           clamp_grid, clamp_eps)


@msda_forward.register_fake
def _msda_forward_fake(value, spatial_shapes, sampling_locations, attention_weights, ndim,
                       clamp_grid, clamp_eps):
    B, _, H, C = value.shape
    return value.new_empty((B, sampling_locations.shape[1], H * C))


@torch.library.custom_op("msda_b200::msda_backward", mutates_args=())
def msda_backward(grad_output: Tensor, value: Tensor, spatial_shapes: Tensor,
                  sampling_locations: Tensor, attention_weights: Tensor, ndim: int,
                  clamp_grid: bool, clamp_eps: float) -> tuple[Tensor, Tensor, Tensor]:
    """(grad_value, grad_sampling_locations, grad_attention_weights), each in the
    dtype of its input."""
    shapes, on_dev = _core.prepare_spatial(spatial_shapes)
    loc, attn = _core.sampling_pair(value, sampling_locations, attention_weights)
    gv, gl, ga = _core.backward(ndim, value.contiguous(), shapes, on_dev, loc, attn, clamp_grid,
                                clamp_eps, grad_output)
    return gv, gl.to(sampling_locations.dtype), ga.to(attention_weights.dtype)


@msda_backward.register_fake
def _msda_backward_fake(grad_output, value, spatial_shapes, sampling_locations,
                        attention_weights, ndim, clamp_grid, clamp_eps):
    fmt = torch.contiguous_format
    return (torch.empty_like(value, memory_format=fmt),
            torch.empty_like(sampling_locations, memory_format=fmt),
            torch.empty_like(attention_weights, memory_format=fmt))


def _setup_context(ctx, inputs, output):
    value, spatial_shapes, loc, attn, ndim, clamp_grid, clamp_eps = inputs
    ctx.save_for_backward(value, spatial_shapes, loc, attn)
    ctx.ndim = ndim
    ctx.clamp_grid = clamp_grid
    ctx.clamp_eps = clamp_eps


def _backward(ctx, grad_output):
    value, spatial_shapes, loc, attn = ctx.saved_tensors
    gv, gl, ga = msda_backward(grad_output.contiguous(), value, spatial_shapes, loc, attn,
                               ctx.ndim, ctx.clamp_grid, ctx.clamp_eps)
    return gv, None, gl, ga, None, None, None


msda_forward.register_autograd(_backward, setup_context=_setup_context)


__all__ = ["msda_forward", "msda_backward"]
