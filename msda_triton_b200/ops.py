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


# ---------------------------------------------------------------- fused prologue
@torch.library.custom_op("msda_b200::msda_fused_forward", mutates_args=())
def msda_fused_forward(value: Tensor, spatial_shapes: Tensor, reference_points: Tensor,
                       sampling_offsets: Tensor, attention_logits: Tensor, ndim: int,
                       clamp_grid: bool, clamp_eps: float) -> Tensor:
    """(B, Q, H*C) output of msda{2,3}d_fused (locations and weights formed in the kernels)."""
    from msda_triton_b200 import fused

    with torch.no_grad():
        return fused.MSDAFusedFn.apply(ndim, value, spatial_shapes, reference_points,
                                       sampling_offsets, attention_logits, clamp_grid, clamp_eps)


@msda_fused_forward.register_fake
def _msda_fused_forward_fake(value, spatial_shapes, reference_points, sampling_offsets,
                             attention_logits, ndim, clamp_grid, clamp_eps):
    B, _, H, C = value.shape
    return value.new_empty((B, sampling_offsets.shape[1], H * C))


@torch.library.custom_op("msda_b200::msda_fused_backward", mutates_args=())
def msda_fused_backward(grad_output: Tensor, value: Tensor, spatial_shapes: Tensor,
                        reference_points: Tensor, sampling_offsets: Tensor,
                        attention_logits: Tensor, ndim: int, clamp_grid: bool,
                        clamp_eps: float) -> tuple[Tensor, Tensor, Tensor, Tensor]:
    """(grad_value, grad_reference_points, grad_sampling_offsets,
    grad_attention_logits), each in the dtype and shape of its input."""
    from msda_triton_b200 import fused

    return fused.fused_backward(ndim, grad_output, value, spatial_shapes, reference_points,
                                sampling_offsets, attention_logits, clamp_grid, clamp_eps)


@msda_fused_backward.register_fake
def _msda_fused_backward_fake(grad_output, value, spatial_shapes, reference_points,
                              sampling_offsets, attention_logits, ndim, clamp_grid, clamp_eps):
    fmt = torch.contiguous_format
    return tuple(torch.empty_like(t, memory_format=fmt)
                 for t in (value, reference_points, sampling_offsets, attention_logits))


def _fused_setup_context(ctx, inputs, output):
    value, spatial_shapes, ref, off, logits, ndim, clamp_grid, clamp_eps = inputs
    ctx.save_for_backward(value, spatial_shapes, ref, off, logits)
    ctx.ndim = ndim
    ctx.clamp_grid = clamp_grid
    ctx.clamp_eps = clamp_eps


def _fused_backward(ctx, grad_output):
    value, spatial_shapes, ref, off, logits = ctx.saved_tensors
    gv, gr, go, gl = msda_fused_backward(grad_output.contiguous(), value, spatial_shapes, ref,
                                         off, logits, ctx.ndim, ctx.clamp_grid, ctx.clamp_eps)
    return gv, None, gr, go, gl, None, None, None


msda_fused_forward.register_autograd(_fused_backward, setup_context=_fused_setup_context)

__all__ += ["msda_fused_forward", "msda_fused_backward"]
