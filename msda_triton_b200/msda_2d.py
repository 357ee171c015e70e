"""2D multi-scale deformable attention on B200 (bilinear sampling).

Drop-in for the reference's src/msda_triton/triton/msda_2d.py: same names
(msda2d, msda2d_fwd, MSDA2DFn), signatures, defaults, tensor contract and
error behaviour; the work runs in the hand-written sm_100a kernels of
libmsda_b200.so.
"""

from __future__ import annotations

import torch

from msda_triton_b200 import _core, ops


def msda2d_fwd(
    value: torch.Tensor,
    value_spatial_shapes: torch.Tensor,
    sampling_locations: torch.Tensor,
    attention_weights: torch.Tensor,
    clamp_grid: bool = True,
    clamp_eps: float = 1e-4,
) -> torch.Tensor:
    """Forward-only 2D MSDA (no autograd graph); use msda2d() for training.

    out[b, q, h*C:(h+1)*C] = sum_{l,p} attention_weights[b,q,h,l,p] *
        bilinear(value[b, level l, h, :], sampling_locations[b,q,h,l,p])

    Args:
        value: (B, K, H, C) features, K = sum_l H_l * W_l flattened level-major.
        value_spatial_shapes: (L, 2) integer (H, W) per level, CPU or CUDA.
        sampling_locations: (B, Q, H, L, P, 2) normalised (x, y) in [0, 1].
        attention_weights: (B, Q, H, L, P).
        clamp_grid: clamp 2*loc-1 to [-1+eps, 1-eps] (grid_sample convention).
        clamp_eps: clamp margin.

    Returns:
        (B, Q, H*C) in value's dtype (fp32 accumulation inside).

    Raises:
        ValueError: non-CUDA inputs, shape mismatch, K != sum of level sizes
            (CPU shapes only).
        NotImplementedError: dtype other than fp32/fp16/bf16.

    Reference: triton/msda_2d.py:654-718.
    """
    if torch.compiler.is_compiling():
        with torch.no_grad():
            return ops.msda_forward(value, value_spatial_shapes, sampling_locations,
                                    attention_weights, 2, clamp_grid, clamp_eps)
    return _core.fwd_entry(2, value, value_spatial_shapes, sampling_locations,
                           attention_weights, clamp_grid, clamp_eps)


class MSDA2DFn(torch.autograd.Function):
    """Autograd Function for 2D MSDA (reference: triton/msda_2d.py:721-853).

    Saves value, the prepared locations/weights and the int32 level shapes;
    the backward produces grad_value, grad_sampling_locations and
    grad_attention_weights in one kernel pass."""

    @staticmethod
    def forward(ctx, value, value_spatial_shapes, sampling_locations, attention_weights,
                clamp_grid=True, clamp_eps=1e-4):
        return _core.fn_forward(2, ctx, value, value_spatial_shapes, sampling_locations,
                                attention_weights, clamp_grid, clamp_eps)

    @staticmethod
    def backward(ctx, grad_output):
        return _core.fn_backward(2, ctx, grad_output)


def msda2d(
    value: torch.Tensor,
    value_spatial_shapes: torch.Tensor,
    sampling_locations: torch.Tensor,
    attention_weights: torch.Tensor,
    clamp_grid: bool = True,
    clamp_eps: float = 1e-4,
) -> torch.Tensor:
    """2D MSDA with autograd -- the training entry point.

    Same arguments and result as msda2d_fwd(); gradients flow to value,
    sampling_locations and attention_weights.  Reference: triton/msda_2d.py:856-907.
    """
    if not value.is_cuda:
        raise ValueError("MSDA2D CUDA kernel requires CUDA tensors. Got CPU tensors instead.")
    if torch.compiler.is_compiling():
        # traced as one opaque op (msda_b200::msda_forward) instead of a graph break
        return ops.msda_forward(value, value_spatial_shapes, sampling_locations,
                                attention_weights, 2, clamp_grid, clamp_eps)
    return MSDA2DFn.apply(value, value_spatial_shapes, sampling_locations, attention_weights,
                          clamp_grid, clamp_eps)


__all__ = ["msda2d", "msda2d_fwd", "MSDA2DFn"]
