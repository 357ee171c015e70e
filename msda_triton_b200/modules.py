"""MSDA2D / MSDA3D nn.Modules whose sampling runs in the sm_100a kernels.

Drop-in for the reference's modules (src/msda_triton/pytorch/msda_2d.py:117-383,
src/msda_triton/pytorch/msda_3d.py:121-394), which sample with grid_sample:
the same constructor arguments, parameter names and shapes (state_dicts load
either way), init_weights() patterns and RNG use, forward signature,
batch_first / query_pos / key_padding_mask / identity handling, query and
head chunking, gradient checkpointing and errors.  The deformable sampling
itself is msda2d / msda3d of this package; with fused_prologue=True (the
default, an extra keyword the reference's modules ignore) the locations and
softmax weights are formed inside the kernels from the raw projections
(msda2d_fused / msda3d_fused) instead of as separate tensors -- for calls
below FUSED_MAX_SAMPLES samples.  Larger calls form them in two passes of
their own (fused.sampling_prologue: the same rounding as the tensor ops,
the fused kernels' softmax) and call msda2d / msda3d, whose backward is then
the cell-sorted pipeline (the fused kernels' backward is the gather/scatter
one).  With fused_prologue=False, mixed dtypes or under torch.compile
tracing, the locations and weights are the reference's tensor ops.

Forward, with q the (batch-first) query and v the projected value:
    offsets = Linear(q) -> (B, Q, H, L, P, d)
    weights = softmax over L*P of Linear(q) -> (B, Q, H, L, P)
    loc     = reference_points[:, :, None, :, None, :] + offsets / (W, H[, D])_l
    out     = output_proj(msda(v, spatial_shapes, loc, weights))
    return dropout(out) + identity
"""

from __future__ import annotations

import math

import torch
from torch import nn
from torch.utils.checkpoint import checkpoint

from msda_triton_b200.fused import (msda2d_fused, msda3d_fused, sampling_prologue,
                                    sampling_prologue_applies)
from msda_triton_b200.msda_2d import msda2d
from msda_triton_b200.msda_3d import msda3d

# Samples (B*Q*H*L*P) per call from which the unfused composition is used
# (the size from which the library's backward takes the cell-sorted plan).
FUSED_MAX_SAMPLES = 1 << 20


# Projections over at least this many rows take _WideLinearFn.
WIDE_LINEAR_MIN_ROWS = 1 << 19


class _WideLinearFn(torch.autograd.Function):
    """nn.Linear over many rows.  The forward is F.linear; the backward takes
    the bias gradient as a product with a ones vector (one cuBLAS GEMM that
    reads the output gradient once at HBM speed) instead of torch's sum
    reduction, which runs at about a third of that and splits inputs above
    2^31 elements into several launches.  The input and weight gradients
    are the usual GEMMs."""

    @staticmethod
    def forward(ctx, x, weight, bias):
        ctx.save_for_backward(x, weight)
        return nn.functional.linear(x, weight, bias)

    @staticmethod
    def backward(ctx, grad):
        x, weight = ctx.saved_tensors
        g2 = grad.reshape(-1, grad.shape[-1])
        gx = gw = gb = None
        if ctx.needs_input_grad[0]:
            gx = grad @ weight
        if ctx.needs_input_grad[1]:
            gw = g2.t() @ x.reshape(-1, x.shape[-1])
        if ctx.needs_input_grad[2]:
            gb = (g2.new_ones((1, g2.shape[0])) @ g2).view(-1)
        return gx, gw, gb


def _project(linear: nn.Linear, x: torch.Tensor) -> torch.Tensor:
    """linear(x), through _WideLinearFn for large CUDA inputs in the
    parameters' dtype (no autocast, no hooks on the layer, not under
    torch.compile tracing)."""
    if (x.is_cuda and linear.bias is not None and x.dtype == linear.weight.dtype
            and x.numel() // max(x.shape[-1], 1) >= WIDE_LINEAR_MIN_ROWS
            and not torch.is_autocast_enabled("cuda") and not torch.compiler.is_compiling()
            and not linear._forward_hooks and not linear._forward_pre_hooks):
        return _WideLinearFn.apply(x, linear.weight, linear.bias)
    return linear(x)


class _MSDAModule(nn.Module):
    """Shared body of MSDA2D / MSDA3D; subclasses set NDIM, the sampling op
    and the init_weights offset pattern."""

    NDIM = 0

    def __init__(self, embed_dims: int, num_heads: int, num_levels: int, num_points: int,
                 dropout: float = 0.1, batch_first: bool = False,
                 query_chunk_size: int | None = None, head_chunk_size: int | None = None,
                 use_checkpoint: bool = False, clamp_grid: bool = True,
                 clamp_eps: float = 1e-4, fused_prologue: bool = True, **kwargs) -> None:
        super().__init__()
        if embed_dims % num_heads != 0:
            raise ValueError(f"embed_dims must be divisible by num_heads, but got {embed_dims} "
                             f"and {num_heads}")
        self.dropout = nn.Dropout(dropout)
        self.batch_first = batch_first
        self.embed_dims = embed_dims
        self.num_levels = num_levels
        self.num_heads = num_heads
        self.num_points = num_points
        self.query_chunk_size = query_chunk_size
        self.head_chunk_size = head_chunk_size
        self.use_checkpoint = use_checkpoint
        self.clamp_grid = clamp_grid
        self.clamp_eps = clamp_eps
        self.fused_prologue = fused_prologue
        samples = num_heads * num_levels * num_points
        # creation order fixes the default-init RNG draws (as in the reference)
        self.sampling_offsets = nn.Linear(embed_dims, samples * self.NDIM)
        self.attention_weights = nn.Linear(embed_dims, samples)
        self.value_proj = nn.Linear(embed_dims, embed_dims)
        self.output_proj = nn.Linear(embed_dims, embed_dims)

    # ------------------------------------------------------------- init
    def _offset_pattern(self, device) -> torch.Tensor:
        """(H, L, P, d) initial sampling offsets (the sampling_offsets bias)."""
        raise NotImplementedError

    def init_weights(self) -> None:
        """Zero offset/weight projections with a per-head offset pattern in the
        bias, Xavier-uniform value/output projections (reference:
        pytorch/msda_3d.py:191-235, pytorch/msda_2d.py:190-233)."""
        nn.init.constant_(self.sampling_offsets.weight, 0.0)
        device = self.sampling_offsets.weight.device
        with torch.no_grad():
            self.sampling_offsets.bias.copy_(self._offset_pattern(device).reshape(-1))
        nn.init.constant_(self.attention_weights.weight, 0.0)
        nn.init.constant_(self.attention_weights.bias, 0.0)
        nn.init.xavier_uniform_(self.value_proj.weight)
        nn.init.constant_(self.value_proj.bias, 0.0)
        nn.init.xavier_uniform_(self.output_proj.weight)
        nn.init.constant_(self.output_proj.bias, 0.0)
        self._is_init = True

    # ------------------------------------------------------------- forward
    def _sample(self, value, spatial_shapes, loc, weights):
        raise NotImplementedError

    def _sample_fused(self, value, spatial_shapes, ref, offsets, logits):
        raise NotImplementedError

    def forward(self, query: torch.Tensor, key: torch.Tensor | None = None,
                value: torch.Tensor | None = None, identity: torch.Tensor | None = None,
                query_pos: torch.Tensor | None = None,
                key_padding_mask: torch.Tensor | None = None,
                reference_points: torch.Tensor | None = None,
                spatial_shapes: torch.Tensor | None = None,
                level_start_index: torch.Tensor | None = None, **kwargs) -> torch.Tensor:
        """query (Q, B, E) or (B, Q, E) with batch_first; value likewise with the
        K = sum of level sizes keys (query if None); reference_points
        (B, Q, L, d) normalised; spatial_shapes (L, d) as (H, W) / (D, H, W).
        `key` and `level_start_index` are unused (API compatibility).
        Returns the query's shape."""
        d, H, L, P = self.NDIM, self.num_heads, self.num_levels, self.num_points
        value_in = query if value is None else value
        identity = query if identity is None else identity
        q = query if query_pos is None else query + query_pos
        if not self.batch_first:
            q = q.permute(1, 0, 2)
            value_in = value_in.permute(1, 0, 2)
        bs, num_query, _ = q.shape
        num_value = value_in.shape[1]
        assert spatial_shapes is not None, "spatial_shapes is required"
        assert reference_points is not None, "reference_points is required"
        # The size check below needs the shapes on the host (the reference
        # syncs here too); the kernels then get the host copy, which lets the
        # backward plan its per-level value-gradient targets.
        shapes_host = spatial_shapes.cpu() if spatial_shapes.is_cuda else spatial_shapes
        total = shapes_host[:, :d].prod(-1).sum()
        assert total == num_value, (
            f"Spatial shapes product {total} doesn't match value size {num_value}")

        v = _project(self.value_proj, value_in)
        if key_padding_mask is not None:
            v = v.masked_fill(key_padding_mask[..., None], 0.0)
        v = v.view(bs, num_value, H, -1)
        if reference_points.shape[-1] != d:
            raise ValueError(f"Last dim of reference_points must be {d}, "
                             f"but got {reference_points.shape[-1]} instead.")
        # (W, H[, D]) per level: the last coordinate axis is x (W-indexed)
        normalizer = spatial_shapes.flip(-1).to(q.device)[None, None, None, :, None, :]

        qc = int(self.query_chunk_size) if self.query_chunk_size else num_query
        hc = (int(self.head_chunk_size)
              if self.head_chunk_size and self.head_chunk_size < H else H)
        c = self.embed_dims // H
        chunks = []
        for q0 in range(0, num_query, qc):
            q1 = min(q0 + qc, num_query)
            qq = q[:, q0:q1]
            offsets = _project(self.sampling_offsets, qq).view(bs, q1 - q0, H, L, P, d)
            logits = _project(self.attention_weights, qq).view(bs, q1 - q0, H, L, P)
            if self.fused_prologue and bs * (q1 - q0) * hc * L * P < FUSED_MAX_SAMPLES:
                # (loc, weights) formed per sample inside the kernels
                ref = reference_points[:, q0:q1]
                run = lambda h0, h1: self._run(self._sample_fused, v[:, :, h0:h1], shapes_host,
                                               ref, offsets[:, :, h0:h1], logits[:, :, h0:h1])
            else:
                ref = reference_points[:, q0:q1]
                if self.fused_prologue and sampling_prologue_applies(ref, offsets, logits):
                    # the locations and weights in two passes of their own
                    # (msda_prologue_fwd / _bwd) instead of the tensor ops
                    loc, weights = sampling_prologue(d, shapes_host[:, :d], ref, offsets, logits)
                else:
                    weights = logits.view(bs, q1 - q0, H, L * P).softmax(-1)
                    weights = weights.view(bs, q1 - q0, H, L, P)
                    loc = ref[:, :, None, :, None, :] + offsets / normalizer
                run = lambda h0, h1: self._run(self._sample, v[:, :, h0:h1], shapes_host,
                                               loc[:, :, h0:h1], weights[:, :, h0:h1])
            if hc == H:
                chunks.append(run(0, H))
                continue
            out = q.new_zeros(bs, q1 - q0, self.embed_dims)
            for h0 in range(0, H, hc):
                h1 = min(h0 + hc, H)
                out[:, :, h0 * c:h1 * c] = run(h0, h1)
            chunks.append(out)
        out = chunks[0] if len(chunks) == 1 else torch.cat(chunks, dim=1)
        out = _project(self.output_proj, out)
        if not self.batch_first:
            out = out.permute(1, 0, 2)
        return self.dropout(out) + identity

    def _run(self, fn, *args):
        if self.use_checkpoint and self.training:
            return checkpoint(fn, *args, use_reentrant=False)
        return fn(*args)


class MSDA3D(_MSDAModule):
    """3D multi-scale deformable attention module (trilinear sampling in the
    sm_100a kernels).  Reference: pytorch/msda_3d.py:121-394."""

    NDIM = 3

    def _offset_pattern(self, device) -> torch.Tensor:
        # head h, point p: angle 2*pi*(h*P + p)/(H*P), radius 0.02*(p+1);
        # (x, y, z) = (r/2 cos a, r/2 sin a, 2r sin 2a), the same on every level
        # (reference: pytorch/msda_3d.py:203-218), evaluated in double.
        H, L, P = self.num_heads, self.num_levels, self.num_points
        idx = torch.arange(H * P, dtype=torch.float64).view(H, P)
        angle = 2.0 * math.pi * idx / (H * P)
        radius = 0.02 * (torch.arange(P, dtype=torch.float64) + 1.0)
        xyz = torch.stack([radius * 0.5 * angle.cos(), radius * 0.5 * angle.sin(),
                           radius * 2.0 * (angle * 2).sin()], -1)          # (H, P, 3)
        return xyz[:, None].expand(H, L, P, 3).to(device=device, dtype=torch.float32)

    def _sample(self, v, spatial_shapes, loc, weights):
        return msda3d(v, spatial_shapes, loc, weights, self.clamp_grid, self.clamp_eps)

    def _sample_fused(self, v, spatial_shapes, ref, offsets, logits):
        return msda3d_fused(v, spatial_shapes, ref, offsets, logits, self.clamp_grid,
                            self.clamp_eps)


class MSDA2D(_MSDAModule):
    """2D multi-scale deformable attention module (bilinear sampling in the
    sm_100a kernels).  Reference: pytorch/msda_2d.py:117-383."""

    NDIM = 2

    def _offset_pattern(self, device) -> torch.Tensor:
        # Deformable-DETR pattern: head h points along angle 2*pi*h/H, scaled so
        # the larger of |cos|, |sin| is 1, times (p+1) for point p, the same on
        # every level (reference: pytorch/msda_2d.py:199-213), in float32.
        H, L, P = self.num_heads, self.num_levels, self.num_points
        theta = torch.arange(H, dtype=torch.float32, device=device) * (2.0 * math.pi / H)
        dirs = torch.stack([theta.cos(), theta.sin()], -1)
        dirs = dirs / dirs.abs().max(-1, keepdim=True)[0]
        scale = torch.arange(1, P + 1, dtype=torch.float32, device=device)
        return (dirs[:, None, None, :] * scale[None, None, :, None]).expand(H, L, P, 2)

    def _sample(self, v, spatial_shapes, loc, weights):
        return msda2d(v, spatial_shapes, loc, weights, self.clamp_grid, self.clamp_eps)

    def _sample_fused(self, v, spatial_shapes, ref, offsets, logits):
        return msda2d_fused(v, spatial_shapes, ref, offsets, logits, self.clamp_grid,
                            self.clamp_eps)


__all__ = ["MSDA2D", "MSDA3D"]
