"""MSDA with the deformable-attention prologue inside the kernels.

A deformable-attention layer (the reference's MSDA2D / MSDA3D modules,
src/msda_triton/pytorch/msda_2d.py:325-339, src/msda_triton/pytorch/msda_3d.py:325-350)
turns two query projections into the kernel's inputs with separate tensor
ops:

    loc     = reference_points[:, :, None, :, None, :] + offsets / (W, H[, D])_l
    weights = softmax(logits over the L*P samples of each (b, q, h))

msda2d_fused / msda3d_fused take reference_points, the raw offsets and the raw
logits instead; the kernels form the locations and weights per sample in
registers (fp32), so neither tensor is written or read from HBM, and the
backward produces the offset, logit and reference-point gradients directly
(the logit gradient is the softmax backward w * (dL/dw - sum w * dL/dw), the
reference-point gradient the location gradient summed over heads and
points).  Results equal msda{2,3}d on the separately computed loc / weights
up to the softmax's summation order (fp32).
"""

from __future__ import annotations

import torch

from msda_triton_b200 import _core, _lib


def _prepare(ndim, value, spatial_shapes, reference_points, offsets, logits):
    if logits.dim() == 4 and offsets.dim() == 6:
        logits = logits.reshape(*offsets.shape[:5])
    _core.validate_inputs(ndim, value, spatial_shapes, offsets, logits)
    B, Q, H, L, P, _ = offsets.shape
    if tuple(reference_points.shape) != (B, Q, L, ndim):
        raise ValueError(f"reference_points must be (B, Q, L, {ndim}) = {(B, Q, L, ndim)}, "
                         f"got {tuple(reference_points.shape)}")
    if not reference_points.is_cuda or reference_points.device != value.device:
        raise ValueError(f"reference_points must be a CUDA tensor on {value.device}, "
                         f"got {reference_points.device}")
    if not reference_points.dtype.is_floating_point:
        raise ValueError(f"reference_points must be floating point, got {reference_points.dtype}")
    shapes, on_dev = _core.prepare_spatial(spatial_shapes)
    off, lg = _core.sampling_pair(value, offsets, logits)
    ref = reference_points.detach().to(torch.float32).contiguous()
    return shapes, on_dev, ref, off, lg


def _args(value, shapes, on_dev, ref, off, lg):
    B, K, H, C = value.shape
    _, Q, _, L, P, _ = off.shape
    return (value.data_ptr(), _core.value_code(value), B, K, H, C,
            shapes.data_ptr(), int(on_dev), L, ref.data_ptr(), off.data_ptr(), lg.data_ptr(),
            _core._DTYPE_CODE[off.dtype], Q, P)


class MSDAFusedFn(torch.autograd.Function):
    """Autograd Function of msda{2,3}d_fused; gradients flow to value,
    reference_points, sampling_offsets and attention_logits."""

    @staticmethod
    def forward(ctx, ndim, value, spatial_shapes, reference_points, sampling_offsets,
                attention_logits, clamp_grid=True, clamp_eps=1e-4):
        shapes, on_dev, ref, off, lg = _prepare(ndim, value, spatial_shapes, reference_points,
                                                sampling_offsets, attention_logits)
        value_c = _core.prepare_value(value)
        B, _, H, C = value_c.shape
        out = torch.empty((B, off.shape[1], H * C), device=value.device, dtype=value.dtype)
        fn = _lib.lib().msda2d_fused_fwd if ndim == 2 else _lib.lib().msda3d_fused_fwd
        with torch.cuda.device(value.device):
            code = fn(*_args(value_c, shapes, on_dev, ref, off, lg), int(bool(clamp_grid)),
                      float(clamp_eps), out.data_ptr(), _core._stream_ptr(value.device))
        _core.check_status(code)
        ctx.save_for_backward(value_c, shapes, ref, off, lg)
        ctx.meta = (ndim, on_dev, bool(clamp_grid), float(clamp_eps), reference_points.dtype,
                    sampling_offsets.dtype, attention_logits.dtype, attention_logits.shape)
        return out

    @staticmethod
    def backward(ctx, grad_output):
        value, shapes, ref, off, lg = ctx.saved_tensors
        ndim, on_dev, clamp, eps, ref_dt, off_dt, lg_dt, lg_shape = ctx.meta
        g_value, g_ref, g_off, g_lg = _backward(ndim, grad_output, value, shapes, on_dev, ref,
                                                off, lg, clamp, eps)
        return (None, g_value, None, g_ref.to(ref_dt), g_off.to(off_dt),
                g_lg.to(lg_dt).reshape(lg_shape), None, None)


def _backward(ndim, grad_output, value, shapes, on_dev, ref, off, lg, clamp, eps):
    """Launch the fused backward on prepared tensors; returns (grad_value,
    grad_reference_points fp32, grad_offsets, grad_logits (B,Q,H,L,P))."""
    go = grad_output.to(value.dtype).contiguous()
    B, K, H, C = value.shape
    _, Q, _, L, P, _ = off.shape
    lib = _lib.lib()
    ws_bytes = lib.msda_fused_bwd_workspace_bytes(ndim, _core.value_code(value), B, K,
                                                  H, C, shapes.data_ptr(), int(on_dev), L, Q,
                                                  P)
    ws = torch.empty((ws_bytes,), device=value.device, dtype=torch.uint8) if ws_bytes else None
    g_value = torch.empty_like(value)
    g_off = torch.empty_like(off)
    g_lg = torch.empty_like(lg)
    partial = torch.empty((B, Q, H, L, ndim), device=value.device, dtype=torch.float32)
    fn = lib.msda2d_fused_bwd if ndim == 2 else lib.msda3d_fused_bwd
    with torch.cuda.device(value.device):
        code = fn(*_args(value, shapes, on_dev, ref, off, lg), int(clamp), eps,
                  go.data_ptr(), g_value.data_ptr(), partial.data_ptr(), g_off.data_ptr(),
                  g_lg.data_ptr(), ws.data_ptr() if ws is not None else None, ws_bytes,
                  _core._stream_ptr(value.device))
    _core.check_status(code)
    return g_value, partial.sum(dim=2), g_off, g_lg


def fused_backward(ndim, grad_output, value, spatial_shapes, reference_points, sampling_offsets,
                   attention_logits, clamp_grid, clamp_eps):
    """The backward of msda{2,3}d_fused as a function of its inputs (the
    torch.library op's implementation): gradients in the inputs' dtypes and
    shapes."""
    shapes, on_dev, ref, off, lg = _prepare(ndim, value, spatial_shapes, reference_points,
                                            sampling_offsets, attention_logits)
    g_value, g_ref, g_off, g_lg = _backward(ndim, grad_output, value.contiguous(), shapes, on_dev,
                                            ref, off, lg, bool(clamp_grid), float(clamp_eps))
    return (g_value, g_ref.to(reference_points.dtype), g_off.to(sampling_offsets.dtype),
            g_lg.to(attention_logits.dtype).reshape(attention_logits.shape))


def _fused(ndim, value, value_spatial_shapes, reference_points, sampling_offsets,
           attention_logits, clamp_grid, clamp_eps):
    if not value.is_cuda:
        raise ValueError(f"MSDA{ndim}D CUDA kernel requires CUDA tensors. Got CPU tensors instead.")
    if torch.compiler.is_compiling():
        from msda_triton_b200 import ops

        # traced as one opaque op (msda_b200::msda_fused_forward), no graph break
        return ops.msda_fused_forward(value, value_spatial_shapes, reference_points,
                                      sampling_offsets, attention_logits, ndim, clamp_grid,
                                      clamp_eps)
    return MSDAFusedFn.apply(ndim, value, value_spatial_shapes, reference_points,
                             sampling_offsets, attention_logits, clamp_grid, clamp_eps)


def msda2d_fused(value: torch.Tensor, value_spatial_shapes: torch.Tensor,
                 reference_points: torch.Tensor, sampling_offsets: torch.Tensor,
                 attention_logits: torch.Tensor, clamp_grid: bool = True,
                 clamp_eps: float = 1e-4) -> torch.Tensor:
    """2D MSDA from the layer's raw projections.

    value (B, K, H, C); value_spatial_shapes (L, 2) as (H, W); reference_points
    (B, Q, L, 2) normalised (x, y); sampling_offsets (B, Q, H, L, P, 2) in cells
    of each level; attention_logits (B, Q, H, L, P) or (B, Q, H, L*P).
    Returns (B, Q, H*C) in value's dtype, with autograd."""
    return _fused(2, value, value_spatial_shapes, reference_points, sampling_offsets,
                  attention_logits, clamp_grid, clamp_eps)


def msda3d_fused(value: torch.Tensor, value_spatial_shapes: torch.Tensor,
                 reference_points: torch.Tensor, sampling_offsets: torch.Tensor,
                 attention_logits: torch.Tensor, clamp_grid: bool = True,
                 clamp_eps: float = 1e-4) -> torch.Tensor:
    """3D MSDA from the layer's raw projections (as msda2d_fused, with
    (L, 3) shapes (D, H, W), (x, y, z) reference points and offsets)."""
    return _fused(3, value, value_spatial_shapes, reference_points, sampling_offsets,
                  attention_logits, clamp_grid, clamp_eps)


class SamplingPrologueFn(torch.autograd.Function):
    """The prologue alone (msda_prologue_fwd / msda_prologue_bwd): locations
    and softmax weights as tensors, for calls that then run msda{2,3}d (the
    large-problem path of the modules, whose cell-sorted backward has no
    fused form).  Two passes replace the module's separate tensor ops and
    their backward: the locations round as `reference_points + offsets /
    normalizer` does in the sampling dtype; the weights are the fused
    kernels' row softmax."""

    @staticmethod
    def forward(ctx, ndim, shapes_host, reference_points, sampling_offsets, attention_logits):
        off = sampling_offsets.contiguous()
        ref = reference_points.contiguous()
        lg = attention_logits.contiguous()
        B, Q, H, L, P, _ = off.shape
        loc = torch.empty_like(off)
        w = torch.empty((B, Q, H, L, P), dtype=off.dtype, device=off.device)
        _core.check_status(_lib.lib().msda_prologue_fwd(
            ndim, B, Q, H, L, P, shapes_host.data_ptr(), ref.data_ptr(), off.data_ptr(),
            lg.data_ptr(), _core._DTYPE_CODE[off.dtype], loc.data_ptr(), w.data_ptr(),
            _core._stream_ptr(off.device)))
        ctx.save_for_backward(w)
        ctx.ndim, ctx.shapes_host = ndim, shapes_host
        ctx.logits_shape = attention_logits.shape
        return loc, w

    @staticmethod
    def backward(ctx, grad_loc, grad_w):
        (w,) = ctx.saved_tensors
        ndim = ctx.ndim
        B, Q, H, L, P = w.shape
        gl = (torch.zeros((B, Q, H, L, P, ndim), dtype=w.dtype, device=w.device)
              if grad_loc is None else grad_loc.to(w.dtype).contiguous())
        gw = torch.zeros_like(w) if grad_w is None else grad_w.to(w.dtype).contiguous()
        goff = torch.empty_like(gl)
        glg = torch.empty_like(w)
        gref_p = torch.empty((B, Q, H, L, ndim), dtype=torch.float32, device=w.device)
        _core.check_status(_lib.lib().msda_prologue_bwd(
            ndim, B, Q, H, L, P, ctx.shapes_host.data_ptr(), w.data_ptr(), gl.data_ptr(),
            gw.data_ptr(), _core._DTYPE_CODE[w.dtype], gref_p.data_ptr(), goff.data_ptr(),
            glg.data_ptr(), _core._stream_ptr(w.device)))
        gref = gref_p.sum(2).to(w.dtype)
        return None, None, gref, goff, glg.view(ctx.logits_shape)


# msda_prologue_{fwd,bwd} take rows of at most this many samples (L*P).
PROLOGUE_MAX_SAMPLES = 2048


def sampling_prologue_applies(reference_points: torch.Tensor, sampling_offsets: torch.Tensor,
                              attention_logits: torch.Tensor) -> bool:
    """Whether SamplingPrologueFn takes these tensors: CUDA, at most
    PROLOGUE_MAX_SAMPLES samples per (b, q, h) row, one of the kernels'
    dtypes for all three, and not under torch.compile tracing (which keeps
    the traceable tensor ops)."""
    dt = sampling_offsets.dtype
    return (sampling_offsets.is_cuda and sampling_offsets.dim() == 6
            and sampling_offsets.shape[3] * sampling_offsets.shape[4] <= PROLOGUE_MAX_SAMPLES
            and reference_points.dtype == dt
            and attention_logits.dtype == dt and dt in _core._DTYPE_CODE
            and reference_points.device == sampling_offsets.device
            and not torch.compiler.is_compiling())


def sampling_prologue(ndim: int, spatial_shapes_host: torch.Tensor,
                      reference_points: torch.Tensor, sampling_offsets: torch.Tensor,
                      attention_logits: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """(sampling_locations, attention_weights) from reference points (B, Q, L,
    d), raw offsets (B, Q, H, L, P, d) and raw logits (B, Q, H, L, P) or (B,
    Q, H, L*P), with autograd; spatial_shapes_host (L, d) on the CPU."""
    shp = spatial_shapes_host.detach().to(torch.int32).contiguous()
    return SamplingPrologueFn.apply(ndim, shp, reference_points, sampling_offsets,
                                    attention_logits)


__all__ = ["msda2d_fused", "msda3d_fused", "MSDAFusedFn", "SamplingPrologueFn",
           "sampling_prologue", "sampling_prologue_applies"]
