"""Dimension-generic host side of the MSDA ops: validation, spatial-shape
preparation, launches through the C ABI, and the autograd Function.

Mirrors the reference's wrappers (src/msda_triton/triton/msda_2d.py:541-907 and
src/msda_triton/triton/msda_3d.py:684-1050): same argument names, same
exception types and messages for the cases the reference checks.  The kernels
run on the current torch CUDA stream of value's device.
"""

from __future__ import annotations

import torch

from msda_triton_b200 import _lib

_DTYPE_CODE = {
    torch.float32: _lib.FLOAT32,
    torch.float16: _lib.FLOAT16,
    torch.bfloat16: _lib.BFLOAT16,
}

_VALUE_ERRORS = {
    _lib.ERROR_INVALID_ARGUMENT,
    _lib.ERROR_SHAPE_MISMATCH,
    _lib.ERROR_TOO_MANY_LEVELS,
    _lib.ERROR_INT32_OVERFLOW,
    _lib.ERROR_MISALIGNED,
    _lib.ERROR_WORKSPACE,
    _lib.ERROR_UNSUPPORTED_CHANNELS,
}


def _name(ndim: int) -> str:
    return f"MSDA{ndim}D"


def check_status(code: int) -> None:
    """Raise the reference's exception type for a non-zero C-ABI status."""
    if code == _lib.SUCCESS:
        return
    msg = _lib.last_error() or _lib.status_string(code)
    if code == _lib.ERROR_UNSUPPORTED_DTYPE:
        raise NotImplementedError(msg)
    if code in _VALUE_ERRORS:
        raise ValueError(msg)
    raise RuntimeError(f"{_lib.status_string(code)}: {msg}")


def validate_inputs(
    ndim: int,
    value: torch.Tensor,
    value_spatial_shapes: torch.Tensor,
    sampling_locations: torch.Tensor,
    attention_weights: torch.Tensor,
) -> None:
    """Device, dtype and shape checks (reference: triton/msda_2d.py:541-583,
    triton/msda_3d.py:684-726).  Raises on the first violation."""
    name = _name(ndim)
    if not value.is_cuda:
        raise ValueError(f"{name} CUDA kernel requires CUDA tensors. Got CPU tensors instead.")
    if value.dtype not in _DTYPE_CODE:
        raise NotImplementedError(
            f"{name} CUDA kernel only supports fp32, fp16, and bf16. Got {value.dtype}. "
            "The kernel accumulates in fp32 internally."
        )
    if value.dim() != 4:
        raise ValueError(f"value must be (B, K, H, C), got {tuple(value.shape)}")
    if sampling_locations.dim() != 6:
        raise ValueError(
            f"sampling_locations must be (B, Q, H, L, P, {ndim}), "
            f"got {tuple(sampling_locations.shape)}"
        )
    bsz, _, num_heads, _ = value.shape
    bsz_s, num_queries, num_heads_s, num_levels, num_points, last = sampling_locations.shape
    if not (bsz == bsz_s and num_heads == num_heads_s and last == ndim):
        raise ValueError(
            f"Shape mismatch: value=(B,K,H,C), sampling_locations=(B,Q,H,L,P,{ndim}). "
            f"Got value={tuple(value.shape)}, sampling_locations={tuple(sampling_locations.shape)}"
        )
    if attention_weights.shape != (bsz, num_queries, num_heads, num_levels, num_points):
        raise ValueError(
            f"attention_weights must be (B,Q,H,L,P), got {tuple(attention_weights.shape)}"
        )
    if value_spatial_shapes.shape != (num_levels, ndim):
        raise ValueError(
            f"value_spatial_shapes must be (L,{ndim}), got {tuple(value_spatial_shapes.shape)}. "
            f"num_levels={num_levels}, expected shape=({num_levels}, {ndim})"
        )
    for t, what in ((sampling_locations, "sampling_locations"), (attention_weights, "attention_weights")):
        if not t.is_cuda or t.device != value.device:
            raise ValueError(f"{what} must be a CUDA tensor on {value.device}, got {t.device}")
        if t.dtype not in _DTYPE_CODE:
            raise NotImplementedError(
                f"{name} CUDA kernel only supports fp32, fp16, and bf16. Got {t.dtype} "
                f"for {what}."
            )
    if value_spatial_shapes.is_cuda and value_spatial_shapes.device != value.device:
        raise ValueError(
            f"value_spatial_shapes must be on the CPU or on {value.device}, "
            f"got {value_spatial_shapes.device}"
        )
    if value_spatial_shapes.dtype.is_floating_point or value_spatial_shapes.dtype == torch.bool:
        raise ValueError(f"value_spatial_shapes must be an integer tensor, got {value_spatial_shapes.dtype}")


def prepare_spatial(value_spatial_shapes: torch.Tensor) -> tuple[torch.Tensor, bool]:
    """int32 contiguous copy of the level shapes, kept where it lives.

    CPU shapes let the library check K against the level sizes for free;
    device shapes are converted on the device and read by the kernels without
    a host synchronisation (reference: triton/msda_2d.py:17-82)."""
    shp = value_spatial_shapes.detach()
    if shp.dtype != torch.int32:
        shp = shp.to(torch.int32)
    return shp.contiguous(), bool(shp.is_cuda)


def sampling_pair(
    value: torch.Tensor, sampling_locations: torch.Tensor, attention_weights: torch.Tensor
) -> tuple[torch.Tensor, torch.Tensor]:
    """Locations and weights in one dtype the kernels take: the value dtype or
    fp32.  Mixed pairs are upcast to fp32 (lossless)."""
    loc, attn = sampling_locations, attention_weights
    if not (loc.dtype == attn.dtype and loc.dtype in (value.dtype, torch.float32)):
        loc, attn = loc.float(), attn.float()
    return loc.contiguous(), attn.contiguous()


def is_head_major(value: torch.Tensor) -> bool:
    """value (B, K, H, C) as a view of a contiguous (B, H, K, C) tensor: each
    head's keys contiguous (what `prepare_value` passes through uncopied)."""
    return (value.dim() == 4 and not value.is_contiguous()
            and value.permute(0, 2, 1, 3).is_contiguous())


def prepare_value(value: torch.Tensor) -> torch.Tensor:
    """value in a layout the kernels read in place: the reference's dense
    (B, K, H, C), or the head-major view of a dense (B, H, K, C) tensor.
    Any other strides are copied to (B, K, H, C)."""
    if value.is_contiguous() or is_head_major(value):
        return value
    return value.contiguous()


def value_code(value: torch.Tensor) -> int:
    """The C ABI's value dtype argument: dtype code, plus the head-major flag."""
    code = _DTYPE_CODE[value.dtype]
    return code | _lib.VALUE_HEAD_MAJOR if is_head_major(value) else code


def _stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _common_args(value, shapes, on_dev, loc, attn):
    B, K, H, C = value.shape
    _, Q, _, L, P, _ = loc.shape
    return (
        value.data_ptr(), value_code(value), B, K, H, C,
        shapes.data_ptr(), int(on_dev), L,
        loc.data_ptr(), attn.data_ptr(), _DTYPE_CODE[loc.dtype], Q, P,
    )


def forward(
    ndim: int,
    value: torch.Tensor,
    shapes: torch.Tensor,
    on_dev: bool,
    loc: torch.Tensor,
    attn: torch.Tensor,
    clamp_grid: bool,
    clamp_eps: float,
) -> torch.Tensor:
    """Launch the forward kernel; inputs already validated and prepared."""
    B, _, H, C = value.shape
    Q = loc.shape[1]
    out = torch.empty((B, Q, H * C), device=value.device, dtype=value.dtype)
    fn = _lib.lib().msda2d_fwd if ndim == 2 else _lib.lib().msda3d_fwd
    with torch.cuda.device(value.device):
        code = fn(
            *_common_args(value, shapes, on_dev, loc, attn),
            int(bool(clamp_grid)), float(clamp_eps),
            out.data_ptr(), _stream_ptr(value.device),
        )
    check_status(code)
    return out


def backward(
    ndim: int,
    value: torch.Tensor,
    shapes: torch.Tensor,
    on_dev: bool,
    loc: torch.Tensor,
    attn: torch.Tensor,
    clamp_grid: bool,
    clamp_eps: float,
    grad_output: torch.Tensor,
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Launch the backward kernel; returns (grad_value, grad_loc, grad_attn)
    in the dtypes of value and of the (prepared) locations."""
    B, K, H, C = value.shape
    go = grad_output
    if go.dtype != value.dtype:
        go = go.to(value.dtype)
    go = go.contiguous()
    grad_value = torch.empty_like(value)
    grad_loc = torch.empty_like(loc)
    grad_attn = torch.empty_like(attn)
    lib = _lib.lib()
    Q, L, P = loc.shape[1], loc.shape[3], loc.shape[4]
    ws_bytes = lib.msda_bwd_workspace_bytes(ndim, value_code(value), B, K, H, C,
                                            shapes.data_ptr(), int(on_dev), L, Q, P)
    ws = torch.empty((ws_bytes,), device=value.device, dtype=torch.uint8) if ws_bytes else None
    fn = lib.msda2d_bwd if ndim == 2 else lib.msda3d_bwd
    with torch.cuda.device(value.device):
        code = fn(
            *_common_args(value, shapes, on_dev, loc, attn),
            int(bool(clamp_grid)), float(clamp_eps),
            go.data_ptr(), grad_value.data_ptr(), grad_loc.data_ptr(), grad_attn.data_ptr(),
            ws.data_ptr() if ws is not None else None, ws_bytes,
            _stream_ptr(value.device),
        )
    check_status(code)
    return grad_value, grad_loc, grad_attn


def backward_accumulate(
    ndim: int,
    value: torch.Tensor,
    shapes: torch.Tensor,
    on_dev: bool,
    loc: torch.Tensor,
    attn: torch.Tensor,
    clamp_grid: bool,
    clamp_eps: float,
    grad_output: torch.Tensor,
    grad_value_accum: torch.Tensor,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Backward scatter only: ADDS the value gradient (fp32) into
    grad_value_accum and returns (grad_loc, grad_attn).  Used where partial
    value gradients are summed before one final cast (query sharding)."""
    if grad_value_accum.dtype != torch.float32 or grad_value_accum.shape != value.shape:
        raise ValueError("grad_value_accum must be an fp32 tensor shaped like value")
    if grad_value_accum.stride() != value.stride():
        raise ValueError("grad_value_accum must have value's layout")
    go = grad_output
    if go.dtype != value.dtype:
        go = go.to(value.dtype)
    go = go.contiguous()
    grad_loc = torch.empty_like(loc)
    grad_attn = torch.empty_like(attn)
    lib = _lib.lib()
    fn = lib.msda2d_bwd_accumulate if ndim == 2 else lib.msda3d_bwd_accumulate
    with torch.cuda.device(value.device):
        code = fn(
            *_common_args(value, shapes, on_dev, loc, attn),
            int(bool(clamp_grid)), float(clamp_eps),
            go.data_ptr(), grad_value_accum.data_ptr(), grad_loc.data_ptr(), grad_attn.data_ptr(),
            _stream_ptr(value.device),
        )
    check_status(code)
    return grad_loc, grad_attn


def cast_from_f32(src: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """Round an fp32 tensor to `dtype` with the library's cast kernel."""
    if dtype == torch.float32:
        return src
    src = src.contiguous()
    dst = torch.empty(src.shape, device=src.device, dtype=dtype)
    with torch.cuda.device(src.device):
        code = _lib.lib().msda_cast_from_f32(src.data_ptr(), dst.data_ptr(), _DTYPE_CODE[dtype],
                                             src.numel(), _stream_ptr(src.device))
    check_status(code)
    return dst


def fwd_entry(ndim, value, value_spatial_shapes, sampling_locations, attention_weights,
              clamp_grid, clamp_eps) -> torch.Tensor:
    validate_inputs(ndim, value, value_spatial_shapes, sampling_locations, attention_weights)
    shapes, on_dev = prepare_spatial(value_spatial_shapes)
    loc, attn = sampling_pair(value, sampling_locations, attention_weights)
    return forward(ndim, prepare_value(value), shapes, on_dev, loc, attn, clamp_grid, clamp_eps)


def fn_forward(ndim, ctx, value, value_spatial_shapes, sampling_locations, attention_weights,
               clamp_grid, clamp_eps) -> torch.Tensor:
    """Body of MSDA{2,3}DFn.forward (reference: triton/msda_2d.py:749-775)."""
    validate_inputs(ndim, value, value_spatial_shapes, sampling_locations, attention_weights)
    shapes, on_dev = prepare_spatial(value_spatial_shapes)
    loc, attn = sampling_pair(value, sampling_locations, attention_weights)
    value_c = prepare_value(value)
    out = forward(ndim, value_c, shapes, on_dev, loc, attn, clamp_grid, clamp_eps)
    ctx.save_for_backward(value_c, loc, attn, shapes)
    ctx.on_dev = on_dev
    ctx.clamp_grid = clamp_grid
    ctx.clamp_eps = clamp_eps
    ctx.loc_dtype = sampling_locations.dtype
    ctx.attn_dtype = attention_weights.dtype
    return out


def fn_backward(ndim, ctx, grad_output):
    """Body of MSDA{2,3}DFn.backward (reference: triton/msda_2d.py:777-853).

    Returns (grad_value, None, grad_sampling_locations, grad_attention_weights,
    None, None): spatial shapes and the clamp arguments get no gradient."""
    value, loc, attn, shapes = ctx.saved_tensors
    grad_value, grad_loc, grad_attn = backward(
        ndim, value, shapes, ctx.on_dev, loc, attn, ctx.clamp_grid, ctx.clamp_eps, grad_output,
    )
    if grad_loc.dtype != ctx.loc_dtype:
        grad_loc = grad_loc.to(ctx.loc_dtype)
    if grad_attn.dtype != ctx.attn_dtype:
        grad_attn = grad_attn.to(ctx.attn_dtype)
    return grad_value, None, grad_loc, grad_attn, None, None
