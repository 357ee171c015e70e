"""ctypes binding of libmsda_b200.so (include/msda_b200.h).

The library is built in-tree by `python -m msda_triton_b200.build` (or
__graft_entry__.build()).  There is no fallback: if the library is missing
or fails to load, every op raises RuntimeError.  MSDA_B200_LIB=<path>
selects another build of the same ABI (e.g. the bounds-checked one).
"""

from __future__ import annotations

import ctypes
import os
import threading

LIB_PATH = os.environ.get("MSDA_B200_LIB") or os.path.join(
    os.path.dirname(os.path.abspath(__file__)), "_lib", "libmsda_b200.so")

# Status codes (msda_status in include/msda_b200.h).
SUCCESS = 0
ERROR_INVALID_ARGUMENT = 1
ERROR_UNSUPPORTED_DTYPE = 2
ERROR_SHAPE_MISMATCH = 3
ERROR_TOO_MANY_LEVELS = 4
ERROR_INT32_OVERFLOW = 5
ERROR_MISALIGNED = 6
ERROR_WORKSPACE = 7
ERROR_UNSUPPORTED_CHANNELS = 8
ERROR_CUDA = 9

# Dtype codes (msda_dtype).
FLOAT32 = 0
FLOAT16 = 1
BFLOAT16 = 2
# ORed into a value dtype code: value / grad_value laid out (B, H, K, C)
VALUE_HEAD_MAJOR = 0x100

MAX_LEVELS = 16
ABI_VERSION = 3

EXPORTED_SYMBOLS = (
    "msda2d_fwd",
    "msda3d_fwd",
    "msda2d_bwd",
    "msda3d_bwd",
    "msda2d_bwd_accumulate",
    "msda3d_bwd_accumulate",
    "msda_cast_from_f32",
    "msda_bwd_static_scratch",
    "msda_bwd_workspace_bytes",
    "msda2d_fused_fwd",
    "msda3d_fused_fwd",
    "msda2d_fused_bwd",
    "msda3d_fused_bwd",
    "msda_fused_bwd_workspace_bytes",
    "msda_prologue_fwd",
    "msda_prologue_bwd",
    "msda_status_string",
    "msda_last_error",
    "msda_abi_version",
)

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None

_i64 = ctypes.c_int64
_int = ctypes.c_int
_vp = ctypes.c_void_p

_FWD_ARGS = [
    _vp, _int, _i64, _i64, _i64, _i64,  # value, value_dtype, B, K, H, C
    _vp, _int, _i64,                    # spatial_shapes, on_device, L
    _vp, _vp, _int, _i64, _i64,         # loc, attn, sampling_dtype, Q, P
    _int, ctypes.c_double,              # clamp_grid, clamp_eps
    _vp, _vp,                           # output, stream
]
_BWD_ARGS = _FWD_ARGS[:-2] + [
    _vp, _vp, _vp, _vp,                 # grad_output, grad_value, grad_loc, grad_attn
    _vp, ctypes.c_size_t, _vp,          # workspace, workspace_bytes, stream
]

_FUSED_FWD_ARGS = [
    _vp, _int, _i64, _i64, _i64, _i64,  # value, value_dtype, B, K, H, C
    _vp, _int, _i64,                    # spatial_shapes, on_device, L
    _vp, _vp, _vp, _int, _i64, _i64,    # reference_points (fp32), offsets, logits, sampling_dtype, Q, P
    _int, ctypes.c_double,              # clamp_grid, clamp_eps
    _vp, _vp,                           # output, stream
]
_FUSED_BWD_ARGS = _FUSED_FWD_ARGS[:-2] + [
    _vp, _vp, _vp, _vp, _vp,            # grad_output, grad_value, grad_reference_partial (fp32),
                                        # grad_sampling_offsets, grad_attention_logits
    _vp, ctypes.c_size_t, _vp,          # workspace, workspace_bytes, stream
]

_PROLOGUE_FWD_ARGS = [
    _int, _i64, _i64, _i64, _i64, _i64,  # ndim, B, Q, H, L, P
    _vp,                                 # spatial_shapes (host int32)
    _vp, _vp, _vp, _int,                 # reference_points, offsets, logits, sampling_dtype
    _vp, _vp, _vp,                       # sampling_locations, attention_weights, stream
]
_PROLOGUE_BWD_ARGS = [
    _int, _i64, _i64, _i64, _i64, _i64,  # ndim, B, Q, H, L, P
    _vp,                                 # spatial_shapes (host int32)
    _vp, _vp, _vp, _int,                 # attention_weights, grad_loc, grad_attn, sampling_dtype
    _vp, _vp, _vp, _vp,                  # grad_reference_partial (fp32), grad_offsets,
                                         # grad_logits, stream
]

_ACC_ARGS = _FWD_ARGS[:-2] + [
    _vp, _vp, _vp, _vp,                 # grad_output, grad_value_accum (fp32), grad_loc, grad_attn
    _vp,                                # stream
]


def lib() -> ctypes.CDLL:
    """Load (once) and return the library, with argument types declared."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"msda_triton_b200: CUDA library not found at {LIB_PATH}; build it with "
                    "`python -m msda_triton_b200.build` (there is no CPU fallback)"
                )
            handle = ctypes.CDLL(LIB_PATH)
            for name in ("msda2d_fwd", "msda3d_fwd"):
                fn = getattr(handle, name)
                fn.argtypes = _FWD_ARGS
                fn.restype = _int
            for name in ("msda2d_bwd", "msda3d_bwd"):
                fn = getattr(handle, name)
                fn.argtypes = _BWD_ARGS
                fn.restype = _int
            for name in ("msda2d_bwd_accumulate", "msda3d_bwd_accumulate"):
                fn = getattr(handle, name)
                fn.argtypes = _ACC_ARGS
                fn.restype = _int
            handle.msda_bwd_static_scratch.argtypes = [_int] + _BWD_ARGS[:-3] + [_vp]
            handle.msda_bwd_static_scratch.restype = _int
            handle.msda_cast_from_f32.argtypes = [_vp, _vp, _int, _i64, _vp]
            handle.msda_cast_from_f32.restype = _int
            handle.msda_bwd_workspace_bytes.argtypes = [_int, _int, _i64, _i64, _i64, _i64, _vp, _int, _i64, _i64, _i64]
            handle.msda_bwd_workspace_bytes.restype = ctypes.c_size_t
            handle.msda_fused_bwd_workspace_bytes.argtypes = handle.msda_bwd_workspace_bytes.argtypes
            handle.msda_fused_bwd_workspace_bytes.restype = ctypes.c_size_t
            for name in ("msda2d_fused_fwd", "msda3d_fused_fwd"):
                getattr(handle, name).argtypes = _FUSED_FWD_ARGS
                getattr(handle, name).restype = _int
            for name in ("msda2d_fused_bwd", "msda3d_fused_bwd"):
                getattr(handle, name).argtypes = _FUSED_BWD_ARGS
                getattr(handle, name).restype = _int
            handle.msda_prologue_fwd.argtypes = _PROLOGUE_FWD_ARGS
            handle.msda_prologue_fwd.restype = _int
            handle.msda_prologue_bwd.argtypes = _PROLOGUE_BWD_ARGS
            handle.msda_prologue_bwd.restype = _int
            handle.msda_status_string.argtypes = [_int]
            handle.msda_status_string.restype = ctypes.c_char_p
            handle.msda_last_error.argtypes = []
            handle.msda_last_error.restype = ctypes.c_char_p
            handle.msda_abi_version.argtypes = []
            handle.msda_abi_version.restype = _int
            ver = handle.msda_abi_version()
            if ver != ABI_VERSION:
                raise RuntimeError(
                    f"msda_triton_b200: library ABI version {ver} != expected {ABI_VERSION}; rebuild"
                )
            _lib = handle
    return _lib


def last_error() -> str:
    return lib().msda_last_error().decode("utf-8", "replace")


def status_string(code: int) -> str:
    return lib().msda_status_string(code).decode("ascii", "replace")
