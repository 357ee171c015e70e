"""ctypes binding of the C oracle (msda_oracle.c).  Test infrastructure only.

Inputs are numpy arrays (or anything np.ascontiguousarray accepts); they are
converted to contiguous float32 (value, loc, attn, grad_out) and int64
(spatial shapes).  Outputs are float32 numpy arrays in the reference's layouts:
out (B, Q, H*C); grad_value (B, K, H, C); grad_loc (B, Q, H, L, P, d);
grad_attn (B, Q, H, L, P).
"""

from __future__ import annotations

import ctypes
import os

import numpy as np

from oracle.build import LIB, build

_lib = None


def _load() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        path = LIB if os.path.exists(LIB) else build()
        lib = ctypes.CDLL(path)
        i64 = ctypes.c_int64
        fp = ctypes.c_void_p
        lib.msda_oracle_fwd.argtypes = [
            ctypes.c_int, fp, fp, i64, i64, i64, i64, i64, i64, i64,
            fp, fp, ctypes.c_int, ctypes.c_double, fp, ctypes.c_int,
        ]
        lib.msda_oracle_fwd.restype = ctypes.c_int
        lib.msda_oracle_bwd.argtypes = [
            ctypes.c_int, fp, fp, i64, i64, i64, i64, i64, i64, i64,
            fp, fp, ctypes.c_int, ctypes.c_double, fp, fp, fp, fp, ctypes.c_int,
        ]
        lib.msda_oracle_bwd.restype = ctypes.c_int
        lib.msda_oracle_cell.argtypes = [ctypes.c_float, i64, ctypes.c_int, ctypes.c_double]
        lib.msda_oracle_cell.restype = i64
        _lib = lib
    return _lib


def _f32(x) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(x, dtype=np.float32))


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


def _dims(value, shapes, loc):
    B, K, H, C = value.shape
    _, Q, _, L, P, d = loc.shape
    if shapes.shape != (L, d):
        raise ValueError(f"spatial shapes must be ({L}, {d}), got {shapes.shape}")
    return B, K, H, C, Q, L, P, d


def msda_fwd_oracle(value, spatial_shapes, sampling_locations, attention_weights,
                    clamp_grid: bool = True, clamp_eps: float = 1e-4,
                    nthreads: int = 0) -> np.ndarray:
    """Forward MSDA on the CPU: returns out (B, Q, H*C) float32."""
    v, loc, attn = _f32(value), _f32(sampling_locations), _f32(attention_weights)
    shp = np.ascontiguousarray(np.asarray(spatial_shapes, dtype=np.int64))
    B, K, H, C, Q, L, P, d = _dims(v, shp, loc)
    out = np.empty((B, Q, H * C), dtype=np.float32)
    rc = _load().msda_oracle_fwd(d, _ptr(v), _ptr(shp), B, K, H, C, Q, L, P,
                                 _ptr(loc), _ptr(attn), int(bool(clamp_grid)),
                                 float(clamp_eps), _ptr(out), int(nthreads))
    if rc != 0:
        raise ValueError(f"msda_oracle_fwd failed with code {rc}")
    return out


def msda_bwd_oracle(value, spatial_shapes, sampling_locations, attention_weights,
                    grad_output, clamp_grid: bool = True, clamp_eps: float = 1e-4,
                    nthreads: int = 0):
    """Backward MSDA on the CPU: returns (grad_value, grad_loc, grad_attn)."""
    v, loc, attn = _f32(value), _f32(sampling_locations), _f32(attention_weights)
    go = _f32(grad_output)
    shp = np.ascontiguousarray(np.asarray(spatial_shapes, dtype=np.int64))
    B, K, H, C, Q, L, P, d = _dims(v, shp, loc)
    if go.shape != (B, Q, H * C):
        raise ValueError(f"grad_output must be {(B, Q, H * C)}, got {go.shape}")
    gv = np.empty_like(v)
    gl = np.empty_like(loc)
    ga = np.empty_like(attn)
    rc = _load().msda_oracle_bwd(d, _ptr(v), _ptr(shp), B, K, H, C, Q, L, P,
                                 _ptr(loc), _ptr(attn), int(bool(clamp_grid)),
                                 float(clamp_eps), _ptr(go), _ptr(gv), _ptr(gl),
                                 _ptr(ga), int(nthreads))
    if rc != 0:
        raise ValueError(f"msda_oracle_bwd failed with code {rc}")
    return gv, gl, ga


def msda_cell_oracle(loc: float, size: int, clamp_grid: bool = True,
                     clamp_eps: float = 1e-4) -> int:
    """Index of the lower corner a normalised coordinate resolves to."""
    return int(_load().msda_oracle_cell(ctypes.c_float(loc), int(size),
                                        int(bool(clamp_grid)), float(clamp_eps)))
