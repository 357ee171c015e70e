"""The C-ABI library on the CPU: it loads, exports every symbol the public
header declares, and rejects bad arguments on the host before any CUDA call
(so these checks need no GPU)."""

from __future__ import annotations

import ctypes
import os
import re

import numpy as np
import pytest

from msda_triton_b200 import _lib

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                      "include", "msda_b200.h")


def _declared_symbols() -> list[str]:
    text = open(HEADER).read()
    return re.findall(r"MSDA_API\s+[\w\s\*]+?\b(\w+)\s*\(", text)


def test_library_loads_and_reports_abi():
    lib = _lib.lib()
    assert lib.msda_abi_version() == _lib.ABI_VERSION


def test_exports_every_declared_symbol():
    declared = _declared_symbols()
    assert set(declared) == set(_lib.EXPORTED_SYMBOLS), declared
    handle = ctypes.CDLL(_lib.LIB_PATH)
    for name in declared:
        assert hasattr(handle, name), f"{name} declared in msda_b200.h but not exported"


def test_status_strings():
    assert _lib.status_string(0) == "MSDA_SUCCESS"
    assert _lib.status_string(_lib.ERROR_SHAPE_MISMATCH) == "MSDA_ERROR_SHAPE_MISMATCH"
    assert _lib.status_string(12345) == "MSDA_ERROR_UNKNOWN"


def _ws(dtype, B, shapes, H, C, Q, P, on_dev=0):
    shp = np.ascontiguousarray(np.array(shapes, dtype=np.int32))
    K = int(sum(np.prod(s) for s in shapes))
    return _lib.lib().msda_bwd_workspace_bytes(len(shapes[0]), dtype, B, K, H, C, shp.ctypes.data,
                                               on_dev, len(shapes), Q, P)


def test_workspace_bytes_gather_path(monkeypatch):
    # The gather/scatter backward: nothing for fp32; for 16-bit values an fp32
    # accumulator over every key by default.
    monkeypatch.delenv("MSDA_BWD_DIRECT16", raising=False)
    assert _ws(_lib.FLOAT32, 2, [(10, 10)], 8, 32, 50, 4) == 0
    assert _ws(_lib.BFLOAT16, 2, [(10, 10)], 8, 32, 50, 4) == 2 * 100 * 8 * 32 * 4
    assert _ws(_lib.FLOAT16, 2, [(10, 10), (5, 5)], 8, 32, 50, 4) == 2 * 125 * 8 * 32 * 4
    # Opt-in (MSDA_BWD_DIRECT16=1): levels with at most 8 expected
    # contributions per element (2^d * Q * P / voxels) reduce straight into
    # grad_value; only the busier levels keep accumulator rows.
    monkeypatch.setenv("MSDA_BWD_DIRECT16", "1")
    # 4 * 50 * 4 / 100 = 8 contributions: direct, no workspace
    assert _ws(_lib.BFLOAT16, 2, [(10, 10)], 8, 32, 50, 4) == 0
    # 4 * 51 * 4 / 100 > 8: the whole level in fp32
    assert _ws(_lib.BFLOAT16, 2, [(10, 10)], 8, 32, 51, 4) == 2 * 100 * 8 * 32 * 4
    # two levels: only the coarse one (4 * 50 * 4 / 25 = 32) is accumulated
    assert _ws(_lib.FLOAT16, 2, [(10, 10), (5, 5)], 8, 32, 50, 4) == 2 * 25 * 8 * 32 * 4
    # 3D: 8 corners per sample
    assert _ws(_lib.BFLOAT16, 1, [(8, 8, 8), (4, 4, 4)], 2, 16, 128, 4) == 64 * 2 * 16 * 4
    assert _ws(_lib.FLOAT16, 0, [(10, 10)], 8, 32, 50, 4) == 0


def _align(x):
    return (x + 255) // 256 * 256


def test_workspace_bytes_sorted_path(monkeypatch):
    # Host shapes and >= 2^20 samples: the cell-sorted backward.  Its
    # workspace: bucket counts (one per cell of the (W+1)(H+1)(D+1) grid plus
    # a dead bucket, per level and (b, h), plus one), scan block sums, a rank
    # and a 32-byte record per sample, the fp32 accumulator of the levels
    # with more than 2 samples per cell, and 16 bytes per sample of the levels
    # whose value slice per batch entry reaches 96 MiB (their dot products
    # run in sorted order and are staged).
    monkeypatch.setenv("MSDA_BWD_PATH", "sorted")
    monkeypatch.delenv("MSDA_VOXEL_DENSITY", raising=False)
    monkeypatch.delenv("MSDA_SORTED_CHUNK_B", raising=False)
    B, H, C, Q, P = 2, 8, 32, 20000, 4
    shapes = [(32, 64, 64), (16, 32, 32), (8, 16, 16)]
    cells = [int(np.prod([s + 1 for s in sh])) for sh in shapes]
    dense = [sh for c, sh in zip(cells, shapes) if Q * P / c > 2.0]
    assert len(dense) == 2  # the finest level is gathered per value row
    acc_keys = sum(int(np.prod(sh)) for sh in dense)
    nkeys = B * H * sum(c + 1 for c in cells)
    n = B * Q * H * len(shapes) * P
    nblk = (nkeys + 4095) // 4096
    expect = (_align((nkeys + 1) * 4) + _align((nblk + 1) * 4) + _align(n * 4)
              + _align(n * 32) + _align(B * acc_keys * H * C * 4))
    # bf16: the finest level holds 64 MiB of value per batch entry, no staging
    assert _ws(_lib.BFLOAT16, B, shapes, H, C, Q, P) == expect
    # fp32 values reduce the dense levels straight into grad_value: no
    # accumulator; the finest level's 128 MiB slice takes the sorted-order dots
    stage = _align(B * Q * H * 1 * P * 16)
    assert _ws(_lib.FLOAT32, B, shapes, H, C, Q, P) == (
        expect - _align(B * acc_keys * H * C * 4) + stage)
    # device-resident shapes cannot be planned on the host: gather path
    K = sum(int(np.prod(s)) for s in shapes)
    assert _ws(_lib.BFLOAT16, B, shapes, H, C, Q, P, on_dev=1) == B * K * H * C * 4
    # MSDA_BWD_PATH=scatter keeps the gather/scatter plan (fp32 accumulator)
    monkeypatch.setenv("MSDA_BWD_PATH", "scatter")
    assert _ws(_lib.BFLOAT16, B, shapes, H, C, Q, P) == B * K * H * C * 4


# A fake device address: every case below fails validation on the host before
# any pointer is dereferenced or any CUDA call is made.
FAKE = 0x10000


def _fwd(ndim=2, vdt=_lib.FLOAT32, B=1, K=20, H=2, C=8, shapes=((4, 5),), L=None,
         sdt=None, Q=3, P=2, clamp=1, eps=1e-4, value=FAKE, out=FAKE, on_dev=0):
    lib = _lib.lib()
    shp = np.ascontiguousarray(np.array(shapes, dtype=np.int32))
    L = len(shapes) if L is None else L
    sdt = vdt if sdt is None else sdt
    fn = lib.msda2d_fwd if ndim == 2 else lib.msda3d_fwd
    return fn(value, vdt, B, K, H, C, shp.ctypes.data, on_dev, L, FAKE, FAKE, sdt, Q, P,
              clamp, eps, out, None)


def test_rejects_bad_dtype():
    assert _fwd(vdt=7) == _lib.ERROR_UNSUPPORTED_DTYPE
    assert "fp32, fp16, and bf16" in _lib.last_error()
    # sampling dtype must be the value dtype or fp32
    assert _fwd(vdt=_lib.FLOAT32, sdt=_lib.BFLOAT16) == _lib.ERROR_UNSUPPORTED_DTYPE


def test_rejects_k_mismatch_with_host_shapes():
    assert _fwd(K=21) == _lib.ERROR_SHAPE_MISMATCH
    assert "does not match sum of spatial shapes" in _lib.last_error()


def test_rejects_too_many_levels():
    shapes = [(1, 1)] * (_lib.MAX_LEVELS + 1)
    assert _fwd(K=len(shapes), shapes=shapes) == _lib.ERROR_TOO_MANY_LEVELS


def test_rejects_int32_overflow():
    assert _fwd(K=2**31, shapes=[(2**16, 2**15)]) == _lib.ERROR_INT32_OVERFLOW
    assert "exceeds int32 range" in _lib.last_error()


def test_rejects_negative_dims_and_bad_eps():
    assert _fwd(Q=-1) == _lib.ERROR_INVALID_ARGUMENT
    assert _fwd(eps=1.5) == _lib.ERROR_INVALID_ARGUMENT


def test_rejects_misaligned_buffers():
    assert _fwd(value=FAKE + 2) == _lib.ERROR_MISALIGNED


def test_rejects_huge_channel_rows():
    assert _fwd(C=4096) == _lib.ERROR_UNSUPPORTED_CHANNELS


def test_empty_problem_is_a_noop():
    # Q = 0: nothing to launch, success without touching any buffer.
    assert _fwd(Q=0) == _lib.SUCCESS
    assert _lib.last_error() == ""


def test_bwd_requires_workspace_for_half_types():
    lib = _lib.lib()
    shp = np.array([[4, 5]], dtype=np.int32)
    # Q=100, P=2 on 20 cells: 40 contributions per element, fp32 accumulation
    rc = lib.msda2d_bwd(FAKE, _lib.BFLOAT16, 1, 20, 2, 8, shp.ctypes.data, 0, 1, FAKE, FAKE,
                        _lib.BFLOAT16, 100, 2, 1, 1e-4, FAKE, FAKE, FAKE, FAKE, None, 0, None)
    assert rc == _lib.ERROR_WORKSPACE
    assert "workspace" in _lib.last_error()


@pytest.mark.parametrize("ndim", [2, 3])
def test_shape_row_order(ndim):
    # Shapes rows are (H, W) / (D, H, W): K is their product sum either way.
    shapes = [(3, 5)] if ndim == 2 else [(2, 3, 5)]
    K = int(np.prod(shapes[0]))
    assert _fwd(ndim=ndim, K=K, shapes=shapes, Q=0) == _lib.SUCCESS
    assert _fwd(ndim=ndim, K=K + 1, shapes=shapes, Q=0) == _lib.ERROR_SHAPE_MISMATCH


def _fused_fwd(ndim=3, ref=FAKE, Q=3, **kw):
    lib = _lib.lib()
    shapes = kw.get("shapes", ((2, 3, 4),) if ndim == 3 else ((4, 5),))
    shp = np.ascontiguousarray(np.array(shapes, dtype=np.int32))
    K = int(sum(np.prod(s) for s in shapes))
    fn = lib.msda3d_fused_fwd if ndim == 3 else lib.msda2d_fused_fwd
    return fn(FAKE, _lib.BFLOAT16, 1, K, 2, 8, shp.ctypes.data, 0, len(shapes), ref, FAKE, FAKE,
              _lib.BFLOAT16, Q, 2, 1, 1e-4, FAKE, None)


@pytest.mark.parametrize("ndim", [2, 3])
def test_fused_entries_validate_reference_points(ndim):
    assert _fused_fwd(ndim, ref=None) == _lib.ERROR_INVALID_ARGUMENT
    assert "reference_points" in _lib.last_error()
    assert _fused_fwd(ndim, ref=FAKE + 2) == _lib.ERROR_MISALIGNED
    assert _fused_fwd(ndim, ref=None, Q=0) == _lib.SUCCESS  # nothing to sample: no pointer needed


def test_fused_workspace_is_the_gather_plan(monkeypatch):
    # The fused backward always takes the gather/scatter path, so its
    # workspace is the gather plan's, whatever MSDA_BWD_PATH says.
    lib = _lib.lib()
    B, H, C, Q, P = 2, 8, 32, 20000, 4
    shapes = [(32, 64, 64), (16, 32, 32), (8, 16, 16)]
    shp = np.ascontiguousarray(np.array(shapes, dtype=np.int32))
    K = int(sum(np.prod(s) for s in shapes))

    def fused():
        return lib.msda_fused_bwd_workspace_bytes(3, _lib.BFLOAT16, B, K, H, C, shp.ctypes.data,
                                                  0, len(shapes), Q, P)

    monkeypatch.setenv("MSDA_BWD_PATH", "scatter")
    gather = _ws(_lib.BFLOAT16, B, shapes, H, C, Q, P)
    assert fused() == gather
    monkeypatch.setenv("MSDA_BWD_PATH", "sorted")
    assert _ws(_lib.BFLOAT16, B, shapes, H, C, Q, P) != gather  # the plain entry sorts
    assert fused() == gather
