"""The cell-sorted backward (msda_sorted.cuh) against the oracle and the
reference's golden vectors.

The sorted pipeline is the default backward for large problems with host
shapes; these tests force it (MSDA_BWD_PATH=sorted) on small problems so the
oracle finishes in seconds, and steer every level through both ways of
forming the value gradient: gathered per value row (MSDA_VOXEL_DENSITY high)
and aggregated per cell with fp32 reductions (MSDA_VOXEL_DENSITY=0).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from msda_triton_b200 import _lib
from tests._util import TOL_FWD_F32, TOL_GRAD_F32, TOL_HALF, make_inputs
from tests.conftest import golden_names, load_golden
from tests.test_msda_gpu import check_all, cuda_fwd_bwd, oracle_all

pytestmark = pytest.mark.gpu

# voxel-density thresholds: every level gathered / default split / every level aggregated
SPLITS = {"voxel": "1e9", "auto": None, "cell": "0"}


# levels whose grad_attn / grad_loc run in sorted order (msda_sdots_kernel):
# the default (only value slices of 96 MiB and more: none at these sizes) or all
SDOTS = {"query": None, "sorted": "0"}


def _env(monkeypatch, split="auto", chunk=None, path="sorted", sdots="query"):
    monkeypatch.setenv("MSDA_BWD_PATH", path)
    if SDOTS[sdots] is None:
        monkeypatch.delenv("MSDA_SORTED_DOTS_MB", raising=False)
    else:
        monkeypatch.setenv("MSDA_SORTED_DOTS_MB", SDOTS[sdots])
    if SPLITS[split] is None:
        monkeypatch.delenv("MSDA_VOXEL_DENSITY", raising=False)
    else:
        monkeypatch.setenv("MSDA_VOXEL_DENSITY", SPLITS[split])
    if chunk is None:
        monkeypatch.delenv("MSDA_SORTED_CHUNK_B", raising=False)
    else:
        monkeypatch.setenv("MSDA_SORTED_CHUNK_B", str(chunk))


def _tols(dtype):
    return (TOL_FWD_F32, TOL_GRAD_F32) if dtype == torch.float32 else (TOL_HALF, TOL_HALF)


def _cast(inp, vdt, sdt):
    value, shp, loc, attn, go = inp
    return value.to(vdt), shp, loc.to(sdt), attn.to(sdt), go.to(vdt)


def _upcast(inp):
    return [x.float() if x.is_floating_point() else x for x in inp]


@pytest.mark.parametrize("split,sdots", [("voxel", "query"), ("cell", "sorted")])
@pytest.mark.parametrize("name", golden_names())
def test_golden_parity_sorted(monkeypatch, name, split, sdots):
    """Every golden fixture through the sorted backward, each level's value
    gradient formed both ways and its dot products taken in both orders,
    against the reference's own outputs."""
    _env(monkeypatch, split, sdots=sdots)
    z = load_golden(name)
    t = {k: torch.from_numpy(z[k]) for k in ("value", "loc", "attn", "grad_out", "shapes")}
    ndim = t["shapes"].shape[1]
    got = cuda_fwd_bwd(ndim, t["value"], t["shapes"], t["loc"], t["attn"], t["grad_out"],
                       bool(z["clamp"]), float(z["eps"]))
    ref = [torch.from_numpy(z[k]) for k in ("out", "grad_value", "grad_loc", "grad_attn")]
    check_all(got, ref, TOL_FWD_F32, TOL_GRAD_F32, f"{name} sorted/{split}")


CASES = [
    # ndim, B, Q, H, C, P, shapes
    (2, 2, 700, 4, 32, 4, [(40, 60), (20, 30), (10, 15), (5, 8)]),
    (3, 2, 900, 4, 32, 4, [(16, 24, 24), (8, 12, 12), (4, 6, 6)]),
    (3, 3, 400, 8, 16, 2, [(3, 4, 4), (12, 16, 20), (2, 3, 3)]),
    (2, 1, 300, 3, 64, 3, [(7, 9), (1, 1), (30, 2)]),
]
DTYPES = [(torch.float32, torch.float32), (torch.bfloat16, torch.bfloat16),
          (torch.float16, torch.float16), (torch.bfloat16, torch.float32),
          (torch.float16, torch.float32)]


@pytest.mark.parametrize("sdots", ["query", "sorted"])
@pytest.mark.parametrize("split", ["voxel", "auto", "cell"])
@pytest.mark.parametrize("dt", DTYPES, ids=lambda d: f"{str(d[0])[6:]}-{str(d[1])[6:]}")
@pytest.mark.parametrize("case", CASES, ids=[f"{c[0]}d-{len(c[6])}lvl-q{c[2]}" for c in CASES])
def test_sorted_matches_oracle(monkeypatch, case, dt, split, sdots):
    ndim, B, Q, H, C, P, shapes = case
    _env(monkeypatch, split, sdots=sdots)
    tf, tg = _tols(dt[0])
    for clamp, rng in ((True, (0.0, 1.0)), (False, (-0.15, 1.15))):
        inp = _cast(make_inputs(B, Q, H, C, P, shapes, seed=Q + C + ndim, loc_range=rng), *dt)
        got = cuda_fwd_bwd(ndim, *inp, clamp=clamp)
        ref = oracle_all(*_upcast(inp), clamp=clamp)
        check_all(got, ref, tf, tg, f"{case} {dt} {split} clamp={clamp}")


@pytest.mark.parametrize("ndim", [2, 3])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_chunks_match_one_pass(monkeypatch, ndim, dtype):
    """Batch entries split over chunks (one, two, then all at once) give the
    oracle's result, each chunk reusing the same workspace."""
    shapes = [(30, 40), (15, 20), (8, 10)] if ndim == 2 else [(12, 16, 16), (6, 8, 8), (3, 4, 4)]
    inp = _cast(make_inputs(5, 300, 4, 32, 4, shapes, seed=7 + ndim), dtype, dtype)
    ref = oracle_all(*_upcast(inp))
    tf, tg = _tols(dtype)
    for chunk, sdots in ((1, "sorted"), (2, "query"), (2, "sorted"), (None, "sorted")):
        _env(monkeypatch, "auto", chunk, sdots=sdots)
        got = cuda_fwd_bwd(ndim, *inp)
        check_all(got, ref, tf, tg, f"chunk={chunk} {sdots}")


@pytest.mark.parametrize("ndim", [2, 3])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_sorted_and_scatter_paths_agree(monkeypatch, ndim, dtype):
    """The two backward plans on one problem: the forward is the same kernel
    (bitwise equal), every gradient agrees at the parity bar (the per-sample
    sums run in another order)."""
    shapes = [(40, 50), (20, 25), (10, 12)] if ndim == 2 else [(16, 20, 20), (8, 10, 10), (4, 5, 5)]
    inp = _cast(make_inputs(2, 800, 8, 32, 4, shapes, seed=31 + ndim), dtype, dtype)
    _env(monkeypatch, "auto")
    srt = cuda_fwd_bwd(ndim, *inp)
    _env(monkeypatch, path="scatter")
    sct = cuda_fwd_bwd(ndim, *inp)
    assert torch.equal(srt[0], sct[0])
    tol = TOL_GRAD_F32 if dtype == torch.float32 else TOL_HALF
    check_all(srt, sct, tol, tol, "sorted vs scatter")


def _clustered(ndim, B, Q, H, C, P, shapes, box, seed, dtype):
    """Every sample of level 0 inside a box of `box` cells per axis at the
    centre of the level (hundreds of samples per cell), the other levels
    uniform."""
    value, shp, loc, attn, go = make_inputs(B, Q, H, C, P, shapes, seed=seed)
    g = torch.Generator().manual_seed(seed + 1)
    for ax in range(ndim):
        n = shapes[0][ndim - 1 - ax]  # (x, y, z) -> W, H, D
        lo = (n // 2 - box / 2) / n
        loc[:, :, :, 0, :, ax] = lo + torch.rand(B, Q, H, P, generator=g) * (box / n)
    return _cast((value, shp, loc, attn, go), dtype, dtype)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("ndim", [2, 3])
@pytest.mark.parametrize("path", ["sorted", "sorted-sdots", "scatter"])
def test_clustered_samples_half_precision(monkeypatch, ndim, dtype, path):
    """Hundreds of contributions per grad_value element on a level the
    density plan rates sparse: every fp16/bf16 backward stays within the
    half-precision bar of the fp32 oracle."""
    shapes = [(64, 96), (32, 48), (16, 24)] if ndim == 2 else [(24, 32, 32), (12, 16, 16), (6, 8, 8)]
    inp = _clustered(ndim, 2, 2000, 4, 32, 4, shapes, 4, 11 + ndim, dtype)
    _env(monkeypatch, "auto", path=path.split("-")[0],
         sdots="sorted" if path.endswith("sdots") else "query")
    got = cuda_fwd_bwd(ndim, *inp)
    ref = oracle_all(*_upcast(inp))
    check_all(got, ref, TOL_HALF, TOL_HALF, f"clustered {dtype} {path}")


def test_workspace_reports_sorted_plan(monkeypatch):
    """The workspace query follows the plan: the sorted plan needs per-sample
    and per-cell arrays, the scatter plan only the fp32 accumulator."""
    shapes = np.array([(16, 24, 24), (8, 12, 12)], dtype=np.int32)
    K = int(np.prod(shapes, axis=1).sum())
    B, Q, H, C, P = 2, 900, 4, 32, 4
    q = lambda: _lib.lib().msda_bwd_workspace_bytes(3, _lib.BFLOAT16, B, K, H, C,
                                                     shapes.ctypes.data, 0, 2, Q, P)
    _env(monkeypatch, "auto")
    sorted_ws = q()
    _env(monkeypatch, path="scatter")
    scatter_ws = q()
    samples = B * Q * H * 2 * P
    assert sorted_ws >= samples * 32
    assert scatter_ws == B * K * H * C * 4


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("case", CASES, ids=[f"{c[0]}d-{len(c[6])}lvl-q{c[2]}" for c in CASES])
def test_dense_cuda_core_and_tensor_core_agree(monkeypatch, case, dtype):
    """16-bit values: the per-cell aggregation of dense levels on the tensor
    cores (weights split into two 16-bit halves; by default for levels with
    at least 8 samples per cell, here for all) and on the CUDA cores
    (MSDA_DENSE_MMA=0) both meet the half-precision bar against the oracle,
    with every level aggregated per cell."""
    ndim, B, Q, H, C, P, shapes = case
    inp = _cast(make_inputs(B, Q, H, C, P, shapes, seed=3 * Q + C), dtype, dtype)
    ref = oracle_all(*_upcast(inp))
    for mma in ("1", "0"):
        _env(monkeypatch, "cell")
        monkeypatch.setenv("MSDA_DENSE_MMA", mma)
        monkeypatch.setenv("MSDA_DENSE_MMA_DENSITY", "0")  # every dense level
        got = cuda_fwd_bwd(ndim, *inp)
        check_all(got, ref, TOL_HALF, TOL_HALF, f"{case} {dtype} dense mma={mma}")


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("case", CASES, ids=[f"{c[0]}d-{len(c[6])}lvl-q{c[2]}" for c in CASES])
def test_voxel_cuda_core_and_tensor_core_agree(monkeypatch, case, dtype):
    """16-bit values: the per-row gather of voxel levels on the tensor cores
    (`mma.sync`, the default for C = 16, 32, 64; weights split into two
    16-bit halves), on the fifth-generation tensor cores (MSDA_VOXEL_MMA=tc:
    tcgen05 with accumulators in tensor memory) and on the CUDA cores
    (MSDA_VOXEL_MMA=0) all meet the half-precision bar against the oracle,
    with every level gathered per row, in-range and clamped (out-of-range)
    locations."""
    ndim, B, Q, H, C, P, shapes = case
    for clamp, rng in ((True, (0.0, 1.0)), (False, (-0.15, 1.15))):
        inp = _cast(make_inputs(B, Q, H, C, P, shapes, seed=5 * Q + C, loc_range=rng),
                    dtype, dtype)
        ref = oracle_all(*_upcast(inp), clamp=clamp)
        for mma in ("1", "tc", "0"):
            _env(monkeypatch, "voxel")
            monkeypatch.setenv("MSDA_VOXEL_MMA", mma)
            got = cuda_fwd_bwd(ndim, *inp, clamp=clamp)
            check_all(got, ref, TOL_HALF, TOL_HALF, f"{case} {dtype} voxel mma={mma} clamp={clamp}")


@pytest.mark.parametrize("ndim", [2, 3])
def test_voxel_tensor_core_many_staging_rounds(monkeypatch, ndim):
    """The tensor-core voxel gather with a shared-memory budget of 24 KB:
    about 24 samples staged per round, so every tile runs many rounds (the
    accumulators carry across them, and a warp's second segment restages
    them).  bf16 against the oracle at the half-precision bar."""
    shapes = [(30, 40), (15, 20)] if ndim == 2 else [(10, 24, 24), (5, 12, 12)]
    inp = _cast(make_inputs(2, 700, 4, 32, 4, shapes, seed=29 + ndim, loc_range=(-0.1, 1.1)),
                torch.bfloat16, torch.bfloat16)
    ref = oracle_all(*_upcast(inp))
    _env(monkeypatch, "voxel")
    monkeypatch.setenv("MSDA_VOXEL_SMEM_KB", "24")
    got = cuda_fwd_bwd(ndim, *inp)
    check_all(got, ref, TOL_HALF, TOL_HALF, f"{ndim}d voxel mma, 24 KB staging")


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("path", ["sorted", "scatter"])
def test_module_like_clustered_half_precision(monkeypatch, path, dtype):
    """Sampling points the way the MSDA3D module forms them -- reference point
    per query plus init_weights' per-head offset pattern (with per-query
    jitter of half a cell) divided by the level size -- with every reference
    point inside a 4-cell box of the finest level: hundreds of contributions
    per value-gradient element on every level.  16-bit values against the
    fp32 oracle at the half-precision bar."""
    from msda_triton_b200.modules import MSDA3D

    shapes = [(12, 16, 16), (6, 8, 8), (3, 4, 4)]
    B, Q, H, C, L, P = 2, 3000, 8, 32, len(shapes), 4
    g = torch.Generator().manual_seed(17)
    m = MSDA3D(embed_dims=H * C, num_heads=H, num_levels=L, num_points=P)
    m.init_weights()
    pattern = m.sampling_offsets.bias.detach().view(H, L, P, 3)           # (H, L, P, 3) in cells
    off = pattern + 0.5 * torch.randn(B, Q, H, L, P, 3, generator=g)
    box = torch.tensor([4.0 / s for s in (16, 16, 12)])                   # 4 cells of level 0 (x, y, z)
    ref = 0.5 - box / 2 + torch.rand(B, Q, L, 3, generator=g) * box
    norm = torch.tensor([[w, h, d] for d, h, w in shapes], dtype=torch.float32)
    loc = ref[:, :, None, :, None, :] + off / norm[None, None, None, :, None, :]
    attn = torch.randn(B, Q, H, L * P, generator=g).softmax(-1).view(B, Q, H, L, P)
    value = torch.randn(B, sum(d * h * w for d, h, w in shapes), H, C, generator=g)
    go = torch.randn(B, Q, H * C, generator=g)
    inp = _cast((value, torch.tensor(shapes), loc, attn, go), dtype, dtype)
    _env(monkeypatch, "auto", path=path)
    got = cuda_fwd_bwd(3, *inp)
    ref_out = oracle_all(*_upcast(inp))
    check_all(got, ref_out, TOL_HALF, TOL_HALF, f"module-like clustered {dtype} {path}")
