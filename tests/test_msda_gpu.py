"""Parity of the CUDA kernels (through msda_triton_b200's public API, which
calls the C ABI) with the CPU oracle and with the reference's golden vectors.

The case list follows the reference's suite (tests/test_msda_2d.py and
tests/test_msda_3d.py of mach9robotics/msda-triton, lines 113-427), with the
tolerances tightened to the parity bar: fp32 forward rtol=atol=1e-5, fp32
gradients 1e-4, fp16/bf16 2e-2 against an fp32 reference on the same
(upcast) inputs.
"""

from __future__ import annotations

import pytest
import torch

import msda_triton_b200 as M
from oracle import msda_bwd_oracle, msda_fwd_oracle
from tests._util import TOL_FWD_F32, TOL_GRAD_F32, TOL_HALF, assert_close, make_inputs
from tests.conftest import golden_names, load_golden

pytestmark = pytest.mark.gpu

FNS = {2: (M.msda2d, M.msda2d_fwd), 3: (M.msda3d, M.msda3d_fwd)}
SHAPES = {
    2: [(32, 32), (16, 16), (8, 8), (4, 4)],
    3: [(4, 5, 5), (2, 3, 3), (3, 4, 4), (2, 2, 2)],
}


def cuda_fwd_bwd(ndim, value, shp, loc, attn, go, clamp=True, eps=1e-4, shapes_on_device=False):
    """Run msda{2,3}d forward + backward on cuda:0 (inputs keep their dtypes);
    returns float32 CPU tensors (out, grad_value, grad_loc, grad_attn)."""
    dev = torch.device("cuda", 0)
    v = value.to(dev).requires_grad_(True)
    lo = loc.to(dev).requires_grad_(True)
    a = attn.to(dev).requires_grad_(True)
    s = shp.to(dev) if shapes_on_device else shp
    out = FNS[ndim][0](v, s, lo, a, clamp, eps)
    out.backward(go.to(dev, out.dtype))
    torch.cuda.synchronize()
    f = lambda t: t.detach().float().cpu()
    return f(out), f(v.grad), f(lo.grad), f(a.grad)


def oracle_all(value, shp, loc, attn, go, clamp=True, eps=1e-4):
    f = lambda t: t.detach().float().cpu().numpy() if torch.is_tensor(t) else t
    out = msda_fwd_oracle(f(value), f(shp), f(loc), f(attn), clamp, eps)
    gv, gl, ga = msda_bwd_oracle(f(value), f(shp), f(loc), f(attn), f(go), clamp, eps)
    return [torch.from_numpy(x) for x in (out, gv, gl, ga)]


def check_all(got, ref, tol_fwd, tol_grad, what):
    for name, g, r, t in zip(("out", "grad_value", "grad_loc", "grad_attn"), got, ref,
                             (tol_fwd, tol_grad, tol_grad, tol_grad)):
        assert_close(g, r, t, f"{what} {name}")


# ---------------------------------------------------------------- golden vectors
@pytest.mark.parametrize("shapes_on_device", [False, True])
@pytest.mark.parametrize("name", golden_names())
def test_golden_parity(name, shapes_on_device):
    """CUDA fwd+bwd vs the reference's own grid_sample outputs and vs the oracle."""
    z = load_golden(name)
    t = {k: torch.from_numpy(z[k]) for k in ("value", "loc", "attn", "grad_out", "shapes")}
    ndim = t["shapes"].shape[1]
    clamp, eps = bool(z["clamp"]), float(z["eps"])
    got = cuda_fwd_bwd(ndim, t["value"], t["shapes"], t["loc"], t["attn"], t["grad_out"],
                       clamp, eps, shapes_on_device)
    ref = [torch.from_numpy(z[k]) for k in ("out", "grad_value", "grad_loc", "grad_attn")]
    check_all(got, ref, TOL_FWD_F32, TOL_GRAD_F32, f"{name} vs reference")
    orc = oracle_all(t["value"], t["shapes"], t["loc"], t["attn"], t["grad_out"], clamp, eps)
    check_all(got, orc, TOL_FWD_F32, TOL_GRAD_F32, f"{name} vs oracle")


# ---------------------------------------------------------------- reference cases
@pytest.mark.parametrize("ndim", [2, 3])
def test_forward_pass_basic(ndim):
    value, shp, loc, attn, go = make_inputs(2, 50, 8, 32, 4, SHAPES[ndim][:2], seed=100 + ndim)
    out = FNS[ndim][1](value.cuda(), shp, loc.cuda(), attn.cuda(), clamp_grid=True, clamp_eps=1e-4)
    assert out.shape == (2, 50, 256) and out.dtype == torch.float32
    assert_close(out.cpu(), msda_fwd_oracle(value, shp, loc, attn), TOL_FWD_F32, "fwd")


@pytest.mark.parametrize("ndim", [2, 3])
@pytest.mark.parametrize("cfg", [(1, 100, 4, 64, 3, 4), (4, 25, 8, 32, 2, 8), (2, 200, 16, 16, 4, 4)])
def test_forward_pass_different_configs(ndim, cfg):
    B, Q, H, C, L, P = cfg
    value, shp, loc, attn, go = make_inputs(B, Q, H, C, P, SHAPES[ndim][:L], seed=hash(cfg) % 1000)
    out = FNS[ndim][1](value.cuda(), shp, loc.cuda(), attn.cuda())
    assert_close(out.cpu(), msda_fwd_oracle(value, shp, loc, attn), TOL_FWD_F32, f"fwd {cfg}")


@pytest.mark.parametrize("ndim", [2, 3])
def test_backward_pass_basic(ndim):
    inp = make_inputs(2, 50, 8, 32, 4, SHAPES[ndim][:2], seed=200 + ndim)
    got = cuda_fwd_bwd(ndim, *inp)
    check_all(got, oracle_all(*inp), TOL_FWD_F32, TOL_GRAD_F32, "basic")


@pytest.mark.parametrize("ndim", [2, 3])
def test_fp64_not_supported(ndim):
    value, shp, loc, attn, _ = make_inputs(1, 10, 2, 8, 4, SHAPES[ndim][:2], seed=1,
                                           dtype=torch.float64, device="cuda")
    with pytest.raises(NotImplementedError) as exc:
        FNS[ndim][1](value, shp, loc, attn)
    assert "fp32, fp16, and bf16" in str(exc.value)
    assert "float64" in str(exc.value)


@pytest.mark.parametrize("ndim", [2, 3])
def test_error_on_cpu_tensors(ndim):
    value, shp, loc, attn, _ = make_inputs(2, 50, 8, 32, 4, SHAPES[ndim][:2], seed=1)
    for fn in FNS[ndim]:
        with pytest.raises(ValueError) as exc:
            fn(value, shp, loc, attn)
        assert "CUDA" in str(exc.value)


@pytest.mark.parametrize("ndim", [2, 3])
def test_edge_case_boundary_and_out_of_bounds(ndim):
    value, shp, loc, attn, go = make_inputs(1, 10, 8, 32, 4, SHAPES[ndim][:2], seed=300 + ndim)
    loc[0, 0, 0, 0, 0, :] = 0.0
    loc[0, 1, 0, 0, 0, :] = 1.0
    loc[0, 2, 0, 0, 0, :] = torch.tensor([0.0, 1.0, 0.5][:ndim])
    loc[0, 3, 0, 0, 0, :] = -0.1
    loc[0, 4, 0, 0, 0, :] = 1.1
    for clamp in (True, False):
        got = cuda_fwd_bwd(ndim, value, shp, loc, attn, go, clamp)
        check_all(got, oracle_all(value, shp, loc, attn, go, clamp), TOL_FWD_F32, TOL_GRAD_F32,
                  f"clamp={clamp}")


@pytest.mark.parametrize("ndim", [2, 3])
def test_gradient_flow_end_to_end(ndim):
    value, shp, loc, attn, _ = make_inputs(2, 20, 4, 16, 4, SHAPES[ndim][:2], seed=400 + ndim)
    v = value.cuda().requires_grad_(True)
    lo = loc.cuda().requires_grad_(True)
    a = attn.cuda().requires_grad_(True)
    out = FNS[ndim][0](v, shp, lo, a)
    loss = (out ** 2).sum()
    loss.backward()
    ref_out = torch.from_numpy(msda_fwd_oracle(value, shp, loc, attn))
    assert abs(loss.item() - float((ref_out.double() ** 2).sum())) < 1e-4 * max(1.0, loss.item())
    gv, gl, ga = msda_bwd_oracle(value, shp, loc, attn, (2 * ref_out).numpy())
    assert_close(v.grad.cpu(), gv, TOL_GRAD_F32, "grad_value")
    assert_close(lo.grad.cpu(), gl, TOL_GRAD_F32, "grad_loc")
    assert_close(a.grad.cpu(), ga, TOL_GRAD_F32, "grad_attn")


@pytest.mark.parametrize("ndim", [2, 3])
def test_no_clamp_grid(ndim):
    inp = make_inputs(2, 50, 8, 32, 4, SHAPES[ndim][:2], seed=500 + ndim, loc_range=(-0.3, 1.3))
    got = cuda_fwd_bwd(ndim, *inp, clamp=False)
    check_all(got, oracle_all(*inp, clamp=False), TOL_FWD_F32, TOL_GRAD_F32, "no clamp")


@pytest.mark.parametrize("ndim", [2, 3])
def test_single_level(ndim):
    inp = make_inputs(2, 50, 8, 32, 4, SHAPES[ndim][:1], seed=600 + ndim)
    got = cuda_fwd_bwd(ndim, *inp)
    check_all(got, oracle_all(*inp), TOL_FWD_F32, TOL_GRAD_F32, "single level")


@pytest.mark.parametrize("ndim", [2, 3])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_half_precision(ndim, dtype):
    """fp16/bf16 fwd AND bwd against the fp32 oracle on the same upcast inputs."""
    value, shp, loc, attn, go = make_inputs(1, 50, 4, 32, 4, SHAPES[ndim][:2], seed=700 + ndim)
    value, loc, attn, go = (t.to(dtype) for t in (value, loc, attn, go))
    got = cuda_fwd_bwd(ndim, value, shp, loc, attn, go)
    ref = oracle_all(value.float(), shp, loc.float(), attn.float(), go.float())
    check_all(got, ref, TOL_HALF, TOL_HALF, f"{dtype}")


# ---------------------------------------------------------------- beyond the reference suite
@pytest.mark.parametrize("ndim", [2, 3])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_mixed_dtype_fp32_sampling(ndim, dtype):
    """Half-precision value with fp32 locations/weights (the usual AMP layout)."""
    value, shp, loc, attn, go = make_inputs(2, 40, 4, 32, 4, SHAPES[ndim][:3], seed=800 + ndim)
    value, go = value.to(dtype), go.to(dtype)
    dev = torch.device("cuda", 0)
    v = value.to(dev).requires_grad_(True)
    lo = loc.to(dev).requires_grad_(True)
    a = attn.to(dev).requires_grad_(True)
    out = FNS[ndim][0](v, shp, lo, a)
    out.backward(go.to(dev))
    assert out.dtype == dtype and lo.grad.dtype == torch.float32 and v.grad.dtype == dtype
    ref = oracle_all(value.float(), shp, loc, attn, go.float())
    got = [t.detach().float().cpu() for t in (out, v.grad, lo.grad, a.grad)]
    check_all(got, ref, TOL_HALF, TOL_HALF, "mixed")


@pytest.mark.parametrize("ndim", [2, 3])
def test_device_and_host_shapes_agree_bitwise(ndim):
    inp = make_inputs(2, 64, 8, 32, 4, SHAPES[ndim], seed=900 + ndim)
    a = cuda_fwd_bwd(ndim, *inp, shapes_on_device=False)
    b = cuda_fwd_bwd(ndim, *inp, shapes_on_device=True)
    assert torch.equal(a[0], b[0])  # forward is deterministic
    for x, y in zip(a[1:], b[1:]):
        assert_close(x, y, 1e-6, "grads host vs device shapes")


@pytest.mark.parametrize("ndim", [2, 3])
def test_forward_deterministic(ndim):
    value, shp, loc, attn, _ = make_inputs(2, 300, 8, 32, 4, SHAPES[ndim], seed=1000 + ndim,
                                           device="cuda")
    o1 = FNS[ndim][1](value, shp, loc, attn)
    o2 = FNS[ndim][1](value, shp, loc, attn)
    assert torch.equal(o1, o2)


@pytest.mark.parametrize("ndim", [2, 3])
def test_non_contiguous_inputs(ndim):
    value, shp, loc, attn, go = make_inputs(2, 30, 4, 16, 4, SHAPES[ndim][:2], seed=1100 + ndim)
    dev = torch.device("cuda", 0)
    # Same logical tensors, stored transposed.
    v_nc = value.to(dev).transpose(1, 2).contiguous().transpose(1, 2)
    l_nc = loc.to(dev).transpose(0, 1).contiguous().transpose(0, 1)
    a_nc = attn.to(dev).transpose(1, 2).contiguous().transpose(1, 2)
    assert not v_nc.is_contiguous() and not l_nc.is_contiguous()
    out = FNS[ndim][1](v_nc, shp, l_nc, a_nc)
    assert_close(out.cpu(), msda_fwd_oracle(value, shp, loc, attn), TOL_FWD_F32, "non-contig")


@pytest.mark.parametrize("ndim", [2, 3])
def test_empty_queries(ndim):
    value, shp, loc, attn, go = make_inputs(2, 0, 8, 32, 4, SHAPES[ndim][:2], seed=1)
    got = cuda_fwd_bwd(ndim, value, shp, loc, attn, go)
    assert got[0].shape == (2, 0, 256)
    assert torch.count_nonzero(got[1]) == 0
    assert got[2].numel() == 0 and got[3].numel() == 0


@pytest.mark.parametrize("ndim", [2, 3])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_zero_points_sample_nothing(ndim, dtype):
    # P = 0: every row is an empty sum -- zero output, zero value gradient,
    # empty location/weight gradients (as the oracle gives).
    value, shp, loc, attn, go = make_inputs(2, 30, 4, 16, 0, SHAPES[ndim][:2], seed=7, dtype=dtype)
    got = cuda_fwd_bwd(ndim, value, shp, loc, attn, go)
    assert got[0].shape == (2, 30, 64) and torch.count_nonzero(got[0]) == 0
    assert got[1].shape == value.shape and torch.count_nonzero(got[1]) == 0
    assert got[2].numel() == 0 and got[3].numel() == 0
    ref = msda_fwd_oracle(value.float(), shp, loc.float(), attn.float())
    assert not ref.any()


@pytest.mark.parametrize("ndim", [2, 3])
@pytest.mark.parametrize("dtype,C", [(torch.float32, 3), (torch.float32, 6), (torch.float32, 256),
                                     (torch.float32, 200), (torch.bfloat16, 5), (torch.bfloat16, 6),
                                     (torch.bfloat16, 512), (torch.float16, 96), (torch.float16, 1)])
def test_channel_layouts(ndim, dtype, C):
    """Chunk-width / lanes-per-row variants: odd C (2- and 4-byte chunks), wide C."""
    inp = make_inputs(1, 12, 3, C, 2, SHAPES[ndim][:2], seed=C)
    inp = [t.to(dtype) if t.is_floating_point() else t for t in inp]
    got = cuda_fwd_bwd(ndim, *inp)
    ref = oracle_all(*[t.float() if t.is_floating_point() else t for t in inp])
    tol_f = TOL_FWD_F32 if dtype == torch.float32 else TOL_HALF
    tol_g = TOL_GRAD_F32 if dtype == torch.float32 else TOL_HALF
    check_all(got, ref, tol_f, tol_g, f"C={C} {dtype}")


@pytest.mark.parametrize("ndim", [2, 3])
def test_max_levels(ndim):
    shapes = [(3, 4)] * 16 if ndim == 2 else [(2, 3, 2)] * 16
    inp = make_inputs(1, 20, 2, 32, 2, shapes, seed=1200 + ndim)
    got = cuda_fwd_bwd(ndim, *inp)
    check_all(got, oracle_all(*inp), TOL_FWD_F32, TOL_GRAD_F32, "16 levels")


def test_too_many_levels_rejected():
    shapes = [(2, 2)] * 17
    value, shp, loc, attn, _ = make_inputs(1, 2, 1, 8, 1, shapes, seed=1, device="cuda")
    with pytest.raises(ValueError):
        M.msda2d_fwd(value, shp, loc, attn)


def test_k_mismatch_rejected_with_host_shapes():
    value, shp, loc, attn, _ = make_inputs(1, 4, 2, 8, 2, [(4, 4)], seed=1, device="cuda")
    with pytest.raises(ValueError, match="does not match sum of spatial shapes"):
        M.msda2d_fwd(value[:, :15], shp, loc, attn)


def test_malformed_device_shapes_do_not_read_out_of_range():
    # Device shapes are not checked against K (no host sync); a level that
    # would reach past K must contribute nothing rather than read past value.
    value, shp, loc, attn, _ = make_inputs(1, 8, 2, 8, 2, [(4, 4), (2, 2)], seed=2, device="cuda")
    bad = torch.tensor([[4, 4], [40, 40]], dtype=torch.int32, device="cuda")
    out = M.msda2d_fwd(value, bad, loc, attn)
    ref = msda_fwd_oracle(value.cpu(), shp, loc.cpu(), attn.cpu() * torch.tensor([1.0, 0.0]).view(1, 1, 1, 2, 1))
    assert_close(out.cpu(), ref, TOL_FWD_F32, "disabled level")


def test_malformed_device_shapes_huge_3d_level():
    # A 3D level of (2^31-1)^3 cells: its size product would overflow int64;
    # it is disabled and contributes nothing, the level before it is intact.
    value, shp, loc, attn, _ = make_inputs(1, 8, 2, 8, 2, [(2, 3, 4), (1, 2, 2)], seed=3,
                                           device="cuda")
    big = 2**31 - 1
    bad = torch.tensor([[2, 3, 4], [big, big, big]], dtype=torch.int32, device="cuda")
    out = M.msda3d_fwd(value, bad, loc, attn)
    keep = torch.tensor([1.0, 0.0]).view(1, 1, 1, 2, 1)
    ref = msda_fwd_oracle(value.cpu(), shp, loc.cpu(), attn.cpu() * keep)
    assert_close(out.cpu(), ref, TOL_FWD_F32, "disabled huge level")


def test_multi_stream_and_device_guard():
    inp = make_inputs(2, 64, 8, 32, 4, SHAPES[2], seed=1300, device="cuda")
    value, shp, loc, attn, _ = inp
    ref = M.msda2d_fwd(value, shp, loc, attn)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        out = M.msda2d_fwd(value, shp, loc, attn)
    s.synchronize()
    assert torch.equal(out, ref)
