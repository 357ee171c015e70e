"""Parity at the BASELINE configurations' full sizes.

The oracle cannot run the whole of the large configs in seconds, so each
case checks, on one full-size forward + backward through the public API:
  * exact slices: for two (batch, head) pairs, the output, grad_value,
    grad_sampling_locations and grad_attention_weights of that slice against
    the oracle (heads and batch entries are independent, so a slice is a
    complete MSDA problem of its own at full K and Q);
  * adjoint identities over the full tensors: out is linear in value and in
    attention_weights, so <out, G> = <value, grad_value> = <weights, grad_weights>;
  * exact homogeneity: scaling value by 2 scales the output by exactly 2.
"""

from __future__ import annotations

import pytest
import torch

import msda_triton_b200 as M
from msda_triton_b200 import _core, _lib
from oracle import msda_bwd_oracle, msda_fwd_oracle
from tests._util import TOL_FWD_F32, TOL_GRAD_F32, TOL_HALF, assert_close

pytestmark = pytest.mark.gpu

SHAPES_2D = [(100, 150), (50, 75), (25, 38), (13, 19)]
CONFIGS = {
    "cfg1_2d_enc": dict(ndim=2, B=4, Q=19947, H=8, C=32, P=4, shapes=SHAPES_2D),
    "cfg2_2d_dec": dict(ndim=2, B=8, Q=900, H=8, C=32, P=4, shapes=SHAPES_2D),
    "cfg3_3d": dict(ndim=3, B=2, Q=20000, H=8, C=32, P=4,
                    shapes=[(32, 64, 64), (16, 32, 32), (8, 16, 16)]),
    "cfg4_3d_xl": dict(ndim=3, B=8, Q=100000, H=8, C=32, P=4,
                       shapes=[(64, 128, 128), (32, 64, 64), (16, 32, 32), (8, 16, 16)]),
}
CASES = [
    ("cfg1_2d_enc", torch.float32), ("cfg1_2d_enc", torch.bfloat16),
    ("cfg2_2d_dec", torch.bfloat16),
    ("cfg3_3d", torch.float32), ("cfg3_3d", torch.bfloat16),
    ("cfg4_3d_xl", torch.bfloat16),
]


def _inputs(cfg, dtype, dev, seed):
    B, Q, H, C, P, d = cfg["B"], cfg["Q"], cfg["H"], cfg["C"], cfg["P"], cfg["ndim"]
    L = len(cfg["shapes"])
    K = sum(int(torch.tensor(s).prod()) for s in cfg["shapes"])
    g = torch.Generator(device=dev).manual_seed(seed)
    value = torch.randn(B, K, H, C, generator=g, device=dev).to(dtype)
    loc = torch.rand(B, Q, H, L, P, d, generator=g, device=dev).to(dtype)
    attn = torch.randn(B, Q, H, L * P, generator=g, device=dev).softmax(-1)
    attn = attn.view(B, Q, H, L, P).to(dtype)
    go = torch.randn(B, Q, H * C, generator=g, device=dev).to(dtype)
    return value, torch.tensor(cfg["shapes"], dtype=torch.int64), loc, attn, go


def _dot(a, b):
    """<a, b> in float64, chunked over the leading dim to bound memory."""
    return sum(float((x.float() * y.float()).sum(dtype=torch.float64)) for x, y in zip(a, b))


@pytest.mark.parametrize("name,dtype", CASES, ids=[f"{n}-{str(d)[6:]}" for n, d in CASES])
def test_full_size(name, dtype):
    cfg = CONFIGS[name]
    dev = torch.device("cuda", 0)
    fn = M.msda3d if cfg["ndim"] == 3 else M.msda2d
    value, shapes, loc, attn, go = _inputs(cfg, dtype, dev, seed=len(name))
    v = value.requires_grad_(True)
    lo = loc.requires_grad_(True)
    a = attn.requires_grad_(True)
    out = fn(v, shapes, lo, a)
    gv, gl, ga = torch.autograd.grad(out, (v, lo, a), go)
    torch.cuda.synchronize()

    half = dtype != torch.float32
    tol_f = TOL_HALF if half else TOL_FWD_F32
    tol_g = TOL_HALF if half else TOL_GRAD_F32
    C = cfg["C"]
    B, H = cfg["B"], cfg["H"]
    for b, h in ((0, 0), (B - 1, H - 1)):
        f = lambda t: t.detach()[b:b + 1, :, h:h + 1].float().cpu().numpy()
        vs, ls, as_ = f(value), f(loc), f(attn)
        gos = go[b:b + 1, :, h * C:(h + 1) * C].float().cpu().numpy()
        ref_out = msda_fwd_oracle(vs, shapes, ls, as_)
        ref_gv, ref_gl, ref_ga = msda_bwd_oracle(vs, shapes, ls, as_, gos)
        tag = f"{name} b={b} h={h}"
        assert_close(out[b, :, h * C:(h + 1) * C].float().cpu(), ref_out[0], tol_f, f"{tag} out")
        assert_close(gv[b, :, h].float().cpu(), ref_gv[0, :, 0], tol_g, f"{tag} grad_value")
        assert_close(gl[b, :, h].float().cpu(), ref_gl[0, :, 0], tol_g, f"{tag} grad_loc")
        assert_close(ga[b, :, h].float().cpu(), ref_ga[0, :, 0], tol_g, f"{tag} grad_attn")

    # The identities hold exactly in real arithmetic; each side carries the
    # rounding of its own tensors, so the bound scales with sum |out * G|
    # (the sums themselves nearly cancel).
    lhs = _dot(out.detach(), go)
    scale = _dot(out.detach().abs(), go.abs())
    rel = 4e-3 if half else 2e-6
    for what, x, gx in (("value", value, gv), ("attention_weights", attn, ga)):
        rhs = _dot(x.detach(), gx)
        assert abs(lhs - rhs) <= rel * scale, \
            f"adjoint <out,G> vs <{what},grad>: {lhs} {rhs} (scale {scale})"

    with torch.no_grad():
        out2 = (M.msda3d_fwd if cfg["ndim"] == 3 else M.msda2d_fwd)(value.detach() * 2, shapes,
                                                                    loc.detach(), attn.detach())
        assert torch.equal(out2, out.detach() * 2)


@pytest.mark.parametrize("ndim", [2, 3])
def test_bwd_accumulate_and_cast_entry_points(ndim):
    """msda{2,3}d_bwd_accumulate adds into a caller fp32 buffer; two calls give
    twice the value gradient; msda_cast_from_f32 rounds it like the full bwd."""
    cfg = dict(ndim=ndim, B=2, Q=300, H=4, C=32, P=4,
               shapes=[(16, 16), (8, 8)] if ndim == 2 else [(8, 8, 8), (4, 4, 4)])
    dev = torch.device("cuda", 0)
    value, shapes, loc, attn, go = _inputs(cfg, torch.bfloat16, dev, seed=5)
    v = value.requires_grad_(True)
    out = (M.msda3d if ndim == 3 else M.msda2d)(v, shapes, loc, attn)
    (gv_ref,) = torch.autograd.grad(out, (v,), go)
    lib = _lib.lib()
    shp, on_dev = _core.prepare_spatial(shapes)
    args = _core._common_args(value.detach(), shp, on_dev, loc, attn)
    acc = torch.zeros(value.shape, device=dev, dtype=torch.float32)
    gl = torch.empty_like(loc)
    ga = torch.empty_like(attn)
    fn = lib.msda3d_bwd_accumulate if ndim == 3 else lib.msda2d_bwd_accumulate
    stream = torch.cuda.current_stream().cuda_stream
    for _ in range(2):
        _core.check_status(fn(*args, 1, 1e-4, go.data_ptr(), acc.data_ptr(), gl.data_ptr(),
                              ga.data_ptr(), stream))
    half_acc = acc * 0.5
    cast = torch.empty_like(value)
    _core.check_status(lib.msda_cast_from_f32(half_acc.data_ptr(), cast.data_ptr(), _lib.BFLOAT16,
                                              half_acc.numel(), stream))
    torch.cuda.synchronize()
    assert_close(cast.float().cpu(), gv_ref.float().cpu(), 1e-2, "accumulate x2 / 2")
    assert torch.equal(cast, half_acc.to(torch.bfloat16))
