"""Cases run against the bounds-checked build of the library (see
tests/test_checked_gpu.py, which starts this file with MSDA_B200_LIB set).

Each case runs forward and backward through the public API on cuda:0,
checks the fp32 results against the CPU oracle, then reads the device word
the checked kernels report out-of-buffer gathers and scatters into.  The last
line printed is a JSON summary: {"cases": n, "violations": [...],
"parity_failures": [...]}.
"""

from __future__ import annotations

import ctypes
import json
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

import torch  # noqa: E402

import msda_triton_b200 as M  # noqa: E402
from msda_triton_b200 import _lib  # noqa: E402
from msda_triton_b200.sharding import msda_query_sharded  # noqa: E402,F401
from oracle import msda_bwd_oracle, msda_fwd_oracle  # noqa: E402
from tests._util import TOL_FWD_F32, TOL_GRAD_F32, make_inputs, max_violation  # noqa: E402

DEV = torch.device("cuda", 0)


def _violations() -> int:
    fn = _lib.lib().msda_checked_violations
    fn.argtypes = [ctypes.c_int]
    fn.restype = ctypes.c_uint
    return int(fn(1))


def _plain(ndim, B, Q, H, C, P, shapes, *, dtype=torch.float32, sdtype=None, loc_range=(0.0, 1.0),
           clamp=True, device_shapes=False, seed=0, env=None, parity=True):
    for k, v in (env or {}).items():
        os.environ[k] = v
    try:
        value, shp, loc, attn, go = make_inputs(B, Q, H, C, P, shapes, seed=seed,
                                                loc_range=loc_range)
        sdtype = sdtype or dtype
        v = value.to(DEV, dtype).requires_grad_(True)
        lo = loc.to(DEV, sdtype).requires_grad_(True)
        a = attn.to(DEV, sdtype).requires_grad_(True)
        s = shp.to(DEV) if device_shapes else shp
        fn = M.msda3d if ndim == 3 else M.msda2d
        out = fn(v, s, lo, a, clamp, 1e-4)
        grads = torch.autograd.grad(out, (v, lo, a), go.to(DEV, dtype))
        torch.cuda.synchronize()
        worst = -1.0
        if parity and dtype == torch.float32 and sdtype == torch.float32:
            ref_out = msda_fwd_oracle(value, shp, loc, attn, clamp)
            ref = (ref_out,) + msda_bwd_oracle(value, shp, loc, attn, go, clamp)
            for i, (got, exp) in enumerate(zip((out,) + grads, ref)):
                tol = TOL_FWD_F32 if i == 0 else TOL_GRAD_F32
                worst = max(worst, max_violation(got.detach().cpu(), exp, tol, tol))
        return worst
    finally:
        for k in (env or {}):
            os.environ.pop(k, None)


def _fused(ndim, dtype=torch.bfloat16, off_scale=3.0, seed=0):
    shapes = [(6, 8, 10), (3, 4, 5)] if ndim == 3 else [(12, 20), (6, 10)]
    B, Q, H, C, P = 2, 300, 4, 32, 4
    L = len(shapes)
    g = torch.Generator().manual_seed(seed)
    K = sum(int(torch.tensor(s).prod()) for s in shapes)
    value = torch.randn(B, K, H, C, generator=g).to(DEV, dtype).requires_grad_(True)
    ref = torch.rand(B, Q, L, ndim, generator=g).to(DEV).requires_grad_(True)
    off = (torch.randn(B, Q, H, L, P, ndim, generator=g) * off_scale).to(DEV, dtype)
    off.requires_grad_(True)
    logits = torch.randn(B, Q, H, L * P, generator=g).to(DEV, dtype).requires_grad_(True)
    fn = M.msda3d_fused if ndim == 3 else M.msda2d_fused
    out = fn(value, torch.tensor(shapes), ref, off, logits)
    torch.autograd.grad(out.float().square().sum(), (value, ref, off, logits))
    torch.cuda.synchronize()
    return -1.0


def main() -> None:
    assert os.environ.get("MSDA_B200_LIB"), "run with MSDA_B200_LIB=<checked library>"
    _violations()  # clear
    s3 = [(6, 8, 10), (3, 4, 5), (2, 2, 3)]
    s2 = [(24, 30), (12, 15), (6, 8)]
    cases = []
    for ndim, shapes in ((3, s3), (2, s2)):
        for dtype, sdt in ((torch.float32, None), (torch.bfloat16, None), (torch.float16, None),
                           (torch.bfloat16, torch.float32)):
            for clamp, lr in ((True, (0.0, 1.0)), (True, (-0.5, 1.5)), (False, (-0.5, 1.5))):
                for dev_shapes in (False, True):
                    cases.append((f"{ndim}d {dtype} {sdt} clamp={clamp} loc={lr} dev={dev_shapes}",
                                  lambda ndim=ndim, shapes=shapes, dtype=dtype, sdt=sdt, clamp=clamp,
                                  lr=lr, dev_shapes=dev_shapes: _plain(
                                      ndim, 2, 257, 4, 32, 4, shapes, dtype=dtype, sdtype=sdt,
                                      loc_range=lr, clamp=clamp, device_shapes=dev_shapes)))
        # every level in fp32 accumulation, then every 16-bit level reduced directly
        cases.append((f"{ndim}d bf16 direct16 off", lambda ndim=ndim, shapes=shapes: _plain(
            ndim, 2, 257, 4, 32, 4, shapes, dtype=torch.bfloat16, env={"MSDA_BWD_DIRECT16": "0"})))
        cases.append((f"{ndim}d bf16 direct16 all", lambda ndim=ndim, shapes=shapes: _plain(
            ndim, 2, 257, 4, 32, 4, shapes, dtype=torch.bfloat16,
            env={"MSDA_BWD_DIRECT16_MAX": "1e9"})))
        # row shapes: wide (several chunks per lane), narrow (one lane per row), ragged C
        for C in (128, 4, 12):
            cases.append((f"{ndim}d fp32 C={C}", lambda ndim=ndim, shapes=shapes, C=C: _plain(
                ndim, 1, 97, 3, C, 3, shapes)))
            cases.append((f"{ndim}d bf16 C={C}", lambda ndim=ndim, shapes=shapes, C=C: _plain(
                ndim, 1, 97, 3, C, 3, shapes, dtype=torch.bfloat16)))
        # the cell-sorted backward with every level gathered per value row:
        # tensor-core and CUDA-core voxel kernels (their layout guard reports
        # bit 8), fp32 with parity
        for vm in ("1", "tc", "0"):
            for C in (16, 32, 64):
                cases.append((f"{ndim}d bf16 sorted voxel mma={vm} C={C}",
                              lambda ndim=ndim, shapes=shapes, vm=vm, C=C: _plain(
                                  ndim, 2, 257, 4, C, 4, shapes, dtype=torch.bfloat16,
                                  loc_range=(-0.5, 1.5), env={"MSDA_BWD_PATH": "sorted",
                                                              "MSDA_VOXEL_DENSITY": "1e9",
                                                              "MSDA_VOXEL_MMA": vm})))
        cases.append((f"{ndim}d fp32 sorted voxel", lambda ndim=ndim, shapes=shapes: _plain(
            ndim, 2, 257, 4, 32, 4, shapes, env={"MSDA_BWD_PATH": "sorted",
                                                 "MSDA_VOXEL_DENSITY": "1e9"})))
        cases.append((f"{ndim}d fused bf16", lambda ndim=ndim: _fused(ndim)))
        cases.append((f"{ndim}d fused fp32 far offsets", lambda ndim=ndim: _fused(
            ndim, torch.float32, off_scale=40.0)))

    violations, parity = [], []
    for name, run in cases:
        worst = run()
        bits = _violations()
        if bits:
            violations.append(f"{name}: bits {bits:#x}")
        if worst > 0:
            parity.append(f"{name}: worst excess {worst:.3g}")
        print(f"{name}: bits {bits} parity {worst:.3g}", flush=True)
    print(json.dumps({"cases": len(cases), "violations": violations, "parity_failures": parity}))


if __name__ == "__main__":
    main()
