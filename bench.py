#!/usr/bin/env python
"""Benchmark of the MSDA hot path on B200 (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl reference]

A step is one forward + backward pass (msda3d / msda2d through the public
autograd API) over one batch of synthetic inputs already resident in HBM.
Default workload: the BASELINE "3D xl" config -- bf16, global B=8, Q=100000,
H=8, C=32, L=4, P=4, levels (64,128,128),(32,64,64),(16,32,32),(8,16,16).

Multi-GPU (torchrun, one process per GPU): batch sharding with no data-path
collective.  By default the global batch is split over the ranks (strong
scaling: B/N entries per rank, BASELINE config 4 as written);
--scaling weak gives every rank its own full batch.  The step time is the
max over ranks (NCCL all_reduce of the CUDA-event time).

--impl reference: the reference's own CPU implementation of the path --
msda{2,3}d_pytorch (grid_sample) from the unmodified package installed
under baseline/_ref, fp32, all host threads -- times a bounded sample of the
same workload; rank 0 only.  Without baseline/_ref the C restatement in
oracle/ stands in (kind "port").
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

SHAPES_2D = [(100, 150), (50, 75), (25, 38), (13, 19)]
WORKLOADS = {
    # the headline (bf16 3D xl fwd+bwd).
    "3d_xl_bf16": dict(ndim=3, B=8, Q=100000, H=8, C=32, P=4, dtype=torch.bfloat16,
                       shapes=[(64, 128, 128), (32, 64, 64), (16, 32, 32), (8, 16, 16)]),
    # BASELINE configs[3].
    "3d_bf16": dict(ndim=3, B=2, Q=20000, H=8, C=32, P=4, dtype=torch.bfloat16,
                    shapes=[(32, 64, 64), (16, 32, 32), (8, 16, 16)]),
    "3d_fp32": dict(ndim=3, B=2, Q=20000, H=8, C=32, P=4, dtype=torch.float32,
                    shapes=[(32, 64, 64), (16, 32, 32), (8, 16, 16)]),
    # BASELINE configs[1].
    "2d_enc_bf16": dict(ndim=2, B=4, Q=19947, H=8, C=32, P=4, dtype=torch.bfloat16, shapes=SHAPES_2D),
    "2d_enc_fp32": dict(ndim=2, B=4, Q=19947, H=8, C=32, P=4, dtype=torch.float32, shapes=SHAPES_2D),
    # the reference's own CPU-runnable case.
    "2d_cfg0_fp32": dict(ndim=2, B=1, Q=300, H=8, C=32, P=4, dtype=torch.float32,
                         shapes=[(32, 32), (16, 16), (8, 8), (4, 4)]),
    # BASELINE configs[2] (inference: forward only).
    "2d_dec_bf16": dict(ndim=2, B=8, Q=900, H=8, C=32, P=4, dtype=torch.bfloat16, shapes=SHAPES_2D,
                        fwd_only=True),
    # The MSDA3D / MSDA2D nn.Modules (projections + sampling + output
    # projection, init_weights() state, reference points U[0,1)) on the
    # shapes of configs 4 and 1; informational, not the headline.
    "module3d_xl_bf16": dict(ndim=3, B=8, Q=100000, H=8, C=32, P=4, dtype=torch.bfloat16,
                             shapes=[(64, 128, 128), (32, 64, 64), (16, 32, 32), (8, 16, 16)],
                             module=True),
    "module2d_enc_bf16": dict(ndim=2, B=4, Q=19947, H=8, C=32, P=4, dtype=torch.bfloat16,
                              shapes=SHAPES_2D, module=True),
}
DTYPE_NAME = {torch.bfloat16: "bf16", torch.float16: "fp16", torch.float32: "fp32"}
L2_BYTES = 126 * 1000 * 1000


def _num_keys(shapes) -> int:
    n = 0
    for s in shapes:
        p = 1
        for v in s:
            p *= v
        n += p
    return n


def dims(wl):
    return wl["B"], _num_keys(wl["shapes"]), wl["H"], wl["C"], wl["Q"], len(wl["shapes"]), wl["P"]


def algorithmic_bytes(wl, B=None):
    """Unique bytes per pass (value/loc/weights/out; grads) -- the roofline basis."""
    B0, K, H, C, Q, L, P = dims(wl)
    B = B0 if B is None else B
    d = wl["ndim"]
    e = torch.tensor([], dtype=wl["dtype"]).element_size()
    smp = B * Q * H * L * P
    fwd = e * (B * K * H * C + smp * d + smp + B * Q * H * C)
    bwd = e * (2 * B * K * H * C + 2 * smp * (d + 1) + B * Q * H * C)
    return {"fwd": fwd, "bwd": bwd, "fwd_bwd": fwd + bwd,
            "samples": smp}


def make_inputs(wl, device, seed):
    """value ~ N(0,1), loc ~ U[0,1), weights = softmax(N(0,1) logits over L*P),
    grad_out ~ N(0,1); generated on the device from a seeded generator."""
    B, K, H, C, Q, L, P = dims(wl)
    d, dt = wl["ndim"], wl["dtype"]
    g = torch.Generator(device=device).manual_seed(seed)
    value = torch.randn(B, K, H, C, generator=g, device=device, dtype=torch.float32).to(dt)
    loc = torch.rand(B, Q, H, L, P, d, generator=g, device=device, dtype=torch.float32).to(dt)
    attn = torch.randn(B, Q, H, L * P, generator=g, device=device, dtype=torch.float32)
    attn = attn.softmax(-1).view(B, Q, H, L, P).to(dt)
    go = torch.randn(B, Q, H * C, generator=g, device=device, dtype=torch.float32).to(dt)
    shapes = torch.tensor(wl["shapes"], dtype=torch.int32)
    return value, shapes, loc, attn, go


# ---------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons during a region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpus):
        self.gpus = gpus
        self.proc = None
        self.path = os.path.join(tempfile.gettempdir(), f"msda_bench_clocks_{os.getpid()}.csv")

    def __enter__(self):
        try:
            os.makedirs(os.path.dirname(self.path), exist_ok=True)
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-i", ",".join(str(g) for g in self.gpus), "-lms", "200"],
                stdout=self.fh, stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except (OSError, ValueError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.fh.close()

    def summary(self):
        if self.proc is None:
            return None
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        try:
            lines = open(self.path).read().strip().splitlines()
        except OSError:
            return None
        for line in lines:
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(smax),
                "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------- our arm
def _peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            pk = json.load(f)
        return float(pk["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


def _traffic(workload, kernel, batch):
    """DRAM bytes per launch from the committed ncu summary (bytes per batch
    entry, which the per-batch head-group schedule keeps proportional to B)."""
    try:
        with open(os.path.join(ROOT, "profiles", "dram_traffic.json")) as f:
            ent = json.load(f).get(workload, {}).get(kernel)
    except (OSError, ValueError):
        return None
    return None if ent is None else float(ent["bytes_per_batch"]) * batch


def time_events(fn, iters, stream):
    """Per-call CUDA-event times (ms) of fn() on `stream` after warm-up."""
    times = []
    for _ in range(iters):
        s = torch.cuda.Event(enable_timing=True)
        e = torch.cuda.Event(enable_timing=True)
        s.record(stream)
        fn()
        e.record(stream)
        e.synchronize()
        times.append(s.elapsed_time(e))
    return times


def run_ours(args, wl, rank, world, local_rank):
    import msda_triton_b200 as M
    from msda_triton_b200 import _core, _lib

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)

    fn = M.msda3d if wl["ndim"] == 3 else M.msda2d
    global_b = wl["B"]
    if args.scaling == "strong" and world > 1:
        if wl["B"] % world:
            raise SystemExit(f"--scaling strong: batch {wl['B']} does not split over {world} GPUs")
        wl = dict(wl, B=wl["B"] // world)
    else:
        global_b = wl["B"] * world
    value, shapes, loc, attn, go = make_inputs(wl, dev, seed=1234 + rank)
    if args.value_layout == "bhkc":
        # the same values stored head-major, handed over as the (B, K, H, C) view
        value = value.permute(0, 2, 1, 3).contiguous().permute(0, 2, 1, 3)
    v = value.requires_grad_(True)
    lo = loc.requires_grad_(True)
    a = attn.requires_grad_(True)
    fwd_only = wl.get("fwd_only", False)

    def step():
        out = fn(v, shapes, lo, a)
        if not fwd_only:
            torch.autograd.grad(out, (v, lo, a), go)

    stream = torch.cuda.current_stream(dev)
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize(dev)

    gpus = list(range(world)) if world > 1 else [local_rank]
    barrier()
    with ClockSampler(gpus) if rank == 0 else _Null() as clk:
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        for _ in range(args.steps):
            step()
        t1.record(stream)
        barrier()
    ms = t0.elapsed_time(t1) / args.steps
    if dist is not None:
        tt = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms = float(tt.item())

    # ---- per-kernel times (one launch each), through the C ABI directly
    lib = _lib.lib()
    B, K, H, C, Q, L, P = dims(wl)
    shp, on_dev = _core.prepare_spatial(shapes)
    args_c = _core._common_args(value.detach(), shp, on_dev, loc.detach(), attn.detach())
    out_buf = torch.empty(B, Q, H * C, device=dev, dtype=wl["dtype"])
    fwd_c = lib.msda3d_fwd if wl["ndim"] == 3 else lib.msda2d_fwd
    bwd_c = lib.msda3d_bwd if wl["ndim"] == 3 else lib.msda2d_bwd
    sp = stream.cuda_stream
    kiters = max(3, min(args.steps, 10))

    def k_fwd():
        _core.check_status(fwd_c(*args_c, 1, 1e-4, out_buf.data_ptr(), sp))

    fwd_times = time_events(k_fwd, kiters + 2, stream)[2:]
    kern = {"fwd": statistics.mean(fwd_times)}
    bwd_launches = 0
    ws_bytes = 0
    if not fwd_only:
        # The backward entry exactly as the autograd path calls it: zero-fill
        # of the value-gradient targets, the scatter kernel and (16-bit
        # values with an fp32 accumulator) the cast kernel.
        ws_bytes = lib.msda_bwd_workspace_bytes(wl["ndim"], _core.value_code(value), B, K,
                                                H, C, shp.data_ptr(), int(on_dev), L, Q, P)
        ws = torch.empty(max(ws_bytes, 1), device=dev, dtype=torch.uint8)
        gv = torch.empty_like(value)
        gl = torch.empty_like(loc)
        ga = torch.empty_like(attn)

        def k_bwd():
            _core.check_status(bwd_c(*args_c, 1, 1e-4, go.data_ptr(), gv.data_ptr(),
                                     gl.data_ptr(), ga.data_ptr(), ws.data_ptr(), ws_bytes, sp))

        kern["bwd"] = statistics.mean(time_events(k_bwd, kiters + 2, stream)[2:])
        bwd_launches = _count_launches(k_bwd)
        if bwd_launches is None:
            bwd_launches = _bwd_launches(wl, ws_bytes)
        del ws, gv, gl, ga
    if dist is not None:
        for k in list(kern):
            tt = torch.tensor([kern[k]], device=dev, dtype=torch.float64)
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            kern[k] = float(tt.item())

    # ---- end to end: pinned host buffers in, results back to the host
    e2e = run_e2e(args, wl, fn, dev, shapes, value, loc, attn, go, fwd_only, dist)

    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return None

    ab = algorithmic_bytes(wl)
    per_pass = ab["fwd"] if fwd_only else ab["fwd_bwd"]
    samples = ab["samples"] * world
    peak, peak_kind = _peaks()
    dom = "fwd" if fwd_only or kern["fwd"] >= kern.get("bwd", 0.0) else "bwd"
    dom_bytes = ab[dom]
    achieved = dom_bytes / (kern[dom] * 1e-3) / 1e9
    traffic = _traffic(args.workload, dom, B)
    pass_gbs = per_pass / (ms * 1e-3) / 1e9
    launches_per_step = 1 + bwd_launches
    res = {
        "metric": "MSDA fwd+bwd Gsamples/s" if not fwd_only else "MSDA fwd Gsamples/s",
        "value": samples / (ms * 1e-3) / 1e9,
        "unit": "Gsamples/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms,
        "higher_is_better": True,
        "scaling": args.scaling,
        "vs_baseline": None,
        "dtype": DTYPE_NAME[wl["dtype"]],
        "data": "synthetic (seeded N(0,1) value/grad_out, U[0,1) locations, softmax weights)",
        "config": {
            "workload": args.workload, "ndim": wl["ndim"], "batch_per_gpu": B,
            "global_batch": global_b, "num_queries": Q, "num_heads": H, "channels": C,
            "num_levels": L, "num_points": P, "spatial_shapes": wl["shapes"],
            "parallelism": f"batch-sharded dp{world} (no collective)",
            "value_layout": "(B, K, H, C)" if args.value_layout == "bkhc" else "(B, H, K, C)",
            "l2": f"inputs larger than L2 (value {value.numel() * value.element_size() / 1e9:.2f} GB"
                  f" > {L2_BYTES / 1e6:.0f} MB); no flush",
        },
        "fwd_ms": kern["fwd"],
        "bwd_ms": kern.get("bwd"),
        "pass_bytes": per_pass,
        "pass_roofline_frac": pass_gbs / peak,
        "roofline": {
            "kernel": "msda_fwd_kernel" if dom == "fwd" else _bwd_entry_name(wl, ws_bytes),
            "bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
            "frac": achieved / peak, "peak_source": peak_kind,
            "algorithmic_bytes": dom_bytes, "traffic": traffic,
        },
        "gpu_launches": launches_per_step * args.steps,
        "clocks": clk.summary(),
        "e2e": e2e,
    }
    # the CPU baseline is a single-GPU figure: rank 0 at N=1 only
    res["cpu_baseline"] = cpu_baseline(args, WORKLOADS[args.workload]) if world == 1 else None
    return res


def _bwd_plan_is_sorted(wl, ws_bytes):
    """Whether the library picked the cell-sorted backward for this workload
    (its workspace holds a 32-byte record per sample)."""
    return ws_bytes >= algorithmic_bytes(wl)["samples"] * 32


def _count_launches(fn):
    """Our kernels (names starting msda_) launched by one call of fn, counted
    from a CUDA activity trace of an untimed call; None if tracing fails."""
    try:
        from torch.autograd import DeviceType
        from torch.profiler import ProfilerActivity, profile
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            fn()
            torch.cuda.synchronize()
        n = sum(1 for e in prof.events()
                if e.device_type == DeviceType.CUDA and "msda_" in e.name)
        return n if n > 0 else None
    except Exception:  # noqa: BLE001 - the trace is optional
        return None


def _bwd_launches(wl, ws_bytes):
    """Our kernel launches in one backward entry when no trace is available:
    the cell-sorted plan runs the dot-product kernel, three scan kernels, the
    placement kernel, the sorted-order dot products, the dense- and
    voxel-level value-gradient kernels and the accumulator cast; the
    gather/scatter plan the scatter kernel and (16-bit values) the cast."""
    if _bwd_plan_is_sorted(wl, ws_bytes):
        return 9
    return 1 + (1 if wl["dtype"] != torch.float32 and ws_bytes > 0 else 0)


def _bwd_entry_name(wl, ws_bytes):
    if _bwd_plan_is_sorted(wl, ws_bytes):
        return ("backward entry, cell-sorted (msda_dots_kernel + scan + msda_place_kernel + "
                "msda_sdots_kernel + msda_dense_kernel / msda_dense_mma_kernel + "
                "msda_voxel_mma_kernel / msda_voxel_kernel + cast)")
    return "backward entry, gather/scatter (zero-fill + msda_bwd_kernel + cast)"


class _Null:
    def __enter__(self):
        return self

    def __exit__(self, *exc):
        return False

    def summary(self):
        return None


def run_e2e(args, wl, fn, dev, shapes, value, loc, attn, go, fwd_only, dist):
    """Same metric through the public API with pinned HOST buffers.  Every
    step uploads its inputs and downloads all of its results (output and,
    for training, the three gradients) inside the timed region.  Steps run
    the way a streaming caller runs them: the upload of step i+1 (copy-in
    stream) and the download of step i-1 (copy-out stream) overlap the
    kernels of step i, with two device slots for the inputs; CUDA events
    order every copy against the compute that reads or writes its buffer."""
    n_in = 3 if fwd_only else 4
    # pinned host copies made directly (no pageable intermediate: 8 ranks on
    # one host each hold these)
    host_in = []
    for t in (value, loc, attn, go)[:n_in]:
        h = torch.empty(t.shape, dtype=t.dtype, pin_memory=True)
        h.copy_(t.detach())
        host_in.append(h)
    h2d = sum(t.numel() * t.element_size() for t in host_in)
    B, K, H, C, Q, L, P = dims(wl)
    outs_shape = [(B, Q, H * C)] + ([] if fwd_only else [tuple(value.shape), tuple(loc.shape),
                                                         tuple(attn.shape)])
    host_out = [torch.empty(s, dtype=wl["dtype"], pin_memory=True) for s in outs_shape]
    d2h = sum(t.numel() * t.element_size() for t in host_out)
    comp = torch.cuda.current_stream(dev)
    s_in = torch.cuda.Stream(dev)
    s_out = torch.cuda.Stream(dev)
    slots = [[torch.empty(t.shape, dtype=t.dtype, device=dev) for t in host_in] for _ in range(2)]
    slot_free = [torch.cuda.Event() for _ in range(2)]
    for e in slot_free:
        e.record(comp)

    def run(iters):
        s_in.wait_stream(comp)
        for i in range(iters):
            k = i % 2
            ev_in = torch.cuda.Event()
            with torch.cuda.stream(s_in):
                s_in.wait_event(slot_free[k])
                for d, h in zip(slots[k], host_in):
                    d.copy_(h, non_blocking=True)
                ev_in.record(s_in)
            comp.wait_event(ev_in)
            v, lo, a = (t.detach().requires_grad_(True) for t in slots[k][:3])
            out = fn(v, shapes, lo, a)
            res = [out]
            if not fwd_only:
                res += list(torch.autograd.grad(out, (v, lo, a), slots[k][3]))
            slot_free[k].record(comp)
            ev_c = torch.cuda.Event()
            ev_c.record(comp)
            with torch.cuda.stream(s_out):
                s_out.wait_event(ev_c)
                for h, r in zip(host_out, res):
                    h.copy_(r.detach(), non_blocking=True)
            for r in res:
                r.record_stream(s_out)
        comp.wait_stream(s_out)
        comp.wait_stream(s_in)

    iters = max(3, min(args.steps, 10))
    run(2)
    torch.cuda.synchronize(dev)
    if dist is not None:
        dist.barrier()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(comp)
    run(iters)
    t1.record(comp)
    torch.cuda.synchronize(dev)
    ms = t0.elapsed_time(t1) / iters
    if dist is not None:
        tt = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms = float(tt.item())
    world = dist.get_world_size() if dist is not None else 1
    samples = algorithmic_bytes(wl)["samples"] * world
    del host_in, host_out, slots
    return {"value": samples / (ms * 1e-3) / 1e9, "unit": "Gsamples/s", "ms_per_step": ms,
            "steps": iters, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "pipeline": "upload i+1 / compute i / download i-1 on three streams"}


# ---------------------------------------------------------------- reference Triton arm
REF_DIR = os.path.join(ROOT, "baseline", "_ref")


def load_reference_triton():
    """The unmodified reference package installed under baseline/_ref, or None."""
    if not os.path.isdir(os.path.join(REF_DIR, "msda_triton")):
        return None
    if REF_DIR not in sys.path:
        sys.path.insert(0, REF_DIR)
    import msda_triton

    return msda_triton


def run_reference_triton(args, wl, rank, world, local_rank):
    """The reference's own Triton kernels on this GPU through its public API
    (msda2d/msda3d with autograd), timed exactly like our arm: same inputs,
    same step, CUDA events, max over ranks.  Informational comparison point."""
    ref = load_reference_triton()
    if ref is None:
        return None if rank else {"impl": "reference-triton",
                                  "unavailable": "reference not installed under baseline/_ref"}
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    fn = ref.msda3d if wl["ndim"] == 3 else ref.msda2d
    global_b = wl["B"] * world
    if args.scaling == "strong" and world > 1 and wl["B"] % world == 0:
        global_b = wl["B"]
        wl = dict(wl, B=wl["B"] // world)
    value, shapes, loc, attn, go = make_inputs(wl, dev, seed=1234 + rank)
    v, lo, a = (t.requires_grad_(True) for t in (value, loc, attn))
    fwd_only = wl.get("fwd_only", False)
    stream = torch.cuda.current_stream(dev)

    def step():
        out = fn(v, shapes, lo, a)
        if not fwd_only:
            torch.autograd.grad(out, (v, lo, a), go)

    def fwd():
        with torch.no_grad():
            fn(v, shapes, lo, a)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    if dist is not None:
        dist.barrier()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for _ in range(args.steps):
        step()
    t1.record(stream)
    torch.cuda.synchronize(dev)
    ms = t0.elapsed_time(t1) / args.steps
    fwd_ms = statistics.mean(time_events(fwd, max(3, min(args.steps, 10)) + 2, stream)[2:])
    if dist is not None:
        tt = torch.tensor([ms, fwd_ms], device=dev, dtype=torch.float64)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms, fwd_ms = (float(x) for x in tt.tolist())
    e2e = run_e2e(args, wl, fn, dev, shapes, value, loc, attn, go, fwd_only, dist)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return None
    B, K, H, C, Q, L, P = dims(wl)
    samples = algorithmic_bytes(wl)["samples"] * world
    return {
        "impl": "reference-triton",
        "metric": "MSDA fwd+bwd Gsamples/s" if not fwd_only else "MSDA fwd Gsamples/s",
        "value": samples / (ms * 1e-3) / 1e9, "unit": "Gsamples/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "fwd_ms": fwd_ms,
        "higher_is_better": True, "scaling": "strong" if global_b == B else "weak",
        "vs_baseline": None,
        "dtype": DTYPE_NAME[wl["dtype"]], "data": "synthetic (same seeded inputs as our arm)",
        "config": {"workload": args.workload, "batch_per_gpu": B, "global_batch": global_b,
                   "num_queries": Q, "source": "unmodified reference from baseline/_ref "
                   "(msda_triton " + getattr(ref, "__version__", "0.1.0") + ")"},
        "e2e": e2e,
    }


# ---------------------------------------------------------------- query sharding
def run_query_sharded(args, wl, rank, world, local_rank):
    """BASELINE config 4 at a batch smaller than the GPU count: every rank holds
    the whole value and a block of the queries; the backward sums the fp32
    partial value gradients with an NCCL reduce-scatter and gathers the
    rounded shards (all-gather in value's dtype).  Total work is fixed
    (strong scaling); time is the max over ranks of CUDA-event times."""
    import datetime

    import torch.distributed as dist

    from msda_triton_b200.sharding import msda_query_sharded, query_shard

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    else:  # one rank: no collective, the rest of the path is the same
        dist.init_process_group("nccl", init_method="tcp://127.0.0.1:29533", rank=0,
                                world_size=1, timeout=datetime.timedelta(seconds=60),
                                device_id=dev)
    value, shapes, loc, attn, go = make_inputs(wl, dev, seed=1234)  # the same on every rank
    sl = query_shard(wl["Q"], rank, world)
    v = value.requires_grad_(True)
    lo = loc[:, sl].contiguous().requires_grad_(True)
    a = attn[:, sl].contiguous().requires_grad_(True)
    g = go[:, sl].contiguous()
    group = dist.group.WORLD

    def step():
        out = msda_query_sharded(wl["ndim"], v, shapes, lo, a, group=group,
                                 reduce_dtype=args.reduce_dtype)
        torch.autograd.grad(out, (v, lo, a), g)

    stream = torch.cuda.current_stream(dev)
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    dist.barrier()
    torch.cuda.synchronize(dev)
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for _ in range(args.steps):
        step()
    t1.record(stream)
    torch.cuda.synchronize(dev)
    ms = t0.elapsed_time(t1) / args.steps
    if world > 1:
        tt = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms = float(tt.item())
    dist.barrier()
    dist.destroy_process_group()
    if rank != 0:
        return None
    B, K, H, C, Q, L, P = dims(wl)
    samples = algorithmic_bytes(wl)["samples"]
    e = value.element_size()
    if args.reduce_dtype == "value":
        how = f"grad_value: one NCCL all_reduce of the partial gradients in {DTYPE_NAME[wl['dtype']]}"
        coll = 2 * B * K * H * C * e * (world - 1) // world
    else:
        how = ("grad_value: fp32 NCCL reduce-scatter + all-gather in the value dtype")
        coll = B * K * H * C * (4 + e) * (world - 1) // world
    return {"metric": "MSDA fwd+bwd Gsamples/s", "value": samples / (ms * 1e-3) / 1e9,
            "unit": "Gsamples/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": DTYPE_NAME[wl["dtype"]], "data": "synthetic (seeded)",
            "config": {"workload": args.workload, "batch": B, "num_queries": Q,
                       "parallelism": f"query-sharded over {world} GPU(s), value replicated; "
                                      + how,
                       "reduce_dtype": args.reduce_dtype,
                       "collective_bytes_per_rank": coll}}


# ---------------------------------------------------------------- module workloads
def run_module(args, wl, rank, world, local_rank):
    """One fwd+bwd step of the nn.Module (ours, or the reference's own module
    from baseline/_ref with --impl reference-triton) on one GPU: same seeded
    parameters (init_weights) and inputs for both; CUDA events."""
    if world > 1:
        raise SystemExit("module workloads run on one GPU")
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    if args.impl == "reference":
        return {"impl": "reference", "unavailable": "module workloads have no CPU arm"}
    if args.impl == "reference-triton":
        ref = load_reference_triton()
        if ref is None:
            return {"impl": "reference-module", "unavailable": "reference not installed under baseline/_ref"}
        from msda_triton.pytorch import MSDA2D, MSDA3D
        impl = "reference-module (grid_sample)"
    else:
        from msda_triton_b200.modules import MSDA2D, MSDA3D
        impl = "ours"
    B, K, H, C, Q, L, P = dims(wl)
    d, dt, E = wl["ndim"], wl["dtype"], H * C
    torch.manual_seed(0)
    kw = {} if impl != "ours" else {"fused_prologue": not args.module_unfused}
    m = (MSDA3D if d == 3 else MSDA2D)(embed_dims=E, num_heads=H, num_levels=L, num_points=P,
                                       dropout=0.0, batch_first=True, **kw)
    m.init_weights()
    m = m.to(dev, dt)
    g = torch.Generator(device=dev).manual_seed(1234)
    query = torch.randn(B, Q, E, generator=g, device=dev).to(dt).requires_grad_(True)
    value = torch.randn(B, K, E, generator=g, device=dev).to(dt).requires_grad_(True)
    refp = torch.rand(B, Q, L, d, generator=g, device=dev).to(dt).requires_grad_(True)
    gout = torch.randn(B, Q, E, generator=g, device=dev).to(dt)
    shapes = torch.tensor(wl["shapes"], dtype=torch.int64, device=dev)
    wrt = [query, value, refp] + list(m.parameters())

    def step():
        out = m(query, value=value, reference_points=refp, spatial_shapes=shapes)
        torch.autograd.grad(out, wrt, gout)

    stream = torch.cuda.current_stream(dev)
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    with ClockSampler([local_rank]) as clk:
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        for _ in range(args.steps):
            step()
        t1.record(stream)
        torch.cuda.synchronize(dev)
    ms = t0.elapsed_time(t1) / args.steps
    samples = algorithmic_bytes(wl)["samples"]
    return {"impl": impl, "metric": "MSDA module fwd+bwd Gsamples/s",
            "value": samples / (ms * 1e-3) / 1e9, "unit": "Gsamples/s", "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": DTYPE_NAME[dt], "data": "synthetic (seeded; init_weights parameters)",
            "config": {"workload": args.workload, "embed_dims": E, "batch": B, "num_queries": Q,
                       "num_keys": K, "num_heads": H, "num_levels": L, "num_points": P,
                       "prologue": ("unfused" if args.module_unfused else "fused")
                       if impl == "ours" else "reference"},
            "clocks": clk.summary()}


# ---------------------------------------------------------------- CPU arms
def _cpu_sample(wl, target_s, per_sample_us):
    """A bounded sample of the workload for the CPU: batch 1, and a query count
    that keeps one fwd+bwd near `target_s` seconds at `per_sample_us`
    microseconds per sample (measured for each implementation)."""
    B, K, H, C, Q, L, P = dims(wl)
    q = int(target_s * 1e6 / per_sample_us / (H * L * P))
    return dict(wl, B=1, Q=max(64, min(Q, q)))


def cpu_inputs(wl, seed=7):
    B, K, H, C, Q, L, P = dims(wl)
    d = wl["ndim"]
    g = torch.Generator().manual_seed(seed)
    value = torch.randn(B, K, H, C, generator=g)
    loc = torch.rand(B, Q, H, L, P, d, generator=g)
    attn = torch.randn(B, Q, H, L * P, generator=g).softmax(-1).view(B, Q, H, L, P)
    go = torch.randn(B, Q, H * C, generator=g)
    shapes = torch.tensor(wl["shapes"], dtype=torch.int64)
    return value, shapes, loc, attn, go


def _reference_pytorch():
    """msda{2,3}d_pytorch of the unmodified reference under baseline/_ref."""
    ref = load_reference_triton()
    if ref is None:
        return None
    from msda_triton.pytorch import msda2d_pytorch, msda3d_pytorch

    return {2: msda2d_pytorch, 3: msda3d_pytorch}


def cpu_step_reference(fns, wl, inputs):
    """One fp32 fwd(+bwd) of the reference's grid_sample path on the host."""
    value, shapes, loc, attn, go = inputs
    fwd_only = wl.get("fwd_only", False)
    v, lo, a = (t.detach().requires_grad_(not fwd_only) for t in (value, loc, attn))
    t = time.perf_counter()
    out = fns[wl["ndim"]](v, shapes, lo, a, True, 1e-4)
    if not fwd_only:
        torch.autograd.grad(out, (v, lo, a), go)
    return time.perf_counter() - t


def cpu_step_port(wl, inputs, nthreads):
    """One fwd(+bwd) of the C restatement (oracle/), the stand-in when the
    reference package is not installed."""
    from oracle import msda_bwd_oracle, msda_fwd_oracle

    value, shapes, loc, attn, go = (t.numpy() for t in inputs)
    t = time.perf_counter()
    msda_fwd_oracle(value, shapes, loc, attn, True, 1e-4, nthreads)
    if not wl.get("fwd_only", False):
        msda_bwd_oracle(value, shapes, loc, attn, go, True, 1e-4, nthreads)
    return time.perf_counter() - t


def cpu_measure(wl, steps, warmup, target_s):
    """Time the CPU implementation on a bounded sample: the reference's own
    msda*_pytorch when installed, else the C port.  Returns (seconds per
    pass list, sample workload, kind, threads)."""
    nthreads = os.cpu_count() or 1
    fns = _reference_pytorch()
    if fns is not None:
        torch.set_num_threads(nthreads)
        swl = _cpu_sample(wl, target_s, 0.8)
        inputs = cpu_inputs(swl)
        for _ in range(warmup):
            cpu_step_reference(fns, swl, inputs)
        ts = [cpu_step_reference(fns, swl, inputs) for _ in range(steps)]
        return ts, swl, "reference", torch.get_num_threads()
    swl = _cpu_sample(wl, target_s, 0.16)
    inputs = cpu_inputs(swl)
    for _ in range(warmup):
        cpu_step_port(swl, inputs, nthreads)
    ts = [cpu_step_port(swl, inputs, nthreads) for _ in range(steps)]
    return ts, swl, "port", nthreads


def _cpu_desc(kind, wl, swl, samples, steps, t):
    what = ("the reference's msda_triton.pytorch grid_sample path (baseline/_ref), fp32"
            if kind == "reference" else "fp32 C port of the reference path (oracle/, OpenMP)")
    return (f"{what}, fwd{'' if wl.get('fwd_only') else '+bwd'} on batch 1, Q={swl['Q']} "
            f"({samples} samples), median of {steps} after 1 warm-up; {t:.2f} s per pass")


def cpu_baseline(args, wl, steps=3, target_s=3.0):
    ts, swl, kind, cores = cpu_measure(wl, steps, 1, target_s)
    t = statistics.median(ts)
    samples = algorithmic_bytes(swl)["samples"]
    return {"value": samples / t / 1e9, "unit": "Gsamples/s", "cores": cores, "kind": kind,
            "sample": _cpu_desc(kind, wl, swl, samples, steps, t)}


def run_reference(args, wl, rank):
    if rank != 0:
        return None
    ts, swl, kind, cores = cpu_measure(wl, args.steps, args.warmup, 2.0)
    t = statistics.median(ts)
    samples = algorithmic_bytes(swl)["samples"]
    val = samples / t / 1e9
    fwd_only = wl.get("fwd_only", False)
    return {
        "impl": "reference",
        "metric": "MSDA fwd+bwd Gsamples/s" if not fwd_only else "MSDA fwd Gsamples/s",
        "value": val, "unit": "Gsamples/s", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": t * 1e3, "higher_is_better": True,
        "scaling": args.scaling,
        "vs_baseline": None, "dtype": "fp32", "data": "synthetic (seeded)",
        "config": {"workload": args.workload, "ndim": wl["ndim"], "batch_per_gpu": 1,
                   "num_queries": swl["Q"], "note": "bounded CPU sample of the workload"},
        "cpu_baseline": {"value": val, "unit": "Gsamples/s", "cores": cores, "kind": kind,
                         "sample": _cpu_desc(kind, wl, swl, samples, args.steps, t)},
        "e2e": {"value": val, "unit": "Gsamples/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--workload", default="3d_xl_bf16", choices=sorted(WORKLOADS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference", "reference-triton"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--module-unfused", action="store_true",
                    help="module workloads: form locations and weights with torch ops and call "
                         "msda2d/msda3d (fused_prologue=False)")
    ap.add_argument("--value-layout", default="bkhc", choices=["bkhc", "bhkc"],
                    help="device-resident value of the timed step: the reference's (B, K, H, C) "
                         "or head-major (B, H, K, C) storage (end-to-end leg: always bkhc)")
    ap.add_argument("--shard", default="batch", choices=["batch", "query"],
                    help="batch: one instance of the workload per GPU (weak scaling); query: "
                         "one instance split by queries across the GPUs (strong scaling)")
    ap.add_argument("--reduce-dtype", default="float32", choices=["float32", "value"],
                    help="--shard query: sum the partial value gradients in fp32 (reduce-scatter "
                         "+ all-gather, one rounding) or in the value dtype (one all_reduce)")
    ap.add_argument("--scaling", default="strong", choices=["strong", "weak"],
                    help="--gpus N: split the workload's batch over the GPUs (strong) or give "
                         "every GPU the whole batch (weak)")
    ap.add_argument("--batch", type=int, default=0,
                    help="per-GPU batch override (a smaller case of the workload, for profiling)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    wl = dict(WORKLOADS[args.workload])
    if args.batch > 0:
        wl["B"] = args.batch
    if args.shard == "query" and args.impl == "ours" and not wl.get("module"):
        res = run_query_sharded(args, wl, rank, world, local_rank)
    elif wl.get("module"):
        res = run_module(args, wl, rank, world, local_rank) if rank == 0 else None
    elif args.impl == "reference":
        res = run_reference(args, wl, rank)
    elif args.impl == "reference-triton":
        res = run_reference_triton(args, wl, rank, world, local_rank)
    else:
        if args.no_cpu_baseline:
            globals()["cpu_baseline"] = lambda *a, **k: None
        res = run_ours(args, wl, rank, world, local_rank)
    if res is not None:
        print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()
