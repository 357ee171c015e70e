"""Multi-GPU runs of the CUDA path (NCCL, one process per GPU): needs >= 2 GPUs.

* query sharding: every rank holds the whole value and a block of queries;
  its output block, its location/weight gradient block and the reduced
  value gradient must match one single-GPU run of the whole problem;
* batch sharding: independent slices -- the concatenated outputs equal the
  single-GPU run bitwise.
"""

from __future__ import annotations

import datetime
import os
import socket
import traceback

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

WORLD = 2


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, ndim, dtype_name, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port),
                          NCCL_NVLS_ENABLE="0")
        dev = torch.device("cuda", rank)
        torch.cuda.set_device(dev)
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                                timeout=datetime.timedelta(seconds=60))
        import msda_triton_b200 as M
        from msda_triton_b200.sharding import batch_shard, msda_query_sharded, query_shard
        from tests._util import make_inputs

        dtype = getattr(torch, dtype_name)
        shapes = [(40, 60), (20, 30), (10, 15)] if ndim == 2 else [(16, 24, 24), (8, 12, 12)]
        B, Q, H, C, P = 2, 1001, 8, 32, 4
        value, shp, loc, attn, go = make_inputs(B, Q, H, C, P, shapes, seed=77, dtype=dtype,
                                                device=dev)
        fn = M.msda3d if ndim == 3 else M.msda2d
        # single-GPU reference on this rank's GPU
        v = value.clone().requires_grad_(True)
        lo = loc.clone().requires_grad_(True)
        a = attn.clone().requires_grad_(True)
        out_ref = fn(v, shp, lo, a)
        gv_ref, gl_ref, ga_ref = torch.autograd.grad(out_ref, (v, lo, a), go)

        # query sharding
        sl = query_shard(Q, rank, world)
        v2 = value.clone().requires_grad_(True)
        lo2 = loc[:, sl].clone().requires_grad_(True)
        a2 = attn[:, sl].clone().requires_grad_(True)
        out = msda_query_sharded(ndim, v2, shp, lo2, a2)
        gv, gl, ga = torch.autograd.grad(out, (v2, lo2, a2), go[:, sl])
        tol = 1e-5 if dtype == torch.float32 else 2e-2
        assert torch.equal(out, out_ref[:, sl]), "query-sharded forward differs"
        torch.testing.assert_close(gl, gl_ref[:, sl], rtol=tol, atol=tol)
        torch.testing.assert_close(ga, ga_ref[:, sl], rtol=tol, atol=tol)
        torch.testing.assert_close(gv.float(), gv_ref.float(), rtol=tol, atol=tol)

        # query sharding, partial value gradients in value's dtype summed by
        # one all_reduce: the same bar (one extra rounding per rank)
        v3 = value.clone().requires_grad_(True)
        lo3 = loc[:, sl].clone().requires_grad_(True)
        a3 = attn[:, sl].clone().requires_grad_(True)
        out3 = msda_query_sharded(ndim, v3, shp, lo3, a3, reduce_dtype="value")
        gv3, gl3, ga3 = torch.autograd.grad(out3, (v3, lo3, a3), go[:, sl])
        assert torch.equal(out3, out_ref[:, sl]), "query-sharded forward differs"
        torch.testing.assert_close(gl3, gl_ref[:, sl], rtol=tol, atol=tol)
        torch.testing.assert_close(ga3, ga_ref[:, sl], rtol=tol, atol=tol)
        torch.testing.assert_close(gv3.float(), gv_ref.float(), rtol=tol, atol=tol)

        # batch sharding: each rank runs its slice; gather and compare bitwise
        bs = batch_shard(B, rank, world)
        out_b = fn(value[bs], shp, loc[bs], attn[bs])
        parts = [torch.empty_like(out_ref[batch_shard(B, r, world)]) for r in range(world)]
        dist.all_gather(parts, out_b.contiguous())
        assert torch.equal(torch.cat(parts), out_ref.detach()), "batch-sharded forward differs"

        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, "ok"))
    except Exception:
        q.put((rank, traceback.format_exc()))


@pytest.mark.parametrize("ndim,dtype_name", [(2, "float32"), (3, "bfloat16")])
def test_query_and_batch_sharding_nccl(ndim, dtype_name):
    if torch.cuda.device_count() < WORLD:
        pytest.skip(f"needs {WORLD} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, WORLD, port, ndim, dtype_name, q))
             for r in range(WORLD)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=300) for _ in range(WORLD))
    for p in procs:
        p.join(timeout=60)
    assert results == {r: "ok" for r in range(WORLD)}, results
