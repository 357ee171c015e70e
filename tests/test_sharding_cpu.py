"""Multi-process (gloo, world size 2, CPU) tests of the sharding host logic.

The compute is injected: a CPU backend built on the oracle stands in for the
CUDA kernels, so these tests check what the sharding layer itself does --
query/batch partition, the fp32 reduce-scatter and all-gather of the partial
value gradients,
gradient routing through autograd -- against a single-process oracle run.
They also check that a rank that disappears turns into an error on the
surviving rank (process-group timeout), not a hang.
"""

from __future__ import annotations

import datetime
import os
import socket
import traceback

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from msda_triton_b200.sharding import batch_shard, msda_query_sharded, query_shard
from oracle import msda_bwd_oracle, msda_fwd_oracle
from tests._util import make_inputs


class OracleBackend:
    """Test-only CPU compute with the CudaBackend interface."""

    @staticmethod
    def prepare(ndim, value, shapes, loc, attn):
        return value.contiguous(), shapes, False, loc.contiguous(), attn.contiguous()

    @staticmethod
    def forward(ndim, value, shapes, on_dev, loc, attn, clamp, eps):
        return torch.from_numpy(msda_fwd_oracle(value.detach().numpy(), shapes.numpy(),
                                                loc.detach().numpy(), attn.detach().numpy(),
                                                clamp, eps))

    @staticmethod
    def backward(ndim, value, shapes, on_dev, loc, attn, clamp, eps, go):
        gv, gl, ga = msda_bwd_oracle(value.detach().numpy(), shapes.numpy(),
                                     loc.detach().numpy(), attn.detach().numpy(),
                                     go.detach().numpy(), clamp, eps)
        return (torch.from_numpy(gv).to(value.dtype), torch.from_numpy(gl),
                torch.from_numpy(ga))

    @staticmethod
    def backward_accumulate(ndim, value, shapes, on_dev, loc, attn, clamp, eps, go, acc):
        gv, gl, ga = msda_bwd_oracle(value.detach().numpy(), shapes.numpy(),
                                     loc.detach().numpy(), attn.detach().numpy(),
                                     go.detach().numpy(), clamp, eps)
        acc += torch.from_numpy(gv)
        return torch.from_numpy(gl), torch.from_numpy(ga)

    @staticmethod
    def cast(acc, dtype):
        return acc.to(dtype)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, timeout_s=60):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))


def _query_sharded_worker(rank, world, port, ndim, reduce_dtype, q):
    try:
        _init(rank, world, port)
        shapes = [(12, 20), (6, 10)] if ndim == 2 else [(6, 8, 10), (3, 4, 5)]
        B, Q, H, C, P = 1, 37, 4, 16, 4
        value, shp, loc, attn, go = make_inputs(B, Q, H, C, P, shapes, seed=21)
        sl = query_shard(Q, rank, world)
        v = value.clone().requires_grad_(True)
        lo = loc[:, sl].clone().requires_grad_(True)
        a = attn[:, sl].clone().requires_grad_(True)
        out = msda_query_sharded(ndim, v, shp, lo, a, backend=OracleBackend,
                                 reduce_dtype=reduce_dtype)
        out.backward(go[:, sl])
        # Reference: the whole problem in one process.
        ref_out = msda_fwd_oracle(value, shp, loc, attn)
        ref_gv, ref_gl, ref_ga = msda_bwd_oracle(value, shp, loc, attn, go)
        np.testing.assert_allclose(out.detach().numpy(), ref_out[:, sl], rtol=1e-6, atol=1e-6)
        np.testing.assert_allclose(v.grad.numpy(), ref_gv, rtol=1e-5, atol=1e-6)
        np.testing.assert_allclose(lo.grad.numpy(), ref_gl[:, sl], rtol=1e-6, atol=1e-6)
        np.testing.assert_allclose(a.grad.numpy(), ref_ga[:, sl], rtol=1e-6, atol=1e-6)
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, "ok"))
    except Exception:  # report to the parent instead of dying silently
        q.put((rank, traceback.format_exc()))


def _run(target, args, world=2, timeout=120):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, world, port, *args, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        rank, msg = q.get(timeout=timeout)
        results[rank] = msg
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    return results


@pytest.mark.parametrize("reduce_dtype", ["float32", "value"])
@pytest.mark.parametrize("ndim", [2, 3])
def test_query_sharded_matches_single_process(ndim, reduce_dtype):
    # fp32 values: both reductions sum fp32 partials, so both match one process
    results = _run(_query_sharded_worker, (ndim, reduce_dtype))
    assert results == {0: "ok", 1: "ok"}, results


def test_query_sharded_rejects_unknown_reduce_dtype():
    with pytest.raises(ValueError, match="reduce_dtype"):
        msda_query_sharded(3, torch.zeros(1), None, None, None, reduce_dtype="fp8")


def test_shard_slices_cover_everything():
    for n in (0, 1, 7, 100, 19947):
        for world in (1, 2, 3, 8):
            parts = [query_shard(n, r, world) for r in range(world)]
            assert parts[0].start == 0 and parts[-1].stop == n
            assert all(a.stop == b.start for a, b in zip(parts, parts[1:]))
            sizes = [p.stop - p.start for p in parts]
            assert max(sizes) - min(sizes) <= 1
            assert batch_shard(n, 0, world) == parts[0]
    with pytest.raises(ValueError):
        query_shard(10, 2, 2)


def _report_and_exit(q, rank, msg):
    # Flush the queue's feeder thread before the hard exit, or the message is lost.
    q.put((rank, msg))
    q.close()
    q.join_thread()
    os._exit(0)


def _lost_rank_worker(rank, world, port, q):
    try:
        _init(rank, world, port, timeout_s=5)
        shapes = [(8, 8)]
        value, shp, loc, attn, go = make_inputs(1, 10, 2, 8, 2, shapes, seed=3)
        sl = query_shard(10, rank, world)
        v = value.clone().requires_grad_(True)
        out = msda_query_sharded(2, v, shp, loc[:, sl], attn[:, sl], backend=OracleBackend)
        if rank == 1:
            # This rank fails between steps: it never joins the backward's
            # collectives and exits.
            _report_and_exit(q, rank, "left")
        try:
            out.backward(go[:, sl])
        except Exception as exc:  # the surviving rank must see an error, not hang
            _report_and_exit(q, rank, f"error: {type(exc).__name__}")
        _report_and_exit(q, rank, "no error")
    except Exception:
        q.put((rank, traceback.format_exc()))


def test_lost_rank_surfaces_as_error():
    results = _run(_lost_rank_worker, (), timeout=90)
    assert results[1] == "left"
    assert results[0].startswith("error"), results[0]
