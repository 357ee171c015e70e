"""Multi-GPU partitioning of the MSDA op (one process per GPU, torch.distributed).

Two partitions of the same op, following the data each rank holds:

* batch sharding -- the batch entries of value / sampling_locations /
  attention_weights are split across ranks.  Batch entries are independent,
  so each rank simply calls msda{2,3}d on its slice: no communication at all
  (`batch_shard` gives the slice).

* query sharding -- for batches smaller than the GPU count.  Every rank holds
  the full `value` (replicated) and the sampling_locations /
  attention_weights of its own contiguous block of queries
  (`query_shard`).  The forward is local (the output is query-sharded like
  the inputs).  In the backward, grad_sampling_locations and
  grad_attention_weights are local, while grad_value is a partial sum on
  every rank: each rank accumulates its part in fp32, a reduce-scatter (NCCL
  over NVLink on GPUs) leaves each rank the fp32 sum of one 1/N shard, the
  rank rounds its shard to value's dtype once, and an all-gather in that
  dtype gives every rank the full grad_value.  For 16-bit values that moves
  3/4 of an fp32 all_reduce's bytes with the same single rounding.
  With reduce_dtype="value" each rank instead runs the single-GPU backward
  (16-bit levels reduce in value's dtype there, busier levels in fp32 rounded
  once) and one all_reduce in value's dtype sums the partial gradients:
  2/3 of the default's bytes for 16-bit values, at the cost of up to one
  rounding per rank instead of one in total.

The reference has no multi-GPU code; this module implements the data-parallel
partition its tensor contract allows.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from msda_triton_b200 import _core


def _split(n: int, rank: int, world_size: int) -> slice:
    if world_size < 1 or not 0 <= rank < world_size:
        raise ValueError(f"bad rank {rank} for world size {world_size}")
    base, extra = divmod(n, world_size)
    start = rank * base + min(rank, extra)
    return slice(start, start + base + (1 if rank < extra else 0))


def batch_shard(batch: int, rank: int, world_size: int) -> slice:
    """Contiguous, balanced slice of the batch owned by `rank`."""
    return _split(batch, rank, world_size)


def query_shard(num_queries: int, rank: int, world_size: int) -> slice:
    """Contiguous, balanced slice of the queries owned by `rank`."""
    return _split(num_queries, rank, world_size)


class CudaBackend:
    """The library's kernels (the only backend the product uses)."""

    @staticmethod
    def prepare(ndim, value, shapes, loc, attn):
        _core.validate_inputs(ndim, value, shapes, loc, attn)
        shp, on_dev = _core.prepare_spatial(shapes)
        loc_p, attn_p = _core.sampling_pair(value, loc, attn)
        return value.contiguous(), shp, on_dev, loc_p, attn_p

    forward = staticmethod(_core.forward)
    backward = staticmethod(_core.backward)
    backward_accumulate = staticmethod(_core.backward_accumulate)
    cast = staticmethod(_core.cast_from_f32)


REDUCE_DTYPES = ("float32", "value")


class _QueryShardedFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, value, value_spatial_shapes, sampling_locations, attention_weights,
                clamp_grid, clamp_eps, ndim, group, backend, reduce_dtype):
        value_c, shp, on_dev, loc, attn = backend.prepare(
            ndim, value, value_spatial_shapes, sampling_locations, attention_weights)
        out = backend.forward(ndim, value_c, shp, on_dev, loc, attn, clamp_grid, clamp_eps)
        ctx.save_for_backward(value_c, loc, attn, shp)
        ctx.meta = (ndim, on_dev, clamp_grid, clamp_eps, group, backend,
                    sampling_locations.dtype, attention_weights.dtype, reduce_dtype)
        return out

    @staticmethod
    def backward(ctx, grad_output):
        value, loc, attn, shp = ctx.saved_tensors
        ndim, on_dev, clamp_grid, clamp_eps, group, backend, loc_dt, attn_dt, rdt = ctx.meta
        world = dist.get_world_size(group)
        if rdt == "value":
            # partial gradients in value's dtype, summed by one all_reduce
            grad_value, grad_loc, grad_attn = backend.backward(
                ndim, value, shp, on_dev, loc, attn, clamp_grid, clamp_eps, grad_output)
            if world > 1:
                dist.all_reduce(grad_value, op=dist.ReduceOp.SUM, group=group)
            return (grad_value, None, grad_loc.to(loc_dt), grad_attn.to(attn_dt),
                    None, None, None, None, None, None)
        n = value.numel()
        pad = (-n) % world
        acc_flat = torch.zeros(n + pad, device=value.device, dtype=torch.float32)
        acc = acc_flat[:n].view(value.shape)
        grad_loc, grad_attn = backend.backward_accumulate(
            ndim, value, shp, on_dev, loc, attn, clamp_grid, clamp_eps, grad_output, acc)
        if world == 1:
            grad_value = backend.cast(acc, value.dtype)
        else:
            # The collectives of the query-sharded backward: the fp32 sum of
            # the partial value gradients lands shard by shard (one shard per
            # rank), each rank rounds its shard, and the rounded shards are
            # gathered on every rank.
            shard = torch.empty((n + pad) // world, device=value.device, dtype=torch.float32)
            dist.reduce_scatter_tensor(shard, acc_flat, op=dist.ReduceOp.SUM, group=group)
            shard_v = backend.cast(shard, value.dtype)
            full = torch.empty(n + pad, device=value.device, dtype=value.dtype)
            dist.all_gather_into_tensor(full, shard_v.contiguous(), group=group)
            grad_value = full[:n].view(value.shape)
        if grad_loc.dtype != loc_dt:
            grad_loc = grad_loc.to(loc_dt)
        if grad_attn.dtype != attn_dt:
            grad_attn = grad_attn.to(attn_dt)
        return grad_value, None, grad_loc, grad_attn, None, None, None, None, None, None


def msda_query_sharded(ndim, value, value_spatial_shapes, sampling_locations,
                       attention_weights, clamp_grid=True, clamp_eps=1e-4, group=None,
                       backend=CudaBackend, reduce_dtype="float32"):
    """MSDA over this rank's queries with a replicated `value`.

    sampling_locations / attention_weights hold only this rank's block of
    queries (see `query_shard`); the result is this rank's block of the
    output.  Gradients: grad_value is summed over all ranks of `group` (an
    fp32 reduce-scatter, then an all-gather in value's dtype; with
    reduce_dtype="value", one all_reduce of value-dtype partials), the other
    gradients stay local.  Every rank must call
    this (and its backward) in the same order, as for any collective.
    """
    if ndim not in (2, 3):
        raise ValueError("ndim must be 2 or 3")
    if reduce_dtype not in REDUCE_DTYPES:
        raise ValueError(f"reduce_dtype must be one of {REDUCE_DTYPES}, got {reduce_dtype!r}")
    if not dist.is_available() or not dist.is_initialized():
        raise RuntimeError("msda query sharding needs an initialised torch.distributed group")
    return _QueryShardedFn.apply(value, value_spatial_shapes, sampling_locations,
                                 attention_weights, clamp_grid, clamp_eps, ndim, group, backend,
                                 reduce_dtype)


def msda2d_query_sharded(value, value_spatial_shapes, sampling_locations, attention_weights,
                         clamp_grid=True, clamp_eps=1e-4, group=None, reduce_dtype="float32"):
    """2D MSDA with queries sharded across the ranks of `group` (see module doc)."""
    return msda_query_sharded(2, value, value_spatial_shapes, sampling_locations,
                              attention_weights, clamp_grid, clamp_eps, group,
                              reduce_dtype=reduce_dtype)


def msda3d_query_sharded(value, value_spatial_shapes, sampling_locations, attention_weights,
                         clamp_grid=True, clamp_eps=1e-4, group=None, reduce_dtype="float32"):
    """3D MSDA with queries sharded across the ranks of `group` (see module doc)."""
    return msda_query_sharded(3, value, value_spatial_shapes, sampling_locations,
                              attention_weights, clamp_grid, clamp_eps, group,
                              reduce_dtype=reduce_dtype)


__all__ = ["batch_shard", "query_shard", "msda2d_query_sharded", "msda3d_query_sharded",
           "msda_query_sharded", "CudaBackend"]
