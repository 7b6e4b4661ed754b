"""Differentiable row collectives of tensor + sequence parallelism.

Under sequence parallelism each rank of a tensor-parallel group holds a contiguous block of
the token rows of the residual stream. Entering a tensor-parallel region gathers the rows
(all-gather; its backward is a reduce-scatter of the gradient), and leaving one sums the
partial outputs of the ranks and hands each rank its rows back (reduce-scatter; its backward
is an all-gather). NCCL runs both as single calls; on gloo (CPU tests), which has no
reduce-scatter, the reduce-scatter is an all-reduce followed by taking this rank's rows.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def _gloo(group) -> bool:
    return dist.get_backend(group) == "gloo"


def all_gather_rows(x: torch.Tensor, group) -> torch.Tensor:
    world = dist.get_world_size(group)
    x = x.contiguous()
    out = torch.empty((x.shape[0] * world,) + tuple(x.shape[1:]), dtype=x.dtype, device=x.device)
    if _gloo(group):
        dist.all_gather(list(out.chunk(world, 0)), x, group=group)
    else:
        dist.all_gather_into_tensor(out, x, group=group)
    return out


def reduce_scatter_rows(x: torch.Tensor, group) -> torch.Tensor:
    world = dist.get_world_size(group)
    x = x.contiguous()
    if x.shape[0] % world:
        raise ValueError(f"reduce_scatter_rows: {x.shape[0]} rows do not split over {world} ranks")
    if _gloo(group):
        y = x.clone()
        dist.all_reduce(y, group=group)
        return y.chunk(world, 0)[dist.get_rank(group)].contiguous()
    out = torch.empty((x.shape[0] // world,) + tuple(x.shape[1:]), dtype=x.dtype, device=x.device)
    dist.reduce_scatter_tensor(out, x, group=group)
    return out


class AllGatherRows(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        return all_gather_rows(x, group)

    @staticmethod
    def backward(ctx, g):
        return reduce_scatter_rows(g, ctx.group), None


class ReduceScatterRows(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        return reduce_scatter_rows(x, group)

    @staticmethod
    def backward(ctx, g):
        return all_gather_rows(g, ctx.group), None


def gather_rows(x, group):
    return AllGatherRows.apply(x, group) if group is not None else x


def scatter_rows(x, group):
    return ReduceScatterRows.apply(x, group) if group is not None else x
