"""Process-group layout for data x pipeline x tensor parallelism.

Ranks are numbered with tensor parallelism innermost, then pipeline, then data parallelism:
    rank = (dp_rank * pp + pp_rank) * tp + tp_rank
the same order the reference's workload export uses (workload_export/export_trace.py:120-122
`rank_of`), so a tensor-parallel group is a run of adjacent ranks (one NVSwitch hop apart on
one node either way, and the groups that move the most bytes share a node first when the job
spans nodes).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch.distributed as dist


def rank_of(dp_rank: int, pp_rank: int, tp_rank: int, pp: int, tp: int) -> int:
    return (dp_rank * pp + pp_rank) * tp + tp_rank


def coords_of(rank: int, pp: int, tp: int):
    """(dp_rank, pp_rank, tp_rank) of a global rank."""
    return rank // (pp * tp), (rank // tp) % pp, rank % tp


@dataclass
class Layout:
    dp: int = 1
    tp: int = 1
    pp: int = 1

    @property
    def world(self) -> int:
        return self.dp * self.tp * self.pp

    def tp_ranks(self, dp_rank, pp_rank):
        return [rank_of(dp_rank, pp_rank, t, self.pp, self.tp) for t in range(self.tp)]

    def dp_ranks(self, pp_rank, tp_rank):
        return [rank_of(d, pp_rank, tp_rank, self.pp, self.tp) for d in range(self.dp)]

    def pp_ranks(self, dp_rank, tp_rank):
        return [rank_of(dp_rank, p, tp_rank, self.pp, self.tp) for p in range(self.pp)]


class ParallelGroups:
    """This rank's coordinates and its tp / pp / dp process groups (None when that degree is 1).

    Every rank creates every group in the same order, as torch.distributed requires."""

    def __init__(self, layout: Layout, rank: int | None = None, backend: str | None = None):
        self.layout = layout
        world = dist.get_world_size() if dist.is_initialized() else 1
        if layout.world != world:
            raise ValueError(f"layout dp{layout.dp} x pp{layout.pp} x tp{layout.tp} needs {layout.world} ranks, "
                             f"the job has {world}")
        self.rank = dist.get_rank() if rank is None and dist.is_initialized() else (rank or 0)
        self.dp_rank, self.pp_rank, self.tp_rank = coords_of(self.rank, layout.pp, layout.tp)
        self.tp_group = self.pp_group = self.dp_group = None
        if world == 1:
            return
        kw = {"backend": backend} if backend else {}
        for d in range(layout.dp):
            for p in range(layout.pp):
                ranks = layout.tp_ranks(d, p)
                g = dist.new_group(ranks, **kw) if layout.tp > 1 else None
                if self.rank in ranks:
                    self.tp_group = g
        for d in range(layout.dp):
            for t in range(layout.tp):
                ranks = layout.pp_ranks(d, t)
                g = dist.new_group(ranks, **kw) if layout.pp > 1 else None
                if self.rank in ranks:
                    self.pp_group = g
                    self.pp_global_ranks = ranks
        for p in range(layout.pp):
            for t in range(layout.tp):
                ranks = layout.dp_ranks(p, t)
                g = dist.new_group(ranks, **kw) if layout.dp > 1 else None
                if self.rank in ranks:
                    self.dp_group = g

    @property
    def tp(self):
        return self.layout.tp

    @property
    def pp(self):
        return self.layout.pp

    @property
    def dp(self):
        return self.layout.dp
