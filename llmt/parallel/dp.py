"""Data parallelism with a ZeRO-1 sharded optimizer over the flat parameter buffers.

The reference has no multi-GPU code: it only models a ring all-reduce of fp32 gradients
(perf_model/scaling.py:163-167) and a ZeRO-1 optimizer (scaling.py:24-25, :169-170).
Here it runs. Per step, after the backward:

  1. reduce-scatter the flat fp32 gradient buffer -> this rank's shard, averaged over ranks
  2. AdamW on the shard only (fp32 master shard + exp_avg/exp_avg_sq shards), which also
     writes the shard of the bf16 shadow weights
  3. all-gather the bf16 shadow shards -> every rank has the full bf16 weights for the next
     forward (this is the bf16 "parameter all-gather"; fp32 masters stay sharded)

Two transports, same math:
  mode="nccl"   NCCL reduce_scatter_tensor / all_gather_into_tensor (the baseline path);
  mode="fused"  one sm_100a kernel per step over NVLink peer memory that reads every peer's
                gradient shard, sums, applies AdamW and stores the new bf16 shard into every
                peer's shadow buffer (llmt.parallel.fused_dp), with bounded device-side waits.

Every rank takes the same collective steps in the same order (warm-up, capture and replay).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from llmt.ops import native as N


class ShardedAdamW:
    """AdamW state for one contiguous shard [lo, hi) of the flat buffers."""

    def __init__(self, flat, lo, hi, lr=3e-4, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1, grad_scale=1.0):
        self.flat, self.lo, self.hi = flat, lo, hi
        dev = flat.master.device
        self.exp_avg = torch.zeros(hi - lo, dtype=torch.float32, device=dev)
        self.exp_avg_sq = torch.zeros(hi - lo, dtype=torch.float32, device=dev)
        self.grad_shard = torch.zeros(hi - lo, dtype=torch.float32, device=dev)
        self.lr_t = torch.full((1,), float(lr), dtype=torch.float32, device=dev)
        self.step_t = torch.zeros(1, dtype=torch.int32, device=dev)
        self.betas, self.eps, self.weight_decay, self.grad_scale = betas, eps, weight_decay, grad_scale

    def set_lr(self, lr):
        self.lr_t.fill_(float(lr))

    @torch.no_grad()
    def step_local(self):
        f = self.flat
        self.step_t.add_(1)
        N.adamw_step(f.master[self.lo:self.hi], self.grad_shard, self.exp_avg, self.exp_avg_sq,
                     f.shadow[self.lo:self.hi], self.lr_t, self.step_t, self.betas[0], self.betas[1], self.eps,
                     self.weight_decay, self.grad_scale)


class DataParallel:
    def __init__(self, world_size: int, rank: int, mode: str = "nccl", group=None):
        self.world_size, self.rank, self.mode, self.group = world_size, rank, mode, group
        self.flat = None
        self.fused = None

    def make_optimizer(self, flat, lr=3e-4, **kw):
        if flat.numel % self.world_size:
            raise ValueError("flat buffer must be padded to a multiple of the world size")
        shard = flat.numel // self.world_size
        self.flat = flat
        lo, hi = self.rank * shard, (self.rank + 1) * shard
        opt = ShardedAdamW(flat, lo, hi, lr=lr, grad_scale=1.0 / self.world_size, **kw)
        # all ranks start from rank 0's weights (the same seed already makes them equal; this
        # makes it a guarantee)
        src = dist.get_global_rank(self.group, 0) if self.group is not None else 0
        dist.broadcast(flat.master, src, group=self.group)
        flat.refresh_shadow()
        if self.mode == "fused":
            from llmt.parallel.fused_dp import FusedDP
            self.fused = FusedDP(flat, opt, self.rank, self.world_size, self.group)
        return opt

    @torch.no_grad()
    def reduce_and_step(self, opt: ShardedAdamW):
        f = self.flat
        if self.fused is not None:
            self.fused.step()
            return
        dist.reduce_scatter_tensor(opt.grad_shard, f.grad, op=dist.ReduceOp.SUM, group=self.group)
        f.grad.zero_()  # gradients accumulate into the flat buffer
        opt.step_local()
        dist.all_gather_into_tensor(f.shadow, f.shadow[opt.lo:opt.hi].clone(), group=self.group)

    def close(self):
        if self.fused is not None:
            self.fused.close()
            self.fused = None
