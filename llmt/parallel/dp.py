"""Data parallelism with a ZeRO-1 sharded optimizer over the flat parameter buffers.

The reference has no multi-GPU code: it only models a ring all-reduce of fp32 gradients
(perf_model/scaling.py:163-167) and a ZeRO-1 optimizer (scaling.py:24-25, :169-170).
Here it runs. Per step, after the backward:

  1. reduce-scatter the flat fp32 gradient buffer -> this rank's shard, averaged over ranks
  2. AdamW on the shard only (fp32 master shard + exp_avg/exp_avg_sq shards), which also
     writes the shard of the bf16 shadow weights
  3. all-gather the bf16 shadow shards -> every rank has the full bf16 weights for the next
     forward (this is the bf16 "parameter all-gather"; fp32 masters stay sharded)

Transports, same math:
  mode="nvls"   the gradient cast to bf16, then one sm_100a kernel that reduces this rank's
                shard inside the NVSwitch (multimem.ld_reduce), applies AdamW and multicasts the
                new bf16 weights to every rank (multimem.st) (llmt.parallel.nvls_dp);
  mode="fused"  one sm_100a kernel per step over NVLink peer memory that reads every peer's
                fp32 gradient shard, sums, applies AdamW and stores the new bf16 shard into
                every peer's shadow buffer (llmt.parallel.fused_dp), with bounded device-side waits;
  mode="nccl"   NCCL reduce_scatter_tensor / all_gather_into_tensor (the baseline path).
"nvls-overlap" and "fused-overlap" run their kernel per bucket on a side stream while the backward
of the earlier blocks computes (bucket-sharded optimizer state).

Every rank takes the same collective steps in the same order (warm-up, capture and replay).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from llmt.ops import native as N


def pick_mode(mode: str, device_index: int) -> str:
    """"auto" -> "nvls" when the device supports NVLink multicast (every rank of one box answers
    the same), else "nccl"; any other mode is returned as given."""
    if mode != "auto":
        return mode
    try:
        import torch.distributed._symmetric_memory as symm
        ok = symm._SymmetricMemory.has_multicast_support(torch._C._autograd.DeviceType.CUDA, device_index)
    except Exception:  # noqa: BLE001 - no symmetric memory in this build
        ok = False
    return "nvls" if ok else "nccl"


class ShardedAdamW:
    """AdamW state for one contiguous shard [lo, hi) of the flat buffers. grad_shard (the
    reduce-scatter output) only exists for the NCCL transport; the fused kernels read the
    gradients where the backward left them."""

    def __init__(self, flat, lo, hi, lr=3e-4, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1, grad_scale=1.0,
                 grad_shard=True):
        self.flat, self.lo, self.hi = flat, lo, hi
        dev = flat.master.device
        self.exp_avg = torch.zeros(hi - lo, dtype=torch.float32, device=dev)
        self.exp_avg_sq = torch.zeros(hi - lo, dtype=torch.float32, device=dev)
        self.grad_shard = torch.zeros(hi - lo, dtype=torch.float32, device=dev) if grad_shard else None
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
        """mode: "auto" (NVLS where the GPUs have NVLink multicast and every rank can allocate its
        buffers, else NCCL), "nvls" (bf16 cast + one multicast kernel after the backward), "nvls-overlap"
        (the same per bucket, overlapped with the backward), "nccl" (reduce-scatter /
        all-gather), "fused" (one peer-memory kernel after the backward) or "fused-overlap"
        (that kernel per bucket, overlapped with the backward)."""
        self.world_size, self.rank, self.mode, self.group = world_size, rank, mode, group
        self.requested = mode  # "auto" resolves here: NVLS where multicast exists, NCCL otherwise
        self.fallback_reason = None
        if mode == "auto":
            self.mode = pick_mode(mode, torch.cuda.current_device() if torch.cuda.is_available() else 0)
        # False when the model's gradient writers store on the step's first write (the NCCL
        # step then skips clearing the buffer, and so does the peer-memory kernel)
        self.zero_grads = True
        self.flat = None
        self.fused = None

    @property
    def overlap(self):
        return self.mode in ("fused-overlap", "nvls-overlap")

    def make_optimizer(self, flat, lr=3e-4, **kw):
        if flat.numel % self.world_size:
            raise ValueError("flat buffer must be padded to a multiple of the world size")
        if self.overlap:
            if not flat.buckets:
                raise ValueError("fused-overlap needs a bucket-padded flat buffer (FlatParams(bucket_pad=True))")
            self.flat = flat
            opt = BucketShardedAdamW(flat, self.rank, self.world_size, lr=lr, **kw)
            src = dist.get_global_rank(self.group, 0) if self.group is not None else 0
            dist.broadcast(flat.master, src, group=self.group)
            flat.refresh_shadow()
            if self.mode == "nvls-overlap":
                from llmt.parallel.nvls_dp import NvlsOverlapDP
                self.fused = NvlsOverlapDP(flat, opt, self.rank, self.world_size, self.group)
            else:
                from llmt.parallel.fused_dp import OverlappedFusedDP
                self.fused = OverlappedFusedDP(flat, opt, self.rank, self.world_size, self.group)
            return opt
        shard = flat.numel // self.world_size
        self.flat = flat
        lo, hi = self.rank * shard, (self.rank + 1) * shard
        opt = ShardedAdamW(flat, lo, hi, lr=lr, grad_scale=1.0 / self.world_size, grad_shard=self.mode == "nccl",
                           **kw)
        # all ranks start from rank 0's weights (the same seed already makes them equal; this
        # makes it a guarantee)
        src = dist.get_global_rank(self.group, 0) if self.group is not None else 0
        dist.broadcast(flat.master, src, group=self.group)
        flat.refresh_shadow()
        if self.mode == "fused":
            from llmt.parallel.fused_dp import FusedDP
            self.fused = FusedDP(flat, opt, self.rank, self.world_size, self.group)
        elif self.mode == "nvls":
            from llmt.parallel.nvls_dp import NvlsDP, NvlsUnavailable
            try:
                self.fused = NvlsDP(flat, opt, self.rank, self.world_size, self.group)
            except NvlsUnavailable as e:
                if self.requested != "auto":
                    raise
                # "auto" falls back to the NCCL step (every rank took the same decision)
                self.fallback_reason = str(e)
                self.mode = "nccl"
                opt.grad_shard = torch.zeros(hi - lo, dtype=torch.float32, device=flat.master.device)
        return opt

    def begin_step(self):
        if self.overlap:
            self.fused.begin_step()

    def bucket_ready(self, b):
        if self.overlap:
            self.fused.bucket_ready(b)

    def gather_master(self, opt):
        """Full fp32 masters on every rank (ZeRO-1 leaves other ranks' shards stale)."""
        f = self.flat
        if isinstance(opt, BucketShardedAdamW):
            opt.gather_master(self.group)
            return
        shard = f.numel // self.world_size
        full = torch.empty_like(f.master)
        dist.all_gather_into_tensor(full, f.master[self.rank * shard:(self.rank + 1) * shard].contiguous(),
                                    group=self.group)
        f.master.copy_(full)

    @torch.no_grad()
    def reduce_and_step(self, opt: ShardedAdamW):
        f = self.flat
        if self.fused is not None and hasattr(self.fused, "clear_grads"):
            self.fused.clear_grads = self.zero_grads  # used from this step's kernels on
        if self.overlap:
            self.fused.finish_step()
            return
        if self.fused is not None:
            self.fused.step()
            return
        dist.reduce_scatter_tensor(opt.grad_shard, f.grad, op=dist.ReduceOp.SUM, group=self.group)
        if self.zero_grads:
            f.grad.zero_()  # gradients accumulate into the flat buffer
        opt.step_local()
        dist.all_gather_into_tensor(f.shadow, f.shadow[opt.lo:opt.hi].clone(), group=self.group)

    def close(self):
        if self.fused is not None:
            self.fused.close()
            self.fused = None


class BucketShardedAdamW:
    """AdamW state for this rank's chunk of every bucket of a bucket-padded flat buffer
    (FlatParams(bucket_pad=True)): bucket (lo, hi) splits into `world` equal chunks and rank r
    owns chunk r of each; m / v hold the owned chunks back to back. The overlapped fused
    data-parallel step updates one bucket as soon as its gradients are final."""

    def __init__(self, flat, rank, world, lr=3e-4, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1):
        self.flat, self.rank, self.world = flat, rank, world
        self.ranges, self.moffs = [], []
        moff = 0
        for lo, hi in flat.buckets:
            c = (hi - lo) // world
            self.ranges.append((lo + rank * c, lo + (rank + 1) * c))
            self.moffs.append(moff)
            moff += c
        dev = flat.master.device
        self.exp_avg = torch.zeros(moff, dtype=torch.float32, device=dev)
        self.exp_avg_sq = torch.zeros(moff, dtype=torch.float32, device=dev)
        self.lr_t = torch.full((1,), float(lr), dtype=torch.float32, device=dev)
        self.step_t = torch.zeros(1, dtype=torch.int32, device=dev)
        self.betas, self.eps, self.weight_decay, self.grad_scale = betas, eps, weight_decay, 1.0 / world

    def set_lr(self, lr):
        self.lr_t.fill_(float(lr))

    def gather_master(self, group=None):
        """Every rank's master chunks -> the full fp32 master on every rank (checkpoints, checks)."""
        f = self.flat
        for (lo, hi) in f.buckets:
            c = (hi - lo) // self.world
            mine = f.master[lo + self.rank * c:lo + (self.rank + 1) * c].clone()
            dist.all_gather_into_tensor(f.master[lo:hi], mine, group=group)
