"""Data-parallel step on NVLink multicast (host side of csrc/comm/dp_nvls.cu).

Replaces NCCL reduce_scatter + sharded AdamW + all_gather (llmt.parallel.dp, mode "nccl") by
a bf16 cast of the gradient and one fused kernel per step:

  cast      the flat fp32 gradient the backward wrote -> a symmetric bf16 buffer (local)
  barrier   every rank's cast is complete (flag barrier over peer memory, bounded)
  fused     multimem.ld_reduce of this rank's gradient shard (summed in the NVSwitch, fp32
            accumulation), AdamW on the fp32 master shard, multimem.st of the new bf16 weights
            into every rank's weight buffer
  barrier   every rank's weights are written before any rank's next forward reads them

Set-up uses PyTorch's symmetric memory (torch.distributed._symmetric_memory) for the plumbing:
the bf16 gradient buffer, the bf16 weight buffer (which becomes the model's shadow weights) and
a small flag pad are symmetric allocations, and the rendezvous binds the first two to NVLink
multicast objects; the kernel only receives their multicast addresses. Ranks that cannot get a
multicast address (no NVSwitch, or a single GPU) raise at set-up.

NvlsOverlapDP runs the same three parts per bucket (a block's parameters, or the trailing
emb / norm_f / head group) on a side stream as soon as the backward has issued the bucket's
gradients, so the reductions and the weight multicasts cross NVLink while the backward of the
earlier blocks computes.
"""
from __future__ import annotations

import os

import torch
import torch.distributed as dist

from llmt.ops import native as N


def _symm():
    import torch.distributed._symmetric_memory as symm
    return symm


class NvlsUnavailable(RuntimeError):
    """Some rank of the group could not allocate the symmetric buffers (every rank raises it)."""


class NvlsDP:
    def __init__(self, flat, opt, rank: int, world: int, group=None):
        self.flat, self.opt, self.rank, self.world = flat, opt, rank, world
        self.group = group if group is not None else dist.group.WORLD
        symm = _symm()
        dev = flat.master.device
        self.device = dev
        # The symmetric buffers come from their own allocator; where one rank cannot get them
        # (device memory) every rank learns it before the collective rendezvous and raises.
        why = ""
        try:
            self.g16 = symm.empty(flat.numel, dtype=torch.bfloat16, device=dev)
            shadow = symm.empty(flat.numel, dtype=torch.bfloat16, device=dev)
            self.pad = symm.empty(64 * world, dtype=torch.int32, device=dev)
        except RuntimeError as e:  # torch.OutOfMemoryError, CUDA driver errors
            why = str(e).splitlines()[0][:200]
            self.g16 = shadow = self.pad = None
            torch.cuda.empty_cache()
        ok = torch.tensor([0 if why else 1], dtype=torch.int32, device=dev)
        dist.all_reduce(ok, op=dist.ReduceOp.MIN, group=self.group)
        if not int(ok.item()):
            self.g16 = shadow = self.pad = None
            torch.cuda.empty_cache()
            raise NvlsUnavailable("NVLS buffers could not be allocated on every rank" + (f": {why}" if why else ""))
        flat.rebind(grad=flat.grad, shadow=shadow)
        flat.refresh_shadow()  # bf16 copy of the (broadcast) masters
        self.pad.zero_()
        torch.cuda.synchronize(dev)
        # the rendezvous binds the buffers to multicast objects (collective); a rank that gets no
        # multicast address reports it and every rank raises together
        why = ""
        try:
            self.h_g = symm.rendezvous(self.g16, self.group)
            self.h_w = symm.rendezvous(flat.shadow, self.group)
            self.h_p = symm.rendezvous(self.pad, self.group)
            if not self.h_g.multicast_ptr or not self.h_w.multicast_ptr:
                why = "symmetric memory reported no NVLink multicast address"
        except RuntimeError as e:
            why = str(e).splitlines()[0][:200]
        ok = torch.tensor([0 if why else 1], dtype=torch.int32, device=dev)
        dist.all_reduce(ok, op=dist.ReduceOp.MIN, group=self.group)
        if not int(ok.item()):
            self.g16 = None
            torch.cuda.empty_cache()
            raise NvlsUnavailable("NVLS multicast set-up failed on some rank" + (f": {why}" if why else ""))
        self.g_mc = self.h_g.multicast_ptr + (self.g16.data_ptr() - self.h_g.buffer_ptrs[rank])
        self.w_mc = self.h_w.multicast_ptr + (flat.shadow.data_ptr() - self.h_w.buffer_ptrs[rank])
        off = self.pad.data_ptr() - self.h_p.buffer_ptrs[rank]
        self.pads_dev = torch.tensor([p + off for p in self.h_p.buffer_ptrs], dtype=torch.int64, device=dev)
        self.my_pad = self.pad.data_ptr()
        self.epoch = torch.zeros(1, dtype=torch.int32, device=dev)
        torch.cuda.synchronize(dev)
        dist.barrier(group=self.group)

    @torch.no_grad()
    def step(self):
        C, o, f = N.ext(), self.opt, self.flat
        C.cast_bf16(f.grad, self.g16)
        C.dp_barrier(self.pads_dev, self.my_pad, self.epoch, self.rank, self.world, 300)
        o.step_t.add_(1)
        b1, b2 = o.betas
        C.dp_nvls_adamw(self.g_mc, self.w_mc, f.master, o.exp_avg, o.exp_avg_sq, o.lo, o.hi - o.lo, o.lr_t, o.step_t,
                        b1, b2, o.eps, o.weight_decay, o.grad_scale)
        C.dp_barrier(self.pads_dev, self.my_pad, self.epoch, self.rank, self.world, 400)

    def error_code(self, reset=False) -> int:
        return N.ext().dp_error_code(reset)

    def close(self):
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)


class NvlsOverlapDP(NvlsDP):
    """The NVLS data-parallel step one bucket at a time, overlapped with the rest of the backward.

    Needs the bucket-sharded optimizer (llmt.parallel.dp.BucketShardedAdamW): rank r owns chunk r
    of every bucket. When a block's backward has been issued (a hook on the gradient of the
    block's input), a side stream waits for that point and, on `sms` SMs that the persistent
    GEMM / attention grids leave free:
      cast      the bucket's fp32 gradients -> the symmetric bf16 buffer
      barrier   every rank's cast of the bucket is complete (so every rank's backward has also
                finished reading the bucket's weights)
      fused     multimem.ld_reduce + AdamW + multimem.st of this rank's chunk of the bucket
    After the backward the trailing bucket follows, then a final barrier (every rank's new
    weights are in every rank's buffer) that the main stream joins before the next forward.
    `sms` defaults to LLMT_DP_SMS or 16."""

    def __init__(self, flat, opt, rank: int, world: int, group=None, sms: int | None = None):
        super().__init__(flat, opt, rank, world, group)
        self.sms = int(os.environ.get("LLMT_DP_SMS", "16")) if sms is None else int(sms)
        # the side kernels run 4 CTAs of 256 threads per reserved SM; one more SM for the barrier
        self.blocks = 4 * max(1, self.sms)
        N.ext().set_reserved_sms(self.sms + 1)
        self.side = torch.cuda.Stream(device=self.device, priority=-1)
        self.armed = False
        self.started = False
        self.done = set()

    def begin_step(self):
        """Arm the bucket hooks for the backward that follows (the last micro-batch's)."""
        self.armed, self.started, self.done = True, False, set()

    def _bucket(self, b):
        C, o, f = N.ext(), self.opt, self.flat
        blo, bhi = f.buckets[b]
        lo, hi = o.ranges[b]
        moff, n = o.moffs[b], hi - lo
        if not self.started:
            o.step_t.add_(1)
            self.started = True
        C.cast_bf16(f.grad[blo:bhi], self.g16[blo:bhi], self.blocks)
        C.dp_barrier(self.pads_dev, self.my_pad, self.epoch, self.rank, self.world, 500)
        b1, b2 = o.betas
        C.dp_nvls_adamw(self.g_mc, self.w_mc, f.master, o.exp_avg[moff:moff + n], o.exp_avg_sq[moff:moff + n], lo, n,
                        o.lr_t, o.step_t, b1, b2, o.eps, o.weight_decay, o.grad_scale, self.blocks)

    def bucket_ready(self, b):
        """Called (from the backward's hooks) when bucket b's gradients have all been issued."""
        if not self.armed or b in self.done:
            return
        self.done.add(b)
        self.side.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(self.side):
            self._bucket(b)

    @torch.no_grad()
    def finish_step(self):
        for b in range(len(self.opt.ranges)):  # the trailing bucket, and any a hook did not reach
            self.bucket_ready(b)
        with torch.cuda.stream(self.side):
            N.ext().dp_barrier(self.pads_dev, self.my_pad, self.epoch, self.rank, self.world, 600)
        torch.cuda.current_stream(self.device).wait_stream(self.side)
        self.armed = False

    def close(self):
        N.ext().set_reserved_sms(0)
        super().close()
