"""Fused data-parallel step over NVLink peer memory (host side of csrc/comm/dp_fused.cu).

Replaces NCCL reduce_scatter + sharded AdamW + all_gather (llmt.parallel.dp, mode "nccl") by
one kernel per step. Set-up: the flat fp32 gradient and bf16 shadow-weight buffers are
re-allocated as CUDA-IPC exportable memory, their 64-byte handles are exchanged over the
process group, and every rank opens every peer's buffers, so the kernel can load and store
peer memory directly through NVSwitch. A small signal pad per rank carries the epoch flags of
the device-side barrier (bounded spins; a timeout sets an error code readable with
error_code()). No multicast is used.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from llmt.ops import native as N


class FusedDP:
    def __init__(self, flat, opt, rank: int, world: int, group=None):
        self.flat, self.opt, self.rank, self.world, self.group = flat, opt, rank, world, group
        C = N.ext()
        dev = flat.master.device
        self.device = dev
        self._own = []
        gp, gh = C.ipc_alloc(flat.numel * 4)
        sp, sh = C.ipc_alloc(flat.numel * 2)
        pp, ph = C.ipc_alloc(4096)
        self._own = [gp, sp, pp]
        grad = C.tensor_from_ptr(gp, flat.numel, torch.float32, dev.index)
        shadow = C.tensor_from_ptr(sp, flat.numel, torch.bfloat16, dev.index)
        grad.copy_(flat.grad)
        shadow.copy_(flat.shadow)
        flat.rebind(grad=grad, shadow=shadow)
        mine = torch.tensor(list(gh + sh + ph), dtype=torch.uint8, device=dev)
        allh = [torch.empty_like(mine) for _ in range(world)]
        dist.all_gather(allh, mine, group=group)
        self._peers = []
        gptr, sptr, pptr = [], [], []
        for p, h in enumerate(allh):
            b = bytes(h.cpu().tolist())
            if p == rank:
                gptr.append(gp)
                sptr.append(sp)
                pptr.append(pp)
                continue
            g_, s_, p_ = C.ipc_open(b[0:64]), C.ipc_open(b[64:128]), C.ipc_open(b[128:192])
            self._peers += [g_, s_, p_]
            gptr.append(g_)
            sptr.append(s_)
            pptr.append(p_)
        self.grads_dev = torch.tensor(gptr, dtype=torch.int64, device=dev)
        self.shadows_dev = torch.tensor(sptr, dtype=torch.int64, device=dev)
        self.pads_dev = torch.tensor(pptr, dtype=torch.int64, device=dev)
        self.my_pad = pp
        self.epoch = torch.zeros(1, dtype=torch.int32, device=dev)
        # zero the gradient shards after reading them; off when the model's first gradient
        # write of a step stores (DataParallel.zero_grads), which saves world x 4 bytes of
        # NVLink stores per parameter
        self.clear_grads = True
        torch.cuda.synchronize(dev)
        dist.barrier(group=group)

    @torch.no_grad()
    def step(self):
        C, o, f = N.ext(), self.opt, self.flat
        C.dp_barrier(self.pads_dev, self.my_pad, self.epoch, self.rank, self.world, 100)
        o.step_t.add_(1)
        b1, b2 = o.betas
        C.dp_fused_adamw(self.grads_dev, self.shadows_dev, f.master, o.exp_avg, o.exp_avg_sq, o.lo, o.hi - o.lo,
                         o.lr_t, o.step_t, b1, b2, o.eps, o.weight_decay, o.grad_scale, self.world,
                         clear=self.clear_grads)
        C.dp_barrier(self.pads_dev, self.my_pad, self.epoch, self.rank, self.world, 200)

    def error_code(self, reset=False) -> int:
        return N.ext().dp_error_code(reset)

    def close(self):
        if not self._own:
            return
        C = N.ext()
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        for p in self._peers:
            C.ipc_close(p)
        self._peers = []
        dist.barrier(group=self.group)
        # the flat views must not outlive the memory: hand the model ordinary buffers back
        grad = self.flat.grad.clone()
        shadow = self.flat.shadow.clone()
        self.flat.rebind(grad=grad, shadow=shadow)
        torch.cuda.synchronize(self.device)
        for p in self._own:
            C.ipc_free(p)
        self._own = []


class OverlappedFusedDP(FusedDP):
    """The fused data-parallel step, one bucket (a block's parameters, or the trailing emb /
    norm_f / head group) at a time, overlapped with the rest of the backward.

    When a block's backward has been issued (a hook on the gradient of the block's input), a
    side stream waits for that point, passes a flag barrier (every rank's gradients of the bucket
    are final) and runs the fused reduce + AdamW + bf16 all-gather on this rank's chunk of the
    bucket, on at most `max_blocks` CTAs so the backward keeps the rest of the GPU. After the
    backward the trailing bucket follows, then a final barrier (every rank's new weights are in
    every peer's buffer) that the main stream joins before the next forward."""

    def __init__(self, flat, opt, rank: int, world: int, group=None, max_blocks: int = 32):
        super().__init__(flat, opt, rank, world, group)
        self.max_blocks = max_blocks
        # persistent GEMM / attention grids leave these SMs to the bucket kernels (one more for
        # the flag barrier), so the two streams do not wait on each other for SMs
        N.ext().set_reserved_sms(max_blocks + 1)
        self.side = torch.cuda.Stream(device=self.device)
        self.armed = False
        self.started = False
        self.done = set()

    def begin_step(self):
        """Arm the bucket hooks for the backward that follows (the last micro-batch's)."""
        self.armed, self.started, self.done = True, False, set()

    def _bucket(self, b):
        C, o, f = N.ext(), self.opt, self.flat
        lo, hi = o.ranges[b]
        moff = o.moffs[b]
        n = hi - lo
        if not self.started:
            o.step_t.add_(1)
            self.started = True
        C.dp_barrier(self.pads_dev, self.my_pad, self.epoch, self.rank, self.world, 700)
        b1, b2 = o.betas
        C.dp_fused_adamw(self.grads_dev, self.shadows_dev, f.master, o.exp_avg[moff:moff + n],
                         o.exp_avg_sq[moff:moff + n], lo, n, o.lr_t, o.step_t, b1, b2, o.eps, o.weight_decay,
                         o.grad_scale, self.world, self.max_blocks, clear=self.clear_grads)

    def bucket_ready(self, b):
        """Called (from the backward's hooks) when bucket b's gradients have all been issued."""
        if not self.armed or b in self.done:
            return
        self.done.add(b)
        cur = torch.cuda.current_stream(self.device)
        self.side.wait_stream(cur)
        with torch.cuda.stream(self.side):
            self._bucket(b)

    def close(self):
        N.ext().set_reserved_sms(0)
        super().close()

    @torch.no_grad()
    def finish_step(self):
        for b in range(len(self.opt.ranges)):  # the trailing bucket, and any a hook did not reach
            self.bucket_ready(b)
        cur = torch.cuda.current_stream(self.device)
        with torch.cuda.stream(self.side):
            N.ext().dp_barrier(self.pads_dev, self.my_pad, self.epoch, self.rank, self.world, 800)
        cur.wait_stream(self.side)
        self.armed = False
