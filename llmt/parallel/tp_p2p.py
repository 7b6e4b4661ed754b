"""Tensor-parallel row collectives over NVLink peer memory, fused with their producers.

Host side of csrc/comm/tp_p2p.cu and of the GEMM's PEER_RS epilogue. Every rank of the
tensor-parallel group allocates CUDA-IPC exportable buffers, the handles are exchanged over
the group and every rank maps every peer's buffers, so kernels read and write peer memory
directly through NVSwitch (no NCCL, no multicast):

  gather sites   one (N, d) bf16 buffer per all-gather site of the forward (two per block):
                 each rank stores its N/tp rows into every peer's buffer; the gathered
                 tensor handed to the next GEMM is this rank's buffer (kept for the backward).
                 Under pipeline parallelism several micro-batches are between their forward
                 and their backward at once: `sets` copies of the site buffers, micro-batch i
                 uses set i % sets (select_set), so a later forward never overwrites rows an
                 earlier micro-batch's backward still reads
  slots          (tp, N/tp, d) bf16, two sets used alternately: the row-parallel GEMMs (wo,
                 w2) store each output row straight into slot `rank` of the row's owner from
                 their epilogue (GEMM -> reduce-scatter in one kernel, the transfer overlapping
                 the remaining tiles), then the owner sums its tp slots
  bwd gather     two (N, d) buffers used alternately for the backward's all-gathers
  pad            barrier flags; a flag barrier (bounded wait, error code on timeout) follows
                 every collective, so a buffer is rewritten only after every rank is done
                 with its previous contents
  gather flags   one counter per 128-row block of every gather buffer (fused gathers)

Alternating sets are safe because between two uses of one set every rank passes the
barrier of the other set's collective, which it reaches only after its kernels that read the
first set have completed (same stream).

Fused all-gathers (fuse_gather, on when every rank's rows are whole 128-row blocks): the
gather is not run when it is asked for. The returned buffer carries it as a pending gather, and
the GEMM that consumes the buffer (qkv, w1||w3 in the forward; the w2 / wo dgrads on the
backward's gathered dy) performs it: its epilogue warps store this rank's rows into every
rank's buffer in 16-row pieces before their first tile, counting each piece in the
destination's flag of that 128-row block, and its TMA producer loads a tile of A only once the
flag of the tile's block has reached this call's count (this rank's own blocks are loaded
first). No barrier follows a fused gather. Its buffers are still rewritten only after every
rank is done with them: a forward site is next written in the next step, after the backward's
reduce-scatter barrier of the same site, which every rank passes only after its weight-gradient
GEMM read the site; between two uses of one backward gather buffer every rank passes a
reduce-scatter barrier (each block's backward runs one between its two gathers). The flag
counts grow by a fixed amount per call on every rank, so they are never reset.
"""
from __future__ import annotations

import os

import torch
import torch.distributed as dist

from llmt.ops import native as N

EPI_PEER_RS = 7


AG_PIECES = 8  # 16-row pieces per 128-row block: each adds one to the block's flag (kAgPieces)


class PendingGather:
    """An all-gather owed by a gather buffer: run by the consuming GEMM (kwargs) or, when the
    first consumer cannot fuse it, on its own (run_unfused)."""

    def __init__(self, comm, x_l, index, dst_ptrs, flag_ptrs):
        self.comm, self.x_l, self.index = comm, x_l, index
        self.dst_ptrs, self.flag_ptrs = dst_ptrs, flag_ptrs

    def kwargs(self):
        c = self.comm
        c.ag_calls[self.index] += 1
        return dict(ag_src=self.x_l, ag_dst=self.dst_ptrs, ag_flags=self.flag_ptrs,
                    ag_expect=c.ag_calls[self.index] * AG_PIECES, ag_tp=c.tp, tp_rank=c.rank, rows_per_rank=c.nl)

    def run_unfused(self):
        self.comm._gather(self.x_l, self.dst_ptrs, 700)


class TPPeerComm:
    def __init__(self, group, rows: int, d: int, sites: int, device, fuse_gather: bool = True, sets: int = 1):
        C = N.ext()
        self.group = group
        self.tp = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if rows % self.tp or d % 32:
            raise ValueError(f"peer collectives need rows % tp == 0 and d % 32 == 0 (rows {rows}, d {d})")
        self.rows, self.d, self.nl = rows, d, rows // self.tp
        dev = torch.device(device)
        self.device = dev
        mat = rows * d * 2  # bytes of one (N, d) bf16 buffer
        self.n_sites = sites
        self.sets, self.set = sets, 0
        sites = sites * sets  # forward site buffers of every set, set-major
        total = (sites + 2 + 2) * mat  # gather sites, 2 slot sets, 2 backward gathers
        fuse_gather = fuse_gather and os.environ.get("LLMT_TP_FUSE_GATHER", "1") != "0"
        self.fuse_gather = fuse_gather and self.nl % 128 == 0 and d % 8 == 0
        self.blocks = rows // 128
        fbytes = max(4096, (sites + 2) * self.blocks * 4)  # flags of the forward sites, 2 backward gathers
        ptr, h = C.ipc_alloc(total)
        pad, ph = C.ipc_alloc(4096)
        flg, fh = C.ipc_alloc(fbytes)
        self._own = [ptr, pad, flg]
        mine = torch.tensor(list(h + ph + fh), dtype=torch.uint8, device=dev)
        allh = [torch.empty_like(mine) for _ in range(self.tp)]
        dist.all_gather(allh, mine, group=group)
        bases, pads, flags = [], [], []
        self._peers = []
        for p, hh in enumerate(allh):
            if p == self.rank:
                bases.append(ptr)
                pads.append(pad)
                flags.append(flg)
                continue
            b = bytes(hh.cpu().tolist())
            bp, pp, fp = C.ipc_open(b[0:64]), C.ipc_open(b[64:128]), C.ipc_open(b[128:192])
            self._peers += [bp, pp, fp]
            bases.append(bp)
            pads.append(pp)
            flags.append(fp)

        def ptrs(off):
            return torch.tensor([b + off for b in bases], dtype=torch.int64, device=dev)

        def local(off, shape):
            n = 1
            for s in shape:
                n *= s
            return C.tensor_from_ptr(ptr + off, n, torch.bfloat16, dev.index).view(*shape)

        self.site_ptrs = [ptrs(s * mat) for s in range(sites)]
        self.site_local = [local(s * mat, (rows, d)) for s in range(sites)]
        self.slot_ptrs = [ptrs((sites + k) * mat) for k in range(2)]
        self.slot_local = [local((sites + k) * mat, (rows, d)) for k in range(2)]
        self.bwd_ptrs = [ptrs((sites + 2 + k) * mat) for k in range(2)]
        self.bwd_local = [local((sites + 2 + k) * mat, (rows, d)) for k in range(2)]
        fl = self.blocks * 4
        self.site_flag_ptrs = [torch.tensor([f + s * fl for f in flags], dtype=torch.int64, device=dev)
                               for s in range(sites + 2)]  # forward sites, then the 2 backward buffers
        self.ag_calls = [0] * (sites + 2)
        self.pads_dev = torch.tensor(pads, dtype=torch.int64, device=dev)
        self.my_pad = pad
        self.epoch = torch.zeros(1, dtype=torch.int32, device=dev)
        self._slot = 0
        self._bwd = 0
        torch.cuda.synchronize(dev)
        dist.barrier(group=group)

    # ------------------------------------------------------------------ primitives
    def barrier(self, code):
        N.ext().dp_barrier(self.pads_dev, self.my_pad, self.epoch, self.rank, self.tp, code)

    def _gather(self, x_l, dst_ptrs, code):
        N.ext().tp_allgather_rows(x_l.contiguous(), dst_ptrs, self.tp, self.rank * self.nl)
        self.barrier(code)

    def select_set(self, k: int):
        """Forward gathers from now on use site-buffer set k (the micro-batch's)."""
        self.set = k % self.sets

    def _pending(self, x_l, buf, index, dst_ptrs):
        out = buf.view_as(buf)
        out._llmt_pending_ag = PendingGather(self, x_l.contiguous(), index, dst_ptrs, self.site_flag_ptrs[index])
        return out

    def all_gather_site(self, x_l, site):
        """(N/tp, d) rows of every rank -> this rank's (N, d) buffer of the site (returned; with
        fused gathers the consuming GEMM fills it)."""
        site += self.set * self.n_sites
        if self.fuse_gather:
            return self._pending(x_l, self.site_local[site], site, self.site_ptrs[site])
        self._gather(x_l, self.site_ptrs[site], 300)
        return self.site_local[site]

    def all_gather_bwd(self, x_l):
        k = self._bwd
        self._bwd ^= 1
        if self.fuse_gather:
            return self._pending(x_l, self.bwd_local[k], self.n_sites * self.sets + k, self.bwd_ptrs[k])
        self._gather(x_l, self.bwd_ptrs[k], 600)
        return self.bwd_local[k]

    def _sum(self, k):
        out = torch.empty((self.nl, self.d), dtype=torch.bfloat16, device=self.device)
        N.ext().tp_sum_slots(self.slot_local[k], out, self.tp)
        return out

    def reduce_scatter(self, partial):
        """(N, d) partial sums of every rank -> this rank's summed (N/tp, d) rows."""
        k = self._slot
        self._slot ^= 1
        N.ext().tp_scatter_rows(partial.contiguous(), self.slot_ptrs[k], self.tp, self.rank)
        self.barrier(400)
        return self._sum(k)

    def gemm_rs(self, x, w16):
        """Row-parallel GEMM x @ w16^T whose epilogue stores each output row into its owner's
        slot; returns this rank's summed rows (N/tp, d)."""
        k = self._slot
        self._slot ^= 1
        N.ext().gemm(x, w16, False, True, EPI_PEER_RS, self.slot_local[k], peer=self.slot_ptrs[k],
                     tp_rank=self.rank, rows_per_rank=self.nl)
        self.barrier(500)
        return self._sum(k)

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
        for p in self._own:
            C.ipc_free(p)
        self._own = []


class AllGatherP2P(torch.autograd.Function):
    """Forward: all-gather of sequence rows into the site's peer-mapped buffer. Backward: the
    reduce-scatter of the gradient over peer memory."""

    @staticmethod
    def forward(ctx, x_l, comm, site):
        ctx.comm = comm
        return comm.all_gather_site(x_l, site)

    @staticmethod
    def backward(ctx, g):
        return ctx.comm.reduce_scatter(g), None, None


class RowLinearRS(torch.autograd.Function):
    """y_rows = reduce-scatter(x @ W^T) with the GEMM storing its rows to their owners (one
    kernel). Backward: all-gather of dy over peer memory, then the dgrad / wgrad GEMMs (the
    wgrad accumulates into W.main_grad)."""

    @staticmethod
    def forward(ctx, x, w, comm):
        ctx.save_for_backward(x)
        ctx.w, ctx.comm = w, comm
        return comm.gemm_rs(x, w.w16)

    @staticmethod
    def backward(ctx, dy):
        (x,) = ctx.saved_tensors
        w, comm = ctx.w, ctx.comm
        dY = comm.all_gather_bwd(dy)
        dx = N.gemm(dY, w.w16, ta=False, tb=False)
        N.gemm(dY, x, ta=True, tb=False, out=w.main_grad, accumulate=True)
        return dx, None, None
