"""One training step over a data x pipeline x tensor parallel layout (`ParallelTrainer`).

Builds this rank's stage (its blocks, tensor-parallel shard), the optimizer (ZeRO-1 AdamW over
the data-parallel group, or the fused AdamW when dp = 1), and runs forward + backward over the
micro-batches (1F1B across stages when pp > 1, plain accumulation otherwise), the tensor-parallel
sum of the replicated norm gradients, then the data-parallel reduce + optimizer step.

impl="native" runs the sm_100a kernels (flat parameter buffers, NCCL); impl="torch" runs the
same layout with plain fp32 torch ops and torch.optim.AdamW (the CPU / gloo reference used
by the tests).

    layout = Layout(dp=2, tp=2, pp=2)
    tr = ParallelTrainer(get_config("llama3-8b"), batch=2, seq=4096, layout=layout, microbatches=4)
    loss = tr.train_step(idx, tgt)      # this data-parallel rank's (batch, seq) tokens
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from llmt.config import ModelConfig
from llmt.parallel.groups import Layout, ParallelGroups, rank_of
from llmt.parallel.pp import NativeStage, Pipeline1F1B, TorchStage, build_stage
from llmt.parallel.tp import sync_replicated_grads


class ParallelTrainer:
    def __init__(self, cfg: ModelConfig, batch: int, seq: int, layout: Layout, microbatches: int = 1,
                 device="cuda", seed: int = 0, lr: float = 3e-4, impl: str = "native", dp_mode: str = "nccl",
                 init: str = "full", ce_chunk: int = 8192, cuda_graph: bool = False, tp_comm: str = "nccl",
                 linear: str = "bf16"):
        self.cfg, self.batch, self.seq, self.layout, self.m = cfg, batch, seq, layout, microbatches
        if batch % microbatches:
            raise ValueError("batch must be a multiple of microbatches")
        self.device = torch.device(device)
        self.impl = impl
        self.groups = g = ParallelGroups(layout)
        self.stage = build_stage(cfg, seq, layout.pp, g.pp_rank, layout.tp, g.tp_rank, seed=seed, device=self.device,
                                 init=init)
        if impl == "native":
            self.x = NativeStage(self.stage, g.tp_group, pad_to=layout.dp, ce_chunk=ce_chunk, comm=tp_comm,
                                 in_flight=layout.pp, linear=linear)
            flat = self.x.flat
            if layout.dp > 1:
                from llmt.parallel.dp import DataParallel
                self.dp = DataParallel(layout.dp, g.dp_rank, mode=dp_mode, group=g.dp_group)
                self.opt = self.dp.make_optimizer(flat, lr=lr)
            else:
                from llmt.optim.adamw import FusedAdamW
                self.dp = None
                self.opt = FusedAdamW(flat.master, flat.grad, flat.shadow, lr=lr)
        elif impl == "torch":
            self.x = TorchStage(self.stage, g.tp_group)
            self.dp = None
            self.opt = torch.optim.AdamW(self.stage.parameters(), lr=lr, betas=(0.9, 0.95), weight_decay=0.1)
        else:
            raise ValueError(f"unknown impl {impl!r}")
        self.pipe = None
        if layout.pp > 1:
            s = g.pp_rank
            prev = rank_of(g.dp_rank, s - 1, g.tp_rank, layout.pp, layout.tp) if s > 0 else None
            nxt = rank_of(g.dp_rank, s + 1, g.tp_rank, layout.pp, layout.tp) if s < layout.pp - 1 else None
            self.pipe = Pipeline1F1B(self.x, s, layout.pp, prev, nxt, g.pp_group, self.device)
        self.loss = torch.zeros((), dtype=torch.float32, device=self.device)
        # whole-step CUDA graph (forward, backward, collectives, optimizer) for layouts without a
        # pipeline: static token buffers, captured after two eager warm-up steps that are undone
        # (the peer-memory tensor-parallel path is not capturable: it runs eager, recorded as
        # cuda_graph false in the bench output)
        self.use_graph = cuda_graph and impl == "native" and layout.pp == 1 and tp_comm != "p2p"
        self.graph = None
        if self.use_graph:
            self.idx_buf = torch.zeros((batch, seq), dtype=torch.long, device=self.device)
            self.tgt_buf = torch.zeros((batch, seq), dtype=torch.long, device=self.device)

    @property
    def is_last_stage(self):
        return self.groups.pp_rank == self.layout.pp - 1

    def forward_backward(self, idx, tgt):
        """Gradients of this step's micro-batches (not yet reduced over data parallel). Returns the
        mean loss on the last pipeline stage, None on the others."""
        mb = self.batch // self.m
        idx = idx.to(self.device, non_blocking=True).view(self.m, mb, self.seq)
        tgt = tgt.to(self.device, non_blocking=True).view(self.m, mb, self.seq)
        if self.pipe is not None:
            loss = self.pipe.step(idx, tgt)
        else:
            losses = []
            for i in range(self.m):
                l_i = self.x.forward_last(self.x.forward_blocks(self.x.forward_first(idx[i]), mb, self.seq), tgt[i])
                (l_i / self.m).backward()
                losses.append(l_i.detach())
            loss = torch.stack(losses).mean()
        sync_replicated_grads(self.stage, self.groups.tp_group, main_grad=self.impl == "native")
        return loss

    def optimizer_step(self):
        if self.impl == "native":
            if self.dp is not None:
                self.dp.reduce_and_step(self.opt)
            else:
                self.opt.step()
            return
        if self.groups.dp_group is not None:
            for p in self.stage.parameters():
                dist.all_reduce(p.grad, group=self.groups.dp_group)
                p.grad /= self.layout.dp
        self.opt.step()
        self.opt.zero_grad(set_to_none=True)

    def _body(self, idx, tgt):
        loss = self.forward_backward(idx, tgt)
        self.optimizer_step()
        if loss is not None:
            self.loss.copy_(loss)

    def run_step(self, idx, tgt):
        """One step without a host sync (graph replay when enabled)."""
        if not self.use_graph:
            self._body(idx, tgt)
            return
        self.idx_buf.copy_(idx, non_blocking=True)
        self.tgt_buf.copy_(tgt, non_blocking=True)
        if self.graph is None:
            # two eager warm-up steps and the capture, then the weights and the optimizer state go
            # back as they were: the first call is one step like every other
            flat = self.x.flat
            state = [flat.master, flat.shadow] + [v for v in vars(self.opt).values() if isinstance(v, torch.Tensor)]
            saved = [t.detach().to("cpu", copy=True) for t in state]
            s = torch.cuda.Stream(device=self.device)
            s.wait_stream(torch.cuda.current_stream(self.device))
            with torch.cuda.stream(s):
                for _ in range(2):
                    self._body(self.idx_buf, self.tgt_buf)
            torch.cuda.current_stream(self.device).wait_stream(s)
            self.graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph):
                self._body(self.idx_buf, self.tgt_buf)
            with torch.no_grad():
                for t, c in zip(state, saved):
                    t.copy_(c)  # in place: the graph holds these buffers
        self.graph.replay()

    def train_step(self, idx, tgt) -> float:
        """Public API: one step on this data-parallel rank's tokens; returns the loss (last stage;
        0.0 on earlier stages)."""
        self.run_step(idx, tgt)
        return float(self.loss.item())

    def close(self):
        self.graph = None  # a graph holding NCCL calls must go before the process group
        if hasattr(self.x, "close"):
            self.x.close()
        if self.dp is not None:
            self.dp.close()
