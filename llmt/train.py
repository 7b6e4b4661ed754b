"""Training engine: model + fused optimizer + (optionally) one CUDA graph per step.

`Trainer` is the public API of the native path:

    tr = Trainer(get_config("medium"), batch=4, seq=1024)
    loss = tr.train_step(idx, targets)      # idx/targets on the host (pinned) or device

One step = forward + backward + AdamW over every parameter, exactly the reference's step()
(bench_train.py:474-490). With cuda_graph=True the whole step (all kernels, including the
optimizer and the data-parallel collectives) is captured once after warm-up and replayed,
which removes the per-kernel launch cost the reference pays from Python (its profile shows
1177-4033 launches per step, README.md:53-62, :117-125). Inputs are copied into static
device buffers before each replay.
"""
from __future__ import annotations

import torch

from llmt.config import ModelConfig
from llmt.models.llama import build_model
from llmt.models.native import NativeLlama
from llmt.ops import functions as Fn
from llmt.ops import native
from llmt.optim.adamw import FusedAdamW


class Trainer:
    """tp_group: tensor + sequence parallel group (the model is then this rank's shard, see
    llmt.parallel.tp); dp: a DataParallel over the data-parallel group (ZeRO-1)."""

    def __init__(self, cfg: ModelConfig, batch: int, seq: int, device="cuda", seed: int = 0, lr: float = 3e-4,
                 cuda_graph: bool = True, microbatches: int = 1, dp=None, ce_chunk: int = 8192, ckpt: bool = False,
                 tp_group=None, init: str = "full", nvtx: bool = False, linear: str = "bf16",
                 first_write: bool = True):
        self.cfg, self.batch, self.seq = cfg, batch, seq
        self.linear = linear
        self.nvtx = nvtx  # NVTX ranges forward / backward / optimizer per step (eager steps; reference --nvtx)
        self.device = torch.device(device)
        self.microbatches = microbatches
        self.dp = dp
        self.tp_group = tp_group
        pad_to = dp.world_size if dp is not None else 1
        if tp_group is not None:
            import torch.distributed as dist
            from llmt.parallel.tp import TPNativeLlama, build_local_model
            tp, r = dist.get_world_size(tp_group), dist.get_rank(tp_group)
            self.model = build_local_model(cfg, seq, tp, r, seed=seed, device=self.device, init=init)
            self.net = TPNativeLlama(self.model, tp_group, ce_chunk=ce_chunk, pad_to=pad_to, ckpt=ckpt, linear=linear)
        else:
            self.model = build_model(cfg, seq, seed=seed, device=self.device)
            overlap = dp is not None and getattr(dp, "overlap", False)
            self.net = NativeLlama(self.model, ce_chunk=ce_chunk, pad_to=pad_to, ckpt=ckpt, nvtx=nvtx,
                                   bucket_pad=overlap, linear=linear)
            if overlap:
                if ckpt:
                    raise ValueError("the overlapped data-parallel step needs ckpt=False")
                self.net.grad_ready = dp.bucket_ready
        flat = self.net.flat
        # First-write gradients (llmt.ops.functions.GRAD): the first micro-batch's backward stores
        # every weight gradient, so nothing clears the 4-byte-per-parameter buffer between steps.
        # Off for the tensor-parallel model, whose collectives' writers always accumulate.
        self.first_write = first_write and tp_group is None
        if dp is not None:
            self.opt = dp.make_optimizer(flat, lr=lr)
            dp.zero_grads = not self.first_write
        else:
            self.opt = FusedAdamW(flat.master, flat.grad, flat.shadow, lr=lr, zero_grad=not self.first_write)
        mb = batch // microbatches
        if mb * microbatches != batch:
            raise ValueError("batch must be a multiple of microbatches")
        self.idx = torch.zeros((microbatches, mb, seq), dtype=torch.long, device=self.device)
        self.tgt = torch.zeros((microbatches, mb, seq), dtype=torch.long, device=self.device)
        self.loss = torch.zeros((), dtype=torch.float32, device=self.device)
        self.use_graph = cuda_graph
        self.graph = None
        self.body_calls = 0

    # ------------------------------------------------------------------ step body
    def _range(self, name):
        if self.nvtx:
            torch.cuda.nvtx.range_push(name)

    def _end(self):
        if self.nvtx:
            torch.cuda.nvtx.range_pop()

    def _body(self):
        self.body_calls += 1
        total = None
        for i in range(self.microbatches):
            self._range("forward")
            loss = self.net(self.idx[i], self.tgt[i])
            self._end()
            self._range("backward")
            if self.dp is not None and i == self.microbatches - 1:
                self.dp.begin_step()  # the last micro-batch's backward releases the buckets
            Fn.GRAD["first"] = self.first_write and i == 0
            try:
                (loss / self.microbatches).backward()
            finally:
                Fn.GRAD["first"] = False
            self._end()
            total = loss.detach() if total is None else total + loss.detach()
        self._range("optimizer")
        if self.tp_group is not None:
            self.net.sync_replicated_grads()
        if self.dp is not None:
            self.dp.reduce_and_step(self.opt)
        else:
            self.opt.step()
        self._end()
        self.loss.copy_(total / self.microbatches)
        if self.linear == "nvfp4":
            native.sr_counter(self.device).add_(1)  # new stochastic-rounding noise every step (graph too)

    def _state_tensors(self):
        """The tensors one step changes: weights (fp32 master, bf16 shadow) and the optimizer's
        state (moments, step count). Communication state (barrier epochs) is not included: the
        peers track it."""
        flat = self.net.flat
        ts = [flat.master, flat.shadow]
        ts += [v for v in vars(self.opt).values() if isinstance(v, torch.Tensor)]
        return ts

    def _capture(self, warmup=2):
        """Warm up (allocator, tensor maps, NCCL communicators) with `warmup` eager steps, capture
        one step, then put the weights and the optimizer state back as they were, so the first
        train_step is one step like every other."""
        state = self._state_tensors()
        need = sum(t.numel() * t.element_size() for t in state)
        free, _ = torch.cuda.mem_get_info(self.device)
        where = self.device if free > 2 * need + (4 << 30) else torch.device("cpu")
        saved = [t.detach().to(where, copy=True) for t in state]
        s = torch.cuda.Stream(device=self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):
            for _ in range(warmup):
                self._body()
        torch.cuda.current_stream(self.device).wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self._body()
        self.graph = g
        with torch.no_grad():
            for t, c in zip(state, saved):
                t.copy_(c)  # in place: the graph holds these buffers
        del saved

    def set_batch(self, idx, tgt):
        """Copy one step's tokens (B, T) into the static device buffers (async from pinned memory)."""
        self.idx.copy_(idx.view(self.idx.shape), non_blocking=True)
        self.tgt.copy_(tgt.view(self.tgt.shape), non_blocking=True)

    def run_step(self):
        """One training step on the current static batch (device-side; no host sync)."""
        if not self.use_graph:
            self._body()
            return
        if self.graph is None:
            self._capture()
        self.graph.replay()

    def train_step(self, idx, tgt) -> float:
        """Public API: H2D copy of the batch, one step, D2H read of the loss."""
        self.set_batch(idx, tgt)
        self.run_step()
        return float(self.loss.item())

    def release(self):
        self.graph = None
