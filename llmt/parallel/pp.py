"""Pipeline parallelism: 1F1B over NCCL point-to-point, executed for real.

The reference only models PP: stage compute plus a bubble of (p-1)/(m+p-1)
(perf_model/scaling.py:155-161) and the 1F1B order of its exported graphs
(workload_export/export_trace.py:125-131). Here each pipeline rank owns a contiguous run of
blocks (`StageModel`: the first stage also the embedding, the last also norm_f and the head)
and runs the same 1F1B order (llmt.export.trace.schedule_1f1b, shared with the exporter):

  warm-up   min(p - s - 1, m) forwards, each activation sent to the next stage
  steady    forward of micro-batch w + j, backward of micro-batch j
  cool-down the remaining backwards

A forward send and the backward receive that follows it (and a backward send with the next
forward receive) go out as one batched NCCL group (batch_isend_irecv): issued one after the
other, two neighbouring stages would each block in a send to the other. Groups that only send
(the warm-up forwards, the last backward) are not waited for on the compute stream: the next
micro-batch's compute overlaps the transfer, and the step waits for them at its end. The stage boundary
carries what the block stack carries: the native path's (pending branch output bf16, fp32
residual) pair, the reference-math path's fp32 residual. Tensor parallelism composes: each
stage is itself sharded over its tensor-parallel group and sends its sequence rows to the
same tensor-parallel rank of the next stage.
"""
from __future__ import annotations

import torch
import torch.distributed as dist
import torch.nn as nn
import torch.nn.functional as F

from llmt.config import ModelConfig
from llmt.export.trace import schedule_1f1b
from llmt.models.llama import Block, RMSNorm, build_model, rope_tables
from llmt.parallel.collectives import gather_rows, scatter_rows


def stage_layers(L: int, pp: int, s: int):
    """Blocks [l0, l1) of stage s; the first L % pp stages take one extra block."""
    base, extra = divmod(L, pp)
    l0 = s * base + min(s, extra)
    return l0, l0 + base + (1 if s < extra else 0)


class StageModel(nn.Module):
    """Blocks [l0, l1) of a (possibly tensor-parallel local) model, the embedding on the first
    stage and norm_f + head on the last. Parameter names keep the global block index, so
    state_dict keys are the reference's."""

    def __init__(self, cfg: ModelConfig, max_seq: int, l0: int, l1: int, first: bool, last: bool):
        super().__init__()
        self.cfg, self.l0, self.l1, self.first, self.last = cfg, l0, l1, first, last
        self.block_offset = l0
        self.blocks = nn.ModuleList([Block(cfg) for _ in range(l1 - l0)])
        self.emb = nn.Embedding(cfg.vocab, cfg.d) if first else None
        self.norm_f = RMSNorm(cfg.d, cfg.eps) if last else None
        self.head = nn.Linear(cfg.d, cfg.vocab, bias=False) if last else None
        cos, sin = rope_tables(max_seq, cfg.hd, cfg.rope_base, device="cpu")
        self.register_buffer("rope_cos", cos, persistent=False)
        self.register_buffer("rope_sin", sin, persistent=False)
        for m in self.modules():
            if isinstance(m, (nn.Linear, nn.Embedding)):
                nn.init.normal_(m.weight, mean=0.0, std=0.02)

    def global_state_dict(self):
        out = {}
        for k, v in self.state_dict().items():
            if k.startswith("blocks."):
                i, rest = k[len("blocks."):].split(".", 1)
                k = f"blocks.{int(i) + self.l0}.{rest}"
            out[k] = v
        return out

    def load_global(self, full: dict):
        own = {}
        for k in self.state_dict():
            if k.startswith("blocks."):
                i, rest = k[len("blocks."):].split(".", 1)
                own[k] = full[f"blocks.{int(i) + self.l0}.{rest}"]
            else:
                own[k] = full[k]
        self.load_state_dict(own)


def build_stage(cfg: ModelConfig, max_seq: int, pp: int, s: int, tp: int = 1, tp_rank: int = 0, seed: int = 0,
                device="cpu", init: str = "full") -> StageModel:
    """This rank's stage (tensor-parallel shard when tp > 1). init="full" slices the seeded full
    model (exact single-GPU weights); init="local" initialises the shard on the device."""
    from llmt.parallel.tp import local_config, shard_state
    lcfg = local_config(cfg, tp) if tp > 1 else cfg
    l0, l1 = stage_layers(cfg.L, pp, s)
    if init == "full":
        full = build_model(cfg, max_seq, seed=seed, device="cpu").state_dict()
        if tp > 1:
            full = shard_state(full, cfg, tp, tp_rank)
        st = StageModel(lcfg, max_seq, l0, l1, s == 0, s == pp - 1)
        st.load_global(full)
        return st.to(device)
    with torch.device(device):
        torch.manual_seed(seed * 1000 + s * 100 + tp_rank)
        st = StageModel(lcfg, max_seq, l0, l1, s == 0, s == pp - 1)
    return st.to(device)  # the rope tables are built on the CPU


# ---------------------------------------------------------------- stage executors
class TorchStage:
    """Reference-math stage (fp32 torch ops; CPU tests). Boundary activation: (x,)."""

    def __init__(self, stage: StageModel, tp_group=None):
        self.m, self.g = stage, tp_group

    def forward_first(self, idx):
        m, g = self.m, self.g
        if g is None:
            return m.emb(idx.reshape(-1))
        vl = m.emb.weight.shape[0]
        ids = idx.reshape(-1) - dist.get_rank(g) * vl
        inside = (ids >= 0) & (ids < vl)
        return scatter_rows(F.embedding(ids.clamp(0, vl - 1), m.emb.weight) * inside[:, None], g)

    def forward_blocks(self, acts, B, T):
        m, g = self.m, self.g
        (x,) = acts if isinstance(acts, tuple) else (acts,)
        d = m.cfg.d
        cos, sin = m.rope_cos[:T], m.rope_sin[:T]
        for blk in m.blocks:
            h = gather_rows(blk.norm1(x), g).view(B, T, d)
            x = x + scatter_rows(blk.attn(h, cos, sin).reshape(B * T, d), g)
            x = x + scatter_rows(blk.mlp(gather_rows(blk.norm2(x), g)), g)
        return (x,)

    def forward_last(self, acts, targets):
        from llmt.parallel.tp import VocabParallelCE
        m, g = self.m, self.g
        (x,) = acts
        if g is None:
            return F.cross_entropy(m.head(m.norm_f(x)).float(), targets.reshape(-1))
        v0 = dist.get_rank(g) * m.head.weight.shape[0]
        return VocabParallelCE.apply(gather_rows(m.norm_f(x), g), m.head.weight, targets.reshape(-1), v0, g)

    def act_specs(self, rows):
        return [((rows, self.m.cfg.d), torch.float32)]


class NativeStage:
    """Stage on the native kernels (flat fp32 master / grad, bf16 shadow; every weight gradient
    into main_grad). Boundary activation: (pending branch output bf16, fp32 residual)."""

    def __init__(self, stage: StageModel, tp_group=None, pad_to: int = 1, ce_chunk: int = 8192, comm: str = "nccl",
                 in_flight: int = 1, linear: str = "bf16"):
        from llmt.models.native import FlatParams
        self.m, self.g, self.ce_chunk = stage, tp_group, ce_chunk
        self.comm_kind, self.comm = comm, None
        # micro-batches between their forward and their backward at once (the pipeline depth):
        # peer-memory gathers keep one set of site buffers per such micro-batch
        self.in_flight = in_flight
        self.micro = 0
        if linear not in ("bf16", "fp8", "mxfp8", "nvfp4"):
            raise ValueError(f"linear must be bf16, fp8, mxfp8 or nvfp4, not {linear!r}")
        if linear != "bf16" and comm == "p2p" and tp_group is not None:
            raise ValueError("low-precision block linears run with NCCL tensor-parallel collectives (tp_comm='nccl')")
        self.linear = linear  # block linears of the stage's blocks (the head stays bf16)
        self.flat = FlatParams(stage, stage.rope_cos.device if stage.emb is None else stage.emb.weight.device,
                               pad_to=pad_to)
        self.tp_rank = dist.get_rank(tp_group) if tp_group is not None else 0

    def forward_first(self, idx):
        from llmt.ops import functions as Fn
        m, g = self.m, self.g
        if g is None:
            return Fn.Embed.apply(idx.reshape(-1), m.emb.weight)
        v0 = self.tp_rank * m.emb.weight.shape[0]
        return scatter_rows(Fn.EmbedVP.apply(idx.reshape(-1), m.emb.weight, v0), g)

    def forward_blocks(self, acts, B, T):
        from llmt.parallel.tp import native_tp_block
        m, g, cfg = self.m, self.g, self.m.cfg
        a, r = acts if isinstance(acts, tuple) else (None, acts)
        cos = m.rope_cos[:T].contiguous()
        sin = m.rope_sin[:T].contiguous()
        comm = self._peer_comm(B * T)
        if comm is not None:
            comm.select_set(self.micro)
        for i, blk in enumerate(m.blocks):
            a, r = native_tp_block(blk, a, r, cos, sin, B, T, cfg, g, comm, i, self.linear)
        return (a, r)

    def _peer_comm(self, rows):
        if self.comm_kind != "p2p" or self.g is None:
            return None
        if self.comm is None or self.comm.rows != rows:
            from llmt.parallel.tp_p2p import TPPeerComm
            if self.comm is not None:
                self.comm.close()
            self.comm = TPPeerComm(self.g, rows, self.m.cfg.d, 2 * len(self.m.blocks), self.flat.master.device,
                                   sets=self.in_flight)
        return self.comm

    def close(self):
        if self.comm is not None:
            self.comm.close()
            self.comm = None

    def forward_last(self, acts, targets):
        from llmt.ops import functions as Fn
        m, g, cfg = self.m, self.g, self.m.cfg
        a, r = acts
        h = Fn.FinalNormFn.apply(a, r, m.norm_f.weight, cfg.eps)
        if g is None:
            return Fn.HeadCE.apply(h, m.head.weight, targets.reshape(-1), self.ce_chunk)
        v0 = self.tp_rank * m.head.weight.shape[0]
        return Fn.HeadCEVP.apply(gather_rows(h, g), m.head.weight, targets.reshape(-1), v0, g, self.ce_chunk)

    def act_specs(self, rows):
        d = self.m.cfg.d
        return [((rows, d), torch.bfloat16), ((rows, d), torch.float32)]


# ---------------------------------------------------------------- 1F1B schedule
class Pipeline1F1B:
    """Runs one step of micro-batches through this rank's stage in the 1F1B order.

    `prev` / `next` are the global ranks of the neighbouring stages (same tensor-parallel and
    data-parallel coordinates). Returns the mean loss on the last stage, None elsewhere."""

    def __init__(self, executor, stage_idx: int, pp: int, prev: int | None, nxt: int | None, pp_group, device):
        self.x, self.s, self.pp = executor, stage_idx, pp
        self.prev, self.next, self.group, self.device = prev, nxt, pp_group, torch.device(device)
        self.first, self.last = stage_idx == 0, stage_idx == pp - 1
        self._inflight = []  # send-only groups not waited for yet: (requests, tensors)

    def _empty(self, rows):
        return [torch.empty(shape, dtype=dt, device=self.device) for shape, dt in self.x.act_specs(rows)]

    def _batch(self, sends, recvs, peer_send, peer_recv):
        """One NCCL group of sends to peer_send and receives from peer_recv. A group with receives
        is waited for, which with NCCL is a dependency of the compute stream on the transfer (the
        host does not block: it goes on queuing the consumer's kernels, which run when the data
        has arrived); a send-only group is not waited for at all: the compute stream goes on with
        the next micro-batch while the transfer runs, and the group is waited for at the end of
        the step (its tensors are kept alive until then)."""
        sends = [t.contiguous() for t in sends]
        ops = [dist.P2POp(dist.isend, t, peer_send, self.group) for t in sends]
        ops += [dist.P2POp(dist.irecv, t, peer_recv, self.group) for t in recvs]
        if not ops:
            return
        reqs = dist.batch_isend_irecv(ops)
        if recvs:
            for req in reqs:
                req.wait()
        else:
            self._inflight.append((reqs, sends))

    def _drain(self):
        for reqs, _ in self._inflight:
            for req in reqs:
                req.wait()
        self._inflight.clear()

    def step(self, idx, tgt):
        """idx, tgt: (m, mb, T) micro-batches of this data-parallel rank."""
        m_count, mb, T = idx.shape
        rows = mb * T
        if self.x.g is not None:
            rows //= dist.get_world_size(self.x.g)
        inputs, outputs, losses = [None] * m_count, [None] * m_count, []

        def fwd(i, acts_in):
            self.x.micro = i  # the executor's per-micro-batch buffers (peer-memory gathers)
            if self.first:
                acts = self.x.forward_blocks(self.x.forward_first(idx[i]), mb, T)
            else:
                for t in acts_in:
                    t.requires_grad_(True)
                acts = self.x.forward_blocks(tuple(acts_in), mb, T)
            inputs[i] = acts_in
            if self.last:
                loss = self.x.forward_last(acts, tgt[i])
                losses.append(loss.detach())
                outputs[i] = loss / m_count
                return None
            outputs[i] = acts
            return acts

        def bwd(i, grads):
            if self.last:
                outputs[i].backward()
            else:
                torch.autograd.backward(list(outputs[i]), list(grads))
            g_in = None if self.first else [t.grad for t in inputs[i]]
            inputs[i] = outputs[i] = None
            return g_in

        def recv_fwd():
            if self.first:
                return None
            bufs = self._empty(rows)
            self._batch([], bufs, None, self.prev)
            return bufs

        def send_fwd(acts):
            if not self.last:
                self._batch(list(acts), [], self.next, None)

        def send_fwd_recv_bwd(acts):
            if self.last:
                return None
            bufs = self._empty(rows)
            self._batch(list(acts), bufs, self.next, self.next)
            return bufs

        specs = self.x.act_specs(rows)

        def as_specs(g):  # gradients leave in the boundary dtypes the receiver expects
            return [t.to(dt) for t, (_, dt) in zip(g, specs)]

        def send_bwd(g):
            if not self.first:
                self._batch(as_specs(g), [], self.prev, None)

        def send_bwd_recv_fwd(g):
            if self.first:
                return None
            bufs = self._empty(rows)
            self._batch(as_specs(g), bufs, self.prev, self.prev)
            return bufs

        def recv_bwd():
            if self.last:
                return None
            bufs = self._empty(rows)
            self._batch([], bufs, None, self.next)
            return bufs

        # the executed order is schedule_1f1b(s, p, m): warm-up forwards, (F, B) pairs, cool-down
        self.order = []
        warm = min(self.pp - self.s - 1, m_count)
        for i in range(warm):
            self.order.append(("F", i))
            send_fwd(fwd(i, recv_fwd()))
        rem = m_count - warm
        acts_in = recv_fwd() if rem > 0 else None
        for j in range(rem):
            self.order += [("F", warm + j), ("B", j)]
            out = fwd(warm + j, acts_in)
            g_in = bwd(j, send_fwd_recv_bwd(out))
            if j == rem - 1:
                send_bwd(g_in)
            else:
                acts_in = send_bwd_recv_fwd(g_in)
        for j in range(rem, m_count):
            self.order.append(("B", j))
            send_bwd(bwd(j, recv_bwd()))
        assert self.order == schedule_1f1b(self.s, self.pp, m_count)
        self._drain()
        return torch.stack(losses).mean() if self.last else None
