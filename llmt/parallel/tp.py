"""Tensor parallelism with sequence parallelism (Megatron-style), executed for real.

The reference only models TP (perf_model/roofline.py:136-160 shards heads, kv heads, ffn and
vocabulary by `tp`; perf_model/scaling.py:151-153 charges four all-reduces per layer). Here
each rank of a tensor-parallel group of size tp holds:

  qkv   the rows of its H/tp query heads, KV/tp key heads and KV/tp value heads
  wo    the matching H/tp * hd input columns                    (row-parallel)
  w1,w3 ffn/tp rows each, w2 the matching ffn/tp input columns
  emb   vocabulary rows [r V/tp, (r+1) V/tp)                    (vocabulary-parallel)
  head  the same vocabulary rows
  norms replicated; their gradients are summed over the group after the backward

and the residual stream is split by token rows (sequence parallelism): rank r keeps rows
[r N/tp, (r+1) N/tp) of the N = B*T tokens, so norms and residual adds touch only N/tp rows.
Per block:

  n1  = rmsnorm(x_r)            -> all-gather rows -> qkv GEMM (+RoPE) -> flash attention
      -> wo GEMM (partial sums) -> reduce-scatter rows -> x_r += ...
  n2  = rmsnorm(x_r)            -> all-gather rows -> w1||w3 GEMM + SwiGLU -> w2 GEMM
      -> reduce-scatter rows    -> x_r += ...

The embedding is vocabulary-parallel (each rank looks up the ids it owns, zeros elsewhere,
and the reduce-scatter that enters the residual stream sums the shards), and so is the head:
each rank computes logits for its vocabulary slice of all N rows, the log-sum-exp is
combined across ranks from the (N,) per-shard values and the target logit comes from the
rank that owns it, so no rank ever holds (N, V) logits.

Each rank's local weights form an ordinary LlamaModel of the *local* shape (H/tp heads,
kv/tp, ffn/tp, V/tp, explicit head_dim), so FlatParams, the fused AdamW, ZeRO-1 over the
data-parallel group and the checkpoint code apply unchanged; `shard_state` / `unshard_state`
convert between the full reference state_dict layout and the shards.
"""
from __future__ import annotations

from dataclasses import replace

import torch
import torch.distributed as dist
import torch.nn.functional as F

from llmt.config import ModelConfig
from llmt.models.llama import LlamaModel, build_model
from llmt.parallel.collectives import gather_rows, scatter_rows


def local_config(cfg: ModelConfig, tp: int) -> ModelConfig:
    for name, v in (("heads", cfg.H), ("kv heads", cfg.kvh), ("ffn", cfg.ffn), ("vocab", cfg.vocab)):
        if v % tp:
            raise ValueError(f"tensor parallel {tp} does not divide {name} = {v}")
    return replace(cfg, H=cfg.H // tp, kv_heads=cfg.kvh // tp, ffn=cfg.ffn // tp, vocab=cfg.vocab // tp,
                   head_dim=cfg.hd)


def _qkv_rows(cfg: ModelConfig, tp: int, r: int):
    hd, H, KV = cfg.hd, cfg.H, cfg.kvh
    hl, kl = H // tp, KV // tp
    return [(r * hl * hd, (r + 1) * hl * hd), (H * hd + r * kl * hd, H * hd + (r + 1) * kl * hd),
            ((H + KV) * hd + r * kl * hd, (H + KV) * hd + (r + 1) * kl * hd)]


def shard_tensor(name: str, t: torch.Tensor, cfg: ModelConfig, tp: int, r: int) -> torch.Tensor:
    """This rank's shard of one full-model tensor (state_dict key `name`)."""
    if name.endswith("attn.qkv.weight"):
        return torch.cat([t[a:b] for a, b in _qkv_rows(cfg, tp, r)], 0)
    if name.endswith("attn.wo.weight") or name.endswith("mlp.w2.weight"):
        n = t.shape[1] // tp
        return t[:, r * n:(r + 1) * n]
    if name.endswith("mlp.w1.weight") or name.endswith("mlp.w3.weight") or name in ("emb.weight", "head.weight"):
        n = t.shape[0] // tp
        return t[r * n:(r + 1) * n]
    return t  # norms: replicated


def shard_state(full: dict, cfg: ModelConfig, tp: int, r: int) -> dict:
    return {k: shard_tensor(k, v, cfg, tp, r).contiguous() for k, v in full.items()}


def unshard_state(shards: list, cfg: ModelConfig) -> dict:
    """Full reference-layout state_dict from every rank's shard dict (rank order)."""
    tp = len(shards)
    out = {}
    for k in shards[0]:
        ts = [s[k] for s in shards]
        if k.endswith("attn.qkv.weight"):
            hd = cfg.hd
            hl, kl = cfg.H // tp * hd, cfg.kvh // tp * hd
            q = [t[:hl] for t in ts]
            kk = [t[hl:hl + kl] for t in ts]
            v = [t[hl + kl:] for t in ts]
            out[k] = torch.cat(q + kk + v, 0)
        elif k.endswith("attn.wo.weight") or k.endswith("mlp.w2.weight"):
            out[k] = torch.cat(ts, 1)
        elif k.endswith("mlp.w1.weight") or k.endswith("mlp.w3.weight") or k in ("emb.weight", "head.weight"):
            out[k] = torch.cat(ts, 0)
        else:
            out[k] = ts[0]
    return out


def build_local_model(cfg: ModelConfig, max_seq: int, tp: int, r: int, seed: int = 0, device="cpu",
                      init: str = "full") -> LlamaModel:
    """The LlamaModel of this rank's shard.

    init="full": build the full model with the reference's seeded init on the CPU and slice it,
                 so the TP job starts from exactly the single-GPU weights (tests, parity);
    init="local": initialise the shard directly on `device`, N(0, 0.02) seeded by (seed, r) --
                 the large shapes (Llama-3-8B) never exist whole on one host."""
    lcfg = local_config(cfg, tp)
    if init == "full":
        full = build_model(cfg, max_seq, seed=seed, device="cpu")
        local = LlamaModel(lcfg, max_seq)
        local.load_state_dict(shard_state(full.state_dict(), cfg, tp, r))
        return local.to(device)
    if init != "local":
        raise ValueError(f"unknown init {init!r}")
    with torch.device(device):
        torch.manual_seed(seed * 1000 + r)
        local = LlamaModel(lcfg, max_seq)
    return local.to(device)  # the rope tables are built on the CPU


def replicated_params(model: LlamaModel):
    """Parameters every tensor-parallel rank holds whole (the RMSNorm weights)."""
    ps = []
    for blk in model.blocks:
        ps += [blk.norm1.weight, blk.norm2.weight]
    if getattr(model, "norm_f", None) is not None:
        ps.append(model.norm_f.weight)
    return ps


def sync_replicated_grads(model: LlamaModel, group, main_grad: bool = False):
    """Sum the replicated weights' gradients over the tensor-parallel group (each rank saw
    only its token rows), in one all-reduce."""
    if group is None:
        return
    gs = [p.main_grad if main_grad else p.grad for p in replicated_params(model)]
    flat = torch.cat([g.reshape(-1) for g in gs])
    dist.all_reduce(flat, group=group)
    off = 0
    for g in gs:
        n = g.numel()
        g.copy_(flat[off:off + n].view_as(g))
        off += n


# ---------------------------------------------------------------- reference-math path (any device)
class VocabParallelCE(torch.autograd.Function):
    """Mean cross entropy over a vocabulary-sharded head, fp32 logits (plain torch ops).

    Forward: logits of this rank's vocabulary slice, per-shard log-sum-exp combined over the
    group, target logit summed from its owner. Backward computes (softmax - onehot) / N for the
    local slice and returns the partial dh; the all-gather that produced h sums the partials."""

    @staticmethod
    def forward(ctx, h, w, targets, v0, group):
        logits = h.float() @ w.float().t()
        vl = w.shape[0]
        lse_l = torch.logsumexp(logits, dim=1)
        tl_local = targets - v0
        inside = (tl_local >= 0) & (tl_local < vl)
        tl = torch.where(inside, logits.gather(1, tl_local.clamp(0, vl - 1)[:, None])[:, 0], torch.zeros_like(lse_l))
        world = dist.get_world_size(group)
        allse = torch.empty((world,) + tuple(lse_l.shape), dtype=lse_l.dtype, device=lse_l.device)
        dist.all_gather(list(allse.unbind(0)), lse_l.contiguous(), group=group)
        lse = torch.logsumexp(allse, dim=0)
        dist.all_reduce(tl, group=group)
        ctx.save_for_backward(h, w, logits, lse, tl_local, inside)
        return (lse - tl).mean()

    @staticmethod
    def backward(ctx, g):
        h, w, logits, lse, tl_local, inside = ctx.saved_tensors
        p = torch.exp(logits - lse[:, None])
        rows = torch.nonzero(inside)[:, 0]
        p[rows, tl_local[rows]] -= 1.0
        p *= g / logits.shape[0]
        dh = (p @ w.float()).to(h.dtype)
        dw = (p.t() @ h.float()).to(w.dtype)
        return dh, dw, None, None, None


class TPTorchLlama(torch.nn.Module):
    """Sequence + tensor parallel forward of a local-shard LlamaModel with plain torch ops (fp32 on
    the CPU with gloo): the oracle for the native path and the CPU test of the sharding math."""

    def __init__(self, local: LlamaModel, group):
        super().__init__()
        self.m = local
        self.group = group

    def forward(self, idx, targets):
        m, g = self.m, self.group
        tp, r = dist.get_world_size(g), dist.get_rank(g)
        B, T = idx.shape
        vl, d = m.emb.weight.shape
        v0 = r * vl
        ids = idx.reshape(-1) - v0
        inside = (ids >= 0) & (ids < vl)
        emb = F.embedding(ids.clamp(0, vl - 1), m.emb.weight) * inside[:, None]
        x = scatter_rows(emb, g)
        cos, sin = m.rope_cos[:T], m.rope_sin[:T]
        for blk in m.blocks:
            h = gather_rows(blk.norm1(x), g).view(B, T, d)
            x = x + scatter_rows(blk.attn(h, cos, sin).reshape(B * T, d), g)
            h2 = gather_rows(blk.norm2(x), g)
            x = x + scatter_rows(blk.mlp(h2), g)
        hf = gather_rows(m.norm_f(x), g)
        return VocabParallelCE.apply(hf, m.head.weight, targets.reshape(-1), v0, g)


# ---------------------------------------------------------------- native path (sm_100a kernels)
def _lowp_regions(linear, cos, sin, B, T, cfg):
    """The block's three linear regions (qkv + attention, wo, SwiGLU MLP) with low-precision
    block linears: tensorwise e4m3 (fp8) or block-scaled MXFP8 / NVFP4, the same functions the
    single-shard model uses. Returns (qkv_attention(x, w), linear(x, w), mlp(x, w1, w2))."""
    if linear == "fp8":
        from llmt.ops import fp8 as F8
        return (lambda x, w: F8.QKVAttentionFP8.apply(x, w, cos, sin, B, T, cfg.H, cfg.kvh, cfg.hd),
                F8.LinearFP8.apply,
                lambda x, w1, w2: F8.SwiGLUMLPFP8.apply(x, w1, w2, cfg.ffn))
    from llmt.ops import mx as MX
    from llmt.ops import native as N
    kind = N.MXFP8 if linear == "mxfp8" else N.NVFP4
    return (lambda x, w: MX.QKVAttentionMX.apply(x, w, cos, sin, B, T, cfg.H, cfg.kvh, cfg.hd, kind),
            lambda x, w: MX.LinearMX.apply(x, w, kind),
            lambda x, w1, w2: MX.SwiGLUMLPMX.apply(x, w1, w2, cfg.ffn, kind))


def native_tp_block(blk, a, r, cos, sin, B, T, cfg, group, comm=None, i=0, linear="bf16"):
    """One block on the native kernels over a tensor-parallel group: NCCL row collectives
    (comm None), or peer-memory ones with the row-parallel GEMMs storing to their owners
    (comm = TPPeerComm; all-gather sites 2i and 2i+1). group None: no tensor parallelism.
    linear: "bf16", or "fp8" / "mxfp8" / "nvfp4" block linears (NCCL collectives only: the
    peer-memory collectives are fused into the bf16 GEMMs). Each rank quantizes its own shards;
    NVFP4's per-tensor scale and tensorwise fp8's scale then come from the shard's amax."""
    if linear != "bf16" and comm is not None:
        raise ValueError("low-precision block linears run with NCCL tensor-parallel collectives "
                         "(tp_comm='nccl'); the peer-memory collectives are fused into the bf16 GEMMs")
    from llmt.ops import functions as Fn
    from llmt.parallel.tp_p2p import AllGatherP2P, RowLinearRS
    if linear != "bf16":
        qkv_attn, lin, mlp = _lowp_regions(linear, cos, sin, B, T, cfg)
        if a is None:
            n1, s1 = Fn.RMSNormFn.apply(r, blk.norm1.weight, cfg.eps), r
        else:
            n1, s1 = Fn.AddRMSNormFn.apply(a, r, blk.norm1.weight, cfg.eps)
        o = qkv_attn(gather_rows(n1, group), blk.attn.qkv.weight)
        att = scatter_rows(lin(o, blk.attn.wo.weight), group)
        n2, s2 = Fn.AddRMSNormFn.apply(att, s1, blk.norm2.weight, cfg.eps)
        return scatter_rows(mlp(gather_rows(n2, group), blk.mlp.w1.weight, blk.mlp.w2.weight), group), s2
    if a is None:
        n1, s1 = Fn.RMSNormFn.apply(r, blk.norm1.weight, cfg.eps), r
    else:
        n1, s1 = Fn.AddRMSNormFn.apply(a, r, blk.norm1.weight, cfg.eps)
    n1g = AllGatherP2P.apply(n1, comm, 2 * i) if comm is not None else gather_rows(n1, group)
    o = Fn.QKVAttention.apply(n1g, blk.attn.qkv.weight, cos, sin, B, T, cfg.H, cfg.kvh, cfg.hd)
    if comm is not None:
        att = RowLinearRS.apply(o, blk.attn.wo.weight, comm)
    else:
        att = scatter_rows(Fn.Linear.apply(o, blk.attn.wo.weight), group)
    n2, s2 = Fn.AddRMSNormFn.apply(att, s1, blk.norm2.weight, cfg.eps)
    n2g = AllGatherP2P.apply(n2, comm, 2 * i + 1) if comm is not None else gather_rows(n2, group)
    if comm is not None:
        return Fn.SwiGLUMLP.apply(n2g, blk.mlp.w1.weight, blk.mlp.w2.weight, cfg.ffn, comm), s2
    mo = Fn.SwiGLUMLP.apply(n2g, blk.mlp.w1.weight, blk.mlp.w2.weight, cfg.ffn)
    return scatter_rows(mo, group), s2

class TPNativeLlama:
    """The sequence + tensor parallel step on the native kernels (bf16 GEMMs, flash attention,
    fused norms, vocabulary-parallel fused head + CE). Row collectives between the regions run
    over NCCL (comm="nccl") or over NVLink peer memory fused with their producers
    (comm="p2p": the wo / w2 GEMMs store their rows straight to the owner ranks). Same
    interface as NativeLlama: forward(idx, targets) -> mean loss, every weight gradient
    accumulated into its parameter's main_grad."""

    def __init__(self, local: LlamaModel, group, ce_chunk: int = 8192, pad_to: int = 1, ckpt: bool = False,
                 comm: str = "nccl", linear: str = "bf16"):
        from llmt.models.native import FlatParams
        self.model = local
        self.cfg = local.cfg
        self.group = group
        self.ckpt = ckpt
        self.ce_chunk = ce_chunk
        dev = local.emb.weight.device
        if dev.type != "cuda":
            raise RuntimeError("the native path runs on CUDA (sm_100a) only")
        self.flat = FlatParams(local, dev, pad_to=pad_to)
        self.tp = dist.get_world_size(group) if group is not None else 1
        self.r = dist.get_rank(group) if group is not None else 0
        self.comm_kind = comm
        self.comm = None  # TPPeerComm, built on the first forward (needs the token count)
        if linear not in ("bf16", "fp8", "mxfp8", "nvfp4"):
            raise ValueError(f"linear must be bf16, fp8, mxfp8 or nvfp4, not {linear!r}")
        if linear != "bf16" and comm == "p2p":
            raise ValueError("low-precision block linears run with NCCL tensor-parallel collectives (comm='nccl')")
        self.linear = linear

    def _peer_comm(self, rows):
        if self.comm_kind != "p2p" or self.group is None:
            return None
        if self.comm is None or self.comm.rows != rows:
            from llmt.parallel.tp_p2p import TPPeerComm
            if self.comm is not None:
                self.comm.close()
            self.comm = TPPeerComm(self.group, rows, self.cfg.d, 2 * len(self.model.blocks),
                                   self.model.emb.weight.device)
        return self.comm

    def forward(self, idx, targets):
        from llmt.ops import functions as Fn
        cfg, m, g = self.cfg, self.model, self.group
        B, T = idx.shape
        if (B * T) % self.tp:
            raise ValueError(f"{B * T} tokens do not split over tensor parallel {self.tp}")
        comm = self._peer_comm(B * T)
        cos = m.rope_cos[:T].contiguous()
        sin = m.rope_sin[:T].contiguous()
        v0 = self.r * m.emb.weight.shape[0]
        x = scatter_rows(Fn.EmbedVP.apply(idx.reshape(-1), m.emb.weight, v0), g)
        a, r = None, x
        for i, blk in enumerate(m.blocks):
            if self.ckpt and torch.is_grad_enabled():
                a, r = torch.utils.checkpoint.checkpoint(native_tp_block, blk, a, r, cos, sin, B, T, cfg, g, comm, i,
                                                      self.linear, use_reentrant=False, preserve_rng_state=False)
            else:
                a, r = native_tp_block(blk, a, r, cos, sin, B, T, cfg, g, comm, i, self.linear)
        h = Fn.FinalNormFn.apply(a, r, m.norm_f.weight, cfg.eps)
        return Fn.HeadCEVP.apply(gather_rows(h, g), m.head.weight, targets.reshape(-1), v0, g, self.ce_chunk)

    def sync_replicated_grads(self):
        sync_replicated_grads(self.model, self.group, main_grad=True)

    def close(self):
        if self.comm is not None:
            self.comm.close()
            self.comm = None

    __call__ = forward
