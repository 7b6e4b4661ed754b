"""Native (sm_100a) execution of the reference-layout LlamaModel.

`NativeLlama(model)` keeps the model's nn.Parameters (so state_dict keys and values are
unchanged) but re-points every parameter at a view of one flat fp32 master buffer, with
matching views into a flat fp32 gradient buffer (`p.main_grad`) and a flat bf16 shadow
buffer (`p.w16`) that the GEMMs read and the fused AdamW rewrites every step. Packing
order puts each block's w1 directly before w3, so the merged gate/up GEMM reads one
(2*ffn, d) weight and writes one (2*ffn, d) gradient without any copy. The flat buffers
are also what the data-parallel engine shards (ZeRO-1) and reduce-scatters.

The reference builds the same network from nn.Linear under bf16 autocast with fp32 master
weights (bench_train.py:458-492); this path keeps fp32 masters and the fp32 residual stream,
runs every GEMM in bf16 with fp32 accumulation, and never materializes logits.
"""
from __future__ import annotations

import torch
import torch.utils.checkpoint

from llmt.models.llama import LlamaModel
from llmt.ops import fp8 as F8
from llmt.ops import mx as MX
from llmt.ops import functions as Fn
from llmt.ops import native as N

ALIGN = 64  # elements; keeps every view 256-byte (fp32) / 128-byte (bf16) aligned


def param_order(model: LlamaModel):
    """(name, parameter) in flat-buffer order: per block qkv, wo, w1, w3, w2, norms; then emb, norm_f, head.

    A pipeline stage (llmt.parallel.pp.StageModel) has only some blocks (named by their global
    index, `block_offset`) and lacks emb or norm_f / head."""
    out = []
    base = getattr(model, "block_offset", 0)
    for i, blk in enumerate(model.blocks):
        p = f"blocks.{base + i}."
        out += [(p + "attn.qkv.weight", blk.attn.qkv.weight), (p + "attn.wo.weight", blk.attn.wo.weight),
                (p + "mlp.w1.weight", blk.mlp.w1.weight), (p + "mlp.w3.weight", blk.mlp.w3.weight),
                (p + "mlp.w2.weight", blk.mlp.w2.weight), (p + "norm1.weight", blk.norm1.weight),
                (p + "norm2.weight", blk.norm2.weight)]
    for name in ("emb", "norm_f", "head"):
        mod = getattr(model, name, None)
        if mod is not None:
            out.append((f"{name}.weight", mod.weight))
    return out


class FlatParams:
    """Flat fp32 master / fp32 grad / bf16 shadow storage behind a model's parameters."""

    def __init__(self, model: LlamaModel, device, pad_to: int = 1, bucket_pad: bool = False):
        """pad_to: the buffer length is a multiple of ALIGN * pad_to (data-parallel sharding).
        bucket_pad: every block's parameters, and the trailing emb / norm_f / head group, start and
        end on such a boundary too, so each of these buckets splits into pad_to equal chunks
        (the overlapped data-parallel step shards every bucket); `buckets` lists them in order."""
        self.names = []
        self.params = []
        self.offsets = []
        self.buckets = []
        off = 0
        unit = ALIGN * pad_to
        cur, b_lo = None, 0
        for name, p in param_order(model):
            group = name.split(".")[1] if name.startswith("blocks.") else "tail"
            if bucket_pad and group != cur:
                if cur is not None:
                    off += (-off) % unit
                    self.buckets.append((b_lo, off))
                cur, b_lo = group, off
            if off % ALIGN:
                off += ALIGN - off % ALIGN
            self.names.append(name)
            self.params.append(p)
            self.offsets.append(off)
            off += p.numel()
        if off % unit:
            off += unit - off % unit
        if bucket_pad and cur is not None:
            self.buckets.append((b_lo, off))
        self.numel = off
        dev = torch.device(device)
        self.master = torch.zeros(off, dtype=torch.float32, device=dev)
        with torch.no_grad():
            for p, o in zip(self.params, self.offsets):
                n = p.numel()
                self.master[o:o + n].copy_(p.detach().reshape(-1).to(dev, torch.float32))
                p.data = self.master[o:o + n].view(p.shape)
        self.blocks = list(model.blocks)
        self.rebind(grad=torch.zeros(off, dtype=torch.float32, device=dev),
                    shadow=torch.zeros(off, dtype=torch.bfloat16, device=dev))
        self.refresh_shadow()

    def rebind(self, grad, shadow):
        """Point every parameter's main_grad / w16 (and the merged w1||w3 views) at new flat buffers."""
        self.grad, self.shadow = grad, shadow
        for p, o in zip(self.params, self.offsets):
            n = p.numel()
            p.main_grad = grad[o:o + n].view(p.shape)
            p.w16 = shadow[o:o + n].view(p.shape)
        pos = {id(p): o for p, o in zip(self.params, self.offsets)}
        for blk in self.blocks:
            w1, w3 = blk.mlp.w1.weight, blk.mlp.w3.weight
            o1, o3 = pos[id(w1)], pos[id(w3)]
            if o3 != o1 + w1.numel():
                raise RuntimeError("w1 and w3 must be adjacent in the flat buffer (ffn*d must be a multiple of 64)")
            ffn, d = w1.shape
            w1.w13_16 = shadow[o1:o1 + 2 * ffn * d].view(2 * ffn, d)
            w1.w13 = self.master[o1:o1 + 2 * ffn * d].view(2 * ffn, d)
            w1.w13_grad = grad[o1:o1 + 2 * ffn * d].view(2 * ffn, d)
            w1.w3_param = w3

    def refresh_shadow(self):
        """bf16 shadow := master (after init or a checkpoint load)."""
        N.cast_bf16(self.master, self.shadow)

    def zero_grad(self):
        self.grad.zero_()


class NativeLlama:
    """Runs `model` on the native kernels. forward(idx, targets) -> mean loss (like the reference).

    A plain wrapper (not an nn.Module), so model.state_dict() keeps the reference keys."""

    def __init__(self, model: LlamaModel, ce_chunk: int = 8192, pad_to: int = 1, ckpt: bool = False,
                 nvtx: bool = False, bucket_pad: bool = False, linear: str = "bf16"):
        """linear: "bf16"; "fp8" for the block linears on tensorwise e4m3 operands (llmt.ops.fp8;
        reference --linear fp8, bench_train.py:33-38); "mxfp8" or "nvfp4" (reference --linear fp4)
        for block-scaled operands (llmt.ops.mx). The head stays bf16."""
        if linear not in ("bf16", "fp8", "mxfp8", "nvfp4"):
            raise ValueError(f"linear must be bf16, fp8, mxfp8 or nvfp4, not {linear!r}")
        self.linear = linear
        self.model = model
        # grad_ready(i) is called from the backward once block i's gradients have all been issued
        # (a hook on the gradient of the block's input): the overlapped data-parallel step uses it
        self.grad_ready = None
        self.ckpt = ckpt
        self.nvtx = nvtx  # NVTX range per block (reference bench_train.py:215-222)
        self.cfg = model.cfg
        dev = model.emb.weight.device
        if dev.type != "cuda":
            raise RuntimeError("the native path runs on CUDA (sm_100a) only")
        self.flat = FlatParams(model, dev, pad_to=pad_to, bucket_pad=bucket_pad)
        self.ce_chunk = ce_chunk

    def forward(self, idx, targets):
        cfg, m = self.cfg, self.model
        B, T = idx.shape
        cos = m.rope_cos[:T].contiguous()
        sin = m.rope_sin[:T].contiguous()
        x = Fn.Embed.apply(idx.reshape(-1), m.emb.weight)
        a, r = None, x
        for i, blk in enumerate(m.blocks):
            if self.grad_ready is not None and r.requires_grad and torch.is_grad_enabled():
                r.register_hook(lambda g, i=i: self.grad_ready(i))
            if self.nvtx:
                torch.cuda.nvtx.range_push(f"block{i}")
            if self.ckpt and torch.is_grad_enabled():
                # per-block recompute (reference bench_train.py:217-218): keep only the block input
                a, r = torch.utils.checkpoint.checkpoint(self._block, blk, a, r, cos, sin, B, T, use_reentrant=False,
                                                      preserve_rng_state=False)
            else:
                a, r = self._block(blk, a, r, cos, sin, B, T)
            if self.nvtx:
                torch.cuda.nvtx.range_pop()
        h = Fn.FinalNormFn.apply(a, r, m.norm_f.weight, cfg.eps)
        return Fn.HeadCE.apply(h, m.head.weight, targets.reshape(-1), self.ce_chunk)

    def _block(self, blk, a, r, cos, sin, B, T):
        cfg = self.cfg
        if a is None:
            n1, s1 = Fn.RMSNormFn.apply(r, blk.norm1.weight, cfg.eps), r
        else:
            n1, s1 = Fn.AddRMSNormFn.apply(a, r, blk.norm1.weight, cfg.eps)
        if self.linear in ("mxfp8", "nvfp4"):
            kind = N.MXFP8 if self.linear == "mxfp8" else N.NVFP4
            o = MX.QKVAttentionMX.apply(n1, blk.attn.qkv.weight, cos, sin, B, T, cfg.H, cfg.kvh, cfg.hd, kind)
            att = MX.LinearMX.apply(o, blk.attn.wo.weight, kind)
            n2, s2 = Fn.AddRMSNormFn.apply(att, s1, blk.norm2.weight, cfg.eps)
            return MX.SwiGLUMLPMX.apply(n2, blk.mlp.w1.weight, blk.mlp.w2.weight, cfg.ffn, kind), s2
        if self.linear == "fp8":
            o = F8.QKVAttentionFP8.apply(n1, blk.attn.qkv.weight, cos, sin, B, T, cfg.H, cfg.kvh, cfg.hd)
            att = F8.LinearFP8.apply(o, blk.attn.wo.weight)
            n2, s2 = Fn.AddRMSNormFn.apply(att, s1, blk.norm2.weight, cfg.eps)
            return F8.SwiGLUMLPFP8.apply(n2, blk.mlp.w1.weight, blk.mlp.w2.weight, cfg.ffn), s2
        o = Fn.QKVAttention.apply(n1, blk.attn.qkv.weight, cos, sin, B, T, cfg.H, cfg.kvh, cfg.hd)
        att = Fn.Linear.apply(o, blk.attn.wo.weight)
        n2, s2 = Fn.AddRMSNormFn.apply(att, s1, blk.norm2.weight, cfg.eps)
        return Fn.SwiGLUMLP.apply(n2, blk.mlp.w1.weight, blk.mlp.w2.weight, cfg.ffn), s2

    __call__ = forward
