"""Reference-stack multi-GPU baseline for the Llama-3-8B-shaped configs (torchrun, one rank per GPU).

The reference trains on one GPU only (plain PyTorch modules, bf16 autocast, SDPA, fused AdamW;
bench_train.py:187-228, :458-492). This is that stack scaled out the stock PyTorch way, with
none of this framework's kernels or engine on the path:

  model     the reference's module structure (pre-norm RMSNorm, packed qkv, rotate-half RoPE,
            SDPA, SwiGLU, untied head) written with module calls so PyTorch's parallel styles can
            hook them; grouped-query attention from this repository's config, since the
            reference's model has none (Llama-3-8B has 8 KV heads)
  TP        torch.distributed.tensor.parallel: qkv / w1 / w3 column-parallel, wo / w2
            row-parallel with sequence-parallel norms, vocabulary-parallel embedding and head
            with loss_parallel (DTensor over NCCL). The packed qkv rows are laid out per rank
            (each rank's contiguous block is its own q | k | v heads), so column sharding
            hands every rank whole heads
  DP        FSDP2 (fully_shard per block and at the root) over the data-parallel mesh dimension,
            bf16 compute and fp32 reduction (MixedPrecisionPolicy); fp32 masters as the reference
  step      forward + backward + fused torch AdamW (lr 3e-4, betas 0.9 / 0.95, wd 0.1)

Times K steps after W warm-up steps with CUDA events between barriers, max over ranks; synthetic
uniform-random tokens, random-init weights. Pipeline parallelism has no stock equivalent in the
reference's stack and is not run here.

    torchrun --nproc-per-node 2 -m llmt.bench.ref_parallel --model llama3-8b --seq 4096 --global-batch 1 --tp 2
"""
from __future__ import annotations

import argparse
import contextlib
import datetime
import json
import os
from dataclasses import replace

import torch
import torch.distributed as dist
import torch.nn as nn
import torch.nn.functional as F


class Attention(nn.Module):
    def __init__(self, cfg):
        super().__init__()
        self.cfg = cfg  # replaced by the per-rank head counts when tensor parallel
        self.qkv = nn.Linear(cfg.d, cfg.qkv_out, bias=False)
        self.wo = nn.Linear(cfg.H * cfg.hd, cfg.d, bias=False)

    def forward(self, x, cos, sin):
        from llmt.models.llama import rope
        B, T, _ = x.shape
        H, KV, hd = self.cfg.H, self.cfg.kvh, self.cfg.hd
        q, k, v = self.qkv(x).view(B, T, H + 2 * KV, hd).split((H, KV, KV), dim=2)
        q, k, v = (t.transpose(1, 2) for t in (q, k, v))
        y = F.scaled_dot_product_attention(rope(q, cos, sin), rope(k, cos, sin), v, is_causal=True,
                                           enable_gqa=KV != H)
        return self.wo(y.transpose(1, 2).reshape(B, T, H * hd))


class MLP(nn.Module):
    def __init__(self, cfg):
        super().__init__()
        self.w1 = nn.Linear(cfg.d, cfg.ffn, bias=False)
        self.w3 = nn.Linear(cfg.d, cfg.ffn, bias=False)
        self.w2 = nn.Linear(cfg.ffn, cfg.d, bias=False)

    def forward(self, x):
        return self.w2(F.silu(self.w1(x)) * self.w3(x))


class Block(nn.Module):
    def __init__(self, cfg):
        super().__init__()
        from llmt.models.llama import RMSNorm
        self.norm1, self.attn = RMSNorm(cfg.d, cfg.eps), Attention(cfg)
        self.norm2, self.mlp = RMSNorm(cfg.d, cfg.eps), MLP(cfg)

    def forward(self, x, cos, sin):
        x = x + self.attn(self.norm1(x), cos, sin)
        return x + self.mlp(self.norm2(x))


class Llama(nn.Module):
    def __init__(self, cfg, seq):
        super().__init__()
        from llmt.models.llama import RMSNorm, rope_tables
        self.cfg = cfg
        self.emb = nn.Embedding(cfg.vocab, cfg.d)
        self.blocks = nn.ModuleList(Block(cfg) for _ in range(cfg.L))
        self.norm_f = RMSNorm(cfg.d, cfg.eps)
        self.head = nn.Linear(cfg.d, cfg.vocab, bias=False)
        cos, sin = rope_tables(seq, cfg.hd, cfg.rope_base, device="cpu")
        self.register_buffer("rope_cos", cos, persistent=False)
        self.register_buffer("rope_sin", sin, persistent=False)

    def forward(self, idx):
        T = idx.shape[1]
        x = self.emb(idx)
        cos, sin = self.rope_cos[:T], self.rope_sin[:T]
        for blk in self.blocks:
            x = blk(x, cos, sin)
        return self.head(self.norm_f(x))


def parallelize(model, mesh, tp, dp):
    from torch.distributed.tensor import Replicate, Shard
    from torch.distributed.tensor.parallel import (ColwiseParallel, PrepareModuleInput, RowwiseParallel,
                                                   SequenceParallel, parallelize_module)
    if tp > 1:
        tp_mesh = mesh["tp"]
        parallelize_module(model, tp_mesh, {
            "emb": RowwiseParallel(input_layouts=Replicate(), output_layouts=Shard(1)),
            "norm_f": SequenceParallel(),
            "head": ColwiseParallel(input_layouts=Shard(1), output_layouts=Shard(-1), use_local_output=False),
        })
        local = replace(model.cfg, H=model.cfg.H // tp, kv_heads=model.cfg.kvh // tp, head_dim=model.cfg.hd)
        for blk in model.blocks:
            parallelize_module(blk, tp_mesh, {
                "norm1": SequenceParallel(),
                "attn": PrepareModuleInput(input_layouts=(Shard(1), None, None),
                                           desired_input_layouts=(Replicate(), None, None)),
                "attn.qkv": ColwiseParallel(),
                "attn.wo": RowwiseParallel(output_layouts=Shard(1)),
                "norm2": SequenceParallel(),
                "mlp": PrepareModuleInput(input_layouts=(Shard(1),), desired_input_layouts=(Replicate(),)),
                "mlp.w1": ColwiseParallel(),
                "mlp.w3": ColwiseParallel(),
                "mlp.w2": RowwiseParallel(output_layouts=Shard(1)),
            })
            blk.attn.cfg = local
    if dp > 1:
        from torch.distributed.fsdp import MixedPrecisionPolicy, fully_shard
        mp = MixedPrecisionPolicy(param_dtype=torch.bfloat16, reduce_dtype=torch.float32)
        for blk in model.blocks:
            fully_shard(blk, mesh=mesh["dp"], mp_policy=mp)
        fully_shard(model, mesh=mesh["dp"], mp_policy=mp)
    return model


def main():
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--model", default="llama3-8b")
    p.add_argument("--seq", type=int, default=4096)
    p.add_argument("--global-batch", type=int, default=1)
    p.add_argument("--dp", type=int, default=1)
    p.add_argument("--tp", type=int, default=1)
    p.add_argument("--steps", type=int, default=5)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--compile", action="store_true", help="torch.compile each block (the reference's row 5)")
    p.add_argument("--json", default=None)
    args = p.parse_args()
    from torch.distributed.device_mesh import init_device_mesh
    from llmt.config import get_config, model_flops_per_token
    from llmt.models.llama import init_weights
    rank, world = int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", rank))
    dev = "cuda" if torch.cuda.is_available() else "cpu"  # cpu: gloo, for the host-side tests
    if dev == "cuda":
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))
    else:
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=300))
    if args.dp * args.tp != world:
        raise SystemExit(f"dp x tp = {args.dp * args.tp} != world size {world}")
    mesh = init_device_mesh(dev, (args.dp, args.tp), mesh_dim_names=("dp", "tp"))
    cfg = get_config(args.model)
    torch.manual_seed(0)
    with torch.device("meta"):
        model = Llama(cfg, args.seq)
    model = parallelize(model, mesh, args.tp, args.dp)
    model.to_empty(device=dev)
    from llmt.models.llama import rope_tables
    cos, sin = rope_tables(args.seq, cfg.hd, cfg.rope_base, dev)
    model.rope_cos.copy_(cos)
    model.rope_sin.copy_(sin)
    with torch.no_grad():
        for name, prm in model.named_parameters():
            if prm.dim() == 1:
                prm.fill_(1.0)
    init_weights(model)
    if args.compile:
        for blk in model.blocks:
            blk.compile()
    opt = torch.optim.AdamW(model.parameters(), lr=3e-4, betas=(0.9, 0.95), weight_decay=0.1,
                            **(dict(fused=True) if dev == "cuda" else dict(foreach=True)))
    B = args.global_batch // args.dp
    g = torch.Generator().manual_seed(1 + mesh["dp"].get_local_rank())
    idx = torch.randint(0, cfg.vocab, (B, args.seq), generator=g).to(dev)
    tgt = torch.randint(0, cfg.vocab, (B, args.seq), generator=g).to(dev)

    def step():
        amp = torch.autocast("cuda", dtype=torch.bfloat16) if args.dp == 1 and dev == "cuda" else contextlib.nullcontext()
        if args.tp > 1:
            from torch.distributed.tensor.parallel import loss_parallel
            lp = loss_parallel()
        else:
            lp = contextlib.nullcontext()
        with lp:
            with amp:
                logits = model(idx)
            loss = F.cross_entropy(logits.float().flatten(0, 1), tgt.flatten())
            loss.backward()
        opt.step()
        opt.zero_grad(set_to_none=True)
        return loss

    for _ in range(max(3, args.warmup) if dev == "cuda" else args.warmup):
        step()
    dist.barrier()
    if dev == "cuda":
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
    t0 = __import__("time").perf_counter()
    for _ in range(args.steps):
        loss = step()
    if dev == "cuda":
        b.record()
        torch.cuda.synchronize()
        step_ms = a.elapsed_time(b) / args.steps
    else:
        step_ms = (__import__("time").perf_counter() - t0) * 1e3 / args.steps
    dist.barrier()
    ms = torch.tensor([step_ms], device=dev)
    dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    mem = torch.tensor([torch.cuda.max_memory_allocated() / 1e9 if dev == "cuda" else 0.0], device=dev)
    dist.all_reduce(mem, op=dist.ReduceOp.MAX)
    tokens = args.global_batch * args.seq
    step_s = ms.item() / 1e3
    if rank == 0:
        from llmt.bench.kernels import peaks
        res = {"impl": "reference-stack (stock PyTorch TP / FSDP2)", "model": args.model, "seq": args.seq,
               "global_batch": args.global_batch, "layout": f"dp{args.dp} tp{args.tp} pp1", "n_gpus": world,
               "compile": args.compile, "ms_per_step": round(ms.item(), 3), "tokens_per_s": round(tokens / step_s, 1),
               "mfu_vs_measured_bf16": round(model_flops_per_token(cfg, args.seq) * tokens / step_s / world
                                             / (peaks()[0] * 1e12), 4),
               "peak_mem_gb": round(mem.item(), 2), "final_loss": float((loss.full_tensor() if hasattr(loss, "full_tensor")
                                                                          else loss).detach()),
               "dtype": "bf16 compute, fp32 masters", "data": "synthetic uniform-random tokens, random-init weights",
               "timing": "CUDA events, max over ranks"}
        print(json.dumps(res), flush=True)
        if args.json:
            with open(args.json, "w") as f:
                json.dump(res, f, indent=1)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
