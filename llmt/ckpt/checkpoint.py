"""Checkpoint save / resume with the reference state_dict layout.

The reference saves nothing (its .gitignore excludes *.pt); the layout kept here is what its
LlamaModel.state_dict() produces (bench_train.py:187-202: emb.weight, blocks.{i}.norm1.weight,
blocks.{i}.attn.qkv.weight, ..., norm_f.weight, head.weight; rope tables not persistent) and
the optimizer state is torch.optim.AdamW's ({"state": {i: {step, exp_avg, exp_avg_sq}},
"param_groups": [...]}), so a checkpoint loads into the reference model and optimizer too.

Two formats:
  gathered  one file `<path>` with {"model", "optimizer", "meta"} -- ZeRO-1 shards (masters and
            Adam state) are gathered to rank 0 first
  sharded   `<path>.rank{r}` per rank with its flat shard, plus `<path>.index.json`
"""
from __future__ import annotations

import json
import os

import torch
import torch.distributed as dist


def _world():
    if dist.is_available() and dist.is_initialized():
        return dist.get_world_size(), dist.get_rank()
    return 1, 0


def _full_flat(buf_shard, numel, world):
    """All-gather equal shards of a flat buffer into the full buffer."""
    full = torch.empty(numel, dtype=buf_shard.dtype, device=buf_shard.device)
    dist.all_gather_into_tensor(full, buf_shard.contiguous())
    return full


def _flat_opt_state(opt, flat):
    """(exp_avg, exp_avg_sq, step) as full-length flat fp32 buffers (gathering ZeRO-1 shards)."""
    world, _ = _world()
    step = int(opt.step_t.item())
    if hasattr(opt, "ranges"):  # BucketShardedAdamW: chunk r of every bucket
        m = torch.zeros(flat.numel, dtype=torch.float32, device=flat.master.device)
        v = torch.zeros_like(m)
        for (lo, hi), moff in zip(flat.buckets, opt.moffs):
            c = (hi - lo) // world
            dist.all_gather_into_tensor(m[lo:hi], opt.exp_avg[moff:moff + c].contiguous())
            dist.all_gather_into_tensor(v[lo:hi], opt.exp_avg_sq[moff:moff + c].contiguous())
        opt.gather_master()
        return m, v, step, flat.master
    if hasattr(opt, "lo"):  # ShardedAdamW
        m = _full_flat(opt.exp_avg, flat.numel, world)
        v = _full_flat(opt.exp_avg_sq, flat.numel, world)
        master = _full_flat(flat.master[opt.lo:opt.hi], flat.numel, world)
    else:
        m, v, master = opt.exp_avg, opt.exp_avg_sq, flat.master
    return m, v, step, master


def state_dicts(model, opt=None, flat=None):
    """(model state_dict with reference keys, AdamW-format optimizer state) on the CPU."""
    master = None
    st = {}
    if opt is not None and flat is not None:
        m, v, step, master = _flat_opt_state(opt, flat)
        for i, (p, o) in enumerate(zip(flat.params, flat.offsets)):
            n = p.numel()
            st[i] = {"step": torch.tensor(float(step)), "exp_avg": m[o:o + n].view(p.shape).cpu().clone(),
                     "exp_avg_sq": v[o:o + n].view(p.shape).cpu().clone()}
    sd = {}
    for k, t in model.state_dict().items():
        sd[k] = t.detach().cpu().clone()
    if master is not None:  # masters of other ranks' shards are only current after the gather
        for name, p, o in zip(flat.names, flat.params, flat.offsets):
            sd[name] = master[o:o + p.numel()].view(p.shape).cpu().clone()
    osd = None
    if opt is not None:
        b1, b2 = opt.betas
        names = flat.names if flat is not None else []
        osd = {"state": st, "param_groups": [{"lr": float(opt.lr_t.item()), "betas": (b1, b2), "eps": opt.eps,
                                              "weight_decay": opt.weight_decay, "params": list(range(len(names))),
                                              "param_names": names}]}
    return sd, osd


def save(path, model, opt=None, flat=None, meta=None, sharded=False):
    world, rank = _world()
    if sharded and flat is not None and opt is not None and hasattr(opt, "lo"):
        torch.save({"lo": opt.lo, "hi": opt.hi, "master": flat.master[opt.lo:opt.hi].cpu(),
                    "exp_avg": opt.exp_avg.cpu(), "exp_avg_sq": opt.exp_avg_sq.cpu(),
                    "step": int(opt.step_t.item()), "lr": float(opt.lr_t.item())}, f"{path}.rank{rank}")
        if rank == 0:
            with open(f"{path}.index.json", "w") as f:
                json.dump({"world": world, "numel": flat.numel, "names": flat.names, "offsets": flat.offsets,
                           "shapes": [list(p.shape) for p in flat.params], "meta": meta or {}}, f)
        return
    sd, osd = state_dicts(model, opt, flat)
    if rank == 0:
        tmp = path + ".tmp"
        torch.save({"model": sd, "optimizer": osd, "meta": meta or {}}, tmp)
        os.replace(tmp, path)
    if world > 1:
        dist.barrier()


def load(path, model, opt=None, flat=None, sharded=False):
    """Restore weights (and optimizer state). Refreshes the bf16 shadow weights when `flat` is given."""
    world, rank = _world()
    if sharded:
        shard = torch.load(f"{path}.rank{rank}", map_location="cpu")
        flat.master[shard["lo"]:shard["hi"]].copy_(shard["master"])
        opt.exp_avg.copy_(shard["exp_avg"])
        opt.exp_avg_sq.copy_(shard["exp_avg_sq"])
        opt.step_t.fill_(shard["step"])
        opt.set_lr(shard["lr"])
        full = _full_flat(flat.master[opt.lo:opt.hi], flat.numel, world)
        flat.master.copy_(full)
        flat.refresh_shadow()
        return {}
    ck = torch.load(path, map_location="cpu")
    with torch.no_grad():
        model.load_state_dict(ck["model"])
    if opt is not None and ck.get("optimizer") and flat is not None:
        st = ck["optimizer"]["state"]
        lo, hi = (opt.lo, opt.hi) if hasattr(opt, "lo") else (0, flat.numel)
        for i, (p, o) in enumerate(zip(flat.params, flat.offsets)):
            s = st.get(i)
            if s is None:
                continue
            n = p.numel()
            a, b = max(o, lo), min(o + n, hi)  # overlap of this parameter with the local shard
            if a >= b:
                continue
            opt.exp_avg[a - lo:b - lo].copy_(s["exp_avg"].reshape(-1)[a - o:b - o])
            opt.exp_avg_sq[a - lo:b - lo].copy_(s["exp_avg_sq"].reshape(-1)[a - o:b - o])
            opt.step_t.fill_(int(float(s["step"])))
        opt.set_lr(ck["optimizer"]["param_groups"][0]["lr"])
    if flat is not None:
        flat.refresh_shadow()
    return ck.get("meta", {})
