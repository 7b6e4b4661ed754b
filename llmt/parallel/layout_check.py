"""Multi-GPU numerics check of a data x tensor x pipeline layout on the native kernels
(torchrun, one rank per GPU).

Every rank runs ParallelTrainer (tiny256, stages sliced from the same seeded full model) on its
data-parallel rank's batch; rank 0 also trains the unsharded model alone on all data-parallel
batches as micro-batches (the same averaged gradient). After a few steps every stage's shard of
the fp32 masters is gathered, reassembled into the reference layout and compared. One JSON
line; exit code 0 when within the bound.

    torchrun --nproc-per-node 8 -m llmt.parallel.layout_check --dp 2 --tp 2 --pp 2 --microbatches 4
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import sys

import torch
import torch.distributed as dist


def main():
    p = argparse.ArgumentParser()
    p.add_argument("--dp", type=int, default=1)
    p.add_argument("--tp", type=int, default=1)
    p.add_argument("--pp", type=int, default=2)
    p.add_argument("--microbatches", type=int, default=4)
    p.add_argument("--steps", type=int, default=3)
    p.add_argument("--dp-mode", default="nccl", choices=["nccl", "fused"])
    p.add_argument("--tp-comm", default="nccl", choices=["nccl", "p2p"])
    p.add_argument("--graph", action="store_true")
    p.add_argument("--seq", type=int, default=128, help="sequence length (peer-memory tensor parallelism fuses "
                   "its all-gathers into the GEMMs when a micro-batch gives each rank whole 128-row blocks)")
    args = p.parse_args()
    from llmt.config import get_config
    from llmt.models.llama import make_batch
    from llmt.ops import native
    from llmt.parallel.engine import ParallelTrainer
    from llmt.parallel.groups import Layout
    from llmt.parallel.tp import unshard_state
    from llmt.train import Trainer
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    cfg = get_config("tiny256", kv_heads=2)
    B, T = args.microbatches, args.seq
    batches = [make_batch(B, T, cfg.vocab, "cpu", seed=d) for d in range(args.dp)]
    lay = Layout(dp=args.dp, tp=args.tp, pp=args.pp)
    tr = ParallelTrainer(cfg, B, T, lay, microbatches=args.microbatches, device=f"cuda:{local}",
                         dp_mode=args.dp_mode, tp_comm=args.tp_comm, cuda_graph=args.graph)
    g = tr.groups
    losses = [tr.train_step(*batches[g.dp_rank]) for _ in range(args.steps)]
    torch.cuda.synchronize()
    codes = {"gemm": native.gemm_error_code(), "attn": native.attn_error_code(), "dp": native.ext().dp_error_code(False)}
    # ZeRO-1 keeps other ranks' master shards stale on this rank: gather the data-parallel
    # shards first so every rank holds its stage's current masters
    if tr.dp is not None:
        tr.dp.gather_master(tr.opt)
    mine = {k: v.detach().float().cpu() for k, v in tr.stage.global_state_dict().items()}
    allsd = [None] * world
    dist.all_gather_object(allsd, {"coords": (g.dp_rank, g.pp_rank, g.tp_rank), "sd": mine, "losses": losses})
    ok = True
    if rank == 0:
        merged = {}
        for s in range(args.pp):
            shards = [next(x["sd"] for x in allsd if x["coords"] == (0, s, t)) for t in range(args.tp)]
            merged.update(unshard_state(shards, cfg) if args.tp > 1 else shards[0])
        last_losses = next(x["losses"] for x in allsd if x["coords"] == (0, args.pp - 1, 0))
        ref = Trainer(cfg, B * args.dp, T, device=f"cuda:{local}", cuda_graph=False,
                      microbatches=args.microbatches * args.dp)
        idx = torch.cat([b[0] for b in batches])
        tgt = torch.cat([b[1] for b in batches])
        ref_losses = [ref.train_step(idx, tgt) for _ in range(args.steps)]
        rsd = ref.model.state_dict()
        num = sum(float((merged[k].to(rsd[k].device) - rsd[k].float()).norm() ** 2) for k in rsd)
        den = sum(float(rsd[k].float().norm() ** 2) for k in rsd)
        rel = (num / den) ** 0.5
        ok = rel < 2e-3 and all(v == 0 for v in codes.values())
        print(json.dumps({"layout": f"dp{args.dp} tp{args.tp} pp{args.pp}", "microbatches": args.microbatches,
                          "tp_comm": args.tp_comm, "graph": args.graph,
                          "rel_err_master": rel, "losses_last_stage_dp0": last_losses, "ref_losses": ref_losses,
                          "error_codes": codes, "ok": ok}), flush=True)
    tr.close()
    dist.barrier()
    dist.destroy_process_group()
    sys.exit(0 if ok else 1)


if __name__ == "__main__":
    main()
