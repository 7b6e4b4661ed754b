"""Multi-GPU numerics check of data parallelism (run under torchrun, one rank per GPU).

Each rank trains the tiny256 model on its own batch with DataParallel in the given mode;
rank 0 also trains the same model alone on the concatenated batches as micro-batches (the
same averaged gradient) and compares the fp32 master weights after a few steps. Prints one
JSON line; exit code 0 when the relative error is within the bound.

    torchrun --nproc-per-node 2 -m llmt.parallel.dp_check --mode fused
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
    p.add_argument("--mode", default="fused", choices=["fused", "nccl", "fused-overlap", "nvls", "nvls-overlap"])
    p.add_argument("--steps", type=int, default=3)
    p.add_argument("--graph", action="store_true")
    args = p.parse_args()
    from llmt.config import get_config
    from llmt.models.llama import make_batch
    from llmt.ops import native
    from llmt.parallel.dp import DataParallel
    from llmt.train import Trainer
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    cfg = get_config("tiny256")
    B, T = 2, 128
    batches = [make_batch(B, T, cfg.vocab, "cpu", seed=r) for r in range(world)]
    dp = DataParallel(world, rank, mode=args.mode)
    tr = Trainer(cfg, B, T, device=f"cuda:{local}", cuda_graph=args.graph, dp=dp)
    for _ in range(args.steps):
        tr.train_step(*batches[rank])
    torch.cuda.synchronize()
    err_code = native.ext().dp_error_code(False)
    # gather the sharded fp32 masters into every rank's view
    f = tr.net.flat
    dp.gather_master(tr.opt)
    full = f.master
    ok = True
    res = {"mode": args.mode, "world": world, "dp_error_code": err_code}
    if rank == 0:
        ref = Trainer(cfg, B * world, T, device=f"cuda:{local}", cuda_graph=False, microbatches=world)
        idx = torch.cat([b[0] for b in batches])
        tgt = torch.cat([b[1] for b in batches])
        for _ in range(args.steps):
            ref.train_step(idx, tgt)
        # compare parameter by parameter: the data-parallel buffer is padded to a multiple of the
        # world size, the single-GPU one is not, so the flat offsets differ
        rf = ref.net.flat
        got = torch.cat([full[o:o + p.numel()] for p, o in zip(f.params, f.offsets)])
        want = torch.cat([rf.master[o:o + p.numel()] for p, o in zip(rf.params, rf.offsets)])
        rel = ((got - want).norm() / want.norm()).item()
        # bf16 shadows every rank uses must equal the master shard rounding
        sh = torch.cat([f.shadow[o:o + p.numel()].float() for p, o in zip(f.params, f.offsets)])
        sh_rel = ((sh - got).norm() / got.norm()).item()
        res.update(rel_err_master=rel, rel_err_shadow=sh_rel)
        ok = rel < 2e-3 and sh_rel < 1e-2 and err_code == 0
        res["ok"] = ok
        print(json.dumps(res), flush=True)
    tr.release()
    dp.close()
    dist.barrier()
    dist.destroy_process_group()
    sys.exit(0 if ok else 1)


if __name__ == "__main__":
    main()
