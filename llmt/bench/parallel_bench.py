"""Throughput of a data x tensor x pipeline layout on the native path, against the scaling
model's prediction for that exact layout (torchrun, one rank per GPU).

Times K steps after W warm-up steps with CUDA events between barriers on every rank and
reports the maximum over ranks; synthetic uniform-random tokens, random-init weights (each
shard initialised on its GPU). The prediction is llmt.perf.scaling.evaluate() for the same
model, sequence, global batch, layout and micro-batch size.

    torchrun --nproc-per-node 8 -m llmt.bench.parallel_bench --model llama3-8b --seq 4096 \\
        --global-batch 16 --dp 2 --tp 2 --pp 2 --microbatches 4
"""
from __future__ import annotations

import argparse
import datetime
import json
import os

import torch
import torch.distributed as dist


def main():
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--model", default="llama3-8b")
    p.add_argument("--seq", type=int, default=4096)
    p.add_argument("--global-batch", type=int, default=16)
    p.add_argument("--dp", type=int, default=1)
    p.add_argument("--tp", type=int, default=1)
    p.add_argument("--pp", type=int, default=1)
    p.add_argument("--microbatches", type=int, default=1)
    p.add_argument("--steps", type=int, default=5)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--dp-mode", default="auto", choices=["auto", "nvls", "nccl", "fused"],
                   help="data-parallel transport (auto: nvls where NVLink multicast exists, else nccl)")
    p.add_argument("--json", default=None)
    p.add_argument("--calibrate", action="store_true",
                   help="also predict from this rank's GEMM / attention shapes timed on the GPU")
    p.add_argument("--graph", action="store_true", help="capture the step in a CUDA graph (pp = 1 only)")
    p.add_argument("--tp-comm", default="nccl", choices=["nccl", "p2p"],
                   help="tensor-parallel row collectives: NCCL, or NVLink peer memory fused with the GEMMs")
    p.add_argument("--linear", default="bf16", choices=["bf16", "fp8", "mxfp8", "nvfp4"],
                   help="block linears (low precision with NCCL tensor-parallel collectives only)")
    p.add_argument("--tp-gather", default="fused", choices=["fused", "separate"],
                   help="peer-memory all-gathers inside the consuming GEMMs, or as their own kernel + barrier")
    args = p.parse_args()
    os.environ["LLMT_TP_FUSE_GATHER"] = "1" if args.tp_gather == "fused" else "0"
    from llmt.config import get_config, model_flops_per_token
    from llmt.parallel.engine import ParallelTrainer
    from llmt.parallel.groups import Layout
    rank, world = int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))
    cfg = get_config(args.model)
    lay = Layout(dp=args.dp, tp=args.tp, pp=args.pp)
    B = args.global_batch // args.dp
    tr = ParallelTrainer(cfg, B, args.seq, lay, microbatches=args.microbatches, device=f"cuda:{local}",
                         init="local", dp_mode=args.dp_mode, cuda_graph=args.graph, tp_comm=args.tp_comm,
                         linear=args.linear)
    dp_mode = tr.dp.mode if tr.dp is not None else None  # what "auto" resolved to
    g = torch.Generator().manual_seed(1 + tr.groups.dp_rank)
    idx = torch.randint(0, cfg.vocab, (B, args.seq), generator=g).pin_memory()
    tgt = torch.randint(0, cfg.vocab, (B, args.seq), generator=g).pin_memory()
    for _ in range(max(3, args.warmup)):
        tr.train_step(idx, tgt)
    dist.barrier()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(args.steps):
        tr.train_step(idx, tgt)
    b.record()
    torch.cuda.synchronize()
    dist.barrier()
    ms = torch.tensor([a.elapsed_time(b) / args.steps], device="cuda")
    dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    mem = torch.tensor([torch.cuda.max_memory_allocated() / 1e9], device="cuda")
    dist.all_reduce(mem, op=dist.ReduceOp.MAX)
    step_s = ms.item() / 1e3
    tokens = args.global_batch * args.seq
    res = {"model": args.model, "seq": args.seq, "global_batch": args.global_batch,
           "layout": f"dp{args.dp} tp{args.tp} pp{args.pp}", "microbatches": args.microbatches, "n_gpus": world,
           "cuda_graph": bool(tr.use_graph), "tp_comm": args.tp_comm, "dp_mode": dp_mode,
           "tp_gather": args.tp_gather if args.tp_comm == "p2p" else None, "linear": args.linear,
           "ms_per_step": round(ms.item(), 3), "tokens_per_s": round(tokens / step_s, 1),
           "mfu_vs_measured_bf16": None, "peak_mem_gb": round(mem.item(), 2),
           "dtype": "bf16" if args.linear == "bf16" else f"{args.linear} block linears, bf16 rest",
           "data": "synthetic uniform-random tokens, random-init weights", "timing": "CUDA events, max over ranks"}
    if rank == 0:
        try:
            from llmt.bench.kernels import peaks
            from llmt.perf.roofline import Machine
            from llmt.perf.scaling import StageCompute, evaluate, load_links
            peak, hbm = peaks()
            res["mfu_vs_measured_bf16"] = round(model_flops_per_token(cfg, args.seq) * tokens / step_s / world
                                                / (peak * 1e12), 4)
            machine = Machine.from_peaks(sustained=True)
            comp = StageCompute(cfg, args.seq, machine)
            pred = evaluate(cfg, args.seq, args.global_batch, world, args.dp, args.tp, args.pp,
                            B // args.microbatches, comp, load_links(), "b200_nvl8_ib")
            if pred:
                res["predicted_ms_per_step"] = round(pred["step_s"] * 1e3, 3)
                res["prediction_error"] = round(pred["step_s"] / step_s - 1, 4)
                res["predicted_breakdown_ms"] = {k: round(v * 1e3, 3) for k, v in pred["breakdown_s"].items()}
            if args.calibrate:
                # the same prediction with this rank's GEMM / attention shapes timed on the GPU
                from llmt.perf.roofline import inventory, measure_shape_times
                ops = inventory(cfg, B // args.microbatches, args.seq, "native", tp=args.tp)
                st = measure_shape_times(ops, "/tmp/llmt_shape_times.json")
                comp_c = StageCompute(cfg, args.seq, machine, shape_times=st)
                pc = evaluate(cfg, args.seq, args.global_batch, world, args.dp, args.tp, args.pp,
                              B // args.microbatches, comp_c, load_links(), "b200_nvl8_ib")
                if pc:
                    res["predicted_calibrated_ms_per_step"] = round(pc["step_s"] * 1e3, 3)
                    res["calibrated_prediction_error"] = round(pc["step_s"] / step_s - 1, 4)
        except Exception as e:  # noqa: BLE001
            res["prediction_unavailable"] = str(e)[:200]
        print(json.dumps(res), flush=True)
        if args.json:
            with open(args.json, "w") as f:
                json.dump(res, f, indent=1)
    tr.close()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
