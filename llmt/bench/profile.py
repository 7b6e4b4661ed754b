"""Where the GPU time of one training step goes (the reference's profile_step.py, native path).

Times the step cleanly first (CUDA events, no profiler), then records a few steps with
torch.profiler (CUPTI) and prints: the top kernels (calls and ms per step, % of GPU time), a
bucket breakdown, launches per step and GPU idle vs the clean step. Buckets follow the
reference's classifier (profile_step.py:44-68) with attention matched before matmul, plus a
`communication` bucket for collective / fused-collective kernels. Kernel names of this
framework carry bucket keywords (gemm_*, flash_*, adamw_*, *rmsnorm*, dp_* / nccl).

    python -m llmt.bench.profile --size medium --batch 4 --seq 1024 [--graph] [--json out.json]
    python -m llmt.bench.profile --impl reference --ref-row "5 + torch.compile"   # a reference row
Profiler numbers are for the breakdown only (shares); the clean step time is the figure.
"""
from __future__ import annotations

import argparse
import json
import statistics
from collections import defaultdict

import torch
from torch.autograd import DeviceType
from torch.profiler import ProfilerActivity, profile

BUCKETS = [
    ("attention", ("flash", "fmha", "attention", "sdpa", "attn")),
    ("communication", ("nccl", "dp_fused", "allreduce", "reduce_scatter", "all_gather", "p2p", "coll_")),
    ("matmul", ("gemm", "cutlass", "cublas", "nvjet", "xmma", "matmul")),
    ("optimizer", ("adam", "multi_tensor", "multitensor")),
    ("memory copies", ("memcpy", "memset", "copy_kernel", "direct_copy", "copy")),
]
OTHER = "elementwise and other"
BUCKET_NAMES = [b for b, _ in BUCKETS] + [OTHER]
WRAPPER_PREFIXES = ("aten::", "autograd::", "Optimizer", "ProfilerStep", "cudaLaunch", "cuda", "Memcpy", "Memset")


def bucket_of(name: str) -> str:
    low = name.lower()
    for bucket, keys in BUCKETS:
        if any(k in low for k in keys):
            return bucket
    return OTHER


def short_name(name: str, n=110) -> str:
    name = name.replace("llmt::", "").replace("(anonymous namespace)::", "").replace("gemm_detail::", "")
    return name if len(name) <= n else name[: n - 3] + "..."


def union_us(intervals):
    """Time during which at least one interval is open (kernels on concurrent streams overlap and
    must not be counted twice): a sweep over the start (+1) and end (-1) boundaries, summing the
    stretches where the open count is positive."""
    edges = sorted([(s, 1) for s, _ in intervals] + [(e, -1) for _, e in intervals],
                   key=lambda t: (t[0], -t[1]))
    busy, depth, opened = 0.0, 0, 0.0
    for t, step in edges:
        if depth == 0 and step > 0:
            opened = t
        depth += step
        if depth == 0:
            busy += t - opened
    return busy


def clean_ms(step, warmup=3, steps=10):
    """Median ms of one step with no profiler attached (an event pair per step, read at the end)."""
    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(steps + 1)]
    ev[0].record()
    for i in range(steps):
        step()
        ev[i + 1].record()
    torch.cuda.synchronize()
    return statistics.median(ev[i].elapsed_time(ev[i + 1]) for i in range(steps))


def profile_step(step, prof_steps=3, top=25, trace=None):
    """Kernel shares of `prof_steps` profiled steps; trace: also write the profiler timeline as a
    Chrome trace (JSON, viewable in chrome://tracing or Perfetto)."""
    with profile(activities=[ProfilerActivity.CPU, ProfilerActivity.CUDA]) as prof:
        for _ in range(prof_steps):
            step()
        torch.cuda.synchronize()
    if trace:
        prof.export_chrome_trace(trace)
    kern = [e for e in prof.events() if e.device_type == DeviceType.CUDA and not e.name.startswith(WRAPPER_PREFIXES)]
    per = defaultdict(lambda: [0, 0.0])
    buckets = defaultdict(float)
    intervals = []
    for e in kern:
        dur = e.time_range.end - e.time_range.start
        per[e.name][0] += 1
        per[e.name][1] += dur
        buckets[bucket_of(e.name)] += dur
        intervals.append((e.time_range.start, e.time_range.end))
    total = sum(v[1] for v in per.values())
    rows = sorted(per.items(), key=lambda kv: -kv[1][1])[:top]
    return {
        "gpu_ms_per_step": total / 1000.0 / prof_steps,
        "busy_ms_per_step": union_us(intervals) / 1000.0 / prof_steps,
        "launches_per_step": sum(v[0] for v in per.values()) / prof_steps,
        "buckets_pct": {b: round(100.0 * buckets[b] / max(total, 1e-9), 2) for b in BUCKET_NAMES},
        "top": [{"kernel": short_name(k), "calls": v[0] / prof_steps, "ms": round(v[1] / 1000.0 / prof_steps, 4),
                 "pct": round(100.0 * v[1] / max(total, 1e-9), 2), "bucket": bucket_of(k)} for k, v in rows],
    }


def reference_step(size, batch, seq, row_name):
    """One training step of a reference ladder row, built by the installed reference's own
    build() (bench_train.py:436-500) from baseline/_ref."""
    import os
    import sys
    ref = os.path.join(os.path.dirname(__file__), "..", "..", "baseline", "_ref")
    sys.path.insert(0, os.path.abspath(ref))
    import bench_train as bt
    row = dict(bt.LADDER)[row_name]
    run = dict(name=row_name, size=size, batch=batch, seq=seq, ckpt=False, nvtx=False, lr=3e-4, **row)
    _, _, step = bt.build(bt.SIZES[size], run, device="cuda")
    return step


def main():
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--size", default="medium")
    p.add_argument("--batch", type=int, default=4)
    p.add_argument("--seq", type=int, default=1024)
    p.add_argument("--graph", action="store_true", help="profile CUDA-graph replays instead of eager steps")
    p.add_argument("--prof-steps", type=int, default=3)
    p.add_argument("--top", type=int, default=25)
    p.add_argument("--json", default=None)
    p.add_argument("--impl", default="native", choices=["native", "reference"])
    p.add_argument("--ref-row", default="5 + torch.compile", help="reference ladder row for --impl reference")
    p.add_argument("--linear", default="bf16", choices=["bf16", "fp8", "mxfp8", "nvfp4"])
    p.add_argument("--trace", default=None, help="write the profiled steps' timeline as a Chrome trace (JSON)")
    p.add_argument("--once", action="store_true",
                   help="run one warm-up step and one step, then exit (a short program for ncu launch lists)")
    args = p.parse_args()
    if args.impl == "reference":
        step = reference_step(args.size, args.batch, args.seq, args.ref_row)
    else:
        from llmt.config import get_config
        from llmt.models.llama import make_batch
        from llmt.train import Trainer
        cfg = get_config(args.size)
        tr = Trainer(cfg, args.batch, args.seq, cuda_graph=args.graph, linear=args.linear)
        idx, tgt = make_batch(args.batch, args.seq, cfg.vocab, "cuda")
        tr.set_batch(idx, tgt)
        step = tr.run_step
    if args.once:
        for _ in range(2):
            step()
        torch.cuda.synchronize()
        print("two steps done")
        return
    ms = clean_ms(step)
    res = profile_step(step, args.prof_steps, args.top, trace=args.trace)
    res["clean_ms_per_step"] = ms
    res["idle_pct"] = round(100.0 * (1 - res["busy_ms_per_step"] / ms), 2) if ms > 0 else None
    res["config"] = {"size": args.size, "batch": args.batch, "seq": args.seq, "graph": args.graph,
                     "impl": args.impl, **({"ref_row": args.ref_row} if args.impl == "reference" else {})}
    print(f"clean step {ms:.3f} ms | GPU kernel time {res['gpu_ms_per_step']:.3f} ms | "
          f"launches/step {res['launches_per_step']:.0f} | idle {res['idle_pct']}%")
    for b, v in res["buckets_pct"].items():
        print(f"  {b:24s} {v:6.2f}%")
    for r in res["top"]:
        print(f"  {r['ms']:8.4f} ms {r['pct']:6.2f}% x{r['calls']:5.1f}  {r['kernel']}")
    if args.json:
        with open(args.json, "w") as f:
            json.dump(res, f, indent=1)


if __name__ == "__main__":
    main()
