"""The optimization ladder on this GPU (reference: bench_train.py --sweep, LADDER rows 1-9).

Rows 1-9 are the reference's own rows, run through its own API (bench_train.build /
run_one from the unmodified install under baseline/_ref: fp32 + naive attention, bf16
autocast, SDPA, fused Adam, torch.compile, Triton kernels, CUDA add+RMSNorm, FP8 and NVFP4
linears). The native rows run this framework's Trainer (tcgen05 GEMMs with fused epilogues,
flash attention, fused AdamW, one CUDA graph per step). Step time is the median of the timed
steps; MFU uses the bf16 matmul peak measured in the same run (the reference's convention)
and, separately, the driver-measured peak in MEASURED_PEAKS.json.

    python -m llmt.bench.ladder --size small --batch 8 --seq 1024 [--rows ref,native] --out results/ladder.json
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import time

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def native_rows():
    """Native rows: bf16 (graph, eager, recompute) and the low-precision block linears that match
    the reference's rows 8 (fp8) and 9 (NVFP4), plus MXFP8."""
    return [("N1 native bf16 (graph)", dict(cuda_graph=True, ckpt=False)),
            ("N2 native bf16 (eager launches)", dict(cuda_graph=False, ckpt=False)),
            ("N3 native bf16 + per-block recompute", dict(cuda_graph=True, ckpt=True)),
            ("N4 native + fp8 linears (e4m3 tensorwise)", dict(cuda_graph=True, ckpt=False, linear="fp8")),
            ("N5 native + MXFP8 linears (e4m3, ue8m0 / 32)", dict(cuda_graph=True, ckpt=False, linear="mxfp8")),
            ("N6 native + NVFP4 linears (e2m1, ue4m3 / 16)", dict(cuda_graph=True, ckpt=False, linear="nvfp4"))]


def run_native(size, B, T, opts, warmup, steps):
    from llmt.config import SIZES, model_flops_per_token
    from llmt.models.llama import make_batch
    from llmt.train import Trainer
    cfg = SIZES[size]
    row = {"name": None, "status": "ok"}
    try:
        torch.cuda.reset_peak_memory_stats()
        tr = Trainer(cfg, B, T, cuda_graph=opts["cuda_graph"], ckpt=opts.get("ckpt", False),
                     linear=opts.get("linear", "bf16"))
        idx, tgt = make_batch(B, T, cfg.vocab, "cuda")
        tr.set_batch(idx, tgt)
        for _ in range(warmup):
            tr.run_step()
        ts = []
        for _ in range(steps):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            tr.run_step()
            b.record()
            torch.cuda.synchronize()
            ts.append(a.elapsed_time(b) / 1e3)
        sec = statistics.median(ts)
        tok = B * T
        row.update(ms_per_step=round(sec * 1e3, 3), tokens_per_s=round(tok / sec),
                   tflops=round(model_flops_per_token(cfg, T) * tok / sec / 1e12, 2),
                   peak_mem_gb=round(torch.cuda.max_memory_allocated() / 1e9, 2), final_loss=round(float(tr.loss.item()), 4))
        tr.release()
        del tr
    except torch.cuda.OutOfMemoryError:
        row["status"] = "oom"
    except Exception as e:  # noqa: BLE001 - one row failing must not stop the ladder
        row.update(status="error", error=f"{type(e).__name__}: {e}"[:300])
    torch.cuda.empty_cache()
    return row


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--size", default="small")
    ap.add_argument("--batch", type=int, default=8)
    ap.add_argument("--seq", type=int, default=1024)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--rows", default="ref,native")
    ap.add_argument("--ref-rows", default="1,2,3,4,5,6,7,8,9")
    ap.add_argument("--out", default=None)
    ap.add_argument("--mem-cap", type=float, default=0.97,
                    help="fraction of the GPU's memory the native rows may allocate (like the reference's runs: "
                         "a row that does not fit is recorded as oom instead of spilling)")
    args = ap.parse_args()
    from llmt.bench.calibrate import env_info, matmul_tflops
    from llmt.perf.roofline import Machine
    bref = matmul_tflops("bf16")["tflops"]
    peak_measured = Machine.from_peaks(sustained=False).bf16_tflops
    rows = []
    if "ref" in args.rows:
        ref = os.path.join(ROOT, "baseline", "_ref")
        sys.path.insert(0, ref)
        import bench_train as bt
        cfg = bt.SIZES[args.size]
        base = dict(size=args.size, batch=args.batch, seq=args.seq, ckpt=False, nvtx=False, lr=3e-4)
        want = {int(x) for x in args.ref_rows.split(",")}
        for name, r in bt.LADDER:
            if int(name.split()[0]) not in want:
                continue
            run = dict(name=name, **base, **r)
            print(f"running {name} ...", flush=True)
            row = bt.run_one(cfg, run, args.warmup, args.steps, bref, None)
            row["impl"] = "reference"
            rows.append(row)
            print(json.dumps({k: row.get(k) for k in ("name", "status", "ms_per_step", "tokens_per_s", "mfu")}), flush=True)
    if "native" in args.rows:
        from llmt.config import SIZES, model_flops_per_token
        cfg = SIZES[args.size]
        if 0 < args.mem_cap < 1:
            torch.cuda.set_per_process_memory_fraction(args.mem_cap)  # this process's allocator only
        for name, opts in native_rows():
            print(f"running {name} ...", flush=True)
            row = run_native(args.size, args.batch, args.seq, opts, args.warmup, args.steps)
            row["name"], row["impl"] = name, "native"
            if row["status"] == "ok":
                row["mfu"] = round(row["tflops"] / bref, 4)
            rows.append(row)
            print(json.dumps({k: row.get(k) for k in ("name", "status", "ms_per_step", "tokens_per_s", "mfu")}), flush=True)
    first = next((r for r in rows if r.get("status") == "ok"), None)
    for r in rows:
        if r.get("status") == "ok" and first:
            r["speedup_vs_first"] = round(first["ms_per_step"] / r["ms_per_step"], 2)
            r["mfu_vs_measured_peak"] = round(r["tflops"] / peak_measured, 4)
    try:
        from tabulate import tabulate
        print(tabulate([[r["name"], r.get("ms_per_step", r.get("status")), r.get("tokens_per_s"), r.get("speedup_vs_first"),
                         r.get("mfu")] for r in rows], headers=["row", "ms/step", "tok/s", "speedup", "MFU (same-run peak)"]))
    except ImportError:
        pass
    res = {**env_info("ladder"), "time": time.strftime("%Y-%m-%d %H:%M:%S"), "size": args.size, "batch": args.batch,
           "seq": args.seq, "bf16_ref_tflops": bref, "measured_peak_tflops": peak_measured, "rows": rows}
    if args.out:
        with open(args.out, "w") as f:
            json.dump(res, f, indent=1)


if __name__ == "__main__":
    main()
