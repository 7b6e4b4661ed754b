"""Fusion ablation: what each fused epilogue saves in a whole training step (the reference's
kernels/ablate_kernels.py, which swaps its Triton ops in and out one at a time).

Runs the native step (CUDA graph) with every fusion on, with each one switched off alone, and
with all of them off; reports ms per step and the saving of each fusion (step time with it off
minus the all-on time). Fusions (llmt.ops.functions): SwiGLU forward in the gate/up GEMM,
SwiGLU backward in the w2 dgrad, RoPE in the qkv GEMM, cross entropy inside the head GEMM.

    python -m llmt.bench.ablate --size medium --batch 4 --seq 1024 [--json out.json]
"""
from __future__ import annotations

import argparse
import json
import statistics

import torch

FUSIONS = ("swiglu_fwd", "swiglu_bwd", "rope", "head_ce")


def _set(on: dict):
    from llmt.ops import functions as Fn
    Fn.SWIGLU_EPILOGUE["fwd"] = on["swiglu_fwd"]
    Fn.SWIGLU_EPILOGUE["bwd"] = on["swiglu_bwd"]
    Fn.FUSION["rope"] = on["rope"]
    Fn.FUSION["head_ce"] = on["head_ce"]  # True: always the fused head (the "all fused" row)


def step_ms(cfg, batch, seq, steps, warmup):
    from llmt.models.llama import make_batch
    from llmt.train import Trainer
    tr = Trainer(cfg, batch, seq, cuda_graph=True)
    idx, tgt = make_batch(batch, seq, cfg.vocab, "cuda")
    tr.set_batch(idx, tgt)
    for _ in range(warmup):
        tr.run_step()
    torch.cuda.synchronize()
    ts = []
    for _ in range(steps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        tr.run_step()
        b.record()
        torch.cuda.synchronize()
        ts.append(a.elapsed_time(b))
    loss = float(tr.loss.item())
    tr.release()
    return statistics.median(ts), loss


def main():
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--size", default="medium")
    p.add_argument("--batch", type=int, default=4)
    p.add_argument("--seq", type=int, default=1024)
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--json", default=None)
    args = p.parse_args()
    from llmt.config import get_config
    cfg = get_config(args.size)
    rows = []
    configs = [("all fused", {f: True for f in FUSIONS})]
    configs += [(f"without {f}", {g: g != f for g in FUSIONS}) for f in FUSIONS]
    configs += [("none fused", {f: False for f in FUSIONS})]
    for name, on in configs:
        _set(on)
        ms, loss = step_ms(cfg, args.batch, args.seq, args.steps, args.warmup)
        rows.append({"config": name, "ms_per_step": round(ms, 3), "loss": round(loss, 4)})
        print(f"{name:22s} {ms:8.3f} ms  loss {loss:.4f}", flush=True)
    _set({f: True for f in FUSIONS})
    from llmt.ops import functions as Fn
    Fn.FUSION["head_ce"] = "auto"
    base = rows[0]["ms_per_step"]
    savings = {r["config"][len("without "):]: round(r["ms_per_step"] - base, 3) for r in rows if r["config"].startswith("without")}
    savings["all"] = round(rows[-1]["ms_per_step"] - base, 3)
    print("saving of each fusion (ms per step):", json.dumps(savings))
    if args.json:
        with open(args.json, "w") as f:
            json.dump({"size": args.size, "batch": args.batch, "seq": args.seq, "rows": rows, "savings_ms": savings}, f,
                      indent=1)


if __name__ == "__main__":
    main()
