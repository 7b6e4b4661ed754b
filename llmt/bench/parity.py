"""Loss parity of the native path against plain PyTorch (the reference's
kernels/check_loss_parity.py): every mode trains the same seeded model on the same fixed
batch for N steps with AdamW (lr 3e-4, betas 0.9/0.95, wd 0.1) and the loss curves are
compared with the fp32 PyTorch run: max |gap| / initial loss, and the step where each run's
loss first drops below 1 (the fixed batch is memorised).

Modes: torch-fp32 (the reference model in fp32), torch-bf16 (bf16 autocast), native-eager,
native-graph (one CUDA graph per step).

    python -m llmt.bench.parity --size small --batch 8 --seq 1024 --steps 100 [--json out.json]
"""
from __future__ import annotations

import argparse
import json

import torch


def torch_losses(cfg, B, T, steps, bf16):
    from llmt.models.llama import build_model, make_batch
    model = build_model(cfg, T, seed=0, device="cuda")
    opt = torch.optim.AdamW(model.parameters(), lr=3e-4, betas=(0.9, 0.95), weight_decay=0.1, fused=True)
    idx, tgt = make_batch(B, T, cfg.vocab, "cuda")
    out = []
    for _ in range(steps):
        with torch.autocast("cuda", dtype=torch.bfloat16, enabled=bf16):
            loss = model(idx, tgt)
        loss.backward()
        opt.step()
        opt.zero_grad(set_to_none=True)
        out.append(float(loss.item()))
    return out


def native_losses(cfg, B, T, steps, graph, linear="bf16"):
    from llmt.models.llama import make_batch
    from llmt.train import Trainer
    tr = Trainer(cfg, B, T, cuda_graph=graph, linear=linear)
    idx, tgt = make_batch(B, T, cfg.vocab, "cpu")
    out = []
    for _ in range(steps):
        out.append(tr.train_step(idx, tgt))
    tr.release()
    return out


def main():
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--size", default="small")
    p.add_argument("--batch", type=int, default=8)
    p.add_argument("--seq", type=int, default=1024)
    p.add_argument("--steps", type=int, default=100)
    p.add_argument("--modes", default="torch-fp32,torch-bf16,native-eager,native-graph",
                   help="also native-fp8, native-mxfp8, native-nvfp4 (low-precision block linears, CUDA graph; "
                        "the reference's triton+fp8 / triton+fp4 modes)")
    p.add_argument("--tol", type=float, default=0.05, help="max |gap| / initial loss accepted against torch-fp32")
    p.add_argument("--json", default=None)
    args = p.parse_args()
    from llmt.config import get_config
    cfg = get_config(args.size)
    runs = {}
    for mode in args.modes.split(","):
        if mode.startswith("torch"):
            runs[mode] = torch_losses(cfg, args.batch, args.seq, args.steps, bf16=mode == "torch-bf16")
        elif mode in ("native-fp8", "native-mxfp8", "native-nvfp4"):
            runs[mode] = native_losses(cfg, args.batch, args.seq, args.steps, graph=True, linear=mode.split("-")[1])
        else:
            runs[mode] = native_losses(cfg, args.batch, args.seq, args.steps, graph=mode == "native-graph")
    ref = runs.get("torch-fp32")
    res = {"size": args.size, "batch": args.batch, "seq": args.seq, "steps": args.steps, "modes": {}}
    ok = True
    for mode, ls in runs.items():
        below = next((i + 1 for i, v in enumerate(ls) if v == v and v < 1.0), None)
        row = {"first_loss": ls[0], "final_loss": ls[-1], "steps_to_loss_below_1": below, "losses": ls}
        if ref is not None:
            gaps = [abs(a - b) for a, b in zip(ls, ref) if a == a]
            row["max_gap_over_initial"] = max(gaps) / ref[0]
            if mode != "torch-fp32":
                ok &= row["max_gap_over_initial"] <= args.tol
        res["modes"][mode] = row
        print(f"{mode:14s} first {ls[0]:.4f} final {ls[-1]:.4f} below-1 at {below} "
              f"gap {row.get('max_gap_over_initial', 0):.4f}", flush=True)
    res["ok"] = ok
    if args.json:
        with open(args.json, "w") as f:
            json.dump(res, f, indent=1)
    raise SystemExit(0 if ok else 1)


if __name__ == "__main__":
    main()
