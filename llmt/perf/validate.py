"""Predicted vs measured step time of the native path (reference: perf_model/validate.py).

For each (size, batch, seq) config: the roofline prediction (peaks only), the calibrated
prediction (each GEMM / attention shape timed on this GPU with this framework's kernels,
elementwise ops at the roofline, CUDA-graph gap per launch), and the measured CUDA-graph step
(CUDA events, median). Reports the error of each and the mean absolute error over the fitting
configs and the held-out ones, plus an MFU-gap breakdown of the measured step.

The "fitted" prediction corrects the calibrated one for the one systematic effect left: GEMM and
attention shapes are timed alone with a flushed L2, while inside the step their operands are
often still in L2. One factor alpha scales the timed (matmul + attention) part; it is fitted by
least squares on the fitting configs only and then applied unchanged to the held-out ones.

    python -m llmt.perf.validate --out results/perf_model_validation.json
"""
from __future__ import annotations

import argparse
import json
import statistics

import torch

from llmt.config import SIZES, model_flops_per_token
from llmt.perf.roofline import Machine, inventory, measure_shape_times, predict

CONFIGS = [("small", 8, 1024), ("medium", 4, 1024), ("large", 2, 1024)]
HOLDOUT = [("small", 4, 2048), ("medium", 8, 1024), ("tiny", 16, 1024)]


def measure_step_ms(size, B, T, steps=10, warmup=3):
    from llmt.models.llama import make_batch
    from llmt.train import Trainer
    cfg = SIZES[size]
    tr = Trainer(cfg, B, T, cuda_graph=True)
    idx, tgt = make_batch(B, T, cfg.vocab, "cuda")
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
    tr.release()
    del tr
    torch.cuda.empty_cache()
    return statistics.median(ts)


def measure_gap_us(n=1000):
    """GPU time between back-to-back kernels replayed from a CUDA graph."""
    x = torch.zeros(1, device="cuda")
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        x.add_(1)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(n):
            x.add_(1)
    g.replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    g.replay()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) * 1e3 / n


TIMED = ("matmul", "attention")


def fitted_ms(row, alpha):
    cats = row["calibrated_by_cat_ms"]
    timed = sum(v for k, v in cats.items() if k in TIMED)
    return row["calibrated_ms"] - timed + alpha * timed


def fit_alpha(rows):
    """Least-squares alpha for measured ~ calibrated - timed + alpha * timed."""
    num = den = 0.0
    for r in rows:
        timed = sum(v for k, v in r["calibrated_by_cat_ms"].items() if k in TIMED)
        rest = r["calibrated_ms"] - timed
        num += timed * (r["measured_ms"] - rest)
        den += timed * timed
    return num / den if den > 0 else 1.0


def mfu_gap(row, peak_tflops, alpha=1.0):
    """Where the measured step's time goes relative to the MFU ideal, in ms (sums to measured_ms).

    ideal: the model FLOPs (the MFU numerator: 6 x matmul params + 12 L d T per token) at the bf16
    peak. The GEMM and attention terms are their calibrated times (scaled by the fitted L2 factor
    alpha) minus their share of the ideal: the GEMMs' share is the 6 x params part, attention's
    the 12 L d T part (counted as full, non-causal attention, as the MFU formula does). The
    memory-bound, optimizer and launch-gap terms are the calibrated prediction's; whatever the
    model does not place (idle time, cache effects across kernels) is the residual."""
    cfg = SIZES[row["size"]]
    tok = row["batch"] * row["seq"]
    peak = peak_tflops * 1e12
    attn_flops = 12 * cfg.L * cfg.d * row["seq"] * tok
    all_flops = model_flops_per_token(cfg, row["seq"]) * tok
    cats = row["calibrated_by_cat_ms"]
    gap = {"model FLOPs at the bf16 peak": all_flops / peak * 1e3,
           "GEMMs below peak": alpha * cats["matmul"] - (all_flops - attn_flops) / peak * 1e3,
           "attention below peak": alpha * cats["attention"] - attn_flops / peak * 1e3,
           "memory-bound ops (norms, elementwise, loss)": cats["elementwise"] + cats["copy/cast"] + cats["loss"],
           "optimizer": cats["optimizer"],
           "kernel launch gaps": row["gap_ms"]}
    gap["residual (not placed by the model)"] = row["measured_ms"] - sum(gap.values())
    return {k: round(v, 3) for k, v in gap.items()}


def run(configs, machine, cache, out_rows, tag):
    for size, B, T in configs:
        cfg = SIZES[size]
        ops = inventory(cfg, B, T, "native")
        st = measure_shape_times(ops, cache)
        p_roof = predict(ops, machine)
        p_cal = predict(ops, machine, st)
        meas = measure_step_ms(size, B, T)
        tok = B * T
        mfu = model_flops_per_token(cfg, T) * tok / (meas / 1e3) / (machine.bf16_tflops * 1e12)
        row = {"set": tag, "size": size, "batch": B, "seq": T, "measured_ms": round(meas, 3),
               "roofline_ms": round(p_roof.total_ms, 3), "calibrated_ms": round(p_cal.total_ms, 3),
               "roofline_err": round((p_roof.total_ms - meas) / meas, 4),
               "calibrated_err": round((p_cal.total_ms - meas) / meas, 4), "mfu": round(mfu, 4),
               "calibrated_by_cat_ms": {k: round(v, 3) for k, v in p_cal.by_cat.items()},
               "gap_ms": round(p_cal.gap_ms, 3)}
        print(json.dumps(row), flush=True)
        out_rows.append(row)


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--out", default=None)
    ap.add_argument("--cache", default="/tmp/llmt_shape_times.json")
    ap.add_argument("--no-holdout", action="store_true")
    ap.add_argument("--gap-from", default=None,
                    help="a results file of this script: add the MFU-gap breakdown to its rows (no GPU needed)")
    args = ap.parse_args()
    if args.gap_from:
        with open(args.gap_from) as f:
            res = json.load(f)
        alpha = res["summary"]["alpha"]
        for r in res["rows"]:
            r["mfu_gap_ms"] = mfu_gap(r, res["machine"]["bf16_tflops"], alpha)
            print(r["size"], r["batch"], r["seq"], json.dumps(r["mfu_gap_ms"]))
        with open(args.out or args.gap_from, "w") as f:
            json.dump(res, f, indent=1)
        return
    gap = measure_gap_us()
    m = Machine.from_peaks(sustained=True, gpu_gap_us=gap)
    rows = []
    run(CONFIGS, m, args.cache, rows, "fit")
    if not args.no_holdout:
        run(HOLDOUT, m, args.cache, rows, "holdout")
    alpha = fit_alpha([r for r in rows if r["set"] == "fit"])
    for r in rows:
        r["fitted_ms"] = round(fitted_ms(r, alpha), 3)
        r["fitted_err"] = round((r["fitted_ms"] - r["measured_ms"]) / r["measured_ms"], 4)
        r["mfu_gap_ms"] = mfu_gap(r, m.bf16_tflops, alpha)
    summ = {"alpha": round(alpha, 4)}
    for tag in ("fit", "holdout"):
        rs = [r for r in rows if r["set"] == tag]
        if rs:
            summ[tag] = {"mae_fitted": round(statistics.mean(abs(r["fitted_err"]) for r in rs), 4),
                         "mae_calibrated": round(statistics.mean(abs(r["calibrated_err"]) for r in rs), 4),
                         "mae_roofline": round(statistics.mean(abs(r["roofline_err"]) for r in rs), 4)}
    res = {"gpu_gap_us": round(gap, 3), "machine": vars(m), "rows": rows, "summary": summ}
    print(json.dumps(res["summary"]))
    if args.out:
        with open(args.out, "w") as f:
            json.dump(res, f, indent=1)


if __name__ == "__main__":
    main()
