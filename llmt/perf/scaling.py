"""DP x TP x PP scaling model: step time, MFU and tokens/s for a global batch on n GPUs
(reference: perf_model/scaling.py, which only predicts; here the intra-node constants are the
B200 pool's measured NVLink 5 numbers and the prediction is checked against real runs).

Per layout (dp, tp, pp, micro-batch mb; m = G / (dp * mb) micro-batches):
  compute   roofline/calibrated prediction (llmt.perf.roofline) of one micro-batch with the
            block GEMMs sharded tp ways, divided over pp stages
  TP        sequence-parallel Megatron: per layer 2 all-gathers (qkv, gate/up inputs) and 2
            reduce-scatters (wo, down outputs) of the (mb, T, d) bf16 activation in the forward,
            the same in the backward; `fused=True` models them inside the GEMMs (overlapped up to
            the GEMM time), else exposed
  PP        1F1B: (m + p - 1) slots per stage, one (mb, T, d) bf16 send per micro-batch per
            direction; sends overlap compute when `overlap_pp`
  DP        ZeRO-1: reduce-scatter fp32 grads + all-gather bf16 weights per step, overlapped
            with the last micro-batch's backward when `overlap_dp`
  optimizer AdamW on params / (tp * pp * dp) (34 B/param incl. bf16 copy and grad zeroing)
  memory    fp32 master + grads (sharded as the layout shards them), bf16 weights, Adam state /
            dp, activations in flight; must fit 90% of the GPU

    python -m llmt.perf.scaling --models medium,llama3-8b --gpus 8,64,1024 --system b200_nvl8_ib
    python -m llmt.perf.scaling --fit <single-stage runs> --holdout <pipelined runs> --json out.json
    python -m llmt.perf.scaling --models llama3-8b --gpus 8,64 --calibration out.json
"""
from __future__ import annotations

import argparse
import json
import math
import os
from dataclasses import dataclass

from llmt.config import SIZES, count_params, model_flops_per_token
from llmt.perf.roofline import Machine, inventory, load_shape_times, predict

HERE = os.path.dirname(os.path.abspath(__file__))
WORKLOADS = {"small": ("small", 1024, 512), "medium": ("medium", 1024, 512), "large": ("large", 1024, 512),
             "llama3-8b": ("llama3-8b", 4096, 1024), "llama3-70b": ("llama3-70b", 4096, 1024)}


@dataclass
class Link:
    bw_gbs: float
    p2p_gbs: float
    latency_us: float


def load_links(path=None):
    with open(path or os.path.join(HERE, "links.json")) as f:
        return json.load(f)


def link(cfg, name) -> Link:
    d = cfg["links"][name]
    return Link(d["bw_gbs"], d.get("p2p_gbs", d["bw_gbs"]), d["latency_us"])


def ring_allreduce_s(nbytes, n, lk: Link):
    if n <= 1:
        return 0.0
    return 2 * (n - 1) / n * nbytes / (lk.bw_gbs * 1e9) + 2 * (n - 1) * lk.latency_us * 1e-6


def reduce_scatter_s(nbytes, n, lk: Link):
    """Half of a ring all-reduce (also the cost of an all-gather of the same total size)."""
    if n <= 1:
        return 0.0
    return (n - 1) / n * nbytes / (lk.bw_gbs * 1e9) + (n - 1) * lk.latency_us * 1e-6


def hier(fn, nbytes, n, g, intra: Link, inter: Link):
    """Inside a node of g GPUs first, then across nodes on the 1/g share."""
    if n <= g:
        return fn(nbytes, n, intra)
    return fn(nbytes, g, intra) + fn(nbytes / g, n // g, inter)


def p2p_s(nbytes, lk: Link):
    return nbytes / (lk.p2p_gbs * 1e9) + lk.latency_us * 1e-6


class StageCompute:
    """Cached per-micro-batch compute time (s) for a tp degree and micro-batch size."""

    def __init__(self, cfg, seq, machine, shape_times=None, path="native"):
        self.cfg, self.seq, self.m, self.st, self.path = cfg, seq, machine, shape_times or {}, path
        self._c = {}

    def get(self, tp, mb, ckpt=False):
        k = (tp, mb, ckpt)
        if k not in self._c:
            ops = inventory(self.cfg, mb, self.seq, self.path, tp=tp)
            ops = [o for o in ops if o.phase != "opt"]
            p = predict(ops, self.m, self.st)
            bwd = sum(o["ms"] for o in p.ops if o["phase"] == "bwd") / 1e3
            tot = p.total_ms / 1e3
            fwd = tot - bwd
            self._c[k] = (tot + (fwd if ckpt else 0.0), bwd + (fwd if ckpt else 0.0))
        return self._c[k]


def evaluate(cfg, seq, G, n, dp, tp, pp, mb, comp: StageCompute, links, system, ckpt=False, fused_tp=True,
             overlap_dp=True, overlap_pp=True, compute_scale=1.0, comm_scale=1.0):
    """compute_scale multiplies the roofline compute of a micro-batch (and so the pipeline
    bubble); comm_scale the tensor-parallel collective time (both fitted by `calibrate`)."""
    if dp * tp * pp != n or G % (dp * mb) or cfg.L % pp or cfg.H % tp or cfg.kvh % tp:
        return None
    m = G // (dp * mb)
    if m < pp and pp > 1:
        return None
    sysd = links["systems"][system]
    g = sysd["gpus_per_node"]
    intra, inter = link(links, sysd["intra"]), link(links, sysd["inter"])
    if tp > g:
        return None
    total, _ = count_params(cfg)
    p_gpu = total / (tp * pp)
    in_flight = min(m, pp)
    act_c = links["activation_bytes_per_token_per_layer_per_d_ckpt" if ckpt else "activation_bytes_per_token_per_layer_per_d"]
    act = act_c * cfg.d * seq * mb * (cfg.L / pp) * in_flight / tp
    mem = p_gpu * (4 + 4 + 2) + p_gpu * 8 / dp + act
    if mem > 0.9 * sysd["gpu_memory_gb"] * 1e9:
        return None
    t_mb, t_mb_bwd = comp.get(tp, mb, ckpt)
    t_mb, t_mb_bwd = t_mb * compute_scale, t_mb_bwd * compute_scale
    t_stage, t_stage_bwd = t_mb / pp, t_mb_bwd / pp
    act_bytes = mb * seq * cfg.d * 2
    tp_link = intra
    t_tp_raw = comm_scale * 8 * (cfg.L / pp) * reduce_scatter_s(act_bytes, tp, tp_link) if tp > 1 else 0.0
    t_tp = max(0.0, t_tp_raw - 0.8 * t_stage) if fused_tp else t_tp_raw
    pp_link = intra if tp * pp <= g else inter
    t_send = p2p_s(act_bytes, pp_link) if pp > 1 else 0.0
    slots = m + pp - 1
    t_pipe = slots * (t_stage + t_tp + (0.0 if overlap_pp else 2 * t_send)) + (2 * t_send * pp if overlap_pp else 0.0)
    g_dp = max(1, g // (tp * pp)) if tp * pp < g else 1
    t_dp = hier(reduce_scatter_s, p_gpu * 4, dp, g_dp, intra, inter) + hier(reduce_scatter_s, p_gpu * 2, dp, g_dp, intra, inter)
    hidden = min(t_dp, t_stage_bwd) if overlap_dp else 0.0
    t_opt = (p_gpu / dp) * 34 / (comp.m.hbm_gbs * 1e9)
    step = t_pipe + (t_dp - hidden) + t_opt
    tokens = G * seq
    mfu = model_flops_per_token(cfg, seq) * tokens / step / n / (comp.m.bf16_tflops * 1e12)
    return {"dp": dp, "tp": tp, "pp": pp, "mb": mb, "m": m, "ckpt": ckpt, "step_s": step, "tokens_per_s": tokens / step,
            "mfu": mfu, "mem_gb": mem / 1e9,
            "breakdown_s": {"compute": m * t_stage, "pipeline bubble": (pp - 1) * t_stage, "tp comm (exposed)": slots * t_tp,
                            "pp sends": (2 * t_send * pp if overlap_pp else slots * 2 * t_send),
                            "dp comm (exposed)": t_dp - hidden, "optimizer": t_opt}}


# ---------------------------------------------------------------- calibration against real runs
# The runs here are the bench JSON lines of llmt.bench.parallel_bench (results/par_*.json). Their
# collectives ran on NCCL, which the step neither fuses into the GEMMs nor overlaps with the
# backward, so they are modeled exposed (fused_tp=False, overlap_dp=False).
RUN_KW = dict(fused_tp=False, overlap_dp=False)


def run_kw(run):
    """How a measured run's collectives are modeled: exposed (RUN_KW), except the peer-memory
    tensor-parallel collectives of a run whose all-gathers ran inside the GEMMs (tp_comm "p2p",
    tp_gather "fused": both the gather and the reduce-scatter are fused into GEMMs, so the
    transfer overlaps the tiles)."""
    kw = dict(RUN_KW)
    if run.get("tp_comm") == "p2p" and run.get("tp_gather") == "fused":
        kw["fused_tp"] = True
    return kw


def run_layout(run):
    """(dp, tp, pp, micro-batch size, global batch) of a parallel-bench result."""
    kv = {p[:2]: int(p[2:]) for p in run["layout"].split()}
    G, m = run["global_batch"], run["microbatches"]
    return kv["dp"], kv["tp"], kv["pp"], G // (kv["dp"] * m), G


def _terms(run, comp, links, system):
    cfg, seq = comp.cfg, comp.seq
    dp, tp, pp, mb, G = run_layout(run)
    r = evaluate(cfg, seq, G, dp * tp * pp, dp, tp, pp, mb, comp, links, system, **run_kw(run))
    b = r["breakdown_s"]
    scaled_c = b["compute"] + b["pipeline bubble"]
    scaled_t = b["tp comm (exposed)"]
    fixed = b["pp sends"] + b["dp comm (exposed)"] + b["optimizer"]
    return scaled_c, scaled_t, fixed


def calibrate(fit_runs, comp, links, system):
    """Least-squares (compute_scale, comm_scale) so that measured = a * compute + c * tp comm +
    the unscaled terms (pipeline sends, data-parallel collectives, optimizer) on `fit_runs`."""
    rows, rhs = [], []
    for run in fit_runs:
        c, t, fixed = _terms(run, comp, links, system)
        rows.append((c, t))
        rhs.append(run["ms_per_step"] / 1e3 - fixed)
    # normal equations of the 2-parameter fit (no numpy needed)
    saa = sum(c * c for c, _ in rows)
    sab = sum(c * t for c, t in rows)
    sbb = sum(t * t for _, t in rows)
    sya = sum(c * y for (c, _), y in zip(rows, rhs))
    syb = sum(t * y for (_, t), y in zip(rows, rhs))
    det = saa * sbb - sab * sab
    if abs(det) < 1e-30:  # no tensor-parallel run: fit the compute scale alone
        return sya / saa, 1.0
    return (sya * sbb - syb * sab) / det, (syb * saa - sya * sab) / det


def predict_run(run, comp, links, system, compute_scale=1.0, comm_scale=1.0):
    dp, tp, pp, mb, G = run_layout(run)
    r = evaluate(comp.cfg, comp.seq, G, dp * tp * pp, dp, tp, pp, mb, comp, links, system,
                 compute_scale=compute_scale, comm_scale=comm_scale, **run_kw(run))
    return r["step_s"] * 1e3


def validate(fit_paths, holdout_paths, machine, links, system="b200_nvl8_ib", shape_times=None):
    """Fit the two scales on `fit_paths` (single-stage runs) and report the error of every run,
    the held-out ones (pipelined / hybrid layouts) separately."""
    def load(ps):
        out = []
        for p in ps:
            with open(p) as f:
                d = json.load(f)
            d["path"] = p
            out.append(d)
        return out
    fit, hold = load(fit_paths), load(holdout_paths)
    model = {r["model"] for r in fit + hold}
    if len(model) != 1:
        raise ValueError(f"one model per validation, got {sorted(model)}")
    run0 = (fit + hold)[0]
    comp = StageCompute(SIZES[run0["model"]], run0["seq"], machine, shape_times)
    a, c = calibrate(fit, comp, links, system)
    res = {"model": run0["model"], "seq": run0["seq"], "system": system, "compute_scale": a, "comm_scale": c,
           "fit": [], "holdout": []}
    for key, runs in (("fit", fit), ("holdout", hold)):
        for r in runs:
            raw = predict_run(r, comp, links, system)
            cal = predict_run(r, comp, links, system, a, c)
            res[key].append({"run": os.path.basename(r["path"]), "layout": r["layout"],
                             "microbatches": r["microbatches"], "global_batch": r["global_batch"],
                             "measured_ms": r["ms_per_step"], "roofline_ms": round(raw, 2),
                             "calibrated_ms": round(cal, 2), "error": round(cal / r["ms_per_step"] - 1, 4)})
    for key in ("fit", "holdout"):
        errs = [abs(x["error"]) for x in res[key]]
        res[f"{key}_mae"] = round(sum(errs) / len(errs), 4) if errs else None
    return res


def no_layout_reason(cfg, seq, G, n, links, system):
    """Why no dp x tp x pp layout of n GPUs works (evaluate() rejected them all): the first of
    a too-small global batch, weights and optimizer state too large even when split as widely as
    the model allows, or divisibility (the remaining case: some split would fit, none divides)."""
    sysd = links["systems"][system]
    widest_tp = max(t for t in (1, 2, 4, 8) if t <= sysd["gpus_per_node"] and cfg.H % t == 0 and cfg.kvh % t == 0)
    widest = widest_tp * cfg.L  # model-parallel GPUs: tp inside a node, one layer per stage
    if G * widest < n:
        return (f"global batch of {G} sequences is too small: at most {widest} model-parallel GPUs per "
                f"replica and one sequence per replica give {G * widest} < {n} GPUs")
    total, _ = count_params(cfg)
    split = min(widest, n)
    if total * (4 + 4 + 2) / split + total * 8 / n > 0.9 * sysd["gpu_memory_gb"] * 1e9:
        return (f"fp32 master + gradient, bf16 weights and the ZeRO-1 Adam state do not fit in "
                f"{sysd['gpu_memory_gb']} GB per GPU even split {split} ways")
    return "no split of the GPUs divides the heads, layers and global batch while fitting in memory"


def divisors(x, cap):
    return [d for d in range(1, min(x, cap) + 1) if x % d == 0]


def all_layouts(cfg, seq, G, n, comp, links, system, restrict=None, **kw):
    out = []
    for tp in (1, 2, 4, 8):
        for pp in divisors(cfg.L, 64):
            if n % (tp * pp):
                continue
            dp = n // (tp * pp)
            for mb in (1, 2, 4, 8, 16):
                for ck in (False, True):
                    if restrict and not restrict(dp, tp, pp, mb):
                        continue
                    r = evaluate(cfg, seq, G, n, dp, tp, pp, mb, comp, links, system, ck, **kw)
                    if r:
                        out.append(r)
    return sorted(out, key=lambda r: -r["tokens_per_s"])


def search(cfg, seq, G, n, comp, links, system, **kw):
    rows = all_layouts(cfg, seq, G, n, comp, links, system, **kw)
    return rows[0] if rows else None


def layout_str(r):
    return f"dp{r['dp']} tp{r['tp']} pp{r['pp']} mb{r['mb']}" + (" ckpt" if r["ckpt"] else "")


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--models", default="medium,llama3-8b")
    ap.add_argument("--gpus", default="8,64,1024")
    ap.add_argument("--system", default="b200_nvl8_ib")
    ap.add_argument("--links", default=None)
    ap.add_argument("--shape-times", default=None)
    ap.add_argument("--show-top", type=int, default=1)
    ap.add_argument("--layout", default=None, help="evaluate one layout, e.g. 'dp2,tp2,pp2,mb1' (needs one --gpus)")
    ap.add_argument("--global-batch", type=int, default=None)
    ap.add_argument("--json", default=None)
    ap.add_argument("--fit", default=None,
                    help="comma list of single-stage parallel-bench results (results/par_*.json) to fit the "
                         "compute and tensor-parallel scales on")
    ap.add_argument("--holdout", default="", help="comma list of results predicted with the fitted scales")
    ap.add_argument("--calibration", default=None,
                    help="a --fit result (JSON): search / evaluate layouts with its compute and "
                         "tensor-parallel scales and NCCL's exposed collectives")
    args = ap.parse_args()
    links = load_links(args.links)
    m = Machine.from_peaks()
    st = load_shape_times(args.shape_times)
    if args.fit:
        res = validate(args.fit.split(","), [p for p in args.holdout.split(",") if p], m, links, args.system, st)
        print(f"{res['model']}: compute x{res['compute_scale']:.3f} of the roofline, tensor-parallel collectives "
              f"x{res['comm_scale']:.3f} of the ring model")
        for key in ("fit", "holdout"):
            for x in res[key]:
                print(f"  {key:8s} {x['layout']:12s} m{x['microbatches']:<2d} measured {x['measured_ms']:8.1f} ms  "
                      f"roofline {x['roofline_ms']:8.1f}  calibrated {x['calibrated_ms']:8.1f}  "
                      f"error {100 * x['error']:+6.1f}%")
            print(f"  {key} mean absolute error {100 * res[key + '_mae']:.1f}%" if res[key + "_mae"] is not None else "")
        if args.json:
            with open(args.json, "w") as f:
                json.dump(res, f, indent=1)
        return
    kw = {}
    if args.calibration:
        with open(args.calibration) as f:
            cal = json.load(f)
        kw = dict(RUN_KW, compute_scale=cal["compute_scale"], comm_scale=cal["comm_scale"])
    res = []
    for name in args.models.split(","):
        size, seq, G = WORKLOADS[name]
        G = args.global_batch or G
        cfg = SIZES[size]
        comp = StageCompute(cfg, seq, m, st)
        for n in (int(x) for x in args.gpus.split(",")):
            if args.layout:
                kv = dict((p[:2], int(p[2:])) for p in args.layout.split(","))
                r = evaluate(cfg, seq, G, n, kv["dp"], kv["tp"], kv["pp"], kv["mb"], comp, links, args.system, **kw)
                rows = [r] if r else []
            else:
                rows = all_layouts(cfg, seq, G, n, comp, links, args.system, **kw)[: args.show_top]
            for r in rows:
                print(f"{name:10s} {n:5d} GPUs  {layout_str(r):22s} {r['step_s'] * 1e3:9.2f} ms "
                      f"{r['tokens_per_s'] / 1e6:8.3f} M tok/s  MFU {100 * r['mfu']:5.1f}%  mem {r['mem_gb']:.1f} GB")
                res.append({"model": name, "gpus": n, **r})
            if not rows:
                print(f"{name:10s} {n:5d} GPUs  no layout fits: {no_layout_reason(cfg, seq, G, n, links, args.system)}")
    if args.json:
        with open(args.json, "w") as f:
            json.dump(res, f, indent=1)


if __name__ == "__main__":
    main()
