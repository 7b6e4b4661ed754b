"""ASTRA-sim driver for the exported Chakra workloads (the reference's
workload_export/run_astra_sim.py).

Writes, next to the per-rank `workload.<r>.et` files of llmt.export.trace, the inputs an
ASTRA-sim analytical run needs -- a network description (one switch level per node of
`gpus_per_node` GPUs at the NVLink 5 constants of llmt/perf/links.json, then the
inter-node link), a system description, an (empty) remote-memory description and the
communicator groups -- and runs the simulator when a binary is given (--bin or the
ASTRA_SIM_BIN environment variable). Acceptance follows the reference's crash-tolerant rule:
a run counts if every rank reported a finish tick and they agree (the simulator's exit code is
not trusted on its own). The predicted step time is then set against llmt.perf.scaling's
prediction for the same layout.

ASTRA-sim is not installed in this image; without a binary the inputs are written and the
result says so.

    python -m llmt.export.astra --size medium --dp 2 --tp 2 --pp 2 --microbatches 4 --out traces
"""
from __future__ import annotations

import argparse
import json
import os
import re
import shutil
import subprocess

from llmt.config import SIZES
from llmt.perf.scaling import load_links


def network_yml(world, gpus_per_node, intra, inter):
    """Two-dimensional switch topology: GPUs of a node behind NVSwitch, nodes behind the IB fabric."""
    nodes = max(1, (world + gpus_per_node - 1) // gpus_per_node)
    per = min(world, gpus_per_node)
    dims = [(per, intra)] + ([(nodes, inter)] if nodes > 1 else [])
    return ("topology: [ " + ", ".join("Switch" for _ in dims) + " ]\n"
            f"npus_count: [ {', '.join(str(n) for n, _ in dims)} ]\n"
            f"bandwidth: [ {', '.join(str(lk['bw_gbs']) for _, lk in dims)} ]  # GB/s\n"
            f"latency: [ {', '.join(str(lk['latency_us'] * 1000.0) for _, lk in dims)} ]  # ns\n")


def system_json(collective="ring"):
    return {"scheduling-policy": "LIFO", "endpoint-delay": 10, "active-chunks-per-dimension": 1,
            "preferred-dataset-splits": 4, "all-reduce-implementation": [collective],
            "all-gather-implementation": [collective], "reduce-scatter-implementation": [collective],
            "all-to-all-implementation": ["direct"], "collective-optimization": "localBWAware",
            "local-mem-bw": 6417, "boost-mode": 0}


def write_inputs(outdir, world, system="b200_nvl8_ib", links=None):
    links = links or load_links()
    sysd = links["systems"][system]
    intra, inter = links["links"][sysd["intra"]], links["links"][sysd["inter"]]
    os.makedirs(outdir, exist_ok=True)
    paths = {"network": os.path.join(outdir, "network.yml"), "system": os.path.join(outdir, "system.json"),
             "memory": os.path.join(outdir, "remote_memory.json")}
    with open(paths["network"], "w") as f:
        f.write(network_yml(world, sysd["gpus_per_node"], intra, inter))
    with open(paths["system"], "w") as f:
        json.dump(system_json(), f, indent=1)
    with open(paths["memory"], "w") as f:
        json.dump({"memory-type": "NO_MEMORY_EXPANSION"}, f)
    return paths


def accept(stdout: str, world: int, tp: int = 1, pp: int = 1):
    """Finish ticks per rank from the simulator log, and whether the run is usable.

    The ranks of one pipeline stage are tied together by their collectives and finish at the same
    tick; different stages finish at different ticks. Accepted when every stage has at least one
    rank that reported and the ranks of each stage agree. (A simulator that crashes while printing
    its statistics after the simulation can drop some ranks' lines; every rank reporting is
    recorded separately by run().) Rank order: tp innermost, then pp, then dp."""
    ticks = {}
    for m in re.finditer(r"sys\[(\d+)\][^\n]*?finished,\s*(\d+)\s*cycles", stdout):
        ticks[int(m.group(1))] = int(m.group(2))
    stages = {}
    for r, t in ticks.items():
        stages.setdefault((r // tp) % pp, set()).add(t)
    ok = len(stages) == pp and all(len(v) == 1 for v in stages.values()) and all(0 <= r < world for r in ticks)
    return ok, ticks


def exposed_comm(stdout: str):
    """Per-rank exposed communication cycles, where the simulator prints them."""
    return {int(m.group(1)): int(m.group(2)) for m in
            re.finditer(r"sys\[(\d+)\][^\n]*?exposed communication\s*(\d+)\s*cycles", stdout)}


def run(outdir, world, binary, timeout_s=3600, tp=1, pp=1):
    paths = write_inputs(outdir, world)
    if not binary or not shutil.which(binary) and not os.path.exists(binary):
        return {"status": "unavailable", "reason": "no ASTRA-sim binary (pass --bin or set ASTRA_SIM_BIN)",
                "inputs": paths}
    cmd = [binary, f"--workload-configuration={os.path.join(outdir, 'workload')}",
           f"--comm-group-configuration={os.path.join(outdir, 'comm_group.json')}",
           f"--system-configuration={paths['system']}", f"--network-configuration={paths['network']}",
           f"--remote-memory-configuration={paths['memory']}"]
    try:
        p = subprocess.run(cmd, capture_output=True, text=True, timeout=timeout_s)
    except subprocess.TimeoutExpired:
        return {"status": "timeout", "cmd": cmd}
    out = p.stdout + p.stderr
    ok, ticks = accept(out, world, tp, pp)
    res = {"status": "ok" if ok else "rejected", "exit_code": p.returncode, "finish_ticks": ticks, "cmd": cmd,
           "all_ranks_reported": len(ticks) == world}
    if ok:
        # the simulator's cycles are nanoseconds; the step ends when the last stage finishes
        res["step_ms"] = max(ticks.values()) / 1e6
        exp = exposed_comm(out)
        if exp:
            res["max_exposed_comm_ms"] = max(exp.values()) / 1e6
    return res


def scaling_prediction(cfg, mb, seq, dp, tp, pp, m, fused_tp=False, system="b200_nvl8_ib"):
    """The scaling model's step for the exported layout (global batch mb x m x dp sequences),
    to set beside the simulated one; None if the model rejects the layout."""
    from llmt.perf.roofline import Machine
    from llmt.perf.scaling import StageCompute, evaluate, load_links
    machine = Machine.from_peaks()
    r = evaluate(cfg, seq, mb * m * dp, dp * tp * pp, dp, tp, pp, mb, StageCompute(cfg, seq, machine), load_links(),
                 system, fused_tp=fused_tp, overlap_dp=False)
    if r is None:
        return None
    return {"step_ms": r["step_s"] * 1e3, "breakdown_ms": {k: v * 1e3 for k, v in r["breakdown_s"].items()}}


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--size", default="medium", choices=list(SIZES))
    ap.add_argument("--batch", type=int, default=4)
    ap.add_argument("--seq", type=int, default=1024)
    ap.add_argument("--dp", type=int, default=2)
    ap.add_argument("--tp", type=int, default=2)
    ap.add_argument("--pp", type=int, default=2)
    ap.add_argument("--microbatches", type=int, default=4)
    ap.add_argument("--out", default="traces")
    ap.add_argument("--bin", default=os.environ.get("ASTRA_SIM_BIN"))
    ap.add_argument("--fused-tp", action="store_true",
                    help="export the tensor-parallel collectives as fused into their GEMMs (the peer-memory path)")
    args = ap.parse_args()
    from llmt.export.trace import export
    cfg = SIZES[args.size]
    graphs, _ = export(cfg, args.batch, args.seq, args.dp, args.tp, args.pp, args.microbatches, outdir=args.out,
                       fused_tp=args.fused_tp)
    res = run(args.out, args.dp * args.tp * args.pp, args.bin, tp=args.tp, pp=args.pp)
    # beside the simulation: rank 0's exported compute and the scaling model's step for this layout
    res["export_compute_ms_rank0"] = round(sum(n["predicted_us"] for n in graphs[0].nodes if n["kind"] == "comp") / 1e3, 3)
    sc = scaling_prediction(cfg, args.batch, args.seq, args.dp, args.tp, args.pp, args.microbatches, args.fused_tp)
    if sc:
        res["scaling_model_step_ms"] = round(sc["step_ms"], 3)
        res["scaling_model_breakdown_ms"] = {k: round(v, 3) for k, v in sc["breakdown_ms"].items()}
        if res.get("step_ms"):
            res["vs_scaling_model_pct"] = round(100 * (res["step_ms"] / sc["step_ms"] - 1), 2)
    print(json.dumps(res))


if __name__ == "__main__":
    main()
