"""Per-rank operator graphs of one DP x TP x PP training step, exported as Chakra traces
(reference: workload_export/export_trace.py, check_export.py).

The graph of each rank is built from this framework's native op inventory
(llmt.perf.roofline.inventory with path="native"): every per-layer op is instantiated for the
layers of the rank's pipeline stage, per micro-batch, in 1F1B order; the embedding sits on
the first stage and the final norm / lm head / loss on the last. Communication nodes follow
the runtime of this framework rather than the reference's all-reduce-only model:
  TP (sequence parallel)  ALL_GATHER of the (mb, T, d) bf16 input before the qkv and w1||w3
                          GEMMs and REDUCE_SCATTER after the wo and w2 GEMMs (forward), the
                          mirror in the backward
  PP                      SEND / RECV of the (mb, T, d) bf16 activation (forward) and its
                          gradient (backward) between neighbour stages
  DP (ZeRO-1)             per layer, after its last micro-batch backward: REDUCE_SCATTER of
                          the fp32 gradients and ALL_GATHER of the bf16 weights
Data dependencies come from tensor names; one in-order compute stream gives control deps.

    python -m llmt.export.trace --size medium --batch 4 --seq 1024 --dp 2 --tp 2 --pp 2 --microbatches 4 --out traces/
"""
from __future__ import annotations

import argparse
import json
import os
from collections import defaultdict

from llmt.config import SIZES
from llmt.export import chakra as ck
from llmt.perf.roofline import Machine, inventory

DT = {"bf16": 2, "fp32": 4}


def rank_of(dp_i, pp_i, tp_i, tp, pp):
    """Rank numbering: tensor parallel innermost, then pipeline, then data parallel."""
    return dp_i * (tp * pp) + pp_i * tp + tp_i


def schedule_1f1b(stage, p, m):
    warm = min(p - stage - 1, m)
    order = [("F", i) for i in range(warm)]
    for i in range(m - warm):
        order += [("F", warm + i), ("B", i)]
    return order + [("B", i) for i in range(m - warm, m)]


def make_groups(dp, tp, pp):
    """Communicator ids (>= 1) -> member ranks; and per-kind lookup tables."""
    table, kinds, nid = {}, {"tp": {}, "dp": {}, "pp": {}}, 1
    for a in range(dp):
        for b in range(pp):
            table[nid] = [rank_of(a, b, t, tp, pp) for t in range(tp)]
            kinds["tp"][(a, b)] = nid
            nid += 1
    for b in range(pp):
        for t in range(tp):
            table[nid] = [rank_of(a, b, t, tp, pp) for a in range(dp)]
            kinds["dp"][(b, t)] = nid
            nid += 1
    return table, kinds


class Graph:
    def __init__(self, rank, machine):
        self.rank, self.m = rank, machine
        self.nodes, self.producer, self.last = [], {}, None

    def add(self, name, kind, cat, phase, ins=(), outs=(), flops=0.0, nbytes=0.0, comm=None, layer=None, mb=None):
        nid = len(self.nodes)
        deps = sorted({self.producer[t] for t in ins if t in self.producer})
        ctrl = []
        if kind == "comp":
            if self.last is not None and self.last not in deps:
                ctrl = [self.last]
            t = max(flops / (self.m.bf16_tflops * 1e12), nbytes / (self.m.hbm_gbs * 1e9)) + self.m.gpu_gap_us * 1e-6
        else:
            t = 0.0
        self.nodes.append({"id": nid, "name": name, "kind": kind, "category": cat, "phase": phase, "layer": layer,
                           "microbatch": mb, "inputs": list(ins), "outputs": list(outs), "flops": flops,
                           "bytes": nbytes, "data_deps": deps, "ctrl_deps": ctrl, "predicted_us": t * 1e6,
                           "comm": comm})
        for o in outs:
            self.producer[o] = nid
        if kind == "comp":
            self.last = nid
        return nid


def _split_inventory(cfg, mb, seq, tp):
    ops = inventory(cfg, mb, seq, "native", tp=tp)
    per_layer, first, last, opt = [], [], [], []
    for o in ops:
        if o.phase == "opt":
            opt.append(o)
            continue
        k, rem = divmod(o.count, cfg.L) if o.count >= cfg.L else (0, o.count)
        if k:
            per_layer.append((o, k))
        if rem:
            (first if "embedding" in o.name else last).append((o, rem))
    return per_layer, first, last, opt


def build_rank(cfg, mb, seq, dp, tp, pp, m, dp_i, pp_i, tp_i, machine, kinds, fused_tp=False):
    """One rank's graph. fused_tp: the tensor-parallel collectives run inside the GEMMs (the
    peer-memory path): an all-gather and the GEMM that consumes it both start from the GEMM's
    input and run concurrently, a reduce-scatter starts with the GEMM that produces its rows, and
    the next operator waits for both (its inputs include the collective's output)."""
    rank = rank_of(dp_i, pp_i, tp_i, tp, pp)
    g = Graph(rank, machine)
    per_layer, first, last, opt = _split_inventory(cfg, mb, seq, tp)
    Lp = cfg.L // pp
    layers = range(pp_i * Lp, (pp_i + 1) * Lp)
    act = mb * seq * cfg.d * 2
    tpg = kinds["tp"][(dp_i, pp_i)]
    dpg = kinds["dp"][(pp_i, tp_i)]
    prev_r = rank_of(dp_i, pp_i - 1, tp_i, tp, pp) if pp_i > 0 else None
    next_r = rank_of(dp_i, pp_i + 1, tp_i, tp, pp) if pp_i < pp - 1 else None

    def coll(name, ctype, nbytes, group, phase, layer, mbi, ins, outs):
        return g.add(name, "coll", "communication", phase, ins, outs, nbytes=nbytes, layer=layer, mb=mbi,
                     comm={"type": ctype, "bytes": nbytes, "pg": group})

    for ph, i in schedule_1f1b(pp_i, pp, m):
        x = f"act.mb{i}"
        if ph == "F":
            if prev_r is not None:
                g.add(f"recv act mb{i}", "recv", "communication", "fwd", (), (x,), nbytes=act, mb=i,
                      comm={"src": prev_r, "dst": rank, "tag": 2 * i, "bytes": act})
            else:
                for o, k in first:
                    if o.phase == "fwd":
                        g.add(o.name, "comp", o.cat, "fwd", (), (x,), o.flops * k, o.bytes * k, mb=i)
            join = ()  # outputs of fused collectives the next operator also waits for
            for li in layers:
                for o, k in per_layer:
                    if o.phase != "fwd":
                        continue
                    ins = (x,) + join
                    join = ()
                    if tp > 1 and ("qkv" in o.name or "w1||w3" in o.name):
                        coll(f"SP all-gather before {o.name} L{li}", ck.ALL_GATHER, act, tpg, "fwd", li, i, ins, (x + ".ag",))
                        if fused_tp:
                            join = (x + ".ag",)
                        else:
                            ins = (x + ".ag",)
                    rs = tp > 1 and (o.name.startswith("wo") or o.name.startswith("w2"))
                    if rs and fused_tp:
                        coll(f"SP reduce-scatter in {o.name} L{li}", ck.REDUCE_SCATTER, act, tpg, "fwd", li, i, ins,
                             (x + ".rs",))
                        join = (x + ".rs",)
                    g.add(f"{o.name} L{li} mb{i}", "comp", o.cat, "fwd", ins, (x,), o.flops * k, o.bytes * k, li, i)
                    if rs and not fused_tp:
                        coll(f"SP reduce-scatter after {o.name} L{li}", ck.REDUCE_SCATTER, act, tpg, "fwd", li, i, (x,), (x,))
            x_out = (x,) + join
            if next_r is not None:
                g.add(f"send act mb{i}", "send", "communication", "fwd", x_out, (), nbytes=act, mb=i,
                      comm={"src": rank, "dst": next_r, "tag": 2 * i, "bytes": act})
            else:
                for o, k in last:
                    if o.phase == "fwd":
                        g.add(f"{o.name} mb{i}", "comp", o.cat, "fwd", x_out, (f"loss.mb{i}",), o.flops * k, o.bytes * k,
                              mb=i)
                        x_out = (x,)
        else:
            gx = f"grad.mb{i}"
            if next_r is not None:
                g.add(f"recv grad mb{i}", "recv", "communication", "bwd", (), (gx,), nbytes=act, mb=i,
                      comm={"src": next_r, "dst": rank, "tag": 2 * i + 1, "bytes": act})
            else:
                for o, k in last:
                    if o.phase == "bwd":
                        g.add(f"{o.name} mb{i}", "comp", o.cat, "bwd", (f"loss.mb{i}",), (gx,), o.flops * k, o.bytes * k, mb=i)
            join = ()
            for li in reversed(layers):
                for o, k in per_layer:
                    if o.phase != "bwd":
                        continue
                    ins = (gx,) + (join if "wgrad" not in o.name else ())
                    if "wgrad" not in o.name:
                        join = ()
                    if tp > 1 and ("w2 dgrad" in o.name or o.name.startswith("wo dgrad")):
                        coll(f"SP all-gather before {o.name} L{li}", ck.ALL_GATHER, act, tpg, "bwd", li, i, ins, (gx + ".ag",))
                        if fused_tp:  # the dgrad GEMM gathers dy itself
                            join = (gx + ".ag",)
                        else:
                            ins = (gx + ".ag",)
                    wout = (f"wgrad.L{li}",) if "wgrad" in o.name else (gx,)
                    if "wgrad" in o.name and fused_tp:
                        ins = ins + tuple(t for t in join if t.endswith(".ag"))  # reads the gathered dy
                    g.add(f"{o.name} L{li} mb{i}", "comp", o.cat, "bwd", ins, wout, o.flops * k, o.bytes * k, li, i)
                    if tp > 1 and (o.name.startswith("qkv dgrad") or o.name.startswith("w1||w3 dgrad")):
                        coll(f"SP reduce-scatter after {o.name} L{li}", ck.REDUCE_SCATTER, act, tpg, "bwd", li, i, (gx,), (gx,))
                if dp > 1 and i == m - 1:
                    nparams = _layer_params(cfg, tp)
                    coll(f"ZeRO-1 grad reduce-scatter L{li}", ck.REDUCE_SCATTER, nparams * 4, dpg, "bwd", li, i,
                         (f"wgrad.L{li}",), (f"gshard.L{li}",))
            if prev_r is not None:
                g.add(f"send grad mb{i}", "send", "communication", "bwd", (gx,), (), nbytes=act, mb=i,
                      comm={"src": rank, "dst": prev_r, "tag": 2 * i + 1, "bytes": act})
            else:
                for o, k in first:
                    if o.phase == "bwd":
                        g.add(f"{o.name} mb{i}", "comp", o.cat, "bwd", (gx,), (), o.flops * k, o.bytes * k, mb=i)
    for o in opt:
        g.add(o.name, "comp", o.cat, "opt", tuple(f"gshard.L{li}" for li in layers) if dp > 1 else (),
              ("weights",), o.flops / (pp * dp), o.bytes / (pp * dp))
    if dp > 1:
        for li in layers:
            coll(f"ZeRO-1 weight all-gather L{li}", ck.ALL_GATHER, _layer_params(cfg, tp) * 2, dpg, "opt", li, None,
                 ("weights",), (f"w16.L{li}",))
    return g


def _layer_params(cfg, tp):
    qkv = cfg.d * cfg.qkv_out
    return (qkv + cfg.H * cfg.hd * cfg.d + 3 * cfg.d * cfg.ffn) // tp + 2 * cfg.d


def to_chakra(n) -> dict:
    typ = {"comp": ck.COMP_NODE, "coll": ck.COMM_COLL_NODE, "send": ck.COMM_SEND_NODE, "recv": ck.COMM_RECV_NODE}[n["kind"]]
    attrs = [("is_cpu_op", "bool_val", False), ("phase", "string_val", n["phase"]), ("category", "string_val", n["category"])]
    if typ == ck.COMP_NODE:
        attrs += [("num_ops", "int64_val", max(1, int(n["flops"]))), ("tensor_size", "uint64_val", int(n["bytes"]))]
    else:
        c = n["comm"]
        attrs.append(("comm_size", "int64_val", int(c["bytes"])))
        if typ == ck.COMM_COLL_NODE:
            attrs += [("comm_type", "int64_val", c["type"]), ("pg_name", "string_val", str(c["pg"]))]
        else:
            attrs += [("comm_src", "int32_val", c["src"]), ("comm_dst", "int32_val", c["dst"]),
                      ("comm_tag", "int32_val", c["tag"])]
    return {"id": n["id"], "name": n["name"], "type": typ, "data_deps": n["data_deps"], "ctrl_deps": n["ctrl_deps"],
            "duration_micros": max(1, round(n["predicted_us"])) if typ == ck.COMP_NODE else 0,
            "inputs": {"shapes": json.dumps(n["inputs"])}, "outputs": {"shapes": json.dumps(n["outputs"])},
            "attrs": attrs}


def export(cfg, mb, seq, dp, tp, pp, m, outdir=None, machine=None, fused_tp=False):
    machine = machine or Machine.from_peaks()
    table, kinds = make_groups(dp, tp, pp)
    graphs = {}
    for a in range(dp):
        for b in range(pp):
            for t in range(tp):
                gr = build_rank(cfg, mb, seq, dp, tp, pp, m, a, b, t, machine, kinds, fused_tp)
                graphs[gr.rank] = gr
    if outdir:
        os.makedirs(outdir, exist_ok=True)
        with open(os.path.join(outdir, "comm_group.json"), "w") as f:
            json.dump({str(k): v for k, v in table.items()}, f)
        for r, gr in graphs.items():
            ck.write_et(os.path.join(outdir, f"workload.{r}.et"), [to_chakra(n) for n in gr.nodes],
                        [("rank", "int64_val", r), ("dp", "int64_val", dp), ("tp", "int64_val", tp), ("pp", "int64_val", pp)])
            with open(os.path.join(outdir, f"graph.rank{r}.json"), "w") as f:
                json.dump(gr.nodes, f)
    return graphs, table


# ---------------------------------------------------------------- checks
def check_graphs(graphs, table) -> dict:
    """Acyclic (deps point backward), every send has one matching recv (src, dst, tag, bytes),
    and every member of a group issues the same collective sequence (type, bytes)."""
    errors = []
    for r, gr in graphs.items():
        for n in gr.nodes:
            if any(d >= n["id"] for d in n["data_deps"] + n["ctrl_deps"]):
                errors.append(f"rank {r} node {n['id']} depends forward")
    sends = defaultdict(int)
    recvs = defaultdict(int)
    for r, gr in graphs.items():
        for n in gr.nodes:
            if n["kind"] == "send":
                c = n["comm"]
                sends[(c["src"], c["dst"], c["tag"], c["bytes"])] += 1
            elif n["kind"] == "recv":
                c = n["comm"]
                recvs[(c["src"], c["dst"], c["tag"], c["bytes"])] += 1
    if sends != recvs:
        errors.append(f"unmatched send/recv: {len(set(sends) ^ set(recvs))} keys differ")
    seqs = defaultdict(dict)
    for r, gr in graphs.items():
        for n in gr.nodes:
            if n["kind"] == "coll":
                c = n["comm"]
                seqs[c["pg"]].setdefault(r, []).append((c["type"], c["bytes"]))
    for pg, per in seqs.items():
        members = table.get(int(pg), [])
        if sorted(per) != sorted(members):
            errors.append(f"group {pg}: ranks {sorted(per)} != members {members}")
        vals = list(per.values())
        if any(v != vals[0] for v in vals):
            errors.append(f"group {pg}: members issue different collective sequences")
    return {"pass": not errors, "errors": errors[:20], "send_recv_pairs": sum(sends.values()),
            "collectives": sum(len(v) for per in seqs.values() for v in per.values())}


def cross_check(cfg, mb, seq, dp, tp, pp, m, graphs) -> dict:
    """FLOPs and bytes of one rank per stage (dp 0, tp 0) == m x step (no optimizer) + optimizer / dp."""
    ops = inventory(cfg, mb, seq, "native", tp=tp)
    want_f = sum(o.total_flops * (1 if o.phase == "opt" else m) for o in ops if o.phase != "opt")
    want_b = sum(o.total_bytes * m for o in ops if o.phase != "opt") + sum(o.total_bytes / dp for o in ops if o.phase == "opt")
    got_f = got_b = 0.0
    for b in range(pp):
        for n in graphs[rank_of(0, b, 0, tp, pp)].nodes:
            if n["kind"] == "comp":
                got_f += n["flops"]
                got_b += n["bytes"]
    ef = abs(got_f - want_f) / want_f
    eb = abs(got_b - want_b) / want_b
    return {"pass": ef < 1e-9 and eb < 1e-9, "flops": [got_f, want_f], "bytes": [got_b, want_b],
            "flops_rel_diff": ef, "bytes_rel_diff": eb}


def check_roundtrip(graphs, outdir) -> dict:
    bad = 0
    for r, gr in graphs.items():
        _, nodes = ck.read_et(os.path.join(outdir, f"workload.{r}.et"))
        if len(nodes) != len(gr.nodes):
            bad += 1
            continue
        for a, b in zip(nodes, (to_chakra(n) for n in gr.nodes)):
            if (a["id"], a["name"], a["type"], a["data_deps"], a["ctrl_deps"]) != (
                    b["id"], b["name"], b["type"], b["data_deps"], b["ctrl_deps"]):
                bad += 1
                break
    return {"pass": bad == 0, "files": len(graphs), "mismatched_files": bad}


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--size", default="medium", choices=list(SIZES))
    ap.add_argument("--batch", type=int, default=4, help="micro-batch size in sequences")
    ap.add_argument("--seq", type=int, default=1024)
    ap.add_argument("--dp", type=int, default=2)
    ap.add_argument("--tp", type=int, default=2)
    ap.add_argument("--pp", type=int, default=2)
    ap.add_argument("--microbatches", type=int, default=4)
    ap.add_argument("--out", default="traces")
    ap.add_argument("--fused-tp", action="store_true",
                    help="tensor-parallel collectives inside the GEMMs (the peer-memory path): each runs "
                         "concurrently with its GEMM instead of before / after it")
    args = ap.parse_args()
    cfg = SIZES[args.size]
    graphs, table = export(cfg, args.batch, args.seq, args.dp, args.tp, args.pp, args.microbatches, args.out,
                           fused_tp=args.fused_tp)
    res = {"graph": check_graphs(graphs, table),
           "cross_check": cross_check(cfg, args.batch, args.seq, args.dp, args.tp, args.pp, args.microbatches, graphs),
           "roundtrip": check_roundtrip(graphs, args.out)}
    print(json.dumps(res, indent=1))


if __name__ == "__main__":
    main()
