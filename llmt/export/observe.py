"""Cross-check of the operator inventory against a real PyTorch execution trace, and of the
Chakra files against the official decoder when it is installed (reference:
workload_export/observe_pytorch.py:48-171, workload_export/check_export.py:55-80).

One training step of the reference-layout model (llmt.models.llama, SDPA attention; fp32 on
the CPU, bf16 autocast on a GPU) runs under torch.profiler.ExecutionTraceObserver, which
records every dispatched aten operator in order with its input shapes. From the trace:

  GEMMs       outermost aten::mm / aten::addmm / aten::bmm calls, as (M, N, K)
  attention   calls of the fused attention kernels (aten::_scaled_dot_product_*), forward and
              backward counted apart

and from the step's inventory (llmt.perf.roofline.inventory, path "eager", the same network
unfused) the GEMM shapes with their call counts, the per-layer forward order and the attention
calls. Passing means: the same multiset of GEMM shapes (a GEMM and its transpose count as one
shape, as PyTorch may compute C^T = B^T A^T), the same forward GEMM order, the same attention
counts.

    python -m llmt.export.observe --size tiny256 --batch 2 --seq 128 [--device cuda] [--et-dir traces]
"""
from __future__ import annotations

import argparse
import json
import os
import tempfile
from collections import Counter

GEMM_OPS = ("aten::mm", "aten::addmm", "aten::bmm")


def _mnk(name, shapes):
    """(M, N, K) of a GEMM call from the recorded input shapes."""
    if name == "aten::addmm":
        shapes = shapes[1:]
    a, b = shapes[0], shapes[1]
    if name == "aten::bmm":
        return (a[-2], b[-1], a[-1])
    return (a[0], b[1], a[1])


def canon(mnk):
    m, n, k = mnk
    return (min(m, n), max(m, n), k)


def parse_trace(trace: dict):
    """Ordered GEMM shapes and attention forward / backward counts of an ET JSON."""
    nodes = sorted(trace["nodes"], key=lambda n: n["id"])
    names = {n["id"]: n["name"] for n in nodes}
    gemms, att_f, att_b = [], 0, 0
    for n in nodes:
        name, parent = n["name"], names.get(n.get("ctrl_deps"))
        if name in GEMM_OPS and parent not in GEMM_OPS:  # a redispatch to itself is recorded twice
            shapes = (n.get("inputs") or {}).get("shapes") or n.get("input_shapes")
            gemms.append(_mnk(name, shapes))
        elif name.startswith("aten::_scaled_dot_product") and not (parent or "").startswith("aten::_scaled_dot_product"):
            if name.endswith("_backward"):
                att_b += 1
            else:
                att_f += 1
    return gemms, att_f, att_b


def expected(cfg, B, T):
    """GEMM multiset, forward GEMM order and attention counts of one step from the inventory."""
    from llmt.perf.roofline import inventory
    ops = inventory(cfg, B, T, "eager", attn="sdpa")
    multiset, per_layer_fwd, head_fwd = Counter(), [], []
    att_f = att_b = 0
    for o in ops:
        if o.key is None:
            continue
        if o.key[0] == "gemm":
            M, N, K = o.key[1:4]
            multiset[canon((M, N, K))] += o.count
            if o.phase == "fwd":
                (per_layer_fwd if o.count == cfg.L else head_fwd).append((M, N, K))
        elif o.key[0] == "sdpa_fwd":
            att_f += o.count
        elif o.key[0] == "sdpa_bwd":
            att_b += o.count
    order = per_layer_fwd * cfg.L + head_fwd
    return multiset, order, att_f, att_b


def capture(cfg, B, T, device="cpu", et_path=None):
    """Execution trace (JSON dict) of one fwd + bwd + AdamW step of the reference-layout model."""
    import torch
    from torch.profiler import ExecutionTraceObserver
    from llmt.models.llama import build_model, make_batch
    model = build_model(cfg, T, seed=0, attn_impl="sdpa", device=device)
    opt = torch.optim.AdamW(model.parameters(), lr=3e-4, betas=(0.9, 0.95), weight_decay=0.1)
    idx, tgt = make_batch(B, T, cfg.vocab, device)
    amp = torch.autocast("cuda", dtype=torch.bfloat16) if device != "cpu" else torch.autocast("cpu", enabled=False)

    def step():
        with amp:
            loss = model(idx, tgt)
        loss.backward()
        opt.step()
        opt.zero_grad(set_to_none=True)

    step()  # warm-up outside the trace
    path = et_path or os.path.join(tempfile.gettempdir(), f"llmt_et_{os.getpid()}.json")
    et = ExecutionTraceObserver()
    et.register_callback(path)
    et.start()
    step()
    if device != "cpu":
        torch.cuda.synchronize()
    et.stop()
    et.unregister_callback()
    with open(path) as f:
        return json.load(f), path


def cross_check(cfg, B, T, device="cpu", et_path=None) -> dict:
    trace, path = capture(cfg, B, T, device, et_path)
    t_gemms, t_af, t_ab = parse_trace(trace)
    e_multi, e_order, e_af, e_ab = expected(cfg, B, T)
    t_multi = Counter(map(canon, t_gemms))
    t_order = [canon(g) for g in t_gemms[:len(e_order)]]
    res = {
        "trace": path, "trace_nodes": len(trace["nodes"]), "trace_gemms": len(t_gemms),
        "inventory_gemms": sum(e_multi.values()),
        "gemm_multiset_match": t_multi == e_multi,
        "forward_order_match": t_order == [canon(g) for g in e_order],
        "attention": {"trace": [t_af, t_ab], "inventory": [e_af, e_ab]},
    }
    if t_multi != e_multi:
        res["only_in_trace"] = {str(k): v for k, v in (t_multi - e_multi).items()}
        res["only_in_inventory"] = {str(k): v for k, v in (e_multi - t_multi).items()}
    res["pass"] = res["gemm_multiset_match"] and res["forward_order_match"] and (t_af, t_ab) == (e_af, e_ab)
    return res


def official_decode(et_dir) -> dict:
    """Decode every workload.*.et in et_dir with Chakra's own protobuf bindings (the chakra
    package's et_def_pb2 and its length-delimited reader), compare node ids / names / types /
    dependencies with this framework's decoder. Skipped when the package is not installed."""
    try:
        from chakra.schema.protobuf.et_def_pb2 import GlobalMetadata, Node  # type: ignore
        from chakra.src.third_party.utils.protolib import decodeMessage, openFileRd  # type: ignore
    except Exception as e:  # noqa: BLE001
        return {"status": "skipped", "reason": f"chakra protobuf bindings not installed ({type(e).__name__})"}
    from llmt.export import chakra as ck
    files = sorted(f for f in os.listdir(et_dir) if f.startswith("workload.") and f.endswith(".et"))
    bad = []
    for fn in files:
        p = os.path.join(et_dir, fn)
        fh = openFileRd(p)
        meta = GlobalMetadata()
        decodeMessage(fh, meta)
        theirs = []
        node = Node()
        while decodeMessage(fh, node):
            theirs.append((node.id, node.name, node.type, list(node.data_deps), list(node.ctrl_deps)))
            node = Node()
        fh.close()
        _, ours = ck.read_et(p)
        mine = [(n["id"], n["name"], n["type"], n["data_deps"], n["ctrl_deps"]) for n in ours]
        if theirs != mine:
            bad.append(fn)
    return {"status": "pass" if not bad else "fail", "files": len(files), "mismatched": bad}


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--size", default="tiny256")
    ap.add_argument("--batch", type=int, default=2)
    ap.add_argument("--seq", type=int, default=128)
    ap.add_argument("--device", default="cpu")
    ap.add_argument("--et-dir", default=None, help="directory of exported workload.*.et files to decode officially")
    ap.add_argument("--out", default=None)
    args = ap.parse_args()
    from llmt.config import get_config
    res = cross_check(get_config(args.size), args.batch, args.seq, args.device)
    if args.et_dir:
        res["official_decoder"] = official_decode(args.et_dir)
    print(json.dumps(res, indent=1))
    if args.out:
        with open(args.out, "w") as f:
            json.dump(res, f, indent=1)
    raise SystemExit(0 if res["pass"] else 1)


if __name__ == "__main__":
    main()
