"""CPU tests: Chakra export checks, perf-model consistency, scaling model, checkpoint layout."""
import math
import os
import sys

import pytest
import torch

from llmt.config import SIZES, get_config, model_flops_per_token
from llmt.export import chakra as ck
from llmt.export import trace
from llmt.perf import roofline, scaling

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_chakra_node_roundtrip(tmp_path):
    nodes = [{"id": 0, "name": "gemm", "type": ck.COMP_NODE, "data_deps": [], "ctrl_deps": [], "duration_micros": 7,
              "inputs": {"shapes": "[[4, 4]]"}, "outputs": {"shapes": "[[4, 4]]"},
              "attrs": [("num_ops", "int64_val", 123), ("tensor_size", "uint64_val", 2 ** 40), ("is_cpu_op", "bool_val", False)]},
             {"id": 1, "name": "rs", "type": ck.COMM_COLL_NODE, "data_deps": [0], "ctrl_deps": [],
              "attrs": [("comm_type", "int64_val", ck.REDUCE_SCATTER), ("comm_size", "int64_val", 4096),
                        ("pg_name", "string_val", "3"), ("neg", "int64_val", -5)]}]
    p = tmp_path / "w.et"
    ck.write_et(p, nodes, [("rank", "int64_val", 0)])
    meta, got = ck.read_et(p)
    assert meta["version"] == ck.SCHEMA_VERSION
    assert [n["id"] for n in got] == [0, 1]
    assert got[1]["data_deps"] == [0]
    assert ck.attr(got[0], "tensor_size") == 2 ** 40
    assert ck.attr(got[1], "neg") == -5
    assert ck.attr(got[1], "pg_name") == "3"


@pytest.mark.parametrize("dp,tp,pp,m", [(2, 2, 2, 4), (1, 1, 4, 8), (4, 2, 1, 2)])
def test_export_graph_checks(tmp_path, dp, tp, pp, m):
    cfg = SIZES["tiny"]
    graphs, table = trace.export(cfg, 2, 256, dp, tp, pp, m, str(tmp_path))
    g = trace.check_graphs(graphs, table)
    assert g["pass"], g["errors"]
    assert trace.cross_check(cfg, 2, 256, dp, tp, pp, m, graphs)["pass"]
    assert trace.check_roundtrip(graphs, str(tmp_path))["pass"]
    if pp > 1:
        assert g["send_recv_pairs"] == 2 * (pp - 1) * m * dp * tp
    kinds = {ck.attr(n, "comm_type") for n in ck.read_et(tmp_path / "workload.0.et")[1] if n["type"] == ck.COMM_COLL_NODE}
    if dp > 1:
        assert ck.REDUCE_SCATTER in kinds and ck.ALL_GATHER in kinds


def test_schedule_1f1b_covers_all_microbatches():
    for p in (1, 2, 4):
        for s in range(p):
            order = trace.schedule_1f1b(s, p, 6)
            assert sorted(i for k, i in order if k == "F") == list(range(6))
            assert sorted(i for k, i in order if k == "B") == list(range(6))
            # a backward never precedes its forward
            pos = {(k, i): j for j, (k, i) in enumerate(order)}
            assert all(pos[("F", i)] < pos[("B", i)] for i in range(6))


def test_native_inventory_matmul_flops_match_model_flops():
    """GEMM FLOPs of the native inventory = 6 x matmul params x tokens + the recomputed lm head."""
    cfg = SIZES["medium"]
    B, T = 4, 1024
    ops = roofline.inventory(cfg, B, T, "native")
    gemm = sum(o.total_flops for o in ops if o.cat in ("matmul", "loss"))
    att = sum(o.total_flops for o in ops if o.cat == "attention")
    N = B * T
    head_recompute = 2.0 * N * cfg.vocab * cfg.d
    norm_params = 2 * cfg.d * cfg.L + cfg.d  # counted by the reference's "matmul params", not GEMMs
    assert math.isclose(gemm - head_recompute,
                        model_flops_per_token(cfg, T) * N - 12 * cfg.L * cfg.d * T * N - 6 * norm_params * N,
                        rel_tol=1e-9)
    # causal attention: fwd 2 + bwd 5 = 7 B H T^2 hd per layer (the 12 L d T term counts full attention)
    assert math.isclose(att, 7.0 * B * cfg.H * T * T * cfg.hd * cfg.L, rel_tol=1e-9)


def test_predict_paths_ordering():
    cfg = SIZES["medium"]
    m = roofline.Machine.from_peaks()
    t = {p: roofline.predict(roofline.inventory(cfg, 4, 1024, p), m, graph=(p == "native")).total_ms
         for p in ("native", "triton", "eager")}
    assert t["native"] < t["triton"] < t["eager"]


def test_scaling_model_layouts():
    cfg = SIZES["medium"]
    links = scaling.load_links()
    comp = scaling.StageCompute(cfg, 1024, roofline.Machine.from_peaks())
    r = scaling.evaluate(cfg, 1024, 16, 8, 2, 2, 2, 1, comp, links, "b200_nvl8_ib")
    assert r is not None and r["step_s"] > 0 and 0 < r["mfu"] < 1
    assert scaling.evaluate(cfg, 1024, 16, 8, 3, 1, 1, 1, comp, links, "b200_nvl8_ib") is None  # 3 x 1 x 1 != 8
    best = scaling.search(cfg, 1024, 512, 64, comp, links, "b200_nvl8_ib")
    assert best and best["dp"] * best["tp"] * best["pp"] == 64
    # more GPUs never lower the aggregate throughput of the best layout here
    b8 = scaling.search(cfg, 1024, 512, 8, comp, links, "b200_nvl8_ib")
    assert best["tokens_per_s"] > b8["tokens_per_s"]


def test_checkpoint_file_loads_into_reference_model(tmp_path):
    """A gathered checkpoint's model state_dict has exactly the reference keys and loads there."""
    from llmt.ckpt import checkpoint
    from llmt.models.llama import build_model
    cfg = get_config("tiny256")
    m = build_model(cfg, 128, seed=3)
    path = str(tmp_path / "ck.pt")
    checkpoint.save(path, m, meta={"step": 7})
    ck_ = torch.load(path)
    assert ck_["meta"]["step"] == 7
    ref = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isfile(os.path.join(ref, "bench_train.py")):
        pytest.skip("reference not installed under baseline/_ref")
    sys.path.insert(0, ref)
    import bench_train as bt
    r = bt.LlamaModel(bt.ModelConfig(d=cfg.d, L=cfg.L, H=cfg.H, ffn=cfg.ffn), 128)
    r.load_state_dict(ck_["model"])
    for k, v in r.state_dict().items():
        assert torch.equal(v, m.state_dict()[k])
    m2 = build_model(cfg, 128, seed=9)
    checkpoint.load(path, m2)
    for k, v in m2.state_dict().items():
        assert torch.equal(v, m.state_dict()[k])


def test_astra_inputs_and_acceptance(tmp_path):
    from llmt.export.astra import accept, run
    res = run(str(tmp_path), 8, None)
    assert res["status"] == "unavailable"
    net = open(res["inputs"]["network"]).read()
    assert "npus_count: [ 8 ]" in net and "725.0" in net
    ok, ticks = accept("sys[0] finished, 100 cycles\nsys[1] finished, 100 cycles", 2)
    assert ok and ticks == {0: 100, 1: 100}
    ok, _ = accept("sys[0] finished, 100 cycles\nsys[1] finished, 90 cycles", 2)
    assert not ok
    # pipeline stages finish at different ticks; the ranks of one stage agree (tp innermost)
    log = "\n".join(f"sys[{r}] finished, {t} cycles, exposed communication 7 cycles"
                     for r, t in ((0, 500), (1, 500), (2, 480), (3, 480)))
    ok, ticks = accept(log, 4, tp=2, pp=2)
    assert ok and max(ticks.values()) == 500
    ok, _ = accept(log.replace("sys[3] finished, 480", "sys[3] finished, 470"), 4, tp=2, pp=2)
    assert not ok
    ok, _ = accept("\n".join(log.splitlines()[:3]), 4, tp=2, pp=2)  # one rank's line lost, both stages seen
    assert ok


def test_execution_trace_cross_check_matches_inventory(tmp_path):
    """A real PyTorch execution trace of one step (tiny256, CPU fp32) has the GEMM shapes, the
    forward GEMM order and the attention calls that the step inventory lists."""
    from llmt.config import get_config
    from llmt.export.observe import cross_check
    res = cross_check(get_config("tiny256"), 2, 64, "cpu", et_path=str(tmp_path / "et.json"))
    assert res["gemm_multiset_match"], res
    assert res["forward_order_match"]
    assert res["attention"]["trace"] == res["attention"]["inventory"] == [4, 4]
    assert res["pass"]


def test_official_chakra_decoder_check_skips_or_passes(tmp_path):
    from llmt.config import get_config
    from llmt.export.observe import official_decode
    from llmt.export.trace import export
    export(get_config("tiny256"), 1, 64, 2, 1, 2, 2, outdir=str(tmp_path))
    res = official_decode(str(tmp_path))
    assert res["status"] in ("skipped", "pass"), res


def test_export_fused_tensor_parallel_collectives(tmp_path):
    """With the collectives inside the GEMMs (--fused-tp) every gather and reduce-scatter still
    appears once per site (same group sequences, checks pass), but no GEMM waits for its gather:
    the gather and the GEMM start from the same input, and the next operator waits for both."""
    from llmt.config import get_config
    from llmt.export import trace
    cfg = get_config("tiny256")
    plain, _ = trace.export(cfg, 2, 256, 1, 2, 2, 2)
    graphs, table = trace.export(cfg, 2, 256, 1, 2, 2, 2, str(tmp_path / "fused"), fused_tp=True)
    assert trace.check_graphs(graphs, table)["pass"]
    assert trace.check_roundtrip(graphs, str(tmp_path / "fused"))["pass"]
    for r, gr in graphs.items():
        colls = [n for n in gr.nodes if n["kind"] == "coll"]
        assert len(colls) == len([n for n in plain[r].nodes if n["kind"] == "coll"])
        ag = {n["id"] for n in colls if n["name"].startswith("SP all-gather")}
        rs = {n["id"] for n in colls if n["name"].startswith("SP reduce-scatter in")}
        assert ag and rs
        consumers = [n for n in gr.nodes if n["kind"] == "comp" and n["phase"] == "fwd"
                     and n["name"].startswith(("qkv", "w1||w3"))]
        assert consumers and not any(ag & set(n["data_deps"]) for n in consumers)
        # every gather and every fused reduce-scatter is waited for by a later node
        assert all(any(i in n["data_deps"] for n in gr.nodes) for i in ag | rs)


def test_mfu_gap_breakdown_sums_to_measured_step():
    """The MFU-gap breakdown of each measured step in the committed validation results places
    every millisecond: its terms sum to the measured step time, the ideal term is the MFU share."""
    import json
    import pathlib
    from llmt.perf.validate import mfu_gap
    res = json.loads((pathlib.Path(__file__).resolve().parents[1] / "results" / "perf_model_validation.json").read_text())
    peak = res["machine"]["bf16_tflops"]
    for r in res["rows"]:
        gap = mfu_gap(r, peak, res["summary"]["alpha"])
        assert abs(sum(gap.values()) - r["measured_ms"]) < 0.01
        assert abs(gap["model FLOPs at the bf16 peak"] / r["measured_ms"] - r["mfu"]) < 0.01
        assert gap["GEMMs below peak"] > 0 and gap["optimizer"] > 0


def test_scaling_model_explains_missing_layouts():
    """When no layout of n GPUs works the scaling model says why: batch too small, or weights and
    optimizer state too large even at the widest split."""
    from llmt.config import SIZES
    from llmt.perf.roofline import Machine
    from llmt.perf.scaling import StageCompute, all_layouts, load_links, no_layout_reason
    links, m = load_links(), Machine.from_peaks()
    for name, G, n, word in (("llama3-8b", 1, 4096, "too small"), ("llama3-70b", 8, 2, "do not fit")):
        cfg = SIZES[name]
        assert not all_layouts(cfg, 4096, G, n, StageCompute(cfg, 4096, m), links, "b200_nvl8_ib")
        assert word in no_layout_reason(cfg, 4096, G, n, links, "b200_nvl8_ib")


def test_scaling_chart_svg():
    """The scaling model's JSON renders as a plain-SVG MFU-vs-GPUs chart, one line per model."""
    from llmt.bench.charts import scaling_chart
    rows = [{"model": m, "gpus": n, "tokens_per_s": 1e6 * n, "mfu": 0.5 - 0.01 * n.bit_length()}
            for m in ("medium", "llama3-8b") for n in (8, 64, 1024)]
    svg = scaling_chart(rows)
    assert svg.startswith("<svg") and svg.count("<polyline") == 2 and "llama3-8b" in svg


def test_untimed_gemm_shapes_run_at_the_timed_efficiency():
    """Shapes without a measured time (too large for one GPU, or never timed) are derated by the
    FLOP-weighted efficiency of the timed GEMMs instead of running at the peak."""
    from llmt.perf.roofline import Machine, gemm_efficiency, gemm_op, predict
    m = Machine.from_peaks()
    peak = m.bf16_tflops * 1e12
    timed = gemm_op("timed", 4096, 4096, 4096, "fwd", 1, "nt")
    st = {"|".join(str(x) for x in timed.key): 2.0 * timed.flops / peak}  # at half the peak
    assert abs(gemm_efficiency(st, peak) - 0.5) < 1e-9
    big = gemm_op("untimed", 8192, 8192, 8192, "fwd", 1, "nt")
    p = predict([timed, big], m, st)
    assert [o["bound"] for o in p.ops] == ["measured", "derated"]
    assert abs(p.ops[1]["ms"] - 2e3 * big.flops / peak) < 1e-3
    assert predict([big], m).ops[0]["bound"] == "compute"  # no shape times: plain roofline
