"""The DP x TP x PP scaling model calibrated on measured single-stage runs predicts the held-out
pipelined and hybrid layouts (results/par_8b_*.json are bench lines measured on B200s)."""
import pathlib

from llmt.perf.roofline import Machine
from llmt.perf.scaling import load_links, validate

R = pathlib.Path(__file__).resolve().parents[1] / "results"


def test_calibrated_scaling_model_predicts_held_out_layouts():
    fit = [str(R / f) for f in ("par_8b_tp2_nccl.json", "par_8b_tp4.json", "par_8b_tp8_nccl.json")]
    hold = [str(R / f) for f in ("par_8b_pp2.json", "par_8b_dp2tp2pp2.json")]
    res = validate(fit, hold, Machine.from_peaks(), load_links())
    # two scales, three single-stage runs: the fit is tight
    assert res["fit_mae"] < 0.01
    # the pipelined (PP2) and hybrid (DP2 x TP2 x PP2) runs were not used to fit
    assert res["holdout_mae"] < 0.05
    for x in res["holdout"]:
        assert abs(x["error"]) < 0.08, x
    # the uncalibrated roofline is far off on the same runs
    assert all(x["roofline_ms"] < 0.8 * x["measured_ms"] for x in res["holdout"])


def test_search_with_calibration_matches_validation():
    """The layout search / evaluation with the fitted scales gives the validated prediction."""
    from llmt.config import SIZES
    from llmt.perf.scaling import RUN_KW, StageCompute, evaluate
    fit = [str(R / f) for f in ("par_8b_tp2_nccl.json", "par_8b_tp4.json", "par_8b_tp8_nccl.json")]
    hold = [str(R / "par_8b_dp2tp2pp2.json")]
    m, links = Machine.from_peaks(), load_links()
    res = validate(fit, hold, m, links)
    comp = StageCompute(SIZES["llama3-8b"], 4096, m)
    r = evaluate(SIZES["llama3-8b"], 4096, 16, 8, 2, 2, 2, 2, comp, links, "b200_nvl8_ib",
                 compute_scale=res["compute_scale"], comm_scale=res["comm_scale"], **RUN_KW)
    assert abs(r["step_s"] * 1e3 - res["holdout"][0]["calibrated_ms"]) < 0.01


def test_fused_tensor_parallel_runs_are_modeled_overlapped():
    """Runs whose tensor-parallel collectives ran inside the GEMMs (peer memory, fused gathers)
    are predicted with the collectives overlapped, from scales fitted on the NCCL runs only."""
    import json
    from llmt.perf.scaling import run_kw
    fused = str(R / "par_8b_tp2_p2p_fused.json")
    assert run_kw(json.load(open(fused)))["fused_tp"]
    assert not run_kw(json.load(open(R / "par_8b_tp2_p2p_separate.json")))["fused_tp"]
    fit = [str(R / f) for f in ("par_8b_tp2_nccl.json", "par_8b_tp4.json", "par_8b_tp8_nccl.json")]
    res = validate(fit, [fused], Machine.from_peaks(), load_links())
    assert abs(res["holdout"][0]["error"]) < 0.05, res["holdout"]
