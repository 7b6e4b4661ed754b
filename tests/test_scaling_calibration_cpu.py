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
