"""The reference-stack multi-GPU baseline (stock PyTorch tensor parallelism / FSDP2 around the
reference's module structure) runs on gloo ranks: two CPU processes, tiny256, TP2 and DP2."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.parametrize("layout,port", [(["--tp", "2"], 29631), (["--dp", "2"], 29632)])
def test_reference_stack_layout_runs_on_gloo(layout, port):
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes", "1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", str(port), "-m", "llmt.bench.ref_parallel",
           "--model", "tiny256", "--seq", "64", "--global-batch", "2", "--steps", "1", "--warmup", "1", *layout]
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="", PYTHONPATH=ROOT)
    out = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-3000:]
    line = [l for l in out.stdout.splitlines() if l.startswith("{")][-1]
    res = json.loads(line)
    assert res["n_gpus"] == 2 and 8.0 < res["final_loss"] < 11.0
