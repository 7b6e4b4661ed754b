"""Data parallelism on 2 GPUs of one box against the 1-GPU model (llmt.parallel.dp_check: every
rank trains on its own batch; rank 0 also trains the model alone on all batches as
micro-batches and compares the fp32 masters and the bf16 shadows after three steps). Runs each
transport as a torchrun child on 127.0.0.1; skipped on a box with one GPU."""
import json
import os
import socket
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _multicast():
    from llmt.parallel.dp import pick_mode
    return pick_mode("auto", 0) == "nvls"


@pytest.mark.parametrize("mode,graph", [("nccl", False), ("nvls", False), ("nvls", True), ("nvls-overlap", True),
                                        ("fused", False)])
def test_dp2_matches_single_gpu(mode, graph):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    if mode.startswith("nvls") and not _multicast():
        pytest.skip("no NVLink multicast on this box")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes", "1",
           "--nproc-per-node", "2", "--master-addr", "127.0.0.1", "--master-port", str(_port()),
           "-m", "llmt.parallel.dp_check", "--mode", mode, "--steps", "3"] + (["--graph"] if graph else [])
    env = dict(os.environ, PYTHONPATH=ROOT, NCCL_DEBUG="WARN", CUDA_VISIBLE_DEVICES="0,1")
    out = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True, timeout=400)
    assert out.returncode == 0, out.stdout[-3000:] + out.stderr[-3000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.startswith("{")]
    res = json.loads(lines[-1])
    assert res["ok"] and res["dp_error_code"] == 0, res
