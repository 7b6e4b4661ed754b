"""Tensor + sequence parallelism over NVLink peer memory on 2 GPUs of one box against the 1-GPU
model (llmt.parallel.layout_check: a few steps of tiny256 sharded over two ranks, the fp32
masters reassembled and compared). At seq 512 each rank owns whole 128-row blocks of every
micro-batch, so the all-gathers run inside the consuming GEMMs (qkv, w1||w3, the w2 / wo
dgrads); at seq 128 they do not, and the separate peer-store gather runs. Skipped on a box with
one GPU."""
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


@pytest.mark.parametrize("seq", [512, 128])
def test_tp2_peer_memory_matches_single_gpu(seq):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes", "1",
           "--nproc-per-node", "2", "--master-addr", "127.0.0.1", "--master-port", str(_port()),
           "-m", "llmt.parallel.layout_check", "--tp", "2", "--pp", "1", "--microbatches", "2", "--tp-comm", "p2p",
           "--seq", str(seq), "--steps", "3"]
    env = dict(os.environ, PYTHONPATH=ROOT, NCCL_DEBUG="WARN", CUDA_VISIBLE_DEVICES="0,1")
    out = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True, timeout=400)
    assert out.returncode == 0, out.stdout[-3000:] + out.stderr[-3000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.startswith("{")]
    res = json.loads(lines[-1])
    assert res["ok"], res


@pytest.mark.parametrize("linear", ["mxfp8", "fp8"])
def test_tp2_low_precision_linears_match_single_gpu(linear):
    """Block linears in MXFP8 (e4m3, ue8m0 per 32) or tensorwise e4m3 under tensor parallelism with
    NCCL collectives, against the single-GPU model with the same linears (tiny256 with ffn 768, so
    every shard's GEMM dimensions are whole block-scaled tiles)."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes", "1",
           "--nproc-per-node", "2", "--master-addr", "127.0.0.1", "--master-port", str(_port()),
           "-m", "llmt.parallel.tp_check", "--linear", linear, "--ffn", "768", "--steps", "3"]
    env = dict(os.environ, PYTHONPATH=ROOT, NCCL_DEBUG="WARN", CUDA_VISIBLE_DEVICES="0,1")
    out = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True, timeout=400)
    assert out.returncode == 0, out.stdout[-3000:] + out.stderr[-3000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.startswith("{")]
    res = json.loads(lines[-1])
    assert res["ok"] and res["linear"] == linear, res
