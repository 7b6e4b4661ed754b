"""Machine calibration on this GPU (reference: bench_train.py:346-433, roofline.py:419-467).

Measures, with CUDA events after warm-up: dense matmul throughput per precision at 8192^3
(torch/cuBLAS for fp32, tf32, fp16, bf16; torch._scaled_mm for fp8 e4m3; this framework's
tcgen05 GEMMs for bf16, fp8, MXFP8 and NVFP4), a 1 GiB device copy (HBM bandwidth, read + write bytes), an L2-resident
copy, the CPU launch cost of an eager kernel and the GPU gap between kernels replayed from a
CUDA graph. Under torchrun with 2+ ranks it adds NVLink probes: a peer copy between rank 0 and
rank 1 and the NCCL all-reduce bus bandwidth at 1 GiB. Never records the product name.

    python -m llmt.bench.calibrate --label b200 [--out results/calibration_b200.json]
    torchrun --nproc-per-node 8 -m llmt.bench.calibrate --links --out results/links_b200.json
"""
from __future__ import annotations

import argparse
import json
import os
import platform
import statistics
import time

import torch


def _time(fn, warmup=3, iters=20, repeats=3):
    """Seconds per call of `fn`: median over `iters * repeats` launches, each bracketed by its own
    pair of CUDA events on the current stream (events are read after one final synchronize)."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    marks = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
             for _ in range(iters * repeats)]
    for a, b in marks:
        a.record()
        fn()
        b.record()
    torch.cuda.synchronize()
    return statistics.median(a.elapsed_time(b) for a, b in marks) / 1e3


def env_info(label):
    p = torch.cuda.get_device_properties(0)
    major, minor = torch.cuda.get_device_capability()
    return {"arch": f"sm_{major}{minor}", "label": label, "torch": torch.__version__, "cuda": torch.version.cuda,
            "os": platform.platform(), "gpu_count": torch.cuda.device_count(), "sm_count": p.multi_processor_count,
            "gpu_mem_gb": round(p.total_memory / 1e9, 1)}


def _square(n, dtype):
    return torch.randn(n, n, device="cuda").to(dtype)


def _torch_mm(dtype, tf32=False):
    def make(n):
        torch.backends.cuda.matmul.allow_tf32 = tf32
        a, b = _square(n, dtype), _square(n, dtype)
        return lambda: torch.mm(a, b)
    return make


def _torch_fp8(n):
    # torch._scaled_mm wants the second operand column-major: a transposed row-major matrix
    a, bt = _square(n, torch.float8_e4m3fn), _square(n, torch.float8_e4m3fn)
    unit = torch.ones((), device="cuda")
    return lambda: torch._scaled_mm(a, bt.t(), scale_a=unit, scale_b=unit, out_dtype=torch.bfloat16)


def _llmt_gemm(kind):
    """This framework's tcgen05 GEMMs; operands are quantized once, outside the timed calls."""
    def make(n):
        from llmt.ops import native as N
        a, b = _square(n, torch.bfloat16), _square(n, torch.bfloat16)
        out = torch.empty(n, n, device="cuda", dtype=torch.bfloat16)
        if kind == "bf16":
            return lambda: N.gemm(a, b, out=out)
        if kind == "fp8":
            (aq, _, sa), (bq, _, sb) = N.fp8_quant(a, transpose=False), N.fp8_quant(b, transpose=False)
            return lambda: N.gemm_fp8(aq, bq, sa, sb, out=out)
        fmt = {"mxfp8": N.MXFP8, "nvfp4": N.NVFP4}[kind]
        ar, br = N.mx_quant(a, fmt)[0], N.mx_quant(b, fmt)[0]
        return lambda: N.gemm_mx(fmt, ar, br, out=out)
    return make


# precision name -> builder(n) returning the call to time (torch / cuBLAS rows first, then ours)
MATMULS = {
    "fp32": _torch_mm(torch.float32), "tf32": _torch_mm(torch.float32, tf32=True),
    "fp16": _torch_mm(torch.float16), "bf16": _torch_mm(torch.bfloat16), "fp8": _torch_fp8,
    "bf16_llmt": _llmt_gemm("bf16"), "fp8_llmt": _llmt_gemm("fp8"), "mxfp8_llmt": _llmt_gemm("mxfp8"),
    "nvfp4_llmt": _llmt_gemm("nvfp4"),
}


def matmul_tflops(precision, n=8192):
    """Dense n^3 matmul throughput of one precision, {"status", "tflops", "ms"}; a precision that
    fails to build or run is reported with its error and does not stop the calibration."""
    saved_tf32 = torch.backends.cuda.matmul.allow_tf32
    try:
        call = MATMULS[precision](n)
        sec = _time(call)
        return {"status": "ok", "tflops": round(2.0 * n ** 3 / sec / 1e12, 1), "ms": round(sec * 1e3, 3)}
    except Exception as e:  # noqa: BLE001
        return {"status": "error", "error": (type(e).__name__ + ": " + str(e))[:300]}
    finally:
        torch.backends.cuda.matmul.allow_tf32 = saved_tf32
        torch.cuda.empty_cache()


def copy_gbs(nbytes=1 << 30):
    src = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    dst = torch.empty_like(src)
    sec = _time(lambda: dst.copy_(src), iters=10)
    return round(2 * nbytes / sec / 1e9, 1)


def graph_gap_us(n=1000):
    from llmt.perf.validate import measure_gap_us
    return round(measure_gap_us(n), 3)


def launch_us():
    x = torch.zeros(1, device="cuda")
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(2000):
        x.add_(1.0)
    t1 = time.perf_counter()
    torch.cuda.synchronize()
    return round((t1 - t0) / 2000 * 1e6, 2)


def calibrate(label):
    info = env_info(label)
    mm = {p: matmul_tflops(p) for p in ("fp32", "tf32", "fp16", "bf16", "fp8", "bf16_llmt", "fp8_llmt", "mxfp8_llmt",
                                        "nvfp4_llmt")}
    return {**info, "time": time.strftime("%Y-%m-%d %H:%M:%S"), "matmul": mm, "hbm_gbs": copy_gbs(),
            "l2_copy_gbs": copy_gbs(16 << 20), "launch_overhead_us": launch_us(), "gpu_gap_us": graph_gap_us()}


def link_probes():
    import datetime

    import torch.distributed as dist
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    out = {"world": world}
    n = 1 << 30
    x = torch.ones(n // 2, dtype=torch.bfloat16, device="cuda")
    sec = _time(lambda: dist.all_reduce(x), warmup=2, iters=5, repeats=2)
    out["nccl_allreduce_busbw_gbs"] = round(2 * (world - 1) / world * n / sec / 1e9, 1)
    y = torch.empty(n // world, dtype=torch.uint8, device="cuda")
    z = torch.empty(n, dtype=torch.uint8, device="cuda")
    sec = _time(lambda: dist.reduce_scatter_tensor(y, z), warmup=2, iters=5, repeats=2)
    out["nccl_reduce_scatter_busbw_gbs"] = round((world - 1) / world * n / sec / 1e9, 1)
    dist.barrier()
    if rank == 0 and world >= 2 and torch.cuda.device_count() >= 2:
        a = torch.empty(n, dtype=torch.uint8, device="cuda:0")
        b = torch.empty(n, dtype=torch.uint8, device="cuda:1")
        sec = _time(lambda: b.copy_(a, non_blocking=True), warmup=2, iters=5, repeats=2)
        out["p2p_copy_gbs"] = round(n / sec / 1e9, 1)
    dist.barrier()
    dist.destroy_process_group()
    return out if rank == 0 else None


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--label", default="b200")
    ap.add_argument("--links", action="store_true", help="NVLink / NCCL probes (run under torchrun)")
    ap.add_argument("--out", default=None)
    args = ap.parse_args()
    res = link_probes() if args.links else calibrate(args.label)
    if res is None:
        return
    print(json.dumps(res, indent=1))
    if args.out:
        with open(args.out, "w") as f:
            json.dump(res, f, indent=1)


if __name__ == "__main__":
    main()
