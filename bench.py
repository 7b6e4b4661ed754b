"""Headline benchmark: training tokens/s (+ MFU) of the 'medium' (~375M) Llama-style model,
data parallel over N B200s (weak scaling: per-GPU batch 4 x seq 1024, synthetic tokens,
random-init weights), full step = forward + backward + AdamW.

    python bench.py [--gpus N --steps K --warmup W] [--impl native|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...      (N > 1)

Timing: W untimed warm-up steps, then exactly K steps bracketed by a barrier and
torch.cuda.synchronize() on both sides, measured with CUDA events on the launching stream,
max over ranks. The step's working set (weights, gradients, optimizer state, activations:
several GB) is far larger than the 126 MB L2, so no explicit flush runs between steps.
An end-to-end figure through the public Trainer API (pinned H2D copy of each step's tokens
and a D2H read of its loss inside the timed loop) is reported as "e2e". SM clocks and
throttle reasons are sampled through NVML during the timed region. Rank 0 prints one JSON line.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

# The reference's published best medium row (FP8 linears, 57,365 tokens/s), measured on ONE sm_120
# GPU: a different part, so vs_baseline is a cross-hardware ratio, labelled as such in the output line.
BASELINE_TOKS = 57365.0
BASELINE_LABEL = "reference's published medium row 8 (FP8 linears) on one sm_120 GPU, not B200"
METRIC = "train tokens/s + MFU, 1/2/4/8 B200, max over ranks; fused-path roofline %"
MODEL = "medium"
PER_GPU_BATCH = 4
SEQ = 1024


class ClockSampler:
    """Samples SM clock and clock-event reasons via NVML every 200 ms (read-only)."""

    REASONS = {
        "sw_power_cap": 0x4, "hw_slowdown": 0x8, "sync_boost": 0x10, "sw_thermal_slowdown": 0x20,
        "hw_thermal_slowdown": 0x40, "hw_power_brake_slowdown": 0x80,
    }

    def __init__(self, device_index):
        self.samples, self.reasons = [], set()
        self.max_mhz = None
        self._stop = threading.Event()
        self._t = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception:  # noqa: BLE001 - NVML is optional
            self.nv = None

    def _run(self):
        while not self._stop.is_set():
            try:
                self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
                mask = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                for k, v in self.REASONS.items():
                    if mask & v:
                        self.reasons.add(k)
            except Exception:  # noqa: BLE001
                pass
            self._stop.wait(0.2)

    def __enter__(self):
        if self.nv is not None:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self._t is not None:
            self._t.join()

    def summary(self):
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None, "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


def setup_dist(n):
    if n > 1 or "RANK" in os.environ:
        rank = int(os.environ.get("RANK", 0))
        world = int(os.environ.get("WORLD_SIZE", 1))
        local = int(os.environ.get("LOCAL_RANK", 0))
        torch.cuda.set_device(local)
        if world > 1:
            import datetime
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                    device_id=torch.device("cuda", local))
        return rank, world, local
    torch.cuda.set_device(0)
    return 0, 1, 0


def max_over_ranks(x, world):
    if world == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world):
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()


def timed(fn, steps, world):
    """K steps between barrier + synchronize; CUDA-event device time (ms) and host wall time."""
    barrier(world)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.perf_counter()
    start.record()
    for _ in range(steps):
        fn()
    end.record()
    torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    barrier(world)
    return start.elapsed_time(end), wall


def peak_tflops():
    """bf16 dense peak for MFU. The timed region is a seconds-long loop under the power cap, so the
    denominator is the sustained cuBLAS figure (not the burst one)."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["bf16_tflops_sustained"])
    except Exception:  # noqa: BLE001
        return 1400.0   # this pool's sustained fallback figure


def run_native(args, rank, world, local):
    from llmt.config import get_config, model_flops_per_token
    from llmt.models.llama import make_batch
    from llmt.ops import native
    from llmt.train import Trainer
    cfg = get_config(MODEL)
    dp = None
    if world > 1:
        from llmt.parallel.dp import DataParallel
        dp = DataParallel(world, rank, mode=args.dp_mode)  # "auto": NVLS where multicast exists
    tr = Trainer(cfg, PER_GPU_BATCH, SEQ, device=f"cuda:{local}", cuda_graph=not args.no_graph, dp=dp,
                 linear=args.linear)
    idx, tgt = make_batch(PER_GPU_BATCH, SEQ, cfg.vocab, "cpu", seed=rank)
    idx, tgt = idx.pin_memory(), tgt.pin_memory()
    tr.set_batch(idx.cuda(local), tgt.cuda(local))
    native.LAUNCHES.reset()
    for _ in range(args.warmup):
        tr.run_step()
    torch.cuda.synchronize()
    launches_per_step = native.LAUNCHES.per_step(tr)
    with ClockSampler(local) as clk:
        ms, _ = timed(tr.run_step, args.steps, world)
        # end to end through the public API: pinned H2D of the tokens + D2H of the loss, every step
        losses = []
        e2e_ms, e2e_wall = timed(lambda: losses.append(tr.train_step(idx, tgt)), args.steps, world)
    ms = max_over_ranks(ms, world)
    e2e_wall = max_over_ranks(e2e_wall * 1000.0, world)
    tokens = PER_GPU_BATCH * SEQ * world
    ms_step = ms / args.steps
    tok_s = tokens / (ms_step / 1e3)
    e2e_tok_s = tokens / (e2e_wall / args.steps / 1e3)
    tflops = model_flops_per_token(cfg, SEQ) * tok_s / world / 1e12
    err = native.gemm_error_code() | native.attn_error_code() | native.ext().dp_error_code(False)
    tr.release()
    dp_mode = dp.mode if dp is not None else None
    if dp is not None:
        dp.close()
    return dict(value=tok_s, ms_per_step=ms_step, mfu=tflops / peak_tflops(), tflops_per_gpu=tflops, dp_mode=dp_mode,
                e2e=dict(value=round(e2e_tok_s, 1), unit="tokens/s", h2d_bytes_per_step=2 * idx.numel() * 8,
                         d2h_bytes_per_step=4, wall_ms_per_step=round(e2e_wall / args.steps, 3)),
                gpu_launches=launches_per_step * args.steps, final_loss=losses[-1] if losses else None,
                kernel_error_code=err, clocks=clk.summary())


def run_reference(args, rank, world, local):
    """The unmodified reference stack (baseline/_ref) through its own build()/LlamaModel API.
    N > 1 wraps its model in stock torch DDP over NCCL (the reference has no multi-GPU code)."""
    ref = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(ref):
        return {"unavailable": "reference not installed under baseline/_ref"}
    sys.path.insert(0, ref)
    import bench_train as bt
    cfg = bt.SIZES[MODEL]
    row = dict(bt.LADDER)[args.ref_row]
    run = dict(name=args.ref_row, size=MODEL, batch=PER_GPU_BATCH, seq=SEQ, ckpt=False, nvtx=False, lr=3e-4, **row)
    device = f"cuda:{local}"
    if world == 1:
        model, opt, step = bt.build(cfg, run, device=device)
    else:
        from torch.nn.parallel import DistributedDataParallel as DDP
        ops = bt.load_ops(run["kernels"], run.get("fused_ops"))
        torch.manual_seed(0)
        model = bt.LlamaModel(cfg, SEQ, run["attn"], ops, False, False, linear=run.get("linear", "bf16")).to(device)
        ddp = DDP(model, device_ids=[local])
        opt = torch.optim.AdamW(model.parameters(), lr=3e-4, betas=(0.9, 0.95), weight_decay=0.1,
                                **(dict(fused=True) if run["fused_adam"] else dict(foreach=True)))
        fwd = torch.compile(ddp) if run["compile"] else ddp
        g = torch.Generator(device="cpu").manual_seed(rank)
        data = torch.randint(0, cfg.vocab, (PER_GPU_BATCH, SEQ + 1), generator=g).to(device)
        idx, tgt = data[:, :-1].contiguous(), data[:, 1:].contiguous()

        def step():
            with bt.set_precision(run["precision"]):
                loss = fwd(idx, tgt)
            loss.backward()
            opt.step()
            opt.zero_grad(set_to_none=True)
            return loss
    # End to end, as for the native arm: every step copies its tokens from pinned host memory into
    # the step's own input tensors and reads the loss back to the host.
    if world == 1:
        cells = dict(zip(step.__code__.co_freevars, (c.cell_contents for c in step.__closure__)))
        idx, tgt = cells["idx"], cells["tgt"]   # the device batch the stock step() closes over
    idx_h, tgt_h = idx.cpu().pin_memory(), tgt.cpu().pin_memory()
    losses = []

    def e2e_step():
        idx.copy_(idx_h, non_blocking=True)
        tgt.copy_(tgt_h, non_blocking=True)
        losses.append(step().item())

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        ms, wall = timed(step, args.steps, world)
        _, e2e_wall = timed(e2e_step, args.steps, world)
    ms = max_over_ranks(ms, world)
    e2e_wall = max_over_ranks(e2e_wall * 1000.0, world)
    tokens = PER_GPU_BATCH * SEQ * world
    ms_step = ms / args.steps
    tok_s = tokens / (ms_step / 1e3)
    tflops = bt.model_flops_per_token(cfg, SEQ) * tok_s / world / 1e12
    e2e = dict(value=round(tokens / (e2e_wall / args.steps / 1e3), 1), unit="tokens/s",
               h2d_bytes_per_step=idx_h.numel() * idx_h.element_size() + tgt_h.numel() * tgt_h.element_size(),
               d2h_bytes_per_step=4, wall_ms_per_step=round(e2e_wall / args.steps, 3))
    return dict(value=tok_s, ms_per_step=ms_step, mfu=tflops / peak_tflops(), tflops_per_gpu=tflops,
                ref_row=args.ref_row, clocks=clk.summary(), e2e=e2e, final_loss=losses[-1])


def main():
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", default="native", choices=["native", "reference"])
    p.add_argument("--ref-row", default="5 + torch.compile",
                   help="reference ladder row (default: its fastest bf16 row on B200)")
    p.add_argument("--dp-mode", default="auto",
                   choices=["auto", "nvls", "nvls-overlap", "fused", "fused-overlap", "nccl"],
                   help="data-parallel transport: auto = nvls where the GPUs support NVLink multicast, else "
                        "nccl; nvls = bf16 gradient cast + one kernel reducing in the NVSwitch, AdamW and "
                        "multicasting the weights; nvls-overlap = the same per bucket during the backward; "
                        "fused = peer-memory kernel; nccl = reduce-scatter / all-gather")
    p.add_argument("--no-graph", action="store_true")
    p.add_argument("--linear", default="bf16", choices=["bf16", "fp8", "mxfp8", "nvfp4"],
                   help="block linears (every GEMM of qkv, wo, w1||w3, w2; the head stays bf16) in bf16, on "
                        "tensorwise e4m3 operands, or block-scaled MXFP8 / NVFP4. With --impl reference, fp8 "
                        "and nvfp4 select the reference's rows '8 + FP8 linears (e4m3)' / '9 + NVFP4 linears "
                        "(e2m1)' unless --ref-row is given")
    args = p.parse_args()
    if args.impl == "reference" and args.ref_row == "5 + torch.compile":
        args.ref_row = {"fp8": "8 + FP8 linears (e4m3)", "nvfp4": "9 + NVFP4 linears (e2m1)"}.get(args.linear,
                                                                                                args.ref_row)
    if args.warmup < 3:
        args.warmup = 3
    rank, world, local = setup_dist(args.gpus)
    try:
        res = run_reference(args, rank, world, local) if args.impl == "reference" else run_native(args, rank, world, local)
    finally:
        pass
    if rank == 0:
        if "unavailable" in res:
            print(json.dumps({"impl": "reference", **res}))
        else:
            par = f"dp{world}"
            line = {
                "metric": METRIC, "value": round(res["value"], 1), "unit": "tokens/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(res["ms_per_step"], 3),
                "higher_is_better": True, "scaling": "weak",
                "vs_baseline": round(res["value"] / BASELINE_TOKS, 3), "vs_baseline_is": BASELINE_LABEL,
                "dtype": {"bf16": "bf16", "fp8": "fp8 e4m3 tensorwise block linears, bf16 rest",
                          "mxfp8": "mxfp8 (e4m3, ue8m0 per 32) block linears, bf16 rest",
                          "nvfp4": "nvfp4 (e2m1, ue4m3 per 16) block linears, bf16 rest"}[args.linear],
                "data": "synthetic uniform-random tokens, random-init weights",
                "config": {"model": MODEL, "global_batch": PER_GPU_BATCH * world, "seq_len": SEQ,
                           "parallelism": par, "l2": "working set >> 126 MB L2; no flush", "linear": args.linear,
                           "mfu": round(res["mfu"], 4), "tflops_per_gpu": round(res["tflops_per_gpu"], 1),
                           "dp_transport": res.get("dp_mode")},
                "clocks": res["clocks"],
            }
            line["e2e"] = res["e2e"]
            line["final_loss"] = res["final_loss"]
            if args.impl == "reference":
                line["impl"] = "reference"
                line["config"]["ref_row"] = res["ref_row"]
            else:
                line["gpu_launches"] = res["gpu_launches"]
                line["kernel_error_code"] = res["kernel_error_code"]
            print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
