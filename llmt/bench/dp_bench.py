"""Data-parallel step kernels alone (torchrun, one rank per GPU): the NVLS fused step and the NCCL
step on a flat buffer of a model's parameter count, timed with CUDA events between barriers,
max over ranks, against their NVLink roofline.

The roofline of one step, per GPU (P parameters, N ranks):
  nccl     reduce-scatter of fp32 gradients and all-gather of bf16 weights: (N - 1) / N x P x 4
           bytes leave (and (N - 1) / N x P x 2 arrive) at the measured peer-copy bandwidth per
           direction (llmt/perf/links.json); HBM for the cast, the AdamW shard (master, m, v read
           and written: 24 B per shard parameter) and the arriving weights in parallel
  nvls     the bf16 cast first (read 4 B, write 2 B per parameter: HBM, in series), then the
           multicast kernel, bound by the larger of its NVLink bytes and its HBM bytes. Through
           the switch every rank's whole bf16 gradient is read once for the ld_reduce of all
           shards (P x 2 leave, this GPU's own shard included) and every shard's new weights
           land in every rank, this one included (P x 2 arrive), plus the shard's reduced
           gradient (P / N x 2 in) and its multicast stores (P / N x 2 out): (1 + 1 / N) x P x 2
           each way. Kernel HBM: the gradient read by the switch (2 B), the AdamW shard
           (24 B / N) and the arriving weights (2 B) per parameter
The NVLS kernel moves bf16 gradients (its cast is part of the timed step); the NCCL step
reduce-scatters the fp32 gradients as the "nccl" mode does.

    torchrun --nproc-per-node 8 -m llmt.bench.dp_bench --model medium --iters 20
"""
from __future__ import annotations

import argparse
import datetime
import json
import os

import torch
import torch.distributed as dist


class _Flat:
    """The parts of llmt.models.native.FlatParams the data-parallel steps touch."""

    def __init__(self, numel, device):
        self.numel = numel
        self.master = torch.randn(numel, device=device) * 0.02
        self.grad = torch.randn(numel, device=device) * 1e-3
        self.shadow = self.master.bfloat16()
        self.buckets = []

    def rebind(self, grad, shadow):
        self.grad, self.shadow = grad, shadow

    def refresh_shadow(self):
        self.shadow.copy_(self.master)


def main():
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--model", default="medium")
    p.add_argument("--iters", type=int, default=20)
    p.add_argument("--modes", default="nvls,nccl")
    p.add_argument("--json", default=None)
    args = p.parse_args()
    from llmt.config import count_params, get_config
    from llmt.parallel.dp import DataParallel
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    total, _ = count_params(get_config(args.model))
    unit = 64 * world
    numel = (total + unit - 1) // unit * unit
    with open(os.path.join(os.path.dirname(os.path.dirname(__file__)), "perf", "links.json")) as f:
        link_gbs = float(json.load(f)["links"]["nvlink5"]["p2p_gbs"])
    from llmt.bench.kernels import peaks
    hbm_gbs = peaks()[1]
    out = {"model": args.model, "params": numel, "world": world, "link_gbs_per_direction": link_gbs,
           "hbm_gbs": hbm_gbs, "modes": {}}
    for mode in args.modes.split(","):
        flat = _Flat(numel, f"cuda:{local}")
        dp = DataParallel(world, rank, mode=mode)
        opt = dp.make_optimizer(flat)
        for _ in range(3):
            dp.reduce_and_step(opt)
        torch.cuda.synchronize()
        dist.barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(args.iters):
            dp.reduce_and_step(opt)
        b.record()
        torch.cuda.synchronize()
        dist.barrier()
        ms = torch.tensor([a.elapsed_time(b) / args.iters], device="cuda")
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        gbytes = 2 if mode == "nvls" else 4
        if mode == "nvls":
            link = (1 + 1 / world) * numel * 2
            serial_hbm = 6 * numel                                  # the cast, before the kernel
            hbm = 2 * numel + 24 * numel / world + 2 * numel        # inside the kernel
        else:
            link = (world - 1) / world * numel * 4
            serial_hbm = 0
            hbm = 4 * numel + 24 * numel / world + 2 * numel
        link_ms = link / (link_gbs * 1e9) * 1e3
        hbm_ms = hbm / (hbm_gbs * 1e9) * 1e3
        serial_ms = serial_hbm / (hbm_gbs * 1e9) * 1e3
        roof_ms = serial_ms + max(link_ms, hbm_ms)
        err = dp.fused.error_code() if dp.fused is not None and hasattr(dp.fused, "error_code") else 0
        out["modes"][mode] = {"ms_per_step": round(ms.item(), 4), "roofline_ms": round(roof_ms, 4),
                              "nvlink_ms": round(link_ms, 4), "hbm_ms": round(hbm_ms, 4),
                              "serial_hbm_ms": round(serial_ms, 4),
                              "fraction_of_roofline": round(roof_ms / ms.item(), 3),
                              "gradient_bytes_per_param": gbytes, "dp_error_code": err}
        dp.close()
        del dp, opt, flat
        torch.cuda.empty_cache()
    if rank == 0:
        print(json.dumps(out), flush=True)
        if args.json:
            with open(args.json, "w") as f:
                json.dump(out, f, indent=1)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
