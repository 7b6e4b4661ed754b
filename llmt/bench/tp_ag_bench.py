"""The tensor-parallel all-gather -> GEMM on one GPU, with stand-ins for the other ranks: the
GEMM with the gather fused into it, against the separate peer-store gather kernel followed by
the GEMM, and against the GEMM alone on an already gathered A (its lower bound).

Every "rank" buffer is local memory here, so the gather's stores run at HBM speed, not over
NVLink: this measures what the fusion costs or saves inside the kernel (the copy on the epilogue
warps, the per-block waits, the own-blocks-first tile order), and it is the case that ncu can
capture (ncu profiles one GPU). The other ranks' blocks are marked as arrived before the timed
calls. The multi-GPU effect is measured by llmt.bench.parallel_bench --tp-comm p2p
--tp-gather fused|separate. L2 is flushed before every timed call.

    python -m llmt.bench.tp_ag_bench --json out.json
    python -m llmt.bench.tp_ag_bench --only "8b tp2 qkv" --modes fused --reps 1 --warmup 1   # under ncu
"""
from __future__ import annotations

import argparse
import json

import torch

PIECES = 8  # 16-row pieces per 128-row block (kAgPieces)

# name, tp, rows per rank, K, N, epilogue  (the consuming GEMMs of a tensor-parallel block)
SHAPES = [
    ("8b tp2 qkv", 2, 2048, 4096, 3072, "rope"),
    ("8b tp2 w13", 2, 2048, 4096, 7168, "swiglu"),
    ("8b tp8 qkv", 8, 512, 4096, 768, "rope"),
    ("medium tp2 qkv", 2, 2048, 1024, 1536, "rope"),
    ("medium tp2 w13", 2, 2048, 1024, 1408, "swiglu"),
]


class Case:
    def __init__(self, tp, rows, K, N, epi, hd=128):
        from llmt.models.llama import rope_tables
        g = torch.Generator(device="cuda").manual_seed(0)
        self.tp, self.rows, self.K, self.N, self.epi = tp, rows, K, N, epi
        M = tp * rows
        self.x_l = torch.randn(rows, K, device="cuda", generator=g).bfloat16()
        self.bufs = [torch.randn(M, K, device="cuda", generator=g).bfloat16() for _ in range(tp)]
        self.flags = [torch.zeros(M // 128, device="cuda", dtype=torch.int32) for _ in range(tp)]
        self.flags[0].fill_(0x7FFFFFFF)  # rank 0's view: every other rank's pieces have arrived
        self.flags[0][: rows // 128] = 0  # ... its own blocks are counted by the kernel
        self.dst = torch.tensor([b.data_ptr() for b in self.bufs], dtype=torch.int64, device="cuda")
        self.fl = torch.tensor([f.data_ptr() for f in self.flags], dtype=torch.int64, device="cuda")
        rows_w = 2 * N if epi == "swiglu" else N
        self.w = (torch.randn(rows_w, K, device="cuda", generator=g) * 0.02).bfloat16()
        self.hd = hd
        self.T = 4096
        self.cos, self.sin = rope_tables(self.T, hd, 10000.0, "cuda")
        self.out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
        self.gu = torch.empty(M, 2 * N, device="cuda", dtype=torch.bfloat16) if epi == "swiglu" else None
        self.calls = 0

    def _gemm(self, **kw):
        from llmt.ops import native as Nn
        C = Nn.ext()
        a = self.bufs[0]
        if self.epi == "swiglu":
            C.gemm(a, self.w, False, True, Nn.EPI_SWIGLU, self.out, aux=self.gu, split=self.N, **kw)
        else:
            C.gemm(a, self.w, False, True, Nn.EPI_ROPE, self.out, cos_t=self.cos, sin_t=self.sin, T=self.T,
                   hd=self.hd, rot_cols=self.N * 2 // 3, **kw)

    def plain(self):
        self._gemm()

    def separate(self):
        from llmt.ops import native as Nn
        Nn.ext().tp_allgather_rows(self.x_l, self.dst, self.tp, 0)
        self._gemm()

    def fused(self):
        self.calls += 1
        self._gemm(ag_src=self.x_l, ag_dst=self.dst, ag_flags=self.fl, ag_expect=self.calls * PIECES, ag_tp=self.tp,
                   tp_rank=0, rows_per_rank=self.rows)


def main():
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--only", default=None, help="one shape name")
    p.add_argument("--modes", default="plain,separate,fused")
    p.add_argument("--reps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--json", default=None)
    args = p.parse_args()
    from llmt.bench.kernels import peaks, time_ms
    from llmt.ops import native as Nn
    Nn.ext()
    peak, _ = peaks()
    rows_out = []
    for name, tp, rows, K, N, epi in SHAPES:
        if args.only and name != args.only:
            continue
        c = Case(tp, rows, K, N, epi)
        flops = 2.0 * tp * rows * K * (2 * N if epi == "swiglu" else N)
        r = {"shape": name, "tp": tp, "M": tp * rows, "N": N, "K": K, "epilogue": epi}
        for mode in args.modes.split(","):
            ms = time_ms(getattr(c, mode), reps=args.reps, warmup=args.warmup)
            r[f"{mode}_us"] = round(ms * 1e3, 1)
            r[f"{mode}_tflops"] = round(flops / (ms / 1e3) / 1e12, 1)
        if "fused_us" in r and "separate_us" in r:
            r["fused_vs_separate"] = round(r["separate_us"] / r["fused_us"], 3)
        r["gemm_error_code"] = Nn.gemm_error_code()
        rows_out.append(r)
        print(json.dumps(r), flush=True)
    if args.json:
        with open(args.json, "w") as f:
            json.dump({"device": torch.cuda.get_device_name(), "measured_bf16_tflops": peak, "rows": rows_out}, f,
                      indent=1)


if __name__ == "__main__":
    main()
