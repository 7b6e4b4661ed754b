"""Kernel microbenchmarks at the model's shapes (the reference's kernels/bench_kernels.py).

Each op is timed with CUDA events, median of repeats, with a 256 MB buffer written between
repeats to flush the 126 MB L2 (reference bench_kernels.py:155-157 flushes the same way).
GEMMs and attention report TFLOP/s and the fraction of the measured bf16 peak; memory-bound
ops report GB/s of algorithmic traffic and the fraction of the measured HBM copy bandwidth
(MEASURED_PEAKS.json). The PyTorch/cuBLAS/SDPA equivalent of each op runs alongside.

    python -m llmt.bench.kernels --size medium --batch 4 --seq 1024 [--ops gemm,fused,attn,mem,lowp]
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics

import torch
import torch.nn.functional as F

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["bf16_tflops"]), float(p["hbm_gbs"])
    except Exception:  # noqa: BLE001
        return 1590.0, 6650.0


_flush = None


def flush_l2():
    global _flush
    if _flush is None:
        _flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device="cuda")
    _flush.fill_(1.0)


def time_ms(fn, reps=10, warmup=3):
    for _ in range(warmup):
        fn()
    ts = []
    for _ in range(reps):
        flush_l2()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        ts.append(a.elapsed_time(b))
    return statistics.median(ts)


def gemm_shapes(cfg, tokens):
    d, f, qo, V = cfg.d, cfg.ffn, cfg.qkv_out, cfg.vocab
    hd_out = cfg.H * cfg.hd
    return [
        # name, M, N, K, ta, tb  (out = op(a) @ op(b))
        ("qkv fwd", tokens, qo, d, False, True), ("qkv dgrad", tokens, d, qo, False, False),
        ("qkv wgrad", qo, d, tokens, True, False),
        ("wo fwd", tokens, d, hd_out, False, True), ("wo dgrad", tokens, hd_out, d, False, False),
        ("wo wgrad", d, hd_out, tokens, True, False),
        ("w13 fwd", tokens, 2 * f, d, False, True), ("w13 dgrad", tokens, d, 2 * f, False, False),
        ("w13 wgrad", 2 * f, d, tokens, True, False),
        ("w2 fwd", tokens, d, f, False, True), ("w2 dgrad", tokens, f, d, False, False),
        ("w2 wgrad", d, f, tokens, True, False),
        ("head fwd", tokens, V, d, False, True), ("head dgrad", tokens, d, V, False, False),
        ("head wgrad", V, d, tokens, True, False),
    ]


def bench_gemm(cfg, tokens, rows, only=None, reps=10):
    from llmt.ops import native as N
    peak, _ = peaks()
    for name, M, Nn, K, ta, tb in gemm_shapes(cfg, tokens):
        if only and name not in only:
            continue
        a = torch.randn((K, M) if ta else (M, K), device="cuda").bfloat16()
        b = torch.randn((Nn, K) if tb else (K, Nn), device="cuda").bfloat16()
        wgrad = ta
        out = torch.empty(M, Nn, device="cuda", dtype=torch.float32 if wgrad else torch.bfloat16)
        # a weight gradient is stored on the step's first write; when the planner splits K for it,
        # the training step zeroes the region and reduce-adds the splits (timed the same way here)
        split = wgrad and N.gemm_plan(M, Nn, K, N.EPI_F32, True)[1] > 1
        if split:
            ours = time_ms(lambda: (out.zero_(), N.gemm(a, b, ta=ta, tb=tb, out=out, accumulate=True)), reps=reps)
        else:
            ours = time_ms(lambda: N.gemm(a, b, ta=ta, tb=tb, out=out), reps=reps)
        aa = a.t() if ta else a
        bb = b.t() if tb else b
        ref = time_ms(lambda: torch.matmul(aa, bb))  # cuBLAS, bf16 out
        fl = 2.0 * M * Nn * K
        rows.append(dict(op=f"gemm {name}", shape=f"{M}x{Nn}x{K}", ms=round(ours, 4), ref_ms=round(ref, 4),
                         tflops=round(fl / ours / 1e9, 1), ref_tflops=round(fl / ref / 1e9, 1),
                         frac_peak=round(fl / ours / 1e9 / peak, 3)))


def bench_fused_gemm(cfg, B, T, rows):
    """The fused-epilogue GEMMs of the native path at the model's shapes (vs the plain GEMM)."""
    from llmt.models.llama import rope_tables
    from llmt.ops import native as N
    peak, _ = peaks()
    tok, d, f = B * T, cfg.d, cfg.ffn
    x = torch.randn(tok, d, device="cuda").bfloat16()
    wqkv = torch.randn(cfg.qkv_out, d, device="cuda").bfloat16()
    cos, sin = rope_tables(T, cfg.hd, cfg.rope_base, "cuda")
    ms = time_ms(lambda: N.gemm_rope(x, wqkv, cos, sin, T, cfg.hd, (cfg.H + cfg.kvh) * cfg.hd))
    fl = 2.0 * tok * cfg.qkv_out * d
    rows.append(dict(op="gemm qkv+rope", shape=f"{tok}x{cfg.qkv_out}x{d}", ms=round(ms, 4), ref_ms=None,
                     tflops=round(fl / ms / 1e9, 1), ref_tflops=0.0, frac_peak=round(fl / ms / 1e9 / peak, 3)))
    w13 = torch.randn(2 * f, d, device="cuda").bfloat16()
    ms = time_ms(lambda: N.gemm_swiglu(x, w13, f))
    fl = 2.0 * tok * 2 * f * d
    rows.append(dict(op="gemm w13+swiglu", shape=f"{tok}x{2 * f}x{d}", ms=round(ms, 4), ref_ms=None,
                     tflops=round(fl / ms / 1e9, 1), ref_tflops=0.0, frac_peak=round(fl / ms / 1e9 / peak, 3)))
    dm = torch.randn(tok, d, device="cuda").bfloat16()
    w2 = torch.randn(d, f, device="cuda").bfloat16()
    gu = torch.randn(tok, 2 * f, device="cuda").bfloat16()
    ms = time_ms(lambda: N.gemm_swiglu_bwd(dm, w2, gu, f))
    fl = 2.0 * tok * f * d
    rows.append(dict(op="gemm w2dgrad+swiglu_bwd", shape=f"{tok}x{f}x{d}", ms=round(ms, 4), ref_ms=None,
                     tflops=round(fl / ms / 1e9, 1), ref_tflops=0.0, frac_peak=round(fl / ms / 1e9 / peak, 3)))
    # the same two steps as a plain GEMM followed by the standalone elementwise kernel
    gu2 = torch.empty(tok, 2 * f, device="cuda", dtype=torch.bfloat16)
    h2 = torch.empty(tok, f, device="cuda", dtype=torch.bfloat16)
    ms = time_ms(lambda: N.swiglu_fwd(*N.gemm(x, w13, ta=False, tb=True, out=gu2).split(f, 1), h=h2))
    fl = 2.0 * tok * 2 * f * d
    rows.append(dict(op="gemm w13, then swiglu", shape=f"{tok}x{2 * f}x{d}", ms=round(ms, 4), ref_ms=None,
                     tflops=round(fl / ms / 1e9, 1), ref_tflops=0.0, frac_peak=round(fl / ms / 1e9 / peak, 3)))

    def unfused_bwd():
        dh = N.gemm(dm, w2, ta=False, tb=False, out=h2)
        g_, u_ = gu.split(f, 1)
        N.swiglu_bwd(dh, g_, u_, dg=g_, du=u_)
    ms = time_ms(unfused_bwd)
    fl = 2.0 * tok * f * d
    rows.append(dict(op="gemm w2dgrad, then swiglu_bwd", shape=f"{tok}x{f}x{d}", ms=round(ms, 4), ref_ms=None,
                     tflops=round(fl / ms / 1e9, 1), ref_tflops=0.0, frac_peak=round(fl / ms / 1e9 / peak, 3)))


def bench_attn(cfg, B, T, rows):
    from llmt.models.llama import rope_tables
    from llmt.ops import native as N
    peak, _ = peaks()
    H, KV, hd = cfg.H, cfg.kvh, cfg.hd
    qkv = torch.randn(B * T, (H + 2 * KV) * hd, device="cuda").bfloat16()
    cos, sin = rope_tables(T, hd, cfg.rope_base, "cuda")
    o, lse = N.flash_attn_fwd(qkv, B, T, H, KV, hd)
    do = torch.randn_like(o)
    fwd = time_ms(lambda: N.flash_attn_fwd(qkv, B, T, H, KV, hd))
    bwd = time_ms(lambda: N.flash_attn_bwd(do, qkv, o, lse, cos, sin, B, T, H, KV, hd))
    q = qkv.view(B, T, -1, hd)[:, :, :H].transpose(1, 2).contiguous().requires_grad_(True)
    k = qkv.view(B, T, -1, hd)[:, :, H:H + KV].transpose(1, 2).repeat_interleave(H // KV, 1).contiguous().requires_grad_(True)
    v = qkv.view(B, T, -1, hd)[:, :, H + KV:].transpose(1, 2).repeat_interleave(H // KV, 1).contiguous().requires_grad_(True)
    y = F.scaled_dot_product_attention(q, k, v, is_causal=True)
    dy = torch.randn_like(y)
    rf = time_ms(lambda: F.scaled_dot_product_attention(q, k, v, is_causal=True))
    rb = time_ms(lambda: torch.autograd.grad(y, (q, k, v), dy, retain_graph=True))
    fl = 4.0 * B * H * T * T * hd / 2  # causal
    rows.append(dict(op="attn fwd", shape=f"B{B} H{H}/{KV} T{T} hd{hd}", ms=round(fwd, 4), ref_ms=round(rf, 4),
                     tflops=round(fl / fwd / 1e9, 1), ref_tflops=round(fl / rf / 1e9, 1),
                     frac_peak=round(fl / fwd / 1e9 / peak, 3)))
    rows.append(dict(op="attn bwd", shape=f"B{B} H{H}/{KV} T{T} hd{hd}", ms=round(bwd, 4), ref_ms=round(rb, 4),
                     tflops=round(2.5 * fl / bwd / 1e9, 1), ref_tflops=round(2.5 * fl / rb / 1e9, 1),
                     frac_peak=round(2.5 * fl / bwd / 1e9 / peak, 3)))


def _bw_row(rows, op, shape, ms, ref_ms, nbytes):
    _, hbm = peaks()
    rows.append(dict(op=op, shape=shape, ms=round(ms, 4), ref_ms=round(ref_ms, 4) if ref_ms else None,
                     gbs=round(nbytes / ms / 1e6, 1), frac_hbm=round(nbytes / ms / 1e6 / hbm, 3)))


def bench_memory_ops(cfg, tokens, rows):
    from llmt.ops import native as N
    d = cfg.d
    r = torch.randn(tokens, d, device="cuda")
    a = torch.randn(tokens, d, device="cuda").bfloat16()
    w = torch.ones(d, device="cuda")
    ms = time_ms(lambda: N.add_rmsnorm_fwd(a, r, w, 1e-5))

    def ref_fwd():
        s = r + a.float()
        return (s * torch.rsqrt(s.pow(2).mean(-1, keepdim=True) + 1e-5) * w).bfloat16(), s
    _bw_row(rows, "add_rmsnorm fwd", f"{tokens}x{d}", ms, time_ms(ref_fwd), tokens * d * (2 + 4 + 4 + 2))
    y, s, rstd = N.add_rmsnorm_fwd(a, r, w, 1e-5)
    dy = torch.randn(tokens, d, device="cuda").bfloat16()
    dw = torch.zeros(d, device="cuda")
    ms = time_ms(lambda: N.rmsnorm_bwd(dy, s, w, rstd, r, dw, False))
    _bw_row(rows, "add_rmsnorm bwd", f"{tokens}x{d}", ms, None, tokens * d * (2 + 4 + 4 + 4 + 2))
    n = sum(p.numel() for p in [torch.empty(0)]) or 100_000_000
    p, g, m, v = (torch.randn(n, device="cuda") for _ in range(4))
    p16 = torch.empty(n, device="cuda", dtype=torch.bfloat16)
    lr = torch.full((1,), 3e-4, device="cuda")
    st = torch.ones(1, device="cuda", dtype=torch.int32)
    ms = time_ms(lambda: N.adamw_step(p, g, m, v, p16, lr, st, 0.9, 0.95, 1e-8, 0.1))
    pp = torch.nn.Parameter(p.clone())
    pp.grad = g.clone()
    opt = torch.optim.AdamW([pp], lr=3e-4, fused=True)
    _bw_row(rows, "adamw (+bf16 copy)", f"{n}", ms, time_ms(opt.step), n * (16 + 12 + 2))


def bench_lowp(cfg, tokens, rows, reps=10):
    """The low-precision block-linear GEMMs (all K-major: fwd, dgrad on W^T, wgrad on the
    transposed activations) per format, and the quantizers (row-wise + transposed copies).
    fp8 is compared with cuBLAS (torch._scaled_mm, tensorwise scales); the fraction is of twice
    the measured bf16 peak (the tensor core's 8-bit rate)."""
    from llmt.ops import native as N
    peak, hbm = peaks()
    d, f, qo = cfg.d, cfg.ffn, cfg.qkv_out
    shapes = [("qkv fwd", tokens, qo, d), ("qkv dgrad", tokens, d, qo), ("qkv wgrad", qo, d, tokens),
              ("w13 fwd", tokens, 2 * f, d), ("w13 dgrad", tokens, d, 2 * f), ("w2 fwd", tokens, d, f),
              ("w2 wgrad", d, f, tokens)]
    for fmt in ("fp8", "mxfp8", "nvfp4"):
        for name, M, Nn, K in shapes:
            a = torch.randn(M, K, device="cuda").bfloat16()
            b = (torch.randn(Nn, K, device="cuda") * 0.05).bfloat16()
            out = torch.empty(M, Nn, device="cuda", dtype=torch.float32 if "wgrad" in name else torch.bfloat16)
            ref = None
            if fmt == "fp8":
                aq, _, sa = N.fp8_quant(a, transpose=False)
                bq, _, sb = N.fp8_quant(b, transpose=False)
                ours = time_ms(lambda: N.gemm_fp8(aq, bq, sa, sb, out=out), reps=reps)
                try:
                    ref = time_ms(lambda: torch._scaled_mm(aq, bq.t(), scale_a=sa.reshape(()), scale_b=sb.reshape(()),
                                                           out_dtype=torch.bfloat16), reps=reps)
                except Exception:  # noqa: BLE001 - cuBLAS fp8 may be unavailable for a shape
                    ref = None
            else:
                kind = N.MXFP8 if fmt == "mxfp8" else N.NVFP4
                ar, _ = N.mx_quant(a, kind)
                br, _ = N.mx_quant(b, kind)
                ours = time_ms(lambda: N.gemm_mx(kind, ar, br, out=out), reps=reps)
            fl = 2.0 * M * Nn * K
            rows.append(dict(op=f"{fmt} {name}", shape=f"{M}x{Nn}x{K}", ms=round(ours, 4),
                             ref_ms=round(ref, 4) if ref else None, tflops=round(fl / ours / 1e9, 1),
                             ref_tflops=round(fl / ref / 1e9, 1) if ref else 0.0,
                             frac_peak=round(fl / ours / 1e9 / (2 * peak), 3)))
    for fmt in ("fp8", "mxfp8", "nvfp4"):
        for name, R, C in (("x", tokens, d), ("h", tokens, f), ("dgu", tokens, 2 * f)):
            x = torch.randn(R, C, device="cuda").bfloat16()
            if fmt == "fp8":
                fn = lambda: N.fp8_quant(x)  # noqa: E731
            else:
                kind = N.MXFP8 if fmt == "mxfp8" else N.NVFP4
                fn = lambda: N.mx_quant(x, kind, row=True, col=True, stochastic=kind == N.NVFP4)  # noqa: E731
            ms = time_ms(fn, reps=reps)
            per = 0.5 if fmt == "nvfp4" else 1.0
            nbytes = R * C * 2 + 2 * R * C * per  # read bf16, write two 8-bit (4-bit) copies
            _bw_row(rows, f"quant {fmt} {name}", f"{R}x{C}", ms, None, nbytes)


def sweep_gemm(cfg, tokens, names):
    """Tile width x split-K sweep for the named GEMM shapes (wgrad shapes accumulate in fp32)."""
    from llmt.ops import native as N
    for name, M, Nn, K, ta, tb in gemm_shapes(cfg, tokens):
        if name not in names:
            continue
        a = torch.randn((K, M) if ta else (M, K), device="cuda").bfloat16()
        b = torch.randn((Nn, K) if tb else (K, Nn), device="cuda").bfloat16()
        out = torch.zeros(M, Nn, device="cuda", dtype=torch.float32 if ta else torch.bfloat16)
        fl = 2.0 * M * Nn * K
        res = []
        for bn in (128, 256):
            for sp in ((1, 2, 3, 4, 6, 8) if ta else (1,)):
                ms = time_ms(lambda: N.gemm(a, b, ta=ta, tb=tb, out=out, accumulate=ta, bn=bn, splits=sp), reps=5)
                res.append(f"bn{bn}/s{sp}:{fl / ms / 1e9:.0f}")
        auto = time_ms(lambda: N.gemm(a, b, ta=ta, tb=tb, out=out, accumulate=ta), reps=5)
        print(f"{name:12s} {M}x{Nn}x{K} auto {fl / auto / 1e9:.0f} TF/s | " + " ".join(res), flush=True)


def main():
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--size", default="medium")
    p.add_argument("--batch", type=int, default=4)
    p.add_argument("--seq", type=int, default=1024)
    p.add_argument("--ops", default="gemm,fused,attn,mem")
    p.add_argument("--json", default=None)
    p.add_argument("--only", default=None, help="comma list of GEMM names, e.g. 'head fwd,wo fwd'")
    p.add_argument("--reps", type=int, default=10)
    args = p.parse_args()
    from llmt.config import get_config
    cfg = get_config(args.size)
    rows = []
    ops = args.ops.split(",")
    if "sweep" in ops:
        sweep_gemm(cfg, args.batch * args.seq, args.only.split(",") if args.only else [n for n, *_ in gemm_shapes(cfg, 1)])
    if "gemm" in ops:
        bench_gemm(cfg, args.batch * args.seq, rows, args.only.split(",") if args.only else None, args.reps)
    if "fused" in ops:
        bench_fused_gemm(cfg, args.batch, args.seq, rows)
    if "attn" in ops:
        bench_attn(cfg, args.batch, args.seq, rows)
    if "mem" in ops:
        bench_memory_ops(cfg, args.batch * args.seq, rows)
    if "lowp" in ops:
        bench_lowp(cfg, args.batch * args.seq, rows, args.reps)
    for r in rows:
        extra = (f"{r['tflops']:7.1f} TF/s (ref {r['ref_tflops']:7.1f}) {100 * r['frac_peak']:5.1f}% of peak"
                 if "tflops" in r else f"{r['gbs']:7.1f} GB/s {100 * r['frac_hbm']:5.1f}% of HBM")
        print(f"{r['op']:22s} {r['shape']:22s} {r['ms']:8.4f} ms (ref {r['ref_ms']}) {extra}")
    if args.json:
        with open(args.json, "w") as f:
            json.dump({"config": vars(args), "rows": rows}, f, indent=1)


if __name__ == "__main__":
    main()
