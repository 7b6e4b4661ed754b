"""Roofline step-time model of one training step (reference: perf_model/roofline.py).

`inventory(cfg, B, T, path)` lists every GPU operation of one step -- forward, backward,
optimizer -- with its FLOPs, bytes moved, kernel launches and a shape key. Three paths:

  eager    the reference's PyTorch rows (bf16 autocast, SDPA or naive attention; separate
           weight casts, multi-kernel norms/RoPE/SwiGLU, full fp32 logits)
  triton   the reference's fused-kernel row (its Triton norm/SwiGLU/RoPE/CE kernels)
  native   this framework: tcgen05 GEMMs with fused epilogues (RoPE in the qkv GEMM, SwiGLU in
           the merged w1||w3 GEMM and its backward in the w2 dgrad), flash attention with the
           RoPE backward fused, CE reduced inside the lm-head GEMM, fp32 grads accumulated by
           TMA reduce-add, one fused AdamW pass that also zeroes the grads, whole step in one
           CUDA graph (no CPU issue cost)

`predict(ops, machine)` takes per op max(FLOPs / peak, bytes / bandwidth) (roofline) or the
measured time of the same GEMM / attention shape when a shape-time table is given
(calibrated), adds the per-launch GPU gap, and for eager paths compares with the CPU issue
time. Tensor parallelism (tp) shards heads, KV heads, the MLP width and the vocabulary.

    python -m llmt.perf.roofline --size medium --batch 4 --seq 1024 --path native
"""
from __future__ import annotations

import argparse
import json
import math
import os
from dataclasses import dataclass, field

from llmt.config import SIZES, ModelConfig, count_params, model_flops_per_token

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
CATEGORIES = ["matmul", "attention", "elementwise", "copy/cast", "loss", "optimizer", "communication"]


@dataclass
class Op:
    name: str
    cat: str
    phase: str              # fwd | bwd | opt
    flops: float = 0.0      # per call
    bytes: float = 0.0      # per call (all kernels of the op)
    launches: int = 1       # kernels per call
    count: int = 1          # calls per step
    key: tuple | None = None  # shape key for measured timing (GEMM / attention)

    @property
    def total_flops(self):
        return self.flops * self.count

    @property
    def total_bytes(self):
        return self.bytes * self.count


def gemm_op(name, M, N, K, phase, count, layout, a_bytes=2, out_bytes=2, epi="plain", cat="matmul"):
    """C (M, N) = op(A) (M, K) @ op(B) (K, N). layout: nt (fwd), nn (dgrad), tn (wgrad)."""
    return Op(name, cat, phase, flops=2.0 * M * N * K, bytes=(M * K + K * N) * a_bytes + M * N * out_bytes,
              launches=1, count=count, key=("gemm", M, N, K, layout, epi))


def ew_op(name, elems, bytes_per_elem, launches, phase, count, cat="elementwise"):
    return Op(name, cat, phase, bytes=float(elems) * bytes_per_elem, launches=launches, count=count)


def inventory(cfg: ModelConfig, B: int, T: int, path: str = "native", attn: str = "sdpa", tp: int = 1,
              ce_chunk: int = 8192, optimizer: str = "fused"):
    if path not in ("native", "triton", "eager"):
        raise ValueError(path)
    N = B * T
    d, L = cfg.d, cfg.L
    V = cfg.vocab // tp
    H, hd, kv = cfg.H // tp, cfg.hd, max(1, cfg.kvh // tp)
    f = cfg.ffn // tp
    dq, dkv = H * hd, kv * hd
    dqkv = dq + 2 * dkv
    n = N * d
    ops = []
    add = ops.append
    native, fused = path == "native", path != "eager"
    linears = [("qkv", dqkv, d), ("wo", d, dq), ("w1", f, d), ("w3", f, d), ("w2", d, f)]
    att_fwd_flops = 2.0 * B * H * T * T * hd    # causal: half of 4 B H T^2 hd
    if native:
        # ---- forward
        add(ew_op("embedding gather", n, 8, 1, "fwd", 1, "loss"))
        add(ew_op("add + rmsnorm (fused)", n, 12, 1, "fwd", 2 * L))
        add(gemm_op("qkv GEMM + RoPE epilogue", N, dqkv, d, "fwd", L, "nt", epi="rope"))
        add(Op("flash attention fwd (tcgen05)", "attention", "fwd", flops=att_fwd_flops,
               bytes=(N * dqkv + N * dq) * 2 + B * H * T * 4, launches=1, count=L, key=("attn_fwd", B, H, kv, T, hd)))
        add(gemm_op("wo GEMM", N, d, dq, "fwd", L, "nt"))
        add(Op("w1||w3 GEMM + SwiGLU epilogue", "matmul", "fwd", flops=2.0 * N * 2 * f * d,
               bytes=(N * d + 2 * f * d) * 2 + N * f * 2 * 3, launches=1, count=L,
               key=("gemm", N, 2 * f, d, "nt", "swiglu")))
        add(gemm_op("w2 GEMM", N, d, f, "fwd", L, "nt"))
        add(ew_op("final add + rmsnorm", n, 12, 1, "fwd", 1))
        nblk = math.ceil(V / 256)
        add(Op("lm head GEMM + CE epilogue (no logits)", "loss", "fwd", flops=2.0 * N * V * d,
               bytes=(N * d + V * d) * 2 + N * nblk * 8, launches=2, count=1, key=("gemm", N, V, d, "nt", "ce_fwd")))
        # ---- backward
        chunks = max(1, math.ceil(N / ce_chunk))
        Nc = math.ceil(N / chunks)
        add(Op("lm head recompute + dlogits epilogue", "loss", "bwd", flops=2.0 * Nc * V * d,
               bytes=(Nc * d + V * d) * 2 + Nc * V * 2, launches=1, count=chunks,
               key=("gemm", Nc, V, d, "nt", "ce_bwd")))
        add(gemm_op("lm head dgrad", Nc, d, V, "bwd", chunks, "nn"))
        add(gemm_op("lm head wgrad (fp32 reduce-add)", V, d, Nc, "bwd", chunks, "tn", out_bytes=8))
        add(ew_op("rmsnorm bwd + dw reduce", n, 26, 2, "bwd", 2 * L + 1))
        add(Op("w2 dgrad GEMM + SwiGLU bwd epilogue", "matmul", "bwd", flops=2.0 * N * f * d,
               bytes=(N * d + d * f) * 2 + N * f * 2 * 4, launches=1, count=L, key=("gemm", N, f, d, "nn", "swiglu_bwd")))
        add(gemm_op("w2 wgrad (fp32 reduce-add)", d, f, N, "bwd", L, "tn", out_bytes=8))
        add(gemm_op("w1||w3 dgrad", N, d, 2 * f, "bwd", L, "nn"))
        add(gemm_op("w1||w3 wgrad (fp32 reduce-add)", 2 * f, d, N, "bwd", L, "tn", out_bytes=8))
        add(gemm_op("wo dgrad", N, dq, d, "bwd", L, "nn"))
        add(gemm_op("wo wgrad (fp32 reduce-add)", d, dq, N, "bwd", L, "tn", out_bytes=8))
        add(Op("flash attention bwd (+RoPE bwd, pre/post)", "attention", "bwd", flops=2.5 * att_fwd_flops,
               bytes=(3 * N * dqkv + 2 * N * dq) * 2 + N * dq * 12, launches=3, count=L,
               key=("attn_bwd", B, H, kv, T, hd)))
        add(gemm_op("qkv dgrad", N, d, dqkv, "bwd", L, "nn"))
        add(gemm_op("qkv wgrad (fp32 reduce-add)", dqkv, d, N, "bwd", L, "tn", out_bytes=8))
        add(ew_op("embedding bwd (atomic scatter)", n, 8, 1, "bwd", 1, "loss"))
        P = count_params_tp(cfg, tp)
        # read p, g, m, v (16 B), write p, m, v, g=0 (16 B), write bf16 shadow (2 B)
        add(ew_op("fused AdamW (+bf16 weights, grad zeroing)", P, 34, 1, "opt", 1, "optimizer"))
        return ops
    # ---------------- reference paths (bf16 autocast) ----------------
    a = 2
    for nm, o, i in linears:
        add(ew_op(f"autocast cast {nm} weight", o * i, 6, 1, "fwd", L, "copy/cast"))
    if fused:
        add(ew_op("rmsnorm (Triton)", n, 4 + a, 1, "fwd", L))
    else:
        add(ew_op("rmsnorm (eager, 7 kernels)", n, 34, 7, "fwd", 2 * L))
    add(gemm_op("qkv projection", N, dqkv, d, "fwd", L, "nt"))
    if fused:
        add(ew_op("rope_qkv (Triton)", N * dqkv, 2 * a, 1, "fwd", L))
    else:
        add(ew_op("rope q,k (eager, 14 kernels)", N * (dq + dkv), 52, 14, "fwd", L))
    if attn == "sdpa":
        add(Op("flash attention forward (SDPA)", "attention", "fwd", flops=att_fwd_flops,
               bytes=(2 * N * dq + 2 * N * dkv) * a + B * H * T * 4, launches=1, count=L,
               key=("sdpa_fwd", B, H, kv, T, hd)))
    else:
        S = B * H * T * T
        add(gemm_op("scores q @ k^T", B * H * T, T, hd, "fwd", L, "nt", cat="attention"))
        add(ew_op("scale, mask, softmax (fp32 casts)", S, 28, 5, "fwd", L, "attention"))
        add(gemm_op("probs @ v", B * H * T, hd, T, "fwd", L, "nn", cat="attention"))
    add(ew_op("attention output transpose copy", N * dq, 2 * a, 1, "fwd", L, "copy/cast"))
    add(gemm_op("output projection", N, d, dq, "fwd", L, "nt"))
    if fused:
        add(ew_op("add_rmsnorm (Triton)", n, 8 + 2 * a, 1, "fwd", L))
    else:
        add(ew_op("residual add", n, 10, 1, "fwd", 2 * L))
    add(gemm_op("w1", N, f, d, "fwd", L, "nt"))
    add(gemm_op("w3", N, f, d, "fwd", L, "nt"))
    add(ew_op("swiglu" + (" (Triton)" if fused else " (eager, 2 kernels)"), N * f, 3 * a if fused else 5 * a,
              1 if fused else 2, "fwd", L))
    add(gemm_op("w2", N, d, f, "fwd", L, "nt"))
    for nm, o, i in linears:
        add(gemm_op(f"{nm} dgrad", N, i, o, "bwd", L, "nn"))
        add(gemm_op(f"{nm} wgrad", o, i, N, "bwd", L, "tn"))
        add(ew_op(f"{nm} grad cast to fp32", o * i, 6, 1, "bwd", L, "copy/cast"))
    add(ew_op("residual grad accumulate + casts", n, 18, 2, "bwd", 2 * L))
    if fused:
        add(ew_op("rmsnorm/add_rmsnorm bwd (Triton + dw sum)", n, 12 + 2 * a, 2, "bwd", 2 * L))
        add(ew_op("swiglu bwd (Triton)", N * f, 5 * a, 1, "bwd", L))
        add(ew_op("rope bwd (Triton)", N * dqkv, 2 * a, 1, "bwd", L))
    else:
        add(ew_op("rmsnorm bwd (eager, 12 kernels)", n, 90, 12, "bwd", 2 * L))
        add(ew_op("swiglu bwd (eager, 3 kernels)", N * f, 9 * a, 3, "bwd", L))
        add(ew_op("rope bwd + dqkv pack (eager)", N * dqkv, 60, 11, "bwd", L))
    add(ew_op("attention output transpose copy bwd", N * dq, 2 * a, 1, "bwd", L, "copy/cast"))
    if attn == "sdpa":
        add(Op("flash attention backward (SDPA)", "attention", "bwd", flops=2.5 * att_fwd_flops,
               bytes=(4 * N * dq + 4 * N * dkv) * a + N * dq * 10, launches=3, count=L,
               key=("sdpa_bwd", B, H, kv, T, hd)))
    else:
        S = B * H * T * T
        for nm in ("dprobs", "dv", "dq", "dk"):
            add(gemm_op(f"attention {nm}", B * H * T, hd if nm != "dprobs" else T, T if nm != "dprobs" else hd,
                        "bwd", L, "nn", cat="attention"))
        add(ew_op("softmax/mask bwd", S, 32, 5, "bwd", L, "attention"))
    add(ew_op("embedding gather", n, 8, 1, "fwd", 1, "loss"))
    add(ew_op("head weight cast", V * d, 6, 1, "fwd", 1, "copy/cast"))
    if fused:
        chunks = math.ceil(N / 2048)
        Nc = N // chunks
        add(gemm_op("lm head logits (chunk)", Nc, V, d, "fwd", chunks, "nt", cat="loss"))
        add(ew_op("CE + dlogits in place (Triton)", Nc * V, 2 * a, 1, "fwd", chunks, "loss"))
        add(gemm_op("lm head dgrad (chunk)", Nc, d, V, "fwd", chunks, "nn", cat="loss"))
        add(gemm_op("lm head wgrad fp32 (chunk)", V, d, Nc, "fwd", chunks, "tn", out_bytes=8, cat="loss"))
        add(ew_op("grad scale + cast", n + V * d, 6, 2, "bwd", 1, "loss"))
    else:
        add(gemm_op("lm head logits", N, V, d, "fwd", 1, "nt", cat="loss"))
        add(ew_op("logits cast + log_softmax + nll (+bwd)", N * V, 36, 7, "fwd", 1, "loss"))
        add(gemm_op("lm head dgrad", N, d, V, "bwd", 1, "nn", cat="loss"))
        add(gemm_op("lm head wgrad", V, d, N, "bwd", 1, "tn", cat="loss"))
    add(ew_op("embedding bwd (zero, sort, index_add)", cfg.vocab * d // tp + n, 10, 7, "bwd", 1, "loss"))
    P = count_params_tp(cfg, tp)
    tensors = 7 * L + 3
    if optimizer == "fused":
        add(ew_op("fused AdamW", P, 28, max(1, tensors // 8), "opt", 1, "optimizer"))
    else:
        add(ew_op("foreach AdamW (8 passes)", P, 84, int(0.85 * tensors), "opt", 1, "optimizer"))
    return ops


def count_params_tp(cfg: ModelConfig, tp: int = 1) -> float:
    total, _ = count_params(cfg)
    if tp == 1:
        return float(total)
    emb = 2 * cfg.vocab * cfg.d
    return float((total - emb) / tp + emb / tp)


@dataclass
class Machine:
    """Measured peaks of one GPU (MEASURED_PEAKS.json / calibration JSON)."""
    bf16_tflops: float
    hbm_gbs: float
    gpu_gap_us: float = 1.0      # GPU time between back-to-back kernels (graph replay)
    launch_us: float = 6.0       # CPU issue cost per kernel from eager PyTorch
    label: str = "b200"

    @classmethod
    def from_peaks(cls, path=None, sustained=True, **kw):
        path = path or os.path.join(ROOT, "MEASURED_PEAKS.json")
        try:
            with open(path) as f:
                p = json.load(f)
            tf = p.get("bf16_tflops_sustained" if sustained else "bf16_tflops") or p["bf16_tflops"]
            return cls(float(tf), float(p["hbm_gbs"]), **kw)
        except (OSError, KeyError, ValueError):
            return cls(1400.0 if sustained else 1590.0, 6650.0, **kw)

    def scaled(self, bw=1.0, peak=1.0, launch=1.0):
        return Machine(self.bf16_tflops * peak, self.hbm_gbs * bw, self.gpu_gap_us * launch, self.launch_us * launch,
                       self.label)


@dataclass
class Prediction:
    total_ms: float
    by_cat: dict = field(default_factory=dict)
    gpu_ms: float = 0.0
    gap_ms: float = 0.0
    cpu_ms: float = 0.0
    launches: int = 0
    flops: float = 0.0
    bytes: float = 0.0
    ops: list = field(default_factory=list)


def gemm_efficiency(shape_times: dict, peak_flops: float, min_gflop: float = 20.0) -> float:
    """Achieved / peak of the timed GEMM shapes of at least min_gflop, FLOP-weighted (total FLOPs
    over total time): the derating applied to GEMM shapes that were not timed (shapes too large
    for one GPU, or a model whose shapes were never measured)."""
    flops = secs = 0.0
    for k, t in shape_times.items():
        f = k.split("|")
        if f[0] != "gemm" or t <= 0:
            continue
        fl = 2.0 * int(f[1]) * int(f[2]) * int(f[3])
        if fl >= min_gflop * 1e9:
            flops += fl
            secs += t
    return min(1.0, flops / secs / peak_flops) if secs > 0 else 1.0


def predict(ops, machine: Machine, shape_times: dict | None = None, graph: bool = True) -> Prediction:
    """Step time: sum over ops of max(compute, memory) (or the measured shape time), plus the
    GPU gap per launch; with graph=False the CPU issue time can bound the step instead. With
    shape times, a GEMM whose shape was not timed runs at the timed GEMMs' efficiency."""
    peak = machine.bf16_tflops * 1e12
    bw = machine.hbm_gbs * 1e9
    p = Prediction(0.0, {c: 0.0 for c in CATEGORIES})
    eff = gemm_efficiency(shape_times, peak) if shape_times else 1.0
    for op in ops:
        tc, tm = op.flops / peak, op.bytes / bw
        if shape_times and op.key is not None and _key(op.key) in shape_times:
            t, bound = shape_times[_key(op.key)], "measured"
        elif shape_times and op.key is not None and op.key[0] == "gemm" and eff < 1.0:
            t, bound = max(tc / eff, tm), "derated"
        else:
            t, bound = max(tc, tm), ("compute" if tc >= tm else "memory")
        p.by_cat[op.cat] += t * op.count * 1e3
        p.launches += op.launches * op.count
        p.flops += op.total_flops
        p.bytes += op.total_bytes
        p.ops.append(dict(name=op.name, cat=op.cat, phase=op.phase, count=op.count, ms=round(t * op.count * 1e3, 4),
                          gflop=round(op.total_flops / 1e9, 3), mbytes=round(op.total_bytes / 1e6, 3), bound=bound))
    p.gap_ms = p.launches * machine.gpu_gap_us / 1e3
    p.gpu_ms = sum(p.by_cat.values()) + p.gap_ms
    p.cpu_ms = 0.0 if graph else p.launches * machine.launch_us / 1e3
    p.total_ms = max(p.gpu_ms, p.cpu_ms)
    return p


def _key(k) -> str:
    return "|".join(str(x) for x in k)


def load_shape_times(path) -> dict:
    if not path:
        return {}
    try:
        with open(path) as f:
            return {k: float(v) for k, v in json.load(f).items()}
    except (OSError, ValueError):
        return {}


def measure_shape_times(ops, cache_path=None, reps=10) -> dict:
    """Times every GEMM / attention shape of `ops` with this framework's kernels (GPU)."""
    import torch

    from llmt.bench.kernels import time_ms
    from llmt.models.llama import rope_tables
    from llmt.ops import native as N
    out = load_shape_times(cache_path) if cache_path else {}
    for op in ops:
        if op.key is None or _key(op.key) in out:
            continue
        k = op.key
        if k[0] == "gemm":
            _, M, Nn, K, layout, epi = k
            ta, tb = layout == "tn", layout == "nt"
            a = torch.randn((K, M) if ta else (M, K), device="cuda").bfloat16()
            if epi == "swiglu":
                w = torch.randn(2 * (Nn // 2), K, device="cuda").bfloat16()
                fn = lambda: N.gemm_swiglu(a, w, Nn // 2)  # noqa: E731
            elif epi == "swiglu_bwd":
                w = torch.randn(K, Nn, device="cuda").bfloat16()
                gu = torch.randn(M, 2 * Nn, device="cuda").bfloat16()
                fn = lambda: N.gemm_swiglu_bwd(a, w, gu, Nn)  # noqa: E731
            elif epi == "rope":
                w = torch.randn(Nn, K, device="cuda").bfloat16()
                cos, sin = rope_tables(1024, 64, 10000.0, "cuda")
                fn = lambda: N.gemm_rope(a, w, cos, sin, 1024, 64, Nn // 2)  # noqa: E731
            elif epi == "ce_fwd":
                w = torch.randn(Nn, K, device="cuda").bfloat16()
                tgt = torch.randint(0, Nn, (M,), device="cuda")
                fn = lambda: N.gemm_ce_fwd(a, w, tgt)  # noqa: E731
            elif epi == "ce_bwd":
                w = torch.randn(Nn, K, device="cuda").bfloat16()
                tgt = torch.randint(0, Nn, (M,), device="cuda")
                lse = torch.zeros(M, device="cuda")
                g = torch.ones(1, device="cuda")
                fn = lambda: N.gemm_ce_bwd(a, w, tgt, lse, g, 1.0 / M)  # noqa: E731
            else:
                b = torch.randn((Nn, K) if tb else (K, Nn), device="cuda").bfloat16()
                o = torch.zeros(M, Nn, device="cuda", dtype=torch.float32 if ta else torch.bfloat16)
                fn = lambda: N.gemm(a, b, ta=ta, tb=tb, out=o, accumulate=ta)  # noqa: E731
        elif k[0] in ("attn_fwd", "attn_bwd"):
            _, B, H, KV, T, hd = k
            qkv = torch.randn(B * T, (H + 2 * KV) * hd, device="cuda").bfloat16()
            o, lse = N.flash_attn_fwd(qkv, B, T, H, KV, hd)
            cos, sin = rope_tables(T, hd, 10000.0, "cuda")
            do = torch.randn_like(o)
            fn = ((lambda: N.flash_attn_fwd(qkv, B, T, H, KV, hd)) if k[0] == "attn_fwd"
                  else (lambda: N.flash_attn_bwd(do, qkv, o, lse, cos, sin, B, T, H, KV, hd)))
        else:
            continue
        out[_key(k)] = time_ms(fn, reps=reps) / 1e3
    if cache_path:
        with open(cache_path, "w") as f:
            json.dump(out, f, indent=1)
    return out


def summarize(p: Prediction, cfg: ModelConfig, B: int, T: int, machine: Machine) -> dict:
    tokens = B * T
    tps = tokens / (p.total_ms / 1e3)
    mfu = model_flops_per_token(cfg, T) * tps / (machine.bf16_tflops * 1e12)
    return {"step_ms": round(p.total_ms, 3), "tokens_per_s": round(tps), "mfu_vs_peak_used": round(mfu, 4),
            "by_cat_ms": {k: round(v, 3) for k, v in p.by_cat.items()}, "gap_ms": round(p.gap_ms, 3),
            "cpu_ms": round(p.cpu_ms, 3), "launches": p.launches, "tflop": round(p.flops / 1e12, 3),
            "gbytes": round(p.bytes / 1e9, 3)}


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--size", default="medium", choices=list(SIZES))
    ap.add_argument("--batch", type=int, default=4)
    ap.add_argument("--seq", type=int, default=1024)
    ap.add_argument("--path", default="native", choices=["native", "triton", "eager"])
    ap.add_argument("--attn", default="sdpa", choices=["sdpa", "naive"])
    ap.add_argument("--tp", type=int, default=1)
    ap.add_argument("--peaks", default=None, help="MEASURED_PEAKS.json-style file")
    ap.add_argument("--shape-times", default=None, help="JSON cache of measured GEMM/attention shape times")
    ap.add_argument("--measure-shapes", action="store_true", help="time the shapes on this GPU (fills the cache)")
    ap.add_argument("--what-if", action="append", default=[], help="bw=2 | peak=2 | launch=0")
    ap.add_argument("--top", type=int, default=12)
    ap.add_argument("--json", action="store_true")
    args = ap.parse_args()
    cfg = SIZES[args.size]
    m = Machine.from_peaks(args.peaks)
    for w in args.what_if:
        k, v = w.split("=")
        m = m.scaled(**{k: float(v)})
    ops = inventory(cfg, args.batch, args.seq, args.path, args.attn, args.tp)
    st = measure_shape_times(ops, args.shape_times) if args.measure_shapes else load_shape_times(args.shape_times)
    p = predict(ops, m, st, graph=args.path == "native")
    s = summarize(p, cfg, args.batch, args.seq, m)
    if args.json:
        print(json.dumps(s))
        return
    print(f"{args.size} b{args.batch} s{args.seq} path={args.path}: {s['step_ms']} ms, {s['tokens_per_s']:,} tok/s, "
          f"MFU {100 * s['mfu_vs_peak_used']:.1f}% | launches {s['launches']} gap {s['gap_ms']} ms")
    for k, v in s["by_cat_ms"].items():
        print(f"  {k:14s} {v:8.3f} ms")
    for o in sorted(p.ops, key=lambda o: -o["ms"])[:args.top]:
        print(f"  {o['ms']:8.3f} ms  {o['bound']:8s} {o['name']}")


if __name__ == "__main__":
    main()
