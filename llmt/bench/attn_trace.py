"""Event timeline of the pipelined attention backward for its first CTA (all query blocks of
key block 0 of (batch 0, head 0)): where each query-block step spends its cycles.

The kernel stamps clock64() at its waits when a trace buffer is set (attn_bwd_set_trace),
with plain stores into four regions (MMA thread, compute warps 2 and 9, TMA thread):
events: 0 start; TMA 30 = Q/dO stage free; MMA 1 = P/dS(n) ready, 2 = Q/dO(n+1) landed
(S/dP(n+1) issued next), 4 = dV/dK(n) issued, 5 = dQ TMEM free,
6 = dQ(n) issued + committed; compute 10 = S/dP ready, 12 = P/dS written, 13 = dQ ready,
14 = dQ drained, 15 = dK/dV ready.

    python -m llmt.bench.attn_trace --size medium --batch 4 --seq 1024
"""
from __future__ import annotations

import argparse
import json

import torch

NAMES = {0: "start", 30: "tma:stage free", 1: "mma:P/dS ready", 2: "mma:S/dP out, next Q landed",
         4: "mma:dV/dK issued", 5: "mma:dQ tmem free", 6: "mma:dQ issued", 10: "S/dP ready", 12: "P/dS written",
         13: "dQ ready", 14: "dQ drained", 15: "dK/dV ready", 7: "mma:tile K/V landed", 8: "mma:tile first Q landed",
         31: "tma:K/V stage free"}
REGIONS = ["mma", "w2", "w9", "tma"]


def main():
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--size", default="medium")
    p.add_argument("--batch", type=int, default=4)
    p.add_argument("--seq", type=int, default=1024)
    p.add_argument("--json", default=None)
    args = p.parse_args()
    from llmt.config import get_config
    from llmt.models.llama import rope_tables
    from llmt.ops import native as N
    cfg = get_config(args.size)
    B, T, H, KV, hd = args.batch, args.seq, cfg.H, cfg.kvh, cfg.hd
    qkv = torch.randn(B * T, (H + 2 * KV) * hd, device="cuda").bfloat16()
    cos, sin = rope_tables(T, hd, cfg.rope_base, "cuda")
    o, lse = N.flash_attn_fwd(qkv, B, T, H, KV, hd)
    do = torch.randn_like(o)
    for _ in range(3):
        N.flash_attn_bwd(do, qkv, o, lse, cos, sin, B, T, H, KV, hd)
    buf = torch.zeros(4096, dtype=torch.int64, device="cuda")
    ext = N.ext()._mod
    ext.attn_bwd_set_trace(buf)
    N.flash_attn_bwd(do, qkv, o, lse, cos, sin, B, T, H, KV, hd)
    torch.cuda.synchronize()
    ext.attn_bwd_set_trace(None)
    spans = buf[1024:1024 + 3 * 1024].view(1024, 3).tolist()
    spans = [(s0, sm, e0) for s0, sm, e0 in spans if s0 > 0]
    if spans:
        t_begin = min(s0 for s0, _, _ in spans)
        t_end = max(e0 for _, _, e0 in spans)
        durs = sorted(e0 - s0 for s0, _, e0 in spans)
        per_sm = {}
        for s0, sm, e0 in spans:
            per_sm.setdefault(sm, []).append((s0, e0))
        busy = [sum(e - b for b, e in v) for v in per_sm.values()]
        print(f"CTAs {len(spans)} on {len(per_sm)} SMs; kernel span {(t_end - t_begin) / 1e3:.1f} us; "
              f"CTA duration us min/median/max {durs[0] / 1e3:.1f}/{durs[len(durs) // 2] / 1e3:.1f}/{durs[-1] / 1e3:.1f}; "
              f"SM busy us min/mean/max {min(busy) / 1e3:.1f}/{sum(busy) / len(busy) / 1e3:.1f}/{max(busy) / 1e3:.1f}")
        by_kb = {}
        nx = B * KV
        for c, (s0, sm, e0) in enumerate(buf[1024:1024 + 3 * 1024].view(1024, 3).tolist()):
            if s0 > 0:
                by_kb.setdefault(c // nx, []).append((e0 - s0) / 1e3)
        print("CTA duration by key block (us, mean):",
              {k: round(sum(v) / len(v), 1) for k, v in sorted(by_kb.items())})
    ev = []
    for reg, vals in enumerate(buf[:1024].view(4, 256).tolist()):
        ev += [(int(x) >> 8, int(x) & 0xFF, REGIONS[reg]) for x in vals if x != 0]
    ev.sort()
    t0 = ev[0][0] if ev else 0
    rows = [{"cycle": t - t0, "event": f"{who}:{NAMES.get(i, str(i))}"} for t, i, who in ev]
    last = 0
    for r in rows:
        print(f"{r['cycle']:8d}  (+{r['cycle'] - last:6d})  {r['event']}")
        last = r["cycle"]
    if args.json:
        with open(args.json, "w") as f:
            json.dump(rows, f)


if __name__ == "__main__":
    main()
