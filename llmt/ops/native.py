"""Thin Python wrappers over the sm_100a extension `llmt._C`.

Every wrapper launches on the current CUDA stream and allocates its outputs through the
PyTorch caching allocator, so the whole training step can be captured in one CUDA graph.
The extension is required: importing a wrapper without the built extension raises instead
of silently falling back to PyTorch.
"""
from __future__ import annotations

import os
from typing import NamedTuple, Optional

import torch

_C = None

EPI_BF16, EPI_F32, EPI_SWIGLU, EPI_SWIGLU_BWD, EPI_ROPE, EPI_CE_FWD, EPI_CE_BWD = range(7)


# Kernels launched per call of an extension entry point (1 unless listed).
_KERNELS_PER_CALL = {"flash_attn_bwd": 3, "gemm_error_code": 0, "attn_error_code": 0, "dp_error_code": 0,
                     "set_reserved_sms": 0, "reserved_sms": 0,
                     "ipc_alloc": 0, "ipc_open": 0, "ipc_close": 0, "ipc_free": 0, "tensor_from_ptr": 0,
                     "sm_count": 0, "bounds_error": 0, "bounds_checking": 0, "fp8_quant": 2, "fp8_amax_slots": 0, "mx_sf_bytes": 0, "gemm_plan": 0}


class LaunchCounter:
    """Counts this library's kernel launches issued from Python (captured graphs replay them)."""

    def __init__(self):
        self.count = 0
        self.bodies = 0

    def reset(self):
        self.count = 0
        self.bodies = 0

    def per_step(self, trainer=None) -> int:
        bodies = trainer.body_calls if trainer is not None else self.bodies
        return int(round(self.count / max(1, bodies)))


LAUNCHES = LaunchCounter()


class _Counted:
    def __init__(self, mod):
        self._mod = mod

    def __getattr__(self, name):
        fn = getattr(self._mod, name)
        if not callable(fn):
            return fn
        k = _KERNELS_PER_CALL.get(name, 1)

        def call(*a, **kw):
            LAUNCHES.count += k
            return fn(*a, **kw)
        return call


def ext():
    """The compiled extension; raises with build instructions when it is missing."""
    global _C
    if _C is None:
        try:
            if os.environ.get("LLMT_BOUNDS") == "1":  # the bounds-checked build (debug)
                from llmt import _C_bounds as c  # noqa: PLC0415
            else:
                from llmt import _C as c  # noqa: PLC0415
        except ImportError as e:  # pragma: no cover - depends on the build
            raise RuntimeError(
                "llmt native extension is not built; run `python setup.py build_ext --inplace` "
                "(or __graft_entry__.build())") from e
        _C = _Counted(c)
    return _C


def available() -> bool:
    try:
        ext()
        return True
    except RuntimeError:
        return False


_tickets: dict[int, torch.Tensor] = {}


def _ticket(device) -> torch.Tensor:
    """Per-device int32 word used by the norm backward's last-CTA-done reduction (self re-arming)."""
    idx = torch.device(device).index or 0
    t = _tickets.get(idx)
    if t is None:
        t = torch.zeros(1, dtype=torch.int32, device=device)
        _tickets[idx] = t
    return t


def _tma_ok(t: torch.Tensor) -> bool:
    return t.stride(-1) == 1 and t.data_ptr() % 16 == 0 and (t.stride(0) * t.element_size()) % 16 == 0


# ---------------------------------------------------------------- norms
def add_rmsnorm_fwd(a, r, w, eps, write_s=True):
    """y = rmsnorm(r + a) * w. a bf16 or None, r fp32, w fp32 -> (y bf16, s fp32 | None, rstd fp32)."""
    y, s, rstd = ext().add_rmsnorm_fwd(a, r, w, float(eps), bool(write_s))
    return y, (s if write_s else None), rstd


def rmsnorm_bwd(dy, s, w, rstd, ds_in, dw, accumulate, write_ds16=True):
    """Returns (ds fp32, ds bf16 | None); writes or accumulates dw (fp32) in place."""
    ds, ds16 = ext().rmsnorm_bwd(dy, s, w, rstd, ds_in, dw, _ticket(s.device), bool(write_ds16), bool(accumulate))
    return ds, (ds16 if write_ds16 else None)


# ---------------------------------------------------------------- GEMM
def _take_ag(a, ta=False):
    """Keyword arguments of an all-gather fused into this GEMM's A loads.

    A tensor returned by the peer-memory tensor-parallel all-gather (TPPeerComm with fused
    gathers) carries the gather it still owes as `_llmt_pending_ag`: its rows are stored into
    every rank's buffer by the first GEMM that reads it with a K-major A. A consumer that cannot
    fuse (an MN-major A, i.e. a weight gradient reading it first) has the gather run on its own
    before it. Either way the pending gather is consumed once."""
    pending = getattr(a, "_llmt_pending_ag", None)
    if pending is None:
        return {}
    del a._llmt_pending_ag
    if ta:
        pending.run_unfused()
        return {}
    return pending.kwargs()


def gemm(a, b, ta=False, tb=True, out=None, out_dtype=torch.bfloat16, accumulate=False, bn=0, splits=0):
    """out = op(a) @ op(b) on the tcgen05 GEMM (bf16 operands, fp32 accumulation).

    ta=False, tb=True  : forward   y  = x  @ W^T
    ta=False, tb=False : dgrad     dx = dy @ W
    ta=True,  tb=False : wgrad     dW = dy^T @ x   (fp32 out, optional accumulate)
    Operands need 16-byte aligned bases and row pitches (TMA); the caller pads otherwise.
    """
    if not (_tma_ok(a) and _tma_ok(b)):
        raise ValueError("gemm operands need 16-byte aligned bases and row pitches (TMA)")
    M = a.shape[1] if ta else a.shape[0]
    N = b.shape[0] if tb else b.shape[1]
    if out is None:
        out = torch.empty((M, N), dtype=out_dtype, device=a.device)
    epi = EPI_F32 if out.dtype == torch.float32 else EPI_BF16
    _take_ag(b, True)  # a pending gather read as B first runs on its own
    ext().gemm(a, b, ta, tb, epi, out, accumulate=accumulate, bn=bn, splits=splits, **_take_ag(a, ta))
    return out


def gemm_swiglu(x, w13, ffn, h=None, gu=None, bn=0):
    """Merged gate/up GEMM with the SwiGLU epilogue: h = silu(x W1^T) * (x W3^T); also saves [g | u]."""
    M = x.shape[0]
    if h is None:
        h = torch.empty((M, ffn), dtype=torch.bfloat16, device=x.device)
    if gu is None:
        gu = torch.empty((M, 2 * ffn), dtype=torch.bfloat16, device=x.device)
    ext().gemm(x, w13, False, True, EPI_SWIGLU, h, aux=gu, split=ffn, bn=bn, **_take_ag(x))
    return h, gu


def gemm_swiglu_bwd(dm, w2, gu, ffn, dgu=None, bn=0):
    """w2 dgrad with the SwiGLU backward epilogue: dh = dm @ W2, then [dg | du] from the saved [g | u]."""
    M = dm.shape[0]
    if dgu is None:
        dgu = torch.empty((M, 2 * ffn), dtype=torch.bfloat16, device=dm.device)
    ext().gemm(dm, w2, False, False, EPI_SWIGLU_BWD, dgu, aux=gu, out2=dgu, split=ffn, bn=bn, **_take_ag(dm))
    return dgu


def gemm_rope(x, wqkv, cos, sin, T, hd, rot_cols, out=None, bn=0):
    """qkv GEMM with RoPE applied to the first rot_cols (q and k) columns in the epilogue."""
    M, N = x.shape[0], wqkv.shape[0]
    if out is None:
        out = torch.empty((M, N), dtype=torch.bfloat16, device=x.device)
    ext().gemm(x, wqkv, False, True, EPI_ROPE, out, cos_t=cos, sin_t=sin, T=T, hd=hd, rot_cols=rot_cols, bn=bn,
               **_take_ag(x))
    return out


def gemm_ce_fwd(h, w, targets, bn=256, return_target_logit=False):
    """Logit tiles reduced in the epilogue: returns (lse fp32 (M,), loss fp32 (M,)); no logits written.
    Targets outside [0, V) contribute no target logit (their loss is 0): a vocabulary-parallel
    shard passes targets shifted by its first row and combines lse / target logits across shards.
    With return_target_logit the (M,) target logits (0 where the target is outside) come third."""
    M, V = h.shape[0], w.shape[0]
    nblk = -(-V // bn)
    part = torch.empty((M, nblk, 2), dtype=torch.float32, device=h.device)
    tl = torch.zeros((M,), dtype=torch.float32, device=h.device)
    dummy = torch.empty((M, 8), dtype=torch.bfloat16, device=h.device)
    ext().gemm(h, w, False, True, EPI_CE_FWD, dummy, tgt=targets, part=part, tlogit=tl, bn=bn)
    lse = torch.empty((M,), dtype=torch.float32, device=h.device)
    loss = torch.empty((M,), dtype=torch.float32, device=h.device)
    ext().ce_combine(part, tl, targets, lse, loss, nblk, V)
    return (lse, loss, tl) if return_target_logit else (lse, loss)


def gemm_ce_bwd(h, w, targets, lse, grad_out, scale, out=None, bn=0):
    """Recomputed logit tiles -> dlogits = (softmax - onehot) * grad_out * scale, bf16 (M, V)."""
    M, V = h.shape[0], w.shape[0]
    if out is None:
        out = torch.empty((M, V), dtype=torch.bfloat16, device=h.device)
    ext().gemm(h, w, False, True, EPI_CE_BWD, out, tgt=targets, lse=lse, grad_out=grad_out, alpha=scale, bn=bn)
    return out


def gemm_plan(M, N, K, epi, can_split):
    """(tile width, split-K factor) the GEMM planner picks for a problem (host only)."""
    return ext().gemm_plan(int(M), int(N), int(K), int(epi), bool(can_split))


def gemm_error_code(reset=False) -> int:
    """Sticky code of the first bounded-wait timeout any GEMM launch hit (0 = none)."""
    return ext().gemm_error_code(reset)


# ---------------------------------------------------------------- fp8 (tensorwise e4m3)
E4M3 = torch.float8_e4m3fn
_AMAX_SLOTS = {}


def fp8_quant(x, transpose=True):
    """Tensorwise e4m3 quantization of a bf16 / fp32 (rows, cols) tensor (reference
    kernels/lowp.py:51-62): scale = 448 / amax, q = e4m3(sat(x * scale)); returns
    (q, q^T or None, inv) with inv a 1-element fp32 device tensor holding 1 / scale (bit-identical to
    llmt.ops.lowp_ref.fp8_quant_ref), so nothing
    leaves the device (the step stays capturable in a CUDA graph)."""
    rows, cols = x.shape
    dev = x.device
    n = _AMAX_SLOTS.get(dev)
    if n is None:
        n = _AMAX_SLOTS[dev] = int(ext().fp8_amax_slots())
    q = torch.empty((rows, cols), dtype=E4M3, device=dev)
    qt = torch.empty((cols, rows), dtype=E4M3, device=dev) if transpose else None
    buf = torch.empty(4 + n, dtype=torch.float32, device=dev)
    inv = buf[:1]
    ext().fp8_quant(x, q, qt, inv, buf[4:])
    return q, qt, inv


def gemm_fp8(a, b, sa, sb, out=None, out_dtype=torch.bfloat16, accumulate=False, bn=0, splits=0):
    """out = (a @ b^T) * sa * sb with e4m3 a (M, K) and b (N, K), fp32 accumulation; bf16 out, or
    fp32 out (+= with accumulate: weight-gradient accumulation into main_grad)."""
    M, N = a.shape[0], b.shape[0]
    if out is None:
        out = torch.empty((M, N), dtype=out_dtype, device=a.device)
    epi = EPI_F32 if out.dtype == torch.float32 else EPI_BF16
    ext().gemm(a, b, False, True, epi, out, accumulate=accumulate, bn=bn, splits=splits, scale_a=sa, scale_b=sb)
    return out


def gemm_fp8_swiglu(xq, w13q, sa, sb, ffn, bn=0):
    """Merged gate/up GEMM on e4m3 operands with the SwiGLU epilogue: (h, [g | u]) in bf16."""
    M = xq.shape[0]
    h = torch.empty((M, ffn), dtype=torch.bfloat16, device=xq.device)
    gu = torch.empty((M, 2 * ffn), dtype=torch.bfloat16, device=xq.device)
    ext().gemm(xq, w13q, False, True, EPI_SWIGLU, h, aux=gu, split=ffn, bn=bn, scale_a=sa, scale_b=sb)
    return h, gu


def gemm_fp8_swiglu_bwd(dmq, w2q_t, sa, sb, gu, ffn, bn=0):
    """w2 dgrad on e4m3 operands (dm and the transposed W2, both K-major) with the SwiGLU
    backward epilogue: [dg | du] in bf16 from the saved [g | u]."""
    M = dmq.shape[0]
    dgu = torch.empty((M, 2 * ffn), dtype=torch.bfloat16, device=dmq.device)
    ext().gemm(dmq, w2q_t, False, True, EPI_SWIGLU_BWD, dgu, aux=gu, out2=dgu, split=ffn, bn=bn, scale_a=sa,
               scale_b=sb)
    return dgu


def gemm_fp8_rope(xq, wq, sa, sb, cos, sin, T, hd, rot_cols, bn=0):
    """qkv GEMM on e4m3 operands with RoPE applied to the first rot_cols columns in the epilogue."""
    M, N = xq.shape[0], wq.shape[0]
    out = torch.empty((M, N), dtype=torch.bfloat16, device=xq.device)
    ext().gemm(xq, wq, False, True, EPI_ROPE, out, cos_t=cos, sin_t=sin, T=T, hd=hd, rot_cols=rot_cols, bn=bn,
               scale_a=sa, scale_b=sb)
    return out


# ---------------------------------------------------------------- block-scaled (MXFP8 / NVFP4)
MXFP8, NVFP4 = 2, 3
SR_STEP = {}  # device -> int64 step counter mixed into the stochastic-rounding seed


class BlockQ(NamedTuple):
    """A block-scaled GEMM operand: q (rows, K) e4m3 or (rows, K / 2) packed e2m1 bytes, its
    scales in the chunked layout, and (NVFP4) the per-tensor decode scale g."""
    q: torch.Tensor
    sf: torch.Tensor
    g: Optional[torch.Tensor]


def sr_counter(device):
    """The device-side step counter of the stochastic rounding (advance it once per step)."""
    dev = torch.device(device)
    if dev not in SR_STEP:
        SR_STEP[dev] = torch.zeros(1, dtype=torch.int64, device=dev)
    return SR_STEP[dev]


_SEEDS = [0]


def mx_quant(x, kind, row=True, col=False, interleave64=False, stochastic=False):
    """Quantize x (rows, cols) for block-scaled GEMMs: `row` along cols (operand of a GEMM that
    contracts over cols), `col` x^T along rows. Returns (BlockQ | None, BlockQ | None).
    kind MXFP8 (ue8m0 per 32) or NVFP4 (ue4m3 per 16 + per-tensor scale; reference recipe
    kernels/lowp.py:110-138, stochastic rounding for gradients). interleave64 writes the row
    copy of a merged [W1; W3] as 64 rows of W1, 64 of W3, ... (the SwiGLU GEMM's B tiles)."""
    rows, cols = x.shape
    dev = x.device
    per = 2 if kind == NVFP4 else 1
    qdt = torch.uint8 if kind == NVFP4 else E4M3
    C = ext()
    q = sf = qt = sft = None
    kblk = 256 if kind == NVFP4 else 128  # values per 128-byte k-block

    def scales(r, c):
        # the kernel writes every scale of the tensor; padding (partial row tiles or k-blocks) is zeroed
        n = C.mx_sf_bytes(kind, r, c)
        alloc = torch.empty if (r % 128 == 0 and c % kblk == 0) else torch.zeros
        return alloc(n, dtype=torch.uint8, device=dev)
    if row:
        q = torch.empty((rows, cols // per), dtype=qdt, device=dev)
        sf = scales(rows, cols)
    if col:
        qt = torch.empty((cols, rows // per), dtype=qdt, device=dev)
        sft = scales(cols, rows)
    g = scratch = None
    if kind == NVFP4:
        n = _AMAX_SLOTS.get(dev)
        if n is None:
            n = _AMAX_SLOTS[dev] = int(C.fp8_amax_slots())
        buf = torch.empty(4 + n, dtype=torch.float32, device=dev)
        g, scratch = buf[:1], buf[4:]
    _SEEDS[0] += 1
    C.mx_quant(kind, x, q, sf, qt, sft, g, scratch, interleave64=interleave64, stochastic=stochastic,
               seed=(_SEEDS[0] * 0x2545F491) & 0x7FFFFFFFFFFFFFFF, seed_dev=sr_counter(dev) if stochastic else None)
    return (BlockQ(q, sf, g) if row else None), (BlockQ(qt, sft, g) if col else None)


def _mx_args(kind, a, b):
    return dict(kind=kind, sfa=a.sf, sfb=b.sf, scale_a=a.g, scale_b=b.g)


def gemm_mx(kind, a, b, out=None, out_dtype=torch.bfloat16, accumulate=False, splits=0):
    """out = a @ b^T on block-scaled operands (BlockQ, both quantized along K); bf16 out, or fp32
    (+= with accumulate)."""
    M, N = a.q.shape[0], b.q.shape[0]
    if out is None:
        out = torch.empty((M, N), dtype=out_dtype, device=a.q.device)
    epi = EPI_F32 if out.dtype == torch.float32 else EPI_BF16
    ext().gemm(a.q, b.q, False, True, epi, out, accumulate=accumulate, splits=splits, **_mx_args(kind, a, b))
    return out


def gemm_mx_swiglu(kind, x, w13, ffn):
    """Merged gate/up GEMM with the SwiGLU epilogue; w13 quantized with interleave64."""
    M = x.q.shape[0]
    h = torch.empty((M, ffn), dtype=torch.bfloat16, device=x.q.device)
    gu = torch.empty((M, 2 * ffn), dtype=torch.bfloat16, device=x.q.device)
    ext().gemm(x.q, w13.q, False, True, EPI_SWIGLU, h, aux=gu, split=ffn, **_mx_args(kind, x, w13))
    return h, gu


def gemm_mx_swiglu_bwd(kind, dm, w2t, gu, ffn):
    """w2 dgrad (dm along d, W2^T along d) with the SwiGLU backward epilogue -> [dg | du]."""
    M = dm.q.shape[0]
    dgu = torch.empty((M, 2 * ffn), dtype=torch.bfloat16, device=dm.q.device)
    ext().gemm(dm.q, w2t.q, False, True, EPI_SWIGLU_BWD, dgu, aux=gu, out2=dgu, split=ffn, **_mx_args(kind, dm, w2t))
    return dgu


def gemm_mx_rope(kind, x, w, cos, sin, T, hd, rot_cols):
    """qkv GEMM on block-scaled operands with RoPE on the first rot_cols columns."""
    M, N = x.q.shape[0], w.q.shape[0]
    out = torch.empty((M, N), dtype=torch.bfloat16, device=x.q.device)
    ext().gemm(x.q, w.q, False, True, EPI_ROPE, out, cos_t=cos, sin_t=sin, T=T, hd=hd, rot_cols=rot_cols,
               **_mx_args(kind, x, w))
    return out


# ---------------------------------------------------------------- elementwise
def swiglu_fwd(g, u, h=None):
    if h is None:
        h = torch.empty(g.shape, dtype=torch.bfloat16, device=g.device)
    ext().swiglu_fwd(g, u, h)
    return h


def swiglu_bwd(dh, g, u, dg=None, du=None):
    if dg is None:
        dg = torch.empty(g.shape, dtype=torch.bfloat16, device=g.device)
    if du is None:
        du = torch.empty(u.shape, dtype=torch.bfloat16, device=u.device)
    ext().swiglu_bwd(dh, g, u, dg, du)
    return dg, du


def rope_inplace(qkv2d, cos, sin, T, n_rot_heads, hd, backward=False):
    ext().rope_inplace(qkv2d, cos, sin, int(T), int(n_rot_heads), int(hd), bool(backward))
    return qkv2d


def embedding_fwd(idx, W, out=None, v0=0, partial=False):
    """x[n] = W[idx[n] - v0]; W holds vocabulary rows [v0, v0 + W.shape[0]). With `partial`
    (a vocabulary-parallel shard) ids outside that range give zero rows."""
    if out is None:
        out = torch.empty((idx.numel(), W.shape[1]), dtype=torch.float32, device=W.device)
    ext().embedding_fwd(idx.reshape(-1), W, out, None, int(v0), bool(partial))
    return out


def embedding_bwd(idx, dx, dW, v0=0):
    """dW[idx[n] - v0] += dx[n] for ids inside the shard."""
    ext().embedding_bwd(idx.reshape(-1), dx, dW, int(v0))


def adamw_step(p, g, m, v, p16, lr, step, b1, b2, eps, wd, grad_scale=1.0, zero_grad=False, max_blocks=0):
    ext().adamw_step(p, g, m, v, p16, lr, step, float(b1), float(b2), float(eps), float(wd), float(grad_scale),
                     bool(zero_grad), int(max_blocks))


def cast_bf16(x, y, max_blocks=0):
    ext().cast_bf16(x, y, int(max_blocks))


def ce_fwd_rows(logits, targets, lse, loss):
    ext().ce_fwd_rows(logits, targets, lse, loss)


def ce_bwd_rows(logits, targets, lse, grad_out, scale):
    ext().ce_bwd_rows(logits, targets, lse, grad_out, float(scale))


# ---------------------------------------------------------------- attention
def flash_attn_fwd(qkv, B, T, H, KV, hd, causal=True, scale=None):
    """Causal flash attention over the packed post-RoPE qkv rows -> (o (B*T, H*hd) bf16, lse (B, H, T))."""
    scale = (1.0 / hd ** 0.5) if scale is None else scale
    o, lse = ext().flash_attn_fwd(qkv, int(B), int(T), int(H), int(KV), int(hd), bool(causal), float(scale))
    return o, lse


def flash_attn_bwd(do, qkv, o, lse, cos, sin, B, T, H, KV, hd, causal=True, scale=None):
    """Gradient w.r.t. the packed *pre-RoPE* qkv rows (the RoPE backward is fused in)."""
    scale = (1.0 / hd ** 0.5) if scale is None else scale
    return ext().flash_attn_bwd(do, qkv, o, lse, cos, sin, int(B), int(T), int(H), int(KV), int(hd), bool(causal),
                                float(scale))


def attn_error_code(reset=False) -> int:
    return ext().attn_error_code(reset)
