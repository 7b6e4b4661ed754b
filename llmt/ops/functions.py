"""Autograd Functions of the native training path.

Each Function covers one fused region of the step and calls only sm_100a kernels of
llmt._C. Weight gradients never go through autograd: every backward accumulates its fp32
weight gradient straight into the parameter's `main_grad` view of the flat gradient buffer
(TMA reduce-add in the GEMM epilogue, so split-K and micro-batch accumulation are free), and
the fused optimizer zeroes the buffer after consuming it. The optimizer and the
data-parallel reduce-scatter read one contiguous buffer.

Regions (reference equivalents in bench_train.py / kernels/triton_ops.py):
  Embed          emb(idx)                                        bench_train.py:213
  RMSNormFn      rmsnorm on the fp32 residual                    triton_ops.py:113-128
  AddRMSNormFn   s = r + a; y = rmsnorm(s)                       triton_ops.py:131-151
  QKVAttention   qkv GEMM (+RoPE epilogue) -> causal flash attn  bench_train.py:130-149
  Linear         y = x W^T (wo)                                  bench_train.py:150
  SwiGLUMLP      w1||w3 GEMM (+SwiGLU epilogue) -> w2 GEMM       bench_train.py:153-163
  HeadCE         lm head + cross entropy, logits never written   triton_ops.py:367-405
"""
from __future__ import annotations

import os

import torch

from llmt.ops import native as N

# SwiGLU inside the GEMM epilogues (True) or as a separate elementwise kernel (False), per direction;
# LLMT_SWIGLU_EPILOGUE="fwd,bwd" / "fwd" / "bwd" / "none" overrides the default.
_sw = os.environ.get("LLMT_SWIGLU_EPILOGUE", "fwd,bwd")
SWIGLU_EPILOGUE = {"fwd": "fwd" in _sw, "bwd": "bwd" in _sw}
# Other fusions that can be switched off (the ablation of llmt.bench.ablate; reference
# kernels/ablate_kernels.py): "rope" = RoPE in the qkv GEMM epilogue (else the standalone
# in-place RoPE kernel after a plain GEMM), "head_ce" = cross entropy reduced inside the head
# GEMM's epilogue with logits never written (else bf16 logits + the row CE kernels).
# LLMT_UNFUSE="rope,head_ce" switches them off. head_ce defaults to "auto": the fused head
# recomputes the logit GEMM in its backward, which costs more than writing and re-reading bf16
# logits while they are small, so logits are materialised up to HEAD_LOGITS_BUDGET bytes and
# never beyond.
# First-write gradients: while GRAD["first"] is set (the first micro-batch of a step whose
# optimizer does not clear the gradient buffer) every weight-gradient writer stores instead of
# adding, so the buffer is never zeroed and the GEMMs never read the old values back from DRAM.
# A split-K GEMM (its splits add into one output) and the embedding's atomic scatter zero their
# own region first.
GRAD = {"first": False}
_unf = os.environ.get("LLMT_UNFUSE", "")
FUSION = {"rope": "rope" not in _unf, "head_ce": False if "head_ce" in _unf else "auto"}
HEAD_LOGITS_BUDGET = 2 << 30


class Embed(torch.autograd.Function):
    @staticmethod
    def forward(ctx, idx, w):
        ctx.save_for_backward(idx)
        ctx.w = w
        return N.embedding_fwd(idx, w)

    @staticmethod
    def backward(ctx, dx):
        (idx,) = ctx.saved_tensors
        first_write_zero(ctx.w.main_grad)  # the scatter adds: rows of absent ids must read zero
        N.embedding_bwd(idx, dx.contiguous(), ctx.w.main_grad)
        return None, None


class EmbedVP(torch.autograd.Function):
    """Vocabulary-parallel embedding: rows for the ids in this shard [v0, v0 + V/tp), zeros
    elsewhere (the reduce-scatter that follows sums the shards)."""

    @staticmethod
    def forward(ctx, idx, w, v0):
        ctx.save_for_backward(idx)
        ctx.w, ctx.v0 = w, v0
        return N.embedding_fwd(idx, w, v0=v0, partial=True)

    @staticmethod
    def backward(ctx, dx):
        (idx,) = ctx.saved_tensors
        N.embedding_bwd(idx, dx.contiguous(), ctx.w.main_grad, v0=ctx.v0)
        return None, None, None


class RMSNormFn(torch.autograd.Function):
    """y = rmsnorm(x) * w on the fp32 residual x (no add); y bf16."""

    @staticmethod
    def forward(ctx, x, w, eps):
        y, _, rstd = N.add_rmsnorm_fwd(None, x, w, eps, write_s=False)
        ctx.save_for_backward(x, rstd)
        ctx.w = w
        return y

    @staticmethod
    def backward(ctx, dy):
        x, rstd = ctx.saved_tensors
        w = ctx.w
        ds, _ = N.rmsnorm_bwd(dy.contiguous(), x, w, rstd, None, w.main_grad, not GRAD["first"], write_ds16=False)
        return ds, None, None


class AddRMSNormFn(torch.autograd.Function):
    """s = r + a (fp32 residual + bf16 branch output), y = rmsnorm(s) * w. Returns (y, s)."""

    @staticmethod
    def forward(ctx, a, r, w, eps):
        y, s, rstd = N.add_rmsnorm_fwd(a, r, w, eps, write_s=True)
        ctx.save_for_backward(s, rstd)
        ctx.w = w
        return y, s

    @staticmethod
    def backward(ctx, dy, ds_in):
        s, rstd = ctx.saved_tensors
        w = ctx.w
        ds, ds16 = N.rmsnorm_bwd(dy.contiguous(), s, w, rstd, ds_in, w.main_grad, not GRAD["first"], write_ds16=True)
        return ds16, ds, None, None


class FinalNormFn(torch.autograd.Function):
    """Final norm: y = rmsnorm(r + a) * w without keeping s as an output."""

    @staticmethod
    def forward(ctx, a, r, w, eps):
        y, s, rstd = N.add_rmsnorm_fwd(a, r, w, eps, write_s=True)
        ctx.save_for_backward(s, rstd)
        ctx.w = w
        return y

    @staticmethod
    def backward(ctx, dy):
        s, rstd = ctx.saved_tensors
        w = ctx.w
        ds, ds16 = N.rmsnorm_bwd(dy.contiguous(), s, w, rstd, None, w.main_grad, not GRAD["first"], write_ds16=True)
        return ds16, ds, None, None


def wgrad_into(dy, x, out):
    """out (M, N) fp32 (+)= dy^T x on the tcgen05 GEMM; on a first write it stores (or zeroes
    first when the planner splits K)."""
    if GRAD["first"]:
        _, splits = N.gemm_plan(dy.shape[1], x.shape[1], dy.shape[0], N.EPI_F32, True)
        if splits == 1:
            N.gemm(dy, x, ta=True, tb=False, out=out, accumulate=False)
            return
        out.zero_()
    N.gemm(dy, x, ta=True, tb=False, out=out, accumulate=True)


def first_write_zero(out):
    """Zero `out` if this is the step's first write and the caller can only accumulate."""
    if GRAD["first"]:
        out.zero_()


def _wgrad(dy, x, p):
    """p.main_grad (out, in) (+)= dy^T x, fp32, on the tcgen05 GEMM."""
    wgrad_into(dy, x, p.main_grad)


class QKVAttention(torch.autograd.Function):
    """o = attention(rope(x Wqkv^T)); x (B*T, d) bf16 -> o (B*T, H*hd) bf16."""

    @staticmethod
    def forward(ctx, x, w, cos, sin, B, T, H, KV, hd):
        if FUSION["rope"]:
            qkv = N.gemm_rope(x, w.w16, cos, sin, T, hd, (H + KV) * hd)
        else:
            qkv = N.gemm(x, w.w16, ta=False, tb=True)
            N.rope_inplace(qkv, cos, sin, T, H + KV, hd)
        o, lse = N.flash_attn_fwd(qkv, B, T, H, KV, hd, causal=True)
        ctx.save_for_backward(x, qkv, o, lse, cos, sin)
        ctx.w = w
        ctx.dims = (B, T, H, KV, hd)
        return o

    @staticmethod
    def backward(ctx, do):
        x, qkv, o, lse, cos, sin = ctx.saved_tensors
        B, T, H, KV, hd = ctx.dims
        w = ctx.w
        dqkv = N.flash_attn_bwd(do.contiguous(), qkv, o, lse, cos, sin, B, T, H, KV, hd, causal=True)
        dx = N.gemm(dqkv, w.w16, ta=False, tb=False)
        _wgrad(dqkv, x, w)
        return dx, None, None, None, None, None, None, None, None


class Linear(torch.autograd.Function):
    """y = x W^T with bf16 operands; W's fp32 gradient goes to W.main_grad."""

    @staticmethod
    def forward(ctx, x, w):
        ctx.save_for_backward(x)
        ctx.w = w
        return N.gemm(x, w.w16, ta=False, tb=True)

    @staticmethod
    def backward(ctx, dy):
        (x,) = ctx.saved_tensors
        w = ctx.w
        dy = dy.contiguous()
        dx = N.gemm(dy, w.w16, ta=False, tb=False)
        _wgrad(dy, x, w)
        return dx, None


class SwiGLUMLP(torch.autograd.Function):
    """m = (silu(x W1^T) * (x W3^T)) W2^T with W1, W3 packed adjacently (one merged GEMM).

    SwiGLU runs either inside the GEMM epilogues (merged gate/up GEMM writes h and keeps [g | u];
    the w2 dgrad writes [dg | du]) or as the standalone elementwise kernel after a plain GEMM;
    SWIGLU_EPILOGUE selects per direction."""

    @staticmethod
    def forward(ctx, x, w1, w2, ffn, comm=None):
        if SWIGLU_EPILOGUE["fwd"]:
            h, gu = N.gemm_swiglu(x, w1.w13_16, ffn)
        else:
            gu = N.gemm(x, w1.w13_16, ta=False, tb=True)
            h = N.swiglu_fwd(gu[:, :ffn], gu[:, ffn:])
        # tensor parallel over peer memory: the w2 GEMM stores its rows to their owner ranks
        m = comm.gemm_rs(h, w2.w16) if comm is not None else N.gemm(h, w2.w16, ta=False, tb=True)
        ctx.save_for_backward(x, h, gu)
        ctx.w1, ctx.w2, ctx.ffn, ctx.comm = w1, w2, ffn, comm
        return m

    @staticmethod
    def backward(ctx, dm):
        x, h, gu = ctx.saved_tensors
        w1, w2, ffn = ctx.w1, ctx.w2, ctx.ffn
        dm = dm.contiguous()
        if ctx.comm is not None:
            dm = ctx.comm.all_gather_bwd(dm)
        if SWIGLU_EPILOGUE["bwd"]:
            dgu = N.gemm_swiglu_bwd(dm, w2.w16, gu, ffn)
            _wgrad(dm, h, w2)
        else:
            _wgrad(dm, h, w2)
            dh = N.gemm(dm, w2.w16, ta=False, tb=False, out=h)  # h is dead after the w2 wgrad
            g, u = gu[:, :ffn], gu[:, ffn:]
            N.swiglu_bwd(dh, g, u, dg=g, du=u)  # [dg | du] overwrite [g | u] in place
            dgu = gu
        dx = N.gemm(dgu, w1.w13_16, ta=False, tb=False)
        wgrad_into(dgu, x, w1.w13_grad)
        return dx, None, None, None, None


class HeadCEVP(torch.autograd.Function):
    """Cross entropy over a vocabulary-parallel head (rows [v0, v0 + V/tp) on this rank).

    Forward: the fused head GEMM reduces this shard's logit tiles to a per-row log-sum-exp and
    target logit (targets shifted by v0; a target outside the shard contributes nothing); the
    (N,) log-sum-exps of all shards are all-gathered and combined, the target logits summed.
    Backward recomputes this shard's logits into bf16 (softmax - onehot) / N chunks and returns
    the partial dh (the all-gather that produced h sums the shards' partials)."""

    @staticmethod
    def forward(ctx, h, w, targets, v0, group, chunk):
        tl_targets = targets - v0
        lse_l, _, tl = N.gemm_ce_fwd(h, w.w16, tl_targets, return_target_logit=True)
        world = torch.distributed.get_world_size(group)
        allse = torch.empty((world,) + tuple(lse_l.shape), dtype=lse_l.dtype, device=lse_l.device)
        torch.distributed.all_gather_into_tensor(allse, lse_l, group=group)
        lse = torch.logsumexp(allse, dim=0)
        torch.distributed.all_reduce(tl, group=group)
        ctx.save_for_backward(h, tl_targets, lse)
        ctx.w, ctx.chunk = w, chunk
        return (lse - tl).mean()

    @staticmethod
    def backward(ctx, g):
        h, targets, lse = ctx.saved_tensors
        w, chunk = ctx.w, ctx.chunk
        n = h.shape[0]
        g = g.reshape(1).float().contiguous()
        dh = torch.empty_like(h)
        for c0 in range(0, n, chunk):
            c1 = min(n, c0 + chunk)
            hc = h[c0:c1]
            dl = N.gemm_ce_bwd(hc, w.w16, targets[c0:c1], lse[c0:c1], g, 1.0 / n)
            N.gemm(dl, w.w16, ta=False, tb=False, out=dh[c0:c1])
            N.gemm(dl, hc, ta=True, tb=False, out=w.main_grad, accumulate=True)
        return dh, None, None, None, None, None


class HeadCE(torch.autograd.Function):
    """Mean cross entropy of the lm head; logits are never written (forward), and are
    recomputed tile by tile into bf16 dlogits chunks of at most `chunk` rows (backward).
    With FUSION["head_ce"] off: bf16 logits are written and the row CE kernels run on them."""

    @staticmethod
    def forward(ctx, h, w, targets, chunk):
        ctx.w, ctx.chunk = w, chunk
        fused = FUSION["head_ce"]
        if fused == "auto":
            fused = h.shape[0] * w.shape[0] * 2 > HEAD_LOGITS_BUDGET
        if not fused:
            logits = N.gemm(h, w.w16, ta=False, tb=True)
            lse = torch.empty(h.shape[0], dtype=torch.float32, device=h.device)
            loss_rows = torch.empty_like(lse)
            N.ce_fwd_rows(logits, targets, lse, loss_rows)
            ctx.save_for_backward(h, targets, lse, logits)
            return loss_rows.mean()
        lse, loss_rows = N.gemm_ce_fwd(h, w.w16, targets)
        ctx.save_for_backward(h, targets, lse)
        return loss_rows.mean()

    @staticmethod
    def backward(ctx, g):
        h, targets, lse = ctx.saved_tensors[:3]
        w, chunk = ctx.w, ctx.chunk
        n = h.shape[0]
        g = g.reshape(1).float().contiguous()
        if len(ctx.saved_tensors) == 4:  # unfused: dlogits in place over the saved logits
            dl = ctx.saved_tensors[3]
            N.ce_bwd_rows(dl, targets, lse, g, 1.0 / n)
            dh = N.gemm(dl, w.w16, ta=False, tb=False)
            wgrad_into(dl, h, w.main_grad)
            return dh, None, None, None
        dh = torch.empty_like(h)
        for c0 in range(0, n, chunk):
            c1 = min(n, c0 + chunk)
            hc = h[c0:c1]
            dl = N.gemm_ce_bwd(hc, w.w16, targets[c0:c1], lse[c0:c1], g, 1.0 / n)
            N.gemm(dl, w.w16, ta=False, tb=False, out=dh[c0:c1])
            if c0 == 0:
                wgrad_into(dl, hc, w.main_grad)
            else:
                N.gemm(dl, hc, ta=True, tb=False, out=w.main_grad, accumulate=True)
        return dh, None, None, None
