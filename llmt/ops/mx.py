"""Block-scaled (MXFP8 / NVFP4) versions of the native block's linear regions.

Block scales run along a GEMM's contraction dimension, so every operand is quantized along the
axis its GEMM contracts (the reference's _FP4Linear, kernels/lowp.py:312-340):
    forward  y  = x  W^T    x along K,  W along K
    dgrad    dx = dy W      dy along N, W^T along N
    wgrad    dW = dy^T x    dy^T along M, x^T along M
One llmt._C.mx_quant pass writes a tensor's row-wise and transposed copies together (weights
once per step: the forward keeps the transposed copy for the dgrad). NVFP4
rounds gradients stochastically and weights / activations to nearest, like the reference; its
per-tensor decode scales are applied in the GEMM epilogue. MXFP8 (ue8m0 scale per 32) is the
Blackwell format the medium and 8B configs name. The GEMMs are the tcgen05 block-scaled kinds
with the native fused epilogues (RoPE in qkv, SwiGLU in the merged gate/up GEMM, whose weight is
quantized with its W1 / W3 rows interleaved by 64 to match the tiles, the SwiGLU backward in the
w2 dgrad, fp32 reduce-add of weight gradients into main_grad). The head stays bf16.
"""
from __future__ import annotations

import torch

from llmt.ops import native as N
from llmt.ops.functions import first_write_zero


def _sr(kind):
    return kind == N.NVFP4


class QKVAttentionMX(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, cos, sin, B, T, H, KV, hd, kind):
        xr, xc = N.mx_quant(x, kind, row=True, col=True)
        wr, wc = N.mx_quant(w, kind, row=True, col=True)
        qkv = N.gemm_mx_rope(kind, xr, wr, cos, sin, T, hd, (H + KV) * hd)
        o, lse = N.flash_attn_fwd(qkv, B, T, H, KV, hd, causal=True)
        ctx.save_for_backward(qkv, o, lse, cos, sin)
        ctx.xc, ctx.wc, ctx.w, ctx.kind, ctx.dims = xc, wc, w, kind, (B, T, H, KV, hd)
        return o

    @staticmethod
    def backward(ctx, do):
        qkv, o, lse, cos, sin = ctx.saved_tensors
        B, T, H, KV, hd = ctx.dims
        kind, w = ctx.kind, ctx.w
        dqkv = N.flash_attn_bwd(do.contiguous(), qkv, o, lse, cos, sin, B, T, H, KV, hd, causal=True)
        dr, dc = N.mx_quant(dqkv, kind, row=True, col=True, stochastic=_sr(kind))
        dx = N.gemm_mx(kind, dr, ctx.wc)
        first_write_zero(w.main_grad)
        N.gemm_mx(kind, dc, ctx.xc, out=w.main_grad, accumulate=True)
        ctx.xc = ctx.wc = None
        return dx, None, None, None, None, None, None, None, None, None


class LinearMX(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, kind):
        xr, xc = N.mx_quant(x, kind, row=True, col=True)
        wr, wc = N.mx_quant(w, kind, row=True, col=True)
        ctx.xc, ctx.wc, ctx.w, ctx.kind = xc, wc, w, kind
        return N.gemm_mx(kind, xr, wr)

    @staticmethod
    def backward(ctx, dy):
        kind, w = ctx.kind, ctx.w
        dr, dc = N.mx_quant(dy.contiguous(), kind, row=True, col=True, stochastic=_sr(kind))
        dx = N.gemm_mx(kind, dr, ctx.wc)
        first_write_zero(w.main_grad)
        N.gemm_mx(kind, dc, ctx.xc, out=w.main_grad, accumulate=True)
        ctx.xc = ctx.wc = None
        return dx, None, None


class SwiGLUMLPMX(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w1, w2, ffn, kind):
        xr, xc = N.mx_quant(x, kind, row=True, col=True)
        # row copy interleaved for the SwiGLU tiles; the transposed copy (dgrad) in natural order
        w13r, w13c = N.mx_quant(w1.w13, kind, row=True, col=True, interleave64=True)
        h, gu = N.gemm_mx_swiglu(kind, xr, w13r, ffn)
        hr, hc = N.mx_quant(h, kind, row=True, col=True)
        w2r, w2c = N.mx_quant(w2, kind, row=True, col=True)
        m = N.gemm_mx(kind, hr, w2r)
        ctx.save_for_backward(gu)
        ctx.xc, ctx.hc, ctx.w2c, ctx.w13c = xc, hc, w2c, w13c
        ctx.w1, ctx.w2, ctx.ffn, ctx.kind = w1, w2, ffn, kind
        return m

    @staticmethod
    def backward(ctx, dm):
        (gu,) = ctx.saved_tensors
        w1, w2, ffn, kind = ctx.w1, ctx.w2, ctx.ffn, ctx.kind
        dmr, dmc = N.mx_quant(dm.contiguous(), kind, row=True, col=True, stochastic=_sr(kind))
        dgu = N.gemm_mx_swiglu_bwd(kind, dmr, ctx.w2c, gu, ffn)
        first_write_zero(w2.main_grad)
        N.gemm_mx(kind, dmc, ctx.hc, out=w2.main_grad, accumulate=True)
        dgr, dgc = N.mx_quant(dgu, kind, row=True, col=True, stochastic=_sr(kind))
        dx = N.gemm_mx(kind, dgr, ctx.w13c)
        first_write_zero(w1.w13_grad)
        N.gemm_mx(kind, dgc, ctx.xc, out=w1.w13_grad, accumulate=True)
        ctx.xc = ctx.hc = ctx.w2c = ctx.w13c = None
        return dx, None, None, None, None
