"""FP8 (tensorwise e4m3) versions of the native block's linear regions.

Same recipe as the reference's _FP8Linear (kernels/lowp.py:73-95): all three GEMMs of a linear
(forward, dgrad, wgrad) run on e4m3 operands with tensorwise current scaling recomputed every
step (scale = 448 / amax) for x, the fp32 weight and dy alike, and x and w are kept as fp8
transposed copies for the backward. The lm head stays bf16 (reference lowp.py:21-22).

Here the GEMMs are the tcgen05 kind::f8f6f4 kernel, both operands K-major (the hardware's fp8
layout, which is why the transposed copies exist), with the native block's fused epilogues and
the inverse scales applied to the fp32 accumulator: RoPE in the qkv GEMM, SwiGLU in the merged
gate/up GEMM, the SwiGLU backward in the w2 dgrad, TMA reduce-add of the fp32 weight gradient
into main_grad. W1 and W3 form one merged (2*ffn, d) tensor with one scale, and their gradients
[dg | du] share one scale too (the reference quantizes w1 and w3 as separate linears).
Quantization is llmt._C.fp8_quant: no host synchronisation, so the step captures in a CUDA graph.
"""
from __future__ import annotations

import torch

from llmt.ops import native as N
from llmt.ops.functions import first_write_zero


class QKVAttentionFP8(torch.autograd.Function):
    """o = attention(rope(x Wqkv^T)) with the qkv GEMM on e4m3 operands."""

    @staticmethod
    def forward(ctx, x, w, cos, sin, B, T, H, KV, hd):
        xq, xqt, sx = N.fp8_quant(x)
        wq, wqt, sw = N.fp8_quant(w)
        qkv = N.gemm_fp8_rope(xq, wq, sx, sw, cos, sin, T, hd, (H + KV) * hd)
        o, lse = N.flash_attn_fwd(qkv, B, T, H, KV, hd, causal=True)
        ctx.save_for_backward(xqt, sx, wqt, sw, qkv, o, lse, cos, sin)
        ctx.w = w
        ctx.dims = (B, T, H, KV, hd)
        return o

    @staticmethod
    def backward(ctx, do):
        xqt, sx, wqt, sw, qkv, o, lse, cos, sin = ctx.saved_tensors
        B, T, H, KV, hd = ctx.dims
        dqkv = N.flash_attn_bwd(do.contiguous(), qkv, o, lse, cos, sin, B, T, H, KV, hd, causal=True)
        dq, dqt, sd = N.fp8_quant(dqkv)
        dx = N.gemm_fp8(dq, wqt, sd, sw)
        first_write_zero(ctx.w.main_grad)
        N.gemm_fp8(dqt, xqt, sd, sx, out=ctx.w.main_grad, accumulate=True)
        return dx, None, None, None, None, None, None, None, None


class LinearFP8(torch.autograd.Function):
    """y = x W^T on e4m3 operands (reference _FP8Linear)."""

    @staticmethod
    def forward(ctx, x, w):
        xq, xqt, sx = N.fp8_quant(x)
        wq, wqt, sw = N.fp8_quant(w)
        ctx.save_for_backward(xqt, sx, wqt, sw)
        ctx.w = w
        return N.gemm_fp8(xq, wq, sx, sw)

    @staticmethod
    def backward(ctx, dy):
        xqt, sx, wqt, sw = ctx.saved_tensors
        dq, dqt, sd = N.fp8_quant(dy.contiguous())
        dx = N.gemm_fp8(dq, wqt, sd, sw)
        first_write_zero(ctx.w.main_grad)
        N.gemm_fp8(dqt, xqt, sd, sx, out=ctx.w.main_grad, accumulate=True)
        return dx, None


class SwiGLUMLPFP8(torch.autograd.Function):
    """m = (silu(x W1^T) * (x W3^T)) W2^T, every GEMM on e4m3 operands."""

    @staticmethod
    def forward(ctx, x, w1, w2, ffn):
        xq, xqt, sx = N.fp8_quant(x)
        w13q, w13qt, s13 = N.fp8_quant(w1.w13)
        h, gu = N.gemm_fp8_swiglu(xq, w13q, sx, s13, ffn)
        hq, hqt, sh = N.fp8_quant(h)
        w2q, w2qt, s2 = N.fp8_quant(w2)
        m = N.gemm_fp8(hq, w2q, sh, s2)
        ctx.save_for_backward(xqt, sx, w13qt, s13, hqt, sh, w2qt, s2, gu)
        ctx.w1, ctx.w2, ctx.ffn = w1, w2, ffn
        return m

    @staticmethod
    def backward(ctx, dm):
        xqt, sx, w13qt, s13, hqt, sh, w2qt, s2, gu = ctx.saved_tensors
        w1, w2, ffn = ctx.w1, ctx.w2, ctx.ffn
        dmq, dmqt, sd = N.fp8_quant(dm.contiguous())
        dgu = N.gemm_fp8_swiglu_bwd(dmq, w2qt, sd, s2, gu, ffn)
        first_write_zero(w2.main_grad)
        N.gemm_fp8(dmqt, hqt, sd, sh, out=w2.main_grad, accumulate=True)
        dgq, dgqt, sg = N.fp8_quant(dgu)
        dx = N.gemm_fp8(dgq, w13qt, sg, s13)
        first_write_zero(w1.w13_grad)
        N.gemm_fp8(dgqt, xqt, sg, sx, out=w1.w13_grad, accumulate=True)
        return dx, None, None, None
