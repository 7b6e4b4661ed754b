"""Plain-PyTorch statement of the fp8 linear recipe: the oracle for the sm_100a kernels.

Tensorwise e4m3 with current scaling, as the reference's _fp8_quant_impl / _FP8Linear
(kernels/lowp.py:51-95): amax = max |x| (at least 1e-12), scale = 448 / amax,
q = e4m3(clamp(x * scale, -448, 448)), inverse scale 1 / scale. The GEMMs here are fp32 matmuls
of the e4m3 values times both inverse scales, which is what a tensor-core fp8 GEMM with fp32
accumulation computes up to summation order. Runs on any device (the CPU tests use it), and
`llmt.ops.native.fp8_quant` must reproduce fp8_quant_ref bit for bit.
"""
from __future__ import annotations

import torch

E4M3_MAX = 448.0


def fp8_quant_ref(x: torch.Tensor):
    """(q e4m3, inv fp32 1-element) of a tensor."""
    amax = x.abs().amax().float().clamp_min(1e-12)
    scale = E4M3_MAX / amax
    q = (x.float() * scale).clamp(-E4M3_MAX, E4M3_MAX).to(torch.float8_e4m3fn)
    return q, scale.reciprocal().reshape(1)


def fp8_matmul_ref(aq, bq, sa, sb):
    """(a @ b^T) * sa * sb in fp32 for e4m3 a (M, K), b (N, K)."""
    return (aq.float() @ bq.float().t()) * (sa * sb)


class FP8LinearRef(torch.autograd.Function):
    """y = x W^T with forward, dgrad and wgrad all on tensorwise e4m3 operands (dy too)."""

    @staticmethod
    def forward(ctx, x, w):
        shape = x.shape
        x2 = x.reshape(-1, shape[-1])
        xq, sx = fp8_quant_ref(x2)
        wq, sw = fp8_quant_ref(w)
        ctx.save_for_backward(xq, sx, wq, sw)
        ctx.shape, ctx.dtype = shape, x.dtype
        return fp8_matmul_ref(xq, wq, sx, sw).to(x.dtype).view(*shape[:-1], w.shape[0])

    @staticmethod
    def backward(ctx, dy):
        xq, sx, wq, sw = ctx.saved_tensors
        dq, sd = fp8_quant_ref(dy.reshape(-1, dy.shape[-1]))
        dx = fp8_matmul_ref(dq, wq.t().contiguous(), sd, sw)
        dw = fp8_matmul_ref(dq.t().contiguous(), xq.t().contiguous(), sd, sx)
        return dx.to(ctx.dtype).view(ctx.shape), dw


def fp8_linear_ref(x, w):
    return FP8LinearRef.apply(x, w)
