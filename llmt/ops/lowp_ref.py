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


# ---------------------------------------------------------------- block-scaled formats
# Chunked scale layout of the block-scaled GEMM: 512-byte chunks of 128 rows x 4 scales, row r
# at (r % 32) * 16 + ((r % 128) // 32) * 4, scale column c at + c % 4, chunks ordered
# [row tile][c // 4]; every row tile holds whole k-blocks of 128 bytes of data (MXFP8: 128
# values = 1 chunk, NVFP4: 256 values = 4 chunks), zero-padded.
FP4_GRID = (0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0)
_FP4_MIDS = (0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0)


def chunks_per_tile(kind: int, cols: int) -> int:
    return -(-cols // 128) if kind == 2 else 4 * (-(-cols // 256))


def to_chunks(sf: torch.Tensor, kind: int, cols: int) -> torch.Tensor:
    """(rows, scale columns) bytes -> the flat chunked layout (zero padding included)."""
    R, S = sf.shape
    ch = chunks_per_tile(kind, cols)
    out = torch.zeros(-(-R // 128) * ch * 512, dtype=torch.uint8, device=sf.device)
    r = torch.arange(R, device=sf.device)[:, None]
    c = torch.arange(S, device=sf.device)[None, :]
    off = ((r // 128) * ch + c // 4) * 512 + (r % 32) * 16 + ((r % 128) // 32) * 4 + c % 4
    out[off.reshape(-1)] = sf.reshape(-1).view(torch.uint8)
    return out


def mxfp8_quant_ref(x: torch.Tensor):
    """MXFP8 along the last dim: (q e4m3 (R, C), scale bytes (R, C / 32) = e + 127) with 2^e the
    smallest power of two that keeps the block's amax within 448."""
    R, C = x.shape
    b = x.float().view(R, C // 32, 32)
    amax = b.abs().amax(-1)
    m, E2 = torch.frexp(amax)  # amax = m 2^E2, m in [0.5, 1)
    e = torch.where(2 * m > 1.75, E2 - 8, E2 - 9)
    e = torch.where(amax < 2.0 ** -126, torch.full_like(e, -127), e).clamp(min=-127)
    q = (b * torch.ldexp(torch.ones_like(amax), -e)[..., None]).clamp(-E4M3_MAX, E4M3_MAX)
    return q.to(torch.float8_e4m3fn).view(R, C), (e + 127).to(torch.uint8)


def mxfp8_dequant(q, sf):
    R, C = q.shape
    s = torch.ldexp(torch.ones(sf.shape, device=q.device), sf.long() - 127)
    return (q.float().view(R, C // 32, 32) * s[..., None]).view(R, C)


def nvfp4_quant_ref(x: torch.Tensor, noise=None):
    """NVFP4 along the last dim (the reference's recipe): packed e2m1 (R, C / 2) with the first
    value in the low nibble, e4m3 block scales (R, C / 16), per-tensor decode scale g (1,)."""
    R, C = x.shape
    xf = x.float()
    # amax / 2688 as PyTorch evaluates it on CUDA: amax times the float reciprocal of 2688
    inv = torch.tensor(1.0, dtype=torch.float32) / torch.tensor(6.0 * E4M3_MAX, dtype=torch.float32)
    g = (xf.abs().amax() * inv.to(x.device)).clamp_min(1e-30)
    b = xf.view(R, C // 16, 16)
    s8 = (b.abs().amax(-1) / (6.0 * g)).clamp(max=E4M3_MAX).to(torch.float8_e4m3fn)
    denom = s8.float() * g
    # one reciprocal per block, as the reference's Triton quantizer (kernels/lowp.py:213-214)
    inv = torch.where(denom > 0, 1.0 / denom, torch.zeros_like(denom))
    v = (b * inv[..., None]).clamp(-6.0, 6.0)
    mag = v.abs()
    if noise is None:
        idx = (mag[..., None] > torch.tensor(_FP4_MIDS, device=x.device)).sum(-1)
    else:
        grid = torch.tensor(FP4_GRID, device=x.device)
        lo = (mag[..., None] >= grid[1:]).sum(-1)
        hi = (lo + 1).clamp(max=7)
        lv, hv = grid[lo], grid[hi]
        frac = torch.where(hv > lv, (mag - lv) / (hv - lv), torch.zeros_like(mag))
        idx = torch.where(noise.view(R, C // 16, 16) < frac, hi, lo)
    code = (idx | (((v < 0) & (idx > 0)).long() << 3)).view(R, C // 2, 2)
    packed = (code[..., 0] | (code[..., 1] << 4)).to(torch.uint8)
    return packed, s8, g.reshape(1)


def nvfp4_dequant(packed, s8, g):
    grid = torch.tensor(FP4_GRID, device=packed.device)
    codes = torch.stack([packed & 15, packed >> 4], -1).long().flatten(-2)
    vals = grid[codes & 7] * torch.where((codes & 8) > 0, -1.0, 1.0)
    R, C = vals.shape
    return (vals.view(R, C // 16, 16) * (s8.float() * g)[..., None]).view(R, C)
