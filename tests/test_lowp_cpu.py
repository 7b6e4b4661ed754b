"""FP8 recipe oracle (llmt.ops.lowp_ref) on CPU: the quantizer's format and the linear's error.

Mirrors the reference's low-precision unit tests (kernels/test_lowp.py:89-106): the fp8 linear's
forward, dgrad and wgrad against fp32 within the e4m3 format's error."""
import pytest
import torch

from llmt.ops.lowp_ref import E4M3_MAX, fp8_linear_ref, fp8_quant_ref
from tests.helpers import rel_err


def test_fp8_quant_scale_and_grid():
    g = torch.Generator().manual_seed(0)
    x = torch.randn(256, 320, generator=g) * 3.0
    q, inv = fp8_quant_ref(x)
    assert q.dtype == torch.float8_e4m3fn and inv.shape == (1,)
    qf = q.float()
    # the largest magnitude lands on the format's maximum; every value is on the e4m3 grid
    assert qf.abs().max().item() == E4M3_MAX
    assert torch.equal(qf.to(torch.float8_e4m3fn).float(), qf)
    assert abs(inv.item() * E4M3_MAX - x.abs().max().item()) < 1e-5 * x.abs().max().item()
    assert rel_err(qf * inv, x) < 0.04


def test_fp8_quant_zero_tensor_is_finite():
    q, inv = fp8_quant_ref(torch.zeros(16, 16))
    assert torch.isfinite(inv).all() and q.float().abs().max().item() == 0.0


@pytest.mark.parametrize("M,N,K", [(128, 96, 64), (256, 688, 256)])
def test_fp8_linear_fwd_dgrad_wgrad(M, N, K):
    g = torch.Generator().manual_seed(1)
    x = torch.randn(M, K, generator=g, requires_grad=True)
    w = (torch.randn(N, K, generator=g) * 0.05).requires_grad_()
    dy = torch.randn(M, N, generator=g)
    y = fp8_linear_ref(x, w)
    y.backward(dy)
    xr, wr = x.detach().clone().requires_grad_(), w.detach().clone().requires_grad_()
    (xr @ wr.t()).backward(dy)
    assert rel_err(y, xr.detach() @ wr.detach().t()) < 0.06
    assert rel_err(x.grad, xr.grad) < 0.06
    assert rel_err(w.grad, wr.grad) < 0.06


def test_mxfp8_oracle_scales_and_error():
    from llmt.ops.lowp_ref import mxfp8_dequant, mxfp8_quant_ref
    g = torch.Generator().manual_seed(2)
    x = torch.randn(128, 256, generator=g) * torch.logspace(-3, 3, 256)  # blocks of very different ranges
    q, s = mxfp8_quant_ref(x)
    blocks = x.view(128, 8, 32).abs().amax(-1)
    scale = torch.ldexp(torch.ones_like(blocks), s.long() - 127)
    # the smallest power of two that keeps each block within the e4m3 range
    assert bool((blocks <= 448 * scale).all()) and bool((blocks > 224 * scale).all())
    assert rel_err(mxfp8_dequant(q, s), x) < 0.04


def test_nvfp4_oracle_grid_and_stochastic_rounding():
    from llmt.ops.lowp_ref import FP4_GRID, nvfp4_dequant, nvfp4_quant_ref
    g = torch.Generator().manual_seed(3)
    x = torch.randn(64, 128, generator=g)
    p, s8, gs = nvfp4_quant_ref(x)
    codes = torch.stack([p & 15, p >> 4], -1).flatten(-2)
    assert int(codes.max()) <= 15 and p.shape == (64, 64)
    d = nvfp4_dequant(p, s8, gs)
    assert rel_err(d, x) < 0.12  # reference round-trip bound (kernels/test_lowp.py:43-47)
    mags = (d.view(64, 8, 16).abs() / (s8.float() * gs)[..., None]).flatten()
    grid = torch.tensor(FP4_GRID)
    assert bool(((mags[:, None] - grid).abs().min(-1).values < 1e-5).all())  # on the e2m1 grid
    acc = torch.zeros_like(x)
    n = 400
    for _ in range(n):
        pp, ss, gg = nvfp4_quant_ref(x, torch.rand(64, 128, generator=g))
        acc += nvfp4_dequant(pp, ss, gg)
    assert rel_err(acc / n, x) < 0.02  # unbiased within 2% over 400 draws (test_lowp.py:53-59)


def test_chunked_scale_layout():
    from llmt.ops.lowp_ref import to_chunks
    sf = torch.arange(256 * 8, dtype=torch.int64).remainder(251).to(torch.uint8).view(256, 8)
    out = to_chunks(sf, 2, 256)
    assert out.numel() == 2 * 2 * 512
    r, c = 37, 5  # tile 0, chunk 1, row 37 -> (37 % 32) * 16 + 1 * 4, scale 5 % 4
    assert out[(0 * 2 + 1) * 512 + 5 * 16 + 1 * 4 + 1] == sf[r, c]
