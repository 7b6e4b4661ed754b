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
