"""Numerics of the memory-bound sm_100a kernels vs plain PyTorch fp32 references.

Mirrors the reference's compare() harness (kernels/test_kernels.py:83-102): same random
inputs and output gradients for the kernel and an fp32 reference, relative L2 error of
every output and every input gradient."""
import pytest
import torch
import torch.nn.functional as F

from tests.helpers import rel_err

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def nat():
    from llmt.ops import native
    native.ext()
    return native


def _rms_ref(s, w, eps):
    return s * torch.rsqrt(s.pow(2).mean(-1, keepdim=True) + eps) * w


@pytest.mark.parametrize("N,D", [(37, 256), (1000, 768), (513, 1024), (64, 2048), (33, 4096), (8, 8192)])
@pytest.mark.parametrize("has_a", [False, True])
def test_add_rmsnorm_fwd_bwd(nat, N, D, has_a):
    g = torch.Generator(device="cuda").manual_seed(0)
    r = torch.randn(N, D, device="cuda", generator=g)
    a = torch.randn(N, D, device="cuda", generator=g).bfloat16() if has_a else None
    w = 1 + 0.1 * torch.randn(D, device="cuda", generator=g)
    y, s, rstd = nat.add_rmsnorm_fwd(a, r, w, 1e-5)
    s_ref = r + (a.float() if has_a else 0)
    assert rel_err(s, s_ref) < 1e-6
    assert rel_err(y, _rms_ref(s_ref, w, 1e-5)) < 1e-2
    dy = torch.randn(N, D, device="cuda", generator=g).bfloat16()
    ds_in = torch.randn(N, D, device="cuda", generator=g)
    sl = s_ref.clone().requires_grad_(True)
    wl = w.clone().requires_grad_(True)
    _rms_ref(sl, wl, 1e-5).backward(dy.float())
    dw = torch.zeros(D, device="cuda")
    ds, ds16 = nat.rmsnorm_bwd(dy, s, w, rstd, ds_in, dw, accumulate=False)
    assert rel_err(ds, sl.grad + ds_in) < 1e-5
    assert rel_err(ds16, sl.grad + ds_in) < 1e-2
    assert rel_err(dw, wl.grad) < 1e-4
    nat.rmsnorm_bwd(dy, s, w, rstd, None, dw, accumulate=True)
    assert rel_err(dw, 2 * wl.grad) < 1e-4


def test_swiglu_standalone(nat):
    g = torch.Generator(device="cuda").manual_seed(1)
    gu = torch.randn(1000, 2 * 1376, device="cuda", generator=g).bfloat16()
    a, b = gu[:, :1376], gu[:, 1376:]
    h = nat.swiglu_fwd(a, b)
    af, bf = a.float().requires_grad_(True), b.float().requires_grad_(True)
    ref = F.silu(af) * bf
    assert rel_err(h, ref) < 1e-2
    dh = torch.randn(1000, 1376, device="cuda", generator=g).bfloat16()
    ref.backward(dh.float())
    dg, du = nat.swiglu_bwd(dh, a, b)
    assert rel_err(dg, af.grad) < 1e-2
    assert rel_err(du, bf.grad) < 1e-2


@pytest.mark.parametrize("H,KV,hd", [(12, 12, 64), (16, 4, 128)])
def test_rope_inplace_fwd_bwd(nat, H, KV, hd):
    from llmt.models.llama import apply_rope, rope_tables
    B, T = 2, 100
    g = torch.Generator(device="cuda").manual_seed(2)
    qkv = torch.randn(B * T, (H + 2 * KV) * hd, device="cuda", generator=g).bfloat16()
    cos, sin = rope_tables(T, hd, 10000.0, "cuda")
    out = nat.rope_inplace(qkv.clone(), cos, sin, T, H + KV, hd)
    v4 = qkv.view(B, T, H + 2 * KV, hd).float()
    rot = apply_rope(v4[:, :, : H + KV].transpose(1, 2), cos, sin).transpose(1, 2)
    ref = v4.clone()
    ref[:, :, : H + KV] = rot
    assert rel_err(out.view(B, T, -1, hd), ref) < 1e-2
    back = nat.rope_inplace(out.clone(), cos, sin, T, H + KV, hd, backward=True)
    assert rel_err(back, qkv) < 2e-2


def test_embedding(nat):
    g = torch.Generator(device="cuda").manual_seed(3)
    W = torch.randn(32000, 768, device="cuda", generator=g)
    idx = torch.randint(0, 32000, (4, 256), device="cuda", generator=g)
    x = nat.embedding_fwd(idx, W)
    assert torch.equal(x, W[idx.reshape(-1)])
    dx = torch.randn(1024, 768, device="cuda", generator=g)
    dW = torch.zeros_like(W)
    nat.embedding_bwd(idx, dx, dW)
    ref = torch.zeros_like(W).index_add_(0, idx.reshape(-1), dx)
    assert rel_err(dW, ref) < 1e-5


def test_adamw_matches_torch(nat):
    g = torch.Generator(device="cuda").manual_seed(4)
    n = 100003
    p = torch.randn(n, device="cuda", generator=g)
    p_ref = torch.nn.Parameter(p.clone())
    opt = torch.optim.AdamW([p_ref], lr=3e-4, betas=(0.9, 0.95), weight_decay=0.1)
    m = torch.zeros_like(p)
    v = torch.zeros_like(p)
    p16 = torch.empty(n, device="cuda", dtype=torch.bfloat16)
    lr = torch.full((1,), 3e-4, device="cuda")
    step = torch.zeros(1, device="cuda", dtype=torch.int32)
    for _ in range(3):
        grad = torch.randn(n, device="cuda", generator=g)
        p_ref.grad = grad.clone()
        opt.step()
        step += 1
        nat.adamw_step(p, grad, m, v, p16, lr, step, 0.9, 0.95, 1e-8, 0.1)
    assert rel_err(p, p_ref.detach()) < 1e-6
    assert rel_err(p16, p_ref.detach()) < 1e-2


@pytest.mark.parametrize("n,blocks", [(8, 0), (1 << 20, 0), (1 << 20, 3), (1000 * 8 + 8, 5), (1001, 2)])
def test_cast_bf16_matches_torch(nat, n, blocks):
    """Vector path (n a multiple of 8, 16-byte aligned) and scalar path, with and without a grid cap
    (the overlapped data-parallel step casts on a few SMs)."""
    g = torch.Generator(device="cuda").manual_seed(9)
    x = torch.randn(n + 8, device="cuda", generator=g)
    y = torch.full((n + 16,), 7.0, device="cuda", dtype=torch.bfloat16)
    nat.ext().cast_bf16(x[:n], y[8:8 + n], blocks)
    assert torch.equal(y[8:8 + n], x[:n].bfloat16())
    assert bool((y[:8] == 7).all() and (y[8 + n:] == 7).all())


def test_ce_rows(nat):
    g = torch.Generator(device="cuda").manual_seed(5)
    R, V = 333, 32000
    logits = (torch.randn(R, V, device="cuda", generator=g) * 3).bfloat16()
    tgt = torch.randint(0, V, (R,), device="cuda", generator=g)
    lse = torch.empty(R, device="cuda")
    loss = torch.empty(R, device="cuda")
    nat.ce_fwd_rows(logits, tgt, lse, loss)
    lf = logits.float()
    assert rel_err(loss, F.cross_entropy(lf, tgt, reduction="none")) < 1e-4
    lg = logits.clone()
    nat.ce_bwd_rows(lg, tgt, lse, None, 1.0 / R)
    ref = (torch.softmax(lf, -1) - F.one_hot(tgt, V).float()) / R
    assert rel_err(lg, ref) < 1e-2
