"""tcgen05 GEMM numerics against an fp32 PyTorch reference of the same op (bf16 inputs)."""
import pytest
import torch

from tests.helpers import rel_err

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def nat():
    from llmt.ops import native
    native.ext()
    return native


# M, N, K: ragged M/K, N a multiple of 8; every row pitch a multiple of 16 bytes.
SHAPES = [(128, 128, 64), (300, 264, 200), (4096, 1024, 1024), (1000, 2816, 1024), (520, 768, 2048)]
# wgrad: (M=out, N=in, K=tokens); its operands are (K, M) and (K, N), so M and N are multiples of 8.
WSHAPES = [(128, 128, 64), (304, 264, 200), (1024, 1024, 4096), (2816, 1024, 1000), (768, 2048, 520)]


@pytest.mark.parametrize("bn", [128, 256])
@pytest.mark.parametrize("M,N,K", SHAPES)
def test_gemm_fwd_nt(nat, M, N, K, bn):
    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    w = torch.randn(N, K, device="cuda", generator=g).bfloat16()
    y = nat.gemm(x, w, ta=False, tb=True, bn=bn)
    ref = x.float() @ w.float().t()
    assert rel_err(y, ref) < 1e-2
    assert nat.gemm_error_code() == 0


@pytest.mark.parametrize("bn", [128, 256])
@pytest.mark.parametrize("M,N,K", SHAPES)
def test_gemm_dgrad_nn(nat, M, N, K, bn):
    g = torch.Generator(device="cuda").manual_seed(1)
    dy = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    w = torch.randn(K, N, device="cuda", generator=g).bfloat16()
    dx = nat.gemm(dy, w, ta=False, tb=False, bn=bn)
    assert rel_err(dx, dy.float() @ w.float()) < 1e-2


@pytest.mark.parametrize("bn", [128, 256])
@pytest.mark.parametrize("M,N,K", WSHAPES)
def test_gemm_wgrad_tn_fp32_accumulate(nat, M, N, K, bn):
    g = torch.Generator(device="cuda").manual_seed(2)
    dy = torch.randn(K, M, device="cuda", generator=g).bfloat16()
    x = torch.randn(K, N, device="cuda", generator=g).bfloat16()
    ref = dy.float().t() @ x.float()
    out = torch.empty(M, N, device="cuda", dtype=torch.float32)
    nat.gemm(dy, x, ta=True, tb=False, out=out, bn=bn)
    assert rel_err(out, ref) < 1e-4
    nat.gemm(dy, x, ta=True, tb=False, out=out, accumulate=True, bn=bn)
    assert rel_err(out, 2 * ref) < 1e-4


def test_gemm_rejects_unaligned_pitch(nat):
    dy = torch.randn(200, 300, device="cuda").bfloat16()   # 600-byte rows: not a TMA pitch
    x = torch.randn(200, 264, device="cuda").bfloat16()
    with pytest.raises(ValueError):
        nat.gemm(dy, x, ta=True, tb=False, out_dtype=torch.float32)


def test_gemm_swiglu_epilogue(nat):
    M, d, F = 777, 512, 688
    g = torch.Generator(device="cuda").manual_seed(3)
    x = torch.randn(M, d, device="cuda", generator=g).bfloat16()
    w13 = (torch.randn(2 * F, d, device="cuda", generator=g) * 0.05).bfloat16()
    for bn in (128, 256):
        h, gu = nat.gemm_swiglu(x, w13, F, bn=bn)
        gr = x.float() @ w13[:F].float().t()
        ur = x.float() @ w13[F:].float().t()
        assert rel_err(gu[:, :F], gr) < 1e-2
        assert rel_err(gu[:, F:], ur) < 1e-2
        assert rel_err(h, torch.nn.functional.silu(gr) * ur) < 1e-2


def test_gemm_swiglu_bwd_epilogue(nat):
    M, d, F = 640, 256, 688
    g = torch.Generator(device="cuda").manual_seed(4)
    dm = torch.randn(M, d, device="cuda", generator=g).bfloat16()
    w2 = (torch.randn(d, F, device="cuda", generator=g) * 0.05).bfloat16()
    gu = torch.randn(M, 2 * F, device="cuda", generator=g).bfloat16()
    dgu = nat.gemm_swiglu_bwd(dm, w2, gu, F)
    dh = dm.float() @ w2.float()
    gg, uu = gu[:, :F].float(), gu[:, F:].float()
    sg = torch.sigmoid(gg)
    assert rel_err(dgu[:, :F], dh * uu * sg * (1 + gg * (1 - sg))) < 1e-2
    assert rel_err(dgu[:, F:], dh * gg * sg) < 1e-2


@pytest.mark.parametrize("hd,H,KV", [(64, 4, 4), (128, 8, 2)])
def test_gemm_rope_epilogue(nat, hd, H, KV):
    from llmt.models.llama import rope_tables
    B, T = 2, 192
    d = H * hd
    g = torch.Generator(device="cuda").manual_seed(5)
    x = torch.randn(B * T, d, device="cuda", generator=g).bfloat16()
    w = (torch.randn((H + 2 * KV) * hd, d, device="cuda", generator=g) * 0.05).bfloat16()
    cos, sin = rope_tables(T, hd, 10000.0, "cuda")
    out = nat.gemm_rope(x, w, cos, sin, T, hd, (H + KV) * hd)
    qkv = (x.float() @ w.float().t()).view(B, T, H + 2 * KV, hd)
    rot = qkv[:, :, : H + KV]
    x1, x2 = rot.chunk(2, dim=-1)
    c = cos.view(1, T, 1, hd)
    s = sin.view(1, T, 1, hd)
    ref = qkv.clone()
    ref[:, :, : H + KV] = rot * c + torch.cat([-x2, x1], -1) * s
    assert rel_err(out.view(B, T, -1, hd), ref) < 1e-2


def test_gemm_ce_epilogues(nat):
    M, d, V = 600, 256, 32000
    g = torch.Generator(device="cuda").manual_seed(6)
    h = torch.randn(M, d, device="cuda", generator=g).bfloat16()
    w = (torch.randn(V, d, device="cuda", generator=g) * 0.05).bfloat16()
    tgt = torch.randint(0, V, (M,), device="cuda", generator=g)
    lse, loss = nat.gemm_ce_fwd(h, w, tgt)
    logits = h.float() @ w.float().t()
    assert rel_err(lse, torch.logsumexp(logits, -1)) < 1e-4
    ref_loss = torch.nn.functional.cross_entropy(logits, tgt, reduction="none")
    assert rel_err(loss, ref_loss) < 1e-3
    go = torch.full((1,), 2.0, device="cuda")
    dl = nat.gemm_ce_bwd(h, w, tgt, lse, go, 1.0 / M)
    ref_dl = (torch.softmax(logits, -1) - torch.nn.functional.one_hot(tgt, V).float()) * 2.0 / M
    assert rel_err(dl, ref_dl) < 1e-2
