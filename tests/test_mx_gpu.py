"""Block-scaled MXFP8 / NVFP4 kernels against the plain-PyTorch oracle (llmt.ops.lowp_ref).

Like the reference's low-precision tests (kernels/test_lowp.py): the quantizers bit for bit
(round to nearest), stochastic rounding unbiased, the block-scaled GEMM against the fp32 matmul
of the dequantized operands (:78-87), and the model / training with these linears."""
import pytest
import torch

from llmt.ops import lowp_ref as R
from tests.helpers import rel_err

pytestmark = pytest.mark.gpu
MX, NV = 2, 3


@pytest.fixture(scope="module")
def nat():
    from llmt.ops import native
    native.ext()
    return native


def _u8(t):
    return t.contiguous().view(torch.uint8)


def _ref_quant(x, kind):
    """Oracle quantization along the last dim -> (q bytes, chunked scales, g or None, dequantized)."""
    if kind == MX:
        q, s = R.mxfp8_quant_ref(x)
        return q, R.to_chunks(s, kind, x.shape[1]), None, R.mxfp8_dequant(q, s)
    p, s8, g = R.nvfp4_quant_ref(x)
    return p, R.to_chunks(s8.view(torch.uint8), kind, x.shape[1]), g, R.nvfp4_dequant(p, s8, g)


@pytest.mark.parametrize("kind", [MX, NV])
@pytest.mark.parametrize("rows,cols,dtype", [(256, 1024, torch.bfloat16), (640, 768, torch.float32),
                                             (128, 2816, torch.bfloat16), (4096, 1024, torch.bfloat16)])
def test_mx_quant_bit_exact(nat, kind, rows, cols, dtype):
    g = torch.Generator(device="cuda").manual_seed(0)
    x = (torch.randn(rows, cols, device="cuda", generator=g) * 3.0).to(dtype)
    x[0, :64] = 0.0  # an all-zero block
    row, col = nat.mx_quant(x, kind, row=True, col=True)
    q, sf, gg, _ = _ref_quant(x, kind)
    qt, sft, _, _ = _ref_quant(x.t().contiguous(), kind)
    assert torch.equal(_u8(row.q), _u8(q)) and torch.equal(row.sf, sf)
    assert torch.equal(_u8(col.q), _u8(qt)) and torch.equal(col.sf, sft)
    if kind == NV:
        assert torch.equal(row.g, gg) and torch.equal(col.g, gg)


@pytest.mark.parametrize("kind", [MX, NV])
def test_mx_quant_interleaved_rows(nat, kind):
    F, d = 192, 256
    w13 = torch.randn(2 * F, d, device="cuda") * 0.05
    row, _ = nat.mx_quant(w13, kind, interleave64=True)
    order = torch.cat([torch.cat([torch.arange(t * 64, t * 64 + 64), F + torch.arange(t * 64, t * 64 + 64)])
                       for t in range(F // 64)])
    q, sf, _, _ = _ref_quant(w13[order.cuda()].contiguous(), kind)
    assert torch.equal(_u8(row.q), _u8(q)) and torch.equal(row.sf, sf)


def test_nvfp4_stochastic_rounding_unbiased(nat):
    x = torch.randn(128, 256, device="cuda")
    rn, _ = nat.mx_quant(x, NV)
    acc = torch.zeros_like(x)
    n = 64
    for _ in range(n):
        sr, _ = nat.mx_quant(x, NV, stochastic=True)
        acc += _dequant_nv(sr, 256)
    one = _dequant_nv(sr, 256)
    assert rel_err(acc / n, x) < 0.35 * rel_err(one, x)  # averaging draws cancels the rounding error
    assert not torch.equal(sr.q, rn.q)


def _dequant_nv(bq, cols):
    """Dequantize a kernel NVFP4 row operand (scales read back from the chunked layout)."""
    rows = bq.q.shape[0]
    ch = R.chunks_per_tile(NV, cols)
    r = torch.arange(rows, device="cuda")[:, None]
    c = torch.arange(cols // 16, device="cuda")[None, :]
    off = ((r // 128) * ch + c // 4) * 512 + (r % 32) * 16 + ((r % 128) // 32) * 4 + c % 4
    s8 = bq.sf[off.reshape(-1)].view(torch.float8_e4m3fn).view(rows, cols // 16)
    return R.nvfp4_dequant(bq.q, s8, bq.g)


def _operand(nat, x, kind):
    q, sf, g, deq = _ref_quant(x, kind)
    return nat.BlockQ(q, sf, g), deq


@pytest.mark.parametrize("kind", [MX, NV])
@pytest.mark.parametrize("M,N,K", [(128, 128, 256), (300, 264, 512), (4096, 1024, 1024), (1000, 2816, 1024)])
def test_gemm_mx_bf16_out(nat, kind, M, N, K):
    g = torch.Generator(device="cuda").manual_seed(1)
    a, da = _operand(nat, torch.randn(M, K, device="cuda", generator=g), kind)
    b, db = _operand(nat, torch.randn(N, K, device="cuda", generator=g) * 0.05, kind)
    y = nat.gemm_mx(kind, a, b)
    assert rel_err(y, da @ db.t()) < 1e-2
    assert nat.gemm_error_code() == 0


@pytest.mark.parametrize("kind", [MX, NV])
@pytest.mark.parametrize("splits", [0, 1, 3])
def test_gemm_mx_f32_accumulate(nat, kind, splits):
    M, N, K = 1024, 768, 4096
    g = torch.Generator(device="cuda").manual_seed(2)
    a, da = _operand(nat, torch.randn(M, K, device="cuda", generator=g), kind)
    b, db = _operand(nat, torch.randn(N, K, device="cuda", generator=g), kind)
    ref = da @ db.t()
    out = torch.zeros(M, N, device="cuda")
    nat.gemm_mx(kind, a, b, out=out, accumulate=True, splits=splits)
    assert rel_err(out, ref) < 1e-5
    nat.gemm_mx(kind, a, b, out=out, accumulate=True, splits=splits)
    assert rel_err(out, 2 * ref) < 1e-5


@pytest.mark.parametrize("kind", [MX, NV])
def test_gemm_mx_swiglu_epilogues(nat, kind):
    M, d, F = 640, 512, 768
    g = torch.Generator(device="cuda").manual_seed(3)
    x, dx_ = _operand(nat, torch.randn(M, d, device="cuda", generator=g), kind)
    w13 = torch.randn(2 * F, d, device="cuda", generator=g) * 0.05
    w13q, _ = nat.mx_quant(w13, kind, interleave64=True)
    _, _, _, dw13 = _ref_quant(w13, kind)  # row-wise blocks: interleaving moves whole rows
    h, gu = nat.gemm_mx_swiglu(kind, x, w13q, F)
    full = dx_ @ dw13.t()
    gr, ur = full[:, :F], full[:, F:]
    assert rel_err(gu[:, :F], gr) < 1e-2 and rel_err(gu[:, F:], ur) < 1e-2
    assert rel_err(h, torch.nn.functional.silu(gr) * ur) < 1e-2
    dm, ddm = _operand(nat, torch.randn(M, d, device="cuda", generator=g), kind)
    w2t, dw2t = _operand(nat, torch.randn(F, d, device="cuda", generator=g) * 0.05, kind)
    dgu = nat.gemm_mx_swiglu_bwd(kind, dm, w2t, gu, F)
    dh = ddm @ dw2t.t()
    gg, uu = gu[:, :F].float(), gu[:, F:].float()
    sg = torch.sigmoid(gg)
    assert rel_err(dgu[:, :F], dh * uu * sg * (1 + gg * (1 - sg))) < 1e-2
    assert rel_err(dgu[:, F:], dh * gg * sg) < 1e-2


@pytest.mark.parametrize("kind", [MX, NV])
def test_gemm_mx_rope_epilogue(nat, kind):
    from llmt.models.llama import rope_tables
    B, T, H, KV, hd = 2, 192, 4, 2, 64
    g = torch.Generator(device="cuda").manual_seed(5)
    x, dx_ = _operand(nat, torch.randn(B * T, H * hd, device="cuda", generator=g), kind)
    w, dw = _operand(nat, torch.randn((H + 2 * KV) * hd, H * hd, device="cuda", generator=g) * 0.05, kind)
    cos, sin = rope_tables(T, hd, 10000.0, "cuda")
    out = nat.gemm_mx_rope(kind, x, w, cos, sin, T, hd, (H + KV) * hd)
    qkv = (dx_ @ dw.t()).view(B, T, H + 2 * KV, hd)
    rot = qkv[:, :, : H + KV]
    x1, x2 = rot.chunk(2, dim=-1)
    ref = qkv.clone()
    ref[:, :, : H + KV] = rot * cos.view(1, T, 1, hd) + torch.cat([-x2, x1], -1) * sin.view(1, T, 1, hd)
    assert rel_err(out.view(B, T, -1, hd), ref) < 1e-2


@pytest.mark.parametrize("linear,loss_tol,grad_tol", [("mxfp8", 2e-2, 0.25), ("nvfp4", 6e-2, 0.8)])
def test_mx_model_loss_and_grads_near_fp32(linear, loss_tol, grad_tol):
    from llmt.config import get_config
    from llmt.models.llama import build_model, make_batch
    from llmt.models.native import NativeLlama
    from llmt.ops import native
    cfg = get_config("tiny256", ffn=768)
    B, T = 2, 128
    ref = build_model(cfg, T, seed=0, device="cuda")
    ours = build_model(cfg, T, seed=0, device="cuda")
    net = NativeLlama(ours, linear=linear)
    idx, tgt = make_batch(B, T, cfg.vocab, "cuda")
    loss_ref = ref(idx, tgt)
    loss_ref.backward()
    loss = net(idx, tgt)
    loss.backward()
    torch.cuda.synchronize()
    assert native.gemm_error_code() == 0 and native.attn_error_code() == 0
    errs = {n: rel_err(p.main_grad, p_ref.grad) for (n, p_ref), p in zip(ref.named_parameters(), ours.parameters())}
    print(linear, "loss", loss.item(), loss_ref.item(), "grad rel err max", max(errs.values()), max(errs, key=errs.get),
          "median", sorted(errs.values())[len(errs) // 2])
    assert abs(loss.item() - loss_ref.item()) / loss_ref.item() < loss_tol
    for n, e in errs.items():
        assert e < grad_tol, (n, e)


@pytest.mark.parametrize("linear,tol", [("mxfp8", 3e-2), ("nvfp4", 8e-2)])
def test_mx_training_tracks_bf16(linear, tol):
    from llmt.config import get_config
    from llmt.models.llama import make_batch
    from llmt.train import Trainer
    cfg = get_config("tiny256", ffn=768)
    idx, tgt = make_batch(2, 128, cfg.vocab, "cpu")
    bf = Trainer(cfg, 2, 128, cuda_graph=True)
    lp = Trainer(cfg, 2, 128, cuda_graph=True, linear=linear)
    lb = [bf.train_step(idx, tgt) for _ in range(8)]
    ll = [lp.train_step(idx, tgt) for _ in range(8)]
    print(linear, "bf16", lb, "low precision", ll)
    assert ll[-1] < ll[0] - 0.5
    assert max(abs(a - b) / b for a, b in zip(ll, lb)) < tol
    bf.release()
    lp.release()
