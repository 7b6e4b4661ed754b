"""tcgen05 flash attention (fwd + bwd with fused RoPE backward) vs an fp32 PyTorch reference."""
import math

import pytest
import torch

from tests.helpers import rel_err

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def nat():
    from llmt.ops import native
    native.ext()
    return native


def _ref_attention(qkv_raw, cos, sin, B, T, H, KV, hd, causal=True):
    """fp32 reference on the packed pre-RoPE rows: rope(q, k) -> (causal) softmax attention -> (B*T, H*hd)."""
    from llmt.models.llama import apply_rope
    x = qkv_raw.float().view(B, T, H + 2 * KV, hd)
    q = apply_rope(x[:, :, :H].transpose(1, 2), cos, sin)
    k = apply_rope(x[:, :, H:H + KV].transpose(1, 2), cos, sin)
    v = x[:, :, H + KV:].transpose(1, 2)
    rep = H // KV
    k = k.repeat_interleave(rep, 1)
    v = v.repeat_interleave(rep, 1)
    s = (q @ k.transpose(-1, -2)) / math.sqrt(hd)
    if causal:
        mask = torch.ones(T, T, dtype=torch.bool, device=s.device).triu(1)
        s = s.masked_fill(mask, float("-inf"))
    lse = torch.logsumexp(s, -1)
    o = torch.softmax(s, -1) @ v
    return o.transpose(1, 2).reshape(B * T, H * hd), lse


CASES = [(2, 256, 4, 4, 64), (1, 384, 4, 2, 128), (2, 200, 4, 4, 64), (1, 1024, 2, 1, 64)]


@pytest.mark.parametrize("B,T,H,KV,hd", CASES)
def test_flash_fwd_bwd(nat, B, T, H, KV, hd):
    from llmt.models.llama import rope_tables
    g = torch.Generator(device="cuda").manual_seed(0)
    qkv_raw = torch.randn(B * T, (H + 2 * KV) * hd, device="cuda", generator=g).bfloat16()
    cos, sin = rope_tables(T, hd, 10000.0, "cuda")
    qkv = nat.rope_inplace(qkv_raw.clone(), cos, sin, T, H + KV, hd)
    o, lse = nat.flash_attn_fwd(qkv, B, T, H, KV, hd)
    torch.cuda.synchronize()
    assert nat.attn_error_code() == 0
    x = qkv_raw.float().clone().requires_grad_(True)
    o_ref, lse_ref = _ref_attention(x, cos, sin, B, T, H, KV, hd)
    assert rel_err(o, o_ref) < 2e-2
    assert rel_err(lse, lse_ref) < 1e-3
    do = torch.randn(B * T, H * hd, device="cuda", generator=g).bfloat16()
    o_ref.backward(do.float())
    dqkv = nat.flash_attn_bwd(do, qkv, o, lse, cos, sin, B, T, H, KV, hd)
    torch.cuda.synchronize()
    assert nat.attn_error_code() == 0
    ref = x.grad.view(B * T, H + 2 * KV, hd)
    got = dqkv.view(B * T, H + 2 * KV, hd)
    assert rel_err(got[:, :H], ref[:, :H]) < 3e-2, "dq"
    assert rel_err(got[:, H:H + KV], ref[:, H:H + KV]) < 3e-2, "dk"
    assert rel_err(got[:, H + KV:], ref[:, H + KV:]) < 3e-2, "dv"


# Forward at the model shapes, causal and not, with scores scaled up (amp) so that the running
# max moves often and the in-TMEM rescale of O is exercised.
@pytest.mark.parametrize("B,T,H,KV,hd", [(4, 1024, 16, 16, 64), (1, 2048, 8, 2, 128), (2, 640, 4, 4, 64)])
@pytest.mark.parametrize("causal", [True, False])
@pytest.mark.parametrize("amp", [1.0, 4.0])
def test_flash_fwd_shapes(nat, B, T, H, KV, hd, causal, amp):
    from llmt.models.llama import rope_tables
    g = torch.Generator(device="cuda").manual_seed(1)
    qkv_raw = (amp * torch.randn(B * T, (H + 2 * KV) * hd, device="cuda", generator=g)).bfloat16()
    cos, sin = rope_tables(T, hd, 10000.0, "cuda")
    qkv = nat.rope_inplace(qkv_raw.clone(), cos, sin, T, H + KV, hd)
    o, lse = nat.flash_attn_fwd(qkv, B, T, H, KV, hd, causal=causal)
    torch.cuda.synchronize()
    assert nat.attn_error_code() == 0
    o_ref, lse_ref = _ref_attention(qkv_raw.float(), cos, sin, B, T, H, KV, hd, causal=causal)
    assert rel_err(o, o_ref) < 2e-2
    assert rel_err(lse, lse_ref) < 1e-3
