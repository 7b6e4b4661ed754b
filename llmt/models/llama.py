"""The plain-PyTorch Llama-style decoder: numerics oracle and parameter-naming tree.

The network is the one the reference trains (bench_train.py:83-228): pre-norm RMSNorm,
one packed qkv projection, rotate-half RoPE on q and k, causal attention, a SwiGLU MLP
(w1 gate, w3 up, w2 down), untied embedding and lm head, N(0, 0.02) weights and unit norm
scales. Two extensions for the Llama-3 shapes: grouped-query attention (`kv_heads`) and a
configurable RoPE base.

Layout of this file: the maths is a set of pure functions over weight tensors
(`rms_norm`, `rope`, `causal_attention`, `swiglu`, `block_forward`, `llama_loss`); the
nn.Module classes exist to own and name the parameters, so that `state_dict()` keys,
shapes and initial values are exactly what the reference's checkpoints hold:

  emb.weight, blocks.{i}.norm1.weight, blocks.{i}.attn.qkv.weight, blocks.{i}.attn.wo.weight,
  blocks.{i}.norm2.weight, blocks.{i}.mlp.w1.weight, blocks.{i}.mlp.w3.weight,
  blocks.{i}.mlp.w2.weight, norm_f.weight, head.weight

The native path (llmt.models.native) reuses these parameters and runs the same maths on
the sm_100a kernels; this file is what it is checked against (fp32 on the CPU, or bf16
autocast on the GPU as the reference-stack baseline).
"""
from __future__ import annotations

import contextlib
import math
from typing import NamedTuple

import torch
import torch.nn as nn
import torch.nn.functional as F
from torch.utils.checkpoint import checkpoint

from llmt.config import ModelConfig


# ---------------------------------------------------------------- pure functions
def rope_tables(T, hd, base, device):
    """Rotation tables for positions 0..T-1, each (T, hd) fp32.

    Column j and column j + hd/2 hold the same angle t * base^(-2j/hd), which is the table
    layout the rotate-half convention (and every native kernel here) indexes."""
    half = hd // 2
    exponent = torch.arange(half, device=device, dtype=torch.float32).mul_(2.0).div_(hd)
    inv_freq = torch.pow(torch.tensor(base, dtype=torch.float32, device=device), exponent).reciprocal_()
    pos = torch.arange(T, device=device, dtype=torch.float32)
    angle = (pos[:, None] * inv_freq[None, :]).repeat(1, 2)
    return torch.cos(angle), torch.sin(angle)


def rope(x, cos, sin):
    """Rotate the two halves of the last dim of x (..., T, hd) by the tables' angles.

    With x = [a | b] and c, s the first half of the tables: [a c - b s | b c + a s].
    Evaluated in fp32; the result has x's dtype."""
    xf = x.float()
    h = xf.shape[-1] // 2
    a, b = xf[..., :h], xf[..., h:]
    c, s = cos[..., :h], sin[..., :h]
    return torch.cat((a * c - b * s, b * c + a * s), dim=-1).to(x.dtype)


# the name the kernel tests use for the oracle rotation
apply_rope = rope


def act_dtype():
    """The autocast dtype in effect (the dtype normalised activations are handed on in), or None."""
    for dev in ("cuda", "cpu"):
        if torch.is_autocast_enabled(dev):
            return torch.get_autocast_dtype(dev)
    return None


def rms_norm(x, weight, eps):
    """y = x / sqrt(mean(x^2) + eps) * weight, computed in fp32. Under autocast the result is
    handed on in the autocast dtype, otherwise in x's dtype."""
    xf = x.float()
    inv_rms = torch.rsqrt(torch.mean(xf * xf, dim=-1, keepdim=True) + eps)
    y = (xf * inv_rms) * weight
    out = act_dtype()
    return y.to(out if out is not None else x.dtype)


def causal_attention(q, k, v, impl="sdpa"):
    """softmax(q k^T / sqrt(hd) + causal mask) v over (B, heads, T, hd); k and v may carry fewer
    heads (grouped-query attention), each shared by heads // kv_heads consecutive query heads."""
    B, H, T, hd = q.shape
    KV = k.shape[1]
    if KV != H:
        k = k[:, :, None].expand(B, KV, H // KV, T, hd).reshape(B, H, T, hd)
        v = v[:, :, None].expand(B, KV, H // KV, T, hd).reshape(B, H, T, hd)
    if impl == "sdpa":
        return F.scaled_dot_product_attention(q, k, v, is_causal=True)
    # "naive": the full (T, T) score matrix, masked above the diagonal, softmax in fp32
    future = torch.triu(torch.full((T, T), True, device=q.device), diagonal=1)
    scores = torch.matmul(q, k.transpose(-1, -2)).mul(1.0 / math.sqrt(hd)).masked_fill(future, float("-inf"))
    return torch.matmul(torch.softmax(scores.float(), dim=-1).to(v.dtype), v)


def attention_forward(cfg: ModelConfig, w_qkv, w_o, x, cos, sin, impl="sdpa"):
    """Packed qkv projection (row blocks q: H*hd, k: KV*hd, v: KV*hd), RoPE on q and k,
    causal attention, heads re-interleaved to (B, T, H*hd), output projection."""
    B, T, _ = x.shape
    H, KV, hd = cfg.H, cfg.kvh, cfg.hd
    q, k, v = F.linear(x, w_qkv).view(B, T, H + 2 * KV, hd).split((H, KV, KV), dim=2)
    q, k, v = (t.permute(0, 2, 1, 3) for t in (q, k, v))
    y = causal_attention(rope(q, cos, sin), rope(k, cos, sin), v, impl)
    return F.linear(y.permute(0, 2, 1, 3).reshape(B, T, H * hd), w_o)


def swiglu(x, w_gate, w_up, w_down):
    """w_down( silu(x w_gate^T) * (x w_up^T) )."""
    return F.linear(F.silu(F.linear(x, w_gate)) * F.linear(x, w_up), w_down)


class BlockWeights(NamedTuple):
    norm1: torch.Tensor
    qkv: torch.Tensor
    wo: torch.Tensor
    norm2: torch.Tensor
    w1: torch.Tensor
    w3: torch.Tensor
    w2: torch.Tensor


def block_forward(cfg: ModelConfig, w: BlockWeights, x, cos, sin, impl="sdpa"):
    """Pre-norm residual block: x + attn(norm1(x)), then + mlp(norm2(.))."""
    x = x + attention_forward(cfg, w.qkv, w.wo, rms_norm(x, w.norm1, cfg.eps), cos, sin, impl)
    return x + swiglu(rms_norm(x, w.norm2, cfg.eps), w.w1, w.w3, w.w2)


def llama_loss(model: "LlamaModel", idx, targets):
    """Mean next-token cross entropy of `model` on idx (B, T) against targets (B, T)."""
    T = idx.shape[1]
    cos, sin = model.rope_cos[:T], model.rope_sin[:T]
    x = F.embedding(idx, model.emb.weight)
    for i, blk in enumerate(model.blocks):
        rng = torch.cuda.nvtx.range(f"block{i}") if model.nvtx else contextlib.nullcontext()
        with rng:
            if model.ckpt and model.training:
                x = checkpoint(blk, x, cos, sin, use_reentrant=False)
            else:
                x = blk(x, cos, sin)
    logits = F.linear(rms_norm(x, model.norm_f.weight, model.cfg.eps), model.head.weight)
    return F.cross_entropy(logits.float().flatten(0, 1), targets.flatten())


# ---------------------------------------------------------------- parameter owners
class RMSNorm(nn.Module):
    """Owns one norm scale (initialised to ones)."""

    def __init__(self, d, eps):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(d))

    def forward(self, x):
        return rms_norm(x, self.weight, self.eps)


class Attention(nn.Module):
    """Owns the packed qkv projection ((H + 2 KV) hd, d) and the output projection (d, H hd)."""

    def __init__(self, cfg: ModelConfig, attn_impl="sdpa"):
        super().__init__()
        self.cfg, self.attn_impl = cfg, attn_impl
        self.qkv = nn.Linear(cfg.d, cfg.qkv_out, bias=False)
        self.wo = nn.Linear(cfg.H * cfg.hd, cfg.d, bias=False)

    def forward(self, x, cos, sin):
        return attention_forward(self.cfg, self.qkv.weight, self.wo.weight, x, cos, sin, self.attn_impl)


class MLP(nn.Module):
    """Owns the SwiGLU projections: w1 (gate) and w3 (up), (ffn, d); w2 (down), (d, ffn)."""

    def __init__(self, cfg: ModelConfig):
        super().__init__()
        self.w1 = nn.Linear(cfg.d, cfg.ffn, bias=False)
        self.w3 = nn.Linear(cfg.d, cfg.ffn, bias=False)
        self.w2 = nn.Linear(cfg.ffn, cfg.d, bias=False)

    def forward(self, x):
        return swiglu(x, self.w1.weight, self.w3.weight, self.w2.weight)


class Block(nn.Module):
    def __init__(self, cfg: ModelConfig, attn_impl="sdpa"):
        super().__init__()
        self.cfg = cfg
        self.norm1 = RMSNorm(cfg.d, cfg.eps)
        self.attn = Attention(cfg, attn_impl)
        self.norm2 = RMSNorm(cfg.d, cfg.eps)
        self.mlp = MLP(cfg)

    def weights(self) -> BlockWeights:
        return BlockWeights(self.norm1.weight, self.attn.qkv.weight, self.attn.wo.weight, self.norm2.weight,
                            self.mlp.w1.weight, self.mlp.w3.weight, self.mlp.w2.weight)

    def forward(self, x, cos, sin):
        return block_forward(self.cfg, self.weights(), x, cos, sin, self.attn.attn_impl)


def init_weights(module: nn.Module, std: float = 0.02):
    """Draw every matrix (projection or embedding) from N(0, std), in parameter order; norm scales
    keep their ones. The draw order is the parameter order, which is the order of the
    reference's own initialiser, so the same seed gives the same weights."""
    with torch.no_grad():
        for name, p in module.named_parameters():
            if p.dim() == 2:
                p.normal_(0.0, std)


class LlamaModel(nn.Module):
    """The decoder; `forward(idx, targets)` returns the mean cross-entropy loss (`llama_loss`)."""

    def __init__(self, cfg: ModelConfig, max_seq: int, attn_impl="sdpa", ckpt=False, nvtx=False):
        super().__init__()
        self.cfg, self.ckpt, self.nvtx, self.max_seq = cfg, ckpt, nvtx, max_seq
        # construction order fixes the parameter order (and the RNG stream the layers consume)
        self.emb = nn.Embedding(cfg.vocab, cfg.d)
        self.blocks = nn.ModuleList(Block(cfg, attn_impl) for _ in range(cfg.L))
        self.norm_f = RMSNorm(cfg.d, cfg.eps)
        self.head = nn.Linear(cfg.d, cfg.vocab, bias=False)
        cos, sin = rope_tables(max_seq, cfg.hd, cfg.rope_base, device="cpu")
        self.register_buffer("rope_cos", cos, persistent=False)
        self.register_buffer("rope_sin", sin, persistent=False)
        init_weights(self)

    def forward(self, idx, targets):
        return llama_loss(self, idx, targets)


def build_model(cfg: ModelConfig, max_seq: int, seed: int = 0, attn_impl="sdpa", ckpt=False, device="cpu"):
    """The model with weights drawn from `seed` (every path starts from the same weights)."""
    torch.manual_seed(seed)
    return LlamaModel(cfg, max_seq, attn_impl=attn_impl, ckpt=ckpt).to(device)


def make_batch(B, T, vocab, device, seed=0):
    """Synthetic data: B rows of T + 1 uniform-random ids from a seeded CPU generator; inputs are
    the first T, targets the last T (next-token prediction)."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    data = torch.randint(0, vocab, (B, T + 1), generator=g)
    return data[:, :-1].contiguous().to(device), data[:, 1:].contiguous().to(device)
