"""Llama-style decoder with the reference's module tree and state_dict layout.

Same network as the reference (bench_train.py:83-228): pre-norm RMSNorm, packed qkv
projection, rotate-half RoPE, causal attention, SwiGLU MLP (w1 gate, w3 up, w2 down),
untied embedding and lm head, N(0, 0.02) init of every Linear/Embedding, RMSNorm weights
ones, non-persistent rope tables. Extended with grouped-query attention (kv_heads) and a
configurable RoPE theta for the Llama-3 shapes.

state_dict keys (identical to the reference):
  emb.weight, blocks.{i}.norm1.weight, blocks.{i}.attn.qkv.weight, blocks.{i}.attn.wo.weight,
  blocks.{i}.norm2.weight, blocks.{i}.mlp.w1.weight, blocks.{i}.mlp.w3.weight,
  blocks.{i}.mlp.w2.weight, norm_f.weight, head.weight

Two execution paths share these parameters:
  plain PyTorch (this file): fp32 or bf16 autocast, naive or SDPA attention -- the numerics
      oracle and the reference-stack baseline;
  native (llmt.models.native): every op on the sm_100a kernels of llmt._C with the
      parameters packed into flat buffers -- the framework's training path.
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn
import torch.nn.functional as F
from torch.utils.checkpoint import checkpoint

from llmt.config import ModelConfig


def rope_tables(T, hd, base, device):
    """cos and sin tables (T, hd) fp32, halves duplicated (rotate-half layout)."""
    inv = 1.0 / (base ** (torch.arange(0, hd, 2, device=device, dtype=torch.float32) / hd))
    t = torch.arange(T, device=device, dtype=torch.float32)
    freqs = torch.outer(t, inv)
    emb = torch.cat([freqs, freqs], dim=-1)
    return emb.cos(), emb.sin()


def rotate_half(x):
    x1, x2 = x.chunk(2, dim=-1)
    return torch.cat([-x2, x1], dim=-1)


def apply_rope(x, cos, sin):
    """x (B, H, T, hd); math in fp32, result in x's dtype."""
    xf = x.float()
    return (xf * cos + rotate_half(xf) * sin).to(x.dtype)


def act_dtype():
    for dev in ("cuda", "cpu"):
        if torch.is_autocast_enabled(dev):
            return torch.get_autocast_dtype(dev)
    return None


class RMSNorm(nn.Module):
    def __init__(self, d, eps):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(d))

    def forward(self, x):
        xf = x.float()
        y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.eps) * self.weight
        dt = act_dtype()
        return y.to(dt) if dt is not None else y.to(x.dtype)


class Attention(nn.Module):
    def __init__(self, cfg: ModelConfig, attn_impl="sdpa"):
        super().__init__()
        self.cfg = cfg
        self.attn_impl = attn_impl
        self.qkv = nn.Linear(cfg.d, cfg.qkv_out, bias=False)   # rows: (H | KV | KV) x hd
        self.wo = nn.Linear(cfg.H * cfg.hd, cfg.d, bias=False)

    def forward(self, x, cos, sin):
        B, T, _ = x.shape
        H, KV, hd = self.cfg.H, self.cfg.kvh, self.cfg.hd
        qkv = self.qkv(x).view(B, T, H + 2 * KV, hd)
        q = qkv[:, :, :H].transpose(1, 2)
        k = qkv[:, :, H:H + KV].transpose(1, 2)
        v = qkv[:, :, H + KV:].transpose(1, 2)
        q = apply_rope(q, cos, sin)
        k = apply_rope(k, cos, sin)
        if KV != H:
            rep = H // KV
            k = k.repeat_interleave(rep, dim=1)
            v = v.repeat_interleave(rep, dim=1)
        if self.attn_impl == "sdpa":
            y = F.scaled_dot_product_attention(q, k, v, is_causal=True)
        else:
            scores = (q @ k.transpose(-2, -1)) * (1.0 / math.sqrt(hd))
            mask = torch.ones(T, T, dtype=torch.bool, device=x.device).triu(1)
            scores = scores.masked_fill(mask, float("-inf"))
            probs = torch.softmax(scores.float(), dim=-1).to(v.dtype)
            y = probs @ v
        y = y.transpose(1, 2).reshape(B, T, H * hd)
        return self.wo(y)


class MLP(nn.Module):
    def __init__(self, cfg: ModelConfig):
        super().__init__()
        self.w1 = nn.Linear(cfg.d, cfg.ffn, bias=False)
        self.w3 = nn.Linear(cfg.d, cfg.ffn, bias=False)
        self.w2 = nn.Linear(cfg.ffn, cfg.d, bias=False)

    def forward(self, x):
        return self.w2(F.silu(self.w1(x)) * self.w3(x))


class Block(nn.Module):
    def __init__(self, cfg: ModelConfig, attn_impl="sdpa"):
        super().__init__()
        self.norm1 = RMSNorm(cfg.d, cfg.eps)
        self.attn = Attention(cfg, attn_impl)
        self.norm2 = RMSNorm(cfg.d, cfg.eps)
        self.mlp = MLP(cfg)

    def forward(self, x, cos, sin):
        x = x + self.attn(self.norm1(x), cos, sin)
        return x + self.mlp(self.norm2(x))


class LlamaModel(nn.Module):
    """The reference network. `forward(idx, targets)` returns the mean cross-entropy loss."""

    def __init__(self, cfg: ModelConfig, max_seq: int, attn_impl="sdpa", ckpt=False, nvtx=False):
        super().__init__()
        self.cfg = cfg
        self.ckpt = ckpt
        self.nvtx = nvtx
        self.max_seq = max_seq
        self.emb = nn.Embedding(cfg.vocab, cfg.d)
        self.blocks = nn.ModuleList([Block(cfg, attn_impl) for _ in range(cfg.L)])
        self.norm_f = RMSNorm(cfg.d, cfg.eps)
        self.head = nn.Linear(cfg.d, cfg.vocab, bias=False)
        cos, sin = rope_tables(max_seq, cfg.hd, cfg.rope_base, device="cpu")
        self.register_buffer("rope_cos", cos, persistent=False)
        self.register_buffer("rope_sin", sin, persistent=False)
        self.apply(self._init)

    @staticmethod
    def _init(m):
        if isinstance(m, (nn.Linear, nn.Embedding)):
            nn.init.normal_(m.weight, mean=0.0, std=0.02)

    def forward(self, idx, targets):
        B, T = idx.shape
        cos, sin = self.rope_cos[:T], self.rope_sin[:T]
        x = self.emb(idx)
        for i, blk in enumerate(self.blocks):
            if self.nvtx:
                torch.cuda.nvtx.range_push(f"block{i}")
            if self.ckpt and self.training:
                x = checkpoint(blk, x, cos, sin, use_reentrant=False)
            else:
                x = blk(x, cos, sin)
            if self.nvtx:
                torch.cuda.nvtx.range_pop()
        logits = self.head(self.norm_f(x))
        return F.cross_entropy(logits.float().view(-1, self.cfg.vocab), targets.reshape(-1))


def build_model(cfg: ModelConfig, max_seq: int, seed: int = 0, attn_impl="sdpa", ckpt=False, device="cpu"):
    """Seeded construction (same initial weights on every path, as the reference's build does)."""
    torch.manual_seed(seed)
    m = LlamaModel(cfg, max_seq, attn_impl=attn_impl, ckpt=ckpt)
    return m.to(device)


def make_batch(B, T, vocab, device, seed=0):
    """Uniform-random token ids from a seeded CPU generator; inputs and next-token targets."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    data = torch.randint(0, vocab, (B, T + 1), generator=g)
    return data[:, :-1].contiguous().to(device), data[:, 1:].contiguous().to(device)
