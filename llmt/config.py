"""Model and run configuration.

Model shapes follow the reference's registries (bench_train.py:49-69 `ModelConfig`/`SIZES`,
perf_model/roofline.py:48-85 `Shape`/`SIZES` with the Llama-3 GQA shapes), plus the
`tiny256` CPU oracle shape of the benchmark contract (d256, 4 layers, 4 heads, ffn 688).
"""
from __future__ import annotations

from dataclasses import asdict, dataclass, replace

VOCAB = 32000


@dataclass(frozen=True)
class ModelConfig:
    d: int
    L: int
    H: int
    ffn: int
    vocab: int = VOCAB
    eps: float = 1e-5
    rope_base: float = 10000.0
    kv_heads: int | None = None   # grouped-query attention; None means kv_heads == H
    head_dim: int | None = None   # None means d // H (set for tensor-parallel shards, where H is local)

    @property
    def hd(self) -> int:
        return self.head_dim or self.d // self.H

    @property
    def kvh(self) -> int:
        return self.kv_heads or self.H

    @property
    def qkv_out(self) -> int:
        """Rows of the packed qkv weight: H*hd query rows, then KV*hd key rows, then KV*hd value rows."""
        return (self.H + 2 * self.kvh) * self.hd

    def to_dict(self):
        return asdict(self)


SIZES = {
    "tiny256": ModelConfig(d=256, L=4, H=4, ffn=688),
    "tiny": ModelConfig(d=512, L=8, H=8, ffn=1408),
    "small": ModelConfig(d=768, L=12, H=12, ffn=2048),
    "medium": ModelConfig(d=1024, L=24, H=16, ffn=2816),
    "large": ModelConfig(d=2048, L=16, H=16, ffn=5504),
    "llama3-8b": ModelConfig(d=4096, L=32, H=32, ffn=14336, vocab=128256, rope_base=500000.0, kv_heads=8),
    "llama3-70b": ModelConfig(d=8192, L=80, H=64, ffn=28672, vocab=128256, rope_base=500000.0, kv_heads=8),
}


def get_config(name: str, **overrides) -> ModelConfig:
    cfg = SIZES[name]
    return replace(cfg, **overrides) if overrides else cfg


def count_params(cfg: ModelConfig):
    """Total parameters and matmul parameters (all but the embedding table).

    Same definition as the reference (bench_train.py:290-294), extended to GQA."""
    qkv = cfg.d * cfg.qkv_out
    per_block = qkv + cfg.H * cfg.hd * cfg.d + 3 * cfg.d * cfg.ffn + 2 * cfg.d
    total = cfg.L * per_block + cfg.d + 2 * cfg.vocab * cfg.d
    return total, total - cfg.vocab * cfg.d


def model_flops_per_token(cfg: ModelConfig, seq: int) -> int:
    """6 x matmul params + 12 x L x d x seq (reference bench_train.py:297-300). Recompute is not counted."""
    _, n_matmul = count_params(cfg)
    return 6 * n_matmul + 12 * cfg.L * cfg.d * seq
