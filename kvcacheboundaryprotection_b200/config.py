"""Decoder architectures used by the capped-KV decode path.

Qwen2-family decoders as the reference's ``TransformerConfig`` describes them
(``src/counterfact_kv_eviction/jax_inference.py:69-133``, ``from_hf_config`` qwen2 branch
at :305-320): GQA attention with a QKV bias (Qwen2) or per-head q/k RMSNorm and no
bias (Qwen3), RoPE over the full head dimension, SwiGLU MLP, RMSNorm with weight ``w``.
"""

from __future__ import annotations

from dataclasses import dataclass, replace
from typing import Dict


@dataclass(frozen=True)
class ModelConfig:
    name: str
    vocab: int
    hidden: int
    n_layers: int
    n_heads: int
    n_kv_heads: int
    ffn: int
    head_dim: int = 128
    rope_theta: float = 1e6
    eps: float = 1e-6
    qkv_bias: bool = True
    qk_norm: bool = False
    tie_embed: bool = False

    @property
    def group(self) -> int:
        return self.n_heads // self.n_kv_heads

    @property
    def qkv_dim(self) -> int:
        return (self.n_heads + 2 * self.n_kv_heads) * self.head_dim

    def param_count(self) -> int:
        h, d = self.hidden, self.head_dim
        per_layer = (
            h * self.qkv_dim
            + (self.qkv_dim if self.qkv_bias else 0)
            + self.n_heads * d * h
            + 3 * h * self.ffn
            + 2 * h
            + (2 * d if self.qk_norm else 0)
        )
        head = 0 if self.tie_embed else self.vocab * h
        return self.vocab * h + head + h + self.n_layers * per_layer

    def with_(self, **kw) -> "ModelConfig":
        return replace(self, **kw)


PRESETS: Dict[str, ModelConfig] = {
    # 4-layer Qwen2-architecture plumbing model (the CPU-runnable parity workload)
    "tiny-qwen2": ModelConfig("tiny-qwen2", 151936, 1024, 4, 8, 2, 2816),
    "qwen2.5-3b": ModelConfig("qwen2.5-3b", 151936, 2048, 36, 16, 2, 11008, tie_embed=True),
    "qwen2.5-7b": ModelConfig("qwen2.5-7b", 152064, 3584, 28, 28, 4, 18944),
    "qwen3-4b": ModelConfig(
        "qwen3-4b", 151936, 2560, 36, 32, 8, 9728, qkv_bias=False, qk_norm=True, tie_embed=True
    ),
    # small shapes for fast parity tests
    "parity-qwen2": ModelConfig("parity-qwen2", 4096, 512, 2, 4, 2, 1024),
    "parity-qwen3": ModelConfig(
        "parity-qwen3", 4096, 512, 2, 8, 2, 768, qkv_bias=False, qk_norm=True, tie_embed=True
    ),
    "parity-g7": ModelConfig("parity-g7", 2048, 896, 2, 7, 1, 1024),
}


def get_config(name: str) -> ModelConfig:
    try:
        return PRESETS[name]
    except KeyError as exc:
        raise ValueError(f"unknown model preset {name!r}; known: {sorted(PRESETS)}") from exc
