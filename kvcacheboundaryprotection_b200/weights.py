"""Seeded random-init decoder weights (no checkpoints are available offline).

Every matrix and bias is drawn N(0, 0.02) in float32 and rounded to bfloat16 (the
reference casts loaded weights to bfloat16, ``jax_inference.py:494,1960``); RMSNorm
weights are ones.  Tensors are drawn in the fixed order of ``weight_names`` from one
``torch.Generator`` seeded with ``seed``, on the device given, so a CPU draw is
reproducible on any host with the same torch version.
"""

from __future__ import annotations

from typing import Dict, List

import torch

from .config import ModelConfig


def weight_names(cfg: ModelConfig) -> List[str]:
    names = ["embed"]
    for i in range(cfg.n_layers):
        names += [f"l{i}.in_norm", f"l{i}.wq", f"l{i}.wk", f"l{i}.wv"]
        if cfg.qkv_bias:
            names += [f"l{i}.bq", f"l{i}.bk", f"l{i}.bv"]
        if cfg.qk_norm:
            names += [f"l{i}.q_norm", f"l{i}.k_norm"]
        names += [f"l{i}.wo", f"l{i}.post_norm", f"l{i}.w_gate", f"l{i}.w_up", f"l{i}.w_down"]
    names.append("final_norm")
    if not cfg.tie_embed:
        names.append("lm_head")
    return names


def weight_shape(cfg: ModelConfig, name: str) -> tuple:
    h, d, f = cfg.hidden, cfg.head_dim, cfg.ffn
    base = name.split(".")[-1]
    return {
        "embed": (cfg.vocab, h),
        "lm_head": (cfg.vocab, h),
        "final_norm": (h,),
        "in_norm": (h,),
        "post_norm": (h,),
        "wq": (cfg.n_heads * d, h),
        "wk": (cfg.n_kv_heads * d, h),
        "wv": (cfg.n_kv_heads * d, h),
        "bq": (cfg.n_heads * d,),
        "bk": (cfg.n_kv_heads * d,),
        "bv": (cfg.n_kv_heads * d,),
        "q_norm": (d,),
        "k_norm": (d,),
        "wo": (h, cfg.n_heads * d),
        "w_gate": (f, h),
        "w_up": (f, h),
        "w_down": (h, f),
    }[base]


def init_weights(cfg: ModelConfig, seed: int = 0, device: str | torch.device = "cpu") -> Dict[str, torch.Tensor]:
    g = torch.Generator(device=device)
    g.manual_seed(int(seed))
    out: Dict[str, torch.Tensor] = {}
    for name in weight_names(cfg):
        shape = weight_shape(cfg, name)
        if name.endswith("norm"):
            out[name] = torch.ones(shape, dtype=torch.bfloat16, device=device)
        else:
            t = torch.randn(shape, generator=g, dtype=torch.float32, device=device)
            out[name] = t.mul_(0.02).to(torch.bfloat16)
            del t
    return out
