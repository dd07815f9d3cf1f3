"""The bf16 noise floor of the forward at the CPU-runnable plumbing configuration
(tiny-qwen2: 4 layers, hidden 1024, vocab 151936, a 1024-token prompt).

Two equally valid restatements with the reference's rounding points -- projections
accumulated in float32 (the oracle) and in float64 -- differ on the step-0 logits by
about 0.027 max-abs (mean 0.0046): 1-2 bf16 ulps per hidden element after four layers
give Gaussian logit deviations whose maximum over 151936 logits sits near 4.5 sigma.
A GPU path is held to that floor, not below it (tests/test_gpu_e2e.py)."""

import numpy as np
import pytest

import oracle.model as om
from kvcacheboundaryprotection_b200.config import get_config
from kvcacheboundaryprotection_b200.weights import init_weights


def test_accumulation_order_alone_moves_logits_past_2e_2(monkeypatch):
    cfg = get_config("tiny-qwen2")
    wn = {k: v.float().numpy() for k, v in init_weights(cfg, seed=0).items()}
    prompt = [int(x) for x in np.random.default_rng(0).integers(0, cfg.vocab, 1024)]
    oc = om.OracleConfig(vocab=cfg.vocab, hidden=cfg.hidden, n_layers=cfg.n_layers, n_heads=cfg.n_heads,
                         n_kv_heads=cfg.n_kv_heads, head_dim=cfg.head_dim, ffn=cfg.ffn, rope_theta=cfg.rope_theta,
                         eps=cfg.eps, qkv_bias=cfg.qkv_bias)

    def logits():
        m = om.OracleModel(oc, wn, max_cache_len=2048)
        return m(input_ids=prompt, past_key_values=None, attention_mask=None, output_attentions=False,
                 use_cache=False).logits[0, -1]

    f32 = logits()
    monkeypatch.setattr(om, "linear", lambda x, w: om.rnd((x.astype(np.float64) @ w.T.astype(np.float64)).astype(np.float32)))
    f64 = logits()
    d = np.abs(f32 - f64)
    assert 2e-2 < d.max() < 5e-2
    assert 2e-3 < d.mean() < 1e-2
    assert np.argmax(f32) == np.argmax(f64) or np.sort(f32)[-1] - np.sort(f32)[-2] <= 2e-2
