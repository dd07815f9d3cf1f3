"""Pins the oracle's forward (oracle/model.py) against an independent implementation of
the same architectures: the Hugging Face ``transformers`` Qwen2 / Qwen3 decoders (eager
attention, float32), loaded with the same weights.

The reference's forward is JAX/XLA (``jax_inference.py:1182-1348``), which cannot run
here.  The oracle restates it with the reference's bfloat16 rounding points.  With those
roundings switched off (``rnd`` -> identity) the oracle must equal transformers' float32
forward to float32 accumulation noise: this checks the wiring -- GQA grouping, RoPE
convention and frequencies, q/k/v bias (Qwen2), per-head q/k RMSNorm (Qwen3), SwiGLU,
residuals, final norm, tied / untied lm_head, causal and decode visibility, and the
per-key attention probabilities the eviction score is built from.  The rounding points
themselves are then the only part not pinned by an independent implementation (they are
read from the reference source, ``jax_inference.py:609-637,949-1050,1089-1107``).
"""

import numpy as np
import pytest
import torch

import oracle.model as om
from kvcacheboundaryprotection_b200.config import get_config
from kvcacheboundaryprotection_b200.weights import init_weights

transformers = pytest.importorskip("transformers")


def _ocfg(cfg):
    return om.OracleConfig(
        vocab=cfg.vocab, hidden=cfg.hidden, n_layers=cfg.n_layers, n_heads=cfg.n_heads, n_kv_heads=cfg.n_kv_heads,
        head_dim=cfg.head_dim, ffn=cfg.ffn, rope_theta=cfg.rope_theta, eps=cfg.eps, qkv_bias=cfg.qkv_bias,
        qk_norm=cfg.qk_norm, tie_embed=cfg.tie_embed,
    )


def _hf_model(cfg, w):
    common = dict(
        vocab_size=cfg.vocab, hidden_size=cfg.hidden, intermediate_size=cfg.ffn, num_hidden_layers=cfg.n_layers,
        num_attention_heads=cfg.n_heads, num_key_value_heads=cfg.n_kv_heads, rms_norm_eps=cfg.eps,
        rope_parameters={"rope_type": "default", "rope_theta": cfg.rope_theta}, max_position_embeddings=4096,
        tie_word_embeddings=cfg.tie_embed, attn_implementation="eager",
    )
    if cfg.qk_norm:
        hcfg = transformers.Qwen3Config(head_dim=cfg.head_dim, attention_bias=cfg.qkv_bias, **common)
        model = transformers.Qwen3ForCausalLM(hcfg)
    else:
        assert cfg.qkv_bias  # Qwen2 attention always carries the q/k/v bias
        hcfg = transformers.Qwen2Config(**common)
        hcfg.head_dim = cfg.head_dim
        model = transformers.Qwen2ForCausalLM(hcfg)
    sd = {"model.embed_tokens.weight": w["embed"], "model.norm.weight": w["final_norm"]}
    if not cfg.tie_embed:
        sd["lm_head.weight"] = w["lm_head"]
    for i in range(cfg.n_layers):
        p, q = f"l{i}.", f"model.layers.{i}."
        sd[q + "input_layernorm.weight"] = w[p + "in_norm"]
        sd[q + "post_attention_layernorm.weight"] = w[p + "post_norm"]
        for a, b in (("wq", "q_proj"), ("wk", "k_proj"), ("wv", "v_proj"), ("wo", "o_proj")):
            sd[q + f"self_attn.{b}.weight"] = w[p + a]
        if cfg.qkv_bias:
            for a, b in (("bq", "q_proj"), ("bk", "k_proj"), ("bv", "v_proj")):
                sd[q + f"self_attn.{b}.bias"] = w[p + a]
        if cfg.qk_norm:
            sd[q + "self_attn.q_norm.weight"] = w[p + "q_norm"]
            sd[q + "self_attn.k_norm.weight"] = w[p + "k_norm"]
        for a, b in (("w_gate", "gate_proj"), ("w_up", "up_proj"), ("w_down", "down_proj")):
            sd[q + f"mlp.{b}.weight"] = w[p + a]
    sd = {k: torch.as_tensor(v, dtype=torch.float32) for k, v in sd.items()}
    missing, unexpected = model.load_state_dict(sd, strict=False)
    assert not unexpected, unexpected
    assert all(k == "lm_head.weight" for k in missing), missing  # tied head only
    return model.float().eval()


@pytest.fixture
def exact_oracle(monkeypatch):
    """The oracle with its bfloat16 rounding points switched off (float32 throughout)."""
    monkeypatch.setattr(om, "rnd", lambda x: np.asarray(x, dtype=np.float32))


@pytest.mark.parametrize("preset", ["parity-qwen2", "parity-qwen3", "parity-g7"])
def test_oracle_forward_matches_transformers_in_float32(preset, exact_oracle):
    cfg = get_config(preset)
    w = {k: v.float().numpy() for k, v in init_weights(cfg, seed=0).items()}
    rng = np.random.default_rng(7)
    P, n_dec = 37, 3
    ids = [int(x) for x in rng.integers(0, cfg.vocab, P + n_dec)]
    hf = _hf_model(cfg, w)
    with torch.no_grad():
        out = hf(input_ids=torch.tensor([ids]), output_attentions=True, use_cache=False)
    hf_logits = out.logits[0].numpy()
    hf_att = [a[0].numpy() for a in out.attentions]  # per layer (Hq, T, T)

    model = om.OracleModel(_ocfg(cfg), w, max_cache_len=512)
    o = model(input_ids=ids[:P], past_key_values=None, attention_mask=None, output_attentions=True, use_cache=True)
    scale = float(np.abs(hf_logits).max())
    tol = 2e-5 * scale + 1e-6
    assert np.abs(o.logits[0, -1] - hf_logits[P - 1]).max() <= tol
    for li in range(cfg.n_layers):  # prefill per-key score: max over heads and query rows
        want = hf_att[li][:, :P, :P].max(axis=(0, 1))
        got = o.attentions[li].reshape(-1)[:P]
        assert np.abs(got - want).max() <= 1e-5
    past = o.past_key_values
    for t in range(n_dec):  # decode steps with every position visible
        mask = [1.0] * (P + t + 1)
        d = model(input_ids=[ids[P + t]], past_key_values=past, attention_mask=mask, output_attentions=True,
                  use_cache=True)
        past = d.past_key_values
        assert np.abs(d.logits[0, -1] - hf_logits[P + t]).max() <= tol
        n = P + t + 1
        for li in range(cfg.n_layers):
            assert np.abs(model.last_probs[li, :, :n] - hf_att[li][:, P + t, :n]).max() <= 1e-5
        want_score = np.max([hf_att[li][:, P + t, :n] for li in range(cfg.n_layers)], axis=(0, 1))
        assert np.abs(d.attentions[0].reshape(-1)[:n] - want_score).max() <= 1e-5


@pytest.mark.parametrize("preset", ["parity-qwen2", "parity-qwen3"])
def test_bf16_rounding_points_stay_within_bf16_noise_of_float32(preset):
    """With its rounding points on, the oracle departs from the float32 forward by bf16
    noise only (a few ulps of the logits' scale), not by a structural difference."""
    cfg = get_config(preset)
    w = {k: v.float().numpy() for k, v in init_weights(cfg, seed=0).items()}
    ids = [int(x) for x in np.random.default_rng(8).integers(0, cfg.vocab, 40)]
    hf = _hf_model(cfg, w)
    with torch.no_grad():
        ref = hf(input_ids=torch.tensor([ids]), use_cache=False).logits[0, -1].numpy()
    got = om.OracleModel(_ocfg(cfg), w, max_cache_len=512)(input_ids=ids, past_key_values=None, attention_mask=None,
                                                          output_attentions=False, use_cache=False).logits[0, -1]
    scale = float(np.abs(ref).max())
    err = np.abs(got - ref)
    assert err.max() <= 0.05 * scale, (err.max(), scale)
    assert np.corrcoef(got, ref)[0, 1] >= 0.995
