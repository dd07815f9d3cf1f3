"""Generate the golden fixtures under tests/golden/ by running the REFERENCE's own code.

Run in a container where the reference project is readable (default path below, or
``--ref DIR``); the fixtures it writes are committed so the tests never need the
reference at run time.  It imports, unmodified:

* ``counterfact_kv_eviction.policies`` (LRUPolicy, H2OFaithfulPolicy, ...),
* ``counterfact_kv_eviction.kv_coupled_generator.KVCoupledQwen35Generator``,
* ``ProtectedPolicyWrapper`` from ``scripts/run_v3_jax.py`` (its module body only
  defines helpers; ``main()`` is not run).

Fixtures:

* ``policy_kats.json``   -- victim lists of every global CLI policy, with and without
  the protection wrapper, on seeded metadata with many ties.
* ``generator_kats.json`` -- full decode/eviction traces of the reference generator
  driven by ``oracle.stub_model.StubScoreModel``.
* ``e2e_parity_qwen2.json`` -- the reference generator driven by the numpy forward
  (``oracle.model``) on the small ``parity-qwen2`` decoder, greedy, with per-step
  logit summaries (used by the GPU parity test).
* ``e2e_tiny_qwen2_lru.json`` -- the same at the CPU-runnable plumbing configuration:
  the 4-layer ``tiny-qwen2`` decoder (hidden 1024, 8/2 heads, vocab 151936), a
  1024-token prompt, LRU, capacity 256, max-cache-len 2048, protect-frac 0.10,
  evict-every 8, 128 greedy tokens.

Usage:  python tests/golden/make_golden.py --ref REFERENCE_DIR [--only NAME]
        (or set KVBP_REFERENCE to the reference project's directory)
"""

from __future__ import annotations

import argparse
import importlib.util
import json
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO))


def _load_reference(ref: Path):
    sys.path.insert(0, str(ref / "src"))
    from counterfact_kv_eviction import policies as P  # noqa: E402
    from counterfact_kv_eviction.interfaces import KVBlockMetadata  # noqa: E402
    from counterfact_kv_eviction.kv_coupled_generator import KVCoupledQwen35Generator  # noqa: E402

    spec = importlib.util.spec_from_file_location("_ref_run_v3_jax", ref / "scripts" / "run_v3_jax.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return P, KVBlockMetadata, KVCoupledQwen35Generator, mod.ProtectedPolicyWrapper


def _policy_factory(P, name: str, capacity: int):
    return {
        "lru": lambda: P.LRUPolicy(),
        "h2o_faithful": lambda: P.H2OFaithfulPolicy(),
        "h2o": lambda: P.HeavyHitterH2OLikePolicy(),
        "snapkv": lambda: P.SnapKVPolicy(),
        "snapkv_faithful": lambda: P.SnapKVFaithfulPolicy(),
        "adakv": lambda: P.AdaKVPolicy(),
        "quest": lambda: P.QUESTPolicy(),
        "streamingllm": lambda: P.StreamingSinkLikePolicy(sink_size=4, recent_window_size=max(0, capacity - 4)),
        "random": lambda: P.RandomEvictionPolicy(),
        "adakv_faithful": lambda: P.AdaKVFaithfulPolicy(),
        "adakv_native": lambda: P.AdaKVNativePolicy(),
        "quest_faithful": lambda: P.QUESTFaithfulPolicy(),
        "quest_native": lambda: P.QUESTNativePolicy(),
    }[name]()


POLICIES = ["lru", "h2o_faithful", "h2o", "snapkv", "snapkv_faithful", "adakv", "quest", "streamingllm", "random"]


def _rand_meta(rng, n_pos_max: int, n_live: int, step: int, tie_level: int):
    """Metadata for ``n_live`` retained positions drawn from [0, n_pos_max)."""
    live = np.sort(rng.choice(n_pos_max, size=n_live, replace=False))
    if tie_level == 0:  # prefill-like: everything ties
        last = np.zeros(n_live, np.int32)
        ins = np.zeros(n_live, np.int32)
        attn = np.zeros(n_live, np.float32)
        cumul = np.zeros(n_live, np.float64)
    else:
        last = rng.integers(0, max(1, step // tie_level + 1), n_live).astype(np.int32) * tie_level
        last = np.minimum(last, step).astype(np.int32)
        ins = np.minimum(rng.integers(0, 3, n_live) * (step // 3), last).astype(np.int32)
        vals = rng.random(8).astype(np.float32)
        attn = vals[rng.integers(0, 8, n_live)] if tie_level > 2 else rng.random(n_live).astype(np.float32)
        cvals = rng.random(6) * 3.0
        cumul = cvals[rng.integers(0, 6, n_live)] if tie_level > 2 else rng.random(n_live) * 3.0
    maxa = np.maximum(attn, (rng.random(n_live) * 0.5).astype(np.float32)).astype(np.float32)
    pre = (rng.random(n_live) ** 2).astype(np.float32)
    cnt = rng.integers(1, 9, n_live).astype(np.int32)
    return live, ins, last, cnt, attn.astype(np.float32), maxa, cumul.astype(np.float64), pre


def make_policy_kats(ref: Path) -> dict:
    P, KVBlockMetadata, _, Wrapper = _load_reference(ref)
    rng = np.random.default_rng(20240501)
    cases = []
    shapes = [
        # (n_pos_max, n_live, capacity, evict_count, step)
        (300, 264, 256, 8, 136),
        (1100, 1024, 256, 768, 0),
        (140, 40, 32, 8, 48),
        (70, 30, 24, 6, 16),
        (2000, 1031, 1024, 8, 200),
        (90, 20, 16, 30, 24),  # evict_count beyond the eligible set
        (50, 12, 8, 0, 8),  # zero evictions
        (130, 100, 4, 96, 0),  # tiny capacity: protection sizes clamp to 4
    ]
    for ci, (nmax, nlive, cap, k, step) in enumerate(shapes):
        for tie in (0, 1, 4):
            live, ins, last, cnt, attn, maxa, cumul, pre = _rand_meta(rng, nmax, nlive, step, tie)
            blocks = {}
            for j, p in enumerate(live):
                blocks[str(int(p))] = KVBlockMetadata(
                    key=str(int(p)),
                    last_access_step=int(last[j]),
                    insert_step=int(ins[j]),
                    access_count=int(cnt[j]),
                    attention_score=float(attn[j]),
                    max_attention_score=float(maxa[j]),
                    cumulative_attention_score=float(cumul[j]),
                    prefill_attention_score=float(pre[j]),
                )
            results = []
            for pol in POLICIES:
                for wrap in ((None, None), (0.10, 0.10), (0.05, 0.05), (0.10, 0.0), (0.0, 0.10)):
                    inner = _policy_factory(P, pol, cap)
                    if wrap[0] is None:
                        policy = inner
                    else:
                        policy = Wrapper(inner, prefix_frac=wrap[0], suffix_frac=wrap[1], capacity=cap)
                    got = policy.select_evictions(dict(blocks), k, step)
                    results.append(
                        {
                            "policy": pol,
                            "protect": wrap[0] is not None,
                            "prefix_frac": wrap[0] if wrap[0] is not None else 0.0,
                            "suffix_frac": wrap[1] if wrap[1] is not None else 0.0,
                            "victims": [int(v) for v in got],
                        }
                    )
            cases.append(
                {
                    "case": ci,
                    "tie": tie,
                    "capacity": cap,
                    "evict_count": k,
                    "step": step,
                    "positions": [int(x) for x in live],
                    "insert_step": [int(x) for x in ins],
                    "last_access": [int(x) for x in last],
                    "access_count": [int(x) for x in cnt],
                    "attn": [float(x) for x in attn],
                    "max_attn": [float(x) for x in maxa],
                    "cumul": [float(x) for x in cumul],
                    "prefill": [float(x) for x in pre],
                    "results": results,
                }
            )
    return {"source": "reference policies.py + run_v3_jax.ProtectedPolicyWrapper", "cases": cases}


GEN_CASES = [
    # name, policy, prompt, capacity, E, max_new, protect (pf, sf) or None, n_kv_heads, regime, seed
    ("lru_p300_c64", "lru", 300, 64, 8, 40, (0.10, 0.10), 2, "decode", 1),
    ("h2of_p300_c64", "h2o_faithful", 300, 64, 8, 40, (0.10, 0.10), 2, "decode", 2),
    ("h2of_noprot", "h2o_faithful", 200, 48, 8, 33, None, 2, "decode", 3),
    ("lru_e1", "lru", 120, 40, 1, 25, (0.10, 0.10), 2, "decode", 4),
    ("lru_short_prompt", "lru", 20, 32, 8, 40, (0.10, 0.10), 2, "decode", 5),
    ("h2o_like", "h2o", 160, 40, 4, 30, (0.05, 0.05), 2, "decode", 6),
    ("snapkv", "snapkv", 160, 40, 8, 30, (0.10, 0.10), 2, "decode", 7),
    ("snapkv_faithful", "snapkv_faithful", 160, 40, 8, 30, (0.10, 0.10), 0, "decode", 8),
    ("adakv", "adakv", 160, 40, 8, 30, (0.10, 0.10), 2, "decode", 9),
    ("quest", "quest", 160, 40, 8, 30, (0.10, 0.10), 2, "decode", 10),
    ("streamingllm", "streamingllm", 160, 40, 8, 30, (0.10, 0.10), 2, "decode", 11),
    ("suffix_zero_hardcap", "lru", 150, 40, 8, 30, (0.10, 0.0), 2, "decode", 12),
    ("tiny_cap_hardcap", "h2o_faithful", 60, 6, 8, 30, (0.10, 0.10), 2, "decode", 13),
    ("prefill_regime", "lru", 120, 40, 8, 20, (0.10, 0.10), 2, "prefill", 14),
    ("lru_1024_256", "lru", 1024, 256, 8, 128, (0.10, 0.10), 2, "decode", 15),
    ("h2of_1024_256", "h2o_faithful", 1024, 256, 8, 128, (0.10, 0.10), 2, "decode", 16),
    ("random_p160_c40", "random", 160, 40, 8, 30, (0.10, 0.10), 2, "decode", 17),
    ("random_noprot_e4", "random", 120, 40, 4, 25, None, 2, "decode", 18),
    ("random_tiny_cap_hardcap", "random", 60, 6, 8, 30, (0.10, 0.10), 2, "decode", 19),
    ("random_1024_256", "random", 1024, 256, 8, 64, (0.10, 0.10), 2, "decode", 20),
    # per-KV-head policies (n_kv_heads > 0 selects the generator's per-head mode)
    ("adakv_faithful", "adakv_faithful", 160, 40, 8, 30, (0.10, 0.10), 2, "decode", 21),
    ("adakv_native", "adakv_native", 160, 40, 8, 30, (0.10, 0.10), 2, "decode", 22),
    ("quest_faithful", "quest_faithful", 160, 40, 8, 30, (0.10, 0.10), 2, "decode", 23),
    ("quest_native", "quest_native", 160, 40, 8, 30, (0.10, 0.10), 2, "decode", 24),
    ("adakv_faithful_noprot", "adakv_faithful", 120, 32, 4, 25, None, 2, "decode", 25),
    ("quest_faithful_e1_short_prompt", "quest_faithful", 30, 40, 1, 20, (0.10, 0.10), 2, "decode", 26),
    ("adakv_faithful_1024_256", "adakv_faithful", 1024, 256, 8, 64, (0.10, 0.10), 2, "decode", 27),
    ("quest_faithful_prefill_regime", "quest_faithful", 120, 40, 8, 20, (0.10, 0.10), 2, "prefill", 28),
    ("adakv_native_tight", "adakv_native", 200, 24, 8, 40, (0.05, 0.05), 2, "decode", 29),
]


def make_generator_kats(ref: Path) -> dict:
    from oracle.stub_model import StubScoreModel

    P, _, Gen, Wrapper = _load_reference(ref)
    out = []
    for name, pol, n_prompt, cap, E, max_new, prot, n_kv, regime, seed in GEN_CASES:
        model = StubScoreModel(vocab=97, n_heads=4, n_kv_heads=2, n_layers=2, max_cache_len=n_prompt + max_new + 8, seed=seed)
        inner = _policy_factory(P, pol, cap)
        policy = inner if prot is None else Wrapper(inner, prefix_frac=prot[0], suffix_frac=prot[1], capacity=cap)
        gen = Gen(model=model, tokenizer=None, policy=policy, capacity=cap, evict_every_n_steps=E, n_kv_heads=n_kv, eviction_regime=regime)
        prompt = [int(x) for x in np.random.default_rng(seed).integers(0, 97, n_prompt)]
        res = gen.generate_with_kv_control(input_ids=prompt, max_new_tokens=max_new)
        out.append(
            {
                "name": name,
                "policy": pol,
                "n_prompt": n_prompt,
                "capacity": cap,
                "evict_every": E,
                "max_new_tokens": max_new,
                "protect": prot,
                "n_kv_heads": n_kv,
                "regime": regime,
                "seed": seed,
                "prompt": prompt,
                "generated_token_ids": res.generated_token_ids,
                "eviction_count": res.eviction_count,
                "positions_retained": res.positions_retained,
                "positions_evicted": res.positions_evicted,
                "retention_mask": res.retention_mask,
                "policy_call_steps": res.policy_call_steps,
                "retained_counts_by_step": res.retained_counts_by_step,
                "prefill_position_count": res.prefill_position_count,
                "faithful_union_retained_max": res.faithful_union_retained_max,
                "faithful_union_overflow_max": res.faithful_union_overflow_max,
                "faithful_union_overflow_steps": res.faithful_union_overflow_steps,
            }
        )
    return {"source": "reference KVCoupledQwen35Generator + oracle.stub_model.StubScoreModel", "cases": out}


def make_e2e(ref: Path, preset: str, n_prompt: int, cap: int, max_cache: int, max_new: int, policy_name: str) -> dict:
    from kvcacheboundaryprotection_b200.config import get_config
    from kvcacheboundaryprotection_b200.weights import init_weights
    from oracle.model import OracleConfig, OracleModel

    P, _, Gen, Wrapper = _load_reference(ref)
    cfg = get_config(preset)
    w = {k: v.float().numpy() for k, v in init_weights(cfg, seed=0).items()}
    ocfg = OracleConfig(
        vocab=cfg.vocab, hidden=cfg.hidden, n_layers=cfg.n_layers, n_heads=cfg.n_heads, n_kv_heads=cfg.n_kv_heads,
        head_dim=cfg.head_dim, ffn=cfg.ffn, rope_theta=cfg.rope_theta, eps=cfg.eps, qkv_bias=cfg.qkv_bias,
        qk_norm=cfg.qk_norm, tie_embed=cfg.tie_embed,
    )

    class Recorder(OracleModel):
        def __init__(self, *a, **k):
            super().__init__(*a, **k)
            self.rec = []

        def __call__(self, **kw):
            out = super().__call__(**kw)
            row = np.asarray(out.logits, np.float32)[0, -1]
            top = np.argsort(-row, kind="stable")[:8]
            self.rec.append({"argmax": int(np.argmax(row)), "top_idx": [int(i) for i in top], "top_val": [float(row[i]) for i in top]})
            return out

    model = Recorder(ocfg, w, max_cache_len=max_cache)
    prompt = [int(x) for x in np.random.default_rng(0).integers(0, cfg.vocab, n_prompt)]
    policy = Wrapper(_policy_factory(P, policy_name, cap), prefix_frac=0.10, suffix_frac=0.10, capacity=cap)
    gen = Gen(model=model, tokenizer=None, policy=policy, capacity=cap, evict_every_n_steps=8, n_kv_heads=cfg.n_kv_heads)
    res = gen.generate_with_kv_control(input_ids=prompt, max_new_tokens=max_new)
    return {
        "source": "reference KVCoupledQwen35Generator + oracle.model.OracleModel",
        "preset": preset,
        "seed": 0,
        "prompt_seed": 0,
        "n_prompt": n_prompt,
        "capacity": cap,
        "max_cache_len": max_cache,
        "max_new_tokens": max_new,
        "policy": policy_name,
        "protect_frac": 0.10,
        "evict_every": 8,
        "generated_token_ids": res.generated_token_ids[n_prompt:],
        "positions_evicted": res.positions_evicted,
        "retained_counts_by_step": res.retained_counts_by_step,
        "policy_call_steps": res.policy_call_steps,
        "eviction_count": res.eviction_count,
        "logit_summaries": model.rec,
    }


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("KVBP_REFERENCE"),
                    help="the reference project's directory (default: $KVBP_REFERENCE)")
    ap.add_argument("--only", default=None)
    a = ap.parse_args()
    if not a.ref:
        ap.error("give --ref or set KVBP_REFERENCE")
    ref = Path(a.ref)
    jobs = {
        "policy_kats.json": lambda: make_policy_kats(ref),
        "generator_kats.json": lambda: make_generator_kats(ref),
        "e2e_parity_qwen2.json": lambda: make_e2e(ref, "parity-qwen2", 300, 64, 512, 40, "lru"),
        "e2e_parity_qwen2_h2o.json": lambda: make_e2e(ref, "parity-qwen2", 300, 64, 512, 40, "h2o_faithful"),
        "e2e_tiny_qwen2_lru.json": lambda: make_e2e(ref, "tiny-qwen2", 1024, 256, 2048, 128, "lru"),
    }
    for fname, fn in jobs.items():
        if a.only and a.only != fname:
            continue
        data = fn()
        (HERE / fname).write_text(json.dumps(data, separators=(",", ":")))
        print("wrote", fname)


if __name__ == "__main__":
    main()
