"""End-to-end parity of the GPU decode path with the oracle (numpy forward + decode loop).

Teacher forcing: both sides consume the oracle's token sequence, so every step is
compared on identical inputs.  Tolerances (bf16 path; the forward numerics are
"parity unpinned" because the reference's JAX/XLA cannot run here):
  * logits: max |diff| <= 2e-2 per step, greedy argmax identical on >= 99 % of steps
    (steps whose top-2 oracle logits tie or sit within 2e-2 are excluded),
  * per-slot step scores: median rel diff <= 1e-3 and |diff| <= 0.08 * p + 1e-3 * max(p)
    per step.  The reference rounds every logit to bfloat16; a one-ulp difference of a
    logit s (from fp32 accumulation order upstream) moves its probability by a factor
    exp(+-ulp(s)), ~|s| * 2^-8, so large logits (Qwen3's q/k RMSNorm) move by a few %.
  * LRU: slot tables, victims and retained counts identical.  Scored policies rank by
    float sums of those probabilities, so near-ties may reorder: >= 90 % of the victims
    must agree (bit-exactness given EQUAL scores is checked in test_gpu_evict.py).
The free-running run (no forcing) is compared against the golden trace produced by the
reference generator with the oracle forward (tests/golden/e2e_parity_qwen2*.json).
"""

import json
import os

import numpy as np
import pytest
import torch

from kvcacheboundaryprotection_b200 import build
from kvcacheboundaryprotection_b200.config import get_config
from kvcacheboundaryprotection_b200.engine import CappedKVEngine, EvictionSpec
from kvcacheboundaryprotection_b200.generator import CappedKVModel, KVCoupledQwen35Generator
from kvcacheboundaryprotection_b200.policies import ProtectedPolicyWrapper, policy_from_name
from kvcacheboundaryprotection_b200.weights import init_weights
from oracle.generator import generate
from oracle.model import OracleConfig, OracleModel
from oracle.policies import PolicySpec

from conftest import GOLDEN

pytestmark = pytest.mark.gpu


def _ocfg(cfg):
    return OracleConfig(
        vocab=cfg.vocab, hidden=cfg.hidden, n_layers=cfg.n_layers, n_heads=cfg.n_heads, n_kv_heads=cfg.n_kv_heads,
        head_dim=cfg.head_dim, ffn=cfg.ffn, rope_theta=cfg.rope_theta, eps=cfg.eps, qkv_bias=cfg.qkv_bias,
        qk_norm=cfg.qk_norm, tie_embed=cfg.tie_embed,
    )


@pytest.fixture(scope="module", autouse=True)
def _lib():
    build.build()


def _run_forced(preset, policy, P, cap, N, max_new, seed=0):
    cfg = get_config(preset)
    w = init_weights(cfg, seed=0)
    wn = {k: v.float().numpy() for k, v in w.items()}
    prompt = [int(x) for x in np.random.default_rng(seed).integers(0, cfg.vocab, P)]
    spec = PolicySpec(policy, cap, True, 0.10, 0.10)
    om = OracleModel(_ocfg(cfg), wn, max_cache_len=N)
    o = generate(om, spec, prompt, max_new, evict_every=8, n_kv_heads=cfg.n_kv_heads, record_logits=True)
    forced = o.generated_token_ids[P:]

    eng = CappedKVEngine(cfg, w, batch=1, evict=EvictionSpec(policy, cap, 8, True, 0.10, 0.10), max_prompt_len=P, max_new_tokens=max_new)
    eng.prefill(torch.tensor([prompt], dtype=torch.int32))
    torch.cuda.synchronize()
    stats = {"logit_diff": [], "argmax_ok": 0, "argmax_n": 0, "score_rel": []}

    def cmp_logits(step_idx):
        got = eng.logits[0].float().cpu().numpy()
        want = o.step_logits[step_idx]
        d = np.abs(got - want)
        stats["logit_diff"].append(float(d.max()))
        stats.setdefault("logit_mean_diff", []).append(float(d.mean()))
        i = int(np.argmax(d))
        ulp = np.float32(2.0) ** (np.floor(np.log2(np.maximum(np.abs(want), 1e-30))) - 7)  # bf16 ulp of each logit
        stats.setdefault("detail", []).append((step_idx, float(d[i]), float(want[i]), float(got[i]),
                                               float((d / ulp).max()), float(np.mean(d <= ulp))))
        top2 = np.sort(want)[-2:]
        if top2[1] - top2[0] > 2e-2:
            stats["argmax_n"] += 1
            stats["argmax_ok"] += int(np.argmax(got) == np.argmax(want))

    cmp_logits(0)
    assert eng.slot_pos[0].cpu().numpy().tolist() == o.slot_tables[0].tolist()
    for s in range(1, max_new + 1):
        eng.tokens.fill_(int(forced[s - 1]))
        eng._append_evict()
        assert eng.slot_pos[0].cpu().numpy().tolist() == o.slot_tables[s].tolist(), f"slot table at step {s}"
        if s == max_new:
            break
        eng._forward()
        sp = eng.slot_pos[0].cpu().numpy()
        # the step's per-slot scores (max over heads and layers), before any update applies them
        got = eng.step_score[0].cpu().numpy()[sp >= 0]
        want = o.step_scores[s - 1][sp[sp >= 0]]
        stats["score_rel"].append(np.abs(got - want) / np.maximum(want, 1e-30))
        stats.setdefault("score_ok", []).append(bool((np.abs(got - want) <= 0.08 * want + 1e-3 * want.max()).all()))
        cmp_logits(s)
        eng._sample_and_score()
    torch.cuda.synchronize()
    eng.check_device_errors()
    n = int(eng.evcount[0].item())
    return o, eng, stats, eng.evlog[0, :n].cpu().numpy().tolist()


@pytest.mark.parametrize("preset,policy", [("parity-qwen2", "lru"), ("parity-qwen2", "h2o_faithful"), ("parity-qwen3", "lru"), ("parity-g7", "h2o_faithful")])
def test_teacher_forced_parity(preset, policy):
    o, eng, st, evicted = _run_forced(preset, policy, P=300, cap=64, N=512, max_new=40)
    assert max(st["logit_diff"]) <= 2e-2, max(st["logit_diff"])
    assert st["argmax_n"] >= 10 and st["argmax_ok"] >= 0.99 * st["argmax_n"]
    rel = np.concatenate(st["score_rel"])
    print(f"{preset}/{policy}: max logit diff {max(st['logit_diff']):.3g}, argmax {st['argmax_ok']}/{st['argmax_n']}, "
          f"score rel max {rel.max():.3g} median {np.median(rel):.3g} p95 {np.percentile(rel, 95):.3g}")
    assert all(st["score_ok"])
    assert np.median(rel) <= 1e-3
    if policy == "lru":
        assert evicted == o.positions_evicted
    else:
        assert len(evicted) == len(o.positions_evicted)
        assert len(set(evicted) & set(o.positions_evicted)) >= 0.9 * len(evicted)


def test_teacher_forced_parity_twenty_sequences_in_one_batch():
    """Twenty sequences decoded in one batch: every decode GEMM then has 17..32 activation
    rows and runs the tcgen05 main loop (the single-sequence runs above take it only for
    the norm-prologue GEMMs).  Each sequence must match its own oracle run as those do:
    logits within 2e-2 per step and identical LRU slot tables and victims."""
    cfg = get_config("parity-qwen2")
    w = init_weights(cfg, seed=0)
    wn = {k: v.float().numpy() for k, v in w.items()}
    B, P, cap, N, max_new = 20, 300, 64, 512, 17  # two eviction cadences
    prompts = [[int(x) for x in np.random.default_rng(100 + b).integers(0, cfg.vocab, P)] for b in range(B)]
    spec = PolicySpec("lru", cap, True, 0.10, 0.10)
    orc = [generate(OracleModel(_ocfg(cfg), wn, max_cache_len=N), spec, p, max_new, evict_every=8,
                    n_kv_heads=cfg.n_kv_heads, record_logits=True) for p in prompts]
    forced = np.array([o.generated_token_ids[P:] for o in orc], dtype=np.int32)  # [B][max_new]

    eng = CappedKVEngine(cfg, w, batch=B, evict=EvictionSpec("lru", cap, 8, True, 0.10, 0.10), max_prompt_len=P,
                         max_new_tokens=max_new)
    eng.prefill(torch.tensor(prompts, dtype=torch.int32))
    torch.cuda.synchronize()
    worst = 0.0

    def check_step(s):
        nonlocal worst
        got = eng.logits.float().cpu().numpy()
        for b in range(B):
            worst = max(worst, float(np.abs(got[b] - orc[b].step_logits[s]).max()))

    check_step(0)
    for s in range(1, max_new + 1):
        eng.tokens.copy_(torch.from_numpy(forced[:, s - 1]).to(eng.tokens.device))
        eng._append_evict()
        sp = eng.slot_pos.cpu().numpy()
        for b in range(B):
            assert sp[b].tolist() == orc[b].slot_tables[s].tolist(), f"slot table of sequence {b} at step {s}"
        if s == max_new:
            break
        eng._forward()
        check_step(s)
        eng._sample_and_score()
    torch.cuda.synchronize()
    eng.check_device_errors()
    print(f"20 sequences: max logit diff {worst:.3g}")
    assert worst <= 2e-2, worst
    for b in range(B):
        n = int(eng.evcount[b].item())
        assert eng.evlog[b, :n].cpu().numpy().tolist() == orc[b].positions_evicted


@pytest.mark.parametrize("fixture", ["e2e_parity_qwen2.json", "e2e_parity_qwen2_h2o.json"])
def test_free_running_against_reference_trace(fixture):
    with open(os.path.join(GOLDEN, fixture)) as f:
        ref = json.load(f)
    cfg = get_config(ref["preset"])
    model = CappedKVModel(cfg, init_weights(cfg, seed=ref["seed"]), device="cuda")
    prompt = [int(x) for x in np.random.default_rng(ref["prompt_seed"]).integers(0, cfg.vocab, ref["n_prompt"])]
    pol = ProtectedPolicyWrapper(policy_from_name(ref["policy"], ref["capacity"]), 0.10, 0.10, ref["capacity"])
    gen = KVCoupledQwen35Generator(model, None, pol, ref["capacity"], 8, cfg.n_kv_heads)
    res = gen.generate_with_kv_control(prompt, ref["max_new_tokens"])
    toks = res.generated_token_ids[ref["n_prompt"]:]
    agree = np.mean(np.asarray(toks) == np.asarray(ref["generated_token_ids"]))
    # greedy decoding diverges for good after the first differing token; bf16 ties
    # make that possible, so require the long common prefix and full agreement of the
    # eviction bookkeeping that does not depend on tokens (counts, call steps).
    assert agree >= 0.99 or toks[:20] == ref["generated_token_ids"][:20]
    assert res.retained_counts_by_step == ref["retained_counts_by_step"]
    assert res.policy_call_steps == ref["policy_call_steps"]
    assert res.eviction_count == ref["eviction_count"]
    if agree == 1.0:
        common = set(res.positions_evicted) & set(ref["positions_evicted"])
        if ref["policy"] == "lru":
            assert res.positions_evicted == ref["positions_evicted"]
        else:
            assert len(common) >= 0.9 * len(ref["positions_evicted"])


def test_graph_replay_equals_eager():
    cfg = get_config("parity-qwen2")
    model = CappedKVModel(cfg, init_weights(cfg, seed=0), device="cuda")
    prompt = [int(x) for x in np.random.default_rng(3).integers(0, cfg.vocab, 200)]
    outs = []
    for use_graph in (False, True):
        pol = ProtectedPolicyWrapper(policy_from_name("h2o_faithful", 48), 0.10, 0.10, 48)
        gen = KVCoupledQwen35Generator(model, None, pol, 48, 8, cfg.n_kv_heads, use_graph=use_graph)
        outs.append(gen.generate_batch([prompt, prompt[::-1]], 30))
    for a, b in zip(*outs):
        assert a.generated_token_ids == b.generated_token_ids
        assert a.positions_evicted == b.positions_evicted


# ---- the CPU-runnable plumbing configuration end to end: 4-layer tiny-qwen2 (hidden 1024,
# 8/2 heads, vocab 151936, weights N(0, 0.02) seed 0 cast to bf16), a 1024-token prompt of
# uniform ids (seed 0), LRU, capacity 256, max-cache-len 2048, protect-frac 0.10,
# evict-every 8, 128 greedy tokens.  The eviction arithmetic gives 768 step-0 victims and
# 8 per cadence step: 896 in all.
TINY = dict(P=1024, cap=256, N=2048, max_new=128)


def test_tiny_qwen2_teacher_forced_parity():
    """Logit tolerance at this configuration: max |diff| <= 5e-2 and mean |diff| <= 1e-2 per
    step.  4 layers of bf16 rounding points over a 1024-token context leave a noise floor
    that no accumulation order gets under: the oracle itself with float64-accumulated
    projections (same rounding points) differs from its float32 form by max 0.027 / mean
    0.0046 on the step-0 logits (tests/test_oracle_noise_floor.py), the same as this path
    (max 0.027 / mean 0.0046 at step 0, <= 0.04 over the 128 steps).  The 2e-2 bound holds
    on the 2-layer parity decoders above."""
    o, eng, st, evicted = _run_forced("tiny-qwen2", "lru", **TINY)
    print(f"tiny-qwen2: max logit diff {max(st['logit_diff']):.3g}, mean {max(st['logit_mean_diff']):.3g}, "
          f"argmax {st['argmax_ok']}/{st['argmax_n']}")
    assert len(st["logit_diff"]) == TINY["max_new"]
    worst = sorted(st["detail"], key=lambda r: -r[1])[:6]
    assert max(st["logit_diff"]) <= 5e-2, ("(step, |diff|, oracle, gpu, max ulps, frac within 1 ulp)", worst)
    assert max(st["logit_mean_diff"]) <= 1e-2
    assert st["argmax_n"] >= 64 and st["argmax_ok"] >= 0.99 * st["argmax_n"]
    assert all(st["score_ok"])
    assert np.median(np.concatenate(st["score_rel"])) <= 1e-3
    assert len(o.positions_evicted) == 896
    assert evicted == o.positions_evicted  # LRU victims identical over all 128 steps


def test_tiny_qwen2_free_running_against_reference_trace():
    """Greedy decoding, no forcing, against the trace of the reference's own generator
    (tests/golden/e2e_tiny_qwen2_lru.json).  bf16 logits of a 151936-entry vocabulary tie
    often: in the trace, 20 of the 128 steps have their two largest logits within one bf16
    ulp (2e-2).  A differently rounded upstream sum may break such a tie the other way, after
    which the two runs continue from different tokens.  So tokens must agree up to the first
    difference, and a difference is only allowed where the trace's chosen token and ours
    both lie within 2e-2 of the trace's maximum logit.  The bookkeeping that does not depend
    on token identity (retained counts per step, policy call steps, 896 evictions) must
    agree over all 128 steps, and the LRU victims up to the divergence."""
    with open(os.path.join(GOLDEN, "e2e_tiny_qwen2_lru.json")) as f:
        ref = json.load(f)
    cfg = get_config(ref["preset"])
    assert (ref["n_prompt"], ref["capacity"], ref["max_new_tokens"]) == (1024, 256, 128)
    model = CappedKVModel(cfg, init_weights(cfg, seed=ref["seed"]), device="cuda")
    prompt = [int(x) for x in np.random.default_rng(ref["prompt_seed"]).integers(0, cfg.vocab, ref["n_prompt"])]
    pol = ProtectedPolicyWrapper(policy_from_name("lru", 256), 0.10, 0.10, 256)
    gen = KVCoupledQwen35Generator(model, None, pol, 256, 8, cfg.n_kv_heads)
    res = gen.generate_with_kv_control(prompt, 128)
    toks = res.generated_token_ids[ref["n_prompt"]:]
    want = ref["generated_token_ids"]
    diff = [i for i in range(128) if toks[i] != want[i]]
    first = diff[0] if diff else 128
    print(f"tiny-qwen2 free-running: {128 - len(diff)}/128 tokens identical, first difference at {first}")
    if diff:
        s = ref["logit_summaries"][first]
        top = dict(zip(s["top_idx"], s["top_val"]))
        assert toks[first] in top, f"step {first}: token {toks[first]} is not among the trace's top 8"
        assert top[want[first]] - top[toks[first]] <= 2e-2, (first, top[want[first]], top[toks[first]])
    assert res.retained_counts_by_step == ref["retained_counts_by_step"]
    assert res.policy_call_steps == ref["policy_call_steps"]
    assert res.eviction_count == ref["eviction_count"] == 896
    # victims chosen at step 0 and at the cadence steps whose scores came from identical tokens
    calls_before = [c for c in ref["policy_call_steps"] if 0 < c <= first + 1]
    n_same = (ref["n_prompt"] - ref["capacity"]) + 8 * len(calls_before)
    assert res.positions_evicted[:n_same] == ref["positions_evicted"][:n_same]


def test_pending_scores_applied_without_append_equal_the_appends_update():
    """The engine defers each step's score update to the next append kernel; after a forward
    with no append to follow, apply_pending_scores runs the same update: the metadata of the
    retained slots equals what the next append's update writes (bit for bit)."""
    cfg = get_config("parity-qwen2")
    w = init_weights(cfg, seed=0)
    prompt = torch.tensor([[int(x) for x in np.random.default_rng(5).integers(0, cfg.vocab, 120)]], dtype=torch.int32)
    engs = []
    for _ in range(2):
        e = CappedKVEngine(cfg, w, batch=1, evict=EvictionSpec("h2o_faithful", 48, 8, True, 0.10, 0.10),
                           max_prompt_len=120, max_new_tokens=12)
        assert e.deferred_score_update
        e.prefill(prompt)
        for _ in range(5):
            e.run_step(use_graph=False)
        engs.append(e)
    a, b = engs
    a.apply_pending_scores()
    b._append_evict()  # applies the pending update, then appends step 6's position
    torch.cuda.synchronize()
    keep = (a.slot_pos >= 0) & (b.slot_pos == a.slot_pos)
    assert int(keep.sum()) >= 40
    for name in ("attn_s", "max_attn", "cumul", "last_access", "access_count"):
        assert torch.equal(getattr(a, name)[keep], getattr(b, name)[keep]), name
    assert int(a.step_score.abs().sum().item()) == 0 and int(a.upd_pending.sum().item()) == 0
    a.check_device_errors()
    b.check_device_errors()
