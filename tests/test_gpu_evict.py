"""Eviction kernels (K2 score update, K3 append/evict, step-0 select + compact) vs. the
reference's own decode/eviction traces, bit for bit, given equal scores.

Each case of tests/golden/generator_kats.json is a run of the reference
``KVCoupledQwen35Generator`` driven by ``oracle.stub_model.StubScoreModel``.  The
oracle generator (checked against the same fixture on the CPU) replays it and records
the per-step score vectors; those exact scores are written into ``step_score`` on the
GPU, so every victim, slot table and count must match exactly.
"""

import ctypes as C
import json
import os

import numpy as np
import pytest
import torch

from kvcacheboundaryprotection_b200 import build, capi
from kvcacheboundaryprotection_b200.policies import ProtectedPolicyWrapper, RandomEvictionPolicy
from oracle.generator import generate, slot_count
from oracle.policies import PolicySpec
from oracle.stub_model import StubScoreModel

from conftest import GOLDEN

pytestmark = pytest.mark.gpu

with open(os.path.join(GOLDEN, "generator_kats.json")) as _f:
    CASES = json.load(_f)["cases"]


class Driver:
    """Minimal state + calls of the eviction kernels for one sequence batch."""

    def __init__(self, B, S, W, evcap, max_new, cfg):
        d = "cuda"
        z = lambda *s, dt=torch.int32: torch.zeros(*s, dtype=dt, device=d)  # noqa: E731
        self.B, self.S, self.W = B, S, W
        self.slot_pos = torch.full((B, S), -1, dtype=torch.int32, device=d)
        self.ins, self.last, self.cnt = z(B, S), z(B, S), z(B, S)
        self.attn, self.maxa, self.pre = z(B, S, dt=torch.float32), z(B, S, dt=torch.float32), z(B, S, dt=torch.float32)
        self.cumul = z(B, S, dt=torch.float64)
        self.posmap = z(B, W)
        self.step_score = z(B, S, dt=torch.float32)
        self.seq_step, self.next_pos, self.cur_pos, self.write_slot = z(B), z(B), z(B), z(B)
        self.tokens = z(B)
        self.token_log = z(B, max(1, max_new))
        self.retained_log = z(B, max_new + 1)
        self.evlog, self.evcount = z(B, evcap), z(B)
        self.err = z(1)
        self.evcap, self.max_new = evcap, max_new
        self.state = capi.State(B, S, W, *[t.data_ptr() for t in (self.slot_pos, self.ins, self.last, self.cnt, self.attn, self.maxa, self.cumul, self.pre, self.posmap)])
        self.cfg = cfg
        self.L = capi.lib()

    @property
    def st(self):
        return torch.cuda.current_stream().cuda_stream

    def prefill(self, P, scores, host=None):
        victim = torch.zeros(self.B, P, dtype=torch.uint8, device="cuda")
        n = C.c_int32()
        sc = None if scores is None else torch.as_tensor(scores, dtype=torch.float32, device="cuda").reshape(self.B, P).contiguous()
        if host is not None:  # random policy: the host's victims, in its order (one sequence)
            vict = [int(k) for k in host.select_evictions({str(p): None for p in range(P)}, max(0, P - self.cfg.capacity), 0)]
            if vict:
                victim[0, torch.tensor(vict, device="cuda")] = 1
                self.evlog[0, : len(vict)] = torch.tensor(vict, dtype=torch.int32, device="cuda")
            n.value = len(vict)
        else:
            capi.check(self.L.kvbp_prefill_select(self.st, self.B, P, C.byref(self.cfg), None if sc is None else sc.data_ptr(), victim.data_ptr(), self.evlog.data_ptr(), self.evcap, C.byref(n), self.err.data_ptr()), "select")
        gsrc = torch.empty(self.B, self.S, dtype=torch.int32, device="cuda")
        capi.check(self.L.kvbp_prefill_compact(self.st, C.byref(self.state), P, self.cfg.capacity, n.value, victim.data_ptr(), None if sc is None else sc.data_ptr(), gsrc.data_ptr(), self.evlog.data_ptr(), self.evcap, self.evcount.data_ptr(), self.seq_step.data_ptr(), self.next_pos.data_ptr(), self.retained_log.data_ptr(), self.max_new, self.step_score.data_ptr(), self.err.data_ptr()), "compact")
        return gsrc

    def append_evict_listed(self, host):
        """Cadence victims drawn by the host policy over the retained positions plus the
        one this step appends (one sequence), then the listed-victims kernel."""
        step = int(self.seq_step[0].item()) + 1
        pos, cnt = torch.zeros(self.B, self.S, dtype=torch.int32, device="cuda"), torch.zeros(self.B, dtype=torch.int32, device="cuda")
        if step % self.cfg.evict_every == 0 and self.cfg.decode_regime:
            sp = self.slot_pos[0].cpu().numpy()
            live = sorted(sp[sp >= 0].tolist() + [int(self.next_pos[0].item())])
            vict = [int(k) for k in host.select_evictions({str(p): None for p in live}, max(0, len(live) - self.cfg.capacity), step)]
            if vict:
                pos[0, : len(vict)] = torch.tensor(vict, dtype=torch.int32, device="cuda")
            cnt[0] = len(vict)
        capi.check(self.L.kvbp_append_evict_listed(self.st, C.byref(self.state), C.byref(self.cfg), self.seq_step.data_ptr(), self.next_pos.data_ptr(), self.cur_pos.data_ptr(), self.write_slot.data_ptr(), self.tokens.data_ptr(), self.token_log.data_ptr(), self.max_new, self.evlog.data_ptr(), self.evcount.data_ptr(), self.evcap, self.retained_log.data_ptr(), pos.data_ptr(), cnt.data_ptr(), self.S, 0, self.err.data_ptr()), "append_evict_listed")

    def append_evict(self):
        capi.check(self.L.kvbp_append_evict(self.st, C.byref(self.state), C.byref(self.cfg), self.seq_step.data_ptr(), self.next_pos.data_ptr(), self.cur_pos.data_ptr(), self.write_slot.data_ptr(), self.tokens.data_ptr(), self.token_log.data_ptr(), self.max_new, self.evlog.data_ptr(), self.evcount.data_ptr(), self.evcap, self.retained_log.data_ptr(), self.err.data_ptr()), "append_evict")

    def score_update(self):
        capi.check(self.L.kvbp_score_update(self.st, C.byref(self.state), self.seq_step.data_ptr(), self.step_score.data_ptr(), self.err.data_ptr()), "score_update")

    def update_append_evict(self, pending):
        capi.check(self.L.kvbp_update_append_evict(self.st, C.byref(self.state), C.byref(self.cfg), self.seq_step.data_ptr(), self.next_pos.data_ptr(), self.cur_pos.data_ptr(), self.write_slot.data_ptr(), self.tokens.data_ptr(), self.token_log.data_ptr(), self.max_new, self.evlog.data_ptr(), self.evcount.data_ptr(), self.evcap, self.retained_log.data_ptr(), self.step_score.data_ptr(), pending.data_ptr(), self.err.data_ptr()), "update_append_evict")

    def metadata(self):
        return [t.clone() for t in (self.slot_pos, self.ins, self.last, self.cnt, self.attn, self.maxa, self.cumul, self.pre, self.posmap, self.seq_step, self.next_pos, self.cur_pos, self.write_slot, self.evcount, self.evlog)]


@pytest.fixture(scope="module", autouse=True)
def _lib():
    build.build()
    capi.lib()


def _spec(case):
    prot = case["protect"]
    return PolicySpec(case["policy"], case["capacity"], prot is not None, *(prot or (0.0, 0.0)))


PER_HEAD = ("adakv_faithful", "adakv_native", "quest_faithful", "quest_native")
GLOBAL_CASES = [c for c in CASES if c["policy"] not in PER_HEAD]
PER_HEAD_CASES = [c for c in CASES if c["policy"] in PER_HEAD]


@pytest.mark.parametrize("case", GLOBAL_CASES, ids=[c["name"] for c in GLOBAL_CASES])
def test_eviction_kernels_match_reference_trace(case):
    P, cap, E, max_new = case["n_prompt"], case["capacity"], case["evict_every"], case["max_new_tokens"]
    model = StubScoreModel(vocab=97, n_heads=4, n_kv_heads=2, n_layers=2, max_cache_len=P + max_new + 8, seed=case["seed"])
    spec = _spec(case)
    o = generate(model, spec, case["prompt"], max_new, evict_every=E, n_kv_heads=case["n_kv_heads"], regime=case["regime"])
    assert o.positions_evicted == case["positions_evicted"]  # oracle == reference

    n_pre, n_suf = capi.protection_sizes(cap, *(case["protect"] or (0.0, 0.0))) if case["protect"] else (0, 0)
    cfg = capi.EvictCfg(cap, E, capi.policy_id(case["policy"]), int(case["protect"] is not None), n_pre, n_suf, int(case["regime"] == "decode"))
    S = slot_count(cap, E, max_new, case["regime"])
    D = Driver(1, S, (P + max_new + 2 + 31) // 32, P + max_new + 2, max_new, cfg)
    host = None
    if case["policy"] == "random":  # victims drawn on the host with the package's policy objects
        host = RandomEvictionPolicy()
        if case["protect"]:
            host = ProtectedPolicyWrapper(host, *case["protect"], cap)
    pre = o.meta.prefill[:P] if case["policy"] not in ("lru", "random") else None
    D.prefill(P, pre, host)
    assert D.slot_pos[0].cpu().numpy().tolist() == o.slot_tables[0].tolist()
    for s in range(1, max_new + 1):
        D.append_evict_listed(host) if host is not None else D.append_evict()
        assert D.slot_pos[0].cpu().numpy().tolist() == o.slot_tables[s].tolist(), f"slot table after step {s}"
        if s == max_new:
            break
        ks = o.step_scores[s - 1]
        sp = D.slot_pos[0].cpu().numpy()
        sc = np.zeros(S, np.float32)
        sc[sp >= 0] = ks[sp[sp >= 0]]
        D.step_score[0].copy_(torch.from_numpy(sc))
        D.score_update()
    torch.cuda.synchronize()
    assert int(D.err.item()) == 0
    n = int(D.evcount[0].item())
    assert D.evlog[0, :n].cpu().numpy().tolist() == case["positions_evicted"]
    assert [P] + D.retained_log[0].cpu().numpy().tolist() == case["retained_counts_by_step"]


DEFERRED_CASES = [c for c in GLOBAL_CASES if c["policy"] != "random"]


@pytest.mark.parametrize("case", DEFERRED_CASES, ids=[c["name"] for c in DEFERRED_CASES])
def test_update_append_evict_equals_separate_update_then_append(case):
    """kvbp_update_append_evict (the previous step's score update run at the start of the
    next append) against the reference trace, and against kvbp_score_update at the end of
    each step + kvbp_append_evict: every metadata array bit-identical after every step."""
    P, cap, E, max_new = case["n_prompt"], case["capacity"], case["evict_every"], case["max_new_tokens"]
    model = StubScoreModel(vocab=97, n_heads=4, n_kv_heads=2, n_layers=2, max_cache_len=P + max_new + 8, seed=case["seed"])
    o = generate(model, _spec(case), case["prompt"], max_new, evict_every=E, n_kv_heads=case["n_kv_heads"], regime=case["regime"])
    n_pre, n_suf = capi.protection_sizes(cap, *(case["protect"] or (0.0, 0.0))) if case["protect"] else (0, 0)
    cfg = capi.EvictCfg(cap, E, capi.policy_id(case["policy"]), int(case["protect"] is not None), n_pre, n_suf, int(case["regime"] == "decode"))
    S = slot_count(cap, E, max_new, case["regime"])
    args = (1, S, (P + max_new + 2 + 31) // 32, P + max_new + 2, max_new, cfg)
    A, Bd = Driver(*args), Driver(*args)  # A: deferred update; Bd: separate launches
    pending = torch.zeros(1, dtype=torch.int32, device="cuda")
    pre = o.meta.prefill[:P] if case["policy"] != "lru" else None
    A.prefill(P, pre)
    Bd.prefill(P, pre)
    for s in range(1, max_new + 1):
        A.update_append_evict(pending)
        Bd.append_evict()
        assert A.slot_pos[0].cpu().numpy().tolist() == o.slot_tables[s].tolist(), f"slot table after step {s}"
        for x, y in zip(A.metadata(), Bd.metadata()):
            assert torch.equal(x, y), f"state differs after step {s}"
        assert int(pending.item()) == 1
        if s == max_new:
            break
        ks = o.step_scores[s - 1]
        sp = A.slot_pos[0].cpu().numpy()
        sc = np.zeros(S, np.float32)
        sc[sp >= 0] = ks[sp[sp >= 0]]
        A.step_score[0].copy_(torch.from_numpy(sc))
        Bd.step_score[0].copy_(torch.from_numpy(sc))
        Bd.score_update()
    torch.cuda.synchronize()
    assert int(A.err.item()) == 0 and int(Bd.err.item()) == 0
    n = int(A.evcount[0].item())
    assert A.evlog[0, :n].cpu().numpy().tolist() == case["positions_evicted"]
    assert [P] + A.retained_log[0].cpu().numpy().tolist() == case["retained_counts_by_step"]


def test_step0_lru_string_order_at_1024():
    # prompt 1024, capacity 256, protect 0.10: first victims follow str(pos) order
    cfg = capi.EvictCfg(256, 8, 0, 1, 25, 25, 1)
    D = Driver(2, 264, 40, 1200, 8, cfg)
    D.prefill(1024, None)
    torch.cuda.synchronize()
    ev = D.evlog[:, :768].cpu().numpy()
    assert ev[0, :8].tolist() == [100, 101, 102, 103, 104, 105, 106, 107]
    assert (ev[0] == ev[1]).all()
    m = PolicySpec("lru", 256, True)
    from oracle.policies import Meta

    assert ev[0].tolist() == m.select(list(range(1024)), Meta.zeros(1024), 768, 0)


@pytest.mark.parametrize("policy", ["h2o_faithful", "h2o", "snapkv", "snapkv_faithful", "adakv", "quest", "streamingllm"])
def test_step0_scored_policies_large_prompt(policy):
    from oracle.policies import Meta

    P, cap = 2048, 256
    rng = np.random.default_rng(7)
    scores = (rng.random(P) ** 4).astype(np.float32)
    scores[rng.integers(0, P, 200)] = scores[5]  # ties on the score component
    n_pre, n_suf = capi.protection_sizes(cap, 0.05, 0.05)
    cfg = capi.EvictCfg(cap, 8, capi.policy_id(policy), 1, n_pre, n_suf, 1)
    D = Driver(1, cap + 8, (P + 40) // 32 + 1, P + 16, 8, cfg)
    D.prefill(P, scores)
    torch.cuda.synchronize()
    m = Meta.zeros(P)
    m.attn[:] = m.max_attn[:] = m.prefill[:] = scores
    m.cumul[:] = scores.astype(np.float64)
    want = PolicySpec(policy, cap, True, 0.05, 0.05).select(list(range(P)), m, P - cap, 0)
    from oracle.policies import hard_cap

    rest = sorted(set(range(P)) - set(want))
    want = want + hard_cap(rest, m, len(rest) - cap)
    n = int(D.evcount[0].item())
    assert D.evlog[0, :n].cpu().numpy().tolist() == want


def test_random_policy_is_rejected_without_a_victim_list():
    cfg = capi.EvictCfg(32, 8, capi.policy_id("random"), 1, 4, 4, 1)
    D = Driver(1, 40, 8, 200, 8, cfg)
    with pytest.raises(capi.KVBPError, match="host"):
        D.append_evict()
    with pytest.raises(capi.KVBPError, match="host"):
        D.prefill(100, None)


def test_random_policy_generator_end_to_end_matches_reference_trace():
    """The drop-in generator with the random policy (host-drawn victims, device slot
    path) reproduces the reference generator's trace of the same policy: victims are
    independent of the model's scores except through the hard-capacity guardrail, which
    these settings never reach."""
    from kvcacheboundaryprotection_b200.config import get_config
    from kvcacheboundaryprotection_b200.generator import CappedKVModel, KVCoupledQwen35Generator
    from kvcacheboundaryprotection_b200.weights import init_weights

    case = next(c for c in CASES if c["name"] == "random_p160_c40")
    cfg = get_config("parity-qwen2").with_(vocab=128 * 8)
    model = CappedKVModel(cfg, init_weights(cfg, seed=0), device="cuda")
    pol = ProtectedPolicyWrapper(RandomEvictionPolicy(), 0.10, 0.10, case["capacity"])
    gen = KVCoupledQwen35Generator(model, None, pol, case["capacity"], case["evict_every"], cfg.n_kv_heads)
    res = gen.generate_with_kv_control(case["prompt"], case["max_new_tokens"])
    assert res.positions_evicted == case["positions_evicted"]
    assert res.retained_counts_by_step == case["retained_counts_by_step"]
    assert res.policy_call_steps == case["policy_call_steps"]
    # the policy object's stream continues across calls, as in the reference
    res2 = gen.generate_with_kv_control(case["prompt"], case["max_new_tokens"])
    assert res2.positions_evicted != res.positions_evicted


@pytest.mark.parametrize("case", PER_HEAD_CASES, ids=[c["name"] for c in PER_HEAD_CASES])
def test_per_head_policies_match_reference_trace(case):
    """Per-KV-head Ada-KV / QUEST through the engine's own per-head path: host selection
    over the device's per-slot signals, listed victims freed on the device, per-head keep
    masks written back -- with the oracle's per-step scores injected into step_score and
    head_score, so victims, slot tables, calls and union statistics must be identical to
    the reference generator's trace."""
    from kvcacheboundaryprotection_b200.config import get_config
    from kvcacheboundaryprotection_b200.engine import CappedKVEngine, EvictionSpec
    from kvcacheboundaryprotection_b200.policies import policy_from_name
    from kvcacheboundaryprotection_b200.weights import init_weights

    P, cap, E, max_new = case["n_prompt"], case["capacity"], case["evict_every"], case["max_new_tokens"]
    mk = lambda: StubScoreModel(vocab=97, n_heads=4, n_kv_heads=2, n_layers=2, max_cache_len=P + max_new + 8,  # noqa: E731
                                seed=case["seed"])
    o = generate(mk(), _spec(case), case["prompt"], max_new, evict_every=E, n_kv_heads=case["n_kv_heads"],
                 regime=case["regime"])
    assert o.positions_evicted == case["positions_evicted"]  # oracle == reference
    pre = mk()(input_ids=case["prompt"], output_attentions=True, use_cache=True).attentions
    layer0 = np.asarray(pre[0], np.float32).reshape(-1)[:P]
    cfg = get_config("parity-qwen2").with_(n_layers=1, vocab=1024)
    assert (cfg.n_heads, cfg.n_kv_heads) == (4, 2)
    pol = policy_from_name(case["policy"], cap)
    prot = case["protect"]
    if prot:
        pol = ProtectedPolicyWrapper(pol, *prot, cap)
    spec = EvictionSpec("quest", cap, E, prot is not None, *(prot or (0.0, 0.0)), regime=case["regime"],
                        protect_capacity=cap)
    eng = CappedKVEngine(cfg, init_weights(cfg, seed=0), batch=1, evict=spec, max_prompt_len=P, max_new_tokens=max_new,
                         host_policy=pol)
    assert eng.per_head and eng.S == slot_count(cap, E, max_new, case["regime"])
    eng.prefill_head_seed = torch.from_numpy(layer0).cuda()[None]
    eng._select_and_compact(P, torch.from_numpy(o.meta.prefill[:P].copy()).cuda()[None])
    eng.prompt_len = P
    assert eng.slot_pos[0].cpu().numpy().tolist() == o.slot_tables[0].tolist()
    heads = iter(o.step_head_scores)
    for s in range(1, max_new + 1):
        eng._append_evict()
        assert eng.slot_pos[0].cpu().numpy().tolist() == o.slot_tables[s].tolist(), f"slot table after step {s}"
        if s == max_new:
            break
        sp = eng.slot_pos[0].cpu().numpy()
        ok = sp >= 0
        sc = np.zeros(eng.S, np.float32)
        sc[ok] = o.step_scores[s - 1][sp[ok]]
        eng.step_score[0].copy_(torch.from_numpy(sc))
        hs = next(heads)
        hsc = np.zeros((2, eng.S), np.float32)
        hsc[:, ok] = hs[:, sp[ok]]
        eng.head_score[0].copy_(torch.from_numpy(hsc))
        eng._sample_and_score()
    torch.cuda.synchronize()
    eng.check_device_errors()
    n = int(eng.evcount[0].item())
    assert eng.evlog[0, :n].cpu().numpy().tolist() == case["positions_evicted"]
    assert [P] + eng.retained_log[0].cpu().numpy().tolist() == case["retained_counts_by_step"]
    assert eng.head_call_steps == case["policy_call_steps"]
    assert eng.union_stats == [case["faithful_union_retained_max"], case["faithful_union_overflow_max"],
                               case["faithful_union_overflow_steps"]]
    sp = eng.slot_pos[0].cpu().numpy()
    ok = sp >= 0
    keep = eng.head_keep[0].cpu().numpy()[:, ok].astype(bool)
    assert (keep == o.head_keep[:, sp[ok]]).all()


@pytest.mark.parametrize("policy,E", [("lru", 24), ("h2o_faithful", 24), ("adakv", 12), ("snapkv", 20)])
def test_eviction_kernels_large_cadence_against_oracle(policy, E):
    """Cadences that evict more than the warp-first top-k selects at once (k > 16) go
    through the block-round selection; both must reproduce the oracle's victims (the
    oracle generator is pinned to the reference's traces on the other cases)."""
    P, cap, max_new, seed = 200, 48, 60, 3
    rng = np.random.default_rng(seed)
    prompt = rng.integers(0, 97, P).tolist()
    model = StubScoreModel(vocab=97, n_heads=4, n_kv_heads=2, n_layers=2, max_cache_len=P + max_new + 8, seed=seed)
    spec = PolicySpec(policy, cap, True, 0.1, 0.1)
    o = generate(model, spec, prompt, max_new, evict_every=E, n_kv_heads=2, regime="decode")
    n_pre, n_suf = capi.protection_sizes(cap, 0.1, 0.1)
    cfg = capi.EvictCfg(cap, E, capi.policy_id(policy), 1, n_pre, n_suf, 1)
    S = slot_count(cap, E, max_new, "decode")
    for deferred in (False, True):
        D = Driver(1, S, (P + max_new + 2 + 31) // 32, P + max_new + 2, max_new, cfg)
        pending = torch.zeros(1, dtype=torch.int32, device="cuda")
        D.prefill(P, o.meta.prefill[:P] if policy != "lru" else None)
        for s in range(1, max_new + 1):
            D.update_append_evict(pending) if deferred else D.append_evict()
            assert D.slot_pos[0].cpu().numpy().tolist() == o.slot_tables[s].tolist(), f"slot table after step {s}"
            if s == max_new:
                break
            ks = o.step_scores[s - 1]
            sp = D.slot_pos[0].cpu().numpy()
            sc = np.zeros(S, np.float32)
            sc[sp >= 0] = ks[sp[sp >= 0]]
            D.step_score[0].copy_(torch.from_numpy(sc))
            if not deferred:
                D.score_update()
        torch.cuda.synchronize()
        assert int(D.err.item()) == 0
        n = int(D.evcount[0].item())
        assert D.evlog[0, :n].cpu().numpy().tolist() == o.positions_evicted


def test_update_append_evict_more_slots_than_one_pass():
    """Above 5120 slots the score update reloads its inputs in a second pass: still bit-
    identical to the separate launches (random prefill scores and step scores)."""
    P, C, E, max_new = 7000, 6000, 8, 20
    cfg = capi.EvictCfg(C, E, capi.policy_id("h2o_faithful"), 1, *capi.protection_sizes(C, 0.1, 0.1), 1)
    S = slot_count(C, E, max_new, "decode")
    assert S > 5120
    args = (2, S, (P + max_new + 2 + 31) // 32, P + max_new + 2, max_new, cfg)
    A, Bd = Driver(*args), Driver(*args)
    pending = torch.zeros(2, dtype=torch.int32, device="cuda")
    rng = np.random.default_rng(7)
    pre = rng.random((2, P)).astype(np.float32)
    A.prefill(P, pre)
    Bd.prefill(P, pre)
    for s in range(1, max_new + 1):
        A.update_append_evict(pending)
        Bd.append_evict()
        for x, y in zip(A.metadata(), Bd.metadata()):
            assert torch.equal(x, y), f"state differs after step {s}"
        sc = torch.from_numpy(rng.random((2, S)).astype(np.float32)).cuda()
        sc[A.slot_pos < 0] = 0
        A.step_score.copy_(sc)
        Bd.step_score.copy_(sc)
        Bd.score_update()
    torch.cuda.synchronize()
    assert int(A.err.item()) == 0 and int(Bd.err.item()) == 0
    assert int(A.evcount[0].item()) > P - C  # the cadence steps evicted
