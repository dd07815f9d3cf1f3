"""Oracle decode/eviction loop vs. traces of the reference generator (same stub model), global
and per-KV-head policies."""

import json
import os

import numpy as np
import pytest

from oracle.generator import generate
from oracle.policies import PolicySpec
from oracle.stub_model import StubScoreModel

from conftest import GOLDEN

with open(os.path.join(GOLDEN, "generator_kats.json")) as _f:
    CASES = json.load(_f)["cases"]


@pytest.mark.parametrize("case", CASES, ids=[c["name"] for c in CASES])
def test_generator_trace(case):
    model = StubScoreModel(
        vocab=97, n_heads=4, n_kv_heads=2, n_layers=2,
        max_cache_len=case["n_prompt"] + case["max_new_tokens"] + 8, seed=case["seed"],
    )
    prot = case["protect"]
    spec = PolicySpec(case["policy"], case["capacity"], prot is not None, *(prot or (0.0, 0.0)))
    res = generate(
        model, spec, case["prompt"], case["max_new_tokens"], evict_every=case["evict_every"],
        n_kv_heads=case["n_kv_heads"], regime=case["regime"],
    )
    for key in ("generated_token_ids", "eviction_count", "positions_retained", "positions_evicted",
                "retention_mask", "policy_call_steps", "retained_counts_by_step", "prefill_position_count",
                "faithful_union_retained_max", "faithful_union_overflow_max", "faithful_union_overflow_steps"):
        assert getattr(res, key) == case[key], key


def test_slot_layout_invariants():
    case = next(c for c in CASES if c["name"] == "lru_p300_c64")
    model = StubScoreModel(vocab=97, n_heads=4, n_kv_heads=2, n_layers=2, max_cache_len=400, seed=case["seed"])
    res = generate(model, PolicySpec("lru", 64, True), case["prompt"], 40, n_kv_heads=2)
    # after step 0 the retained prompt positions fill slots 0..63 in ascending order
    t0 = res.slot_tables[0]
    assert (t0[:64] == np.sort(t0[:64])).all() and (t0[64:] == -1).all()
    # every slot table holds exactly the retained positions
    kept = set(np.flatnonzero(res.retention_mask).tolist())
    assert set(res.slot_tables[-1][res.slot_tables[-1] >= 0].tolist()) == kept
