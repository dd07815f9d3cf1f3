"""Oracle policy restatement vs. victim lists produced by the reference's own code."""

import json
import os

import numpy as np
import pytest

from oracle.policies import Meta, PolicySpec, protection_sizes

from conftest import GOLDEN


def _cases():
    with open(os.path.join(GOLDEN, "policy_kats.json")) as f:
        return json.load(f)["cases"]


def _meta(case):
    pos = np.asarray(case["positions"], np.int64)
    n = int(pos.max()) + 1
    m = Meta.zeros(n)
    m.insert_step[pos] = case["insert_step"]
    m.last_access[pos] = case["last_access"]
    m.access_count[pos] = case["access_count"]
    m.attn[pos] = np.asarray(case["attn"], np.float32)
    m.max_attn[pos] = np.asarray(case["max_attn"], np.float32)
    m.cumul[pos] = np.asarray(case["cumul"], np.float64)
    m.prefill[pos] = np.asarray(case["prefill"], np.float32)
    return pos.tolist(), m


def test_policy_kats_bit_exact():
    n = 0
    for case in _cases():
        pos, m = _meta(case)
        for r in case["results"]:
            spec = PolicySpec(r["policy"], case["capacity"], r["protect"], r["prefix_frac"], r["suffix_frac"])
            got = spec.select(pos, m, case["evict_count"], case["step"])
            assert got == r["victims"], (case["case"], case["tie"], r["policy"], r["protect"], r["suffix_frac"])
            n += 1
    assert n >= 900


def test_string_tiebreak_first_victims():
    # all-tied LRU keys over positions 0..1023: victims follow decimal-string order
    m = Meta.zeros(1024)
    spec = PolicySpec("lru", 256, True, 0.10, 0.10)
    got = spec.select(list(range(1024)), m, 768, 0)
    assert got[:8] == [100, 101, 102, 103, 104, 105, 106, 107]
    assert len(got) == 768


@pytest.mark.parametrize("cap,frac,expect", [(256, 0.10, 25), (1024, 0.10, 102), (4096, 0.10, 409), (256, 0.05, 12), (8, 0.1, 4)])
def test_protection_sizes(cap, frac, expect):
    assert protection_sizes(cap, frac, frac) == (expect, expect)


def test_attention_mass_alias():
    m = Meta.zeros(50)
    m.cumul[:] = np.linspace(1, 0, 50)
    a = PolicySpec("attention-mass", 20, True).select(list(range(50)), m, 10, 3)
    b = PolicySpec("h2o_faithful", 20, True).select(list(range(50)), m, 10, 3)
    assert a == b


def test_int8_roundtrip_restatement():
    """The oracle's int8 demotion: zero rows stay zero, the row maximum maps to +-127 * scale,
    every value is a multiple of the scale, and re-demotion is nearly idempotent."""
    import numpy as np

    from oracle.bf16 import rnd
    from oracle.model import int8_roundtrip

    rng = np.random.default_rng(0)
    x = rnd(rng.standard_normal((6, 128)).astype(np.float32) * 3)
    x[2] = 0.0
    y = int8_roundtrip(x)
    assert (y[2] == 0).all()
    scale = rnd(np.abs(x).max(axis=-1, keepdims=True) / np.float32(127))
    q = y / np.where(scale == 0, 1, scale)
    assert np.abs(q).max() <= 127.0 * (1 + 2 ** -8)  # q * scale is rounded to bf16
    assert np.allclose(np.abs(y).max(axis=-1), (127 * scale[:, 0]), rtol=1e-2)
    assert np.abs(int8_roundtrip(y) - y).max() <= np.abs(y).max() * 2 ** -7
