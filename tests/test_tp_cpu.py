"""Tensor-parallel plan and weight sharding (CPU): every head, FFN column and vocabulary
row is owned exactly as the plan says, and the shards' partial products sum back to the
unsharded projections."""

import pytest
import torch

from kvcacheboundaryprotection_b200.config import get_config
from kvcacheboundaryprotection_b200.tp import local_config, shard_weights, tp_plan
from kvcacheboundaryprotection_b200.weights import init_weights


@pytest.mark.parametrize("preset,world", [("qwen2.5-7b", 1), ("qwen2.5-7b", 2), ("qwen2.5-7b", 4),
                                          ("qwen2.5-7b", 8), ("qwen2.5-3b", 8), ("qwen3-4b", 8),
                                          ("tiny-qwen2", 2), ("tiny-qwen2", 4)])
def test_plan_covers_everything_once(preset, world):
    cfg = get_config(preset)
    plans = [tp_plan(cfg, world, r) for r in range(world)]
    qs = sorted(q for p in plans for q in p.q_heads)
    assert qs == list(range(cfg.n_heads))  # every query head on exactly one rank
    for p in plans:
        G = cfg.group
        assert all(q // G in p.kv_heads for q in p.q_heads)  # a query head sits with its KV head
        assert 1 <= len(p.q_heads) // len(p.kv_heads) <= 8
        assert p.kv_replicas == max(1, world // cfg.n_kv_heads)
    kvs = sorted(k for p in plans for k in p.kv_heads)
    assert kvs == sorted(list(range(cfg.n_kv_heads)) * max(1, world // cfg.n_kv_heads))
    for lo_key, hi_key, total in (("ffn_lo", "ffn_hi", cfg.ffn), ("vocab_lo", "vocab_hi", cfg.vocab)):
        spans = [(getattr(p, lo_key), getattr(p, hi_key)) for p in plans]
        assert spans[0][0] == 0 and spans[-1][1] == total
        assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
        assert all((hi - lo) % 128 == 0 and hi > lo for lo, hi in spans)
        sizes = [hi - lo for lo, hi in spans]
        assert max(sizes) - min(sizes) <= 128


def test_bad_world_sizes_are_rejected():
    with pytest.raises(ValueError):
        tp_plan(get_config("qwen2.5-7b"), 3, 0)  # 4 KV heads do not split over 3 ranks
    with pytest.raises(ValueError):
        tp_plan(get_config("tiny-qwen2"), 16, 0)  # 8 replicas of a KV head, 4 query heads each


@pytest.mark.parametrize("world", [2, 4])
def test_sharded_projections_sum_to_the_full_ones(world):
    cfg = get_config("tiny-qwen2").with_(n_layers=1, vocab=1024)
    w = {k: v.float() for k, v in init_weights(cfg, seed=3).items()}
    g = torch.Generator().manual_seed(0)
    x = torch.randn(3, cfg.hidden, generator=g)
    att = torch.randn(3, cfg.n_heads * cfg.head_dim, generator=g)
    act = torch.randn(3, cfg.ffn, generator=g)
    o_full = att @ w["l0.wo"].t()
    d_full = act @ w["l0.w_down"].t()
    o_sum = torch.zeros_like(o_full)
    d_sum = torch.zeros_like(d_full)
    logits = []
    for r in range(world):
        p = tp_plan(cfg, world, r)
        lc = local_config(cfg, p)
        s = shard_weights(cfg, w, p)
        assert s["l0.wq"].shape == (lc.n_heads * 128, cfg.hidden)
        assert s["l0.wk"].shape == (lc.n_kv_heads * 128, cfg.hidden)
        assert s["l0.w_gate"].shape == (lc.ffn, cfg.hidden) and s["l0.w_down"].shape == (cfg.hidden, lc.ffn)
        att_r = torch.cat([att[:, q * 128 : (q + 1) * 128] for q in p.q_heads], 1)
        o_sum += att_r @ s["l0.wo"].t()
        d_sum += act[:, p.ffn_lo : p.ffn_hi] @ s["l0.w_down"].t()
        # column-parallel q rows are the full projection's rows of the rank's heads
        q_full = x @ w["l0.wq"].t()
        q_r = x @ s["l0.wq"].t()
        for i, q in enumerate(p.q_heads):
            assert torch.allclose(q_r[:, i * 128 : (i + 1) * 128], q_full[:, q * 128 : (q + 1) * 128])
        logits.append(x @ s["lm_head"].t())
    assert torch.allclose(o_sum, o_full, atol=1e-4)
    assert torch.allclose(d_sum, d_full, atol=1e-4)
    assert torch.allclose(torch.cat(logits, 1), x @ w["lm_head"].t(), atol=1e-4)


def test_split_k_choices():
    """The split rule reproduces the burst sweep's best (or within a few %) choices."""
    from kvcacheboundaryprotection_b200.engine import CappedKVEngine

    cfg = get_config("qwen2.5-7b")
    H, F, V = cfg.hidden, cfg.ffn, cfg.vocab
    qkv_n = (cfg.n_heads + 2 * cfg.n_kv_heads) * cfg.head_dim
    pick = CappedKVEngine._pick_splits
    assert [pick(qkv_n, H), pick(H, H), pick(2 * F, H), pick(H, F), pick(V, H)] == [7, 8, 1, 8, 1]
    assert pick(128 * 148, H) == 2       # 148 tiles: exactly two CTAs per SM
    assert pick(128 * 149, H) == 1       # 149 tiles: any split adds a second wave
    assert pick(128 * 172, 2048) == 1    # the Qwen2.5-3B gate/up (measured 29.7 vs 33.8 us at 3)
    assert pick(128 * 297, H) == 2       # one tile past a whole wave (the TP=4 lm_head shard)
    assert pick(128 * 594, H) == 1
    assert pick(768, H) == 16            # 6 tiles (q/k/v at TP=8)
    # tensor parallel: each rank picks for its own shard
    from kvcacheboundaryprotection_b200.tp import allreduce_splits

    assert allreduce_splits(cfg, 2) == {"o": 8, "down": 8}
    assert allreduce_splits(cfg, 8, 0) == {"o": 4, "down": 8}  # 4 query heads on rank 0


def test_allreduce_slots_are_independent_of_the_call():
    """The o and down fused-allreduce GEMMs share one symmetric buffer with different
    split counts (7B at TP=8: 3 and 7).  Every (parity, source rank, row, column pair) has
    its own 16-byte slot inside the buffer; o (even call index) and down (odd) never share
    one, whatever their split counts, and the layout does not depend on the split count."""
    from kvcacheboundaryprotection_b200.tp import allreduce_buffer_bytes, allreduce_slot, allreduce_splits

    cfg = get_config("qwen2.5-7b")
    world, M, N = 8, 16, cfg.hidden
    sp = allreduce_splits(cfg, world)
    assert sp["o"] != sp["down"]  # the case that used to overlap
    size = allreduce_buffer_bytes(world, M, N)
    seen = set()
    for parity in (0, 1):
        for src in range(world):
            offs = [allreduce_slot(world, M, N, parity, src, r, c) for r in range(M) for c in range(0, N, 2)]
            assert len(set(offs)) == len(offs)
            assert all(o % 16 == 0 and 0 <= o and o + 16 <= size for o in offs)
            assert not (seen & set(offs))
            seen |= set(offs)
    assert len(seen) * 16 == size


def test_reference_tp_clamp_and_groups():
    """The tensor-parallel size follows the reference's clamp (jax_inference.py:1846-1861:
    the largest size <= the requested one dividing the query heads, the KV heads and the
    FFN width); the remaining factor of the world becomes data-parallel groups of
    consecutive ranks."""
    from kvcacheboundaryprotection_b200.tp import reference_tp_size, tp_groups

    q7, q4, q3 = get_config("qwen2.5-7b"), get_config("qwen3-4b"), get_config("qwen2.5-3b")
    assert [reference_tp_size(q7, n) for n in (1, 2, 4, 8)] == [1, 2, 4, 4]  # 4 KV heads
    assert [reference_tp_size(q4, n) for n in (1, 2, 4, 8)] == [1, 2, 4, 8]  # 8 KV heads
    assert [reference_tp_size(q3, n) for n in (1, 2, 4, 8)] == [1, 2, 2, 2]  # 2 KV heads
    assert tp_groups(8, 4) == [[0, 1, 2, 3], [4, 5, 6, 7]]
    assert tp_groups(4, 4) == [[0, 1, 2, 3]]
    with pytest.raises(ValueError):
        tp_groups(8, 3)
