"""Policy objects with the reference's names and constructor arguments.

The scored policies carry configuration only: their victim selection runs on the GPU in
``kvbp_append_evict`` / ``kvbp_prefill_select``.  ``RandomEvictionPolicy`` is the
exception: its victims are Python ``random.Random(seed).sample`` draws over the eligible
keys, so it (and ``ProtectedPolicyWrapper`` around it) selects on the host through the
reference's ``select_evictions(blocks, evict_count, step)`` protocol and the engine
hands the victims to ``kvbp_append_evict_listed``.  Names, defaults and the protection
wrapper follow ``src/counterfact_kv_eviction/policies.py`` and
``scripts/run_v3_jax.py:102-136,500-527``.  ``"attention-mass"`` is accepted as the
name of the pure cumulative-attention-mass policy (``h2o_faithful``).
"""

from __future__ import annotations

import random
from dataclasses import dataclass, field
from typing import Any, Dict, List, Sequence

import numpy as np

from .capi import POLICY_IDS, protection_sizes


@dataclass
class LRUPolicy:
    name: str = "lru"


@dataclass
class H2OFaithfulPolicy:
    name: str = "h2o_faithful"


@dataclass
class HeavyHitterH2OLikePolicy:
    heavy_hitter_weight: float = 0.7
    attention_weight: float = 0.1
    recent_window: int = 64
    recent_bonus: float = 1.0
    name: str = "h2o"

    def __post_init__(self):
        if (self.heavy_hitter_weight, self.attention_weight, self.recent_window, self.recent_bonus) != (0.7, 0.1, 64, 1.0):
            raise ValueError("the CUDA kernel implements the reference defaults (0.7, 0.1, 64, 1.0) only")


@dataclass
class SnapKVPolicy:
    name: str = "snapkv"


@dataclass
class SnapKVFaithfulPolicy:
    name: str = "snapkv_faithful"


@dataclass
class AdaKVPolicy:
    alpha: float = 0.5
    name: str = "adakv"

    def __post_init__(self):
        if self.alpha != 0.5:
            raise ValueError("the CUDA kernel implements alpha = 0.5 (the reference default) only")


@dataclass
class QUESTPolicy:
    name: str = "quest"


@dataclass
class StreamingSinkLikePolicy:
    sink_size: int = 4
    recent_window_size: int = 8
    name: str = "streaming_sink_like"


@dataclass
class RandomEvictionPolicy:
    """Uniform random eviction (policies.py:1553-1582).  One ``random.Random(seed)`` stream
    per policy object, consumed across calls (and across the sequences a generator decodes
    with this object, one after another); each call samples ``min(evict_count, len(blocks))``
    keys in the blocks' order.  The draws must be Python's own to match the reference bit
    for bit, so this runs on the host."""

    seed: int = 42
    name: str = "random"
    _rng: random.Random = field(init=False, repr=False, compare=False)

    def __post_init__(self) -> None:
        self._rng = random.Random(self.seed)

    def select_evictions(self, blocks: Dict[str, Any], evict_count: int, step: int) -> List[str]:
        k = min(max(0, int(evict_count)), len(blocks))
        if k <= 0:
            return []
        return self._rng.sample(list(blocks.keys()), k)


class ProtectedPolicyWrapper:
    """Excludes the lowest/highest retained positions from eviction (run_v3_jax.py:102-136).
    The scored policies apply it on the GPU from (prefix_frac, suffix_frac, capacity);
    ``select_evictions`` is the host form, used around host-side inner policies."""

    def __init__(self, inner_policy: Any, prefix_frac: float = 0.10, suffix_frac: float = 0.10, capacity: int = 0):
        self.inner = inner_policy
        self.name = f"protected-{inner_policy.name}"
        self.prefix_frac = prefix_frac
        self.suffix_frac = suffix_frac
        self.capacity = capacity

    def select_evictions(self, blocks: Dict[str, Any], evict_count: int, step: int) -> List[str]:
        if evict_count <= 0 or not blocks:
            return []
        cap = self.capacity if self.capacity > 0 else len(blocks)
        n_pre, n_suf = protection_sizes(cap, self.prefix_frac, self.suffix_frac)
        ordered = sorted(int(k) for k in blocks)
        protected = {str(p) for p in ordered[:n_pre]}
        protected.update(str(p) for p in ordered[-n_suf:])  # n_suf == 0: the whole list
        eligible = {k: v for k, v in blocks.items() if k not in protected}
        if not eligible:
            return []
        return self.inner.select_evictions(eligible, min(evict_count, len(eligible)), step)


# ---- per-KV-head policies -------------------------------------------------------------
# Each KV head keeps its own top-k positions by a per-head signal; the generator evicts
# what no head keeps.  The selection is numpy on the host, with the reference's numpy
# operations in the same order (np.argpartition's choice among equal signals -- e.g. the
# all-zero rows of heads 1.. at step 0 -- is part of the result), over signals the GPU
# accumulates per slot; the GPU applies the per-head masks in attention and frees the
# victims' slots.


def _protected(retained: np.ndarray, n_prefix: int, n_suffix: int) -> np.ndarray:
    """Positions 0..n_prefix-1 and the n_suffix highest retained positions."""
    prot = np.zeros(retained.shape[0], dtype=bool)
    prot[:n_prefix] = True
    if n_suffix > 0:
        live = np.where(retained)[0]
        if len(live) > 0:
            prot[live[-n_suffix:]] = True
    return prot


def _top_b_per_head(signal: np.ndarray, evictable: np.ndarray, budgets, keep: np.ndarray) -> None:
    for h in range(signal.shape[0]):
        b_h = min(int(budgets[h]), len(evictable))
        if b_h >= len(evictable):
            keep[h, evictable] = True
            continue
        top = np.argpartition(signal[h, evictable], -b_h)[-b_h:]
        keep[h, evictable[top]] = True


@dataclass
class AdaKVFaithfulPolicy:
    """Ada-KV with per-head budgets (policies.py:1585-1642, :95-178): a shared budget of
    (capacity - protected) per head is split across heads by inverse attention entropy
    of the cumulative per-head signal; each head keeps its top-B_h."""

    name: str = "adakv_faithful"
    static_suffix_mode: bool = False
    native_per_head = False

    def __post_init__(self):
        if self.static_suffix_mode:
            raise ValueError("static_suffix_mode is not supported on the GPU path")

    def _budgets(self, head_attn: np.ndarray, budget: int) -> np.ndarray:
        H = head_attn.shape[0]
        if budget <= 0 or H <= 0:
            return np.zeros(H, dtype=int)
        if self.native_per_head:
            return np.full(H, budget, dtype=int)
        total = budget * H
        row = np.maximum(head_attn.sum(axis=1, keepdims=True), 1e-12)
        probs = head_attn / row
        ent = -np.sum(probs * np.log(np.maximum(probs, 1e-12)), axis=1)
        inv = 1.0 / np.maximum(ent, 1e-6)
        b = np.maximum(np.round(inv / inv.sum() * total).astype(int), 1)
        while b.sum() > total:
            b[np.argmax(b)] -= 1
        while b.sum() < total:
            b[np.argmin(b)] += 1
        return b

    def select_per_head_retention(self, per_head_cumul_attn: np.ndarray, retention_mask: Sequence[bool],
                                  capacity: int, n_protected: int = 0, n_suffix_protected: int = 0,
                                  orig_prompt_len: int = 0) -> np.ndarray:
        H, n = per_head_cumul_attn.shape
        retained = np.array(list(retention_mask)[:n], dtype=bool)
        prot = _protected(retained, n_protected, n_suffix_protected) & retained
        keep = np.tile(prot, (H, 1))
        budget = max(0, int(capacity) - int(prot.sum()))
        ev = np.where(retained & ~prot)[0]
        if budget <= 0 or len(ev) == 0:
            return keep
        _top_b_per_head(per_head_cumul_attn, ev, self._budgets(per_head_cumul_attn[:, ev], budget), keep)
        return keep


@dataclass
class AdaKVNativePolicy(AdaKVFaithfulPolicy):
    """Ada-KV with the full unprotected budget for every head (policies.py:1645-1672)."""

    name: str = "adakv_native"
    native_per_head = True


@dataclass
class QUESTFaithfulPolicy:
    """QUEST per head (policies.py:1452-1538): each head keeps its top (capacity -
    protected) positions by the latest step's per-head attention."""

    name: str = "quest_faithful"
    static_suffix_mode: bool = False

    def __post_init__(self):
        if self.static_suffix_mode:
            raise ValueError("static_suffix_mode is not supported on the GPU path")

    def select_per_head_retention(self, per_head_attn: np.ndarray, retention_mask: Sequence[bool], capacity: int,
                                  n_protected: int = 0, n_suffix_protected: int = 0,
                                  orig_prompt_len: int = 0) -> np.ndarray:
        H, n = per_head_attn.shape
        retained = np.array(list(retention_mask)[:n], dtype=bool)
        prot = _protected(retained, n_protected, n_suffix_protected)
        keep = np.tile(prot & retained, (H, 1))
        budget = max(0, int(capacity) - int(prot.sum()))  # the raw protected count
        ev = np.where(retained & ~prot)[0]
        if budget <= 0 or len(ev) == 0:
            return keep
        _top_b_per_head(per_head_attn, ev, [budget] * H, keep)
        return keep


@dataclass
class QUESTNativePolicy(QUESTFaithfulPolicy):
    """Named alias of QUESTFaithfulPolicy (policies.py:1541-1550)."""

    name: str = "quest_native"


def union_trim(keep: np.ndarray, signal: np.ndarray, retained: np.ndarray, capacity: int, n_prefix: int,
               n_suffix: int) -> np.ndarray:
    """Global retention = the heads' union, trimmed to ``capacity`` by fewest votes, then
    lowest summed signal, outside the prefix/suffix (kv_coupled_generator.py:398-427).
    Clears trimmed positions in ``keep`` too; returns the union."""
    union = keep.any(axis=0)
    n_union = int(union.sum())
    if n_union > capacity:
        n = keep.shape[1]
        prot = np.zeros(n, dtype=bool)
        prot[:n_prefix] = True
        if n_suffix > 0:
            live = np.where(retained[:n])[0]
            if len(live) >= n_suffix:
                prot[live[-n_suffix:]] = True
        cand = np.where(union & ~prot)[0]
        if len(cand) > 0:
            votes = keep[:, cand].sum(axis=0).astype(np.float64)
            attn = signal[:, cand].sum(axis=0)
            order = np.lexsort((attn, votes))
            trim = cand[order[: min(n_union - capacity, len(cand))]]
            union[trim] = False
            keep[:, trim] = False
    return union


PER_HEAD_CLASSES = (AdaKVFaithfulPolicy, QUESTFaithfulPolicy)


def per_head(policy: Any) -> bool:
    """True for the per-KV-head (faithful / native) Ada-KV and QUEST policies."""
    return isinstance(getattr(policy, "inner", policy), PER_HEAD_CLASSES)


def host_selected(policy: Any) -> bool:
    """True when the (possibly wrapped) policy picks its victims on the host."""
    return isinstance(getattr(policy, "inner", policy), RandomEvictionPolicy) or per_head(policy)


def policy_from_name(name: str, capacity: int) -> Any:
    """The CLI's policy_map (run_v3_jax.py:500-518) for the GPU-supported policies."""
    table = {
        "lru": LRUPolicy,
        "h2o_faithful": H2OFaithfulPolicy,
        "attention-mass": H2OFaithfulPolicy,
        "attention_mass": H2OFaithfulPolicy,
        "h2o": HeavyHitterH2OLikePolicy,
        "snapkv": SnapKVPolicy,
        "snapkv_faithful": SnapKVFaithfulPolicy,
        "adakv": AdaKVPolicy,
        "quest": QUESTPolicy,
        "random": RandomEvictionPolicy,
        "adakv_faithful": AdaKVFaithfulPolicy,
        "adakv_native": AdaKVNativePolicy,
        "quest_faithful": QUESTFaithfulPolicy,
        "quest_native": QUESTNativePolicy,
    }
    if name == "streamingllm":
        return StreamingSinkLikePolicy(sink_size=4, recent_window_size=max(0, capacity - 4))
    if name not in table:
        raise ValueError(f"policy {name!r} is not available on the GPU path; supported: {sorted(POLICY_IDS)}")
    return table[name]()


def kernel_policy_name(policy: Any, capacity: int) -> str:
    """Canonical kernel policy name of a (possibly wrapped) policy object."""
    inner = getattr(policy, "inner", policy)
    name = inner.name
    if isinstance(inner, QUESTFaithfulPolicy):
        return "quest"  # the device key of its global fallback call (policies.py:1467-1478)
    if isinstance(inner, AdaKVFaithfulPolicy):
        return "quest"  # never called globally: the cumulative signal always exists
    if name == "streaming_sink_like":
        if getattr(inner, "sink_size", 4) != 4 or getattr(inner, "recent_window_size", capacity - 4) != max(0, capacity - 4):
            raise ValueError("streamingllm on the GPU path uses sink_size=4, recent_window_size=capacity-4")
        return "streamingllm"
    if name not in POLICY_IDS:
        raise ValueError(f"policy {name!r} is not available on the GPU path")
    return name
