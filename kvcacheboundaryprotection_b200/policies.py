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
from typing import Any, Dict, List

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


def host_selected(policy: Any) -> bool:
    """True when the (possibly wrapped) policy picks its victims on the host."""
    return isinstance(getattr(policy, "inner", policy), RandomEvictionPolicy)


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
    if name == "streaming_sink_like":
        if getattr(inner, "sink_size", 4) != 4 or getattr(inner, "recent_window_size", capacity - 4) != max(0, capacity - 4):
            raise ValueError("streamingllm on the GPU path uses sink_size=4, recent_window_size=capacity-4")
        return "streamingllm"
    if name not in POLICY_IDS:
        raise ValueError(f"policy {name!r} is not available on the GPU path")
    return name
