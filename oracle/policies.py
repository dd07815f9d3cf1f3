"""Restatement of the reference's global eviction policies (test infrastructure).

Per-position metadata is held in numpy arrays indexed by absolute position (the
reference keeps one ``KVBlockMetadata`` object per position keyed by
``str(position)``, ``src/counterfact_kv_eviction/kv_coupled_generator.py:69-81``).
Every policy here ranks candidates by a composite key and evicts the ``k`` smallest,
returned in ascending key order -- the behaviour of ``_top_k_smallest_keys`` /
``heapq.nsmallest`` (``src/counterfact_kv_eviction/policies.py:12-63``).  The last key
component is the decimal string of the position, so ties between equal numeric
components fall back to *string* order ("100" < "11" < "9").
"""

from __future__ import annotations

import random
from dataclasses import dataclass, field
from typing import Callable, Dict, List, Optional, Sequence

import numpy as np

# Name used on the command line -> canonical reference policy name.  "attention-mass"
# is the cumulative-attention-mass policy, which the reference calls "h2o_faithful"
# (policies.py:1338-1367).
ALIASES = {"attention-mass": "h2o_faithful", "attention_mass": "h2o_faithful"}

GLOBAL_POLICIES = (
    "lru",
    "h2o_faithful",
    "h2o",
    "snapkv",
    "snapkv_faithful",
    "adakv",
    "quest",
    "streamingllm",
    "random",
)


def canonical(name: str) -> str:
    return ALIASES.get(name, name)


@dataclass
class Meta:
    """Per-position metadata arrays (index = absolute position)."""

    insert_step: np.ndarray  # int32
    last_access: np.ndarray  # int32
    access_count: np.ndarray  # int32
    attn: np.ndarray  # float32, latest per-step score
    max_attn: np.ndarray  # float32, running max of per-step scores
    cumul: np.ndarray  # float64, sum of per-step scores
    prefill: np.ndarray  # float32, prefill score

    @classmethod
    def zeros(cls, n: int) -> "Meta":
        return cls(
            insert_step=np.zeros(n, np.int32),
            last_access=np.zeros(n, np.int32),
            access_count=np.ones(n, np.int32),
            attn=np.zeros(n, np.float32),
            max_attn=np.zeros(n, np.float32),
            cumul=np.zeros(n, np.float64),
            prefill=np.zeros(n, np.float32),
        )


def _signal(m: Meta, p: int) -> float:
    # max(attention_score, max_attention_score), policies.py:66-67
    return max(float(m.attn[p]), float(m.max_attn[p]))


def _key_fn(policy: str, m: Meta, step: int) -> Callable[[int], tuple]:
    """Composite eviction key for one position (smaller = evicted first)."""
    if policy == "lru":  # policies.py:181-196
        return lambda p: (int(m.last_access[p]), int(m.insert_step[p]), str(p))
    if policy == "h2o_faithful":  # policies.py:1338-1367
        return lambda p: (float(m.cumul[p]), int(m.last_access[p]), int(m.insert_step[p]), str(p))
    if policy == "h2o":  # HeavyHitterH2OLikePolicy, policies.py:1190-1218

        def k(p: int) -> tuple:
            recent = 1.0 if (step - int(m.last_access[p])) <= 64 else 0.0
            keep = 0.7 * float(m.cumul[p]) + 0.1 * _signal(m, p) + 1.0 * recent
            return (keep, int(m.last_access[p]), int(m.insert_step[p]), str(p))

        return k
    if policy == "snapkv":  # policies.py:1267-1299
        return lambda p: (float(m.cumul[p]) + _signal(m, p), int(m.last_access[p]), str(p))
    if policy == "snapkv_faithful":  # policies.py:1302-1335
        return lambda p: (float(m.prefill[p]), int(m.last_access[p]), str(p))
    if policy == "adakv":  # AdaKVPolicy alpha=0.5, policies.py:1375-1412
        return lambda p: (float(m.cumul[p]) + 0.5 * float(m.max_attn[p]), int(m.last_access[p]), str(p))
    if policy in ("quest", "quest_faithful", "quest_native"):  # policies.py:1415-1449, fallback :1467-1478
        return lambda p: (float(m.attn[p]), int(m.last_access[p]), str(p))
    if policy in ("adakv_faithful", "adakv_native"):  # global fallback, policies.py:1600-1612
        return lambda p: (float(m.cumul[p]), int(m.last_access[p]), str(p))
    raise ValueError(f"unknown policy {policy!r}")


def smallest(positions: Sequence[int], k: int, key: Callable[[int], tuple]) -> List[int]:
    """The k smallest positions by ``key``, ascending (policies.py:12-27,48-63)."""
    if k <= 0 or not positions:
        return []
    return sorted(positions, key=key)[:k]


def inner_select(policy: str, positions: Sequence[int], m: Meta, k: int, step: int, capacity: int,
                 rng: Optional[random.Random] = None) -> List[int]:
    """One call of the unwrapped policy's ``select_evictions``."""
    policy = canonical(policy)
    if policy == "random":
        # RandomEvictionPolicy (policies.py:1553-1582): the policy's own Random(42) stream,
        # ``sample`` over the candidate keys in the order given (ascending positions)
        k = min(max(0, k), len(positions))
        if k <= 0:
            return []
        return [int(x) for x in rng.sample([str(p) for p in positions], k)]
    if policy == "streamingllm":
        # StreamingSinkLikePolicy(sink_size=4, recent_window_size=max(0, capacity-4)),
        # policies.py:1221-1264 with the CLI's construction at run_v3_jax.py:504-507.
        if k <= 0 or not positions:
            return []
        sink = smallest(positions, 4, lambda p: (int(m.insert_step[p]), str(p)))
        recent_n = max(0, capacity - 4)
        by_recent = sorted(
            positions, key=lambda p: (int(m.last_access[p]), int(m.insert_step[p]), str(p)), reverse=True
        )[:recent_n]
        keep = set(sink) | set(by_recent)
        cand = [p for p in positions if p not in keep] or list(positions)
        return smallest(cand, k, lambda p: (int(m.last_access[p]), int(m.insert_step[p]), str(p)))
    return smallest(positions, k, _key_fn(policy, m, step))


def protection_sizes(capacity: int, prefix_frac: float, suffix_frac: float) -> tuple[int, int]:
    """(prefix, suffix) protected counts, run_v3_jax.py:119-121 (Python float math)."""
    n_pre = max(4, int(capacity * prefix_frac)) if prefix_frac > 0 else 0
    n_suf = max(4, int(capacity * suffix_frac)) if suffix_frac > 0 else 0
    return n_pre, n_suf


@dataclass
class PolicySpec:
    """A policy plus the optional structural-protection wrapper.

    Mirrors ``ProtectedPolicyWrapper`` (run_v3_jax.py:102-136) when ``protect`` is true.
    """

    name: str
    capacity: int
    protect: bool = False
    prefix_frac: float = 0.10
    suffix_frac: float = 0.10
    rng: Optional[random.Random] = field(default=None, init=False, repr=False)

    def __post_init__(self) -> None:
        if canonical(self.name) == "random":  # one stream per policy object, seed 42
            self.rng = random.Random(42)

    def select(self, positions: Sequence[int], m: Meta, evict_count: int, step: int) -> List[int]:
        if not self.protect:
            return inner_select(self.name, positions, m, evict_count, step, self.capacity, self.rng)
        if evict_count <= 0 or not positions:
            return []
        cap = self.capacity if self.capacity > 0 else len(positions)
        n_pre, n_suf = protection_sizes(cap, self.prefix_frac, self.suffix_frac)
        ordered = sorted(int(p) for p in positions)
        prot = set(ordered[:n_pre])
        # ``all_positions[-n_suf:]``: with n_suf == 0 this slice is the WHOLE list, so a
        # zero suffix fraction protects every position (reference behaviour, kept).
        prot.update(ordered[-n_suf:])
        eligible = [p for p in positions if p not in prot]
        if not eligible:
            return []
        return inner_select(self.name, eligible, m, min(evict_count, len(eligible)), step, self.capacity, self.rng)


def hard_cap(retained: Sequence[int], m: Meta, overflow: int) -> List[int]:
    """Guardrail victims, kv_coupled_generator.py:588-604: (last, insert, int pos) order."""
    if overflow <= 0:
        return []
    order = sorted(retained, key=lambda p: (int(m.last_access[p]), int(m.insert_step[p]), int(p)))
    return order[:overflow]


# ---- per-KV-head ("faithful" / "native") policies -----------------------------------
# AdaKVFaithfulPolicy / AdaKVNativePolicy (policies.py:1585-1672, helpers :69-178) and
# QUESTFaithfulPolicy / QUESTNativePolicy (:1452-1551).  Each KV head keeps its own top-k
# positions by a per-head signal; the generator evicts what no head keeps.
PER_HEAD_POLICIES = ("adakv_faithful", "adakv_native", "quest_faithful", "quest_native")


def per_head_uses_current(name: str) -> bool:
    """QUEST ranks by the latest step's per-head attention, Ada-KV by the cumulative one."""
    return canonical(name).startswith("quest")


def _prefix_suffix(retained: np.ndarray, n_prefix: int, n_suffix: int) -> np.ndarray:
    """Positions 0..n_prefix-1 and the n_suffix highest retained positions."""
    prot = np.zeros(retained.shape[0], bool)
    prot[:n_prefix] = True
    if n_suffix > 0:
        live = np.flatnonzero(retained)
        if live.size:
            prot[live[-n_suffix:]] = True
    return prot


def adakv_budgets(head_attn: np.ndarray, budget: int, native: bool) -> np.ndarray:
    """Per-head budgets (policies.py:95-125): the same budget for every head (native), or a
    shared budget split by inverse attention entropy, each head at least 1."""
    H = head_attn.shape[0]
    if budget <= 0 or H <= 0:
        return np.zeros(H, dtype=int)
    if native:
        return np.full(H, budget, dtype=int)
    total = budget * H
    probs = head_attn / np.maximum(head_attn.sum(axis=1, keepdims=True), 1e-12)
    ent = -np.sum(probs * np.log(np.maximum(probs, 1e-12)), axis=1)
    inv = 1.0 / np.maximum(ent, 1e-6)
    out = np.maximum(np.round(inv / inv.sum() * total).astype(int), 1)
    while out.sum() > total:
        out[np.argmax(out)] -= 1
    while out.sum() < total:
        out[np.argmin(out)] += 1
    return out


def select_per_head_retention(name: str, signal: np.ndarray, retention_mask: Sequence[bool], capacity: int,
                              n_prefix: int, n_suffix: int) -> np.ndarray:
    """(n_kv_heads, n_positions) keep mask of one per-head policy call."""
    name = canonical(name)
    H, n = signal.shape
    retained = np.array(list(retention_mask)[:n], dtype=bool)
    prot_raw = _prefix_suffix(retained, n_prefix, n_suffix)
    if name.startswith("adakv"):
        prot = prot_raw & retained
        budget = max(0, int(capacity) - int(prot.sum()))
        evictable_mask = retained & ~prot
    else:  # quest: the budget counts the raw protected set
        prot = prot_raw & retained
        budget = max(0, int(capacity) - int(prot_raw.sum()))
        evictable_mask = retained & ~prot_raw
    keep = np.tile(prot, (H, 1))
    if budget <= 0:
        return keep
    ev = np.flatnonzero(evictable_mask)
    if ev.size == 0:
        return keep
    if name.startswith("adakv"):
        budgets = adakv_budgets(signal[:, ev], budget, native=(name == "adakv_native"))
    else:
        budgets = np.full(H, budget, dtype=int)
    for h in range(H):
        b_h = min(int(budgets[h]), ev.size)
        if b_h >= ev.size:
            keep[h, ev] = True
            continue
        top = np.argpartition(signal[h, ev], -b_h)[-b_h:]
        keep[h, ev[top]] = True
    return keep


def union_trim(keep: np.ndarray, signal: np.ndarray, retained: np.ndarray, capacity: int, n_prefix: int,
               n_suffix: int) -> np.ndarray:
    """Global retention = union of the heads' keep masks, trimmed to capacity by fewest
    votes then lowest summed signal (kv_coupled_generator.py:398-427); modifies ``keep``."""
    union = keep.any(axis=0)
    n_union = int(union.sum())
    if n_union > capacity:
        n = keep.shape[1]
        prot = np.zeros(n, bool)
        prot[:n_prefix] = True
        if n_suffix > 0:
            live = np.flatnonzero(retained[:n])
            if live.size >= n_suffix:
                prot[live[-n_suffix:]] = True
        cand = np.flatnonzero(union & ~prot)
        if cand.size:
            votes = keep[:, cand].sum(axis=0).astype(np.float64)
            attn = signal[:, cand].sum(axis=0)
            order = np.lexsort((attn, votes))
            trim = cand[order[: min(n_union - capacity, cand.size)]]
            union[trim] = False
            keep[:, trim] = False
    return union
