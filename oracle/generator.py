"""Restatement of the reference's global-mask decode/eviction loop (test infrastructure).

Follows ``KVCoupledQwen35Generator.generate_with_kv_control`` and ``_maybe_evict``
(``src/counterfact_kv_eviction/kv_coupled_generator.py:135-604``), including the per-KV-head
mode of the faithful / native Ada-KV and QUEST policies (:216-325 at step 0, :373-433 in
the decode loop, signal updates :470-497).  The model is any callable with the JAX
adapter's signature (``src/counterfact_kv_eviction/jax_inference.py:1575-1583``).

On top of the reference behaviour it tracks the slot layout that the CUDA path
defines, since the reference keeps a position-indexed cache and has no slots:

* after the step-0 eviction the retained prompt positions occupy slots
  ``0..R-1`` in ascending position order, all other slots are free;
* each decode step's new position takes the lowest free slot *before* that step's
  cadence eviction;
* every victim's slot becomes free.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any, Dict, List, Optional, Sequence

import numpy as np

from .policies import (PER_HEAD_POLICIES, Meta, PolicySpec, canonical, hard_cap, per_head_uses_current,
                       protection_sizes, select_per_head_retention, union_trim)


@dataclass
class OracleResult:
    generated_token_ids: List[int]
    eviction_count: int
    positions_retained: int
    positions_evicted: List[int]
    retention_mask: List[bool]
    policy_call_steps: List[int]
    retained_counts_by_step: List[int]
    prefill_position_count: int
    # per decode step s (1-based, index s-1): victims chosen at that step
    victims_by_step: List[List[int]] = field(default_factory=list)
    # slot table (slot -> position, -1 = free) after step 0 and after each step's eviction
    slot_tables: List[np.ndarray] = field(default_factory=list)
    # per decode forward: the per-position score vector ks (float32) it produced
    step_scores: List[np.ndarray] = field(default_factory=list)
    # logits row used for sampling at each step (float32), when recorded
    step_logits: List[np.ndarray] = field(default_factory=list)
    meta: Optional[Meta] = None
    faithful_union_retained_max: int = 0
    faithful_union_overflow_max: int = 0
    faithful_union_overflow_steps: int = 0
    # per-head mode: the (n_kv_heads, positions) keep mask after each step's selection
    head_keep: Optional[np.ndarray] = None
    # per-head mode, per decode forward: the (n_kv_heads, n_pos) signal rows it produced
    step_head_scores: List[np.ndarray] = field(default_factory=list)


class SlotTable:
    """Slot <-> position map with the lowest-free-slot rule."""

    def __init__(self, n_slots: int):
        self.pos = np.full(n_slots, -1, np.int64)

    def compact(self, retained_sorted: Sequence[int]) -> None:
        if len(retained_sorted) > len(self.pos):
            raise ValueError("retained prompt positions exceed the slot count")
        self.pos[:] = -1
        self.pos[: len(retained_sorted)] = np.asarray(retained_sorted, np.int64)

    def assign(self, position: int) -> int:
        free = np.flatnonzero(self.pos < 0)
        if free.size == 0:
            raise ValueError("no free KV slot")
        s = int(free[0])
        self.pos[s] = position
        return s

    def release(self, position: int) -> None:
        hit = np.flatnonzero(self.pos == position)
        if hit.size:
            self.pos[hit[0]] = -1


def slot_count(capacity: int, evict_every: int, max_new_tokens: int, regime: str) -> int:
    """Slots a sequence needs under the lowest-free-slot rule."""
    if regime == "prefill":
        return capacity + max(1, max_new_tokens)
    return capacity + evict_every


def _per_key_max(attentions: Any, n: int) -> np.ndarray:
    """Max over every leading axis of the attention outputs (kv_coupled_generator.py:636-658)."""
    if attentions is None or len(attentions) == 0:
        return np.zeros(0, np.float32)
    rows = [np.asarray(a, np.float32).reshape(-1, np.asarray(a).shape[-1]) for a in attentions]
    return np.concatenate(rows, axis=0).max(axis=0)


def generate(
    model: Any,
    policy: PolicySpec,
    input_ids: Sequence[int],
    max_new_tokens: int,
    *,
    evict_every: int = 8,
    n_kv_heads: int = 0,
    eos_token_ids: Optional[set] = None,
    temperature: float = 0.0,
    rng: Optional[np.random.Generator] = None,
    regime: str = "decode",
    n_slots: Optional[int] = None,
    record_logits: bool = False,
    forced_tokens: Optional[Sequence[int]] = None,
) -> OracleResult:
    """Run the capped-cache decode loop; returns the reference's result fields.

    ``forced_tokens`` (teacher forcing, tests only) replaces the sampled token at
    step ``s`` by ``forced_tokens[s-1]``.
    """
    cap = int(policy.capacity)
    if cap <= 0:
        raise ValueError("capacity must be > 0")
    if evict_every <= 0:
        raise ValueError("evict_every_n_steps must be > 0")
    if regime not in ("decode", "prefill"):
        raise ValueError("eviction_regime must be 'decode' or 'prefill'")
    if max_new_tokens < 0:
        raise ValueError("max_new_tokens must be >= 0")
    if len(input_ids) == 0:
        raise ValueError("input_ids must be non-empty")

    n_prompt = len(input_ids)
    n_alloc = n_prompt + max_new_tokens + 2
    meta = Meta.zeros(n_alloc)
    retained = np.zeros(n_alloc, bool)
    evicted: List[int] = []
    calls: List[int] = []
    counts: List[int] = []
    victims_by_step: List[List[int]] = []
    slot_tables: List[np.ndarray] = []
    step_scores: List[np.ndarray] = []
    step_logits: List[np.ndarray] = []
    slots = SlotTable(n_slots or slot_count(cap, evict_every, max_new_tokens, regime))

    # per-KV-head mode (AdaKV / QUEST faithful and native), kv_coupled_generator.py:115-133
    per_head = canonical(policy.name) in PER_HEAD_POLICIES
    use_cur = per_head and per_head_uses_current(policy.name)
    ph_cumul = ph_cur = ph_keep = None
    ph_ready = False
    n_pref = n_suff = 0
    if per_head and policy.protect:
        n_pref, n_suff = protection_sizes(cap, policy.prefix_frac, policy.suffix_frac)
    if per_head and n_kv_heads > 0:
        ph_cumul = np.zeros((n_kv_heads, n_alloc), np.float64)
        ph_cur = np.zeros((n_kv_heads, n_alloc), np.float32)
        ph_keep = np.ones((n_kv_heads, n_alloc), bool)
    union_stats = [0, 0, 0]  # retained max, overflow max, overflow steps
    step_head_scores: List[np.ndarray] = []

    def per_head_select(step: int) -> List[int]:
        """One per-head policy call + union trim; returns the evicted positions (ascending)."""
        signal = ph_cur if use_cur else ph_cumul
        rmask = retained[:n_pos]
        keep = select_per_head_retention(policy.name, signal[:, :n_pos], rmask.tolist(), cap, n_pref, n_suff)
        n_union = int(keep.any(axis=0).sum())
        union_stats[0] = max(union_stats[0], n_union)
        union_stats[1] = max(union_stats[1], max(0, n_union - cap))
        union_stats[2] += int(n_union > cap)
        union = union_trim(keep, signal[:, :n_pos], rmask, cap, n_pref, n_suff)
        ph_keep[:, :n_pos] = keep
        out_v = [p for p in range(n_pos) if retained[p] and not union[p]]
        for p in out_v:
            retained[p] = False
        evicted.extend(out_v)
        calls.append(step)
        return out_v

    # --- prefill (kv_coupled_generator.py:160-209) ---------------------------------
    need_attn = canonical(getattr(policy, "name", "")) != "lru"
    out = model(input_ids=list(input_ids), output_attentions=need_attn, use_cache=True)
    past = out.past_key_values
    pre = _per_key_max(out.attentions, n_prompt)
    n_pre = min(len(pre), n_prompt)
    meta.attn[:n_pre] = pre[:n_pre]
    meta.max_attn[:n_pre] = pre[:n_pre]
    meta.cumul[:n_pre] = pre[:n_pre]
    meta.prefill[:n_pre] = pre[:n_pre]
    retained[:n_prompt] = True
    n_pos = n_prompt
    counts.append(n_pos)

    def evict(step: int, forced: bool) -> List[int]:
        """_maybe_evict (kv_coupled_generator.py:549-604)."""
        live = np.flatnonzero(retained[:n_pos]).tolist()
        if not (step % evict_every == 0 or (forced and len(live) > cap)):
            return []
        k = max(0, len(live) - cap)
        chosen = policy.select(live, meta, k, step)
        calls.append(step)
        out_v: List[int] = []
        for p in chosen:
            if 0 <= p < n_pos and retained[p]:
                retained[p] = False
                out_v.append(p)
        live = np.flatnonzero(retained[:n_pos]).tolist()
        for p in hard_cap(live, meta, len(live) - cap):
            retained[p] = False
            out_v.append(p)
        evicted.extend(out_v)
        return out_v

    if not per_head:
        evict(0, True)
    elif n_prompt > cap and ph_keep is not None:
        # step 0 per head: the first attention output seeds head 0's signal
        # (kv_coupled_generator.py:240-271: a (1, 1, 1, N) prefill array gives one row)
        raw = out.attentions
        if raw is not None and len(raw) > 0:
            arr = np.asarray(raw[0], np.float32)
            if arr.ndim == 4:
                arr = arr[0, :, -1, :]
            if arr.ndim == 2:
                hh, cc = min(arr.shape[0], n_kv_heads), min(arr.shape[1], n_prompt)
                if hh > 0 and cc > 0:
                    ph_cumul[:hh, :cc] += arr[:hh, :cc]
                    ph_cur[:hh, :cc] = arr[:hh, :cc]
                    ph_ready = True
        if not use_cur or ph_ready:
            per_head_select(0)
    if ph_keep is not None and evicted:
        ph_keep[:, evicted] = False
    slots.compact(np.flatnonzero(retained[:n_pos]).tolist())
    slot_tables.append(slots.pos.copy())
    counts.append(int(retained[:n_pos].sum()))

    generated = [int(t) for t in input_ids]
    last_logits = np.asarray(out.logits, np.float32)

    # --- decode loop (kv_coupled_generator.py:336-516) -----------------------------
    for step in range(1, max_new_tokens + 1):
        row = last_logits[0, -1]
        if record_logits:
            step_logits.append(row.copy())
        if temperature > 0.0 and rng is not None:
            z = row / temperature
            z -= z.max()
            prob = np.exp(z) / np.exp(z).sum()
            tok = int(rng.choice(len(prob), p=prob))
        else:
            tok = int(np.argmax(row))
        if forced_tokens is not None:
            tok = int(forced_tokens[step - 1])
        generated.append(tok)
        if eos_token_ids and tok in eos_token_ids:
            break

        new_pos = n_pos
        n_pos += 1
        retained[new_pos] = True
        meta.insert_step[new_pos] = step
        meta.last_access[new_pos] = step
        meta.access_count[new_pos] = 1
        slots.assign(new_pos)

        cadence = step % evict_every == 0
        if per_head and cadence and regime == "decode" and ph_keep is not None and (not use_cur or ph_ready):
            vict = per_head_select(step)
        else:
            vict = evict(step, False) if regime == "decode" else []
        if ph_keep is not None and vict:
            ph_keep[:, vict] = False
        for p in vict:
            slots.release(p)
        victims_by_step.append(vict)
        slot_tables.append(slots.pos.copy())
        counts.append(int(retained[:n_pos].sum()))

        if step == max_new_tokens:
            break

        if per_head and ph_keep is not None:
            mask_arg = ph_keep[:, :n_pos].astype(np.float32)
        elif n_kv_heads > 0:
            mask_arg = np.broadcast_to(retained[:n_pos].astype(np.float32), (n_kv_heads, n_pos)).copy()
        else:
            mask_arg = [1.0 if r else 0.0 for r in retained[:n_pos]]
        out = model(
            input_ids=[tok], past_key_values=past, attention_mask=mask_arg, output_attentions=True, use_cache=True
        )
        past = out.past_key_values
        last_logits = np.asarray(out.logits, np.float32)

        if per_head and out.attentions is not None and len(out.attentions) > 0:
            # per-head scores (Hq, C); rows 0..n_kv_heads-1 feed the per-head signals
            # (kv_coupled_generator.py:470-497: the first n_kv_heads QUERY heads)
            arr = np.asarray(out.attentions[0], np.float32)
            if ph_cumul is not None and arr.ndim == 2:
                hh, cc = min(arr.shape[0], n_kv_heads), min(arr.shape[1], n_pos)
                ph_cumul[:hh, :cc] += arr[:hh, :cc]
                ph_cur[:, :n_pos] = 0.0
                ph_cur[:hh, :cc] = arr[:hh, :cc]
                ph_ready = cc > 0
                step_head_scores.append(arr[:hh, :n_pos].copy())
            ks = arr.max(axis=0)[:n_pos].astype(np.float32)
        else:
            ks = _per_key_max(out.attentions, n_pos)[:n_pos].astype(np.float32)
        if ks.size:
            step_scores.append(ks.copy())
            rm = retained[:n_pos]
            top = float(ks.max())
            thr = np.float32(0.05 * top)
            meta.attn[:n_pos] = np.where(rm, ks, meta.attn[:n_pos])
            np.maximum(meta.max_attn[:n_pos], rm * ks, out=meta.max_attn[:n_pos])
            meta.cumul[:n_pos] += rm * ks
            hit = rm & (ks > thr)
            meta.last_access[:n_pos] = np.where(hit, np.int32(step), meta.last_access[:n_pos])
            meta.access_count[:n_pos] += hit.astype(np.int32)

    return OracleResult(
        generated_token_ids=generated,
        eviction_count=len(evicted),
        positions_retained=int(retained[:n_pos].sum()),
        positions_evicted=evicted,
        retention_mask=[bool(r) for r in retained[:n_pos]],
        policy_call_steps=calls,
        retained_counts_by_step=counts,
        prefill_position_count=n_prompt,
        victims_by_step=victims_by_step,
        slot_tables=slot_tables,
        step_scores=step_scores,
        step_logits=step_logits,
        meta=meta,
        faithful_union_retained_max=union_stats[0],
        faithful_union_overflow_max=union_stats[1],
        faithful_union_overflow_steps=union_stats[2],
        head_keep=None if ph_keep is None else ph_keep[:, :n_pos].copy(),
        step_head_scores=step_head_scores,
    )
