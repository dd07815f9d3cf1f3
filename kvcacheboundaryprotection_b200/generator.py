"""Drop-in generator for the capped-KV decode loop, running on the GPU.

``KVCoupledQwen35Generator`` keeps the reference's constructor and
``generate_with_kv_control`` signature and returns the reference's
``KVCoupledGeneratorResult`` fields
(``src/counterfact_kv_eviction/kv_coupled_generator.py:28-51,84-547``).  The model
argument is a ``CappedKVModel`` (config + weights on the device).  Every step -- slot
allocation, cadence eviction, forward, greedy sampling, score update -- runs on the
device; the host replays one CUDA graph per step and reads the logs once at the end.
``generate_batch`` decodes several prompts of equal length in lockstep.

With ``eos_token_ids`` or ``temperature > 0`` the loop synchronises with the host
every step (EOS check / numpy sampling with the caller's ``rng``, exactly as the
reference samples), which is also how the end-to-end timing is taken.
"""

from __future__ import annotations

import time
from dataclasses import dataclass
from typing import Any, Dict, List, Optional, Sequence

import numpy as np
import torch

from .config import ModelConfig
from .engine import CappedKVEngine, EvictionSpec, FusedWeights
from .policies import host_selected, kernel_policy_name


@dataclass
class KVCoupledGeneratorResult:
    generated_token_ids: List[int]
    generated_text: str
    eviction_count: int
    positions_retained: int
    positions_evicted: List[int]
    retention_mask: List[bool]
    policy_call_steps: List[int]
    retained_counts_by_step: List[int]
    prefill_position_count: int
    faithful_union_retained_max: int = 0
    faithful_union_overflow_max: int = 0
    faithful_union_overflow_steps: int = 0
    policy_compute_time_s: float = 0.0
    prefill_wall_s: float = 0.0
    decode_phase_wall_s: float = 0.0
    decode_step_n: int = 0
    decode_step_mean_ms: float = 0.0
    decode_step_p50_ms: float = 0.0
    decode_step_p95_ms: float = 0.0
    decode_step_p99_ms: float = 0.0


class CappedKVModel:
    """Decoder config + weights resident on one GPU."""

    def __init__(self, cfg: ModelConfig, weights: Dict[str, torch.Tensor], device: Any = "cuda"):
        self.cfg = cfg
        self.config = cfg
        self.device = torch.device(device)
        self.weights = FusedWeights(cfg, weights, self.device)


def _percentiles(ms: List[float]):
    if not ms:
        return 0, 0.0, 0.0, 0.0, 0.0
    a = np.asarray(ms, np.float64)
    return int(a.size), float(a.mean()), float(np.percentile(a, 50)), float(np.percentile(a, 95)), float(np.percentile(a, 99))


class KVCoupledQwen35Generator:
    def __init__(
        self,
        model: CappedKVModel,
        tokenizer: Any,
        policy: Any,
        capacity: int,
        evict_every_n_steps: int = 8,
        n_kv_heads: int = 0,
        eviction_regime: str = "decode",
        use_graph: bool = True,
    ) -> None:
        if capacity <= 0:
            raise ValueError("capacity must be > 0")
        if evict_every_n_steps <= 0:
            raise ValueError("evict_every_n_steps must be > 0")
        if eviction_regime not in {"decode", "prefill"}:
            raise ValueError("eviction_regime must be 'decode' or 'prefill'")
        self.model = model
        self.tokenizer = tokenizer
        self.policy = policy
        self.capacity = int(capacity)
        self.evict_every_n_steps = int(evict_every_n_steps)
        self.eviction_regime = eviction_regime
        self.use_graph = use_graph
        protect = hasattr(policy, "inner")
        self.spec = EvictionSpec(
            policy=kernel_policy_name(policy, self.capacity),
            capacity=self.capacity,
            evict_every=self.evict_every_n_steps,
            protect=protect,
            prefix_frac=float(getattr(policy, "prefix_frac", 0.0)) if protect else 0.0,
            suffix_frac=float(getattr(policy, "suffix_frac", 0.0)) if protect else 0.0,
            regime=eviction_regime,
        )
        if protect:
            wcap = int(getattr(policy, "capacity", 0) or 0)
            if wcap <= 0:
                raise ValueError("ProtectedPolicyWrapper(capacity=0) sizes protection per call; pass capacity > 0")
            self.spec.protect_capacity = wcap
        self.last_engine: Optional[CappedKVEngine] = None

    # ------------------------------------------------------------------
    def generate_with_kv_control(
        self,
        input_ids: Sequence[int],
        max_new_tokens: int,
        eos_token_ids: Optional[set] = None,
        temperature: float = 0.0,
        rng: Optional[np.random.Generator] = None,
    ) -> KVCoupledGeneratorResult:
        return self.generate_batch([list(input_ids)], max_new_tokens, eos_token_ids, temperature, rng)[0]

    def generate_batch(
        self,
        batch_input_ids: Sequence[Sequence[int]],
        max_new_tokens: int,
        eos_token_ids: Optional[set] = None,
        temperature: float = 0.0,
        rng: Optional[np.random.Generator] = None,
        forced_tokens: Optional[np.ndarray] = None,
    ) -> List[KVCoupledGeneratorResult]:
        if max_new_tokens < 0:
            raise ValueError("max_new_tokens must be >= 0")
        if not batch_input_ids or any(len(x) == 0 for x in batch_input_ids):
            raise ValueError("input_ids must be non-empty")
        P = len(batch_input_ids[0])
        if any(len(x) != P for x in batch_input_ids):
            raise ValueError("generate_batch needs prompts of equal length")
        B = len(batch_input_ids)
        host_pol = self.policy if host_selected(self.policy) else None
        if host_pol is not None and B > 1:
            # one random stream consumed sequence after sequence, as the reference's loop does
            return [
                self.generate_batch([ids], max_new_tokens, eos_token_ids, temperature, rng,
                                    None if forced_tokens is None else forced_tokens[b : b + 1])[0]
                for b, ids in enumerate(batch_input_ids)
            ]
        eng = CappedKVEngine(
            self.model.cfg, self.model.weights, batch=B, evict=self.spec, max_prompt_len=P,
            max_new_tokens=max(1, max_new_tokens), device=self.model.device, host_policy=host_pol,
        )
        self.last_engine = eng
        ids = torch.tensor(np.asarray(batch_input_ids, np.int64), dtype=torch.int32)
        dev = self.model.device
        host_loop = (bool(eos_token_ids) or (temperature > 0.0 and rng is not None) or forced_tokens is not None
                     or host_pol is not None)

        torch.cuda.synchronize(dev)
        t0 = time.perf_counter()
        eng.prefill(ids)
        torch.cuda.synchronize(dev)
        prefill_s = time.perf_counter() - t0
        t1 = time.perf_counter()

        stop = [max_new_tokens] * B  # last step whose token was appended
        eos_tok: List[Optional[int]] = [None] * B
        step_ms: List[float] = []
        if max_new_tokens > 0:
            if host_loop:
                self._host_loop(eng, max_new_tokens, eos_token_ids, temperature, rng, forced_tokens, stop, eos_tok, step_ms)
            else:
                if self.use_graph and max_new_tokens > 1:
                    eng.capture()
                ev = [torch.cuda.Event(enable_timing=True) for _ in range(max_new_tokens)]
                ev[0].record()
                for s in range(1, max_new_tokens):
                    eng.run_step(use_graph=self.use_graph)
                    ev[s].record()
                eng.final_step()
                torch.cuda.synchronize(dev)
                step_ms = [ev[s - 1].elapsed_time(ev[s]) for s in range(1, max_new_tokens)]
        torch.cuda.synchronize(dev)
        decode_s = time.perf_counter() - t1
        eng.check_device_errors()
        return [self._assemble(eng, b, batch_input_ids[b], max_new_tokens, stop[b], eos_tok[b], prefill_s, decode_s, step_ms) for b in range(B)]

    # ------------------------------------------------------------------
    def _host_loop(self, eng, max_new, eos, temperature, rng, forced, stop, eos_tok, step_ms):
        """Per-step host synchronisation: EOS checks, numpy temperature sampling or forced tokens."""
        B = eng.B
        tok_host = torch.empty(B, dtype=torch.int32, pin_memory=True)
        active = [True] * B
        for s in range(1, max_new + 1):
            # token for step s: sampled from the logits of the previous forward
            if temperature > 0.0 and rng is not None:
                rows = eng.logits.float().cpu().numpy()
                for b in range(B):
                    z = rows[b] / temperature
                    z -= z.max()
                    p = np.exp(z) / np.exp(z).sum()
                    tok_host[b] = int(rng.choice(len(p), p=p))
                eng.tokens.copy_(tok_host, non_blocking=True)
            if forced is not None:
                tok_host.copy_(torch.from_numpy(np.asarray(forced[:, s - 1], np.int32)))
                eng.tokens.copy_(tok_host, non_blocking=True)
            if eos:
                tok_host.copy_(eng.tokens, non_blocking=True)
                torch.cuda.current_stream(eng.dev).synchronize()
                for b in range(B):
                    if active[b] and int(tok_host[b]) in eos:
                        active[b] = False
                        stop[b] = s - 1
                        eos_tok[b] = int(tok_host[b])
                if not any(active):
                    return
            t = time.perf_counter()
            if s == max_new:
                eng.final_step()
            else:
                eng.run_step(use_graph=False)
                torch.cuda.current_stream(eng.dev).synchronize()
                step_ms.append((time.perf_counter() - t) * 1000.0)

    def _assemble(self, eng, b, prompt, max_new, stop, eos_tok, prefill_s, decode_s, step_ms) -> KVCoupledGeneratorResult:
        P = len(prompt)
        E = self.evict_every_n_steps
        tokens = eng.token_log[b].cpu().numpy().tolist()[:stop] if max_new > 0 else []
        retained = eng.retained_log[b].cpu().numpy().tolist()  # index s: after step s
        evlog = eng.evlog[b].cpu().numpy()
        evcount = int(eng.evcount[b].item())
        # evictions up to and including step ``stop``
        n0 = P - retained[0] if max_new >= 0 else 0
        n_ev = n0
        for s in range(1, stop + 1):
            n_ev += retained[s - 1] + 1 - retained[s]
        n_ev = min(n_ev, evcount)
        evicted = [int(x) for x in evlog[:n_ev]]
        n_pos = P + stop
        mask = np.ones(n_pos, bool)
        mask[evicted] = False
        if getattr(eng, "per_head", False):  # the per-head branch records only the calls it made
            calls = [s for s in eng.head_call_steps if s <= stop]
        else:
            calls = [0] + ([s for s in range(1, stop + 1) if s % E == 0] if self.eviction_regime == "decode" else [])
        gen = [int(t) for t in prompt] + [int(t) for t in tokens]
        if eos_tok is not None:
            gen.append(int(eos_tok))
        text = ""
        if self.tokenizer is not None and hasattr(self.tokenizer, "decode"):
            text = str(self.tokenizer.decode(gen))
        n, m, p50, p95, p99 = _percentiles(step_ms)
        return KVCoupledGeneratorResult(
            generated_token_ids=gen,
            generated_text=text,
            eviction_count=len(evicted),
            positions_retained=int(mask.sum()),
            positions_evicted=evicted,
            retention_mask=mask.tolist(),
            policy_call_steps=calls,
            retained_counts_by_step=[P] + [int(x) for x in retained[: stop + 1]],
            prefill_position_count=P,
            prefill_wall_s=prefill_s,
            decode_phase_wall_s=decode_s,
            decode_step_n=n,
            decode_step_mean_ms=m,
            decode_step_p50_ms=p50,
            decode_step_p95_ms=p95,
            decode_step_p99_ms=p99,
            **({"faithful_union_retained_max": eng.union_stats[0], "faithful_union_overflow_max": eng.union_stats[1],
                "faithful_union_overflow_steps": eng.union_stats[2]} if getattr(eng, "per_head", False) else {}),
        )
