"""Deterministic score source with the JAX adapter's call signature (test infrastructure).

``StubScoreModel`` stands in for ``JAXModelAdapter.__call__``
(``src/counterfact_kv_eviction/jax_inference.py:1575-1790``) when only the
decode/eviction loop is under test: it returns seeded logits and per-key attention
probabilities whose shapes follow the adapter exactly --

* prefill with ``output_attentions``: one ``(1, 1, 1, N)`` array per layer, zero at
  positions >= the prompt length (jax_inference.py:1777-1789);
* decode with a 2-D ``(n_kv_heads, n_pos)`` mask: ``[(Hq, N)]`` per-head scores
  (jax_inference.py:1666-1673); with a 1-D mask: ``[(1, 1, 1, N)]``.

Masked columns get probability exactly 0, as the real softmax gives them
(``exp(-1e9 - m)`` underflows to 0 in float32).
"""

from __future__ import annotations

from typing import Any, List, Optional, Sequence

import numpy as np


class _Out:
    def __init__(self, logits, past_key_values, attentions):
        self.logits = logits
        self.past_key_values = past_key_values
        self.attentions = attentions


class StubScoreModel:
    def __init__(
        self,
        *,
        vocab: int = 512,
        n_heads: int = 4,
        n_kv_heads: int = 2,
        n_layers: int = 2,
        max_cache_len: int = 4096,
        seed: int = 0,
        spread: float = 2.0,
    ):
        self.vocab = vocab
        self.n_heads = n_heads
        self.n_kv_heads = n_kv_heads
        self.n_layers = n_layers
        self.max_cache_len = max_cache_len
        self.seed = seed
        self.spread = spread
        self.calls = 0

    def _rng(self) -> np.random.Generator:
        self.calls += 1
        return np.random.default_rng([self.seed, self.calls])

    def __call__(
        self,
        *,
        input_ids: Sequence[int],
        past_key_values: Optional[tuple] = None,
        attention_mask: Any = None,
        output_attentions: bool = False,
        use_cache: bool = True,
    ) -> _Out:
        rng = self._rng()
        n_in = len(input_ids)
        cache_pos = 0 if past_key_values is None else int(past_key_values[0])
        n_max = self.max_cache_len
        logits = rng.standard_normal((1, 1, self.vocab)).astype(np.float32)
        if n_in > 1:  # prefill
            end = cache_pos + n_in
            atts = None
            if output_attentions:
                atts = []
                for _ in range(self.n_layers):
                    a = np.zeros(n_max, np.float32)
                    a[:end] = rng.random(end).astype(np.float32) ** 3
                    atts.append(a.reshape(1, 1, 1, -1))
            return _Out(logits, (end,), atts)
        # decode: the new token sits at cache_pos and sees columns < cache_pos + 1
        n_pos = cache_pos + 1
        if isinstance(attention_mask, np.ndarray) and attention_mask.ndim == 2:
            keep = attention_mask[0] > 0.5
            per_head = True
        else:
            keep = np.asarray(attention_mask, np.float32) > 0.5 if attention_mask is not None else np.ones(n_pos, bool)
            per_head = False
        keep = np.concatenate([keep[:n_pos], np.zeros(max(0, n_pos - len(keep)), bool)])[:n_pos]
        probs = np.zeros((self.n_layers, self.n_heads, n_max), np.float32)
        for layer in range(self.n_layers):
            z = (rng.standard_normal((self.n_heads, n_pos)) * self.spread).astype(np.float32)
            z = np.where(keep[None, :], z, np.float32(-1e9))
            z = z - z.max(axis=1, keepdims=True)
            e = np.exp(z)
            probs[layer, :, :n_pos] = e / e.sum(axis=1, keepdims=True)
        if not output_attentions:
            atts = None
        elif per_head:
            atts = [probs.max(axis=0)]
        else:
            atts = [probs.max(axis=(0, 1)).reshape(1, 1, 1, -1)]
        return _Out(logits, (n_pos,), atts)
