"""numpy restatement of the reference's Qwen2/Qwen3 forward (test infrastructure).

Follows ``JAXModelAdapter`` and ``_forward_jittable`` in
``src/counterfact_kv_eviction/jax_inference.py``:

* ``rms_norm`` (:609-618): float32 mean of squares, ``x * rsqrt(var + eps) * w`` in
  float32, cast back to bfloat16; Qwen2/Qwen3 use ``w`` (not ``1 + w``).
* ``rotary_embedding`` (:621-637): float32 angles, cos/sin cast to bfloat16, then
  ``[x1*c - x2*s, x2*c + x1*s]`` as bfloat16 ops (each op rounds).
* ``_attention_layer`` GQA branch (:942-1084): q/k/v projections with bfloat16
  output, bias added as a bfloat16 op (Qwen2, :953-956), optional per-head q/k
  RMSNorm (Qwen3, :975-978), RoPE, K/V written at ``cache_pos`` (:1011-1012),
  ``s = bf16(bf16(q.k) * bf16(1/sqrt(128)))`` over every cache column, additive
  ``0 / -1e9`` float32 mask, float32 softmax, ``p @ float32(V)`` cast to bfloat16.
* ``_mlp_layer`` (:1089-1107): ``silu(g) * u`` as bfloat16 ops, then ``down``.
* ``_forward_jittable`` (:1182-1348): embed, L x (norm, attn, +res, norm, mlp, +res),
  final norm, lm_head with bfloat16 output returned as float32.
* adapter decode branch (:1606-1682): per-KV-head mask repeated over the query
  group, per-head scores = max over layers ``(Hq, N)``; prefill branch
  (:1684-1790): per-layer running max over heads and real query rows, zero at
  positions >= the prompt end.

Matrix products run as float32 BLAS on bfloat16-valued operands (float32
accumulation), rounded to bfloat16 where the reference's output dtype is bfloat16.
XLA's own accumulation order and transcendental implementations are not
reproduced (JAX cannot run here), so these numerics are "parity unpinned" beyond the
rounding points listed above.

Unlike the reference, the prefill is not split into 256-token chunks: chunking only
changes which rows are computed together, and padded rows never reach a real
output (causal mask), so the real rows are identical.  Prefill logits are returned
for the last prompt position only (the generator reads ``logits[0, -1]``).
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Any, Dict, List, Optional, Sequence

import numpy as np

from .bf16 import rnd

F32 = np.float32
NEG = F32(-1e9)


@dataclass
class OracleConfig:
    vocab: int
    hidden: int
    n_layers: int
    n_heads: int
    n_kv_heads: int
    head_dim: int
    ffn: int
    rope_theta: float = 1e6
    eps: float = 1e-6
    qkv_bias: bool = True
    qk_norm: bool = False
    tie_embed: bool = False


def inv_freq_table(head_dim: int, theta: float) -> np.ndarray:
    """RoPE inverse frequencies exactly as jax_inference.py:623-624 in float32."""
    half = head_dim // 2
    expo = np.arange(0, half, dtype=F32) / F32(half)
    return (F32(1.0) / (F32(theta) ** expo)).astype(F32)


def scale_bf16(head_dim: int) -> np.float32:
    """``1/sqrt(head_dim)`` as the bfloat16 value the reference multiplies by."""
    return rnd(np.array([1.0 / math.sqrt(head_dim)], F32))[0]


def rms_norm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    var = np.mean(x * x, axis=-1, keepdims=True, dtype=F32)
    normed = x * (F32(1.0) / np.sqrt(var + F32(eps)))
    return rnd(normed * w)


def rope(x: np.ndarray, pos: np.ndarray, inv_freq: np.ndarray) -> np.ndarray:
    """x: (n, heads, D) bf16-valued; pos: (n,) int."""
    half = x.shape[-1] // 2
    ang = pos.astype(F32)[:, None] * inv_freq[None, :]
    c = rnd(np.cos(ang))[:, None, :]
    s = rnd(np.sin(ang))[:, None, :]
    x1, x2 = x[..., :half], x[..., half:]
    return np.concatenate([rnd(rnd(x1 * c) - rnd(x2 * s)), rnd(rnd(x2 * c) + rnd(x1 * s))], axis=-1)


def silu_mul(g: np.ndarray, u: np.ndarray) -> np.ndarray:
    with np.errstate(over="ignore"):
        sig = rnd(F32(1.0) / (F32(1.0) + np.exp(-g)))
    return rnd(rnd(g * sig) * u)


def linear(x: np.ndarray, w: np.ndarray) -> np.ndarray:
    return rnd(x @ w.T)


class _Out:
    def __init__(self, logits, past_key_values, attentions):
        self.logits = logits
        self.past_key_values = past_key_values
        self.attentions = attentions


class OracleModel:
    """Callable with the ``JAXModelAdapter.__call__`` signature (jax_inference.py:1575)."""

    def __init__(self, cfg: OracleConfig, weights: Dict[str, np.ndarray], max_cache_len: int = 2048, chunk: int = 256):
        self.cfg = cfg
        self.w = weights
        self.max_cache_len = int(max_cache_len)
        self.chunk = int(chunk)
        self.inv_freq = inv_freq_table(cfg.head_dim, cfg.rope_theta)
        self.scale = scale_bf16(cfg.head_dim)
        # last decode's per-layer/per-head probabilities (L, Hq, N), for tests
        self.last_probs: Optional[np.ndarray] = None

    # -- one decoder layer over rows at absolute positions ``pos`` --------------------
    def _layer(self, i, h, pos, ck, cv, allow):
        """h: (n, H); ck/cv: (Hkv, N, D) cache (updated in place); ``allow(n, Hq, ncols)``
        returns the boolean visibility; returns (h_out, probs (n, Hq, ncols))."""
        c, w = self.cfg, self.w
        G = c.n_heads // c.n_kv_heads
        D = c.head_dim
        n = h.shape[0]
        x = rms_norm(h, w[f"l{i}.in_norm"], c.eps)
        q = linear(x, w[f"l{i}.wq"])
        k = linear(x, w[f"l{i}.wk"])
        v = linear(x, w[f"l{i}.wv"])
        if c.qkv_bias:
            q = rnd(q + w[f"l{i}.bq"])
            k = rnd(k + w[f"l{i}.bk"])
            v = rnd(v + w[f"l{i}.bv"])
        q = q.reshape(n, c.n_heads, D)
        k = k.reshape(n, c.n_kv_heads, D)
        v = v.reshape(n, c.n_kv_heads, D)
        if c.qk_norm:
            q = rms_norm(q, w[f"l{i}.q_norm"], c.eps)
            k = rms_norm(k, w[f"l{i}.k_norm"], c.eps)
        q = rope(q, pos, self.inv_freq)
        k = rope(k, pos, self.inv_freq)
        ck[:, pos, :] = k.transpose(1, 0, 2)
        cv[:, pos, :] = v.transpose(1, 0, 2)
        ncols = int(pos.max()) + 1
        vis = allow(n, c.n_heads, ncols)  # (n, Hq, ncols) bool
        probs = np.empty((n, c.n_heads, ncols), F32)
        attn = np.empty((n, c.n_heads, D), F32)
        for g in range(c.n_kv_heads):
            qg = q[:, g * G : (g + 1) * G, :]  # (n, G, D)
            s = rnd(qg @ ck[g, :ncols, :].T)  # (n, G, ncols)
            s = rnd(s * self.scale)
            s = s + np.where(vis[:, g * G : (g + 1) * G, :], F32(0.0), NEG)
            s = s - s.max(axis=-1, keepdims=True)
            e = np.exp(s)
            p = e / e.sum(axis=-1, keepdims=True)
            probs[:, g * G : (g + 1) * G, :] = p
            attn[:, g * G : (g + 1) * G, :] = rnd(p @ cv[g, :ncols, :])
        o = linear(attn.reshape(n, c.n_heads * D), w[f"l{i}.wo"])
        h = rnd(h + o)
        x2 = rms_norm(h, w[f"l{i}.post_norm"], c.eps)
        act = silu_mul(linear(x2, w[f"l{i}.w_gate"]), linear(x2, w[f"l{i}.w_up"]))
        h = rnd(h + linear(act, w[f"l{i}.w_down"]))
        return h, probs

    def _logits(self, h_last: np.ndarray) -> np.ndarray:
        c, w = self.cfg, self.w
        x = rms_norm(h_last, w["final_norm"], c.eps)
        head = w["embed"] if c.tie_embed else w["lm_head"]
        return linear(x, head).astype(F32)

    def _new_cache(self):
        c = self.cfg
        shape = (c.n_kv_heads, self.max_cache_len, c.head_dim)
        return [np.zeros(shape, F32) for _ in range(c.n_layers)], [np.zeros(shape, F32) for _ in range(c.n_layers)]

    def __call__(
        self,
        *,
        input_ids: Sequence[int],
        past_key_values: Optional[tuple] = None,
        attention_mask: Any = None,
        output_attentions: bool = False,
        use_cache: bool = True,
    ) -> _Out:
        c = self.cfg
        N = self.max_cache_len
        ids = np.asarray(list(input_ids), np.int64)
        n = len(ids)
        if n == 0:
            raise ValueError("input_ids must be non-empty")
        if past_key_values is not None:
            ck, cv, cache_pos = past_key_values
        else:
            ck, cv = self._new_cache()
            cache_pos = 0
        h = self.w["embed"][ids]

        if n == 1:  # decode branch, jax_inference.py:1606-1682
            if cache_pos >= N:
                raise ValueError(f"cache_pos {cache_pos} >= max_cache_len {N}.")
            per_head = isinstance(attention_mask, np.ndarray) and attention_mask.ndim == 2
            ncols_live = cache_pos + 1
            if attention_mask is None:
                flags = np.ones((c.n_heads, ncols_live), bool)
            elif per_head:
                m = np.asarray(attention_mask, F32)
                if m.shape[1] < ncols_live:
                    m = np.pad(m, ((0, 0), (0, ncols_live - m.shape[1])))
                flags = np.repeat(m[:, :ncols_live] > 0.5, c.n_heads // m.shape[0], axis=0)
            else:
                m = np.asarray(list(attention_mask), F32)
                if len(m) > N:
                    raise ValueError(f"attention_mask length {len(m)} exceeds max_cache_len {N}")
                if len(m) < ncols_live:
                    m = np.pad(m, (0, ncols_live - len(m)))
                flags = np.broadcast_to(m[:ncols_live] > 0.5, (c.n_heads, ncols_live))

            def allow(nr, nh, ncols):
                return flags[None, :, :ncols]

            pos = np.array([cache_pos], np.int64)
            layer_probs = np.zeros((c.n_layers, c.n_heads, N), F32)
            for i in range(c.n_layers):
                h, pr = self._layer(i, h, pos, ck[i], cv[i], allow)
                layer_probs[i, :, : pr.shape[-1]] = pr[0]
            self.last_probs = layer_probs
            logits = self._logits(h[-1:])[None]  # (1, 1, V)
            atts = None
            if output_attentions:
                if per_head:
                    atts = [layer_probs.max(axis=0)]
                else:
                    atts = [layer_probs.max(axis=(0, 1)).reshape(1, 1, 1, -1)]
            return _Out(logits, (ck, cv, cache_pos + 1) if use_cache else None, atts)

        # prefill branch, jax_inference.py:1684-1790
        end = cache_pos + n
        padded = ((n + self.chunk - 1) // self.chunk) * self.chunk
        if cache_pos + padded > N:
            raise ValueError(
                f"Prefill chunk would exceed cache: cur_pos={cache_pos} + effective_len={padded} > max_cache_len={N}."
            )
        pos = np.arange(cache_pos, end, dtype=np.int64)
        causal = pos[:, None, None] >= np.arange(end)[None, None, :]

        def allow(nr, nh, ncols):
            return np.broadcast_to(causal[:, :, :ncols], (nr, nh, ncols))

        accum = [np.zeros(N, F32) for _ in range(c.n_layers)]
        for i in range(c.n_layers):
            h, pr = self._layer(i, h, pos, ck[i], cv[i], allow)
            if output_attentions:
                accum[i][: pr.shape[-1]] = pr.max(axis=(0, 1))
                accum[i][end:] = 0.0
        logits = self._logits(h[-1:])[None]
        atts = [a.reshape(1, 1, 1, -1) for a in accum] if output_attentions else None
        return _Out(logits, (ck, cv, end) if use_cache else None, atts)


def weight_names(cfg: OracleConfig) -> List[str]:
    names = ["embed"]
    for i in range(cfg.n_layers):
        names += [f"l{i}.in_norm", f"l{i}.wq", f"l{i}.wk", f"l{i}.wv"]
        if cfg.qkv_bias:
            names += [f"l{i}.bq", f"l{i}.bk", f"l{i}.bv"]
        if cfg.qk_norm:
            names += [f"l{i}.q_norm", f"l{i}.k_norm"]
        names += [f"l{i}.wo", f"l{i}.post_norm", f"l{i}.w_gate", f"l{i}.w_up", f"l{i}.w_down"]
    names.append("final_norm")
    if not cfg.tie_embed:
        names.append("lm_head")
    return names


def int8_roundtrip(rows: np.ndarray) -> np.ndarray:
    """Lossy int8 demotion of K/V rows (last axis = head_dim), restating
    ``_demote_kv_positions`` (src/counterfact_kv_eviction/online_credit_generator.py:
    676-691): per row absmax scale, round-half-even, clip to [-127, 127], dequantise --
    each op on bfloat16 values, computed in float32 and rounded to bfloat16."""
    x = rnd(np.asarray(rows, F32))
    scale = rnd(np.abs(x).max(axis=-1, keepdims=True) / F32(127.0))
    den = np.maximum(scale, rnd(np.array([1e-10], F32))[0])
    q = np.clip(np.round(rnd(x / den)), F32(-127.0), F32(127.0))
    return rnd(q * scale)
