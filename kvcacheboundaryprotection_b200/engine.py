"""Device-resident capped-KV decode engine (B200, sm_100a).

``CappedKVEngine`` owns, for a batch of B sequences decoded in lockstep:

* the decoder weights (bf16; q/k/v and gate/up fused into one matrix each),
* the slot KV cache ``[L][B][Hkv][S][128]`` bf16 with S = capacity + evict_every
  (capacity + max_new_tokens under ``--eviction-regime prefill``),
* the per-slot eviction metadata (``kvbp_state``) and the position bitmap,
* activation buffers, the eviction / token / retained-count logs.

One decode step is::

    kvbp_update_append_evict   the previous step's score update, then the new position
                               -> lowest free slot; cadence eviction
    kvbp_embed
    kvbp_row_sumsq
    L x [ kvbp_decode_qkv_gemm   (RMSNorm prologue; bias, q/k norm, RoPE, K/V slot store)
          kvbp_decode_attn_score (attention over the slots + per-slot score)
          kvbp_decode_gemm o     (residual epilogue)
          kvbp_decode_gemm gu    (RMSNorm prologue, SwiGLU epilogue)
          kvbp_decode_gemm down  (residual epilogue) ]
    kvbp_decode_gemm lm_head (final RMSNorm prologue), kvbp_argmax

(the host-selected and per-KV-head policies and the tensor-parallel engine append with
their own kernels and end the step with kvbp_score_update instead).
Every step-dependent value (step counter, positions, slots) lives on the device, so
one captured CUDA graph replays every step.  The decode GEMMs are this package's
weight-streaming sm_100a kernels over packed weights (``gemm="kvbp"``, the default);
``gemm="cublas"`` runs them as torch.mm with bf16 output and float32 accumulation,
with standalone norm / RoPE / SwiGLU kernels around them.  The prefill projections run
on the tcgen05 prefill GEMM (``gemm="kvbp"``) or cuBLAS.

The reference computes the same step in ``KVCoupledQwen35Generator`` (host loop,
``src/counterfact_kv_eviction/kv_coupled_generator.py:336-516``) around
``JAXModelAdapter``'s jitted forward (``jax_inference.py:1182-1348,1606-1682``).
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Dict, List, Optional

import numpy as np
import torch

from . import capi
from .capi import EvictCfg, State, check, lib
from .config import ModelConfig


def inv_freq_table(head_dim: int, theta: float) -> np.ndarray:
    """RoPE inverse frequencies as float32 ops (jax_inference.py:623-624)."""
    half = head_dim // 2
    expo = np.arange(0, half, dtype=np.float32) / np.float32(half)
    return (np.float32(1.0) / (np.float32(theta) ** expo)).astype(np.float32)


def scale_bf16(head_dim: int) -> float:
    return float(torch.tensor(1.0 / math.sqrt(head_dim), dtype=torch.float32).to(torch.bfloat16).item())


def _ptr(t: Optional[torch.Tensor]):
    return None if t is None else t.data_ptr()


@dataclass
class EvictionSpec:
    """Eviction configuration of the harness (scripts/run_v3_jax.py:141-206)."""

    policy: str = "lru"
    capacity: int = 256
    evict_every: int = 8
    protect: bool = True
    prefix_frac: float = 0.10
    suffix_frac: float = 0.10
    regime: str = "decode"
    # capacity the protection wrapper sizes its prefix/suffix from (its own ``capacity``
    # field, run_v3_jax.py:119); None = the eviction capacity
    protect_capacity: Optional[int] = None

    def sizes(self) -> tuple:
        if not self.protect:
            return 0, 0
        cap = self.capacity if self.protect_capacity is None else self.protect_capacity
        return capi.protection_sizes(cap, self.prefix_frac, self.suffix_frac)


def interleave_gate_up(gate: torch.Tensor, up: torch.Tensor, block: int = 64) -> torch.Tensor:
    """[2F, H] with rows 128t..128t+63 = gate rows 64t.. and 128t+64.. = the matching up rows
    (the layout the SwiGLU epilogue of kvbp_decode_gemm expects)."""
    F, H = gate.shape
    if F % block:
        raise ValueError(f"ffn {F} must be a multiple of {block}")
    return torch.stack([gate.view(F // block, block, H), up.view(F // block, block, H)], 1).reshape(2 * F, H).contiguous()


def deinterleave_gate_up(gu: torch.Tensor, block: int = 64) -> torch.Tensor:
    """[rows, 2F] GEMM output in interleaved feature order -> [rows, 2F] as [gate | up]."""
    R, F2 = gu.shape
    v = gu.view(R, F2 // (2 * block), 2, block)
    return torch.cat([v[:, :, 0, :].reshape(R, F2 // 2), v[:, :, 1, :].reshape(R, F2 // 2)], 1)


def pack_weight(w: torch.Tensor) -> torch.Tensor:
    """Row-major bf16 [N, K] -> the decode GEMM's packed layout (same shape and size;
    kvbp_pack_weight describes the element order)."""
    N, K = w.shape
    out = torch.empty_like(w)
    check(lib().kvbp_pack_weight(torch.cuda.current_stream(w.device).cuda_stream, N, K, _ptr(w), _ptr(out)),
          "pack_weight")
    return out


def unpack_weight(w: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Inverse of pack_weight (into ``out`` when given)."""
    N, K = w.shape
    if out is None:
        out = torch.empty_like(w)
    check(lib().kvbp_unpack_weight(torch.cuda.current_stream(w.device).cuda_stream, N, K, _ptr(w), _ptr(out)),
          "unpack_weight")
    return out


class FusedWeights:
    """Decoder weights on the device in the engine's layout (bf16): q/k/v stacked into
    one [(Hq+2Hkv)*128, H] matrix (+ stacked bias); gate/up interleaved in blocks of 64
    rows for the own decode GEMM (``gemm="kvbp"``) or stacked [gate; up] for cuBLAS.
    With ``gemm="kvbp"`` the projection matrices and lm_head are stored packed
    (pack_weight); ``rowmajor`` gives a row-major view for the prefill's cuBLAS GEMMs."""

    PACKED = ("w_qkv", "w_o", "w_gu", "w_down")

    def __init__(self, cfg: ModelConfig, w: Dict[str, torch.Tensor], device: torch.device, gemm: str = "kvbp"):
        c, d, bf = cfg, torch.device(device), torch.bfloat16
        if gemm not in ("kvbp", "cublas"):
            raise ValueError("gemm must be 'kvbp' or 'cublas'")
        self.gemm = gemm

        def g(name):
            return w[name].to(device=d, dtype=bf).contiguous()

        self.cfg = cfg
        self.embed_w = g("embed")
        self.lm_w = self.embed_w if c.tie_embed else g("lm_head")
        self.final_norm = g("final_norm")
        self.layers = []
        for i in range(c.n_layers):
            self.layers.append(
                {
                    "in_norm": g(f"l{i}.in_norm"),
                    "post_norm": g(f"l{i}.post_norm"),
                    "w_qkv": torch.cat([g(f"l{i}.wq"), g(f"l{i}.wk"), g(f"l{i}.wv")], 0).contiguous(),
                    "b_qkv": torch.cat([g(f"l{i}.bq"), g(f"l{i}.bk"), g(f"l{i}.bv")], 0).contiguous()
                    if c.qkv_bias
                    else None,
                    "q_norm": g(f"l{i}.q_norm") if c.qk_norm else None,
                    "k_norm": g(f"l{i}.k_norm") if c.qk_norm else None,
                    "w_o": g(f"l{i}.wo"),
                    "w_gu": interleave_gate_up(g(f"l{i}.w_gate"), g(f"l{i}.w_up"))
                    if gemm == "kvbp"
                    else torch.cat([g(f"l{i}.w_gate"), g(f"l{i}.w_up")], 0).contiguous(),
                    "w_down": g(f"l{i}.w_down"),
                }
            )
        self.inv_freq = torch.from_numpy(inv_freq_table(c.head_dim, c.rope_theta)).to(d)
        self._scratch = None
        if gemm == "kvbp":
            with torch.cuda.device(d):
                for L in self.layers:
                    for k in self.PACKED:
                        L[k] = pack_weight(L[k])
                self.lm_w = pack_weight(self.lm_w)

    def rowmajor(self, w: torch.Tensor) -> torch.Tensor:
        """Row-major copy of a packed projection matrix (a reused scratch buffer, valid
        until the next call); the tensor itself when the weights are not packed."""
        if self.gemm != "kvbp":
            return w
        n = w.numel()
        if self._scratch is None or self._scratch.numel() < n:
            biggest = max(L[k].numel() for L in self.layers for k in self.PACKED)
            self._scratch = torch.empty(max(n, biggest), dtype=torch.bfloat16, device=w.device)
        return unpack_weight(w, self._scratch[:n].view(w.shape))

    def streamed_bytes(self, batch: int) -> int:
        """Weight bytes one decode step reads: every matrix, bias and norm, the lm_head in
        full, but only ``batch`` rows of the embedding table (a lookup, not a stream)."""
        return self.nbytes() - 2 * self.embed_w.numel() + 2 * batch * self.cfg.hidden

    def nbytes(self) -> int:
        n = self.embed_w.numel() + (0 if self.lm_w is self.embed_w else self.lm_w.numel()) + self.final_norm.numel()
        for L in self.layers:
            n += sum(t.numel() for t in L.values() if t is not None)
        return 2 * n


class CappedKVEngine:
    def __init__(
        self,
        cfg: ModelConfig,
        weights: Dict[str, torch.Tensor],
        *,
        batch: int,
        evict: EvictionSpec,
        max_prompt_len: int,
        max_new_tokens: int,
        device: Optional[torch.device] = None,
        kv_heads: Optional[List[int]] = None,
        gemm: str = "kvbp",
        host_policy=None,
    ):
        if cfg.head_dim != 128:
            raise ValueError("only head_dim 128 is supported")
        if cfg.group > 8:
            raise ValueError("query group size > 8 is not supported by the decode kernel")
        if evict.capacity <= 0:
            raise ValueError("capacity must be > 0")
        if evict.evict_every <= 0:
            raise ValueError("evict_every_n_steps must be > 0")
        if evict.regime not in ("decode", "prefill"):
            raise ValueError("eviction_regime must be 'decode' or 'prefill'")
        lib()  # fail loudly when the CUDA library is missing
        # a policy that draws its victims on the host (the random policy) through the
        # reference's select_evictions protocol; the device applies them
        from .policies import per_head as _is_per_head

        self.host_policy = host_policy
        self.per_head = host_policy is not None and _is_per_head(host_policy)
        if evict.policy == "random" and host_policy is None:
            raise ValueError("the random policy needs its policy object (host_policy)")
        if host_policy is not None and not (self.per_head or evict.policy == "random"):
            raise ValueError("host_policy is for the random and the per-KV-head policies only")
        if host_policy is not None and int(batch) != 1:
            raise ValueError("a host-selected policy runs one sequence per engine: batch must be 1")
        inner = getattr(host_policy, "inner", host_policy)
        self.head_uses_current = self.per_head and inner.name.startswith("quest")
        self.dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        if self.dev.type != "cuda":
            raise ValueError("CappedKVEngine runs on CUDA devices only")
        torch.backends.cuda.matmul.allow_tf32 = False
        torch.backends.cuda.matmul.allow_bf16_reduced_precision_reduction = False
        self.cfg = cfg
        self.ev = evict
        self.B = int(batch)
        self.max_prompt = int(max_prompt_len)
        self.max_new = int(max_new_tokens)
        self.policy_id = capi.policy_id(evict.policy)
        self.n_prefix, self.n_suffix = evict.sizes()
        C = evict.capacity
        self.S = C + (evict.evict_every if evict.regime == "decode" else max(1, self.max_new))
        self.W = (self.max_prompt + self.max_new + 2 + 31) // 32
        self.evcap = self.max_prompt + self.max_new + 2
        self.gemm = weights.gemm if isinstance(weights, FusedWeights) else gemm
        if self.gemm == "kvbp" and self.B > 32:
            raise ValueError("the decode GEMM handles up to 32 sequences per GPU")
        self._load_weights(weights)
        self._alloc()
        self.graph: Optional[torch.cuda.CUDAGraph] = None
        self.prompt_len = 0
        self.step = 0

    # ------------------------------------------------------------------ setup
    def _load_weights(self, w) -> None:
        fw = w if isinstance(w, FusedWeights) else FusedWeights(self.cfg, w, self.dev, gemm=self.gemm)
        self.fw = fw
        self.embed_w, self.lm_w, self.final_norm = fw.embed_w, fw.lm_w, fw.final_norm
        self.layers = fw.layers
        self.inv_freq = fw.inv_freq

    def _alloc(self) -> None:
        c, d, B, S = self.cfg, self.dev, self.B, self.S
        i32, f32, bf = torch.int32, torch.float32, torch.bfloat16
        L = c.n_layers
        self.kc = torch.zeros(L, B, c.n_kv_heads, S, c.head_dim, dtype=bf, device=d)
        self.vc = torch.zeros_like(self.kc)
        z = lambda *s, dt=i32: torch.zeros(*s, dtype=dt, device=d)  # noqa: E731
        self.slot_pos = torch.full((B, S), -1, dtype=i32, device=d)
        self.insert_step = z(B, S)
        self.last_access = z(B, S)
        self.access_count = z(B, S)
        self.attn_s = z(B, S, dt=f32)
        self.max_attn = z(B, S, dt=f32)
        self.cumul = z(B, S, dt=torch.float64)
        self.prefill_s = z(B, S, dt=f32)
        self.posmap = z(B, self.W, dt=torch.int32)
        self.step_score = z(B, S, dt=f32)
        self.seq_counter = z(B)  # arrivals per sequence of the fused score update (zero between launches)
        self.upd_pending = z(B)  # 1 while a forwarded step's scores await the next append's update
        self._forwarded = False  # the last launched step forwarded (its scores are pending)
        self.seq_step = z(B)
        self.next_pos = z(B)
        self.cur_pos = z(B)
        self.write_slot = z(B)
        self.tokens = z(B)
        self.token_log = z(B, max(1, self.max_new))
        self.retained_log = z(B, self.max_new + 1)
        self.evlog = z(B, self.evcap)
        self.evcount = z(B)
        if self.host_policy is not None:  # victims listed by the host at cadence steps
            self.ext_pos = z(B, S)
            self.ext_n = z(B)
        if self.per_head:  # per-KV-head retention masks and signals, slot-indexed
            Hkv = c.n_kv_heads
            self.head_keep = torch.ones(B, Hkv, S, dtype=torch.uint8, device=d)
            self.head_score = z(B, Hkv, S, dt=f32)
            self.head_cumul = z(B, Hkv, S, dt=torch.float64)
            self.head_current = z(B, Hkv, S, dt=f32)
            self.head_ready = False
            self.union_stats = [0, 0, 0]  # retained max, overflow max, overflow steps
            self.head_call_steps: List[int] = []
        self.dev_err = z(1)
        H, F, V = c.hidden, c.ffn, c.vocab
        self.h = z(B, H, dt=bf)
        self.x = z(B, H, dt=bf)
        self.qkv = z(B, c.qkv_dim, dt=bf)
        self.q = z(B, c.n_heads, c.head_dim, dt=bf)
        self.attn_out = z(B, c.n_heads * c.head_dim, dt=bf)
        self.o = z(B, H, dt=bf)
        self.gu = z(B, 2 * F, dt=bf)
        self.act = z(B, F, dt=bf)
        self.dn = z(B, H, dt=bf)
        self.logits = z(B, V, dt=bf)
        # own-GEMM RMSNorm partial sums and split-K cluster sizes
        self.ss_a = z(max(1, H // 128), 32, dt=f32)
        self.ss_b = z(max(1, H // 128), 32, dt=f32)
        self.splits = {
            name: self._pick_splits(N, K)
            for name, (N, K) in {"qkv": (c.qkv_dim, H), "o": (H, c.n_heads * c.head_dim), "gu": (2 * F, H),
                                 "down": (H, F), "lm": (V, H)}.items()
        }
        self._state = State(
            B, S, self.W,
            self.slot_pos.data_ptr(), self.insert_step.data_ptr(), self.last_access.data_ptr(),
            self.access_count.data_ptr(), self.attn_s.data_ptr(), self.max_attn.data_ptr(),
            self.cumul.data_ptr(), self.prefill_s.data_ptr(), self.posmap.data_ptr(),
        )
        self._cfg = EvictCfg(
            self.ev.capacity, self.ev.evict_every, self.policy_id, int(self.ev.protect), self.n_prefix,
            self.n_suffix, int(self.ev.regime == "decode"),
        )

    @staticmethod
    def _pick_splits(N: int, K: int, sms: int = 148) -> int:
        """Split-K factor (CTAs per 128-column tile, one thread-block cluster) of a decode
        GEMM with N / 128 column tiles and K / 128 k-blocks, from a burst sweep of every
        per-rank shape of the 7B, Qwen2.5-3B and Qwen3-4B decoders at 1, 2, 4 and 8 GPUs on
        B200 (and of 149 .. 240-tile shapes at 1, 16 and 32 rows):
        * a few tiles past one whole wave of 2 CTAs per SM (up to 1/8 of a wave more): 2
          splits, so the CTAs left over for a second wave carry half a k range (297 tiles,
          the TP = 4 lm_head shard: 61.4-63.6 us against 65.5-66.4 us unsplit);
        * otherwise more tiles than SMs: no split -- a split only adds a second wave (172
          tiles of the 3B gate/up: 29.7 us unsplit against 33.8 us with 3 splits; 149, 152,
          160, 200 and 594 tiles alike);
        * >= ~2/3 tile per SM: the split whose whole waves of 2 CTAs per SM carry the most
          work per wave (148 tiles: 2 splits, one full wave);
        * 24.. tiles: about 256 CTAs, at most 8 per cluster (the single-GPU 7B q/k/v, o and
          down shapes, re-swept inside the decode step: 7, 8, 8);
        * fewer tiles: about 210 CTAs in all, at most 16 per cluster."""
        tiles = max(1, N // 128)
        kc = max(1, K // 128)
        slots = 2 * sms
        if slots < tiles <= slots + slots // 8:
            return 2
        if tiles > sms:
            return 1
        if tiles * 3 >= slots:
            cands = range(1, min(4, kc) + 1)
            return min(cands, key=lambda s: (math.ceil(tiles * s / slots) / s, s))
        if tiles >= 24:
            return max(1, min((256 * sms // 148) // tiles, 8, kc))
        return max(1, min(round(210 * sms / 148 / tiles), 16, kc))

    @property
    def stream(self) -> int:
        return torch.cuda.current_stream(self.dev).cuda_stream

    def kv_bytes_per_layer(self) -> int:
        return self.kc[0].numel() * 2 * 2

    # ------------------------------------------------------------------ prefill
    def _prefill_attention(self, q, kbuf, vbuf, need_scores, colmax):
        """Causal prefill attention with the reference's rounding points on the tcgen05
        tensor cores (kvbp_prefill_attn_score).

        q [P, Hq, D] bf16; kbuf/vbuf [Hkv, P, D] bf16.  Returns [P, Hq*D] bf16 and folds
        the per-key max over heads and query rows of the probabilities into ``colmax``
        (jax_inference.py:1018-1050 with the causal mask :1169-1179, per-key max
        :1754-1760).
        """
        c = self.cfg
        P = q.shape[0]
        out = torch.empty(P, c.n_heads, c.head_dim, dtype=torch.bfloat16, device=self.dev)
        check(
            lib().kvbp_prefill_attn_score(
                self.stream, P, c.n_heads, c.n_kv_heads, c.head_dim, _ptr(q), _ptr(kbuf), _ptr(vbuf), _ptr(out),
                _ptr(colmax) if need_scores else None, _ptr(self.dev_err),
            ),
            "prefill_attn_score",
        )
        return out.reshape(P, c.n_heads * c.head_dim)

    def prefill(self, input_ids: torch.Tensor) -> None:
        """Step 0 for the whole batch: forward the prompts, score positions (non-LRU),
        evict down to capacity (forced), compact into slots and sample step 1's token."""
        c, d, st = self.cfg, self.dev, self.stream
        L = lib()
        ids = input_ids.to(device=d, dtype=torch.int32).contiguous()
        B, P = ids.shape
        if B != self.B:
            raise ValueError(f"batch {B} != engine batch {self.B}")
        if P <= 0:
            raise ValueError("input_ids must be non-empty")
        if P > self.max_prompt:
            raise ValueError(f"prompt length {P} > max_prompt_len {self.max_prompt}")
        need_scores = capi.POLICY_IDS[self.ev.policy] != 0
        Hkv, D = c.n_kv_heads, c.head_dim
        pre_k = torch.empty(c.n_layers, B, Hkv, P, D, dtype=torch.bfloat16, device=d)
        pre_v = torch.empty_like(pre_k)
        scores = torch.zeros(B, P, dtype=torch.float32, device=d) if need_scores else None
        # per-head mode seeds head 0 with the FIRST layer's per-key max only: the generator
        # reads attentions[0] of the prefill output (kv_coupled_generator.py:244-262)
        self.prefill_head_seed = torch.zeros(B, P, dtype=torch.float32, device=d) if self.per_head else None
        positions = torch.arange(P, dtype=torch.int32, device=d)
        H = c.hidden
        if self.gemm == "kvbp":
            # own tcgen05 projections over the prompt rows of several sequences at once
            group = max(1, min(B, self.PREFILL_ROWS // P))
            for g0 in range(0, B, group):
                self._prefill_group(ids[g0 : g0 + group], g0, pre_k, pre_v, scores, need_scores, positions)
            self._select_and_compact(P, scores, pre_k, pre_v)
            check(L.kvbp_argmax(st, B, c.vocab, c.vocab, _ptr(self.logits), _ptr(self.tokens)), "argmax")
            return
        for b in range(B):
            h = torch.empty(P, H, dtype=torch.bfloat16, device=d)
            check(L.kvbp_embed(st, P, c.vocab, H, _ptr(self.embed_w), _ptr(ids[b]), _ptr(h), _ptr(self.dev_err)), "embed")
            x = torch.empty_like(h)
            delta = None
            colmax = torch.zeros(P, dtype=torch.float32, device=d) if need_scores else None
            for li, Lw in enumerate(self.layers):
                check(L.kvbp_add_rmsnorm(st, P, H, _ptr(h), _ptr(delta), _ptr(Lw["in_norm"]), _ptr(x), c.eps), "rmsnorm")
                qkv = torch.mm(x, self.fw.rowmajor(Lw["w_qkv"]).t())
                q = torch.empty(P, c.n_heads, D, dtype=torch.bfloat16, device=d)
                kb, vb = pre_k[li, b], pre_v[li, b]
                check(
                    L.kvbp_qkv_rope_scatter(
                        st, P, P, c.n_heads, Hkv, D, P, _ptr(qkv), c.qkv_dim, _ptr(Lw["b_qkv"]), _ptr(Lw["q_norm"]),
                        _ptr(Lw["k_norm"]), c.eps, _ptr(self.inv_freq), _ptr(positions), _ptr(positions), _ptr(q),
                        _ptr(kb), _ptr(vb), _ptr(self.dev_err),
                    ),
                    "qkv_rope_scatter",
                )
                lcol = torch.zeros(P, dtype=torch.float32, device=d) if need_scores else None
                att = self._prefill_attention(q, kb, vb, need_scores, lcol)
                if need_scores:
                    torch.maximum(colmax, lcol, out=colmax)
                    if li == 0 and self.prefill_head_seed is not None:
                        self.prefill_head_seed[b].copy_(lcol)
                o = torch.mm(att, self.fw.rowmajor(Lw["w_o"]).t())
                check(L.kvbp_add_rmsnorm(st, P, H, _ptr(h), _ptr(o), _ptr(Lw["post_norm"]), _ptr(x), c.eps), "rmsnorm")
                gu = torch.mm(x, self.fw.rowmajor(Lw["w_gu"]).t())
                if self.gemm == "kvbp":
                    gu = deinterleave_gate_up(gu)
                act = torch.empty(P, c.ffn, dtype=torch.bfloat16, device=d)
                check(L.kvbp_silu_mul(st, P, c.ffn, _ptr(gu), _ptr(act)), "silu_mul")
                delta = torch.mm(act, self.fw.rowmajor(Lw["w_down"]).t())
                del gu, act, qkv, q
            hl = h[P - 1 : P].contiguous()
            dl = delta[P - 1 : P].contiguous()
            xl = torch.empty_like(hl)
            check(L.kvbp_add_rmsnorm(st, 1, H, _ptr(hl), _ptr(dl), _ptr(self.final_norm), _ptr(xl), c.eps), "rmsnorm")
            if self.gemm == "kvbp":  # lm_head is packed: one row through the decode GEMM
                check(
                    L.kvbp_decode_gemm(st, 0, 1, c.vocab, H, _ptr(self.lm_w), _ptr(xl), H, None, 0, None, c.eps,
                                       _ptr(self.logits[b : b + 1]), c.vocab, None, self.splits["lm"], _ptr(self.dev_err)),
                    "decode_gemm[lm]",
                )
            else:
                torch.mm(xl, self.lm_w.t(), out=self.logits[b : b + 1])
            if need_scores:
                scores[b] = colmax
        self._select_and_compact(P, scores, pre_k, pre_v)
        check(L.kvbp_argmax(st, B, c.vocab, c.vocab, _ptr(self.logits), _ptr(self.tokens)), "argmax")

    PREFILL_ROWS = 65536  # prompt rows forwarded together by the tcgen05 prefill path

    def _prefill_group(self, ids, b0, pre_k, pre_v, scores, need_scores, positions) -> None:
        """Prompt forward of sequences b0 .. b0 + n - 1 (ids [n, P]) with every projection on
        the tcgen05 prefill GEMM over all n * P rows at once (packed weights read directly,
        the gate/up product finished as SwiGLU in its epilogue); RoPE + K/V scatter for all
        rows in one launch; causal attention with the per-key score per sequence."""
        c, d, st, L = self.cfg, self.dev, self.stream, lib()
        n, P = ids.shape
        R, H, D, Hkv = n * P, c.hidden, c.head_dim, c.n_kv_heads
        bf = torch.bfloat16
        flat = ids.reshape(-1).contiguous()
        pos = positions.repeat(n).contiguous()
        err = _ptr(self.dev_err)

        def gemm(epi, N, K, w, x, out):
            check(L.kvbp_prefill_gemm(st, epi, R, N, K, _ptr(w), _ptr(x), x.stride(0), _ptr(out), out.stride(0), err),
                  "prefill_gemm")

        h = torch.empty(R, H, dtype=bf, device=d)
        check(L.kvbp_embed(st, R, c.vocab, H, _ptr(self.embed_w), _ptr(flat), _ptr(h), err), "embed")
        x = torch.empty_like(h)
        qkv = torch.empty(R, c.qkv_dim, dtype=bf, device=d)
        q = torch.empty(R, c.n_heads, D, dtype=bf, device=d)
        att = torch.empty(R, c.n_heads * D, dtype=bf, device=d)
        o = torch.empty(R, H, dtype=bf, device=d)
        act = torch.empty(R, c.ffn, dtype=bf, device=d)
        delta = None
        colmax = torch.zeros(n, P, dtype=torch.float32, device=d) if need_scores else None
        for li, Lw in enumerate(self.layers):
            check(L.kvbp_add_rmsnorm(st, R, H, _ptr(h), _ptr(delta), _ptr(Lw["in_norm"]), _ptr(x), c.eps), "rmsnorm")
            gemm(0, c.qkv_dim, H, Lw["w_qkv"], x, qkv)
            kc, vc = pre_k[li, b0 : b0 + n], pre_v[li, b0 : b0 + n]
            check(
                L.kvbp_qkv_rope_scatter(
                    st, R, P, c.n_heads, Hkv, D, P, _ptr(qkv), c.qkv_dim, _ptr(Lw["b_qkv"]), _ptr(Lw["q_norm"]),
                    _ptr(Lw["k_norm"]), c.eps, _ptr(self.inv_freq), _ptr(pos), _ptr(pos), _ptr(q), _ptr(kc), _ptr(vc),
                    err,
                ),
                "qkv_rope_scatter",
            )
            for j in range(n):
                lcol = torch.zeros(P, dtype=torch.float32, device=d) if need_scores else None
                att[j * P : (j + 1) * P] = self._prefill_attention(q[j * P : (j + 1) * P], kc[j], vc[j], need_scores,
                                                                    lcol)
                if need_scores:
                    torch.maximum(colmax[j], lcol, out=colmax[j])
                    if li == 0 and self.prefill_head_seed is not None:
                        self.prefill_head_seed[b0 + j].copy_(lcol)
            gemm(0, H, c.n_heads * D, Lw["w_o"], att, o)
            check(L.kvbp_add_rmsnorm(st, R, H, _ptr(h), _ptr(o), _ptr(Lw["post_norm"]), _ptr(x), c.eps), "rmsnorm")
            gemm(2, 2 * c.ffn, H, Lw["w_gu"], x, act)
            delta = o  # o is free again: the down projection lands there
            gemm(0, H, c.ffn, Lw["w_down"], act, delta)
        last = torch.arange(n, device=d) * P + (P - 1)
        hl = h[last].contiguous()
        dl = delta[last].contiguous()
        xl = torch.empty_like(hl)
        check(L.kvbp_add_rmsnorm(st, n, H, _ptr(hl), _ptr(dl), _ptr(self.final_norm), _ptr(xl), c.eps), "rmsnorm")
        check(
            L.kvbp_decode_gemm(st, 0, n, c.vocab, H, _ptr(self.lm_w), _ptr(xl), H, None, 0, None, c.eps,
                               _ptr(self.logits[b0 : b0 + n]), c.vocab, None, self.splits["lm"], err),
            "decode_gemm[lm]",
        )
        if need_scores:
            scores[b0 : b0 + n] = colmax

    def _host_victims(self, retained_sorted: List[int], evict_count: int, step: int) -> List[int]:
        """One ``_maybe_evict`` policy call on the host (kv_coupled_generator.py:563-577):
        blocks keyed by str(position) in ascending position order."""
        blocks = {str(p): None for p in retained_sorted}
        out, seen = [], set()
        for key in self.host_policy.select_evictions(blocks, evict_count, step):
            p = int(key)
            if str(p) in blocks and p not in seen:
                seen.add(p)
                out.append(p)
        return out

    def _select_and_compact(self, P, scores, pre_k=None, pre_v=None) -> None:
        L, st = lib(), self.stream
        victim = torch.zeros(self.B, P, dtype=torch.uint8, device=self.dev)
        self.evlog.zero_()
        nvict = capi.C.c_int32()
        head_state = None
        if self.per_head:
            vict, head_state = self._per_head_step0(P, scores)
            if vict:
                victim[0, torch.tensor(vict, dtype=torch.long, device=self.dev)] = 1
                self.evlog[0, : len(vict)] = torch.tensor(vict, dtype=torch.int32, device=self.dev)
            nvict.value = len(vict)
        elif self.host_policy is not None:
            # step 0 (force_if_over_capacity): evict_count = P - capacity, victims in the
            # policy's order, then the compaction's hard-capacity guardrail
            vict = self._host_victims(list(range(P)), max(0, P - self.ev.capacity), 0)
            if vict:
                victim[0, torch.tensor(vict, dtype=torch.long, device=self.dev)] = 1
                self.evlog[0, : len(vict)] = torch.tensor(vict, dtype=torch.int32, device=self.dev)
            nvict.value = len(vict)
        else:
            check(
                L.kvbp_prefill_select(
                    st, self.B, P, capi.C.byref(self._cfg), _ptr(scores), _ptr(victim), _ptr(self.evlog), self.evcap,
                    capi.C.byref(nvict), _ptr(self.dev_err),
                ),
                "prefill_select",
            )
        self.gather_src = torch.empty(self.B, self.S, dtype=torch.int32, device=self.dev)
        self.retained_log.zero_()
        self.upd_pending.zero_()  # no forwarded decode step yet
        self._forwarded = False
        check(
            L.kvbp_prefill_compact(
                st, capi.C.byref(self._state), P, self.ev.capacity, nvict.value, _ptr(victim), _ptr(scores),
                _ptr(self.gather_src), _ptr(self.evlog), self.evcap, _ptr(self.evcount), _ptr(self.seq_step),
                _ptr(self.next_pos), _ptr(self.retained_log), self.max_new, _ptr(self.step_score), _ptr(self.dev_err),
            ),
            "prefill_compact",
        )
        if self.per_head:
            self._per_head_load(head_state)
        if pre_k is not None:
            c = self.cfg
            check(
                L.kvbp_gather_kv(
                    st, _ptr(pre_k), _ptr(pre_v), _ptr(self.kc), _ptr(self.vc), _ptr(self.gather_src), c.n_layers,
                    self.B, c.n_kv_heads, P, self.S,
                ),
                "gather_kv",
            )
        self.prompt_len = P
        self.step = 0
        self.n_policy_victims_step0 = nvict.value

    def synthetic_prefill(self, prompt_len: int, seed: int = 0) -> None:
        """Post-prefill state of ``prompt_len``-token prompts without running the prefill:
        seeded N(0,1) K/V in every slot, U(0,1) prefill scores through the real step-0
        selection and compaction kernels, random first tokens.  For decode throughput
        measurement, where prefill is excluded from the metric."""
        g = torch.Generator(device=self.dev)
        g.manual_seed(int(seed))
        P = int(prompt_len)
        scores = torch.rand(self.B, P, generator=g, device=self.dev, dtype=torch.float32)
        need_scores = capi.POLICY_IDS[self.ev.policy] != 0
        self.prefill_head_seed = None  # per-head mode: the scores stand in for layer 0's
        self._select_and_compact(P, scores if need_scores else None)
        for t in (self.kc, self.vc):
            for li in range(t.shape[0]):
                t[li].normal_(generator=g)
        self.tokens.copy_(torch.randint(0, self.cfg.vocab, (self.B,), generator=g, device=self.dev, dtype=torch.int32))

    # ------------------------------------------------------------------ decode
    def _append_evict(self) -> None:
        self._forwarded = False  # the update kernel consumes the pending scores (deferred mode)
        if self.per_head:
            self._append_evict_per_head()
            return
        if self.host_policy is not None:
            self._append_evict_listed()
            return
        if self.deferred_score_update:
            check(
                lib().kvbp_update_append_evict(
                    self.stream, capi.C.byref(self._state), capi.C.byref(self._cfg), _ptr(self.seq_step),
                    _ptr(self.next_pos), _ptr(self.cur_pos), _ptr(self.write_slot), _ptr(self.tokens),
                    _ptr(self.token_log), self.max_new, _ptr(self.evlog), _ptr(self.evcount), self.evcap,
                    _ptr(self.retained_log), _ptr(self.step_score), _ptr(self.upd_pending), _ptr(self.dev_err),
                ),
                "update_append_evict",
            )
            return
        check(
            lib().kvbp_append_evict(
                self.stream, capi.C.byref(self._state), capi.C.byref(self._cfg), _ptr(self.seq_step),
                _ptr(self.next_pos), _ptr(self.cur_pos), _ptr(self.write_slot), _ptr(self.tokens),
                _ptr(self.token_log), self.max_new, _ptr(self.evlog), _ptr(self.evcount), self.evcap,
                _ptr(self.retained_log), _ptr(self.dev_err),
            ),
            "append_evict",
        )

    # ------------------------------------------------------------------ per-KV-head mode
    def _per_head_call(self, signal: np.ndarray, retained: np.ndarray, step: int):
        """One per-head policy call and the union trim (kv_coupled_generator.py:383-433);
        returns (keep (Hkv, n), union (n,))."""
        from .policies import union_trim

        inner = getattr(self.host_policy, "inner", self.host_policy)
        C = self.ev.capacity
        keep = inner.select_per_head_retention(signal, retained.tolist(), C, n_protected=self.n_prefix,
                                               n_suffix_protected=self.n_suffix, orig_prompt_len=self.prompt_len)
        n_union = int(keep.any(axis=0).sum())
        st = self.union_stats
        st[0] = max(st[0], n_union)
        st[1] = max(st[1], max(0, n_union - C))
        st[2] += int(n_union > C)
        union = union_trim(keep, signal, retained, C, self.n_prefix, self.n_suffix)
        self.head_call_steps.append(step)
        return keep, union

    def _per_head_step0(self, P: int, scores):
        """Step 0 in per-head mode (kv_coupled_generator.py:216-325): when the prompt
        exceeds the capacity, the prefill score seeds head 0's signals and one per-head
        call picks the victims (no global policy call otherwise)."""
        Hkv = self.cfg.n_kv_heads
        self.head_ready = False
        self.head_call_steps = []
        self.union_stats = [0, 0, 0]
        if P <= self.ev.capacity:
            return [], None
        seed = (self.prefill_head_seed if getattr(self, "prefill_head_seed", None) is not None else scores)
        seed = np.zeros(P, np.float32) if seed is None else seed[0].float().cpu().numpy()[:P]
        cumul = np.zeros((Hkv, P), np.float64)
        cumul[:1, :P] += seed[None, :]
        cur = np.zeros((Hkv, P), np.float32)
        cur[:1, :P] = seed[None, :]
        self.head_ready = True
        keep, union = self._per_head_call(cur if self.head_uses_current else cumul, np.ones(P, bool), 0)
        return [p for p in range(P) if not union[p]], (keep, cumul, cur)

    def _per_head_load(self, head_state) -> None:
        """Slot-indexed per-head state after the step-0 compaction."""
        self.head_keep.fill_(1)
        self.head_cumul.zero_()
        self.head_current.zero_()
        self.head_score.zero_()
        if head_state is None:
            return
        keep, cumul, cur = head_state
        sp = self.slot_pos[0].cpu().numpy()
        ok = sp >= 0
        kk = np.ones(keep.shape[:1] + sp.shape, np.uint8)
        kk[:, ok] = keep[:, sp[ok]]
        self.head_keep[0].copy_(torch.from_numpy(kk))
        cu = np.zeros(kk.shape, np.float64)
        cu[:, ok] = cumul[:, sp[ok]]
        self.head_cumul[0].copy_(torch.from_numpy(cu))
        cr = np.zeros(kk.shape, np.float32)
        cr[:, ok] = cur[:, sp[ok]]
        self.head_current[0].copy_(torch.from_numpy(cr))

    def _append_evict_per_head(self) -> None:
        """Decode-step bookkeeping in per-head mode.  At a cadence step the host builds the
        position-indexed signals from the device's per-slot ones, runs the per-head call
        and the union trim, and the kernel frees the positions no head keeps (no guardrail,
        as in the reference); then every slot's keep row is written for the next forward.
        If the signal is not ready yet (QUEST before any forward), the reference falls back
        to its global policy call, which is the device's QUEST key."""
        step = int(self.seq_step[0].item()) + 1
        cadence = self.ev.regime == "decode" and step % self.ev.evict_every == 0
        if not cadence or (self.head_uses_current and not self.head_ready):
            check(
                lib().kvbp_append_evict(
                    self.stream, capi.C.byref(self._state), capi.C.byref(self._cfg), _ptr(self.seq_step),
                    _ptr(self.next_pos), _ptr(self.cur_pos), _ptr(self.write_slot), _ptr(self.tokens),
                    _ptr(self.token_log), self.max_new, _ptr(self.evlog), _ptr(self.evcount), self.evcap,
                    _ptr(self.retained_log), _ptr(self.dev_err),
                ),
                "append_evict",
            )
            if cadence:  # global fallback call: freed slots become visible to every head
                self.head_call_steps.append(step)
                free = self.slot_pos[0] < 0
                self.head_keep[0][:, free] = 1
            return
        sp = self.slot_pos[0].cpu().numpy()
        new_pos = int(self.next_pos[0].item())
        n = new_pos + 1
        ok = sp >= 0
        retained = np.zeros(n, bool)
        retained[sp[ok]] = True
        retained[new_pos] = True
        src = (self.head_current if self.head_uses_current else self.head_cumul)[0].cpu().numpy()
        signal = np.zeros((src.shape[0], n), src.dtype)
        signal[:, sp[ok]] = src[:, ok]
        keep, union = self._per_head_call(signal, retained, step)
        vict = [p for p in range(n) if retained[p] and not union[p]]
        if vict:
            self.ext_pos[0, : len(vict)] = torch.tensor(vict, dtype=torch.int32, device=self.dev)
        self.ext_n.fill_(len(vict))
        check(
            lib().kvbp_append_evict_listed(
                self.stream, capi.C.byref(self._state), capi.C.byref(self._cfg), _ptr(self.seq_step),
                _ptr(self.next_pos), _ptr(self.cur_pos), _ptr(self.write_slot), _ptr(self.tokens),
                _ptr(self.token_log), self.max_new, _ptr(self.evlog), _ptr(self.evcount), self.evcap,
                _ptr(self.retained_log), _ptr(self.ext_pos), _ptr(self.ext_n), self.S, capi.LISTED_NO_HARDCAP,
                _ptr(self.dev_err),
            ),
            "append_evict_listed",
        )
        sp2 = self.slot_pos[0].cpu().numpy()
        ok2 = sp2 >= 0
        kk = np.ones((keep.shape[0], sp2.shape[0]), np.uint8)
        kk[:, ok2] = keep[:, sp2[ok2]]
        self.head_keep[0].copy_(torch.from_numpy(kk))

    def _append_evict_listed(self) -> None:
        """Decode-step bookkeeping with host-drawn victims: at a cadence step the host
        reads the retained positions (plus the one this step appends), runs the policy
        call and lists its victims; the kernel appends, frees them and applies the
        hard-capacity guardrail.  Synchronises with the device every step."""
        step = int(self.seq_step[0].item()) + 1
        n = 0
        if self.ev.regime == "decode" and step % self.ev.evict_every == 0:
            sp = self.slot_pos[0].cpu().numpy()
            retained = sorted(sp[sp >= 0].tolist() + [int(self.next_pos[0].item())])
            vict = self._host_victims(retained, max(0, len(retained) - self.ev.capacity), step)
            n = len(vict)
            if n:
                self.ext_pos[0, :n] = torch.tensor(vict, dtype=torch.int32, device=self.dev)
        self.ext_n.fill_(n)
        check(
            lib().kvbp_append_evict_listed(
                self.stream, capi.C.byref(self._state), capi.C.byref(self._cfg), _ptr(self.seq_step),
                _ptr(self.next_pos), _ptr(self.cur_pos), _ptr(self.write_slot), _ptr(self.tokens),
                _ptr(self.token_log), self.max_new, _ptr(self.evlog), _ptr(self.evcount), self.evcap,
                _ptr(self.retained_log), _ptr(self.ext_pos), _ptr(self.ext_n), self.S, 0, _ptr(self.dev_err),
            ),
            "append_evict_listed",
        )

    def _gemm(self, name, epi, N, K, w, x, ldx, out, ldo, norm_w=None, ss_in=None, n_parts=0, ss_out=None):
        c = self.cfg
        check(
            lib().kvbp_decode_gemm(
                self.stream, epi, self.B, N, K, _ptr(w), _ptr(x), ldx, _ptr(ss_in), n_parts, _ptr(norm_w), c.eps,
                _ptr(out), ldo, _ptr(ss_out), self.splits[name], _ptr(self.dev_err),
            ),
            f"decode_gemm[{name}]",
        )

    def _forward(self) -> None:
        if self.gemm == "kvbp":
            self._forward_kvbp()
        else:
            self._forward_cublas()
        self._forwarded = True

    def _forward_kvbp(self) -> None:
        """Forward with the own decode GEMMs: the RMSNorms ride in the GEMM prologues; the
        q/k/v bias, norm, RoPE and cache store, the residual adds and SwiGLU in the
        epilogues (5 launches per layer)."""
        c, st, L, B = self.cfg, self.stream, lib(), self.B
        H, D, F = c.hidden, c.head_dim, c.ffn
        nt_h = H // 128
        check(L.kvbp_embed(st, B, c.vocab, H, _ptr(self.embed_w), _ptr(self.tokens), _ptr(self.h), _ptr(self.dev_err)), "embed")
        check(L.kvbp_row_sumsq(st, B, H, _ptr(self.h), _ptr(self.ss_a)), "row_sumsq")
        ss_in, n_in = self.ss_a, 1
        for li, Lw in enumerate(self.layers):
            check(
                L.kvbp_decode_qkv_gemm(
                    st, B, c.n_heads, c.n_kv_heads, H, _ptr(Lw["w_qkv"]), _ptr(self.h), H, _ptr(ss_in), n_in,
                    _ptr(Lw["in_norm"]), c.eps, _ptr(Lw["b_qkv"]), _ptr(Lw["q_norm"]), _ptr(Lw["k_norm"]),
                    _ptr(self.inv_freq), _ptr(self.cur_pos), _ptr(self.write_slot), self.S, _ptr(self.q),
                    _ptr(self.kc[li]), _ptr(self.vc[li]), self.splits["qkv"], _ptr(self.dev_err),
                ),
                "decode_qkv_gemm",
            )
            self._attention(li)
            self._gemm("o", 1, H, c.n_heads * D, Lw["w_o"], self.attn_out, c.n_heads * D, self.h, H, ss_out=self.ss_b)
            self._gemm("gu", 2, 2 * F, H, Lw["w_gu"], self.h, H, self.act, F, Lw["post_norm"], self.ss_b, nt_h)
            self._gemm("down", 1, H, F, Lw["w_down"], self.act, F, self.h, H, ss_out=self.ss_a)
            ss_in, n_in = self.ss_a, nt_h
        self._gemm("lm", 0, c.vocab, H, self.lm_w, self.h, H, self.logits, c.vocab, self.final_norm, ss_in, n_in)

    @property
    def deferred_score_update(self) -> bool:
        """A step's score update runs at the start of the next step's append kernel
        (kvbp_update_append_evict), so the step needs no launch of its own for it; the
        scores of the last forwarded step stay in step_score until then
        (``apply_pending_scores`` applies them without appending)."""
        return not self.per_head and self.host_policy is None and type(self) is CappedKVEngine

    def apply_pending_scores(self) -> None:
        """Apply a forwarded step's scores that no append has consumed yet (deferred mode)."""
        if not self.deferred_score_update or not self._forwarded:
            return
        check(lib().kvbp_score_update(self.stream, capi.C.byref(self._state), _ptr(self.seq_step),
                                      _ptr(self.step_score), _ptr(self.dev_err)), "score_update")
        self.upd_pending.zero_()
        self._forwarded = False

    def _attention(self, li: int) -> None:
        c, L = self.cfg, lib()
        if self.per_head:
            check(
                L.kvbp_decode_attn_score_heads(
                    self.stream, self.B, c.n_heads, c.n_kv_heads, c.head_dim, self.S, _ptr(self.q), _ptr(self.kc[li]),
                    _ptr(self.vc[li]), _ptr(self.slot_pos), _ptr(self.write_slot), _ptr(self.head_keep),
                    _ptr(self.attn_out), _ptr(self.step_score), _ptr(self.head_score), _ptr(self.dev_err),
                ),
                "decode_attn_score_heads",
            )
            return
        check(
            L.kvbp_decode_attn_score(
                self.stream, self.B, c.n_heads, c.n_kv_heads, c.head_dim, self.S, _ptr(self.q), _ptr(self.kc[li]),
                _ptr(self.vc[li]), _ptr(self.slot_pos), _ptr(self.write_slot), _ptr(self.attn_out),
                _ptr(self.step_score), _ptr(self.dev_err),
            ),
            "decode_attn_score",
        )

    def _forward_cublas(self) -> None:
        """Forward the token of every sequence at cur_pos, writing its K/V to write_slot."""
        c, st, L, B = self.cfg, self.stream, lib(), self.B
        H, D = c.hidden, c.head_dim
        check(L.kvbp_embed(st, B, c.vocab, H, _ptr(self.embed_w), _ptr(self.tokens), _ptr(self.h), _ptr(self.dev_err)), "embed")
        delta = None
        for li, Lw in enumerate(self.layers):
            check(L.kvbp_add_rmsnorm(st, B, H, _ptr(self.h), _ptr(delta), _ptr(Lw["in_norm"]), _ptr(self.x), c.eps), "rmsnorm")
            torch.mm(self.x, Lw["w_qkv"].t(), out=self.qkv)
            check(
                L.kvbp_qkv_rope_scatter(
                    st, B, 1, c.n_heads, c.n_kv_heads, D, self.S, _ptr(self.qkv), c.qkv_dim, _ptr(Lw["b_qkv"]),
                    _ptr(Lw["q_norm"]), _ptr(Lw["k_norm"]), c.eps, _ptr(self.inv_freq), _ptr(self.cur_pos),
                    _ptr(self.write_slot), _ptr(self.q), _ptr(self.kc[li]), _ptr(self.vc[li]), _ptr(self.dev_err),
                ),
                "qkv_rope_scatter",
            )
            self._attention(li)
            torch.mm(self.attn_out, Lw["w_o"].t(), out=self.o)
            check(L.kvbp_add_rmsnorm(st, B, H, _ptr(self.h), _ptr(self.o), _ptr(Lw["post_norm"]), _ptr(self.x), c.eps), "rmsnorm")
            torch.mm(self.x, Lw["w_gu"].t(), out=self.gu)
            check(L.kvbp_silu_mul(st, B, c.ffn, _ptr(self.gu), _ptr(self.act)), "silu_mul")
            torch.mm(self.act, Lw["w_down"].t(), out=self.dn)
            delta = self.dn
        check(L.kvbp_add_rmsnorm(st, B, H, _ptr(self.h), _ptr(self.dn), _ptr(self.final_norm), _ptr(self.x), c.eps), "rmsnorm")
        torch.mm(self.x, self.lm_w.t(), out=self.logits)

    def _sample_and_score(self) -> None:
        L, st, c = lib(), self.stream, self.cfg
        check(L.kvbp_argmax(st, self.B, c.vocab, c.vocab, _ptr(self.logits), _ptr(self.tokens)), "argmax")
        if not self.deferred_score_update:
            check(L.kvbp_score_update(st, capi.C.byref(self._state), _ptr(self.seq_step), _ptr(self.step_score), _ptr(self.dev_err)), "score_update")
        self._head_signal_update()

    def _head_signal_update(self) -> None:
        if self.per_head:
            check(lib().kvbp_head_signal_update(self.stream, self.B, self.cfg.n_kv_heads, self.S, _ptr(self.write_slot),
                                                _ptr(self.head_score), _ptr(self.head_cumul), _ptr(self.head_current),
                                                _ptr(self.dev_err)), "head_signal_update")
            self.head_ready = True

    def decode_step_launches(self, *, forward: bool = True, sample: bool = True) -> None:
        """Enqueue one decode step (no host synchronisation)."""
        self._append_evict()
        if forward:
            self._forward()
            if sample:
                self._sample_and_score()
            else:
                if not self.deferred_score_update:
                    check(lib().kvbp_score_update(self.stream, capi.C.byref(self._state), _ptr(self.seq_step), _ptr(self.step_score), _ptr(self.dev_err)), "score_update")
                self._head_signal_update()

    def capture(self) -> None:
        """Capture one full decode step (append/evict + forward + sample + score) as a graph."""
        if self.host_policy is not None:
            raise ValueError("a host-selected policy synchronises every step: run eager steps, not a graph")
        s = torch.cuda.Stream(self.dev)
        s.wait_stream(torch.cuda.current_stream(self.dev))
        # cuBLAS creates its handle and workspace lazily; do that outside the capture
        if self.gemm == "cublas":
            with torch.cuda.stream(s):
                L0 = self.layers[0]
                for a, w, o in ((self.x, L0["w_qkv"], self.qkv), (self.attn_out, L0["w_o"], self.o),
                                (self.x, L0["w_gu"], self.gu), (self.act, L0["w_down"], self.dn),
                                (self.x, self.lm_w, self.logits)):
                    torch.mm(a, w.t(), out=o)
        s.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                self.decode_step_launches()
        torch.cuda.current_stream(self.dev).wait_stream(s)
        self.graph = g

    def run_step(self, *, use_graph: bool = True) -> None:
        """One decode step for steps 1..max_new-1 (append/evict, forward, sample, score)."""
        if use_graph and self.graph is not None:
            self.graph.replay()
            self._forwarded = True
        else:
            self.decode_step_launches()
        self.step += 1

    def final_step(self) -> None:
        """Step max_new: the sampled token is appended (and evicted at cadence) but not forwarded."""
        self._append_evict()
        self.step += 1

    def demote_positions(self, positions) -> List[List[int]]:
        """Lossy int8 round trip of the K/V of retained positions, every layer and kv head
        (the online-credit generator's demotion, online_credit_generator.py:643-704).
        ``positions[b]`` lists sequence b's positions; positions already demoted, or not
        retained, are skipped.  Returns the positions demoted now, per sequence."""
        if len(positions) != self.B:
            raise ValueError("one position list per sequence")
        if not hasattr(self, "demoted"):
            self.demoted = [set() for _ in range(self.B)]
        sp = self.slot_pos.cpu().numpy()
        done, rows = [], []
        for b in range(self.B):
            where = {int(p): s for s, p in enumerate(sp[b]) if p >= 0}
            new = [int(p) for p in positions[b] if int(p) in where and int(p) not in self.demoted[b]]
            new = list(dict.fromkeys(new))
            self.demoted[b].update(new)
            done.append(new)
            rows.append([where[p] for p in new])
        stride = max(1, max(len(r) for r in rows))
        slots = torch.full((self.B, stride), -1, dtype=torch.int32)
        for b, r in enumerate(rows):
            slots[b, : len(r)] = torch.tensor(r, dtype=torch.int32)
        counts = torch.tensor([len(r) for r in rows], dtype=torch.int32)
        if int(counts.sum()):
            slots_d, counts_d = slots.to(self.dev), counts.to(self.dev)
            c = self.cfg
            check(lib().kvbp_demote_int8(self.stream, _ptr(self.kc), _ptr(self.vc), c.n_layers, self.B, c.n_kv_heads,
                                         self.S, _ptr(slots_d), stride, _ptr(counts_d), _ptr(self.dev_err)),
                  "demote_int8")
            torch.cuda.current_stream(self.dev).synchronize()
        return done

    def check_device_errors(self) -> None:
        word = int(self.dev_err.item())
        if word:
            raise capi.KVBPError("device reported: " + "; ".join(capi.decode_dev_errors(word)))
