"""Tensor parallelism over KV-head groups for the capped-KV decode path.

One process per GPU; rank r of ``world`` holds

* the KV heads ``plan.kv_heads`` and the query heads of their groups (when there are
  fewer KV heads than ranks, each KV head is replicated on ``world / Hkv`` ranks and
  its query group is split between them as evenly as possible), with their slot KV
  cache and the column-parallel q/k/v rows;
* the o projection's columns of those query heads (row-parallel: partial sums);
* a contiguous share of the FFN (gate/up rows, down columns) in 128-wide blocks;
* a contiguous share of the vocabulary (lm_head rows) in 128-wide blocks;
* the full embedding table, norms and the (identical) eviction metadata.

Per decode step the ranks exchange: an allreduce-SUM of the fp32 o and down partial
sums (2 per layer), an allreduce-MAX of the per-slot step score (once, after the last
layer, before the score update), and an allreduce-MAX of the (value, index) argmax key
over the vocabulary shards.  Every rank then holds the same residual stream, tokens and
scores, and runs the same eviction kernels, so victims agree without a broadcast.  This
is the sharding of the reference's mesh (``jax_inference.py:568-588``: q/k/v, gate, up
column-parallel; o, down row-parallel) with the per-slot score reduced as
``max over heads`` (``jax_inference.py:1345``, ``kv_coupled_generator.py:484,497``).

The step is written as a generator that yields ``(op, tensor)`` at each collective
point, so the same code runs with NCCL (``NcclCollective``, one rank per process) and
with all ranks emulated in one process on one GPU (``run_lockstep``), which the tests
use to check the sharded arithmetic against the unsharded engine.
"""

from __future__ import annotations

from dataclasses import dataclass, replace
from typing import Callable, Dict, Iterator, List, Sequence, Tuple

import torch

from . import capi
from .capi import check, lib
from .config import ModelConfig
from .engine import CappedKVEngine, FusedWeights, _ptr, deinterleave_gate_up

Phase = Tuple[str, torch.Tensor]  # ("sum" | "max", tensor reduced in place)


def _split(n: int, parts: int, i: int) -> Tuple[int, int]:
    """[lo, hi) of part i when n items are split into contiguous, balanced parts."""
    base, extra = divmod(n, parts)
    lo = i * base + min(i, extra)
    return lo, lo + base + (1 if i < extra else 0)


@dataclass(frozen=True)
class TPPlan:
    world: int
    rank: int
    kv_heads: Tuple[int, ...]  # global KV head indices held by this rank
    q_heads: Tuple[int, ...]   # global query head indices, grouped by local KV head
    kv_replicas: int           # ranks holding each KV head (1 when Hkv >= world)
    ffn_lo: int
    ffn_hi: int
    vocab_lo: int
    vocab_hi: int


def tp_plan(cfg: ModelConfig, world: int, rank: int) -> TPPlan:
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    Hq, Hkv, G = cfg.n_heads, cfg.n_kv_heads, cfg.group
    if Hkv >= world:
        if Hkv % world:
            raise ValueError(f"{Hkv} KV heads do not split over {world} ranks")
        per = Hkv // world
        kv = tuple(range(rank * per, (rank + 1) * per))
        q = tuple(k * G + j for k in kv for j in range(G))
        rep = 1
    else:
        if world % Hkv:
            raise ValueError(f"{world} ranks do not replicate {Hkv} KV heads evenly")
        rep = world // Hkv
        if rep > G:
            raise ValueError(f"{rep} replicas of a KV head but only {G} query heads per group")
        k, j = divmod(rank, rep)
        lo, hi = _split(G, rep, j)
        kv = (k,)
        q = tuple(k * G + i for i in range(lo, hi))
    if cfg.ffn % 128 or cfg.vocab % 128:
        raise ValueError("ffn and vocab must be multiples of 128 for tensor parallelism")
    flo, fhi = _split(cfg.ffn // 128, world, rank)
    vlo, vhi = _split(cfg.vocab // 128, world, rank)
    return TPPlan(world, rank, kv, q, rep, flo * 128, fhi * 128, vlo * 128, vhi * 128)


def reference_tp_size(cfg: ModelConfig, devices: int) -> int:
    """The tensor-parallel size the reference runs on ``devices`` devices: the largest
    size <= devices that divides the query heads, the KV heads and the FFN width
    (jax_inference.py:1846-1861 clamps a requested TP size this way; Qwen2.5-7B's 4 KV
    heads make it 4 on 8 devices, Qwen3-4B's 8 KV heads keep 8)."""
    t = max(1, int(devices))
    while t > 1 and (cfg.n_heads % t or cfg.n_kv_heads % t or cfg.ffn % t):
        t -= 1
    return t


def tp_groups(world: int, tp_size: int) -> List[List[int]]:
    """Ranks of the tensor-parallel groups when ``world`` ranks run ``world // tp_size``
    data-parallel replicas of a ``tp_size``-way tensor-parallel decode: consecutive ranks
    form a group (on one node they share the NVSwitch fabric equally)."""
    if tp_size < 1 or world % tp_size:
        raise ValueError(f"tensor-parallel size {tp_size} does not divide {world} ranks")
    return [list(range(g * tp_size, (g + 1) * tp_size)) for g in range(world // tp_size)]


def local_config(cfg: ModelConfig, plan: TPPlan) -> ModelConfig:
    """The shapes one rank computes with (its heads, FFN share and vocabulary share)."""
    return replace(
        cfg,
        n_heads=len(plan.q_heads),
        n_kv_heads=len(plan.kv_heads),
        ffn=plan.ffn_hi - plan.ffn_lo,
        vocab=plan.vocab_hi - plan.vocab_lo,
        tie_embed=False,
    )


def shard_weights(cfg: ModelConfig, w: Dict[str, torch.Tensor], plan: TPPlan) -> Dict[str, torch.Tensor]:
    """This rank's weights under the names of ``weights.weight_names`` (local shapes);
    ``embed`` stays whole (token lookup), ``lm_head`` is the rank's vocabulary rows."""
    D = cfg.head_dim

    def heads(t, hs, dim=0):
        return torch.cat([t.narrow(dim, h * D, D) for h in hs], dim)

    out = {"embed": w["embed"], "final_norm": w["final_norm"]}
    out["lm_head"] = (w["embed"] if cfg.tie_embed else w["lm_head"])[plan.vocab_lo : plan.vocab_hi]
    f = slice(plan.ffn_lo, plan.ffn_hi)
    for i in range(cfg.n_layers):
        p = f"l{i}."
        out[p + "in_norm"] = w[p + "in_norm"]
        out[p + "post_norm"] = w[p + "post_norm"]
        out[p + "wq"] = heads(w[p + "wq"], plan.q_heads)
        out[p + "wk"] = heads(w[p + "wk"], plan.kv_heads)
        out[p + "wv"] = heads(w[p + "wv"], plan.kv_heads)
        if cfg.qkv_bias:
            out[p + "bq"] = heads(w[p + "bq"], plan.q_heads)
            out[p + "bk"] = heads(w[p + "bk"], plan.kv_heads)
            out[p + "bv"] = heads(w[p + "bv"], plan.kv_heads)
        if cfg.qk_norm:
            out[p + "q_norm"] = w[p + "q_norm"]
            out[p + "k_norm"] = w[p + "k_norm"]
        out[p + "wo"] = heads(w[p + "wo"], plan.q_heads, dim=1)
        out[p + "w_gate"] = w[p + "w_gate"][f]
        out[p + "w_up"] = w[p + "w_up"][f]
        out[p + "w_down"] = w[p + "w_down"][:, f]
    return out


class NcclCollective:
    """Runs a phase's reduction with torch.distributed (NCCL) on the current stream."""

    def __init__(self, group=None):
        self.group = group

    def __call__(self, op: str, t: torch.Tensor) -> None:
        import torch.distributed as dist

        dist.all_reduce(t, op=dist.ReduceOp.SUM if op == "sum" else dist.ReduceOp.MAX, group=self.group)


class SymmetricBuffer:
    """A device buffer mapped into every rank of the process group (torch symmetric
    memory): ``peers`` is a device array of the ranks' base addresses, for the decode
    GEMM's fused allreduce -- of ranks ``peer_ranks`` only (default: all), so that a
    tensor-parallel group inside a larger job passes the kernel its own ranks' buffers."""

    def __init__(self, nbytes: int, device: torch.device, group=None, peer_ranks: Sequence[int] = None):
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm_mem

        group = group or dist.group.WORLD
        self.nbytes = (int(nbytes) + 255) // 256 * 256
        self.buf = symm_mem.empty(self.nbytes, dtype=torch.uint8, device=device)
        self.handle = symm_mem.rendezvous(self.buf, group.group_name)
        ptrs = list(self.handle.buffer_ptrs)
        if peer_ranks is not None:
            ptrs = [ptrs[r] for r in peer_ranks]
        self.peers = torch.tensor(ptrs, dtype=torch.int64, device=device)
        self.group = group
        self.reset()

    def reset(self) -> None:
        """Zero the flags and receive areas on every rank, then synchronise the ranks."""
        import torch.distributed as dist

        self.buf.zero_()
        torch.cuda.synchronize(self.buf.device)
        dist.barrier(group=self.group)


def allreduce_slot(world: int, M: int, N: int, parity: int, src_rank: int, row: int, col: int) -> int:
    """Byte offset, in every rank's symmetric buffer, of the 16-byte slot {x, tag, y, tag}
    that ``src_rank`` writes for (row, columns col & ~1, col | 1) in a call of this parity."""
    assert 0 <= src_rank < world and 0 <= row < M and 0 <= col < N and parity in (0, 1)
    return (((parity * world + src_rank) * M + row) * (N // 2) + col // 2) * 16


def allreduce_buffer_bytes(world: int, M: int, N: int) -> int:
    """Size of the symmetric buffer kvbp_decode_gemm_allreduce needs (include/kvbp.h):
    [2 parities][world source ranks][M][N / 2] slots of 16 bytes."""
    return 2 * world * M * N * 8


def allreduce_splits(cfg: ModelConfig, world: int, rank: int = 0) -> dict:
    """Split-K factors of this rank's row-parallel o and down GEMMs under tensor
    parallelism: the single-GPU rule on the rank's own K.  The fused allreduce pairs
    values by (source rank, row, column) only, so the ranks need not agree on them."""
    p = tp_plan(cfg, world, rank)
    return {"o": CappedKVEngine._pick_splits(cfg.hidden, len(p.q_heads) * cfg.head_dim),
            "down": CappedKVEngine._pick_splits(cfg.hidden, p.ffn_hi - p.ffn_lo)}


class TPEngine(CappedKVEngine):
    """One rank of a tensor-parallel decode.  ``weights`` is the FULL weight dict (it is
    sharded here) or this rank's prebuilt ``FusedWeights``.  ``collective`` performs the
    reductions when the step runs as one rank of a process group.  With
    ``fused_allreduce`` (one rank per GPU in a real process group) the o/down partial sums
    are reduced inside the GEMMs over NVLink instead of by ``collective``.  ``group`` /
    ``group_ranks``: the tensor-parallel group when the process group holds several
    (data-parallel replicas of the tensor-parallel decode); default the whole world."""

    def __init__(self, cfg: ModelConfig, weights, *, plan: TPPlan, collective: Callable = None,
                 fused_allreduce: bool = False, group=None, group_ranks: Sequence[int] = None, **kw):
        if kw.get("gemm", "kvbp") != "kvbp":
            raise ValueError("tensor parallelism runs on the own decode GEMMs")
        self.full_cfg = cfg
        self.plan = plan
        self.group = group
        self.coll = collective or NcclCollective(group)
        lcfg = local_config(cfg, plan)
        if not isinstance(weights, FusedWeights):
            dev = kw.get("device")
            weights = FusedWeights(lcfg, shard_weights(cfg, weights, plan), torch.device(dev) if dev else
                                   torch.device("cuda", torch.cuda.current_device()))
        super().__init__(lcfg, weights, **kw)
        self.part = torch.zeros(self.B, cfg.hidden, dtype=torch.float32, device=self.dev)
        self.keys = torch.zeros(self.B, dtype=torch.int64, device=self.dev)
        self.splits.update(allreduce_splits(cfg, plan.world, plan.rank))
        self.symm = None
        if fused_allreduce and plan.world > 1:
            # mapped over the whole process group (every rank makes the same call), the
            # kernel given its own group's ranks
            self.symm = SymmetricBuffer(allreduce_buffer_bytes(plan.world, self.B, cfg.hidden), self.dev,
                                        peer_ranks=group_ranks)

    def _allreduce_gemm(self, name, K, w, x, ldx, call, ss_out) -> None:
        c = self.cfg
        check(
            lib().kvbp_decode_gemm_allreduce(
                self.stream, self.B, c.hidden, K, _ptr(w), _ptr(x), ldx, _ptr(self.h), _ptr(ss_out), self.splits[name],
                _ptr(self.symm.peers), self.plan.world, self.plan.rank, call, _ptr(self.seq_step), self.symm.nbytes,
                _ptr(self.dev_err),
            ),
            f"decode_gemm_allreduce[{name}]",
        )

    # ------------------------------------------------------------------ decode
    def _forward_phases(self, sample: bool = True) -> Iterator[Phase]:
        c, st, L, B = self.cfg, self.stream, lib(), self.B
        H, D, F = c.hidden, c.head_dim, c.ffn
        nt_h = H // 128
        check(L.kvbp_embed(st, B, self.full_cfg.vocab, H, _ptr(self.embed_w), _ptr(self.tokens), _ptr(self.h),
                           _ptr(self.dev_err)), "embed")
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
            check(
                L.kvbp_decode_attn_score(
                    st, B, c.n_heads, c.n_kv_heads, D, self.S, _ptr(self.q), _ptr(self.kc[li]), _ptr(self.vc[li]),
                    _ptr(self.slot_pos), _ptr(self.write_slot), _ptr(self.attn_out), _ptr(self.step_score),
                    _ptr(self.dev_err),
                ),
                "decode_attn_score",
            )
            if self.symm is not None:  # allreduce fused into the GEMM over NVLink
                self._allreduce_gemm("o", c.n_heads * D, Lw["w_o"], self.attn_out, c.n_heads * D, 2 * li, self.ss_b)
            else:
                self._gemm("o", 3, H, c.n_heads * D, Lw["w_o"], self.attn_out, c.n_heads * D, self.part, H)
                yield ("sum", self.part)
                check(L.kvbp_residual_add(st, B, H, _ptr(self.h), _ptr(self.part), _ptr(self.ss_b)), "residual_add")
            self._gemm("gu", 2, 2 * F, H, Lw["w_gu"], self.h, H, self.act, F, Lw["post_norm"], self.ss_b, nt_h)
            if self.symm is not None:
                self._allreduce_gemm("down", F, Lw["w_down"], self.act, F, 2 * li + 1, self.ss_a)
            else:
                self._gemm("down", 3, H, F, Lw["w_down"], self.act, F, self.part, H)
                yield ("sum", self.part)
                check(L.kvbp_residual_add(st, B, H, _ptr(self.h), _ptr(self.part), _ptr(self.ss_a)), "residual_add")
            ss_in, n_in = self.ss_a, nt_h
        if sample:
            self._gemm("lm", 0, c.vocab, H, self.lm_w, self.h, H, self.logits, c.vocab, self.final_norm, ss_in, n_in)
            check(L.kvbp_argmax_key(st, B, c.vocab, c.vocab, _ptr(self.logits), self.plan.vocab_lo, _ptr(self.keys)),
                  "argmax_key")
            yield ("max", self.keys)
            check(L.kvbp_key_to_token(st, B, _ptr(self.keys), _ptr(self.tokens)), "key_to_token")

    def step_phases(self, *, forward: bool = True, sample: bool = True) -> Iterator[Phase]:
        """One decode step: append/evict, forward (with its reductions), the score
        allreduce-MAX and the score update."""
        self._append_evict()
        if forward:
            yield from self._forward_phases(sample)
            yield ("max", self.step_score)
            check(lib().kvbp_score_update(self.stream, capi.C.byref(self._state), _ptr(self.seq_step),
                                          _ptr(self.step_score), _ptr(self.dev_err)), "score_update")

    def decode_step_launches(self, *, forward: bool = True, sample: bool = True) -> None:
        for op, t in self.step_phases(forward=forward, sample=sample):
            self.coll(op, t)

    def capture(self) -> None:
        # the communicator is created lazily: do one reduction before the capture
        self.coll("sum", torch.zeros(1, device=self.dev))
        torch.cuda.synchronize(self.dev)
        super().capture()

    # ------------------------------------------------------------------ prefill
    def synthetic_prefill(self, prompt_len: int, seed: int = 0) -> None:
        """As ``CappedKVEngine.synthetic_prefill``, drawing the FULL caches from the seed
        and keeping this rank's KV heads, so every rank (and a replica of a KV head) sees
        the same state."""
        g = torch.Generator(device=self.dev)
        g.manual_seed(int(seed))
        P = int(prompt_len)
        scores = torch.rand(self.B, P, generator=g, device=self.dev, dtype=torch.float32)
        need_scores = capi.POLICY_IDS[self.ev.policy] != 0
        self._select_and_compact(P, scores if need_scores else None)
        fc = self.full_cfg
        kv = list(self.plan.kv_heads)
        for t in (self.kc, self.vc):
            for li in range(t.shape[0]):
                full = torch.empty(self.B, fc.n_kv_heads, self.S, fc.head_dim, dtype=t.dtype, device=self.dev)
                full.normal_(generator=g)
                t[li].copy_(full[:, kv])
                del full
        self.tokens.copy_(torch.randint(0, fc.vocab, (self.B,), generator=g, device=self.dev, dtype=torch.int32))
        if self.symm is not None:
            self.symm.reset()

    def prefill_phases(self, input_ids: torch.Tensor) -> Iterator[Phase]:
        """Step 0 (prompt forward, scores, forced eviction, compaction, first token) with
        this rank's shards; the o/down partial sums, the per-key score and the argmax key
        are the reduction points.  With the own GEMMs (gemm="kvbp") every projection runs on
        the tcgen05 prefill GEMM from the packed shards: q/k/v plain, gate/up with the
        SwiGLU epilogue, o/down as fp32 partial sums (reduced over the ranks, then rounded);
        with gemm="cublas", torch.mm (fp32 for the row-parallel partials)."""
        c, fc, d, st = self.cfg, self.full_cfg, self.dev, self.stream
        L = lib()
        ids = input_ids.to(device=d, dtype=torch.int32).contiguous()
        B, P = ids.shape
        if B != self.B:
            raise ValueError(f"batch {B} != engine batch {self.B}")
        if P <= 0 or P > self.max_prompt:
            raise ValueError(f"prompt length {P} outside 1..{self.max_prompt}")
        need_scores = capi.POLICY_IDS[self.ev.policy] != 0
        Hkv, D, H = c.n_kv_heads, c.head_dim, c.hidden
        pre_k = torch.empty(c.n_layers, B, Hkv, P, D, dtype=torch.bfloat16, device=d)
        pre_v = torch.empty_like(pre_k)
        scores = torch.zeros(B, P, dtype=torch.float32, device=d) if need_scores else None
        positions = torch.arange(P, dtype=torch.int32, device=d)
        fw = self.fw
        own = self.gemm == "kvbp"

        def pgemm(epi, N, K, w, xin, out):
            check(L.kvbp_prefill_gemm(st, epi, P, N, K, _ptr(w), _ptr(xin), xin.stride(0), _ptr(out), out.stride(0),
                                      _ptr(self.dev_err)), "prefill_gemm")

        for b in range(B):
            h = torch.empty(P, H, dtype=torch.bfloat16, device=d)
            check(L.kvbp_embed(st, P, fc.vocab, H, _ptr(self.embed_w), _ptr(ids[b]), _ptr(h), _ptr(self.dev_err)),
                  "embed")
            x = torch.empty_like(h)
            delta = None
            colmax = torch.zeros(P, dtype=torch.float32, device=d) if need_scores else None
            for li, Lw in enumerate(self.layers):
                check(L.kvbp_add_rmsnorm(st, P, H, _ptr(h), _ptr(delta), _ptr(Lw["in_norm"]), _ptr(x), c.eps),
                      "rmsnorm")
                if own:
                    qkv = torch.empty(P, c.qkv_dim, dtype=torch.bfloat16, device=d)
                    pgemm(0, c.qkv_dim, H, Lw["w_qkv"], x, qkv)
                else:
                    qkv = torch.mm(x, fw.rowmajor(Lw["w_qkv"]).t())
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
                if own:
                    part = torch.empty(P, H, dtype=torch.float32, device=d)
                    pgemm(3, H, c.n_heads * D, Lw["w_o"], att, part)
                else:
                    part = att.float() @ fw.rowmajor(Lw["w_o"]).float().t()
                yield ("sum", part)
                o = part.to(torch.bfloat16)
                check(L.kvbp_add_rmsnorm(st, P, H, _ptr(h), _ptr(o), _ptr(Lw["post_norm"]), _ptr(x), c.eps),
                      "rmsnorm")
                act = torch.empty(P, c.ffn, dtype=torch.bfloat16, device=d)
                if own:
                    pgemm(2, 2 * c.ffn, H, Lw["w_gu"], x, act)
                else:
                    gu = deinterleave_gate_up(torch.mm(x, fw.rowmajor(Lw["w_gu"]).t()))
                    check(L.kvbp_silu_mul(st, P, c.ffn, _ptr(gu), _ptr(act)), "silu_mul")
                    del gu
                if own:
                    part = torch.empty(P, H, dtype=torch.float32, device=d)
                    pgemm(3, H, c.ffn, Lw["w_down"], act, part)
                else:
                    part = act.float() @ fw.rowmajor(Lw["w_down"]).float().t()
                yield ("sum", part)
                delta = part.to(torch.bfloat16)
                del act, qkv, q, part
            hl = h[P - 1 : P].contiguous()
            dl = delta[P - 1 : P].contiguous()
            xl = torch.empty_like(hl)
            check(L.kvbp_add_rmsnorm(st, 1, H, _ptr(hl), _ptr(dl), _ptr(self.final_norm), _ptr(xl), c.eps), "rmsnorm")
            check(
                L.kvbp_decode_gemm(st, 0, 1, c.vocab, H, _ptr(self.lm_w), _ptr(xl), H, None, 0, None, c.eps,
                                   _ptr(self.logits[b : b + 1]), c.vocab, None, self.splits["lm"], _ptr(self.dev_err)),
                "decode_gemm[lm]",
            )
            if need_scores:
                yield ("max", colmax)
                scores[b] = colmax
        self._select_and_compact(P, scores, pre_k, pre_v)
        check(L.kvbp_argmax_key(st, B, c.vocab, c.vocab, _ptr(self.logits), self.plan.vocab_lo, _ptr(self.keys)),
              "argmax_key")
        yield ("max", self.keys)
        check(L.kvbp_key_to_token(st, B, _ptr(self.keys), _ptr(self.tokens)), "key_to_token")

    def prefill(self, input_ids: torch.Tensor) -> None:
        for op, t in self.prefill_phases(input_ids):
            self.coll(op, t)
        if self.symm is not None:
            self.symm.reset()


def run_lockstep(phase_iters: Sequence[Iterator[Phase]]) -> None:
    """Run the ranks' phase generators of one emulated process group (all on one device
    and stream) in lockstep: at each collective point the tensors are reduced in rank
    order and every rank receives the result."""
    its: List[Iterator[Phase]] = list(phase_iters)
    while True:
        items = []
        for it in its:
            try:
                items.append(next(it))
            except StopIteration:
                items.append(None)
        if all(x is None for x in items):
            return
        if any(x is None for x in items) or len({x[0] for x in items}) != 1:
            raise RuntimeError("ranks reached different collectives")
        op = items[0][0]
        acc = items[0][1].clone()
        for _, t in items[1:]:
            if op == "sum":
                acc += t
            else:
                torch.maximum(acc, t, out=acc)
        for _, t in items:
            t.copy_(acc)
