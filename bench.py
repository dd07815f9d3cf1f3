#!/usr/bin/env python3
"""Benchmark of the capped-KV decode path on B200.

Headline (``--workload qwen2.5-7b``, the default): decode tokens/s of the
Qwen2.5-7B-architecture decoder (28 layers, hidden 3584, 28 q / 4 kv heads, ffn 18944,
vocab 152064, random bf16 weights) with a 1024-slot capped KV cache, attention-mass
(h2o_faithful) eviction every 8 steps with 10 % prefix/suffix protection, batch 16
sequences per GPU, 32768-token prompts.  Prefill is excluded from the metric (as the
reference's decode_step_* fields exclude it): decoding starts from the post-prefill
state of the prompts -- seeded N(0,1) K/V in the retained slots and U(0,1) prefill
scores passed through the real step-0 selection/compaction kernels.

One step = one decode step of every sequence (slot append + cadence eviction,
28-layer forward, greedy argmax, score update), replayed from one CUDA graph.
Inputs are larger than L2 (15 GB of weights are streamed every step).

Multi-GPU: one process per GPU.  The headline at N > 1 decodes the same 16 sequences
tensor-parallel over KV-head groups (strong scaling; o/down allreduce fused into the
GEMMs over NVLink, score and argmax allreduce-MAX by NCCL).  The tensor-parallel size is
the reference's clamp (the largest size <= N dividing the query heads, KV heads and FFN
width: 2, 4, 4 for the 7B model at N = 2, 4, 8); the rest of N becomes data-parallel
replicas of the group that split the sequences (``--tp-size`` overrides).  The run checks
itself ("tp_check": bit-identical state on the ranks of each group, and logits / victims
against one GPU decoding the same state).  Beside it: "data_parallel" (16 independent sequences per GPU, no
collective, weak scaling) and "configs" -- the Qwen2.5-3B-arch workload (32 sequences
per GPU, capacity 256, LRU, data parallel) and the Qwen3-4B-arch single 65536-token
sequence (capacity 4096, LRU, tensor parallel over its 8 KV heads).  Time = max over
ranks of the device time.

Run ``--impl reference`` for the CPU reference arm (the oracle port of the
reference's decode step timed on the host cores).
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

WORKLOADS = {
    # name: preset, batch, capacity, prompt, policy, multi-GPU parallelism
    # (dp: independent sequences shard with no data-path collective -- every rank decodes
    #  its own `batch` sequences, weak scaling; tp: one decode of `batch` sequences over
    #  all ranks' KV-head groups, strong scaling).  The 7B workload is tensor parallel at
    #  N > 1 (its configuration names tensor parallelism over KV-head groups); its
    #  data-parallel decode is measured beside it ("data_parallel").
    "qwen2.5-7b": ("qwen2.5-7b", 16, 1024, 32768, "attention-mass", "tp"),
    "qwen2.5-3b": ("qwen2.5-3b", 32, 256, 2048, "lru", "dp"),
    "qwen3-4b": ("qwen3-4b", 1, 4096, 65536, "lru", "tp"),
    "tiny-qwen2": ("tiny-qwen2", 1, 256, 1024, "lru", "dp"),
}
ALSO_DP = {"qwen2.5-7b"}
OTHER_CONFIGS = ("qwen2.5-3b", "qwen3-4b")  # measured beside the 7B headline (--no-configs skips)
METRIC = "decode tok/s (Qwen2.5-7B arch, cap 1024) at 1/2/4/8 B200; kernel HBM GB/s"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="qwen2.5-7b", choices=sorted(WORKLOADS))
    ap.add_argument("--batch", type=int, default=None,
                    help="sequences (per GPU under data parallelism, in total under tensor parallelism)")
    ap.add_argument("--parallel", default="auto", choices=["auto", "tp", "dp"],
                    help="multi-GPU scheme (auto: the workload's own, see WORKLOADS)")
    ap.add_argument("--tp-size", type=int, default=None,
                    help="tensor parallelism: ranks per tensor-parallel group (default: the reference's clamp, the "
                         "largest size <= N dividing the query heads, KV heads and FFN width; N / size data-parallel "
                         "groups then split the sequences)")
    ap.add_argument("--no-micro", action="store_true", help="skip the operator microbench sweep")
    ap.add_argument("--no-configs", action="store_true", help="skip the other workloads measured beside the headline")
    ap.add_argument("--no-check", action="store_true", help="skip the tensor-parallel correctness check")
    ap.add_argument("--nccl-allreduce", action="store_true",
                    help="tensor parallelism: reduce the o/down partials with NCCL instead of the fused NVLink GEMM")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline")
    ap.add_argument("--e2e-steps", type=int, default=16)
    ap.add_argument("--micro-only", type=int, default=None, metavar="CAPACITY",
                    help="run only the operator microbench at this capacity (lru, protect 0.10) and exit")
    ap.add_argument("--micro-attn", action="store_true",
                    help="run only the decode attention microbench at the workload's shape and exit")
    ap.add_argument("--micro-prefill", type=int, default=None, metavar="PROMPT_LEN",
                    help="run only the tcgen05 prefill attention microbench at this prompt length and exit")
    ap.add_argument("--micro-prefill-gemm", type=int, default=None, metavar="ROWS",
                    help="run only the tcgen05 prefill projection GEMM microbench over this many prompt rows and exit")
    ap.add_argument("--micro-gemm", action="store_true",
                    help="run only the decode GEMM microbench (one layer's projections + lm_head) and exit")
    return ap.parse_args()


def peaks():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), float(d.get("bf16_tflops", 1590.0)), "measured"
    return 6650.0, 1590.0, "fallback"


# ------------------------------------------------------------------------ clocks
class ClockSampler:
    FIELDS = (
        "index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
        "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap"
    )

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.idx}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL,
            )
        except Exception:
            self.proc = None

    def stop(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        with open(self.path) as f:
            for line in f:
                parts = [x.strip() for x in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    sm.append(float(parts[1]))
                    smax.append(float(parts[2]))
                except ValueError:
                    continue
                for n, v in zip(names, parts[5:9]):
                    if v.lower() == "active":
                        reasons.add(n)
        os.unlink(self.path)
        return {
            "sm_mhz": statistics.median(sm) if sm else None,
            "sm_max_mhz": max(smax) if smax else None,
            "samples": len(sm),
            "reasons": sorted(reasons),
        }


# ------------------------------------------------------------------------ ours
_TP_GROUPS = {}  # tensor-parallel size -> the process groups (created once, by every rank)


def tp_layout(a, cfg, world, rank, B):
    """(tp size, data-parallel replicas, this rank's replica, rank in its group, group,
    group ranks) of a tensor-parallel decode of B sequences over ``world`` ranks: the tp
    size is --tp-size or the reference's clamp (tp.reference_tp_size); the replicas split
    the sequences; with one replica the group is the whole world."""
    import torch.distributed as dist

    from kvcacheboundaryprotection_b200.tp import reference_tp_size, tp_groups

    t = min(a.tp_size or reference_tp_size(cfg, world), world)
    if t < 1 or world % t or B % (world // t):
        t = world  # the sequences do not split over the replicas: one group of every rank
    dp = world // t
    if dp == 1:
        return t, 1, 0, rank, None, None
    groups = tp_groups(world, t)
    if t not in _TP_GROUPS:
        _TP_GROUPS[t] = [dist.new_group(r) for r in groups]  # collective: every rank, every group
    g = rank // t
    return t, dp, g, rank % t, _TP_GROUPS[t][g], groups[g]


def _build_engine(a, workload, tp, rank, world, dev, B, n_new, seed_rank):
    """The workload's engine on this rank: tensor-parallel (TPEngine over its group's
    KV-head shards, the same synthetic post-prefill state on every rank of a group, B /
    replicas sequences per group) or one GPU's independent sequences (CappedKVEngine, its
    own seeded state)."""
    import torch

    from kvcacheboundaryprotection_b200.config import get_config
    from kvcacheboundaryprotection_b200.engine import CappedKVEngine, EvictionSpec, FusedWeights
    from kvcacheboundaryprotection_b200.weights import init_weights

    preset, _, C, P, policy, _ = WORKLOADS[workload]
    cfg = get_config(preset)
    spec = EvictionSpec(policy, C, 8, True, 0.10, 0.10)
    weights = init_weights(cfg, seed=0, device=dev)
    if tp:
        from kvcacheboundaryprotection_b200.tp import TPEngine, local_config, shard_weights, tp_plan

        t, dp, g, trank, group, granks = tp_layout(a, cfg, world, rank, B)
        plan = tp_plan(cfg, t, trank)
        fw = FusedWeights(local_config(cfg, plan), shard_weights(cfg, weights, plan), dev)
        del weights
        torch.cuda.empty_cache()
        eng = TPEngine(cfg, fw, plan=plan, fused_allreduce=not a.nccl_allreduce, batch=B // dp, evict=spec,
                       max_prompt_len=P, max_new_tokens=n_new, device=dev, group=group, group_ranks=granks)
        eng.tp_size, eng.replicas, eng.replica = t, dp, g
        eng.synthetic_prefill(P, seed=1234 + g)
    else:
        fw = FusedWeights(cfg, weights, dev)
        del weights
        torch.cuda.empty_cache()
        eng = CappedKVEngine(cfg, fw, batch=B, evict=spec, max_prompt_len=P, max_new_tokens=n_new, device=dev)
        eng.synthetic_prefill(P, seed=1234 + seed_rank)
    torch.cuda.synchronize()
    return cfg, eng, fw


def decode_run(a, workload, par, rank, world, local_rank, *, steps, warmup, full=True):
    """Decode throughput of one workload: K graph replays timed with device events
    between barriers, max over ranks.  ``par``: "tp" (one decode of the workload's
    sequences over all ranks, strong scaling) or "dp" (each rank decodes its own
    sequences, no data-path collective, weak scaling).  With ``full`` also the end-to-end
    number through host buffers and clocks; always the per-kernel table and rooflines."""
    import torch
    import torch.distributed as dist

    dev = torch.device("cuda", local_rank)
    preset, B0, C, P, policy, _ = WORKLOADS[workload]
    tp = world > 1 and par == "tp"
    B = (a.batch or B0) if workload == a.workload else B0
    K, W = steps, warmup
    n_new = W + K + (a.e2e_steps if full else 0) + 16
    cfg, eng, fw = _build_engine(a, workload, tp, rank, world, dev, B, n_new, rank)
    Br = eng.B  # this rank's sequences (a tensor-parallel group's share of the B under tp)
    eng.capture()
    for _ in range(W):
        eng.run_step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks = None
    if full:
        cvd = [x for x in os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",") if x.strip().isdigit()]
        clocks = ClockSampler(int(cvd[local_rank]) if len(cvd) > local_rank else local_rank)
        clocks.start()
        time.sleep(0.3)
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(K):
        eng.run_step()
    e1.record()
    torch.cuda.synchronize()
    ck = clocks.stop() if clocks else None
    ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        dist.barrier()
    seqs = B if tp else world * B  # sequences decoded per step by the whole job
    value = seqs * K / (ms / 1000.0)
    eng.check_device_errors()

    e2e = None
    if full:
        # end to end through host buffers: the host feeds each step's tokens and reads them back
        pin_in = torch.empty(Br, dtype=torch.int32, pin_memory=True)
        pin_out = torch.empty(Br, dtype=torch.int32, pin_memory=True)
        pin_in.copy_(eng.tokens.cpu())
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(a.e2e_steps):
            eng.tokens.copy_(pin_in, non_blocking=True)
            eng.run_step()
            pin_out.copy_(eng.tokens, non_blocking=True)
            torch.cuda.current_stream().synchronize()
            pin_in.copy_(pin_out)
        e2e_s = time.perf_counter() - t0
        if world > 1:
            t = torch.tensor([e2e_s], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            e2e_s = float(t.item())
        e2e = {
            "value": round(seqs * a.e2e_steps / e2e_s, 2),
            "unit": "tok/s",
            "h2d_bytes_per_step": 4 * Br,  # per rank
            "d2h_bytes_per_step": 4 * Br,
            "how": "host copies each step's token ids in from pinned memory, replays the step, reads the sampled ids back and synchronises",
        }

    # ---- live per-kernel timing (the step's launches of each kind replayed as a burst)
    km = measure_kernels_in_step(eng, steps=2)
    hbm, tf, peak_kind = peaks()
    avg_valid = C + 3.5  # retained slots per (sequence, kv head): C .. C+E-1 over a cadence
    kbytes = kernel_algorithmic_bytes(eng.cfg, Br, avg_valid)  # this rank's shapes
    per_step = {"attention": cfg.n_layers, "qkv": cfg.n_layers, "o": cfg.n_layers, "gate_up": cfg.n_layers,
                "down": cfg.n_layers, "lm_head": 1}
    kernels = {}
    for k, te in km["eager"].items():
        t = km["burst"].get(k, te)
        gbs = kbytes[k] / (t * 1e-3) / 1e9
        kernels[k] = {"avg_launch_us": round(t * 1000, 2),
                      "timing": "burst" if k in km["burst"] else "eager",
                      "eager_launch_us": round(te * 1000, 2), "launches_per_step": per_step[k],
                      "algorithmic_bytes_per_launch": int(kbytes[k]), "achieved_gbs": round(gbs, 1),
                      "frac": round(gbs / hbm, 4), "traffic": None if tp else NCU_TRAFFIC.get((preset, k))}
    dominant = max(kernels, key=lambda k: kernels[k]["avg_launch_us"] * per_step[k])

    def roofline_of(k):
        d = kernels[k]
        return {"kernel": k, "bound": "hbm", "achieved": d["achieved_gbs"], "peak": hbm,
                "peak_kind": f"{peak_kind} HBM copy bandwidth", "unit": "GB/s", "frac": d["frac"],
                "traffic": d["traffic"], "avg_launch_us": d["avg_launch_us"],
                "timing": (d["timing"] + ": the step's launches of this kernel back to back in a CUDA graph, "
                           "events around the replays" if d["timing"] == "burst" else
                           d["timing"] + ": events around each eager launch"),
                "algorithmic_bytes_per_launch": d["algorithmic_bytes_per_launch"]}

    if tp:
        tsz, reps = getattr(eng, "tp_size", world), getattr(eng, "replicas", 1)
        tp_par = f"tp{tsz}" + (f"xdp{reps}" if reps > 1 else "")
        tp_desc = (f"{B} sequences tensor-parallel over {world} GPUs" if reps == 1 else
                   f"{B} sequences: {reps} data-parallel groups of {Br}, each tensor-parallel over {tsz} GPUs "
                   f"(the reference's TP clamp for {eng.full_cfg.n_kv_heads} KV heads)")
    lc = eng.cfg
    step_bytes = fw.streamed_bytes(Br) + cfg.n_layers * algorithmic_attn_bytes(Br, lc.n_heads, lc.n_kv_heads, avg_valid)
    step_ms = ms / K
    out = {
        "metric": METRIC,
        "value": round(value, 2),
        "unit": "tok/s",
        "n_gpus": world,
        "steps": K,
        "warmup": W,
        "ms_per_step": round(step_ms, 4),
        "higher_is_better": True,
        "scaling": "strong" if tp else "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded random bf16 weights N(0,0.02); decode from a synthetic post-prefill state)",
        "config": {
            "workload": f"{preset} decode, capacity {C}, {policy} eviction every 8 steps, protect-frac 0.10, "
            + (tp_desc if tp else f"{B} sequences/GPU")
            + f", prompt {P}, greedy",
            "batch_per_gpu": Br,
            "global_batch": seqs,
            "capacity": C,
            "prompt_len": P,
            "policy": policy,
            "parallelism": tp_par if tp else f"dp{world}",
            "allreduce": "fused NVLink GEMM epilogue (o, down) + NCCL (score, argmax)" if tp else None,
            "l2": "inputs larger than L2 (all weights streamed every step)",
        },
        "roofline": roofline_of(dominant),
        "roofline_attention": roofline_of("attention"),
        "kernels": kernels,
        "step_roofline": {
            "bytes_per_step": int(step_bytes),
            "achieved_gbs": round(step_bytes / (step_ms * 1e-3) / 1e9, 1),
            "frac": round(step_bytes / (step_ms * 1e-3) / 1e9 / hbm, 4),
            "note": "bytes one decode step must read on one GPU (every weight matrix and the lm_head of this rank; "
                    "B rows of the embedding table; K/V, q, out) / measured step time (all kernels own sm_100a)",
        },
        "gpu_launches": K * launches_per_step(cfg, tp),
    }
    if e2e:
        out["e2e"] = e2e
    if ck:
        out["clocks"] = ck
    return out, eng, fw


def _checksum(t):
    """Order-sensitive integer digest of a tensor's bytes (for cross-rank identity)."""
    import torch

    b = t.contiguous().view(-1).view(torch.uint8).to(torch.int64)
    w = torch.arange(b.numel(), device=b.device, dtype=torch.int64) % 65521 + 1
    return int((b * w).sum().item())


def tp_check(a, workload, rank, world, local_rank, eng, steps=8):
    """Correctness of the tensor-parallel run (the fused NVLink allreduce included).

    1. After the timed steps every rank must hold bit-identical token logs, eviction
       logs and counts, slot tables, float64 cumulative scores and residual streams
       (the allreduce sums the ranks' partials in rank order on every rank).
    2. From one fresh synthetic state, ``steps`` teacher-forced decode steps (the last one
       an eviction cadence step) of the tensor-parallel engine against one GPU decoding
       the same state with the full weights (CappedKVEngine).  Summing the row-parallel
       partials in another order moves bf16 results by an ulp here and there, which
       compounds over the layers, so the tolerance is calibrated in the same run: the
       single-GPU engine is run a second time with other split-K counts for its o / down
       projections (another summation order, equally valid), and the tensor-parallel
       logits must stay within twice that noise floor (max and mean |diff| over the
       steps before the cadence step) with identical greedy tokens wherever the top-2
       gap exceeds the floor; at the cadence step >= 90 % of the victims must agree."""
    import torch
    import torch.distributed as dist

    from kvcacheboundaryprotection_b200.engine import CappedKVEngine, EvictionSpec, FusedWeights
    from kvcacheboundaryprotection_b200.weights import init_weights

    dev = torch.device("cuda", local_rank)
    names = ["token_log", "evlog", "evcount", "slot_pos", "cumul", "h", "tokens", "retained_log"]
    mine = torch.tensor([_checksum(getattr(eng, n)) for n in names], dtype=torch.int64, device=dev)
    # the ranks of one tensor-parallel group decode the same sequences (data-parallel
    # replicas of the group decode others)
    allv = [torch.empty_like(mine) for _ in range(eng.plan.world)]
    dist.all_gather(allv, mine, group=eng.group)
    differ = [names[i] for i in range(len(names)) if any(int(v[i]) != int(allv[0][i]) for v in allv)]
    gate = torch.tensor([1 if differ else 0], dtype=torch.int32, device=dev)
    dist.all_reduce(gate, op=dist.ReduceOp.MAX)  # any group's ranks differ
    if int(gate.item()) and not differ:
        differ = ["(another tensor-parallel group)"]

    preset, B0, C, P, policy, _ = WORKLOADS[workload]
    B = eng.B  # this group's sequences
    cfg = eng.full_cfg
    ref = CappedKVEngine(cfg, FusedWeights(cfg, init_weights(cfg, seed=0, device=dev), dev), batch=B,
                         evict=EvictionSpec(policy, C, 8, True, 0.10, 0.10), max_prompt_len=P,
                         max_new_tokens=steps + 4, device=dev)
    torch.cuda.empty_cache()
    lo, hi = eng.plan.vocab_lo, eng.plan.vocab_hi

    def run(e, forced=None):
        e.synthetic_prefill(P, seed=4321)
        logits, toks = [], []
        for s in range(steps):
            if forced is not None:
                e.tokens.copy_(forced[s])
            toks.append(e.tokens.clone())
            e.decode_step_launches()
            torch.cuda.synchronize()
            logits.append(e.logits.float().clone())
        n = int(e.evcount.max().item())
        return logits, toks, e.evlog[:, :n].clone(), e.evcount.clone()

    l1, toks, ev1, n1 = run(ref)
    default = dict(ref.splits)
    ref.splits.update(o=max(1, default["o"] // 2), down=max(1, default["down"] // 2))
    l2, _, _, _ = run(ref, toks)
    ref.splits.update(default)
    lt, _, evt, nt = run(eng, toks)
    eng.check_device_errors()
    ref.check_device_errors()
    del ref
    torch.cuda.empty_cache()
    pre = steps - 1  # steps before the cadence step
    floor_max = max(float((l2[s] - l1[s]).abs().max()) for s in range(pre))
    floor_mean = max(float((l2[s] - l1[s]).abs().mean()) for s in range(pre))
    tp_max = max(float((lt[s] - l1[s][:, lo:hi]).abs().max()) for s in range(pre))
    tp_mean = max(float((lt[s] - l1[s][:, lo:hi]).abs().mean()) for s in range(pre))
    # greedy tokens: where the reference's top-2 gap exceeds the tolerance and its
    # maximum lies in this rank's vocabulary shard, the shard's argmax must match it
    shard_ok = 0
    shard_n = 0
    for s in range(pre):
        top2 = l1[s].topk(2, dim=1).values
        dec = (top2[:, 0] - top2[:, 1]) > 2 * floor_max + 2e-2
        want = l1[s].argmax(1)
        in_shard = (want >= lo) & (want < hi) & dec
        got = lt[s].argmax(1) + lo
        shard_n += int(in_shard.sum())
        shard_ok += int((in_shard & (got == want)).sum())
    cnt = torch.tensor([shard_ok, shard_n], dtype=torch.int64, device=dev)
    dist.all_reduce(cnt)
    common = sum(len(set(ev1[b, : int(n1[b])].tolist()) & set(evt[b, : int(nt[b])].tolist())) for b in range(B))
    total = int(n1.sum())
    vals = torch.tensor([tp_max, tp_mean, floor_max, floor_mean], device=dev)
    dist.all_reduce(vals, op=dist.ReduceOp.MAX)
    tp_max, tp_mean, floor_max, floor_mean = (float(x) for x in vals)
    overlap = common / max(1, total)
    ov = torch.tensor([overlap], device=dev)
    dist.all_reduce(ov, op=dist.ReduceOp.MIN)
    overlap = float(ov)
    argmax_ok = int(cnt[0]) == int(cnt[1])
    ok = (not differ and tp_max <= 2 * floor_max + 1e-2 and tp_mean <= 2 * floor_mean + 1e-3 and argmax_ok
          and overlap >= 0.9)
    return {
        "status": "ok" if ok else "FAILED",
        "ranks_identical": not differ,
        "ranks_differ_in": differ,
        "vs_1gpu_steps": steps,
        "vs_1gpu_max_logit_diff": round(tp_max, 5),
        "vs_1gpu_mean_logit_diff": round(tp_mean, 6),
        "noise_floor_max_logit_diff": round(floor_max, 5),
        "noise_floor_mean_logit_diff": round(floor_mean, 6),
        "decisive_argmax_agree": f"{int(cnt[0])}/{int(cnt[1])}",
        "cadence_victim_overlap": round(overlap, 4),
        "how": "bit-identical state across ranks after the timed steps; then teacher-forced steps from one fresh "
               "state against a single-GPU engine with the full weights, tolerance = 2x the noise floor of the "
               "same single-GPU engine with other o/down split-K counts",
    }


def launches_per_step(cfg, tp: bool = False) -> int:
    # own kernels: update_append_evict (the previous step's score update runs in it), embed,
    # row_sumsq, per layer (q/k/v GEMM, attention, o GEMM, gate/up GEMM, down GEMM),
    # lm_head GEMM, argmax; tensor parallel: append_evict, argmax_key + key_to_token and a
    # separate score_update; NCCL's own kernels are not counted
    return 1 + 1 + 1 + cfg.n_layers * 5 + 1 + (2 if tp else 1) + (1 if tp else 0)


def algorithmic_attn_bytes(B, Hq, Hkv, valid_slots):
    """Bytes one decode_attn_score launch must move: K+V of every valid slot, q in,
    out, plus the per-slot score read-modify-write."""
    kv = 2 * B * Hkv * valid_slots * 128 * 2
    qo = 2 * B * Hq * 128 * 2
    score = B * valid_slots * 4 * 2
    return kv + qo + score


def measure_kernels_in_step(eng, steps=3, reps=5):
    """Device time (ms) of each kind of heavy kernel of the decode step, two ways, on the
    launching stream.  Keys: attention, qkv, o, gate_up, down, lm_head.

    burst: the launches of one real step of that kind (one per layer, with the step's own
    arguments) captured back to back into a CUDA graph, replayed ``reps`` times between
    two events; per launch = elapsed / launches.  Consecutive launches overlap only as
    they do inside the step (programmatic dependent launch), and their operands (one
    layer's weights or KV cache each) add up to more than L2 holds.  This is the kernel
    duration the roofline uses.
    eager: CUDA events around each eager launch of ``steps`` steps; it includes the
    front-end gap of an isolated launch (a few microseconds per launch).

    The fused-allreduce GEMMs of the tensor-parallel engine are not replayed (their
    cross-rank flags are tied to the step's call sequence): their burst time is absent."""
    import torch

    from kvcacheboundaryprotection_b200.capi import lib

    c = eng.cfg
    times = {}
    stream = torch.cuda.current_stream()
    L = lib()

    def kind_of_gemm(args):
        epi, N, K = args[1], args[3], args[4]
        if epi == 2:
            return "gate_up"
        if epi in (1, 3):  # residual in place, or fp32 partial sums under tensor parallelism
            return "down" if K == c.ffn else "o"
        return "lm_head"

    def wrap(orig, kind):
        def f(*args):
            a = torch.cuda.Event(enable_timing=True)
            b = torch.cuda.Event(enable_timing=True)
            a.record(stream)
            r = orig(*args)
            b.record(stream)
            times.setdefault(kind(args) if callable(kind) else kind, []).append((a, b))
            return r

        return f

    calls = {}

    def record(orig, kind, name):
        def f(*args):
            calls.setdefault(kind(args) if callable(kind) else kind, []).append((name, orig, args))
            return orig(*args)

        return f

    names = {"kvbp_decode_attn_score": "attention", "kvbp_decode_attn_score_update": "attention",
             "kvbp_decode_qkv_gemm": "qkv", "kvbp_decode_gemm": kind_of_gemm,
             "kvbp_decode_gemm_allreduce": lambda args: "down" if args[3] == c.ffn else "o"}
    saved = {n: getattr(L, n) for n in names}
    try:
        for n, kind in names.items():
            setattr(L, n, wrap(saved[n], kind))
        for _ in range(steps):
            eng.decode_step_launches()
            eng.step += 1
        torch.cuda.synchronize()
        for n, kind in names.items():
            setattr(L, n, record(saved[n], kind, n))
        eng.decode_step_launches()
        eng.step += 1
        torch.cuda.synchronize()
    finally:
        for n, f in saved.items():
            setattr(L, n, f)
    eager = {k: sum(a.elapsed_time(b) for a, b in v) / len(v) for k, v in times.items()}
    burst = {}
    for k, lst in calls.items():
        if any(n == "kvbp_decode_gemm_allreduce" for n, _, _ in lst):
            continue
        side = torch.cuda.Stream()
        side.wait_stream(stream)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(side):
            with torch.cuda.graph(g, stream=side):
                h = torch.cuda.current_stream().cuda_stream
                for _, orig, args in lst:
                    orig(h, *args[1:])
        stream.wait_stream(side)
        g.replay()
        torch.cuda.synchronize()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            g.replay()
        e1.record(stream)
        torch.cuda.synchronize()
        burst[k] = e0.elapsed_time(e1) / (reps * len(lst))
        del g
    return {"burst": burst, "eager": eager}


def kernel_algorithmic_bytes(cfg, B, avg_valid):
    """Bytes each heavy kernel of the decode step must move per launch (weights read
    once; activations in and out; K/V of the valid slots for attention)."""
    H, F, V, D = cfg.hidden, cfg.ffn, cfg.vocab, cfg.head_dim
    qkv_n = (cfg.n_heads + 2 * cfg.n_kv_heads) * D
    return {
        "attention": algorithmic_attn_bytes(B, cfg.n_heads, cfg.n_kv_heads, avg_valid),
        "qkv": qkv_n * H * 2 + B * H * 2 + B * qkv_n * 2,
        "o": H * cfg.n_heads * D * 2 + B * cfg.n_heads * D * 2 + 2 * B * H * 2,
        "gate_up": 2 * F * H * 2 + B * H * 2 + B * F * 2,
        "down": H * F * 2 + B * F * 2 + 2 * B * H * 2,
        "lm_head": V * H * 2 + B * H * 2 + B * V * 2,
    }


# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of one launch, from ncu
# captures on B200 at the qwen2.5-7b shapes: the attention from this file's --micro-attn
# run, the GEMMs from run_gemm_microbench("qwen2.5-7b", M=16) (its q/k/v launch is the
# same main loop and weight stream as the step's, with the plain epilogue).
NCU_TRAFFIC = {
    ("qwen2.5-7b", "attention"): 34129152,
    ("qwen2.5-7b", "qkv"): 33217536,
    ("qwen2.5-7b", "o"): 25949440,
    ("qwen2.5-7b", "gate_up"): 271760384 + 384000,
    ("qwen2.5-7b", "down"): 136550144 + 708096,
    ("qwen2.5-7b", "lm_head"): 1090553600 + 4642560,
}


# ------------------------------------------------------------------------ microbench
def run_microbench(cap_list=(256, 1024, 4096), policies=("lru", "attention-mass"), fracs=(0.10, 0.05), iters=16):
    """Operator microbench: one fused decode attention + eviction step for 64 sequences,
    8 kv heads x group 4, head_dim 128.  The step is two launches: kvbp_update_append_evict
    (the previous step's score update, then slot append + cadence protection / top-k / hard
    cap) and kvbp_decode_attn_score_update without state (scatter of the new K/V row into
    its slot, attention + per-slot score); q and the new K/V rows are the operator's inputs,
    and every step applies the previous step's scores (steady state).  "unfused_step_us"
    times the same step as four launches (append, q/k RoPE + K/V scatter, attention, score
    update).  Each timed step is preceded by an L2 flush (a 512 MB read, which leaves no
    dirty lines behind) outside the CUDA-event pair."""
    import ctypes as C_

    import torch

    from kvcacheboundaryprotection_b200 import capi
    from kvcacheboundaryprotection_b200.capi import check, lib
    from kvcacheboundaryprotection_b200.engine import inv_freq_table

    L = lib()
    dev = torch.device("cuda")
    B, Hkv, G, D, E = 64, 8, 4, 128, 8
    Hq = Hkv * G
    hbm, _, peak_kind = peaks()
    flush = torch.empty(512 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)
    out = []
    for C in cap_list:
        S = C + E
        g = torch.Generator(device=dev).manual_seed(C)
        kc = torch.randn(B, Hkv, S, D, generator=g, device=dev).to(torch.bfloat16)
        vc = torch.randn(B, Hkv, S, D, generator=g, device=dev).to(torch.bfloat16)
        P0 = 4 * C
        for pol in policies:
            for frac in fracs:
                st = _micro_state(B, S, C, P0, dev, g)
                n_pre, n_suf = capi.protection_sizes(C, frac, frac)
                cfg = capi.EvictCfg(C, E, capi.policy_id(pol), 1, n_pre, n_suf, 1)
                qkv = (torch.randn(B, (Hq + 2 * Hkv) * D, generator=g, device=dev) / math.sqrt(D)).to(torch.bfloat16)
                q = torch.empty(B, Hq, D, dtype=torch.bfloat16, device=dev)
                attn_out = torch.empty_like(q)
                inv = torch.from_numpy(inv_freq_table(D, 1e6)).to(dev)
                err = torch.zeros(1, dtype=torch.int32, device=dev)
                qf = (torch.randn(B, Hq, D, generator=g, device=dev) / math.sqrt(D)).to(torch.bfloat16)
                knew = torch.randn(B, Hkv, D, generator=g, device=dev).to(torch.bfloat16)
                vnew = torch.randn(B, Hkv, D, generator=g, device=dev).to(torch.bfloat16)
                pending = torch.ones(B, dtype=torch.int32, device=dev)

                def fused_step():
                    s = torch.cuda.current_stream().cuda_stream
                    check(L.kvbp_update_append_evict(s, C_.byref(st["state"]), C_.byref(cfg), st["seq_step"].data_ptr(), st["next_pos"].data_ptr(), st["cur_pos"].data_ptr(), st["write_slot"].data_ptr(), None, None, 0, st["evlog"].data_ptr(), st["evcount"].data_ptr(), st["evcap"], None, st["step_score"].data_ptr(), pending.data_ptr(), err.data_ptr()), "update_append")
                    check(L.kvbp_decode_attn_score_update(s, B, Hq, Hkv, D, S, qf.data_ptr(), knew.data_ptr(), vnew.data_ptr(), kc.data_ptr(), vc.data_ptr(), st["slot_pos"].data_ptr(), st["write_slot"].data_ptr(), attn_out.data_ptr(), st["step_score"].data_ptr(), None, None, None, err.data_ptr()), "attn_scatter")

                def step(ev=None):
                    s = torch.cuda.current_stream().cuda_stream
                    mark = (lambda i: ev[i].record()) if ev else (lambda i: None)
                    mark(0)
                    check(L.kvbp_append_evict(s, C_.byref(st["state"]), C_.byref(cfg), st["seq_step"].data_ptr(), st["next_pos"].data_ptr(), st["cur_pos"].data_ptr(), st["write_slot"].data_ptr(), None, None, 0, st["evlog"].data_ptr(), st["evcount"].data_ptr(), st["evcap"], None, err.data_ptr()), "append")
                    mark(1)
                    check(L.kvbp_qkv_rope_scatter(s, B, 1, Hq, Hkv, D, S, qkv.data_ptr(), (Hq + 2 * Hkv) * D, None, None, None, 1e-6, inv.data_ptr(), st["cur_pos"].data_ptr(), st["write_slot"].data_ptr(), q.data_ptr(), kc.data_ptr(), vc.data_ptr(), err.data_ptr()), "qkv")
                    mark(2)
                    check(L.kvbp_decode_attn_score(s, B, Hq, Hkv, D, S, q.data_ptr(), kc.data_ptr(), vc.data_ptr(), st["slot_pos"].data_ptr(), st["write_slot"].data_ptr(), attn_out.data_ptr(), st["step_score"].data_ptr(), err.data_ptr()), "attn")
                    mark(3)
                    check(L.kvbp_score_update(s, C_.byref(st["state"]), st["seq_step"].data_ptr(), st["step_score"].data_ptr(), err.data_ptr()), "score")
                    mark(4)

                def graph_of(fn):
                    for _ in range(3):
                        fn()
                    gr_ = torch.cuda.CUDAGraph()
                    side = torch.cuda.Stream()
                    side.wait_stream(torch.cuda.current_stream())
                    with torch.cuda.stream(side):
                        with torch.cuda.graph(gr_, stream=side):
                            fn()
                    torch.cuda.current_stream().wait_stream(side)
                    return gr_

                def timed_replays(gr_):
                    gr_.replay()  # the first replay of a graph pays its upload: not a step's time
                    torch.cuda.synchronize()
                    t = 0.0
                    for it in range(iters):
                        flush.sum()
                        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                        e0.record()
                        gr_.replay()
                        e1.record()
                        torch.cuda.synchronize()
                        t += e0.elapsed_time(e1)
                    return t

                gr = graph_of(fused_step)
                tot = timed_replays(gr)
                del gr
                gr = graph_of(step)
                tot_unfused = timed_replays(gr)
                del gr

                def attn_alone():
                    check(L.kvbp_decode_attn_score(torch.cuda.current_stream().cuda_stream, B, Hq, Hkv, D, S, q.data_ptr(), kc.data_ptr(), vc.data_ptr(), st["slot_pos"].data_ptr(), st["write_slot"].data_ptr(), attn_out.data_ptr(), st["step_score"].data_ptr(), err.data_ptr()), "attn")

                # attention kernel alone (a one-launch graph, same L2 discipline)
                gr = graph_of(attn_alone)
                attn_only = timed_replays(gr)
                # the step's kernels one by one (eager, events between launches), over one
                # eviction cycle of E steps
                per = [0.0] * 4
                for it in range(E):
                    ev = [torch.cuda.Event(enable_timing=True) for _ in range(5)]
                    step(ev)
                    torch.cuda.synchronize()
                    for k in range(4):
                        per[k] += ev[k].elapsed_time(ev[k + 1]) * 1000 / E
                torch.cuda.synchronize()
                if int(err.item()):
                    raise RuntimeError("device error in microbench: " + str(capi.decode_dev_errors(int(err.item()))))
                us = tot / iters * 1000
                us_unfused = tot_unfused / iters * 1000
                valid = C + E / 2
                byts = micro_bytes(B, Hq, Hkv, valid, E)
                ab = algorithmic_attn_bytes(B, Hq, Hkv, valid)
                aus = attn_only / iters * 1000
                out.append(
                    {
                        "capacity": C,
                        "policy": pol,
                        "protect_frac": frac,
                        "step_us": round(us, 2),
                        "step_gbs": round(byts / (us * 1e-6) / 1e9, 1),
                        "step_frac": round(byts / (us * 1e-6) / 1e9 / hbm, 4),
                        "launches": 2,
                        "unfused_step_us": round(us_unfused, 2),
                        "unfused_step_frac": round(byts / (us_unfused * 1e-6) / 1e9 / hbm, 4),
                        "attn_us": round(aus, 2),
                        "attn_gbs": round(ab / (aus * 1e-6) / 1e9, 1),
                        "attn_frac": round(ab / (aus * 1e-6) / 1e9 / hbm, 4),
                        "eager_us": {"append_evict": round(per[0], 2), "qkv_rope_scatter": round(per[1], 2),
                                     "attention": round(per[2], 2), "score_update": round(per[3], 2)},
                    }
                )
                del gr
        del kc, vc
    return {"peak_gbs": hbm, "peak_kind": peak_kind, "batch": B, "kv_heads": Hkv, "group": G, "rows": out}


def run_attn_microbench(preset="qwen2.5-7b", B=16, C=1024, E=8, layers=8, iters=5):
    """Operator microbench of kvbp_decode_attn_score at a decode workload's shape: B
    sequences, the preset's heads, S = C + E slots of which C + E/2 are valid (the mean
    over an eviction cycle).  The launches cycle over ``layers`` separate caches (more
    bytes than L2 holds), as the decode step does."""
    import torch

    from kvcacheboundaryprotection_b200.capi import check, lib
    from kvcacheboundaryprotection_b200.config import get_config

    L = lib()
    cfg = get_config(preset)
    dev = torch.device("cuda")
    hbm, _, peak_kind = peaks()
    Hq, Hkv, D, S = cfg.n_heads, cfg.n_kv_heads, cfg.head_dim, C + E
    g = torch.Generator(device=dev).manual_seed(0)
    kcs = [torch.randn(B, Hkv, S, D, generator=g, device=dev).to(torch.bfloat16) for _ in range(layers)]
    vcs = [torch.randn(B, Hkv, S, D, generator=g, device=dev).to(torch.bfloat16) for _ in range(layers)]
    valid = C + E // 2
    slot_pos = torch.arange(S, dtype=torch.int32, device=dev).repeat(B, 1)
    slot_pos[:, valid:] = -1
    q = (torch.randn(B, Hq, D, generator=g, device=dev) / math.sqrt(D)).to(torch.bfloat16)
    out = torch.empty_like(q)
    score = torch.zeros(B, S, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)

    def launch(li):
        check(L.kvbp_decode_attn_score(torch.cuda.current_stream().cuda_stream, B, Hq, Hkv, D, S, q.data_ptr(),
                                       kcs[li].data_ptr(), vcs[li].data_ptr(), slot_pos.data_ptr(), None,
                                       out.data_ptr(), score.data_ptr(), err.data_ptr()), "decode_attn_score")

    for li in range(layers):
        launch(li)
    torch.cuda.synchronize()
    # eager: events around each launch (includes the front-end gap of an isolated launch)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(iters * layers)]
    for it in range(iters):
        for li in range(layers):
            a, b = ev[it * layers + li]
            a.record()
            launch(li)
            b.record()
    torch.cuda.synchronize()
    eager_us = statistics.median([a.elapsed_time(b) * 1000 for a, b in ev])
    # burst: the ``layers`` launches back to back in a CUDA graph, as in the decode step
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(side):
        with torch.cuda.graph(graph, stream=side):
            for li in range(layers):
                launch(li)
    torch.cuda.current_stream().wait_stream(side)
    graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        graph.replay()
    e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1000 / (iters * layers)
    del graph
    if int(err.item()):
        raise RuntimeError("device error in attention microbench")
    byts = algorithmic_attn_bytes(B, Hq, Hkv, valid)
    return {"preset": preset, "batch": B, "capacity": C, "slots": S, "valid_slots": valid, "us": round(us, 2),
            "timing": "burst: the launches over the layers' caches back to back in a CUDA graph",
            "eager_us": round(eager_us, 2), "algorithmic_bytes": byts, "gbs": round(byts / us / 1e3, 1), "frac": round(byts / us / 1e3 / hbm, 4),
            "peak_gbs": hbm, "peak_kind": peak_kind}


def planted_prompt(vocab: int, P: int, seed: int = 0, span: int = 16):
    """Uniform-random token ids with one key span: tokens [r, r + span) copied to the last
    ``span`` positions (r uniform), the synthetic stand-in for a needle-in-a-haystack prompt."""
    rng = np.random.default_rng(seed)
    ids = rng.integers(0, vocab, P)
    r = int(rng.integers(0, P - 2 * span))
    ids[P - span:] = ids[r : r + span]
    return ids


def run_prefill_e2e(workload="qwen2.5-7b", batch=1):
    """Step 0 of the workload end to end through CappedKVEngine.prefill: prompt forward
    (cuBLAS projections, tcgen05 causal attention with the per-key score), the forced
    eviction down to the capacity, compaction into the slot cache and the first greedy
    token, for ``batch`` prompts with a planted key span.  Reported apart from the decode
    metric (which excludes prefill, as the reference's decode_step_* fields do)."""
    import torch

    from kvcacheboundaryprotection_b200.config import get_config
    from kvcacheboundaryprotection_b200.engine import CappedKVEngine, EvictionSpec, FusedWeights
    from kvcacheboundaryprotection_b200.weights import init_weights

    preset, _, C, P, policy, _ = WORKLOADS[workload]
    cfg = get_config(preset)
    dev = torch.device("cuda")
    fw = FusedWeights(cfg, init_weights(cfg, seed=0, device=dev), dev)
    eng = CappedKVEngine(cfg, fw, batch=batch, evict=EvictionSpec(policy, C, 8, True, 0.10, 0.10), max_prompt_len=P,
                         max_new_tokens=8, device=dev)
    ids = torch.tensor(np.stack([planted_prompt(cfg.vocab, P, seed=b) for b in range(batch)]), dtype=torch.int32)
    eng.prefill(ids)  # warm-up of the same shapes
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.perf_counter()
    e0.record()
    eng.prefill(ids)
    e1.record()
    torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    ms = e0.elapsed_time(e1)
    eng.check_device_errors()
    out = {"workload": f"{preset}, {batch} x {P}-token prompt with a planted 16-token key span, capacity {C}, {policy}",
           "ms": round(ms, 1), "wall_ms": round(wall * 1000, 1), "prefill_tok_s": round(batch * P / (ms / 1000), 1),
           "retained_after_step0": int((eng.slot_pos[0] >= 0).sum().item()),
           "how": "CUDA events around CappedKVEngine.prefill (after one warm-up prefill of the same shapes)"}
    del eng, fw
    torch.cuda.empty_cache()
    return out


def run_prefill_microbench(preset="qwen2.5-7b", P=8192, iters=3):
    """Operator microbench of kvbp_prefill_attn_score (tcgen05 causal prefill attention
    with the per-key score) for one layer of one sequence at the preset's heads.
    Algorithmic FLOPs = 4 * (P^2 / 2) * 128 * Hq (Q.K^T and P.V over the causal half);
    the kernel executes twice that on the tensor cores (Q.K^T in both passes, P.V as bf16
    hi + lo parts)."""
    import torch

    from kvcacheboundaryprotection_b200.capi import check, lib
    from kvcacheboundaryprotection_b200.config import get_config

    L = lib()
    cfg = get_config(preset)
    dev = torch.device("cuda")
    _, tf, peak_kind = peaks()
    Hq, Hkv, D = cfg.n_heads, cfg.n_kv_heads, cfg.head_dim
    g = torch.Generator(device=dev).manual_seed(0)
    q = torch.randn(P, Hq, D, generator=g, device=dev).to(torch.bfloat16)
    k = torch.randn(Hkv, P, D, generator=g, device=dev).to(torch.bfloat16)
    v = torch.randn(Hkv, P, D, generator=g, device=dev).to(torch.bfloat16)
    out = torch.empty(P, Hq, D, dtype=torch.bfloat16, device=dev)
    colmax = torch.zeros(P, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)

    def run():
        check(L.kvbp_prefill_attn_score(torch.cuda.current_stream().cuda_stream, P, Hq, Hkv, D, q.data_ptr(),
                                        k.data_ptr(), v.data_ptr(), out.data_ptr(), colmax.data_ptr(),
                                        err.data_ptr()), "prefill_attn_score")

    run()
    torch.cuda.synchronize()
    ts = []
    for _ in range(iters):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        run()
        e1.record()
        torch.cuda.synchronize()
        ts.append(e0.elapsed_time(e1))
    if int(err.item()):
        raise RuntimeError("device error in prefill microbench")
    ms = statistics.median(ts)
    alg = 4.0 * (P * P / 2.0) * D * Hq
    return {"preset": preset, "prompt": P, "heads": [Hq, Hkv], "ms": round(ms, 3),
            "algorithmic_tflops": round(alg / (ms * 1e-3) / 1e12, 1),
            "tensor_tflops_executed": round(2 * alg / (ms * 1e-3) / 1e12, 1),
            "peak_tflops": tf, "peak_kind": f"{peak_kind} dense bf16 (cuBLAS)",
            "frac_executed": round(2 * alg / (ms * 1e-3) / 1e12 / tf, 4)}


def run_prefill_gemm_microbench(preset="qwen2.5-7b", R=16384, iters=5):
    """Operator microbench of kvbp_prefill_gemm (tcgen05) on one decoder layer's prefill
    projections of ``preset`` over R prompt rows: q/k/v, o, gate/up (SwiGLU epilogue) and
    down, each as 3 warm-up + ``iters`` timed launches (CUDA events, median), then the same
    product through torch.mm (cuBLAS, row-major weights, plain output) for context.  The
    launch order is fixed (per shape: own launches, then cuBLAS), so an ncu capture can
    select a shape by its launch index."""
    import torch

    from kvcacheboundaryprotection_b200 import capi
    from kvcacheboundaryprotection_b200.config import get_config
    from kvcacheboundaryprotection_b200.engine import pack_weight

    L = capi.lib()
    cfg = get_config(preset)
    dev = torch.device("cuda")
    _, bf16_peak, _ = peaks()
    H, F = cfg.hidden, cfg.ffn
    qkv_n = (cfg.n_heads + 2 * cfg.n_kv_heads) * cfg.head_dim
    shapes = (("qkv", qkv_n, H, 0), ("o", H, cfg.n_heads * cfg.head_dim, 0), ("gate_up", 2 * F, H, 2), ("down", H, F, 0))
    g = torch.Generator(device=dev).manual_seed(0)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    rows = []
    for name, N, K, epi in shapes:
        x = torch.randn(R, K, generator=g, device=dev).to(torch.bfloat16)
        w = (torch.randn(N, K, generator=g, device=dev) * 0.02).to(torch.bfloat16)
        wp = pack_weight(w)
        oc = N // 2 if epi == 2 else N
        out = torch.empty(R, oc, dtype=torch.bfloat16, device=dev)
        ref = torch.empty(R, N, dtype=torch.bfloat16, device=dev)

        def own():
            capi.check(L.kvbp_prefill_gemm(torch.cuda.current_stream().cuda_stream, epi, R, N, K, wp.data_ptr(),
                                           x.data_ptr(), K, out.data_ptr(), oc, err.data_ptr()), "prefill_gemm")

        def cublas():
            torch.mm(x, w.t(), out=ref)

        row = {"shape": name, "N": N, "K": K, "epilogue": "swiglu" if epi == 2 else "plain"}
        for tag, fn in (("own", own), ("cublas", cublas)):
            for _ in range(3):
                fn()
            torch.cuda.synchronize()
            ts = []
            for _ in range(iters):
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                fn()
                e1.record()
                torch.cuda.synchronize()
                ts.append(e0.elapsed_time(e1) * 1000)
            us = sorted(ts)[len(ts) // 2]
            tf = 2 * R * N * K / us / 1e6
            row[tag] = {"us": round(us, 1), "tflops": round(tf, 1), "frac": round(tf / bf16_peak, 4)}
        if int(err.item()):
            raise RuntimeError("device error in prefill GEMM microbench: " + str(capi.decode_dev_errors(int(err.item()))))
        rows.append(row)
        del x, w, wp, out, ref
    return {"rows_R": R, "peak_tflops": bf16_peak, "rows": rows}


def run_gemm_microbench(preset="qwen2.5-7b", M=16, iters=10, sweep=False):
    """Operator microbench of kvbp_decode_gemm on one decoder layer's projections (and the
    lm_head) of ``preset``: M activation rows against bf16 weights streamed from HBM, each
    with the epilogue and norm prologue the decode step uses and the engine's split-K
    choice (``sweep``: also other split counts).  A 512 MB read flushes L2 before every
    timed launch; the same shapes through torch.mm (cuBLAS, plain output, row-major
    weights) are timed beside it for context."""
    import torch

    from kvcacheboundaryprotection_b200.capi import check, lib
    from kvcacheboundaryprotection_b200.config import get_config
    from kvcacheboundaryprotection_b200.engine import CappedKVEngine, pack_weight

    L = lib()
    cfg = get_config(preset)
    dev = torch.device("cuda")
    hbm, _, peak_kind = peaks()
    H, F, V = cfg.hidden, cfg.ffn, cfg.vocab
    qkv_n = (cfg.n_heads + 2 * cfg.n_kv_heads) * cfg.head_dim
    shapes = (  # name, N, K, epilogue (0 plain, 1 residual, 2 SwiGLU), norm prologue
        ("qkv", qkv_n, H, 0, True),
        ("o", H, cfg.n_heads * cfg.head_dim, 1, False),
        ("gate_up", 2 * F, H, 2, True),
        ("down", H, F, 1, False),
        ("lm_head", V, H, 0, True),
    )
    flush = torch.empty(512 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)
    g = torch.Generator(device=dev).manual_seed(0)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    rows = []
    for name, N, K, epi, norm in shapes:
        W = (torch.randn(N, K, generator=g, device=dev) * 0.02).to(torch.bfloat16)
        Wp = pack_weight(W)
        x = torch.randn(M, K, generator=g, device=dev).to(torch.bfloat16)
        out = torch.zeros(M, N // 2 if epi == 2 else N, dtype=torch.bfloat16, device=dev)
        nw = torch.ones(K, dtype=torch.bfloat16, device=dev)
        ss_parts = torch.ones(1, 32, device=dev)
        ss_out = torch.zeros(N // 128, 32, device=dev)
        pick = CappedKVEngine._pick_splits(N, K)
        cands = [pick]
        if sweep:
            cands += [sp for sp in (1, 2, 3, 4, 5, 6, 7, 8, 10, 12, 16) if sp != pick and sp <= K // 128]

        def timed(fn):
            fn()
            ts = []
            for it in range(iters):
                flush.sum()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                fn()
                e1.record()
                torch.cuda.synchronize()
                ts.append(e0.elapsed_time(e1) * 1000)
            return statistics.median(ts)

        byts = N * K * 2 + M * K * 2 + out.numel() * 2 * (2 if epi == 1 else 1)
        cub = timed(lambda: torch.mm(x, W.t()))
        for sp in cands:
            def ours(sp=sp):
                s = torch.cuda.current_stream().cuda_stream
                check(L.kvbp_decode_gemm(s, epi, M, N, K, Wp.data_ptr(), x.data_ptr(), K,
                                         ss_parts.data_ptr() if norm else None, 1, nw.data_ptr() if norm else None,
                                         1e-6, out.data_ptr(), out.shape[1], ss_out.data_ptr() if epi == 1 else None,
                                         sp, err.data_ptr()), "decode_gemm")

            us = timed(ours)
            rows.append({"gemm": name, "N": N, "K": K, "splits": sp, "us": round(us, 2),
                         "gbs": round(byts / us / 1e3, 1), "frac": round(byts / us / 1e3 / hbm, 4),
                         "cublas_us": round(cub, 2)})
        del W, Wp
    torch.cuda.synchronize()
    if int(err.item()):
        raise RuntimeError("device error in GEMM microbench")
    return {"peak_gbs": hbm, "peak_kind": peak_kind, "rows_M": M, "preset": preset, "rows": rows}


def micro_bytes(B, Hq, Hkv, valid, E):
    """Algorithmic bytes of one fused step: attention bytes + new K/V write + metadata
    (step score, attn, max, cumul f64, last, count: read+write per valid slot) +
    selection reads on cadence steps amortised over E steps."""
    attn = algorithmic_attn_bytes(B, Hq, Hkv, valid)
    kvw = 2 * B * Hkv * 128 * 2
    meta = B * valid * (4 + 4 + 4 + 8 + 4 + 4 + 4) * 2
    sel = B * valid * (4 + 4 + 4 + 8) / E
    return attn + kvw + meta + sel


def _micro_state(B, S, C, P0, dev, g):
    import torch

    from kvcacheboundaryprotection_b200 import capi

    i32 = torch.int32
    pos = torch.stack([torch.sort(torch.randperm(P0, generator=g, device=dev)[:C]).values for _ in range(B)]).to(i32)
    slot_pos = torch.full((B, S), -1, dtype=i32, device=dev)
    slot_pos[:, :C] = pos
    step0 = 64
    W = (P0 + 4096 + 31) // 32
    posmap = torch.zeros(B, W, dtype=torch.int64, device=dev)
    # bit set for each retained position
    words = (pos // 32).long()
    bits = torch.ones_like(words) << (pos % 32).long()
    posmap.scatter_add_(1, words, bits)
    posmap = posmap.to(torch.int64).bitwise_and(0xFFFFFFFF)
    posmap = torch.where(posmap >= 2**31, posmap - 2**32, posmap).to(i32)
    st = {
        "slot_pos": slot_pos,
        "ins": torch.zeros(B, S, dtype=i32, device=dev),
        "last": torch.randint(0, step0, (B, S), generator=g, device=dev, dtype=i32),
        "cnt": torch.ones(B, S, dtype=i32, device=dev),
        "attn": torch.rand(B, S, generator=g, device=dev),
        "maxa": torch.rand(B, S, generator=g, device=dev),
        "cumul": torch.rand(B, S, generator=g, device=dev, dtype=torch.float64) * 4,
        "pre": torch.rand(B, S, generator=g, device=dev),
        "posmap": posmap.contiguous(),
        "step_score": torch.zeros(B, S, device=dev),
        "seq_step": torch.full((B,), step0, dtype=i32, device=dev),
        "next_pos": torch.full((B,), P0, dtype=i32, device=dev),
        "cur_pos": torch.zeros(B, dtype=i32, device=dev),
        "write_slot": torch.zeros(B, dtype=i32, device=dev),
        "evcap": 1 << 16,
    }
    st["evlog"] = torch.zeros(B, st["evcap"], dtype=i32, device=dev)
    st["evcount"] = torch.zeros(B, dtype=i32, device=dev)
    st["state"] = capi.State(
        B, S, W, *[st[k].data_ptr() for k in ("slot_pos", "ins", "last", "cnt", "attn", "maxa", "cumul", "pre", "posmap")]
    )
    return st


# ------------------------------------------------------------------------ CPU reference / baseline
def cpu_threads() -> int:
    """Sets numpy's BLAS pool to every host core, whatever OMP_NUM_THREADS torchrun put in
    the environment, and returns the thread count the pool actually has."""
    n = os.cpu_count() or 1
    try:
        import threadpoolctl

        threadpoolctl.threadpool_limits(limits=n, user_api="blas")
        info = [p for p in threadpoolctl.threadpool_info() if p.get("user_api") == "blas"]
        if info:
            return int(info[0]["num_threads"])
    except Exception:  # noqa: BLE001 - no controllable BLAS pool: report one thread
        return 1
    return n


def cpu_reference_step_times(workload, steps, warmup, budget_s=90.0):
    """Time the oracle port of the reference's decode step on the host cores.

    The reference decodes one sequence at a time (batch 1): a sequence's decode step is a
    forward of one token through every layer with attention over the retained positions,
    the full lm_head, then the per-step eviction bookkeeping (score update; the policy
    call every 8 steps over the retained positions).  Whole steps are timed at the
    workload's real shapes.  One layer's weights are drawn and used for all the layers
    (a full fp32 weight set would need ~4x the bf16 model in host memory; every layer
    still streams its ~1 GB of fp32 weights from DRAM, more than any CPU cache).  Stops
    after ``budget_s`` seconds of timed steps (at least 2).  Returns (per-step seconds,
    sample description, BLAS threads)."""
    import oracle.model as om
    from oracle.bf16 import rnd
    from oracle.policies import Meta, PolicySpec
    from kvcacheboundaryprotection_b200.config import get_config

    threads = cpu_threads()
    preset, _, C, P, policy, _ = WORKLOADS[workload]
    cfg = get_config(preset)
    rng = np.random.default_rng(0)
    H, D, F = cfg.hidden, cfg.head_dim, cfg.ffn

    def w(*shape):
        return rnd(rng.standard_normal(shape, dtype=np.float32) * np.float32(0.02))

    weights = {
        "l0.in_norm": np.ones(H, np.float32), "l0.post_norm": np.ones(H, np.float32),
        "l0.wq": w(cfg.n_heads * D, H), "l0.wk": w(cfg.n_kv_heads * D, H), "l0.wv": w(cfg.n_kv_heads * D, H),
        "l0.wo": w(H, cfg.n_heads * D), "l0.w_gate": w(F, H), "l0.w_up": w(F, H), "l0.w_down": w(H, F),
        "final_norm": np.ones(H, np.float32),
        "lm_head": w(cfg.vocab, H),
    }
    if cfg.qkv_bias:
        weights.update({"l0.bq": w(cfg.n_heads * D), "l0.bk": w(cfg.n_kv_heads * D), "l0.bv": w(cfg.n_kv_heads * D)})
    if cfg.qk_norm:
        weights.update({"l0.q_norm": np.ones(D, np.float32), "l0.k_norm": np.ones(D, np.float32)})
    ocfg = om.OracleConfig(vocab=cfg.vocab, hidden=H, n_layers=1, n_heads=cfg.n_heads, n_kv_heads=cfg.n_kv_heads,
                           head_dim=D, ffn=F, rope_theta=cfg.rope_theta, eps=cfg.eps, qkv_bias=cfg.qkv_bias,
                           qk_norm=cfg.qk_norm, tie_embed=False)
    model = om.OracleModel(ocfg, weights, max_cache_len=C + 16)
    # every layer's cache: C retained positions + the new one (visibility = retained slots)
    ck = [rnd(rng.standard_normal((cfg.n_kv_heads, C + 16, D), dtype=np.float32)) for _ in range(cfg.n_layers)]
    cv = [rnd(rng.standard_normal((cfg.n_kv_heads, C + 16, D), dtype=np.float32)) for _ in range(cfg.n_layers)]
    h0 = rnd(rng.standard_normal((1, H), dtype=np.float32))
    spec = PolicySpec(policy, C, True, 0.10, 0.10)
    meta = Meta.zeros(P + 4096)
    meta.cumul[:] = rng.random(P + 4096)
    live = sorted(rng.choice(P, C, replace=False).tolist())

    def allow(n, nh, ncols):
        return np.ones((1, nh, ncols), bool)

    times = []
    t_start = None
    for it in range(warmup + steps):
        t0 = time.perf_counter()
        pos = np.array([C], np.int64)  # the new token attends over C + 1 positions
        hh = h0
        ks = None
        for li in range(cfg.n_layers):
            hh, probs = model._layer(0, hh, pos, ck[li], cv[li], allow)
            pk = probs.max(axis=(0, 1))
            ks = pk if ks is None else np.maximum(ks, pk)  # per-slot score: max over heads, layers
        _ = model._logits(hh)
        ks = ks.astype(np.float32)
        n = len(ks)
        thr = np.float32(0.05 * float(ks.max()))
        meta.cumul[:n] += ks
        hit = ks > thr
        meta.last_access[:n] = np.where(hit, np.int32(it), meta.last_access[:n])
        if it % 8 == 0:
            spec.select(live + [P + it], meta, 8, it + 1)
        dt = time.perf_counter() - t0
        if it >= warmup:
            times.append(dt)
            t_start = t_start or t0
            if len(times) >= 2 and time.perf_counter() - t_start > budget_s:
                break
    sample = (
        f"{len(times)} whole batch-1 decode steps of {preset} at capacity {C} ({cfg.n_layers} layers, full "
        f"{cfg.vocab}-row lm_head, eviction bookkeeping; one layer's weights reused by every layer); numpy "
        f"float32 (bf16-rounded) oracle port, {threads} BLAS threads"
    )
    return times, sample, threads


def run_reference(a, rank):
    if rank != 0:
        return None
    times, sample, threads = cpu_reference_step_times(a.workload, a.steps, a.warmup)
    tok_s = 1.0 / (sum(times) / len(times))
    preset, B0, C, P, policy, par = WORKLOADS[a.workload]
    tp = a.gpus > 1 and (par if a.parallel == "auto" else a.parallel) == "tp"
    return {
        "impl": "reference",
        "metric": METRIC,
        "value": round(tok_s, 4),
        "unit": "tok/s",
        "n_gpus": a.gpus,
        "steps": len(times),
        "warmup": a.warmup,
        "ms_per_step": round(1000 * sum(times) / len(times), 3),
        "higher_is_better": True,
        "scaling": "strong" if tp else "weak",
        "vs_baseline": None,
        "dtype": "f32 (bf16-rounded values)",
        "data": "synthetic",
        "config": {"workload": f"{preset} decode, capacity {C}, {policy}, batch 1 (the reference decodes one "
                   f"sequence per generate call: tok/s of many sequences is the same)", "capacity": C},
        "cpu_baseline": {"value": round(tok_s, 4), "unit": "tok/s", "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": round(tok_s, 4), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


# ------------------------------------------------------------------------ main
def main():
    a = parse()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if a.impl == "reference":
        out = run_reference(a, rank)
        if out is not None:
            print(json.dumps(out), flush=True)
        return
    import torch
    import torch.distributed as dist

    if a.micro_only is not None:
        from kvcacheboundaryprotection_b200 import build as kbuild

        kbuild.build()
        print(json.dumps(run_microbench(cap_list=(a.micro_only,), policies=("lru",), fracs=(0.10,), iters=16)), flush=True)
        return
    if a.micro_attn:
        from kvcacheboundaryprotection_b200 import build as kbuild

        kbuild.build()
        preset, B0, C0 = WORKLOADS[a.workload][:3]
        print(json.dumps(run_attn_microbench(preset, a.batch or B0, C0)), flush=True)
        return
    if a.micro_prefill is not None:
        from kvcacheboundaryprotection_b200 import build as kbuild

        kbuild.build()
        print(json.dumps(run_prefill_microbench(WORKLOADS[a.workload][0], a.micro_prefill)), flush=True)
        return
    if a.micro_prefill_gemm is not None:
        from kvcacheboundaryprotection_b200 import build as kbuild

        kbuild.build()
        print(json.dumps(run_prefill_gemm_microbench(WORKLOADS[a.workload][0], a.micro_prefill_gemm)), flush=True)
        return
    if a.micro_gemm:
        from kvcacheboundaryprotection_b200 import build as kbuild

        kbuild.build()
        print(json.dumps(run_gemm_microbench(WORKLOADS[a.workload][0], sweep=True)), flush=True)
        return
    if world > 1:
        torch.cuda.set_device(local_rank)
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local_rank))
    from kvcacheboundaryprotection_b200 import build as kbuild

    kbuild.build()
    torch.cuda.set_device(local_rank)
    par = WORKLOADS[a.workload][5] if a.parallel == "auto" else a.parallel
    out, eng, fw = decode_run(a, a.workload, par, rank, world, local_rank, steps=a.steps, warmup=a.warmup)
    if world > 1 and par == "tp" and not a.no_check:
        eng.graph = None
        out["tp_check"] = tp_check(a, a.workload, rank, world, local_rank, eng)
    eng.graph = None  # a graph holding NCCL calls goes before the process group
    del eng, fw
    torch.cuda.empty_cache()
    side_k, side_w = min(a.steps, 20), min(a.warmup, 3)
    if world > 1 and a.parallel == "auto" and a.workload in ALSO_DP:
        r, e, f = decode_run(a, a.workload, "dp", rank, world, local_rank, steps=side_k, warmup=side_w, full=False)
        e.graph = None
        del e, f
        torch.cuda.empty_cache()
        out["data_parallel"] = {k: r[k] for k in ("value", "unit", "ms_per_step", "scaling", "config", "roofline",
                                                  "step_roofline")}
    if not a.no_configs and a.workload == "qwen2.5-7b" and a.batch is None:
        out["configs"] = {}
        for w in OTHER_CONFIGS:
            wpar = WORKLOADS[w][5]
            r, e, f = decode_run(a, w, wpar, rank, world, local_rank, steps=side_k, warmup=side_w, full=False)
            entry = {k: r[k] for k in ("value", "unit", "ms_per_step", "scaling", "config", "roofline",
                                       "roofline_attention", "step_roofline", "kernels")}
            if world > 1 and wpar == "tp" and not a.no_check:
                e.graph = None
                entry["tp_check"] = tp_check(a, w, rank, world, local_rank, e)
            e.graph = None
            del e, f
            torch.cuda.empty_cache()
            out["configs"][w] = entry
    fw = None
    if rank == 0 and world == 1:
        if not a.no_micro:
            out["kernel_microbench"] = run_microbench()
            out["gemm_microbench"] = run_gemm_microbench(WORKLOADS[a.workload][0])
            preset, B0, C0 = WORKLOADS[a.workload][:3]
            out["attn_microbench"] = run_attn_microbench(preset, a.batch or B0, C0)
            out["prefill_microbench"] = run_prefill_microbench(preset, 8192)
            out["prefill_e2e"] = run_prefill_e2e(a.workload)
        if not a.no_cpu:
            times, sample, threads = cpu_reference_step_times(a.workload, 3, 1, budget_s=20.0)
            v = 1.0 / (sum(times) / len(times))
            out["cpu_baseline"] = {"value": round(v, 4), "unit": "tok/s", "cores": threads, "kind": "port", "sample": sample}
    if rank == 0:
        print(json.dumps(out), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
