"""One rank of a tensor-parallel decode, one process per GPU (launched under torchrun by
test_gpu_tp_multiproc.py).  Run A decodes greedily with the NCCL allreduce of the
o/down partial sums; run B replays A's tokens (teacher forcing) from a captured CUDA
graph with the allreduce fused into the GEMMs over NVLink.  Rank 0 writes the per-step
logit differences, token agreement and eviction logs to the JSON file in argv[1]."""

import json
import os
import sys
from datetime import timedelta

import numpy as np
import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from kvcacheboundaryprotection_b200 import capi  # noqa: E402
from kvcacheboundaryprotection_b200.config import get_config  # noqa: E402
from kvcacheboundaryprotection_b200.engine import EvictionSpec  # noqa: E402
from kvcacheboundaryprotection_b200.tp import TPEngine, tp_plan  # noqa: E402
from kvcacheboundaryprotection_b200.weights import init_weights  # noqa: E402


def gathered_logits(eng, world):
    # vocabulary shards may differ in size by one 128-block: pad to the largest
    V = eng.full_cfg.vocab
    lens = [tp_plan(eng.full_cfg, world, r).vocab_hi - tp_plan(eng.full_cfg, world, r).vocab_lo for r in range(world)]
    m = max(lens)
    pad = torch.zeros(eng.B, m, dtype=eng.logits.dtype, device=eng.dev)
    pad[:, : eng.logits.shape[1]] = eng.logits
    parts = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(parts, pad)
    full = torch.cat([p[:, :n] for p, n in zip(parts, lens)], 1)
    assert full.shape[1] == V
    return full.float().cpu().numpy()


def main():
    out_path = sys.argv[1]
    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=timedelta(seconds=60), device_id=dev)
    capi.lib()
    cfg = get_config("parity-qwen2")
    w = init_weights(cfg, seed=0, device=dev)
    B, P, cap, max_new = 2, 200, 48, 24
    rng = np.random.default_rng(7)
    ids = torch.tensor(rng.integers(0, cfg.vocab, (B, P)), dtype=torch.int32)
    spec = EvictionSpec("lru", cap, 8, True, 0.10, 0.10)
    plan = tp_plan(cfg, world, rank)

    # run A: NCCL allreduces, eager, greedy
    a = TPEngine(cfg, w, plan=plan, batch=B, evict=spec, max_prompt_len=P, max_new_tokens=max_new, device=dev)
    a.prefill(ids)
    toks_in, logits_a, toks_a = [], [], []
    for s in range(1, max_new):
        toks_in.append(a.tokens.clone())
        a.decode_step_launches()
        a.step += 1
        logits_a.append(gathered_logits(a, world))
        toks_a.append(a.tokens.cpu().numpy().tolist())
    torch.cuda.synchronize()
    a.check_device_errors()

    # run B: fused NVLink allreduce, CUDA graph, A's input tokens
    b = TPEngine(cfg, w, plan=plan, fused_allreduce=True, batch=B, evict=spec, max_prompt_len=P,
                 max_new_tokens=max_new, device=dev)
    b.prefill(ids)
    b.capture()
    diffs, agree, decisive = [], 0, 0
    for s in range(1, max_new):
        b.tokens.copy_(toks_in[s - 1])
        b.run_step()
        lb = gathered_logits(b, world)
        la = logits_a[s - 1]
        diffs.append(float(np.abs(lb - la).max()))
        for r in range(B):
            top2 = np.sort(la[r])[-2:]
            if top2[1] - top2[0] > 2e-2:
                decisive += 1
                agree += int(int(b.tokens[r].item()) == toks_a[s - 1][r])
    torch.cuda.synchronize()
    b.check_device_errors()
    # every rank holds the same tokens and eviction state
    same = torch.tensor([int(torch.equal(b.slot_pos, a.slot_pos)), 1], device=dev)
    tok = b.tokens.clone()
    all_tok = [torch.empty_like(tok) for _ in range(world)]
    dist.all_gather(all_tok, tok)
    same[1] = int(all(torch.equal(t, tok) for t in all_tok))
    dist.all_reduce(same, op=dist.ReduceOp.MIN)
    if rank == 0:
        n = [int(x) for x in a.evcount.tolist()]
        res = {
            "world": world,
            "max_logit_diff": max(diffs),
            "argmax_agree": agree,
            "argmax_decisive": decisive,
            "slot_tables_equal": bool(same[0].item()),
            "tokens_equal_across_ranks": bool(same[1].item()),
            "evlog_a": [a.evlog[i, : n[i]].tolist() for i in range(B)],
            "evlog_b": [b.evlog[i, : int(b.evcount[i].item())].tolist() for i in range(B)],
        }
        with open(out_path, "w") as f:
            json.dump(res, f)
    del b.graph
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
