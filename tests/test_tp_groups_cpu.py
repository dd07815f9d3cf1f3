"""Tensor-parallel groups inside a larger job, with world-size-4 gloo ranks on CPU (no GPU).

bench.tp_layout picks the tensor-parallel size (the reference's clamp, or --tp-size) and
splits the ranks into data-parallel replicas of the group; each replica's collectives
must reach its own ranks only, and sizes that do not split the sequences fall back to one
group of every rank."""

import os
import socket
from types import SimpleNamespace

import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    import bench
    from kvcacheboundaryprotection_b200.config import get_config

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        q7 = get_config("qwen2.5-7b")
        out = {}
        # default: the reference clamp keeps TP = 4 on 4 ranks (4 KV heads): one group
        t, dp, g, trank, group, granks = bench.tp_layout(SimpleNamespace(tp_size=None), q7, world, rank, 16)
        out["default"] = (t, dp, g, trank, group is None, granks)
        # --tp-size 2: two replicas of a 2-rank group, 8 sequences each
        t, dp, g, trank, group, granks = bench.tp_layout(SimpleNamespace(tp_size=2), q7, world, rank, 16)
        x = torch.tensor([float(rank + 1)])
        dist.all_reduce(x, group=group)  # sums over the rank's own group only
        out["tp2"] = (t, dp, g, trank, tuple(granks), float(x))
        # 3 sequences do not split over 2 replicas: one group of every rank
        t, dp, g, trank, group, granks = bench.tp_layout(SimpleNamespace(tp_size=2), q7, world, rank, 3)
        out["fallback"] = (t, dp, g, trank, group is None)
        q.put((rank, out))
    finally:
        dist.destroy_process_group()


def test_tp_replica_groups_on_four_gloo_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    world = 4
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r in range(world):
        o = got[r]
        assert o["default"] == (4, 1, 0, r, True, None)
        g = r // 2
        members = (2 * g, 2 * g + 1)
        assert o["tp2"] == (2, 2, g, r % 2, members, float(sum(m + 1 for m in members)))
        assert o["fallback"] == (4, 1, 0, r, True)
