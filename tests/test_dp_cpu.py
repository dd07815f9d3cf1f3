"""Data-parallel host logic with world-size-2 gloo ranks on CPU (no GPU).

Each rank decodes its contiguous shard of sequences with the oracle loop + stub score
model; the gathered results must equal a single-process run over all sequences."""

import os
import socket

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from kvcacheboundaryprotection_b200.parallel import max_over_ranks, run_data_parallel, shard_range


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _prompts():
    import numpy as np

    rng = np.random.default_rng(5)
    return [[int(x) for x in rng.integers(0, 97, 120)] for _ in range(5)]


def _gen(prompts):
    from oracle.generator import generate
    from oracle.policies import PolicySpec
    from oracle.stub_model import StubScoreModel

    out = []
    for p in prompts:
        m = StubScoreModel(vocab=97, n_heads=4, n_kv_heads=2, n_layers=2, max_cache_len=200, seed=sum(p) % 1000)
        r = generate(m, PolicySpec("h2o_faithful", 40, True), p, 24, n_kv_heads=2)
        out.append((r.generated_token_ids, r.positions_evicted, r.retained_counts_by_step))
    return out


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        res = run_data_parallel(_gen, _prompts())
        t = max_over_ranks(float(rank + 1))
        if rank == 0:
            q.put((res, t))
    finally:
        dist.destroy_process_group()


def test_shard_range_covers_everything():
    for n in (0, 1, 5, 16, 17):
        for w in (1, 2, 3, 8):
            got = [shard_range(n, r, w) for r in range(w)]
            assert got[0][0] == 0 and got[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(got, got[1:]))
            assert max(h - l for l, h in got) - min(h - l for l, h in got) <= 1
    with pytest.raises(ValueError):
        shard_range(4, 2, 2)


def test_two_gloo_ranks_match_single_process():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res, t = q.get(timeout=300)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert t == 2.0
    assert [tuple(map(tuple, r)) for r in res] == [tuple(map(tuple, r)) for r in _gen(_prompts())]
