"""Tensor parallelism over KV-head groups, emulated on one GPU: the ranks of a process
group run in lockstep in one process (``tp.run_lockstep``), each with its own shards,
caches and metadata, and their reductions are done in rank order.  Compared with the
oracle on the same teacher-forced tokens and with the same tolerances as the single-GPU
parity tests (test_gpu_e2e.py); in addition every rank must hold bit-identical slot
tables, eviction metadata, residual stream and tokens (they decide evictions
independently and must agree without a broadcast)."""

import numpy as np
import pytest
import torch

from kvcacheboundaryprotection_b200 import build, capi
from kvcacheboundaryprotection_b200.config import get_config
from kvcacheboundaryprotection_b200.engine import EvictionSpec
from kvcacheboundaryprotection_b200.tp import TPEngine, run_lockstep, tp_plan
from kvcacheboundaryprotection_b200.weights import init_weights
from oracle.generator import generate
from oracle.model import OracleModel
from oracle.policies import PolicySpec

from test_gpu_e2e import _ocfg

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _lib():
    build.build()


def _same_on_all_ranks(engs, name):
    ref = getattr(engs[0], name)
    for e in engs[1:]:
        assert torch.equal(getattr(e, name), ref), f"{name} differs across ranks"


def _run_forced_tp(preset, policy, world, P=300, cap=64, N=512, max_new=40, seed=0):
    cfg = get_config(preset)
    w = init_weights(cfg, seed=0)
    wn = {k: v.float().numpy() for k, v in w.items()}
    prompt = [int(x) for x in np.random.default_rng(seed).integers(0, cfg.vocab, P)]
    o = generate(OracleModel(_ocfg(cfg), wn, max_cache_len=N), PolicySpec(policy, cap, True, 0.10, 0.10), prompt,
                 max_new, evict_every=8, n_kv_heads=cfg.n_kv_heads, record_logits=True)
    forced = o.generated_token_ids[P:]
    wd = {k: v.cuda() for k, v in w.items()}
    spec = EvictionSpec(policy, cap, 8, True, 0.10, 0.10)
    engs = [TPEngine(cfg, wd, plan=tp_plan(cfg, world, r), batch=1, evict=spec, max_prompt_len=P,
                     max_new_tokens=max_new) for r in range(world)]
    run_lockstep([e.prefill_phases(torch.tensor([prompt], dtype=torch.int32)) for e in engs])
    torch.cuda.synchronize()
    L = capi.lib()
    stats = {"logit_diff": [], "argmax_ok": 0, "argmax_n": 0, "score_rel": [], "score_ok": []}

    def cmp_logits(step_idx):
        got = torch.cat([e.logits[0] for e in engs]).float().cpu().numpy()
        want = o.step_logits[step_idx]
        stats["logit_diff"].append(float(np.abs(got - want).max()))
        # the vocabulary-sharded argmax is the argmax of the gathered logits, on every rank
        assert all(int(e.tokens[0].item()) == int(np.argmax(got)) for e in engs)
        top2 = np.sort(want)[-2:]
        if top2[1] - top2[0] > 2e-2:
            stats["argmax_n"] += 1
            stats["argmax_ok"] += int(np.argmax(got) == np.argmax(want))

    cmp_logits(0)
    assert engs[0].slot_pos[0].cpu().numpy().tolist() == o.slot_tables[0].tolist()
    for s in range(1, max_new + 1):
        for e in engs:
            e.tokens.fill_(int(forced[s - 1]))
            e._append_evict()
        assert engs[0].slot_pos[0].cpu().numpy().tolist() == o.slot_tables[s].tolist(), f"slot table at step {s}"
        _same_on_all_ranks(engs, "slot_pos")
        if s == max_new:
            break
        run_lockstep([e._forward_phases(sample=True) for e in engs])
        run_lockstep([iter([("max", e.step_score)]) for e in engs])
        sp = engs[0].slot_pos[0].cpu().numpy()
        got = engs[0].step_score[0].cpu().numpy()[sp >= 0]
        want = o.step_scores[s - 1][sp[sp >= 0]]
        stats["score_rel"].append(np.abs(got - want) / np.maximum(want, 1e-30))
        stats["score_ok"].append(bool((np.abs(got - want) <= 0.08 * want + 1e-3 * want.max()).all()))
        cmp_logits(s)
        for e in engs:
            capi.check(L.kvbp_score_update(e.stream, capi.C.byref(e._state), e.seq_step.data_ptr(),
                                           e.step_score.data_ptr(), e.dev_err.data_ptr()), "score_update")
    torch.cuda.synchronize()
    for e in engs:
        e.check_device_errors()
    for name in ("h", "slot_pos", "cumul", "last_access", "evlog", "evcount", "tokens"):
        _same_on_all_ranks(engs, name)
    n = int(engs[0].evcount[0].item())
    return o, stats, engs[0].evlog[0, :n].cpu().numpy().tolist()


@pytest.mark.parametrize("preset,policy,world", [("parity-qwen2", "lru", 2), ("parity-qwen2", "h2o_faithful", 4),
                                                 ("parity-qwen3", "lru", 4), ("parity-g7", "h2o_faithful", 2)])
def test_tp_teacher_forced_parity(preset, policy, world):
    o, st, evicted = _run_forced_tp(preset, policy, world)
    assert max(st["logit_diff"]) <= 2e-2, max(st["logit_diff"])
    assert st["argmax_n"] >= 10 and st["argmax_ok"] >= 0.99 * st["argmax_n"]
    rel = np.concatenate(st["score_rel"])
    print(f"tp{world} {preset}/{policy}: max logit diff {max(st['logit_diff']):.3g}, argmax "
          f"{st['argmax_ok']}/{st['argmax_n']}, score rel max {rel.max():.3g} median {np.median(rel):.3g}")
    assert all(st["score_ok"])
    assert np.median(rel) <= 1e-3
    if policy == "lru":
        assert evicted == o.positions_evicted
    else:
        assert len(evicted) == len(o.positions_evicted)
        assert len(set(evicted) & set(o.positions_evicted)) >= 0.9 * len(evicted)


def test_argmax_key_over_vocabulary_shards():
    g = torch.Generator(device="cuda").manual_seed(5)
    B, V, shards = 6, 4096, 4
    logits = torch.randn(B, V, generator=g, device="cuda").to(torch.bfloat16)
    logits[1, 100] = logits[1, 3000] = 9.0  # tie across shards: the lower index wins
    logits[2, 1024] = logits[2, 1025] = 9.0  # tie inside a shard
    logits[3] = -1.0  # all equal and negative: index 0
    L = capi.lib()
    st = torch.cuda.current_stream().cuda_stream
    keys = torch.full((B,), torch.iinfo(torch.int64).min, dtype=torch.int64, device="cuda")
    per = V // shards
    for r in range(shards):
        k = torch.empty(B, dtype=torch.int64, device="cuda")
        part = logits[:, r * per : (r + 1) * per].contiguous()
        capi.check(L.kvbp_argmax_key(st, B, per, per, part.data_ptr(), r * per, k.data_ptr()), "argmax_key")
        torch.maximum(keys, k, out=keys)
    tok = torch.empty(B, dtype=torch.int32, device="cuda")
    capi.check(L.kvbp_key_to_token(st, B, keys.data_ptr(), tok.data_ptr()), "key_to_token")
    ref = torch.empty(B, dtype=torch.int32, device="cuda")
    capi.check(L.kvbp_argmax(st, B, V, V, logits.data_ptr(), ref.data_ptr()), "argmax")
    torch.cuda.synchronize()
    assert tok.tolist() == ref.tolist()
    assert tok[1].item() == 100 and tok[2].item() == 1024 and tok[3].item() == 0


def test_residual_add_matches_torch():
    g = torch.Generator(device="cuda").manual_seed(2)
    M, H = 13, 1024
    h = torch.randn(M, H, generator=g, device="cuda").to(torch.bfloat16)
    d = torch.randn(M, H, generator=g, device="cuda")
    ss = torch.full((H // 128, 32), 5.0, device="cuda")
    want = (h.float() + d.to(torch.bfloat16).float()).to(torch.bfloat16)
    capi.check(capi.lib().kvbp_residual_add(torch.cuda.current_stream().cuda_stream, M, H, h.data_ptr(), d.data_ptr(),
                                            ss.data_ptr()), "residual_add")
    torch.cuda.synchronize()
    assert torch.equal(h, want)
    ss_ref = (want.float() ** 2).view(M, H // 128, 128).sum(-1).t()
    assert torch.allclose(ss[:, :M], ss_ref, rtol=1e-5)
    assert (ss[:, M:] == 0).all()


@pytest.mark.parametrize("M", [16, 32])  # 32 rows: the tcgen05 main loop
def test_gemm_fp32_epilogue_is_the_unrounded_sum(M):
    from kvcacheboundaryprotection_b200.engine import pack_weight

    g = torch.Generator(device="cuda").manual_seed(4)
    N, K = 512, 1024
    W = (torch.randn(N, K, generator=g, device="cuda") * 0.05).to(torch.bfloat16)
    x = torch.randn(M, K, generator=g, device="cuda").to(torch.bfloat16)
    for splits in (1, 4):
        out = torch.zeros(M, N, device="cuda")
        capi.check(capi.lib().kvbp_decode_gemm(torch.cuda.current_stream().cuda_stream, 3, M, N, K,
                                               pack_weight(W).data_ptr(), x.data_ptr(), K, None, 0, None, 1e-6,
                                               out.data_ptr(), N, None, splits, None), "gemm")
        torch.cuda.synchronize()
        ref = x.float() @ W.float().t()
        assert torch.allclose(out, ref, rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("M,splits", [(5, 1), (16, 4), (32, 2)])  # 32 rows: the tcgen05 main loop
def test_fused_allreduce_gemm_single_rank_equals_residual_gemm(M, splits):
    """kvbp_decode_gemm_allreduce with one rank (its own symmetric buffer the only peer) is
    the residual GEMM: h = bf16(h + bf16(acc)) bit for bit and the same per-tile sums of
    squares of the new h -- the allreduce epilogue's push, tag wait and rank-order sum
    reduce to the identity."""
    from kvcacheboundaryprotection_b200.engine import pack_weight

    g = torch.Generator(device="cuda").manual_seed(11)
    N, K = 1024, 2048
    W = (torch.randn(N, K, generator=g, device="cuda") * 0.03).to(torch.bfloat16)
    x = torch.randn(M, K, generator=g, device="cuda").to(torch.bfloat16)
    h0 = torch.randn(M, N, generator=g, device="cuda").to(torch.bfloat16)
    Wp = pack_weight(W)
    L = capi.lib()
    st = torch.cuda.current_stream().cuda_stream
    h_ref, ss_ref = h0.clone(), torch.zeros(N // 128, 32, device="cuda")
    capi.check(L.kvbp_decode_gemm(st, 1, M, N, K, Wp.data_ptr(), x.data_ptr(), K, None, 0, None, 1e-6,
                                  h_ref.data_ptr(), N, ss_ref.data_ptr(), splits, None), "residual gemm")
    buf_bytes = 2 * 1 * M * N * 8
    buf = torch.zeros(buf_bytes // 4, dtype=torch.int32, device="cuda")
    peers = torch.tensor([buf.data_ptr()], dtype=torch.int64, device="cuda")
    epoch = torch.ones(1, dtype=torch.int32, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    h, ss = h0.clone(), torch.zeros(N // 128, 32, device="cuda")
    capi.check(L.kvbp_decode_gemm_allreduce(st, M, N, K, Wp.data_ptr(), x.data_ptr(), K, h.data_ptr(), ss.data_ptr(),
                                            splits, peers.data_ptr(), 1, 0, 0, epoch.data_ptr(), buf_bytes,
                                            err.data_ptr()), "allreduce gemm")
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert torch.equal(h, h_ref)
    assert torch.allclose(ss[:, :M], ss_ref[:, :M], rtol=1e-5, atol=0)
