"""K1 decode attention + per-slot score vs. a plain PyTorch fp32 reference of the same op.

The reference op (jax_inference.py:1018-1050): s = bf16(bf16(q.k) * bf16(1/sqrt(128))),
float32 softmax over the valid slots, out = bf16(p @ float32(V)); per-slot score =
max over the group's heads of p, max-accumulated into step_score.

Tolerances: q.k is accumulated in fp32 in a different order (tensor-core mma vs. the
fp32 GEMM), so a logit can land on the neighbouring bfloat16 value; such slots move
their probabilities by <= 2^-8 relative.  We require
  * out:   max |diff| <= 1.6e-2 and >= 97 % of elements bit-identical,
  * score: rel diff <= 1e-5 on >= 97 % of slots and <= 2e-2 everywhere.
"""

import math

import pytest
import torch

from kvcacheboundaryprotection_b200 import build, capi

pytestmark = pytest.mark.gpu

SCALE = float(torch.tensor(1.0 / math.sqrt(128)).to(torch.bfloat16))


def torch_reference(q, kc, vc, slot_pos):
    B, Hq, D = q.shape
    Hkv, S = kc.shape[1], kc.shape[2]
    G = Hq // Hkv
    out = torch.zeros(B, Hq, D, dtype=torch.float32, device=q.device)
    score = torch.zeros(B, S, dtype=torch.float32, device=q.device)
    for b in range(B):
        valid = slot_pos[b] >= 0
        for g in range(Hkv):
            K = kc[b, g].float()
            V = vc[b, g].float()
            qg = q[b, g * G : (g + 1) * G].float()
            s = (qg @ K.t()).to(torch.bfloat16).float()
            s = (s * SCALE).to(torch.bfloat16).float()
            s = torch.where(valid[None, :], s, torch.tensor(float("-inf"), device=q.device))
            p = torch.softmax(s, dim=-1)
            out[b, g * G : (g + 1) * G] = (p @ V).to(torch.bfloat16).float()
            score[b] = torch.maximum(score[b], p.max(0).values)
    return out, score


def run_kernel(q, kc, vc, slot_pos, score_init=None, cluster=0, persist=None):
    L = capi.lib()
    B, Hq, D = q.shape
    Hkv, S = kc.shape[1], kc.shape[2]
    out = torch.empty_like(q)
    score = score_init.clone() if score_init is not None else torch.zeros(B, S, dtype=torch.float32, device=q.device)
    err = torch.zeros(1, dtype=torch.int32, device=q.device)
    st = torch.cuda.current_stream().cuda_stream
    args = (st, B, Hq, Hkv, D, S, q.data_ptr(), kc.data_ptr(), vc.data_ptr(), slot_pos.data_ptr(), None,
            out.data_ptr(), score.data_ptr(), err.data_ptr())
    if persist is not None:
        capi.check(L.kvbp_decode_attn_score_cfg(*args, cluster, persist), "attn")
    elif cluster:
        capi.check(L.kvbp_decode_attn_score_cs(*args, cluster), "attn")
    else:
        capi.check(L.kvbp_decode_attn_score(*args), "attn")
    torch.cuda.synchronize()
    assert int(err.item()) == 0, capi.decode_dev_errors(int(err.item()))
    return out.float(), score


def make_case(B, Hq, Hkv, S, free_frac, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    q = (torch.randn(B, Hq, 128, generator=g, device="cuda") / math.sqrt(128)).to(torch.bfloat16)
    kc = torch.randn(B, Hkv, S, 128, generator=g, device="cuda").to(torch.bfloat16)
    vc = torch.randn(B, Hkv, S, 128, generator=g, device="cuda").to(torch.bfloat16)
    pos = torch.randperm(S * 4, generator=g, device="cuda")[:S].to(torch.int32).repeat(B, 1)
    free = torch.rand(B, S, generator=g, device="cuda") < free_frac
    pos[free] = -1
    pos[:, 0] = 0  # at least one valid slot
    return q, kc, vc, pos.contiguous()


def assert_close(out, score, ref_out, ref_score, valid):
    d = (out - ref_out).abs()
    assert d.max().item() <= 1.6e-2, d.max().item()
    assert (d == 0).float().mean().item() >= 0.97
    rel = ((score - ref_score).abs() / ref_score.clamp_min(1e-30))[valid]
    assert rel.max().item() <= 2e-2, rel.max().item()
    assert (rel <= 1e-5).float().mean().item() >= 0.97
    assert (score[~valid] == 0).all()


CASES = [
    # B, Hq, Hkv, S, free fraction
    (2, 8, 2, 264, 0.05),  # tiny-qwen2 heads, capacity 256 + 8
    (3, 4, 1, 100, 0.3),
    (2, 28, 4, 1032, 0.01),  # Qwen2.5-7B group of 7
    (1, 32, 8, 4104, 0.002),  # Qwen3-4B / microbench group of 4, capacity 4096
    (2, 16, 2, 136, 0.0),  # group of 8
    (1, 3, 3, 70, 0.1),  # group of 1
    (2, 6, 2, 200, 0.2),  # group of 3
    (1, 10, 2, 77, 0.1),  # group of 5
    (1, 12, 2, 129, 0.1),  # group of 6
    (4, 32, 8, 1, 0.0),  # a single slot
]


@pytest.fixture(scope="module", autouse=True)
def _lib():
    build.build()
    capi.lib()


@pytest.mark.parametrize("B,Hq,Hkv,S,free", CASES)
def test_attention_matches_torch_reference(B, Hq, Hkv, S, free):
    q, kc, vc, pos = make_case(B, Hq, Hkv, S, free, seed=S * 7 + Hq)
    out, score = run_kernel(q, kc, vc, pos)
    ref_out, ref_score = torch_reference(q, kc, vc, pos)
    assert_close(out, score, ref_out, ref_score, pos >= 0)


@pytest.mark.parametrize("cluster", [1, 2, 3, 5, 8])
def test_attention_every_cluster_size(cluster):
    q, kc, vc, pos = make_case(2, 28, 4, 1032, 0.05, seed=11)
    out, score = run_kernel(q, kc, vc, pos, cluster=cluster)
    ref_out, ref_score = torch_reference(q, kc, vc, pos)
    assert_close(out, score, ref_out, ref_score, pos >= 0)


def test_step_score_is_max_accumulated():
    q, kc, vc, pos = make_case(2, 8, 2, 264, 0.1, seed=5)
    init = torch.rand(2, 264, device="cuda") * 0.02
    init[pos < 0] = 0
    _, score = run_kernel(q, kc, vc, pos, score_init=init)
    _, fresh = run_kernel(q, kc, vc, pos)
    assert torch.equal(score, torch.maximum(init, fresh))


def test_large_batch_microbench_shape_runs_clean():
    # B=64, Hkv=8, G=4, capacity 1024: the operator microbench shape
    q, kc, vc, pos = make_case(64, 32, 8, 1032, 0.0, seed=3)
    out, score = run_kernel(q, kc, vc, pos)
    ref_out, ref_score = torch_reference(q[:4], kc[:4], vc[:4], pos[:4])
    assert_close(out[:4], score[:4], ref_out, ref_score, pos[:4] >= 0)
    assert torch.isfinite(out).all()


@pytest.mark.parametrize("cluster", [0, 1, 3])
def test_early_streaming_with_write_slot_matches_plain(cluster):
    """With write_slot the kernel stages its first tiles before the preceding K/V store
    finishes and reloads the written row; the result must equal a call without it."""
    from kvcacheboundaryprotection_b200.engine import inv_freq_table

    g = torch.Generator(device="cuda").manual_seed(17)
    B, Hq, Hkv, D, S = 4, 28, 4, 128, 1032
    tiles = (S + 63) // 64
    cs = cluster or 4
    kc = torch.randn(B, Hkv, S, D, generator=g, device="cuda").to(torch.bfloat16)
    vc = torch.randn(B, Hkv, S, D, generator=g, device="cuda").to(torch.bfloat16)
    slot_pos = torch.arange(S, device="cuda", dtype=torch.int32).repeat(B, 1)
    slot_pos[:, 1000:] = -1
    t0_rank1 = (1 * tiles) // cs if cs > 1 else 1
    ws = torch.tensor([3, t0_rank1 * 64 + 5, 999, -1], dtype=torch.int32, device="cuda")
    qkv = torch.randn(B, (Hq + 2 * Hkv) * D, generator=g, device="cuda").to(torch.bfloat16)
    pos = torch.tensor([7, 900, 4000, 12], dtype=torch.int32, device="cuda")
    inv = torch.from_numpy(inv_freq_table(D, 1e6)).cuda()
    q = torch.empty(B, Hq, D, dtype=torch.bfloat16, device="cuda")
    L = capi.lib()
    st = torch.cuda.current_stream().cuda_stream
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    outs = []
    for use_ws in (True, False):
        kc_i, vc_i = kc.clone(), vc.clone()
        out = torch.zeros(B, Hq, D, dtype=torch.bfloat16, device="cuda")
        score = torch.zeros(B, S, dtype=torch.float32, device="cuda")
        torch.cuda.synchronize()
        capi.check(L.kvbp_qkv_rope_scatter(st, B, 1, Hq, Hkv, D, S, qkv.data_ptr(), (Hq + 2 * Hkv) * D, None, None,
                                           None, 1e-6, inv.data_ptr(), pos.data_ptr(), ws.data_ptr(), q.data_ptr(),
                                           kc_i.data_ptr(), vc_i.data_ptr(), err.data_ptr()), "rope")
        capi.check(L.kvbp_decode_attn_score_cs(st, B, Hq, Hkv, D, S, q.data_ptr(), kc_i.data_ptr(), vc_i.data_ptr(),
                                               slot_pos.data_ptr(), ws.data_ptr() if use_ws else None,
                                               out.data_ptr(), score.data_ptr(), err.data_ptr(), cluster), "attn")
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        outs.append((out, score, kc_i))
    assert torch.equal(outs[0][0], outs[1][0])
    assert torch.equal(outs[0][1], outs[1][1])
    # and the written rows really are part of the attention (the reference agrees)
    ref_out, ref_score = torch_reference(q, outs[1][2], vc_i, slot_pos)
    assert (outs[0][0].float() - ref_out).abs().max().item() <= 1.6e-2


def _state(B, S, pos, seed):
    """kvbp_state arrays with seeded metadata for the score update."""
    g = torch.Generator(device="cuda").manual_seed(seed)
    d = "cuda"
    st = {
        "slot_pos": pos,  # shared: neither path changes slot positions
        "insert_step": torch.randint(0, 5, (B, S), generator=g, device=d, dtype=torch.int32),
        "last_access": torch.randint(0, 9, (B, S), generator=g, device=d, dtype=torch.int32),
        "access_count": torch.randint(1, 9, (B, S), generator=g, device=d, dtype=torch.int32),
        "attn": torch.rand(B, S, generator=g, device=d),
        "max_attn": torch.rand(B, S, generator=g, device=d),
        "cumul": torch.rand(B, S, generator=g, device=d, dtype=torch.float64) * 3,
        "prefill": torch.rand(B, S, generator=g, device=d),
        "posmap": torch.zeros(B, 64, dtype=torch.int32, device=d),
    }
    s = capi.State(B, S, 64, *[st[k].data_ptr() for k in ("slot_pos", "insert_step", "last_access", "access_count",
                                                        "attn", "max_attn", "cumul", "prefill", "posmap")])
    return st, s


@pytest.mark.parametrize("B,Hq,Hkv,S", [(64, 32, 8, 264), (16, 28, 4, 1032), (3, 8, 2, 4104)])
def test_fused_scatter_and_score_update_equal_separate_launches(B, Hq, Hkv, S):
    """kvbp_decode_attn_score_update (new K/V row stored by the attention kernel, score
    update by the last CTA of each sequence) gives bit for bit the state of the separate
    launches: the row copied into the cache, kvbp_decode_attn_score, kvbp_score_update --
    on two calls in a row (the per-sequence arrival counters reset themselves)."""
    import ctypes as C

    L = capi.lib()
    stream = torch.cuda.current_stream().cuda_stream
    q, kc, vc, pos = make_case(B, Hq, Hkv, S, 0.2, seed=S)
    g = torch.Generator(device="cuda").manual_seed(7)
    knew = torch.randn(B, Hkv, 128, generator=g, device="cuda").to(torch.bfloat16)
    vnew = torch.randn(B, Hkv, 128, generator=g, device="cuda").to(torch.bfloat16)
    ws = torch.randint(0, S, (B,), generator=g, device="cuda", dtype=torch.int32)
    ws[0] = -1  # a sequence whose new position was evicted before its forward
    pos[torch.arange(B, device="cuda")[1:], ws[1:].long()] = 10 ** 6  # the written slots hold the new position
    seq_step = torch.full((B,), 9, dtype=torch.int32, device="cuda")
    kc_a, vc_a, kc_b, vc_b = kc.clone(), vc.clone(), kc.clone(), vc.clone()
    sa, state_a = _state(B, S, pos, 1)
    sb, state_b = _state(B, S, pos, 1)
    counter = torch.zeros(B, dtype=torch.int32, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    for rep in range(2):
        out_a, out_b = torch.empty_like(q), torch.empty_like(q)
        sc_a = torch.zeros(B, S, device="cuda")
        sc_b = torch.zeros(B, S, device="cuda")
        for b in range(1, B):  # separate: the scatter, attention, score update
            kc_a[b, :, ws[b]] = knew[b]
            vc_a[b, :, ws[b]] = vnew[b]
        capi.check(L.kvbp_decode_attn_score(stream, B, Hq, Hkv, 128, S, q.data_ptr(), kc_a.data_ptr(), vc_a.data_ptr(),
                                            pos.data_ptr(), ws.data_ptr(), out_a.data_ptr(), sc_a.data_ptr(),
                                            err.data_ptr()), "attn")
        capi.check(L.kvbp_score_update(stream, C.byref(state_a), seq_step.data_ptr(), sc_a.data_ptr(), err.data_ptr()),
                   "score_update")
        capi.check(L.kvbp_decode_attn_score_update(stream, B, Hq, Hkv, 128, S, q.data_ptr(), knew.data_ptr(),
                                                   vnew.data_ptr(), kc_b.data_ptr(), vc_b.data_ptr(), pos.data_ptr(),
                                                   ws.data_ptr(), out_b.data_ptr(), sc_b.data_ptr(), C.byref(state_b),
                                                   seq_step.data_ptr(), counter.data_ptr(), err.data_ptr()), "fused")
        torch.cuda.synchronize()
        assert int(err.item()) == 0, capi.decode_dev_errors(int(err.item()))
        assert torch.equal(out_a, out_b)
        assert torch.equal(kc_a, kc_b) and torch.equal(vc_a, vc_b)
        for k in ("attn", "max_attn", "cumul", "last_access", "access_count"):
            assert torch.equal(sa[k], sb[k]), k
        assert not sc_b.any() and not sc_a.any()
        assert not counter.any()
        knew, vnew = vnew, knew  # second call: other rows
        seq_step += 1


# more (sequence, kv head) pairs than one wave of two CTAs per SM holds: the persistent
# kernel (a single wave of clusters walking the pairs round-robin) is chosen by default; it
# must be bit-identical to one cluster per pair at the same cluster size
PERSIST_CASES = [
    # B, Hq, Hkv, S, free fraction, cluster size
    (64, 32, 8, 1032, 0.01, 1),  # operator microbench, capacity 1024
    (64, 32, 8, 1032, 0.01, 4),
    (64, 32, 8, 264, 0.05, 1),  # capacity 256 (one consumer group)
    (64, 32, 8, 4104, 0.002, 4),  # capacity 4096
    (64, 32, 8, 4104, 0.002, 3),  # uneven tile split over the cluster
    (40, 16, 8, 520, 0.1, 2),  # group of 2
    (75, 12, 4, 300, 0.1, 1),  # group of 3, 4 kv heads
]


@pytest.mark.parametrize("B,Hq,Hkv,S,free,cs", PERSIST_CASES)
def test_persistent_kernel_bit_identical_to_one_cluster_per_pair(B, Hq, Hkv, S, free, cs):
    q, kc, vc, pos = make_case(B, Hq, Hkv, S, free, seed=S + B + cs)
    init = torch.rand(B, S, device="cuda") * 1e-3  # step_score already holds earlier layers' maxima
    init[pos < 0] = 0
    out_p, score_p = run_kernel(q, kc, vc, pos, score_init=init, cluster=cs, persist=0)
    out_1, score_1 = run_kernel(q, kc, vc, pos, score_init=init, cluster=cs, persist=-1)
    assert torch.equal(out_p, out_1)
    assert torch.equal(score_p, score_1)
    # fewer clusters than one wave holds (each walks more pairs) gives the same results
    out_f, score_f = run_kernel(q, kc, vc, pos, score_init=init, cluster=cs, persist=7)
    assert torch.equal(out_f, out_1)
    assert torch.equal(score_f, score_1)
    if B <= 40:  # the fp32 reference loop is slow: check the smaller cases against it too
        out0, score0 = run_kernel(q, kc, vc, pos)
        ref_out, ref_score = torch_reference(q, kc, vc, pos)
        assert_close(out0, score0, ref_out, ref_score, pos >= 0)


def test_persistent_kernel_fused_scatter():
    """The new K/V row stored by the persistent kernel (st == NULL: scatter only) equals the
    row copied into the cache first and the plain kernel run on it."""
    B, Hq, Hkv, S = 64, 32, 8, 1032
    q, kc, vc, pos = make_case(B, Hq, Hkv, S, 0.01, seed=5)
    g = torch.Generator(device="cuda").manual_seed(6)
    knew = torch.randn(B, Hkv, 128, generator=g, device="cuda").to(torch.bfloat16)
    vnew = torch.randn(B, Hkv, 128, generator=g, device="cuda").to(torch.bfloat16)
    ws = torch.randint(0, S, (B,), generator=g, device="cuda").to(torch.int32)
    bi = torch.arange(B, device="cuda")
    pos[bi, ws.long()] = 10 ** 6 + bi.to(torch.int32)
    kc_a, vc_a = kc.clone(), vc.clone()
    kc_b, vc_b = kc.clone(), vc.clone()
    kc_b[bi, :, ws.long()] = knew
    vc_b[bi, :, ws.long()] = vnew
    L = capi.lib()
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    out_a, sc_a = torch.empty_like(q), torch.zeros(B, S, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    capi.check(L.kvbp_decode_attn_score_update(st, B, Hq, Hkv, 128, S, q.data_ptr(), knew.data_ptr(), vnew.data_ptr(),
                                               kc_a.data_ptr(), vc_a.data_ptr(), pos.data_ptr(), ws.data_ptr(),
                                               out_a.data_ptr(), sc_a.data_ptr(), None, None, None, err.data_ptr()),
               "attn_scatter")
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    out_b, sc_b = run_kernel(q, kc_b, vc_b, pos, cluster=1, persist=-1)
    assert torch.equal(kc_a, kc_b) and torch.equal(vc_a, vc_b)
    assert torch.equal(out_a.float(), out_b)
    assert torch.equal(sc_a, sc_b)
