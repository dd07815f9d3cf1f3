"""Lossy int8 demotion of cache rows (kvbp_demote_int8) against the oracle's restatement
of the reference's round trip (online_credit_generator.py:643-704), bit for bit: the
operations are single bf16-rounded float32 ops, so there is no accumulation order to
differ in."""

import numpy as np
import pytest
import torch

from kvcacheboundaryprotection_b200 import build, capi
from oracle.model import int8_roundtrip

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _lib():
    build.build()


def test_demote_rows_match_oracle_and_leave_others_alone():
    L, B, Hkv, S = 3, 4, 2, 40
    g = torch.Generator(device="cuda").manual_seed(0)
    kc = (torch.randn(L, B, Hkv, S, 128, generator=g, device="cuda") * 3).to(torch.bfloat16)
    vc = torch.randn(L, B, Hkv, S, 128, generator=g, device="cuda").to(torch.bfloat16)
    kc[0, 1, 0, 5] = 0.0                     # all-zero row: scale 0, stays 0
    kc[1, 2, 1, 7, :4] = torch.tensor([127.0, 63.5, -0.5, 1.5])  # exact half-way quotients
    slots = torch.tensor([[5, 7, -1], [5, 0, 39], [7, 3, 3], [1, 2, 4]], dtype=torch.int32, device="cuda")
    counts = torch.tensor([2, 3, 1, 0], dtype=torch.int32, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    k0, v0 = kc.clone(), vc.clone()
    capi.check(capi.lib().kvbp_demote_int8(torch.cuda.current_stream().cuda_stream, kc.data_ptr(), vc.data_ptr(),
                                           L, B, Hkv, S, slots.data_ptr(), 3, counts.data_ptr(), err.data_ptr()),
               "demote_int8")
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    want_k, want_v = k0.float().cpu().numpy(), v0.float().cpu().numpy()
    for b in range(B):
        for j in range(int(counts[b])):
            s = int(slots[b, j])
            want_k[:, b, :, s] = int8_roundtrip(want_k[:, b, :, s])
            want_v[:, b, :, s] = int8_roundtrip(want_v[:, b, :, s])
    assert np.array_equal(kc.float().cpu().numpy(), want_k)
    assert np.array_equal(vc.float().cpu().numpy(), want_v)
    assert (kc[0, 1, 0, 5] == 0).all()
    assert not torch.equal(kc, k0)  # something was demoted


def test_out_of_range_slot_sets_the_index_error():
    kc = torch.zeros(1, 1, 1, 8, 128, dtype=torch.bfloat16, device="cuda")
    vc = torch.zeros_like(kc)
    slots = torch.tensor([[9]], dtype=torch.int32, device="cuda")
    counts = torch.tensor([1], dtype=torch.int32, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    capi.check(capi.lib().kvbp_demote_int8(torch.cuda.current_stream().cuda_stream, kc.data_ptr(), vc.data_ptr(),
                                           1, 1, 1, 8, slots.data_ptr(), 1, counts.data_ptr(), err.data_ptr()), "demote")
    torch.cuda.synchronize()
    assert int(err.item()) & 4  # KVBP_DEV_INDEX


def test_engine_demotes_retained_positions_once():
    from kvcacheboundaryprotection_b200.config import get_config
    from kvcacheboundaryprotection_b200.engine import CappedKVEngine, EvictionSpec
    from kvcacheboundaryprotection_b200.weights import init_weights

    cfg = get_config("parity-qwen2").with_(n_layers=1, vocab=1024)
    eng = CappedKVEngine(cfg, init_weights(cfg, seed=0), batch=2, evict=EvictionSpec("lru", 32, 8, True), max_prompt_len=64,
                         max_new_tokens=4)
    eng.synthetic_prefill(64, seed=3)
    sp = eng.slot_pos.cpu().numpy()
    live = [int(p) for p in sp[0] if p >= 0][:3]
    before = eng.kc.clone()
    got = eng.demote_positions([live + [10 ** 6], []])  # an unknown position is skipped
    assert got == [live, []]
    after = eng.kc.clone()
    for p in live:
        s = int(np.flatnonzero(sp[0] == p)[0])
        want = int8_roundtrip(before[0, 0, :, s].float().cpu().numpy())
        assert np.array_equal(after[0, 0, :, s].float().cpu().numpy(), want)
    assert eng.demote_positions([live, []]) == [[], []]  # already demoted: skipped
    assert torch.equal(eng.kc, after)
