"""kvbp_prefill_evict_noalloc vs. kvbp_prefill_select + kvbp_prefill_compact.

The no-allocation entry point exists for callers that cannot allocate device memory
(e.g. a jax.ffi / XLA custom-call handler, which may only use the buffers XLA assigns
it).  It must produce exactly what the two-call path with a caller-provided flag
buffer produces.  Two calls in a row with different shapes and policies check that the
shared fixed scratch array carries nothing over from the previous call.  This file is
collected last (tests/test_zz_*) so a run that stops at the first failure has already
run every other test; it also passes alone in a fresh process.
"""

import ctypes as C

import numpy as np
import pytest
import torch

from kvcacheboundaryprotection_b200 import build, capi

pytestmark = pytest.mark.gpu


class _State:
    def __init__(self, B, S, W, evcap, log_steps):
        d = "cuda"
        z = lambda *s, dt=torch.int32: torch.zeros(*s, dtype=dt, device=d)  # noqa: E731
        self.t = {
            "slot_pos": torch.full((B, S), -7, dtype=torch.int32, device=d),
            "ins": z(B, S), "last": z(B, S), "cnt": z(B, S),
            "attn": z(B, S, dt=torch.float32), "maxa": z(B, S, dt=torch.float32),
            "cumul": z(B, S, dt=torch.float64), "pre": z(B, S, dt=torch.float32),
            "posmap": z(B, W),
            "gather_src": z(B, S), "evlog": z(B, evcap), "evcount": z(B),
            "seq_step": z(B) + 5, "next_pos": z(B), "retained_log": z(B, log_steps + 1),
            "step_score": torch.ones(B, S, dtype=torch.float32, device=d), "err": z(1),
        }
        t = self.t
        self.state = capi.State(B, S, W, *[t[k].data_ptr() for k in ("slot_pos", "ins", "last", "cnt", "attn", "maxa", "cumul", "pre", "posmap")])
        self.evcap, self.log_steps = evcap, log_steps

    def host(self):
        torch.cuda.synchronize()
        return {k: v.cpu().numpy() for k, v in self.t.items()}


def _run_pair(B, P, cap, policy, frac, seed):
    L = capi.lib()
    st = torch.cuda.current_stream().cuda_stream
    n_pre, n_suf = capi.protection_sizes(cap, frac, frac)
    cfg = capi.EvictCfg(cap, 8, capi.policy_id(policy), 1, n_pre, n_suf, 1)
    S, W, evcap, log_steps = cap + 8, (P + 64 + 31) // 32, P + 64, 16
    rng = np.random.default_rng(seed)
    scores = torch.from_numpy((rng.random((B, P)) ** 3).astype(np.float32)).cuda() if policy != "lru" else None
    sp = None if scores is None else scores.data_ptr()

    ref = _State(B, S, W, evcap, log_steps)
    victim = torch.zeros(B, P, dtype=torch.uint8, device="cuda")
    n = C.c_int32()
    r = ref.t
    capi.check(L.kvbp_prefill_select(st, B, P, C.byref(cfg), sp, victim.data_ptr(), r["evlog"].data_ptr(), evcap, C.byref(n), r["err"].data_ptr()), "select")
    capi.check(L.kvbp_prefill_compact(st, C.byref(ref.state), P, cap, n.value, victim.data_ptr(), sp, r["gather_src"].data_ptr(), r["evlog"].data_ptr(), evcap, r["evcount"].data_ptr(), r["seq_step"].data_ptr(), r["next_pos"].data_ptr(), r["retained_log"].data_ptr(), log_steps, r["step_score"].data_ptr(), r["err"].data_ptr()), "compact")

    got = _State(B, S, W, evcap, log_steps)
    g = got.t
    capi.check(L.kvbp_prefill_evict_noalloc(st, C.byref(got.state), P, C.byref(cfg), sp, g["gather_src"].data_ptr(), g["evlog"].data_ptr(), evcap, g["evcount"].data_ptr(), g["seq_step"].data_ptr(), g["next_pos"].data_ptr(), g["retained_log"].data_ptr(), log_steps, g["step_score"].data_ptr(), g["err"].data_ptr()), "noalloc")
    return ref.host(), got.host()


@pytest.fixture(scope="module", autouse=True)
def _lib():
    build.build()
    capi.lib()


def test_noalloc_matches_two_call_path_on_consecutive_calls():
    # call 1: larger batch x prompt, scored policy; call 2: smaller, LRU -- the second
    # call must not see any flag left over from the first
    for B, P, cap, policy, frac, seed in ((4, 3000, 256, "h2o_faithful", 0.10, 1), (3, 1100, 300, "lru", 0.05, 2)):
        ref, got = _run_pair(B, P, cap, policy, frac, seed)
        assert int(ref["err"][0]) == 0 and int(got["err"][0]) == 0
        for k in ref:
            if k == "err":
                continue
            if k == "evlog":
                for b in range(B):
                    n = int(ref["evcount"][b])
                    assert np.array_equal(ref[k][b, :n], got[k][b, :n]), (policy, k, b)
            else:
                assert np.array_equal(ref[k], got[k]), (policy, k)


def test_noalloc_rejects_sizes_beyond_its_scratch():
    L = capi.lib()
    st = capi.State(1024, 16, 1, *([0] * 9))
    cfg = capi.EvictCfg(8, 8, 0, 1, 4, 4, 1)
    status = L.kvbp_prefill_evict_noalloc(None, C.byref(st), 2048, C.byref(cfg), None, None, None, 0, None, None, None, None, 0, None, None)
    assert status == 1
    assert b"exceeds the fixed scratch" in L.kvbp_last_error()
