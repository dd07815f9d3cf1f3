"""C-ABI library checks that need no GPU: it loads, exports every declared symbol,
and its host-side validation / pure host helpers behave."""

import ctypes as C
import os
import re

import pytest

from kvcacheboundaryprotection_b200 import build, capi

from conftest import REPO


def _declared():
    text = open(os.path.join(REPO, "include", "kvbp.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(kvbp_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def L():
    build.build()
    return capi.lib()


def test_exports_every_declared_symbol(L):
    names = _declared()
    assert len(names) >= 15
    for n in names:
        assert hasattr(L, n), n
    assert set(names) == set(capi.SIGNATURES), "ctypes signatures out of sync with include/kvbp.h"


def test_version_and_policy_ids(L):
    assert b"sm_100a" in L.kvbp_version()
    assert capi.policy_id("lru") == 0
    assert capi.policy_id("attention-mass") == capi.policy_id("h2o_faithful") == 1
    assert L.kvbp_policy_id(b"random") == 8 and L.kvbp_policy_id(b"no_such_policy") == -1
    with pytest.raises(ValueError):
        capi.policy_id("adakv_faithful")


@pytest.mark.parametrize(
    "cap,pf,sf,expect",
    [(256, 0.10, 0.10, (25, 25)), (1024, 0.10, 0.10, (102, 102)), (4096, 0.10, 0.10, (409, 409)),
     (256, 0.05, 0.05, (12, 12)), (8, 0.10, 0.0, (4, 0)), (1000, 0.07, 0.0, (70, 0)), (30, 0.0, 0.5, (0, 15))],
)
def test_protection_sizes_match_python(L, cap, pf, sf, expect):
    py = (max(4, int(cap * pf)) if pf > 0 else 0, max(4, int(cap * sf)) if sf > 0 else 0)
    assert capi.protection_sizes(cap, pf, sf) == py == expect


def test_host_validation_rejects_bad_arguments(L):
    # null pointers are rejected on the host before any CUDA call
    st = L.kvbp_decode_attn_score(None, 1, 4, 1, 128, 64, None, None, None, None, None, None, None, None)
    assert st == 1 and b"null" in L.kvbp_last_error()
    st = L.kvbp_decode_attn_score(None, 1, 4, 1, 64, 64, 1, 1, 1, 1, None, 1, 1, None)
    assert st == 2  # head_dim 64 unsupported
    st = L.kvbp_decode_attn_score(None, 1, 18, 2, 128, 64, 16, 16, 16, 16, None, 16, 16, None)
    assert st == 2  # group of 9 heads unsupported
    assert L.kvbp_argmax(None, 1, 100, 50, 16, 16) == 1  # ld < vocab
    assert L.kvbp_argmax(None, 1, 100, 101, 16, 16) == 1  # rows not 16-byte aligned (ld % 8 != 0)
    cfg = capi.EvictCfg(0, 8, 0, 1, 25, 25, 1)
    n = C.c_int32()
    assert L.kvbp_prefill_select(None, 1, 100, C.byref(cfg), None, 16, 16, 10, C.byref(n), None) == 1
    with pytest.raises(capi.KVBPError):
        capi.check(L.kvbp_embed(None, 1, 10, 12, 16, 16, 16, None), "embed")


def test_host_validation_of_the_operator_step_and_prefill_gemm_entries(L):
    # kvbp_update_append_evict needs its step scores and pending flags
    st_ = capi.State(1, 64, 4, *([16] * 9))
    cfg = capi.EvictCfg(32, 8, 0, 1, 4, 4, 1)
    args = (None, C.byref(st_), C.byref(cfg), 16, 16, 16, 16, None, None, 0, 16, 16, 8, None)
    assert L.kvbp_update_append_evict(*args, None, 16, None) == 1
    assert b"step_score and pending" in L.kvbp_last_error()
    assert L.kvbp_update_append_evict(*args, 16, None, None) == 1
    # attention + scatter without state needs the new row
    st = L.kvbp_decode_attn_score_update(None, 1, 4, 1, 128, 64, 16, None, None, 16, 16, 16, 16, 16, 16, None, None,
                                         None, None)
    assert st == 1 and b"nothing to fuse" in L.kvbp_last_error()
    # prefill GEMM: epilogues 0 (plain), 2 (SwiGLU) and 3 (fp32) only; sizes multiples of 128
    assert L.kvbp_prefill_gemm(None, 1, 128, 128, 128, 16, 16, 128, 16, 128, None) == 2
    assert L.kvbp_prefill_gemm(None, 0, 128, 100, 128, 16, 16, 128, 16, 128, None) == 1
    assert L.kvbp_prefill_gemm(None, 2, 128, 256, 128, 16, 16, 128, 16, 64, None) == 1  # SwiGLU: ldo 64 < N/2
    assert L.kvbp_prefill_gemm(None, 0, 128, 128, 128, None, 16, 128, 16, 128, None) == 1  # null weights
