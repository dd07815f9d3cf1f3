"""ctypes binding of ``libkvbp.so`` (declared in ``include/kvbp.h``).

Every call enqueues on the caller's CUDA stream (torch's current stream by default)
and raises ``KVBPError`` when the library reports a host-side error.  There is no
fallback: if the library is missing, ``lib()`` raises.
"""

from __future__ import annotations

import ctypes as C
import os
from pathlib import Path
from typing import Optional

LIB_PATH = Path(__file__).resolve().parent / "lib" / "libkvbp.so"

KVBP_OK = 0
LISTED_NO_HARDCAP = 1
DEV_ERRORS = {
    1: "no free KV slot",
    2: "NaN score",
    4: "index out of range (access skipped)",
    8: "bounded wait timed out",
    16: "no valid slot for a (sequence, kv head)",
    32: "eviction log overflow",
    64: "bounded wait for another GPU timed out",
}

POLICY_IDS = {
    "lru": 0,
    "h2o_faithful": 1,
    "attention-mass": 1,
    "attention_mass": 1,
    "h2o": 2,
    "snapkv": 3,
    "snapkv_faithful": 4,
    "adakv": 5,
    "quest": 6,
    "streamingllm": 7,
    "random": 8,  # victims sampled on the host, applied by kvbp_append_evict_listed
}


class KVBPError(RuntimeError):
    pass


class State(C.Structure):
    _fields_ = [
        ("B", C.c_int32),
        ("S", C.c_int32),
        ("W", C.c_int32),
        ("slot_pos", C.c_void_p),
        ("insert_step", C.c_void_p),
        ("last_access", C.c_void_p),
        ("access_count", C.c_void_p),
        ("attn", C.c_void_p),
        ("max_attn", C.c_void_p),
        ("cumul", C.c_void_p),
        ("prefill", C.c_void_p),
        ("posmap", C.c_void_p),
    ]


class EvictCfg(C.Structure):
    _fields_ = [
        ("capacity", C.c_int32),
        ("evict_every", C.c_int32),
        ("policy", C.c_int32),
        ("protect", C.c_int32),
        ("n_prefix", C.c_int32),
        ("n_suffix", C.c_int32),
        ("decode_regime", C.c_int32),
    ]


# name -> (restype, argtypes) for every symbol in include/kvbp.h
P, I32, I64, F32, F64 = C.c_void_p, C.c_int32, C.c_int64, C.c_float, C.c_double
SIGNATURES = {
    "kvbp_version": (C.c_char_p, []),
    "kvbp_last_error": (C.c_char_p, []),
    "kvbp_policy_id": (C.c_int, [C.c_char_p]),
    "kvbp_protection_sizes": (None, [I32, F64, F64, C.POINTER(C.c_int32), C.POINTER(C.c_int32)]),
    "kvbp_decode_attn_score": (C.c_int, [P, I32, I32, I32, I32, I32, P, P, P, P, P, P, P, P]),
    "kvbp_qkv_rope_scatter": (
        C.c_int,
        [P, I32, I32, I32, I32, I32, I32, P, I32, P, P, P, F32, P, P, P, P, P, P, P],
    ),
    "kvbp_score_update": (C.c_int, [P, C.POINTER(State), P, P, P]),
    "kvbp_append_evict": (
        C.c_int,
        [P, C.POINTER(State), C.POINTER(EvictCfg), P, P, P, P, P, P, I32, P, P, I32, P, P],
    ),
    "kvbp_update_append_evict": (
        C.c_int,
        [P, C.POINTER(State), C.POINTER(EvictCfg), P, P, P, P, P, P, I32, P, P, I32, P, P, P, P],
    ),
    "kvbp_append_evict_listed": (
        C.c_int,
        [P, C.POINTER(State), C.POINTER(EvictCfg), P, P, P, P, P, P, I32, P, P, I32, P, P, P, I32, I32, P],
    ),
    "kvbp_decode_attn_score_heads": (C.c_int, [P, I32, I32, I32, I32, I32, P, P, P, P, P, P, P, P, P, P]),
    "kvbp_decode_attn_score_update": (
        C.c_int,
        [P, I32, I32, I32, I32, I32, P, P, P, P, P, P, P, P, P, C.POINTER(State), P, P, P],
    ),
    "kvbp_head_signal_update": (C.c_int, [P, I32, I32, I32, P, P, P, P, P]),
    "kvbp_prefill_select": (C.c_int, [P, I32, I32, C.POINTER(EvictCfg), P, P, P, I32, C.POINTER(C.c_int32), P]),
    "kvbp_prefill_compact": (
        C.c_int,
        [P, C.POINTER(State), I32, I32, I32, P, P, P, P, I32, P, P, P, P, I32, P, P],
    ),
    "kvbp_prefill_evict_noalloc": (
        C.c_int,
        [P, C.POINTER(State), I32, C.POINTER(EvictCfg), P, P, P, I32, P, P, P, P, I32, P, P],
    ),
    "kvbp_gather_kv": (C.c_int, [P, P, P, P, P, P, I32, I32, I32, I32, I32]),
    "kvbp_embed": (C.c_int, [P, I32, I32, I32, P, P, P, P]),
    "kvbp_add_rmsnorm": (C.c_int, [P, I32, I32, P, P, P, P, F32]),
    "kvbp_silu_mul": (C.c_int, [P, I32, I32, P, P]),
    "kvbp_argmax": (C.c_int, [P, I32, I32, I64, P, P]),
    "kvbp_row_sumsq": (C.c_int, [P, I32, I32, P, P]),
    "kvbp_decode_gemm": (C.c_int, [P, I32, I32, I32, I32, P, P, I32, P, I32, P, F32, P, I32, P, I32, P]),
    "kvbp_decode_qkv_gemm": (C.c_int, [P, I32, I32, I32, I32, P, P, I32, P, I32, P, F32, P, P, P, P, P, P, I32, P, P,
                                       P, I32, P]),
    "kvbp_prefill_attn_score": (C.c_int, [P, I32, I32, I32, I32, P, P, P, P, P, P]),
    "kvbp_decode_gemm_allreduce": (C.c_int, [P, I32, I32, I32, P, P, I32, P, P, I32, P, I32, I32, I32, P, I64, P]),
    "kvbp_pack_weight": (C.c_int, [P, I32, I32, P, P]),
    "kvbp_argmax_key": (C.c_int, [P, I32, I32, I64, P, I32, P]),
    "kvbp_key_to_token": (C.c_int, [P, I32, P, P]),
    "kvbp_residual_add": (C.c_int, [P, I32, I32, P, P, P]),
    "kvbp_demote_int8": (C.c_int, [P, P, P, I32, I32, I32, I32, P, I32, P, P]),
    "kvbp_prefill_gemm": (C.c_int, [P, I32, I32, I32, I32, P, P, I32, P, I32, P]),
    "kvbp_unpack_weight": (C.c_int, [P, I32, I32, P, P]),
}
EXTRA_SIGNATURES = {
    "kvbp_decode_attn_score_cs": (C.c_int, [P, I32, I32, I32, I32, I32, P, P, P, P, P, P, P, P, I32]),
    "kvbp_decode_attn_score_cfg": (C.c_int, [P, I32, I32, I32, I32, I32, P, P, P, P, P, P, P, P, I32, I32]),
}

_LIB: Optional[C.CDLL] = None


def lib() -> C.CDLL:
    """Load libkvbp.so (built in-tree by ``kvcacheboundaryprotection_b200.build``)."""
    global _LIB
    if _LIB is None:
        path = Path(os.environ.get("KVBP_LIB", str(LIB_PATH)))
        if not path.exists():
            raise KVBPError(
                f"{path} not found: build it with `python -m kvcacheboundaryprotection_b200.build` "
                "(the CUDA library is required; there is no CPU fallback)"
            )
        L = C.CDLL(str(path))
        for name, (res, args) in {**SIGNATURES, **EXTRA_SIGNATURES}.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = L
    return _LIB


def check(status: int, what: str) -> None:
    if status != KVBP_OK:
        msg = lib().kvbp_last_error().decode(errors="replace")
        raise KVBPError(f"{what} failed with status {status}: {msg}")


def decode_dev_errors(word: int) -> list:
    return [msg for bit, msg in DEV_ERRORS.items() if word & bit]


def protection_sizes(capacity: int, prefix_frac: float, suffix_frac: float) -> tuple:
    a, b = C.c_int32(), C.c_int32()
    lib().kvbp_protection_sizes(int(capacity), float(prefix_frac), float(suffix_frac), C.byref(a), C.byref(b))
    return a.value, b.value


def policy_id(name: str) -> int:
    pid = lib().kvbp_policy_id(name.encode())
    if pid < 0:
        raise ValueError(f"policy {name!r} has no CUDA eviction kernel; supported: {sorted(POLICY_IDS)}")
    return pid
